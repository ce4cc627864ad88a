// nq8_conv.cu -- conv1d and conv_transpose1d through the Q8_0 / bf16 GEMMs.
//
// The Kokoro ISTFTNet decoder's convolutions (src/kokoro/decoder.rs; Triton
// kernels conv1d_k, im2col_conv1d and the fused leaky-ReLU variants of
// kernels/kokoro_kernels.py:182,426-525; backend entries conv1d, im2col,
// matmul_bias, conv_transpose1d of src/kokoro/gpu_backend.rs:59-110).  The
// reference GPU path lowers a conv1d to im2col + matmul_bias over the weight's
// GGUF 2-D form [C_out, C_in * K]; here the same lowering feeds the tensor-core
// GEMMs of this library:
//   conv1d:            im2col (NCW input -> token-major rows [T_out][C_in*K],
//                      optional leaky ReLU on load) -> nq_linear (bias and
//                      activation fused in the GEMM epilogue) -> transpose to
//                      NCW [C_out][T_out].
//   conv_transpose1d:  transpose the input to token-major rows (optional leaky
//                      ReLU) -> GEMM against the transposed weight [C_out*K,
//                      C_in] (f32 columns [T_in][C_out*K]) -> col2im: each
//                      output sums its (ceil(K / stride) at most) taps in
//                      ascending tap order, then bias and activation.
#include <algorithm>

#include "nq8_common.cuh"
#include "nq8_kernels.h"
#include "nq8_sm100_pair.cuh"

namespace nq {
namespace {

__device__ __forceinline__ float load_x(const void *x, int x_dtype, int64_t i) {
  return x_dtype == 0 ? static_cast<const float *>(x)[i] : __bfloat162float(static_cast<const __nv_bfloat16 *>(x)[i]);
}
__device__ __forceinline__ float leaky(float v, float slope) { return v >= 0.f ? v : v * slope; }

// rows[t][e] for e < c_in * K: x[ci][t * stride - pad + j * dil] with
// ci = e / K, j = e % K (zero outside [0, t_in)); zero for e in [c_in * K, ld).
// A block covers tt output rows and the channel chunk [ci0, ci0 + cb): the
// cb x W input window it reads (W = (tt - 1) stride + (K - 1) dil + 1
// samples) is staged once in shared memory -- loads coalesced along time,
// leaky ReLU and zero padding applied -- and each row's segment
// [ci0 K, (ci0 + cb) K) is written 8 elements (16 bytes of bf16) per thread.
// The block of the last chunk also zero-fills [c_in K, ld).  ld % 8 == 0 and
// cb K % 8 == 0 unless cb == c_in keep every 8-element group aligned.
constexpr int kIcTTMax = 32;
__global__ void __launch_bounds__(256) im2col_kernel(const void *__restrict__ x, int x_dtype, int64_t ldx, int c_in,
                                                     int t_in, int K, int stride, int pad, int dil, float slope,
                                                     int t_out, int64_t ld, int a_dtype, void *__restrict__ rows, int cb,
                                                     int tt, int W, int pitch) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sx[];  // [cb][pitch]
  const int ci0 = blockIdx.x * cb;
  const int cbn = min(cb, c_in - ci0);
  for (int t0 = blockIdx.y * tt; t0 < t_out; t0 += gridDim.y * tt) {
    const int tb = t0 * stride - pad;
    __syncthreads();  // the previous tile's window is no longer read
    for (int idx = threadIdx.x; idx < cbn * W; idx += blockDim.x) {
      const int cl = idx / W, w = idx - cl * W;
      const int ti = tb + w;
      sx[cl * pitch + w] =
          (ti >= 0 && ti < t_in) ? leaky(load_x(x, x_dtype, static_cast<int64_t>(ci0 + cl) * ldx + ti), slope) : 0.f;
    }
    __syncthreads();
    const int seg = cbn * K;                            // this chunk's elements of a row
    const int64_t e_base = static_cast<int64_t>(ci0) * K;
    const int64_t seg_w = ci0 + cbn == c_in ? ld - e_base : seg;  // the last chunk also pads the row
    const int rows_here = min(tt, t_out - t0);
    const int groups = static_cast<int>((seg_w + 7) / 8);
    for (int g = threadIdx.x; g < rows_here * groups; g += blockDim.x) {
      const int r = g / groups;
      const int q = (g - r * groups) * 8;  // first element of the group within the segment
      float v[8];
      int cl = q / K, j = q - cl * K;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        v[u] = q + u < seg ? sx[cl * pitch + r * stride + j * dil] : 0.f;
        if (++j == K) {
          j = 0;
          ++cl;
        }
      }
      const int64_t o = static_cast<int64_t>(t0 + r) * ld + e_base + q;
      const int n = seg_w - q < 8 ? static_cast<int>(seg_w - q) : 8;
      if (a_dtype == 0) {
        float *dst = static_cast<float *>(rows) + o;
        if (n == 8) {
          reinterpret_cast<float4 *>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
          reinterpret_cast<float4 *>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
          for (int u = 0; u < n; ++u) dst[u] = v[u];
        }
      } else {
        __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(rows) + o;
        if (n == 8) {
          uint4 pk;
          pk.x = pack_bf16x2(v[0], v[1]);
          pk.y = pack_bf16x2(v[2], v[3]);
          pk.z = pack_bf16x2(v[4], v[5]);
          pk.w = pack_bf16x2(v[6], v[7]);
          *reinterpret_cast<uint4 *>(dst) = pk;
        } else {
          for (int u = 0; u < n; ++u) dst[u] = __float2bfloat16_rn(v[u]);
        }
      }
    }
  }
}

// Token-major operand planes of the implicit convs: hi[t][c] =
// bf16(leaky(x[c][t])), lo[t][c] = bf16(v - hi) (f32 x only).  A block moves
// a 64-channel x 32-frame tile through shared memory.  Loads run along time,
// 16 bytes per thread where the vector lies inside the row (issued before
// their use).  Stores write whole 128-byte channel runs per frame.
constexpr int kTokT = 32;
__global__ void __launch_bounds__(256) conv_tokens_kernel(const void *__restrict__ x, int x_dtype, int64_t ldx, int c_in,
                                                          int t_in, float slope, __nv_bfloat16 *__restrict__ hi,
                                                          __nv_bfloat16 *__restrict__ lo, int vec) {
  pdl_wait();
  pdl_trigger();
  __shared__ float tile[64][kTokT + 1];
  const int t0 = blockIdx.x * kTokT, c0 = blockIdx.y * 64;
  if (x_dtype != 0) {
    // bf16: 8 frames per vector, 4 vectors per channel row of the tile, one per thread
    const __nv_bfloat16 *xb = static_cast<const __nv_bfloat16 *>(x);
    const int q = threadIdx.x, c = q >> 2, tl = (q & 3) * 8, t = t0 + tl;
    const __nv_bfloat16 *src = xb + static_cast<int64_t>(c0 + c) * ldx + t;
    uint4 v;
    if (vec && t + 8 <= t_in) {
      v = __ldg(reinterpret_cast<const uint4 *>(src));
    } else {
      uint16_t e[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) e[u] = t + u < t_in ? __bfloat16_as_ushort(src[u]) : 0;
      v = make_uint4(e[0] | (uint32_t(e[1]) << 16), e[2] | (uint32_t(e[3]) << 16), e[4] | (uint32_t(e[5]) << 16),
                     e[6] | (uint32_t(e[7]) << 16));
    }
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      tile[c][tl + 2 * u] = leaky(bf16_bits_to_f32(w[u] & 0xffffu), slope);
      tile[c][tl + 2 * u + 1] = leaky(bf16_bits_to_f32(w[u] >> 16), slope);
    }
  } else {
    // f32: 4 frames per vector, 8 vectors per channel row of the tile, two per thread
    const float *xf = static_cast<const float *>(x);
    float4 v[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int q = threadIdx.x + i * 256, c = q >> 3, t = t0 + (q & 7) * 4;
      const float *src = xf + static_cast<int64_t>(c0 + c) * ldx + t;
      if (vec && t + 4 <= t_in) {
        v[i] = __ldg(reinterpret_cast<const float4 *>(src));
      } else {
        v[i] = make_float4(t < t_in ? src[0] : 0.f, t + 1 < t_in ? src[1] : 0.f, t + 2 < t_in ? src[2] : 0.f,
                           t + 3 < t_in ? src[3] : 0.f);
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int q = threadIdx.x + i * 256, c = q >> 3, tl = (q & 7) * 4;
      tile[c][tl] = leaky(v[i].x, slope);
      tile[c][tl + 1] = leaky(v[i].y, slope);
      tile[c][tl + 2] = leaky(v[i].z, slope);
      tile[c][tl + 3] = leaky(v[i].w, slope);
    }
  }
  __syncthreads();
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int r = ty; r < kTokT; r += 8) {
    const int t = t0 + r;
    if (t >= t_in) break;
    const float v0 = tile[2 * tx][r], v1 = tile[2 * tx + 1][r];
    const uint32_t h = pack_bf16x2(v0, v1);
    const int64_t o = static_cast<int64_t>(t) * c_in + c0 + 2 * tx;
    *reinterpret_cast<uint32_t *>(hi + o) = h;
    if (lo) *reinterpret_cast<uint32_t *>(lo + o) = pack_bf16x2(v0 - bf16_bits_to_f32(h & 0xffffu), v1 - bf16_bits_to_f32(h >> 16));
  }
}

// dst[r][j c_in + ci] = src[r][ci K + j]: eight consecutive destination
// elements (one 16-byte store) per thread.
__global__ void conv_tap_weight_kernel(const __nv_bfloat16 *__restrict__ src, int64_t ld_src, int rows, int c_in, int K,
                                       __nv_bfloat16 *__restrict__ dst) {
  const int64_t ld_dst = static_cast<int64_t>(K) * c_in;
  const int64_t groups = static_cast<int64_t>(rows) * (ld_dst / 8);
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < groups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = g / (ld_dst / 8);
    const int64_t e0 = (g - r * (ld_dst / 8)) * 8;
    const int j = static_cast<int>(e0 / c_in);
    const int ci0 = static_cast<int>(e0 - static_cast<int64_t>(j) * c_in);
    const __nv_bfloat16 *s = src + r * ld_src + static_cast<int64_t>(ci0) * K + j;
    uint16_t v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = reinterpret_cast<const uint16_t *>(s)[static_cast<int64_t>(u) * K];
    *reinterpret_cast<uint4 *>(dst + r * ld_dst + e0) =
        make_uint4(v[0] | (uint32_t(v[1]) << 16), v[2] | (uint32_t(v[3]) << 16), v[4] | (uint32_t(v[5]) << 16),
                   v[6] | (uint32_t(v[7]) << 16));
  }
}

// dst[co s + r][i c_in + ci] = src[co K + r + s i][ci] (zero when the tap or
// the row does not exist): eight consecutive destination elements per thread.
__global__ void conv_poly_weight_kernel(const __nv_bfloat16 *__restrict__ src, int64_t ld_src, int c_out, int K,
                                        int s, int c_in, int taps, int rows, __nv_bfloat16 *__restrict__ dst) {
  const int64_t ld_dst = static_cast<int64_t>(taps) * c_in;
  const int64_t groups = static_cast<int64_t>(rows) * (ld_dst / 8);
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < groups;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = g / (ld_dst / 8);
    const int64_t e0 = (g - n * (ld_dst / 8)) * 8;
    const int i = static_cast<int>(e0 / c_in);
    const int ci0 = static_cast<int>(e0 - static_cast<int64_t>(i) * c_in);
    const int co = static_cast<int>(n / s), r = static_cast<int>(n - static_cast<int64_t>(co) * s);
    const int j = r + s * i;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (co < c_out && j < K) v = *reinterpret_cast<const uint4 *>(src + (static_cast<int64_t>(co) * K + j) * ld_src + ci0);
    *reinterpret_cast<uint4 *>(dst + n * ld_dst + e0) = v;
  }
}

// y[c][t] (ldy) = src[t][c] (lds): 32 x 32 tiles through shared memory.
__global__ void transpose_out_kernel(const void *__restrict__ src, int src_dtype, int64_t lds, int rows_t, int cols_c,
                                     void *__restrict__ y, int y_dtype, int64_t ldy) {
  pdl_wait();
  pdl_trigger();
  __shared__ float tile[32][33];
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int t = t0 + r, c = c0 + threadIdx.x;
    tile[r][threadIdx.x] = (t < rows_t && c < cols_c) ? load_x(src, src_dtype, static_cast<int64_t>(t) * lds + c) : 0.f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int c = c0 + r, t = t0 + threadIdx.x;
    if (c < cols_c && t < rows_t) {
      const float v = tile[threadIdx.x][r];
      const int64_t o = static_cast<int64_t>(c) * ldy + t;
      if (y_dtype == 0) static_cast<float *>(y)[o] = v;
      else static_cast<__nv_bfloat16 *>(y)[o] = __float2bfloat16_rn(v);
    }
  }
}

// y[co][t] = act(bias[co] + sum over taps j ascending with (t + pad - j) % stride
// == 0 and ti = (t + pad - j) / stride in [0, t_in) of cols[ti][co * K + j]).
__global__ void col2im_kernel(const float *__restrict__ cols, int64_t ldc, int t_in, int c_out, int K, int stride,
                              int pad, int t_out, const float *__restrict__ bias, int epi, void *__restrict__ y,
                              int y_dtype, int64_t ldy) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = static_cast<int64_t>(c_out) * t_out;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int co = static_cast<int>(i / t_out);
    const int t = static_cast<int>(i - static_cast<int64_t>(co) * t_out);
    float acc = 0.f;
    const int tp = t + pad;
    for (int j = tp % stride; j < K; j += stride) {
      const int ti = (tp - j) / stride;
      if (ti < 0) break;  // ti only decreases with j
      if (ti < t_in) acc += cols[static_cast<int64_t>(ti) * ldc + static_cast<int64_t>(co) * K + j];
    }
    float v = acc + (bias ? bias[co] : 0.f);
    switch (epi) {
      case kEpiSilu: v = act_t<kEpiSilu>(v); break;
      case kEpiGeluErf: v = act_t<kEpiGeluErf>(v); break;
      case kEpiRelu: v = act_t<kEpiRelu>(v); break;
      default: break;
    }
    const int64_t o = static_cast<int64_t>(co) * ldy + t;
    if (y_dtype == 0) static_cast<float *>(y)[o] = v;
    else static_cast<__nv_bfloat16 *>(y)[o] = __float2bfloat16_rn(v);
  }
}

int grid_for(int64_t total, int threads) {
  return static_cast<int>(std::min<int64_t>((total + threads - 1) / threads, 148 * 16));
}

}  // namespace

cudaError_t launch_im2col(const void *x, int x_dtype, int64_t ldx, int c_in, int t_in, int K, int stride, int pad,
                          int dil, float slope, int t_out, int64_t ld, int a_dtype, void *rows, cudaStream_t s) {
  if (t_out == 0 || ld == 0) return cudaSuccess;
  if (ld % 8) return cudaErrorInvalidValue;
  if (static_cast<int64_t>(K - 1) * dil > 8192 || stride > 64) return cudaErrorInvalidValue;
  // Channel chunk: 64 (a multiple of 8, so chunk boundaries keep rows 8-aligned)
  // or all of c_in.  Time tile: 32 rows, halved (to 8) until the grid has
  // about four blocks per SM, so the window loads of some blocks overlap the
  // stores of others.
  const int cb0 = c_in <= 64 ? c_in : 64;
  const int chunks0 = (c_in + cb0 - 1) / cb0;
  int tt = kIcTTMax;
  while (tt > 8 && static_cast<int64_t>(chunks0) * ((t_out + tt - 1) / tt) < 4 * 148) tt /= 2;
  const int W = (tt - 1) * stride + (K - 1) * dil + 1;
  const int pitch = W | 1;  // odd: the taps of consecutive elements spread over the banks
  int cb = cb0;  // halved while its window exceeds 48 KB
  while (cb > 8 && static_cast<size_t>(cb) * pitch * 4 > 48 * 1024) cb /= 2;
  if (cb < c_in && (cb * K) % 8) return cudaErrorInvalidValue;
  const size_t smem = static_cast<size_t>(cb) * pitch * 4;
  if (smem > 48 * 1024) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>((c_in + cb - 1) / cb),
                  static_cast<unsigned>(std::min((t_out + tt - 1) / tt, 65535)));
  return launch_pdl(im2col_kernel, grid, dim3(256), smem, s, 1, x, x_dtype, ldx, c_in, t_in, K, stride, pad, dil,
                    slope, t_out, ld, a_dtype, rows, cb, tt, W, pitch);
}

cudaError_t launch_conv_tokens(const void *x, int x_dtype, int64_t ldx, int c_in, int t_in, float slope,
                               __nv_bfloat16 *hi, __nv_bfloat16 *lo, cudaStream_t s) {
  if (t_in == 0) return cudaSuccess;
  if (c_in % 64) return cudaErrorInvalidValue;
  // 16-byte loads need 16-byte aligned rows (base and row stride)
  const int per_vec = x_dtype == 0 ? 4 : 8;
  const int vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0 && ldx % per_vec == 0) ? 1 : 0;
  const dim3 grid((t_in + kTokT - 1) / kTokT, c_in / 64);
  return launch_pdl(conv_tokens_kernel, grid, dim3(256), 0, s, 1, x, x_dtype, ldx, c_in, t_in, slope, hi, lo, vec);
}

cudaError_t launch_conv_tap_weight(const __nv_bfloat16 *src, int64_t ld_src, int rows, int c_in, int K,
                                   __nv_bfloat16 *dst, cudaStream_t s) {
  if (c_in % 8) return cudaErrorInvalidValue;
  const int64_t groups = static_cast<int64_t>(rows) * K * c_in / 8;
  if (groups == 0) return cudaSuccess;
  conv_tap_weight_kernel<<<grid_for(groups, 256), 256, 0, s>>>(src, ld_src, rows, c_in, K, dst);
  return cudaGetLastError();
}

cudaError_t launch_conv_poly_weight(const __nv_bfloat16 *src, int64_t ld_src, int c_out, int K, int s, int c_in,
                                   int taps, int rows, __nv_bfloat16 *dst, cudaStream_t stream) {
  if (c_in % 8 || ld_src % 8) return cudaErrorInvalidValue;
  const int64_t groups = static_cast<int64_t>(rows) * taps * c_in / 8;
  if (groups == 0) return cudaSuccess;
  conv_poly_weight_kernel<<<grid_for(groups, 256), 256, 0, stream>>>(src, ld_src, c_out, K, s, c_in, taps, rows, dst);
  return cudaGetLastError();
}

cudaError_t launch_transpose_out(const void *src, int src_dtype, int64_t lds, int rows_t, int cols_c, void *y,
                                 int y_dtype, int64_t ldy, cudaStream_t s) {
  if (rows_t == 0 || cols_c == 0) return cudaSuccess;
  const dim3 grid((rows_t + 31) / 32, (cols_c + 31) / 32);
  return launch_pdl(transpose_out_kernel, grid, dim3(32, 8), 0, s, 1, src, src_dtype, lds, rows_t, cols_c, y, y_dtype,
                    ldy);
}

cudaError_t launch_col2im(const float *cols, int64_t ldc, int t_in, int c_out, int K, int stride, int pad, int t_out,
                          const float *bias, int epi, void *y, int y_dtype, int64_t ldy, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(c_out) * t_out;
  if (total == 0) return cudaSuccess;
  return launch_pdl(col2im_kernel, dim3(grid_for(total, 256)), dim3(256), 0, s, 1, cols, ldc, t_in, c_out, K, stride,
                    pad, t_out, bias, epi, y, y_dtype, ldy);
}

}  // namespace nq
