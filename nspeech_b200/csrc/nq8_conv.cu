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
// A thread writes 8 consecutive elements of one row (one 16-byte store for
// bf16 rows, two for f32), walking (ci, j) incrementally; ld % 8 == 0.
__global__ void im2col_kernel(const void *__restrict__ x, int x_dtype, int64_t ldx, int c_in, int t_in, int K,
                              int stride, int pad, int dil, float slope, int t_out, int64_t ld, int a_dtype,
                              void *__restrict__ rows) {
  pdl_wait();
  pdl_trigger();
  const int ck = c_in * K;
  for (int t = blockIdx.y; t < t_out; t += gridDim.y) {
    const int tbase = t * stride - pad;
    for (int64_t e0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; e0 < ld;
         e0 += static_cast<int64_t>(gridDim.x) * blockDim.x * 8) {
      float v[8];
      int ci = static_cast<int>(e0 / K), j = static_cast<int>(e0 - static_cast<int64_t>(ci) * K);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        v[q] = 0.f;
        if (e0 + q < ck) {
          const int ti = tbase + j * dil;
          if (ti >= 0 && ti < t_in) v[q] = leaky(load_x(x, x_dtype, static_cast<int64_t>(ci) * ldx + ti), slope);
        }
        if (++j == K) {
          j = 0;
          ++ci;
        }
      }
      if (a_dtype == 0) {
        float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(rows) + static_cast<int64_t>(t) * ld + e0);
        dst[0] = make_float4(v[0], v[1], v[2], v[3]);
        dst[1] = make_float4(v[4], v[5], v[6], v[7]);
      } else {
        uint4 pk;
        pk.x = pack_bf16x2(v[0], v[1]);
        pk.y = pack_bf16x2(v[2], v[3]);
        pk.z = pack_bf16x2(v[4], v[5]);
        pk.w = pack_bf16x2(v[6], v[7]);
        *reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(rows) + static_cast<int64_t>(t) * ld + e0) = pk;
      }
    }
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
  const int threads = 128;
  const dim3 grid(static_cast<unsigned>((ld / 8 + threads - 1) / threads), static_cast<unsigned>(std::min(t_out, 65535)));
  return launch_pdl(im2col_kernel, grid, dim3(threads), 0, s, 1, x, x_dtype, ldx, c_in, t_in, K, stride, pad, dil,
                    slope, t_out, ld, a_dtype, rows);
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
