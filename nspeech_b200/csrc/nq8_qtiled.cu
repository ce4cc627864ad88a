// nq8_qtiled.cu -- the QTiled semantics of MatMul::from_qtensor on sm_100a.
//
// Reference: QTiledOp::cpu_fwd (src/fast_matmul.rs:71-125) over
// tiled_matmul_inner (:30-62).  The activations are quantized per 32-element
// block to Q8_0 with ggml's rule (from_float, :42: d = amax / 127,
// q = roundf(x / d), d stored as f16) and every output is the per-block
// integer dot product scaled by both blocks' f16 scales (vec_dot, :57):
//     y[m, n] = sum over blocks b, in order, of ((float)sumi_b * d_w) * d_x
// with f32 rounding after each multiply and add -- the association order of
// the CPU oracle (oracle/nq8_oracle.c oq_matmul_qtiled), so results are
// bit-identical to it.  candle's own vec_dot order is not visible (the crate is
// not vendored); the reference's tolerance contract covers the difference.
//
// Two kernels:
//   qtiled_quantize_x  one warp per 32-element block (lane = element): amax by
//                      shuffles, IEEE divide, roundf, f16 scale; writes int8
//                      rows [M][K_pad] and f32 scales [M][K_pad / 32] (zero
//                      past K, like the weight's zero blocks).
//   qtiled_kernel      each warp owns 16 weight rows and 8 * TN tokens; per
//                      32-k block one mma.sync m16n8k32 s8 per 8 tokens gives
//                      the exact int32 sums, which are scaled and added in
//                      block order.  The weight fragments come straight from
//                      the packed tiles (a 16-row slab of one 16-k chunk is
//                      256 contiguous bytes: coalesced 32-bit loads, no shared
//                      memory); every output is owned by one thread, so no
//                      split over k and no cross-thread reduction.
#include <algorithm>

#include "nq8_common.cuh"
#include "nq8_kernels.h"
#include "nq8_sm100_pair.cuh"

namespace nq {
namespace {

constexpr int kQtWarps = 4;  // warps per CTA (16 weight rows each)

__global__ void __launch_bounds__(256) qtiled_quantize_x(const void *x, int x_dtype, int64_t ldx, int M, int64_t K,
                                                         int kb_pad, int8_t *xq, float *dx) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  for (int m = blockIdx.y; m < M; m += gridDim.y)
  for (int b = blockIdx.x * 8 + (threadIdx.x >> 5); b < kb_pad; b += gridDim.x * 8) {
    const int64_t k = static_cast<int64_t>(b) * 32 + lane;
    float v = 0.f;
    if (k < K) {
      v = x_dtype == 0 ? static_cast<const float *>(x)[m * ldx + k]
                       : __bfloat162float(static_cast<const __nv_bfloat16 *>(x)[m * ldx + k]);
    }
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const float q = roundf(__fmul_rn(v, id));
    xq[static_cast<int64_t>(m) * kb_pad * 32 + k] = static_cast<int8_t>(q);
    if (lane == 0) dx[static_cast<int64_t>(m) * kb_pad + b] = __half2float(__float2half_rn(d));
  }
}

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %11, %12, %13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ uint32_t ldg32(const uint8_t *p) {
  return __ldg(reinterpret_cast<const unsigned int *>(p));
}

template <int TN>
__global__ void __launch_bounds__(32 * kQtWarps) qtiled_kernel(const QtiledParams p) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int row0 = (blockIdx.x * kQtWarps + warp) * 16;  // first weight row of this warp (packed = logical order)
  if (row0 >= p.n_tiles * kPackRows) return;
  const int tile = row0 / kPackRows, r_in = row0 % kPackRows;
  const int kb_pad = p.kc * 2;
  const uint8_t *wt = p.w + static_cast<size_t>(tile) * p.kc * kTileBytes;
  for (int m0 = blockIdx.y * (8 * TN); m0 < p.M; m0 += gridDim.y * (8 * TN)) {

  // B operand rows (token g of each 8-token group) and scale rows (tokens
  // tig*2, tig*2+1); tokens past M read row 0 and are never stored.
  const int8_t *xb[TN];
  const float *sx0[TN], *sx1[TN];
#pragma unroll
  for (int t = 0; t < TN; ++t) {
    const int mb = m0 + t * 8 + g, ms = m0 + t * 8 + tig * 2;
    xb[t] = p.xq + static_cast<int64_t>(mb < p.M ? mb : 0) * kb_pad * 32;
    sx0[t] = p.dx + static_cast<int64_t>(ms < p.M ? ms : 0) * kb_pad;
    sx1[t] = p.dx + static_cast<int64_t>(ms + 1 < p.M ? ms + 1 : 0) * kb_pad;
  }
  float acc[TN][4];
#pragma unroll
  for (int t = 0; t < TN; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;

  for (int c = 0; c < p.kc; ++c) {
    const uint8_t *ch = wt + static_cast<size_t>(c) * kTileBytes;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int kb = 2 * c + h;
      uint32_t a[4];
      a[0] = ldg32(ch + qs_offset(r_in + g, 2 * h) + tig * 4);
      a[1] = ldg32(ch + qs_offset(r_in + g + 8, 2 * h) + tig * 4);
      a[2] = ldg32(ch + qs_offset(r_in + g, 2 * h + 1) + tig * 4);
      a[3] = ldg32(ch + qs_offset(r_in + g + 8, 2 * h + 1) + tig * 4);
      const float dw0 = __half2float(__ldg(reinterpret_cast<const __half *>(ch + scale_offset(r_in + g, h))));
      const float dw1 = __half2float(__ldg(reinterpret_cast<const __half *>(ch + scale_offset(r_in + g + 8, h))));
#pragma unroll
      for (int t = 0; t < TN; ++t) {
        const int8_t *xr = xb[t] + kb * 32 + tig * 4;
        const uint32_t b0 = __ldg(reinterpret_cast<const unsigned int *>(xr));
        const uint32_t b1 = __ldg(reinterpret_cast<const unsigned int *>(xr + 16));
        int d[4];
        mma_s8(d, a, b0, b1);
        const float x0 = __ldg(sx0[t] + kb), x1 = __ldg(sx1[t] + kb);
        // (n = g, m = 2 tig), (g, 2 tig + 1), (g + 8, 2 tig), (g + 8, 2 tig + 1)
        acc[t][0] = __fadd_rn(acc[t][0], __fmul_rn(__fmul_rn(__int2float_rn(d[0]), dw0), x0));
        acc[t][1] = __fadd_rn(acc[t][1], __fmul_rn(__fmul_rn(__int2float_rn(d[1]), dw0), x1));
        acc[t][2] = __fadd_rn(acc[t][2], __fmul_rn(__fmul_rn(__int2float_rn(d[2]), dw1), x0));
        acc[t][3] = __fadd_rn(acc[t][3], __fmul_rn(__fmul_rn(__int2float_rn(d[3]), dw1), x1));
      }
    }
  }

#pragma unroll
  for (int t = 0; t < TN; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = m0 + t * 8 + tig * 2 + (i & 1);
      const int64_t n = row0 + g + (i >> 1) * 8;
      if (m >= p.M || n >= p.N) continue;
      float v = acc[t][i] + (p.bias ? p.bias[n] : 0.f);
      switch (p.epi) {
        case kEpiSilu: v = act_t<kEpiSilu>(v); break;
        case kEpiGeluErf: v = act_t<kEpiGeluErf>(v); break;
        case kEpiRelu: v = act_t<kEpiRelu>(v); break;
        default: break;
      }
      const int64_t off = static_cast<int64_t>(m) * p.ldy + n;
      if (p.y_dtype == 0) static_cast<float *>(p.y)[off] = v;
      else static_cast<__nv_bfloat16 *>(p.y)[off] = __float2bfloat16_rn(v);
    }
  }  // token tiles
}

template <int TN>
cudaError_t launch_t(const QtiledParams &p, cudaStream_t stream) {
  const int rows = p.n_tiles * kPackRows;
  const dim3 grid((rows / 16 + kQtWarps - 1) / kQtWarps, std::min((p.M + 8 * TN - 1) / (8 * TN), 65535));
  return launch_pdl(qtiled_kernel<TN>, grid, dim3(32 * kQtWarps), 0, stream, 1, p);
}

}  // namespace

size_t qtiled_x_bytes(int64_t M, int kc) {
  const size_t q = static_cast<size_t>(M) * kc * kPackK;
  return (q + 255) / 256 * 256 + static_cast<size_t>(M) * kc * 2 * sizeof(float);
}

cudaError_t launch_qtiled_quantize(const void *x, int x_dtype, int64_t ldx, int64_t M, int64_t K, int kc, int8_t *xq,
                                   float *dx, cudaStream_t stream) {
  const int kb_pad = kc * 2;
  const dim3 grid(std::min((kb_pad + 7) / 8, 64), static_cast<unsigned>(std::min<int64_t>(M, 65535)));
  return launch_pdl(qtiled_quantize_x, grid, dim3(256), 0, stream, 1, x, x_dtype, ldx, static_cast<int>(M), K, kb_pad,
                    xq, dx);
}

cudaError_t launch_qtiled(const QtiledParams &p, cudaStream_t stream) {
  if (p.M <= 8) return launch_t<1>(p, stream);
  if (p.M <= 16) return launch_t<2>(p, stream);
  return launch_t<8>(p, stream);
}

}  // namespace nq
