// nq8_kernels.h -- launch interfaces between the C-ABI layer (nq8_api.cu) and
// the kernels (nq8_gemv.cu, nq8_gemm.cu, nq8_aux.cu).  Internal header.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "nq8_common.cuh"

namespace nq {

// One weight's share of a GEMV launch (up to three for the fused Q/K/V call).
struct GemvProblem {
  const uint8_t *w;  // packed tiles
  int n_tiles;       // ceil(N_pad / 128)
  int kc_total;      // k chunks of 64
  int64_t N;         // logical output rows of W
  int glu;           // weight packed NQ_PACK_GLU
  int64_t n_out;     // output columns (N, or N/2 for GLU)
  const float *bias;
  void *y;
  int64_t ldy;
  float *partials;  // [splits][n_tiles][16][128] f32 (split-K only)
  int *counters;    // [n_tiles], zero between calls
};

struct GemvParams {
  GemvProblem prob[3];
  const void *x;
  int x_dtype;  // 0 f32, 1 bf16
  int64_t ldx;
  int M;
  int64_t K;
  int epi;
  int y_dtype;
  int splits;
  int cps;  // k chunks per split
  DevCtl ctl;
};

size_t gemv_smem_bytes(int mrows, bool splitx, int cps);
cudaError_t launch_gemv(const GemvParams &p, int nprob, int grid_x, bool splitx, cudaStream_t stream);

struct GemmParams {
  const uint8_t *w;
  int n_tiles;
  int kc_total;
  int64_t N;
  int glu;
  int64_t n_out;
  int M;
  const float *bias;
  int epi;
  void *y;
  int y_dtype;
  int64_t ldy;
  int splits;
  int cps;
  int grid_n;       // 128-row weight tiles (= n_tiles)
  int grid_m;       // token tiles of BT rows
  float *partials;  // [splits][grid_m][grid_n][128][BT] f32 (split-K only)
  int *counters;    // [grid_m * grid_n]
  DevCtl ctl;
};

// Which compiled token-tile configuration to launch.
enum GemmVariant : int { kGemmBt256 = 0, kGemmBt128 = 1, kGemmBt64 = 2, kGemmBt128SplitX = 3 };
int gemm_block_t(GemmVariant v);
size_t gemm_smem_bytes(GemmVariant v);
// Persistent launch: `grid` CTAs (<= one per SM) walk grid_n * grid_m * splits
// work units.
cudaError_t launch_gemm(GemmVariant v, const CUtensorMap &a_hi, const CUtensorMap &a_lo,
                        const GemmParams &p, int grid, cudaStream_t stream);

// f32 -> bf16 planes: hi = bf16(x), lo = bf16(x - hi) (lo may be null); rows
// of k_pad elements, zero beyond K.  Also used for bf16 -> bf16 copies when a
// caller's bf16 activations are not TMA-aligned.
cudaError_t launch_split_x(const void *x, int x_dtype, int64_t ldx, int64_t M, int64_t K,
                           int64_t k_pad, __nv_bfloat16 *hi, __nv_bfloat16 *lo, cudaStream_t stream);

cudaError_t launch_wait_timeout_probe(DevCtl ctl, cudaStream_t stream);

}  // namespace nq
