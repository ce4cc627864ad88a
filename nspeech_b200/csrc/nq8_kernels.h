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
  int64_t N;         // logical output rows of W
  int glu;           // weight packed NQ_PACK_GLU
  int64_t n_out;     // output columns (N, or N/2 for GLU)
  const float *bias;
  void *y;
  int64_t ldy;
  float *partials;  // [upt][M][n_tiles * 128] f32: slot j holds unit j of every tile
};

struct GemvParams {
  GemvProblem prob[3];
  const __nv_bfloat16 *xh;  // activations: bf16 rows of ldx elements, zero beyond K up to kc * 64
  const __nv_bfloat16 *xl;  // bf16(x - hi) rows for f32 activations, else null
  int64_t ldx;              // multiple of 8 elements; xh / xl 16-byte aligned
  int M;
  int epi;
  int y_dtype;
  int nprob;   // problems (weights) sharing x
  int kc;      // 64-wide k chunks per tile (same for every problem)
  int unit;    // k chunks per work unit
  int upt;     // units per tile: ceil(kc / unit)
  int units;   // units of all problems, tile-major
  int ctas;    // CTAs launched; CTA c starts with unit c
  int *sched;  // [0] work counter, [1] cluster form's tile arrivals: zero between calls (re-armed by the kernels)
  int sm_count;
  int path;    // 0: the cost rule below, 1: always the split + reduce form, 2: the cluster form where it applies
  // Decoder-step epilogue (one problem; res_out non-null selects it): the
  // row is y = W x + bias, res_out = res_in + y, prob[0].y = LN(res_out).
  const float *res_in;
  float *res_out;
  int64_t ld_res;
  const float *ln_g;  // LayerNorm gamma [N]
  const float *ln_b;  // LayerNorm beta [N] or null
  float ln_eps;
  DevCtl ctl;
};
constexpr int kGemvLnMaxN = 8192;  // row width the residual + LayerNorm epilogue holds

// Work split of one GEMV launch (fixed by the shape and the SM count).
struct GemvPlan {
  int unit, upt, units, ctas;
};
GemvPlan gemv_plan(int sm_count, int total_tiles, int kc, int m);
// The GEMV (ctas CTAs) and its gemv_reduce: two launches.  Latency-bound
// plain calls (at most 8 rows, at most 5 k chunks per CTA with the tile's k
// over a cluster of up to 8 CTAs, all CTAs in one wave) instead run the
// cluster form: one launch, the partial sums meet in distributed shared
// memory.
cudaError_t launch_gemv(const GemvParams &p, int ctas, cudaStream_t stream);
// Cluster size the cluster form uses for a call (0: the split + reduce form).
int gemv_cluster_size(int total_tiles, int kc, int sm_count, int path, bool resadd, int m);

// Decode chain (nq8_chain.cu): the dependent M = 1 GEMV steps of a decoder
// token in one cooperative launch.  Step s reads a bf16 vector x (or, with
// x_ln, the LayerNorm of step s - 1's residual row, computed on load) and
// either stores y = act(W x + bias) (GLU for GLU-packed weights) or, with
// res_out set, res_out = res_in + W x + bias; a residual step's LayerNorm
// output (bf16, y) is stored by the CTA of the next step's tile 0, or by the
// completer when it is the last step.  One CTA computes a whole 128-row tile.
constexpr int kChainMaxK = 4096;  // input length a step stages in shared memory
constexpr int kChainMaxLnN = 4096;
constexpr int kChainCluster = 4;  // CTAs that share one tile of a split step
struct ChainStep {
  const uint8_t *w;  // packed Q8_0 tiles [n_tiles][kc]
  int n_tiles, kc;
  int64_t N;         // weight rows
  int glu;
  int64_t n_out;     // outputs: N, or N / 2 for GLU
  int epi;
  const float *bias;
  int x_ln;          // input = LayerNorm of step s - 1's res_out
  const __nv_bfloat16 *x;  // input vector (x_ln == 0)
  int K;             // input length
  const float *res_in;
  float *res_out;    // residual step when set
  const float *ln_g, *ln_b;
  float ln_eps;
  void *y;           // output, or a residual step's LayerNorm output (bf16); may be null for the latter
  int y_dtype;
  int split;         // tiles go to clusters (chunk c to rank c % kChainCluster), else to CTAs
  int rot;           // cluster (split) or CTA of tile 0
};
struct ChainParams {
  const ChainStep *steps;  // device array
  int n_steps;
  int *ready;              // [n_steps] completed tiles per step, zero between calls
  DevCtl ctl;
};
size_t chain_smem_bytes();
int chain_threads();
// CTAs of one cooperative launch on this device (all resident at once).
cudaError_t chain_max_ctas(int sm_count, int *ctas);
cudaError_t launch_chain(const ChainParams &p, int ctas, cudaStream_t stream);

// K1: fused Q8_0 GEMM (dequantizes in the kernel; best below a few thousand
// tokens, where the weights dominate the traffic).
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
  int grid_n;       // weight pair tiles: ceil(n_tiles / 2), 256 rows each
  int grid_m;       // token tiles of BT rows
  float *partials;  // split-K only: [splits][M][ldp] f32, token-major, summed by splitk_reduce
  int ldp;          // n_tiles * 128
  DevCtl ctl;
};

// Which compiled configuration to launch (bf16 activations, or f32 ones as
// hi/lo bf16 planes).
enum GemmVariant : int { kGemmBt256 = 0, kGemmBt128 = 1, kGemmBt64 = 2, kGemmBt128SplitX = 3 };
// Tokens per work unit of an SM pair (each CTA stages half of them).
int gemm_block_t(GemmVariant v);
size_t gemm_smem_bytes(GemmVariant v);
// Persistent cluster launch: up to `pairs` two-CTA clusters (capped at the
// number that fit on the device at once) walk grid_n * grid_m * splits units.
cudaError_t launch_gemm(GemmVariant v, const CUtensorMap &a_hi, const CUtensorMap &a_lo,
                        const GemmParams &p, int pairs, cudaStream_t stream);

// K3: bf16 x bf16 GEMM over a dequantized copy of the weights (packed row
// order: row t*128 + r is row r of packed tile t), for large token counts.
struct GemmBf16Params {
  int64_t N;        // logical weight rows
  int n_rows;       // rows of the dequantized matrix (n_tiles * 128)
  int glu;
  int64_t n_out;
  int M;
  int kc_total;
  const float *bias;
  int epi;
  void *y;
  int y_dtype;
  int64_t ldy;
  int splits;
  int cps;
  int grid_n;       // 256-row weight pair tiles
  int grid_m;       // token tiles of the unit width
  float *partials;  // split-K only: [splits][M][n_rows] f32
  // Tail split (splits == 1 only): tiles [0, full_units) run whole; each
  // later tile runs as tail_pieces units of tail_cps k chunks on different
  // pairs.  A piece stores its raw accumulator to tail_part and counts on
  // tail_cnt; the last piece to arrive sums all pieces in piece order and
  // applies the epilogue (so results do not depend on arrival order), then
  // re-arms the counter.  tail_pieces <= 1: no tail split.
  int full_units;
  int tail_pieces;
  int tail_cps;
  float *tail_part;  // [tail tiles][pieces][2 CTAs][16 warps][unit tokens / 4][32] f32
  int *tail_cnt;     // [tail tiles][2 CTAs][16] counters, zero between calls
  int w_static;      // the weight is not written by any kernel of this stream (kept bf16 copy)
  int pair_stores;   // bf16 epilogue through lane pairs (4-byte stores); the host sets it when
                     // every unit runs in one round, where each unit's epilogue is exposed
  // Implicit conv1d (stride 1): the token operand of k chunk c is the
  // token-major input [t_in][channels] at channel offset 64 (c % conv_cpt),
  // rows t + j conv_dil - conv_pad for output token t and tap j = c / conv_cpt
  // (rows outside [0, t_in) read as zero).  conv_cpt = 0: a plain GEMM.
  int conv_cpt;
  int conv_dil;
  int conv_pad;
  int y_cm;          // channel-major output y[n][ldy] (NCW); no GLU, no split-K
  // Polyphase conv_transpose1d (poly_s > 0, with conv_cpt): weight row
  // n = co * poly_s + r holds phase r of output channel co; token m is input
  // position q = poly_q0 + m, and its value goes to y[co][q * poly_s + r -
  // poly_pad] when that frame is in [0, t_out); bias is indexed by co.
  int poly_s;
  int poly_q0;
  int poly_pad;
  int64_t t_out;
  DevCtl ctl;
};
int gemm_bf16_block_t();              // default tokens per pair unit
int gemm_bf16_block_w();              // weight rows per pair unit
bool gemm_bf16_unit_ok(int tokens);   // unit widths the kernel is built for (64, 128, 256)
int gemm_bf16_token_box(int unit_tokens);  // token rows per TMA box (per CTA and sub-tile)
// unit_tokens: tokens per pair unit (grid_m in p counts units of that width;
// the token tensor maps have boxes of gemm_bf16_token_box(unit_tokens) rows).
cudaError_t launch_gemm_bf16(bool splitx, int unit_tokens, const CUtensorMap &w, const CUtensorMap &a_hi,
                             const CUtensorMap &a_lo, const GemmBf16Params &p, int pairs, cudaStream_t stream);

// Packed Q8_0 tiles -> bf16 [n_tiles * 128][kc * 64] (row-major, packed row
// order), each element bf16(f32(d) * q).
cudaError_t launch_dequant_tiles(const uint8_t *w, int n_tiles, int kc, __nv_bfloat16 *out, cudaStream_t stream);

// Deterministic split-K reduction: y[m, j] = act(sum_s P[s][m][row(j)] + bias)
// with the splits summed in order (GLU: value row and gate row of column j).
struct SplitkReduceParams {
  const float *partials;
  int splits;
  int M;
  int ldp;
  int64_t n_out;
  int glu;
  const float *bias;
  int epi;
  void *y;
  int y_dtype;
  int64_t ldy;
};
cudaError_t launch_splitk_reduce(const SplitkReduceParams &p, cudaStream_t stream);

// f32 -> bf16 planes: hi = bf16(x), lo = bf16(x - hi) (lo may be null); rows
// of k_pad elements, zero beyond K.  Also used for bf16 -> bf16 copies when a
// caller's bf16 activations are not TMA-aligned.
cudaError_t launch_split_x(const void *x, int x_dtype, int64_t ldx, int64_t M, int64_t K,
                           int64_t k_pad, __nv_bfloat16 *hi, __nv_bfloat16 *lo, cudaStream_t stream);

// QTiled semantics (MatMul::from_qtensor, src/fast_matmul.rs:71-125): x
// quantized per 32 to Q8_0, per-block int8 dot products scaled by both f16
// scales and summed in block order (nq8_qtiled.cu).
struct QtiledParams {
  const uint8_t *w;  // packed tiles (not GLU-packed)
  int n_tiles, kc;
  int64_t N;
  int M;
  const int8_t *xq;  // [M][kc * 64] quantized activations
  const float *dx;   // [M][kc * 2] their Q8_0 scales (f16 values)
  const float *bias;
  int epi;           // NONE, SILU, GELU_ERF or RELU
  void *y;
  int y_dtype;
  int64_t ldy;
};
// Workspace bytes of the quantized activations of M rows (int8 rows, then the
// f32 scales at the returned offset's 256-byte-aligned split).
size_t qtiled_x_bytes(int64_t M, int kc);
cudaError_t launch_qtiled_quantize(const void *x, int x_dtype, int64_t ldx, int64_t M, int64_t K, int kc, int8_t *xq,
                                   float *dx, cudaStream_t stream);
cudaError_t launch_qtiled(const QtiledParams &p, cudaStream_t stream);

// conv1d / conv_transpose1d glue (nq8_conv.cu).
// Implicit conv1d operands: token-major planes hi[t][c] = bf16(leaky(x[c][t]))
// (lo = bf16(v - hi) for f32 x; lo may be null), rows of c_in elements.
cudaError_t launch_conv_tokens(const void *x, int x_dtype, int64_t ldx, int c_in, int t_in, float slope,
                               __nv_bfloat16 *hi, __nv_bfloat16 *lo, cudaStream_t s);
// Polyphase weight of a conv_transpose1d from its transposed GEMM form src
// [c_out K][c_in] (rows (co, j), ld_src elements): dst row co * s + r, column
// i c_in + ci = src[co K + r + s i][ci] when r + s i < K, else 0; rows up to
// `rows` (zero past c_out * s).
cudaError_t launch_conv_poly_weight(const __nv_bfloat16 *src, int64_t ld_src, int c_out, int K, int s, int c_in,
                                   int taps, int rows, __nv_bfloat16 *dst, cudaStream_t stream);
// Tap-major copy of a conv weight: dst[r][j c_in + ci] = src[r][ci K + j] for
// rows r < rows (src rows ld_src elements, dst rows K c_in).
cudaError_t launch_conv_tap_weight(const __nv_bfloat16 *src, int64_t ld_src, int rows, int c_in, int K,
                                   __nv_bfloat16 *dst, cudaStream_t s);
// rows[t][e] = leaky(x[e / K][t * stride - pad + (e % K) * dil]) for e < c_in * K,
// zero up to ld; x NCW with row stride ldx; a_dtype 0 f32, 1 bf16.
cudaError_t launch_im2col(const void *x, int x_dtype, int64_t ldx, int c_in, int t_in, int K, int stride, int pad,
                          int dil, float slope, int t_out, int64_t ld, int a_dtype, void *rows, cudaStream_t s);
// y[c][t] = src[t][c] (NCW output from token-major rows).
cudaError_t launch_transpose_out(const void *src, int src_dtype, int64_t lds, int rows_t, int cols_c, void *y,
                                 int y_dtype, int64_t ldy, cudaStream_t s);
// conv_transpose1d overlap-add of GEMM columns cols[t_in][c_out * K] (f32).
cudaError_t launch_col2im(const float *cols, int64_t ldc, int t_in, int c_out, int K, int stride, int pad, int t_out,
                          const float *bias, int epi, void *y, int y_dtype, int64_t ldy, cudaStream_t s);

cudaError_t launch_wait_timeout_probe(DevCtl ctl, cudaStream_t stream);

}  // namespace nq
