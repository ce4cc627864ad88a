/*
 * nq8.h -- C ABI of the B200 (sm_100a) GGUF Q8_0 contraction library, libnq8.so.
 *
 * Drop-in boundary for nspeech's Q8_0 matmul path.  Every entry point lists
 * the reference interface it replaces (paths relative to the dropbox/nspeech
 * source tree).  Plain C types only: device pointers are `void*`/`float*`,
 * a CUDA stream is passed as `void*` (NULL = legacy default stream).
 *
 * Conventions
 *   - Every function returns NQ_OK (0) or a negative NQ_ERR_* code; the
 *     message of the last failure on the calling thread is kept for
 *     nq_last_error().  No entry point falls back to a CPU path.
 *   - Weights are opaque handles owned by the library (device memory,
 *     immutable after creation, safe to share across threads/streams).
 *   - Activations x, outputs y and bias live in caller-owned device memory
 *     (the `enc_*` convention of src/triton_kernels.rs:862-1397).
 *   - The library owns a per-(device, stream) workspace (activation split
 *     planes, partial sums, work counters).  It grows on demand,
 *     so the first call of a given size on a stream may cudaMalloc; make that
 *     call once before capturing the stream into a CUDA graph.
 *   - Calls on different streams may run concurrently; calls on one stream
 *     are ordered by the stream.
 *
 * Numerics: y = act(x . bf16(dequant(W))^T + bias) with f32 accumulation, the
 * FbgemmBf16Op semantics of src/fast_matmul.rs:138-167 (weights rounded to
 * bf16 after Q8_0 dequantization).  f32 activations are carried at f32
 * precision (split into two bf16 planes); bf16 activations are used as is.
 */
#ifndef NQ8_H
#define NQ8_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define NQ_OK 0
#define NQ_ERR_ARG (-1)         /* null pointer, unknown enum value */
#define NQ_ERR_SHAPE (-2)       /* K % 32 != 0, last dim != K, GLU with odd N, ... */
#define NQ_ERR_ALIGN (-3)       /* pointer or leading dimension misaligned */
#define NQ_ERR_DTYPE (-4)       /* unsupported dtype (GGUF tensor not Q8_0, ...) */
#define NQ_ERR_CUDA (-5)        /* a CUDA runtime call failed */
#define NQ_ERR_TIMEOUT (-6)     /* a kernel's bounded wait ran out (device status) */
#define NQ_ERR_FORMAT (-7)      /* malformed GGUF file */
#define NQ_ERR_IO (-8)          /* file open / mmap failure */
#define NQ_ERR_NOT_INIT (-9)    /* nq_init was not called on this thread's device */
#define NQ_ERR_UNSUPPORTED (-10)/* e.g. GLU epilogue on a weight not packed for it */
#define NQ_ERR_DEVICE (-11)     /* device status word reported a kernel-side error */

/* ---- element types of activations / outputs ---------------------------- */
#define NQ_F32 0
#define NQ_BF16 1

/* ---- fused epilogues (applied after the bias add) ----------------------- */
#define NQ_EPI_NONE 0
#define NQ_EPI_SILU 1        /* Parakeet FFN w1 (src/parakeet/fast_conformer.rs:207) */
#define NQ_EPI_GELU_ERF 2    /* Moonshine encoder fc1 (src/moonshine/encoder.rs:105) */
#define NQ_EPI_GLU_SIGMOID 3 /* pointwise_conv1: a*sigmoid(b) (fast_conformer.rs:479-484) */
#define NQ_EPI_GLU_SILU 4    /* Moonshine decoder fc1: x*silu(gate) (moonshine/decoder.rs:403-410) */
#define NQ_EPI_RELU 5        /* subsampling pointwise convs (fast_conformer.rs:180-183) */

/* ---- weight packing flags ----------------------------------------------- */
#define NQ_PACK_DEFAULT 0
/* Rows [0, N/2) are the value half and [N/2, N) the gate half of a GLU
 * projection; they are interleaved per 128-row tile so that the GLU epilogues
 * fuse into the matmul.  Required for NQ_EPI_GLU_*; output width is N/2. */
#define NQ_PACK_GLU 1
/* Compute with the QTiled semantics of MatMul::from_qtensor
 * (src/fast_matmul.rs:184, dispatched to QTiledOp at :212; QTiledOp::cpu_fwd
 * :71-125 over tiled_matmul_inner :30-62): every nq_linear call quantizes the
 * activation rows per 32 elements to Q8_0 (ggml rule: d = amax / 127,
 * q = roundf(x / d), d rounded to f16) and computes
 *   y[m, n] = sum over blocks b, in order, of ((float)sumi_b * d_w) * d_x
 * with the exact int8 block dot products sumi_b, then bias and activation.
 * Without the flag a weight computes FbgemmBf16Op's semantics (below).  Not
 * combinable with NQ_PACK_GLU; nq_gemv_noalloc and nq_gemv_resadd_ln reject
 * it. */
#define NQ_MODE_QTILED 2

/* ---- device status bits (nq_status) -------------------------------------- */
#define NQ_DEV_TIMEOUT_PRODUCER 0x1
#define NQ_DEV_TIMEOUT_CONSUMER 0x2
#define NQ_DEV_TIMEOUT_MMA 0x4
#define NQ_DEV_TIMEOUT_EPILOGUE 0x8
#define NQ_DEV_TIMEOUT_DRAIN 0x10

typedef struct nq_weight nq_weight;

/* Bind the calling thread to a device and create its context (status word,
 * tensor-map entry point).  Per process, per GPU.  Replaces the device probe
 * of src/parakeet/mod.rs:309-325 (get_device). */
int nq_init(int device_ordinal);

/* Library version string, e.g. "nq8 0.1 sm_100a". */
const char *nq_version(void);

/* Upload a GGUF Q8_0 weight of logical shape [n, k] (GGUF ne0 = k): n*k/32
 * blocks of 34 bytes (f16 d, 32 x int8), host memory or an mmap.  Repacks once
 * into the tiled HBM layout.  Replaces MatMul::from_qtensor
 * (src/fast_matmul.rs:184) and EncoderBackend::upload_matmul_weight
 * (src/moonshine/gpu_encoder.rs:33-35). */
int nq_weight_from_q8_0(const void *blocks, int64_t n, int64_t k, int flags, nq_weight **out);

/* Upload an f32 [n, k] weight.  A tensor dequantized from Q8_0 (the way the
 * reference calls it: new_mm, src/moonshine/encoder.rs:29-39) re-quantizes
 * losslessly and is stored as Q8_0.  Any other finite tensor is kept at bf16
 * precision (round to nearest even), as the reference's PackedMatrixBf16
 * packing does: a bf16-only weight, which every nq_linear call runs on the
 * bf16 tensor-core GEMM (M <= 16 included) and which has no Q8_0 form
 * (nq_weight_to_q8_0, nq_weights_fuse, nq_gemv_noalloc, nq_gemv_resadd_ln
 * and NQ_MODE_QTILED reject it).  Either way y = x . bf16(W)^T with f32
 * accumulation.  NaN or infinite elements fail with NQ_ERR_DTYPE.
 * Replaces MatMul::from_tensor (src/fast_matmul.rs:191-208). */
int nq_weight_from_f32(const float *w, int64_t n, int64_t k, int flags, nq_weight **out);

/* mmap a GGUF v2/v3 file, find `tensor_name`, check it is Q8_0 and 2-D, and
 * upload it.  Replaces the mmap GGUF loader + QTensor path of
 * src/parakeet/transducer.rs:1759-1865. */
int nq_weight_from_gguf(const char *path, const char *tensor_name, int flags, nq_weight **out);

/* Host-only: parse a GGUF file and report tensor `tensor_name`'s ggml type
 * id (Q8_0 = 8) and its 2-D shape [n, k] (k = ne0).  No device work. */
int nq_gguf_tensor_info(const char *path, const char *tensor_name, int *ggml_type, int64_t *n, int64_t *k);

/* Concatenate weights along N (fused QKV [q;k;v], or [value; gate] with
 * NQ_PACK_GLU) into a new handle; all must share K.  Mirrors the fused QKV
 * upload of src/moonshine/gpu_encoder.rs:276-292. */
int nq_weights_fuse(const nq_weight *const *ws, int count, int flags, nq_weight **out);

/* Copy a weight back to GGUF Q8_0 blocks (n*k/32*34 bytes of host memory). */
int nq_weight_to_q8_0(const nq_weight *w, void *blocks_out);

int nq_weight_shape(const nq_weight *w, int64_t *n, int64_t *k, int *flags);
void nq_weight_free(nq_weight *w);
/* keep != 0: dequantize the weight once into an owned bf16 copy (2 bytes per
 * element, next to the Q8_0 tiles) that every later GEMM with M >= 128 reads
 * directly -- the reference's pre-dequantized MatMul::PackedBf16 /
 * FbgemmBf16Op weights (src/fast_matmul.rs:127-167, :176-226); the values
 * and results are the same as without it.  keep == 0 frees the copy (after a
 * device synchronize).  GEMV and M < 128 calls keep reading the Q8_0 tiles.
 * Synchronous; call on the weight's device. */
int nq_weight_keep_bf16(nq_weight *w, int keep);

/* y[m, :] = act(x[m, :K] . W^T + bias), m in [0, M).
 *   x: device, x_dtype NQ_F32 | NQ_BF16, row stride ldx elements (>= K).
 *   bias: device f32 [N] or NULL.  epilogue: NQ_EPI_*.
 *   y: device, y_dtype NQ_F32 | NQ_BF16, row stride ldy (>= N_out; N_out = N/2
 *      for GLU epilogues).  M = 0 is a no-op.
 * M <= 16 runs the GEMV kernel (dynamically scheduled units of k, fixed-order
 * sum of their partials), larger M the tcgen05 GEMM.
 * Replaces MatMul::forward / FbgemmBf16Op::cpu_fwd (src/fast_matmul.rs:
 * 138-167, 210-226) and QLinear::forward (src/parakeet/quantized_layers.rs:
 * 31-38). */
int nq_linear(const nq_weight *w, const void *x, int x_dtype, int64_t m, int64_t ldx,
              const float *bias, int epilogue, void *y, int y_dtype, int64_t ldy, void *stream);

/* Named dispatch entry points of src/triton_kernels.rs (contiguous rows). */
/* triton_matmul :170-211 / enc_matmul :1205-1231: c = a . W^T */
int nq_matmul(const nq_weight *w, const void *a, int a_dtype, void *c, int c_dtype, int64_t m,
              void *stream);
/* triton_matmul_bias :217-260 / enc_matmul_bias :1233-1260 */
int nq_matmul_bias(const nq_weight *w, const void *a, int a_dtype, const float *bias, void *c,
                   int c_dtype, int64_t m, void *stream);
/* triton_matmul_bias_gelu :266-309 / enc_matmul_bias_gelu :1262-1289 */
int nq_matmul_bias_gelu(const nq_weight *w, const void *a, int a_dtype, const float *bias,
                        void *c, int c_dtype, int64_t m, void *stream);
/* enc_gemv_splitk :1077-1115 and enc_gemv_splitk_bias :1036-1075 (bias may be
 * NULL); x is one row. */
int nq_gemv_splitk(const nq_weight *w, const void *x, int x_dtype, const float *bias, void *out,
                   int out_dtype, void *stream);
/* enc_gemv_glu_splitk :1163-1202: out = silu(gate) * value, W packed NQ_PACK_GLU */
int nq_gemv_glu_splitk(const nq_weight *w, const void *x, int x_dtype, const float *bias,
                       void *out, int out_dtype, void *stream);
/* enc_gemv_qkv_splitk :1117-1161: three projections of one row in one launch
 * sequence; weights must share K.  Outputs q, k, v are separate buffers. */
int nq_gemv_qkv_splitk(const nq_weight *wq, const nq_weight *wk, const nq_weight *wv,
                       const void *x, int x_dtype, void *q, void *k, void *v, int out_dtype,
                       void *stream);
/* DecoderBackend::gemv_resadd_ln (src/moonshine/gpu_decoder.rs:67-70) with the
 * fused split-K reduce + residual add + LayerNorm of
 * kernels/moonshine_kernels.py:1109-1146: for each row m < M (M <= 16),
 *   y = x[m] . W^T + bias (bias may be NULL),
 *   res_out[m] = res_in[m] + y                     (f32; res_out may be res_in),
 *   norm_out[m] = LN(res_out[m]) * gamma + beta    (beta may be NULL).
 * LN uses the mean and biased variance of the row in f32 (the CPU decoder's
 * arithmetic; the Metal kernel's f16 round of y is not reproduced).  N <=
 * 8192, W not GLU-packed; residual rows of ld_res floats, output rows of
 * ld_out elements of out_dtype.  Two launches (the GEMV and its epilogue). */
int nq_gemv_resadd_ln(const nq_weight *w, const void *x, int x_dtype, int64_t m, int64_t ldx,
                      const float *bias, const float *res_in, float *res_out, int64_t ld_res,
                      const float *ln_gamma, const float *ln_beta, float eps, void *norm_out,
                      int out_dtype, int64_t ld_out, void *stream);
/* ---- decode chain ----------------------------------------------------------
 * The dependent M = 1 projections of a decoder token (the calls of
 * src/moonshine/decoder.rs through DecoderBackend::gemv and ::gemv_resadd_ln,
 * src/moonshine/gpu_decoder.rs:67-70), recorded once and run as ONE
 * cooperative kernel per token instead of two launches per call: a
 * persistent grid streams every step's weights, waits on device counters
 * between dependent steps, and computes the LayerNorm of a residual step in
 * the CTAs of the step that reads it.  No counterpart in the reference; each
 * step computes the corresponding nq_linear (M = 1) / nq_gemv_resadd_ln call
 * -- the same bf16 weight products -- with f32 sums in another fixed order
 * (deterministic; one CTA owns a whole 128-row tile).  Steps: Q8_0 weights
 * (no QTiled, no bf16-only), K and a residual step's N at most 4096, x bf16
 * (one row), y of a plain step
 * f32 or bf16, a residual step's LayerNorm output bf16.  Buffers are bound by
 * address when a step is added.  A step's input may be an external vector or
 * any earlier step's output; inputs that equal the previous residual step's
 * LayerNorm output are computed on load.  Rejected (NQ_ERR_UNSUPPORTED):
 * a step whose input overlaps its outputs, two residual steps in a row, and a
 * step that writes over the previous step's residual or LayerNorm output.
 * The first nq_chain_run uploads the chain (allocations, not capturable);
 * later runs are one launch each and may be captured in a CUDA graph.  Runs
 * of one chain must not overlap.  After a device status error (a bounded wait
 * ran out), nq_status re-arms the chain's counters. */
typedef struct nq_chain nq_chain;
int nq_chain_create(nq_chain **out);  /* on the current device */
/* y = act(W x + bias), as nq_linear with M = 1. */
int nq_chain_linear(nq_chain *c, const nq_weight *w, const void *x, const float *bias, int epilogue, void *y,
                    int y_dtype);
/* res_out = res_in + W x + bias; norm_out = LN(res_out) * gamma + beta (bf16),
 * as nq_gemv_resadd_ln with M = 1 (res_out may be res_in; norm_out may be
 * NULL when no later step or caller reads it). */
int nq_chain_gemv_resadd_ln(nq_chain *c, const nq_weight *w, const void *x, const float *bias, const float *res_in,
                            float *res_out, const float *ln_gamma, const float *ln_beta, float eps, void *norm_out);
int nq_chain_steps(const nq_chain *c);
int nq_chain_run(nq_chain *c, void *stream);
void nq_chain_free(nq_chain *c);  /* no run of the chain may be in flight */

/* No counterpart in the reference.  The GEMV of nq_linear (M <= 16 rows,
 * same arguments and result) without any allocation: its partial sums,
 * staged activations and work counter live in a static device array of this
 * library (4 MiB of partials, 2 MiB of bf16 activation planes and the
 * counter, per device) instead of the
 * per-stream workspace nq_linear grows with cudaMalloc.  For callers that
 * cannot allocate at call time: a streaming decoder step on a latency budget
 * (cudaMalloc / cudaFree can synchronize the device and stall every stream),
 * or a process running at a fixed device-memory cap where a workspace growth
 * could fail mid-stream.  Requires nq_init on the device.  The first call on
 * a device looks up the array's address (cudaGetSymbolAddress, which may load
 * the module), so make that first call before any stream capture.  Every
 * call on a device shares the one array and leaves its contents behind (the
 * counter is re-armed by each call): calls that overlap on the GPU -- on
 * two streams, or from two threads -- race and give wrong results; serialize
 * them.  A call whose partial sums or staged activations (f32 or
 * unaligned x, or K not a multiple of 64) exceed the array is rejected with
 * NQ_ERR_SHAPE before any launch; M > 16 too. */
int nq_gemv_noalloc(const nq_weight *w, const void *x, int x_dtype, int64_t m, int64_t ldx,
                    const float *bias, int epilogue, void *y, int y_dtype, int64_t ldy,
                    void *stream);

/* ---- Kokoro conv1d / conv_transpose1d (configs 4) -------------------------
 * One sequence, NCW layouts as the reference's decoder: x is [c_in][ldx]
 * (channel rows of >= t_in elements), y is [c_out][ldy].  x_leaky is the
 * slope of a leaky ReLU applied to x on load (1.0 = none), the fused
 * leaky_relu + conv variants of the reference (conv1d_lrelu001,
 * conv_transpose1d_lrelu).  bias (f32 [c_out], nullable) and epilogue
 * (NONE, SILU, GELU_ERF, RELU) apply to the output. */

/* Output frames of a conv1d: (t_in + 2 padding - dilation (kernel - 1) - 1) /
 * stride + 1, or a negative NQ_ERR_* code. */
int64_t nq_conv1d_out_len(int64_t t_in, int kernel, int stride, int padding, int dilation);

/* y[co][t] = act(bias[co] + sum over ci, j of W[co, ci * kernel + j] *
 * leaky(x[ci][t * stride - padding + j * dilation])), zero padding.  `w` is
 * the conv weight in its GGUF 2-D form [c_out, c_in * kernel] (n = c_out,
 * k = c_in * kernel): a Q8_0 weight, or a bf16-only one from
 * nq_weight_from_f32 when c_in * kernel is not a multiple of 32.  Lowered as
 * im2col -> nq_linear (tensor cores) -> transpose to NCW, the reference's GPU
 * lowering (im2col + matmul_bias), or, for stride-1 convs with c_in a multiple
 * of 64 and more than 16 output frames, as an implicit GEMM over a tap-major
 * bf16 copy of the weight (nq_set_conv_path).  That copy is built and kept on
 * the first such call with the weight, which therefore must not run under
 * stream capture (NQ_ERR_UNSUPPORTED).  Scratch: a per-stream conv workspace
 * (grows with cudaMalloc on first use of a size).  Replaces
 * KokoroGpuBackend::conv1d / conv1d_k / conv1d_lrelu001 / im2col +
 * matmul_bias (src/kokoro/gpu_backend.rs:59-110; kernels conv1d_k and
 * im2col_conv1d, kernels/kokoro_kernels.py:182,426). */
int nq_conv1d(const nq_weight *w, const void *x, int x_dtype, int64_t c_in, int64_t t_in, int64_t ldx, int kernel,
              int stride, int padding, int dilation, float x_leaky, const float *bias, int epilogue, void *y,
              int y_dtype, int64_t ldy, void *stream);

/* Output frames of a conv_transpose1d: (t_in - 1) stride - 2 padding + kernel
 * + output_padding, or a negative NQ_ERR_* code. */
int64_t nq_conv_transpose1d_out_len(int64_t t_in, int kernel, int stride, int padding, int output_padding);

/* The weight of a conv_transpose1d from its (dequantized) values in the
 * reference's layout [c_in][c_out][kernel] (ConvTranspose1d, groups 1),
 * stored transposed as a bf16-only weight [c_out * kernel, c_in] (values
 * rounded to bf16, the fast_matmul packing). */
int nq_conv_transpose1d_weight(const float *w, int64_t c_in, int64_t c_out, int kernel, nq_weight **out);

/* y[co][t] = act(bias[co] + sum over ci, j with t = ti * stride - padding + j
 * of W[ci][co][j] * leaky(x[ci][ti])).  For c_in a multiple of 64 (and more
 * than 16 input positions reaching the output) one polyphase implicit GEMM:
 * output phase r = (t + padding) mod stride is a stride-1 conv over the input
 * with taps r, r + stride, ..., computed against a polyphase bf16 copy of the
 * weight built on the first such call (not under stream capture).  Otherwise
 * (or with nq_set_conv_path(NQ_CONV_IM2COL)) one GEMM to the columns
 * [t_in][c_out * kernel] (f32), then an overlap-add that sums each output's
 * taps in ascending j.  Both are deterministic.  Replaces
 * KokoroGpuBackend::conv_transpose1d / conv_transpose1d_lrelu
 * (src/kokoro/gpu_backend.rs:72-81; decoder.rs generator.ups). */
int nq_conv_transpose1d(const nq_weight *w, const void *x, int x_dtype, int64_t c_in, int64_t t_in, int64_t ldx,
                        int kernel, int stride, int padding, int output_padding, float x_leaky, const float *bias,
                        int epilogue, void *y, int y_dtype, int64_t ldy, void *stream);

/* ---- FastConformer encoder (the caller of the Q8_0 path for configs 2/5) ---
 * Mirrors FastConformerConfig (src/parakeet/fast_conformer.rs:31-45) and
 * FastConformerEncoder::forward (:1072-1104, blocks :967-999): dw-striding
 * 8x subsampling, x*sqrt(d), relative positions, then per layer macaron FFN
 * (x0.5), rel-pos MHSA, conv module (pw1+GLU, depthwise, BN, SiLU, pw2),
 * FFN, norm_out.  Every contraction with a rank-2 / pointwise weight runs on
 * the Q8_0 kernels with bf16 activations; the residual stream is f32.
 * Batches of padded segments reproduce per-segment results (masks). */
typedef struct nq_encoder_config {
  int feat_in;      /* log-mel bins (128) */
  int d_model;      /* 1024 (512 also supported); head dim must be 128 */
  int n_heads;      /* 8 */
  int ff_mult;      /* 4 */
  int n_layers;     /* 24 */
  int conv_kernel;  /* 9 (odd, <= 31) */
  int sub_channels; /* 256 */
  int scale_input;  /* 1: multiply the subsampled input by sqrt(d_model) */
} nq_encoder_config;

typedef struct nq_encoder nq_encoder;

/* Empty encoder bound to the current device; fill with nq_encoder_set_tensor
 * or nq_encoder_load_gguf, then nq_encoder_finalize. */
int nq_encoder_create(const nq_encoder_config *cfg, nq_encoder **out);

/* Stage one tensor by its reference name (e.g.
 * "encoder.layers.3.self_attn.q_proj.weight", the names produced by
 * remap_nemo_tensor_name, src/parakeet/transducer.rs:1279-1302).
 * ggml_type 0 = F32 data, 8 = Q8_0 blocks; dims outermost first (candle
 * order, e.g. a linear weight is [out, in]).  Q8_0 matrices given as F32 are
 * quantized with ggml semantics.  Host memory; copied. */
int nq_encoder_set_tensor(nq_encoder *enc, const char *name, int ggml_type, const void *data,
                          const int64_t *dims, int n_dims);

/* Stage every "encoder.*" tensor of a GGUF file (Q8_0 or F32). */
int nq_encoder_load_gguf(nq_encoder *enc, const char *path);

/* Check completeness, fill the defaults the reference loader adds (zero
 * biases, BN running mean 0 / var 1: src/parakeet/transducer.rs:1955-1996),
 * fuse Q/K/V, pack the pointwise_conv1 weight for the fused GLU, upload. */
int nq_encoder_finalize(nq_encoder *enc);

/* Encoder frames produced from t_mel input frames (three stride-2 stages). */
int nq_encoder_out_frames(int t_mel);

/* mel: device f32 [batch, t_mel, feat_in]; lengths: host int32 [batch] valid
 * mel frames per segment (<= t_mel; NULL = all t_mel).  out: device f32
 * [batch, T, d_model] with T = nq_encoder_out_frames(t_mel), frames beyond a
 * segment's own length zeroed; out_lengths (host, may be NULL) receives the
 * per-segment encoder lengths.  Replaces TransducerModel::run_encoder
 * (src/parakeet/transducer.rs:387-404) for a batch of VAD segments.
 * Each stream gets its own activation arena (allocated on its first
 * forward, grown for larger batches): forwards on one stream run in stream
 * order, forwards on different streams share only the weights and may run
 * concurrently (two streams fill the GPU while one forward's kernels leave
 * SMs idle). */
int nq_encoder_forward(nq_encoder *enc, const float *mel, const int32_t *lengths, int batch, int t_mel,
                       float *out, int32_t *out_lengths, void *stream);

/* Same with host buffers: copies mel in and the output back on `stream`
 * (pinned host memory recommended) and synchronizes it. */
int nq_encoder_forward_host(nq_encoder *enc, const float *mel_host, const int32_t *lengths, int batch,
                            int t_mel, float *out_host, int32_t *out_lengths, void *stream);

/* Queued form of nq_encoder_forward_host for a stream of batches (configs[4]:
 * many VAD segments); no counterpart in the reference, whose run_encoder is
 * synchronous.  Enqueues the copy of mel_host to the device, the forward on
 * `stream` and the copy of the output to out_host, then returns: the copies
 * run on the encoder's own copy streams and overlap the forwards of the
 * neighbouring calls (two device staging slots, event-ordered).  mel_host and
 * out_host must be pinned host memory and stay untouched until
 * nq_encoder_wait returns; out_lengths is filled before this returns.
 * Calls from several threads are serialized by the encoder (they share its
 * two staging slots). */
int nq_encoder_forward_host_async(nq_encoder *enc, const float *mel_host, const int32_t *lengths, int batch,
                                  int t_mel, float *out_host, int32_t *out_lengths, void *stream);
/* Block until every queued nq_encoder_forward_host_async output is in host memory. */
int nq_encoder_wait(nq_encoder *enc);

/* Number of kernels nq_encoder_forward launches for (batch, t_mel). */
int nq_encoder_launch_count(const nq_encoder *enc, int batch, int t_mel);

void nq_encoder_free(nq_encoder *enc);

/* ---- per-kernel timing --------------------------------------------------
 * When enabled, every Q8_0 kernel launch of this process is bracketed by CUDA
 * events on its own stream (the per-op timing of the reference's
 * TRITON_ENCODER_PROFILE / forward_profile, src/moonshine/gpu_encoder.rs:
 * 367-369,508).  Kernel classes: */
#define NQ_KCLASS_GEMM 0    /* tcgen05 GEMM (M > 16) */
#define NQ_KCLASS_GEMV 1    /* GEMV (M <= 16), its partial-sum pass included */
#define NQ_KCLASS_DEQUANT 2 /* Q8_0 -> bf16 weight pass of the large-M GEMM */
#define NQ_KCLASS_REDUCE 3  /* split-K reduction after a split GEMM */
#define NQ_KCLASS_ATTENTION 4 /* encoder relative-position attention; FLOPs
                               * 6 B Tp^2 D (QK^T, the relative band, PV over
                               * padded frames), bytes q, k, v, rel. keys, out */
#define NQ_KCLASS_NORM 5      /* encoder residual add + LayerNorm; no FLOPs
                               * counted, bytes per token row: the f32 residual
                               * read and written, the added row read, the
                               * bf16 normalized row written */
int nq_profile_enable(int on);
/* Synchronizes the recorded events and reports for one class: launches,
 * summed device ms, summed algorithmic FLOPs (2MNK) and bytes
 * (N*K*34/32 + M*K*sx + M*N*sy + 4N).  reset != 0 clears that class's
 * records. */
int nq_profile_read(int kernel_class, int64_t *launches, double *total_ms, double *flops, double *bytes,
                    int reset);

/* Kernels this library has launched in this process (all devices and
 * streams); reset != 0 returns the count and zeroes it.  No counterpart in
 * the reference: launch accounting for benchmarks and tests. */
int nq_launch_counter(int64_t *count, int reset);

/* Thread-local message of the last failure ("" if none); returns its length. */
int nq_last_error(char *buf, int len);

/* Synchronize `stream`, then read and clear this device's status word.
 * Returns NQ_OK, or NQ_ERR_TIMEOUT with the NQ_DEV_* bits in *bits. */
int nq_status(void *stream, int *bits);

/* Cycle budget of every bounded wait in the kernels (default ~2^31 cycles,
 * about one second).  Lowered only by tests. */
int nq_set_wait_limit(int64_t cycles);

/* Which kernel serves a GEMM call (M > 16).  No counterpart in the
 * reference: a B200 dispatch knob.  AUTO (default) dequantizes the weight
 * once into scratch and runs the bf16 tcgen05 GEMM from 128 tokens, and
 * runs the fused in-kernel-dequantizing GEMM below that; FUSED and DEQUANT
 * force one of them (tests use this to cover both on the same shapes).
 * Process-wide; returns NQ_ERR_ARG for an unknown value. */
#define NQ_GEMM_AUTO 0
#define NQ_GEMM_FUSED 1
#define NQ_GEMM_DEQUANT 2
int nq_set_gemm_path(int path);

/* Tokens per 2-SM work unit of the dequantize-once (bf16 tcgen05) GEMM: 64,
 * 128 or 256, or 0 (default) for a per-call choice by a cost model (narrower
 * units give calls with few 256-token tiles more units for the SM pairs).
 * No counterpart in the reference: a B200 dispatch knob.  Process-wide;
 * returns NQ_ERR_ARG for other values. */
int nq_set_gemm_unit_tokens(int tokens);

/* Tail split of the dequantize-once GEMM.  No counterpart in the reference: a
 * B200 dispatch knob.  When a call's output tiles (256 weight rows x the unit
 * width in tokens) leave the last round of SM pairs partly idle, the tiles of
 * that round are cut into k pieces that run on the idle pairs; the last piece
 * of each tile to finish adds the pieces in piece order (deterministic) and
 * writes the output, in the same launch.  0 (default): a cost model decides
 * per call; 1: never; 2..16: that many pieces whenever a partial round exists
 * (tests).  Results differ from the unsplit sums only by f32 summation order.
 * A forced piece count runs on 256-token units unless nq_set_gemm_unit_tokens
 * sets a width.  Process-wide. */
int nq_set_gemm_tail_split(int mode);

/* Which kernel runs the encoder's relative-position attention.  No
 * counterpart in the reference: a B200 dispatch knob.  TCGEN05 (default):
 * tcgen05 MMAs with the scores and the output in tensor memory; MMA_SYNC:
 * the earlier warp-level mma.sync kernel (kept for comparison).  Both compute
 * the same attention; results differ by f32 / bf16 rounding only.
 * Process-wide; returns NQ_ERR_ARG for other values. */
#define NQ_ATTENTION_TCGEN05 0
#define NQ_ATTENTION_MMA_SYNC 1
int nq_set_attention_kernel(int kernel);

/* Which form serves a GEMV call (M <= 16: nq_linear, the named GEMV entries,
 * nq_gemv_resadd_ln, nq_gemv_noalloc).  No counterpart in the reference: a
 * B200 dispatch knob.  SPLIT: k cut into units over all SMs (dynamic work
 * counter), then a reduce launch -- two launches, best for large weights.
 * CLUSTER: each 128-row tile's k over a thread-block cluster of up to 8 CTAs,
 * the partial sums added through distributed shared memory -- one launch;
 * a residual + LayerNorm call's LayerNorm is computed by the cluster that
 * finishes last.  AUTO (default): CLUSTER for calls of at most 8 rows
 * without the residual + LayerNorm epilogue whose CTAs get at most 5 k
 * chunks, with all CTAs in one wave (the latency-bound decoder projections),
 * else SPLIT.  CLUSTER forces
 * the cluster form wherever it applies (at most 8 chunks per CTA), residual
 * calls included; elsewhere SPLIT runs.  The two forms add the same products
 * in different f32 orders.  Process-wide; returns NQ_ERR_ARG for other
 * values. */
#define NQ_GEMV_AUTO 0
#define NQ_GEMV_SPLIT 1
#define NQ_GEMV_CLUSTER 2
int nq_set_gemv_path(int path);

/* How nq_conv1d and nq_conv_transpose1d lower a convolution.  No
 * counterpart in the reference: a B200 dispatch knob.  AUTO (default):
 * stride-1 conv1d and conv_transpose1d whose c_in is a multiple of 64 (and
 * more than 16 output frames / input positions) run as implicit GEMMs
 * (token-major input planes, a tap-major or polyphase bf16 copy of the
 * weight, shifted-row loads, NCW output from the GEMM epilogue); other convs
 * as im2col + nq_linear + transpose, or column GEMM + overlap-add.  IM2COL
 * forces the second forms (tests compare the two).  Results differ by f32
 * summation order only.  Process-wide; returns NQ_ERR_ARG for other values. */
#define NQ_CONV_AUTO 0
#define NQ_CONV_IM2COL 1
int nq_set_conv_path(int path);

/* DEBUG ONLY -- a test hook for failure detection, not part of the matmul
 * API: launches a kernel that waits on an mbarrier nothing arrives on,
 * bounded by the wait limit; the kernel records NQ_DEV_TIMEOUT_CONSUMER and
 * returns, leaving the context usable.  No counterpart in the reference. */
int nq_debug_wait_timeout(void *stream);

#ifdef __cplusplus
}
#endif

#endif /* NQ8_H */
