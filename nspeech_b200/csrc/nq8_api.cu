// nq8_api.cu -- the C ABI of libnq8.so (declared in include/nq8.h).
//
// Host runtime around the kernels: per-device contexts (status word, driver
// entry point for tensor maps), immutable weight handles, a per-(device,
// stream) workspace, shape/alignment validation and the GEMV / GEMM dispatch.
// There is no CPU compute path: if a kernel cannot run, the call fails.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/nq8.h"
#include "nq8_attention.h"
#include "nq8_encoder.h"
#include "nq8_host.h"
#include "nq8_kernels.h"

struct nq_weight {
  int device = 0;
  int64_t n = 0, k = 0;
  int flags = 0;
  int n_tiles = 0, kc = 0;
  uint8_t *dev = nullptr;
  size_t bytes = 0;
  // Optional dequantized copy, bf16 [n_tiles * 128][kc * 64] in packed row
  // order (nq_weight_keep_bf16): the dequantize-once GEMM reads it instead of
  // dequantizing per call.
  __nv_bfloat16 *bf16 = nullptr;
  // bf16-only weight (no Q8_0 tiles, dev == nullptr): an f32 tensor that is not
  // a Q8_0 dequantization kept at bf16 precision (MatMul::from_tensor's
  // packing), or a transposed conv weight.  Every call runs the bf16 GEMM.
  bool bf16_only = false;
  // Tap-major bf16 copy for the implicit conv1d, [n_tiles * 128][tap_k *
  // tap_cin] with element (r, j tap_cin + ci) = W[r, ci tap_k + j]: built on the
  // first nq_conv1d call that takes that path, freed with the weight.
  mutable __nv_bfloat16 *tap = nullptr;
  mutable int64_t tap_cin = 0;
  mutable int tap_k = 0;
  // Polyphase copy of a conv_transpose1d weight for stride poly_s:
  // [ceil(c_out poly_s / 128) * 128][ceil(K / poly_s) * c_in], row
  // co * poly_s + r, column i c_in + ci = W[ci][co][r + poly_s i]; built on the
  // first nq_conv_transpose1d call that takes the implicit path, freed with
  // the weight.
  mutable __nv_bfloat16 *poly = nullptr;
  mutable int poly_s = 0;
};

struct nq_chain {
  int device = 0;
  struct Range {
    uintptr_t lo = 0, hi = 0;  // [lo, hi)
    bool overlaps(const Range &o) const { return lo < o.hi && o.lo < hi; }
  };
  std::vector<nq::ChainStep> steps;
  std::vector<Range> x_range, y_range, res_range;  // per step (empty ranges where absent)
  double flops = 0, bytes = 0;
  bool uploaded = false;
  int ctas = 0;
  nq::ChainStep *d_steps = nullptr;
  int *d_counters = nullptr;  // completed tiles per step
  size_t counter_bytes = 0;
};

namespace {

constexpr int kMaxDevices = 64;
constexpr int kSmCountB200 = 148;

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct Workspace {
  uint8_t *buf = nullptr;
  size_t bytes = 0;
  int *counters = nullptr;  // kCounterSlots ints, zero between calls
};
constexpr size_t kCounterSlots = 1 << 16;

struct DeviceCtx {
  bool ready = false;
  int *status = nullptr;
  int sm_count = kSmCountB200;
  EncodeTiledFn encode = nullptr;
  std::mutex mu;
  std::map<cudaStream_t, Workspace> ws;
  // Scratch of the conv entry points (im2col rows, GEMM outputs), separate from
  // `ws` so that the GEMM's own workspace growth cannot free it mid-call.
  std::map<cudaStream_t, Workspace> conv_ws;
  // Counters of the decode chains on this device (re-zeroed with the
  // workspace counters when a status bit reports a kernel that gave up).
  std::map<int *, size_t> chain_counters;
};

DeviceCtx g_ctx[kMaxDevices];
std::mutex g_init_mu;
long long g_wait_limit = 1LL << 31;
int g_gemm_path = NQ_GEMM_AUTO;
int g_gemm_unit_tokens = 0;  // 0: the kernel's default unit width
int g_attention_kernel = NQ_ATTENTION_TCGEN05;
int g_tail_split = 0;        // 0: cost model, 1: off, >= 2: that many pieces when a tail exists
int g_conv_path = NQ_CONV_AUTO;
int g_gemv_path = NQ_GEMV_AUTO;
std::mutex g_tap_mu;         // builds of weights' tap-major copies
// Token count from which a GEMM call dequantizes the weight once and runs
// the bf16 tensor-core GEMM (measured crossover on B200).
constexpr int64_t kDequantMinM = 128;
// Cost model of the bf16 GEMM's split-K choice, measured on B200: time of one
// 64-wide k step of a 256 x 256 pair unit within a full wave, and the split-K
// reduction's partial-sum traffic rate and fixed launch cost.
constexpr double kNsPerUnitStep = 390.0;
constexpr double kReduceBytesPerNs = 5000.0;
constexpr double kReduceLaunchNs = 3000.0;
// Tail split: each piece of a 256-token unit stores 128 KB of f32
// accumulators per CTA and the last piece reads every piece back from L2
// (about 130 GB/s per SM), modelled per piece; measured on B200 from 1024^3
// (no split 10.5 us, 4 pieces 15.3 us) and 2048 x 4096 -> 1024 (28.2 us,
// 2 pieces 22.8 us).  A narrower unit's piece moves width / 256 of it.
constexpr double kTailFixupNsPerPiece = 2200.0;
// Workspace counters: slot 0 is the GEMV work counter; the tail split's
// per-(tile, CTA, warp group) counters start here.
constexpr size_t kTailCounterBase = 64;
thread_local std::string t_err;

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  return fail(NQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int current_ctx(DeviceCtx **out, int *dev_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices || !g_ctx[dev].ready)
    return fail(NQ_ERR_NOT_INIT, "nq_init(%d) was not called", dev);
  *out = &g_ctx[dev];
  if (dev_out) *dev_out = dev;
  return NQ_OK;
}

// Grow-only workspace for `stream`; counters are zeroed once at allocation
// and re-armed by the kernels.  `conv` selects the conv entry points' scratch.
int get_workspace(DeviceCtx *ctx, cudaStream_t stream, size_t bytes, Workspace **out, bool conv = false) {
  std::lock_guard<std::mutex> lk(ctx->mu);
  Workspace &w = (conv ? ctx->conv_ws : ctx->ws)[stream];
  if (!w.counters) {
    cudaError_t e = cudaMalloc(&w.counters, kCounterSlots * sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(workspace counters)");
    e = cudaMemset(w.counters, 0, kCounterSlots * sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(workspace counters)");
  }
  if (w.bytes < bytes) {
    if (w.buf) {
      cudaError_t e = cudaStreamSynchronize(stream);
      if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize(workspace growth)");
      cudaFree(w.buf);
      w.buf = nullptr;
      w.bytes = 0;
    }
    size_t sz = std::max(bytes, static_cast<size_t>(16) << 20);
    cudaError_t e = cudaMalloc(&w.buf, sz);
    if (e != cudaSuccess) return fail(NQ_ERR_CUDA, "cudaMalloc(workspace %zu bytes): %s", sz, cudaGetErrorString(e));
    w.bytes = sz;
  }
  *out = &w;
  return NQ_OK;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int upload_packed(const uint8_t *blocks, int64_t n, int64_t k, int flags, nq_weight **out) {
  DeviceCtx *ctx = nullptr;
  int dev = 0;
  int rc = current_ctx(&ctx, &dev);
  if (rc) return rc;
  std::unique_ptr<nq_weight> w(new nq_weight);
  w->device = dev;
  w->n = n;
  w->k = k;
  w->flags = flags;
  w->n_tiles = nq::pack_n_tiles(n, flags);
  w->kc = nq::pack_k_chunks(k);
  w->bytes = static_cast<size_t>(w->n_tiles) * w->kc * nq::kTileBytes;
  std::vector<uint8_t> host(w->bytes);
  nq::pack_q8_0(blocks, n, k, flags, host.data());
  cudaError_t e = cudaMalloc(&w->dev, w->bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(weight)");
  e = cudaMemcpy(w->dev, host.data(), w->bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(w->dev);
    return cuda_fail(e, "cudaMemcpy(weight)");
  }
  *out = w.release();
  return NQ_OK;
}

// A bf16-only weight from f32 values [n, k] (rounded to bf16, packed row order).
int upload_bf16_only(const float *wf, int64_t n, int64_t k, int flags, nq_weight **out) {
  DeviceCtx *ctx = nullptr;
  int dev = 0;
  int rc = current_ctx(&ctx, &dev);
  if (rc) return rc;
  std::unique_ptr<nq_weight> w(new nq_weight);
  w->device = dev;
  w->n = n;
  w->k = k;
  w->flags = flags;
  w->n_tiles = nq::pack_n_tiles(n, flags);
  w->kc = nq::pack_k_chunks(k);
  w->bf16_only = true;
  const size_t elems = static_cast<size_t>(w->n_tiles) * nq::kPackRows * w->kc * nq::kPackK;
  std::vector<uint16_t> host(elems);
  nq::pack_bf16_rows(wf, n, k, flags, host.data());
  cudaError_t e = cudaMalloc(&w->bf16, elems * 2);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(bf16 weight)");
  e = cudaMemcpy(w->bf16, host.data(), elems * 2, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(w->bf16);
    return cuda_fail(e, "cudaMemcpy(bf16 weight)");
  }
  *out = w.release();
  return NQ_OK;
}

int check_weight_shape(int64_t n, int64_t k, int flags) {
  if (n <= 0 || k <= 0) return fail(NQ_ERR_SHAPE, "weight shape [%lld, %lld] must be positive", (long long)n, (long long)k);
  if (k % 32) return fail(NQ_ERR_SHAPE, "K=%lld is not a multiple of the Q8_0 block (32)", (long long)k);
  if (flags & ~(NQ_PACK_GLU | NQ_MODE_QTILED)) return fail(NQ_ERR_ARG, "unknown weight flags 0x%x", flags);
  if ((flags & NQ_PACK_GLU) && (flags & NQ_MODE_QTILED))
    return fail(NQ_ERR_UNSUPPORTED, "NQ_MODE_QTILED weights cannot be GLU-packed");
  if ((flags & NQ_PACK_GLU) && (n % 2)) return fail(NQ_ERR_SHAPE, "GLU weight needs an even N (got %lld)", (long long)n);
  if (n > (1LL << 31) || k > (1LL << 31)) return fail(NQ_ERR_SHAPE, "weight too large");
  return NQ_OK;
}

int make_tmap(DeviceCtx *ctx, CUtensorMap *map, const void *ptr, int64_t kdim, int64_t rows, int64_t ld_elems,
              int box_rows) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kdim), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_elems) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = ctx->encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return NQ_OK;
}

struct LinearArgs {
  const nq_weight *w;
  const float *bias;
  void *y;
  int64_t ldy;
};

int64_t out_width(const nq_weight *w) { return (w->flags & NQ_PACK_GLU) ? w->n / 2 : w->n; }

int validate(const nq_weight *w, const void *x, int x_dtype, int64_t m, int64_t ldx, int epilogue, const void *y,
             int y_dtype, int64_t ldy) {
  if (!w) return fail(NQ_ERR_ARG, "null weight");
  if (m < 0) return fail(NQ_ERR_SHAPE, "negative M");
  if (x_dtype != NQ_F32 && x_dtype != NQ_BF16) return fail(NQ_ERR_DTYPE, "x dtype %d unsupported", x_dtype);
  if (y_dtype != NQ_F32 && y_dtype != NQ_BF16) return fail(NQ_ERR_DTYPE, "y dtype %d unsupported", y_dtype);
  if (epilogue < NQ_EPI_NONE || epilogue > NQ_EPI_RELU) return fail(NQ_ERR_ARG, "unknown epilogue %d", epilogue);
  const bool glu_epi = epilogue == NQ_EPI_GLU_SIGMOID || epilogue == NQ_EPI_GLU_SILU;
  const bool glu_w = (w->flags & NQ_PACK_GLU) != 0;
  if (glu_epi && !glu_w) return fail(NQ_ERR_UNSUPPORTED, "GLU epilogue needs a weight packed with NQ_PACK_GLU");
  if (!glu_epi && glu_w) return fail(NQ_ERR_UNSUPPORTED, "weight packed with NQ_PACK_GLU needs a GLU epilogue");
  if (m == 0) return NQ_OK;
  if (!x || !y) return fail(NQ_ERR_ARG, "null activation or output pointer");
  if (ldx < w->k) return fail(NQ_ERR_SHAPE, "ldx=%lld < K=%lld", (long long)ldx, (long long)w->k);
  if (ldy < out_width(w)) return fail(NQ_ERR_SHAPE, "ldy=%lld < output width %lld", (long long)ldy, (long long)out_width(w));
  if (m > (1LL << 30)) return fail(NQ_ERR_SHAPE, "M too large");
  return NQ_OK;
}

// ------------------------------------------------------------ profiling
// Event pairs around each kernel launch while profiling is on; read back
// (synchronizing the events) by nq_profile_read.
struct ProfRecord {
  int kclass;
  cudaEvent_t start, stop;
  double flops, bytes;
};
struct Profiler {
  std::mutex mu;
  bool on = false;
  std::vector<ProfRecord> records;
  std::vector<cudaEvent_t> pool;
  cudaEvent_t take() {
    if (!pool.empty()) {
      cudaEvent_t e = pool.back();
      pool.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }
};
Profiler g_prof;

struct ProfScope {
  ProfRecord rec{};
  cudaStream_t stream;
  bool active = false;
  ProfScope(int kclass, cudaStream_t s, double flops, double bytes) : stream(s) {
    std::lock_guard<std::mutex> lk(g_prof.mu);
    if (!g_prof.on) return;
    rec = ProfRecord{kclass, g_prof.take(), g_prof.take(), flops, bytes};
    active = rec.start && rec.stop;
    if (active) cudaEventRecord(rec.start, stream);
  }
  ~ProfScope() {
    if (!active) return;
    cudaEventRecord(rec.stop, stream);
    std::lock_guard<std::mutex> lk(g_prof.mu);
    g_prof.records.push_back(rec);
  }
};

// ------------------------------------------------------------------ GEMV
// GEMV work plan: about two CTAs per SM, each owning one k split and a
// strided set of weight tiles (persistent), at least four k chunks per split
// when K allows, and at most as many chunks per split as the staged
// activation slice holds.
// The GEMV reads bf16 activation rows in place when they are 16-byte aligned
// rows of whole 64-wide chunks; otherwise split_x first writes zero-padded
// bf16 planes (hi, and lo for f32) to the workspace.
bool gemv_x_direct(const void *x, int x_dtype, int64_t ldx, int64_t k) {
  return x_dtype == NQ_BF16 && (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (ldx % 8 == 0) &&
         (k % nq::kPackK == 0);
}

size_t gemv_partial_bytes(const nq::GemvPlan &plan, int n_tiles, int64_t m) {
  return align_up(static_cast<size_t>(plan.upt) * m * n_tiles * nq::kPackRows * sizeof(float), 256);
}

// Decoder-step epilogue of a one-weight GEMV (nq_gemv_resadd_ln).
struct GemvResLn {
  const float *res_in;
  float *res_out;
  int64_t ld_res;
  const float *g;
  const float *b;
  float eps;
};

// Algorithmic FLOPs and bytes of `nprob` weights applied to M rows (the
// profiler's per-launch figures): 2MNK, and N*K*34/32 + M*K*sx + M*N*sy + 4N.
void linear_cost(const LinearArgs *args, int nprob, int64_t m, int x_dtype, int y_dtype, double *flops,
                 double *bytes) {
  *flops = 0;
  *bytes = 0;
  for (int i = 0; i < nprob; ++i) {
    const nq_weight *w = args[i].w;
    *flops += 2.0 * m * w->n * w->k;
    *bytes += w->n * (w->k / 32) * 34.0 + m * w->k * (x_dtype == NQ_F32 ? 4.0 : 2.0) +
              m * out_width(w) * (y_dtype == NQ_F32 ? 4.0 : 2.0) + (args[i].bias ? 4.0 * w->n : 0.0);
  }
}

int run_gemv(DeviceCtx *ctx, const LinearArgs *args, int nprob, const void *x, int x_dtype, int64_t m, int64_t ldx,
             int epilogue, int y_dtype, cudaStream_t stream, const GemvResLn *rl = nullptr) {
  const nq_weight *w0 = args[0].w;
  int total_tiles = 0;
  for (int i = 0; i < nprob; ++i) total_tiles += args[i].w->n_tiles;
  const int kc = w0->kc;
  const nq::GemvPlan plan = nq::gemv_plan(ctx->sm_count, total_tiles, kc, static_cast<int>(m));
  const bool splitx = x_dtype == NQ_F32;
  const bool direct = gemv_x_direct(x, x_dtype, ldx, w0->k);
  const int64_t k_pad = static_cast<int64_t>(kc) * nq::kPackK;

  // Workspace: [activation planes][partials of problem 0, 1, 2].
  const size_t plane = align_up(static_cast<size_t>(m) * k_pad * 2, 256);
  const size_t x_bytes = direct ? 0 : plane * (splitx ? 2 : 1);
  size_t part_bytes = 0;
  for (int i = 0; i < nprob; ++i) part_bytes += gemv_partial_bytes(plan, args[i].w->n_tiles, m);
  Workspace *ws = nullptr;
  int rc = get_workspace(ctx, stream, x_bytes + part_bytes, &ws);
  if (rc) return rc;

  nq::GemvParams p;
  std::memset(&p, 0, sizeof(p));
  size_t part_off = x_bytes;
  for (int i = 0; i < nprob; ++i) {
    const nq_weight *w = args[i].w;
    nq::GemvProblem &pr = p.prob[i];
    pr.w = w->dev;
    pr.n_tiles = w->n_tiles;
    pr.N = w->n;
    pr.glu = (w->flags & NQ_PACK_GLU) ? 1 : 0;
    pr.n_out = out_width(w);
    pr.bias = args[i].bias;
    pr.y = args[i].y;
    pr.ldy = args[i].ldy;
    pr.partials = reinterpret_cast<float *>(ws->buf + part_off);
    part_off += gemv_partial_bytes(plan, w->n_tiles, m);
  }
  p.sched = ws->counters;  // work counter, tile arrivals
  p.sm_count = ctx->sm_count;
  p.path = g_gemv_path;
  if (direct) {
    p.xh = static_cast<const __nv_bfloat16 *>(x);
    p.ldx = ldx;
  } else {
    __nv_bfloat16 *hi = reinterpret_cast<__nv_bfloat16 *>(ws->buf);
    __nv_bfloat16 *lo = splitx ? reinterpret_cast<__nv_bfloat16 *>(ws->buf + plane) : nullptr;
    cudaError_t e = nq::launch_split_x(x, x_dtype, ldx, m, w0->k, k_pad, hi, lo, stream);
    if (e != cudaSuccess) return cuda_fail(e, "split_x launch");
    p.xh = hi;
    p.xl = lo;
    p.ldx = k_pad;
  }
  p.M = static_cast<int>(m);
  p.epi = epilogue;
  p.y_dtype = y_dtype;
  p.nprob = nprob;
  p.kc = kc;
  p.unit = plan.unit;
  p.upt = plan.upt;
  p.units = plan.units;
  p.ctas = plan.ctas;
  if (rl) {
    p.res_in = rl->res_in;
    p.res_out = rl->res_out;
    p.ld_res = rl->ld_res;
    p.ln_g = rl->g;
    p.ln_b = rl->b;
    p.ln_eps = rl->eps;
  }
  p.ctl.status = ctx->status;
  p.ctl.wait_limit = g_wait_limit;
  double flops = 0, bytes = 0;
  linear_cost(args, nprob, m, x_dtype, y_dtype, &flops, &bytes);
  ProfScope ps(NQ_KCLASS_GEMV, stream, flops, bytes);
  cudaError_t e = nq::launch_gemv(p, plan.ctas, stream);
  if (e != cudaSuccess) return cuda_fail(e, "GEMV launch");
  return NQ_OK;
}

// ------------------------------------------------------------------ GEMM
// How one GEMM call (M > 16) is carried out.
struct GemmPlan {
  bool deq = false;      // dequantize-once path (dequant_tiles + K3), else fused K1
  bool cached = false;   // deq with the weight's kept bf16 copy: no dequantize launch
  bool split_x = false;  // activations staged to bf16 planes first (f32, or unaligned bf16)
  int bt = 256;          // tokens per pair unit
  int grid_m = 0, grid_n = 0, splits = 1, cps = 0, pairs = 1;
  int full_units = 0, tail_pieces = 1, tail_cps = 0;  // K3 tail split (tail_pieces > 1)
  int tail_tiles() const { return tail_pieces > 1 ? grid_m * grid_n - full_units : 0; }
  int launches() const { return 1 + (deq && !cached ? 1 : 0) + (splits > 1 ? 1 : 0) + (split_x ? 1 : 0); }
};

// Measured time of one 64-wide k step of a pair unit in a full wave, by unit
// width: it barely shrinks with the width, because the unit's 256-row weight
// tile (32 KB per pair and step) streams whole whatever the token count.
double unit_step_ns(int bt) { return bt >= 256 ? kNsPerUnitStep : bt >= 128 ? 360.0 : 330.0; }

// The bf16 GEMM (K3) at unit width bt: split-K or tail split with the least
// estimated time.  Full waves of units times their k steps, plus, when split,
// one write and one read of the f32 partials and the reduction launch; the
// tail split (256-token units) runs the R full rounds whole and cuts the L
// tiles of the last, partial round into S k pieces on S x L <= pairs pairs,
// the last piece of each tile summing them (no extra launch).  Returns the
// estimate.
// narrow_tail: the cost model may also tail-split 64- and 128-token units
// (f32 activations: two MMAs per k step, so a piece saves enough; measured
// on B200, configs[0] at M = 125 with f32 x: 81.9 -> 74.7 us, but with bf16 x
// 54.8 -> 56.7 us).  A forced split (nq_set_gemm_tail_split) always applies.
double plan_bf16_width(GemmPlan *gp, int bt, int64_t m, int kc, int ldp, bool splitk = true,
                       bool narrow_tail = false) {
  GemmPlan &g = *gp;
  g.bt = bt;
  g.grid_m = static_cast<int>((m + g.bt - 1) / g.bt);
  const int tiles = g.grid_m * g.grid_n;
  const double step = unit_step_ns(bt);
  double best = 1e300;
  const int max_splits = splitk ? std::max(1, std::min(8, kc / 4)) : 1;
  for (int sp = 1; sp <= max_splits; ++sp) {
    const int cps = (kc + sp - 1) / sp;
    const int splits = (kc + cps - 1) / cps;
    if (splits != sp) continue;
    const int64_t units = static_cast<int64_t>(tiles) * splits;
    const int64_t rounds = (units + g.pairs - 1) / g.pairs;
    double t = static_cast<double>(rounds) * cps * step;
    if (splits > 1) t += 2.0 * splits * static_cast<double>(m) * ldp * 4.0 / kReduceBytesPerNs + kReduceLaunchNs;
    if (t < best) {
      best = t;
      g.splits = splits;
      g.cps = cps;
    }
  }
  const int R = tiles / g.pairs, L = tiles - R * g.pairs;
  g.full_units = tiles;
  g.tail_pieces = 1;
  g.tail_cps = 0;
  if (g_tail_split != 1 && L > 0 && (g.bt == 256 || narrow_tail || g_tail_split >= 2)) {
    const double fixup = kTailFixupNsPerPiece * g.bt / 256.0;
    const int s_cap = std::min(std::min(g.pairs / L, kc / 2), 16);
    double best_tail = 1e300;
    int pick = 1, pick_cps = kc;
    for (int sp = 2; sp <= s_cap; ++sp) {
      const int cps = (kc + sp - 1) / sp;
      if ((kc + cps - 1) / cps != sp) continue;
      const double t = (static_cast<double>(R) * kc + cps) * step + (sp + 1) * fixup;
      if (g_tail_split >= 2 ? sp == g_tail_split : t < best_tail) {
        best_tail = t;
        pick = sp;
        pick_cps = cps;
      }
    }
    if (pick > 1 && (g_tail_split >= 2 || best_tail < best)) {
      g.splits = 1;
      g.cps = kc;
      g.tail_pieces = pick;
      g.tail_cps = pick_cps;
      g.full_units = R * g.pairs;
      best = best_tail;
    }
  }
  return best;
}

// Unit width of a bf16 GEMM call: the one with the least estimated time,
// unless a width or a tail split is forced.  Narrow units give a call with
// few 256-token tiles more units for the SM pairs, at a k step that costs
// nearly as much (the weight tile streams whole either way).
GemmPlan plan_bf16(const GemmPlan &g0, int64_t m, int kc, int ldp, bool splitk, bool narrow_tail = false) {
  GemmPlan g = g0;
  if (g_gemm_unit_tokens || g_tail_split >= 2) {  // a forced tail split without a forced width: 256
    plan_bf16_width(&g, g_gemm_unit_tokens ? g_gemm_unit_tokens : 256, m, kc, ldp, splitk, narrow_tail);
    return g;
  }
  GemmPlan best_plan = g;
  double best_t = 1e300;
  for (int bt : {256, 128, 64}) {
    GemmPlan c = g;
    const double t = plan_bf16_width(&c, bt, m, kc, ldp, splitk, narrow_tail);
    if (t < best_t) {
      best_t = t;
      best_plan = c;
    }
  }
  return best_plan;
}

// The fused kernel (K1) re-dequantizes the weight for every 192-token tile
// and is issue-bound; the dequantize-once path is tensor-bound and wins from
// kDequantMinM tokens (measured on B200), unless a path is forced.
GemmPlan plan_gemm(int sm_count, const nq_weight *w, int64_t m, int x_dtype, bool direct) {
  GemmPlan g;
  const bool splitx = x_dtype == NQ_F32;
  // A weight with a kept bf16 copy needs no dequantize pass: K3 on the copy
  // is the faster path down to small M as well (M = 125, 1024 -> 4096:
  // 10.0 vs 14.9 us for the fused kernel).
  g.deq = w->bf16_only || g_gemm_path == NQ_GEMM_DEQUANT ||
          (g_gemm_path == NQ_GEMM_AUTO && (m >= kDequantMinM || w->bf16 != nullptr));
  g.cached = g.deq && w->bf16 != nullptr;
  g.split_x = !direct;
  g.pairs = std::max(1, sm_count / 2);
  g.grid_n = (w->n_tiles + 1) / 2;
  const int kc = w->kc;
  if (!g.deq) {
    // Fused kernel: split K when the output tiles do not fill the SM pairs
    // (>= 4 k chunks per split).
    g.bt = nq::gemm_block_t(splitx ? nq::kGemmBt128SplitX : nq::kGemmBt128);
    g.grid_m = static_cast<int>((m + g.bt - 1) / g.bt);
    const int tiles = g.grid_m * g.grid_n;
    int splits = 1;
    if (tiles < g.pairs) splits = std::max(1, std::min((g.pairs + tiles - 1) / tiles, std::max(1, kc / 4)));
    g.cps = (kc + splits - 1) / splits;
    g.splits = (kc + g.cps - 1) / g.cps;
    return g;
  }
  return plan_bf16(g, m, kc, w->n_tiles * nq::kPackRows, true, splitx);
}

bool direct_bf16(const void *x, int x_dtype, int64_t ldx) {
  return x_dtype == NQ_BF16 && (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (ldx % 8 == 0);
}

int run_gemm(DeviceCtx *ctx, const LinearArgs &a, const void *x, int x_dtype, int64_t m, int64_t ldx, int epilogue,
             int y_dtype, cudaStream_t stream) {
  const nq_weight *w = a.w;
  const int kc = w->kc;
  const int64_t k_pad = static_cast<int64_t>(kc) * nq::kPackK;
  const bool splitx = x_dtype == NQ_F32;
  const bool direct = direct_bf16(x, x_dtype, ldx);
  const GemmPlan plan = plan_gemm(ctx->sm_count, w, m, x_dtype, direct);
  const bool deq = plan.deq;
  const int pairs = plan.pairs, bt = plan.bt, grid_m = plan.grid_m, grid_n = plan.grid_n;
  const int splits = plan.splits, cps = plan.cps;
  const int ldp = w->n_tiles * nq::kPackRows;  // rows of partials / of the dequantized weight

  // Workspace: [activation planes][dequantized weight][split-K partials]
  // [tail-split pieces].
  size_t xbytes = 0;
  if (!direct) xbytes = align_up(static_cast<size_t>(m) * k_pad * 2, 1024) * (splitx ? 2 : 1);
  const size_t wbytes = deq && !plan.cached ? align_up(static_cast<size_t>(ldp) * k_pad * 2, 1024) : 0;
  const size_t part_bytes = splits > 1 ? align_up(static_cast<size_t>(splits) * m * ldp * sizeof(float), 256) : 0;
  // one piece: 2 CTAs x 16 epilogue warps x (bt / 4) tokens x 32 rows of f32
  const size_t tail_bytes = static_cast<size_t>(plan.tail_tiles()) * plan.tail_pieces * 2 * 16 * (bt / 4) * 32 * 4;
  if (kTailCounterBase + static_cast<size_t>(plan.tail_tiles()) * 2 * 16 > kCounterSlots)
    return fail(NQ_ERR_SHAPE, "tail split needs more counters than the workspace holds");
  Workspace *ws = nullptr;
  int rc = get_workspace(ctx, stream, xbytes + wbytes + part_bytes + tail_bytes, &ws);
  if (rc) return rc;
  float *partials = splits > 1 ? reinterpret_cast<float *>(ws->buf + xbytes + wbytes) : nullptr;
  float *tail_part = tail_bytes ? reinterpret_cast<float *>(ws->buf + xbytes + wbytes + part_bytes) : nullptr;

  const void *a_ptr = x;
  int64_t a_k = w->k, a_ld = ldx;
  __nv_bfloat16 *lo = nullptr;
  if (!direct) {
    __nv_bfloat16 *hi = reinterpret_cast<__nv_bfloat16 *>(ws->buf);
    if (splitx) lo = reinterpret_cast<__nv_bfloat16 *>(ws->buf + xbytes / 2);
    cudaError_t e = nq::launch_split_x(x, x_dtype, ldx, m, w->k, k_pad, hi, lo, stream);
    if (e != cudaSuccess) return cuda_fail(e, "activation split launch");
    a_ptr = hi;
    a_k = k_pad;
    a_ld = k_pad;
  }
  CUtensorMap tm_a, tm_alo;
  rc = make_tmap(ctx, &tm_a, a_ptr, a_k, m, a_ld, deq ? nq::gemm_bf16_token_box(bt) : bt / 2);
  if (rc) return rc;
  if (splitx) {
    rc = make_tmap(ctx, &tm_alo, lo, a_k, m, a_ld, deq ? nq::gemm_bf16_token_box(bt) : bt / 2);
    if (rc) return rc;
  } else {
    tm_alo = tm_a;
  }

  const double flops = 2.0 * m * w->n * w->k;
  const double bytes = w->n * (w->k / 32) * 34.0 + m * w->k * (x_dtype == NQ_F32 ? 4.0 : 2.0) +
                       m * out_width(w) * (y_dtype == NQ_F32 ? 4.0 : 2.0) + (a.bias ? 4.0 * w->n : 0.0);
  const int units = grid_m * grid_n * splits;
  if (deq) {
    __nv_bfloat16 *wb = plan.cached ? w->bf16 : reinterpret_cast<__nv_bfloat16 *>(ws->buf + xbytes);
    if (!plan.cached) {
      ProfScope ps(NQ_KCLASS_DEQUANT, stream, 0.0, w->bytes + static_cast<double>(ldp) * k_pad * 2);
      cudaError_t e = nq::launch_dequant_tiles(w->dev, w->n_tiles, kc, wb, stream);
      if (e != cudaSuccess) return cuda_fail(e, "weight dequantize launch");
    }
    CUtensorMap tm_w;
    rc = make_tmap(ctx, &tm_w, wb, k_pad, ldp, k_pad, nq::gemm_bf16_block_w() / 2);
    if (rc) return rc;
    nq::GemmBf16Params p;
    std::memset(&p, 0, sizeof(p));
    p.N = w->n;
    p.n_rows = ldp;
    p.glu = (w->flags & NQ_PACK_GLU) ? 1 : 0;
    p.n_out = out_width(w);
    p.M = static_cast<int>(m);
    p.kc_total = kc;
    p.bias = a.bias;
    p.epi = epilogue;
    p.y = a.y;
    p.y_dtype = y_dtype;
    p.ldy = a.ldy;
    p.splits = splits;
    p.cps = cps;
    p.grid_n = grid_n;
    p.grid_m = grid_m;
    p.partials = partials;
    p.full_units = plan.full_units;
    p.tail_pieces = plan.tail_pieces;
    p.tail_cps = plan.tail_cps;
    p.tail_part = tail_part;
    p.tail_cnt = ws->counters + kTailCounterBase;
    p.w_static = plan.cached ? 1 : 0;
    p.ctl.status = ctx->status;
    p.ctl.wait_limit = g_wait_limit;
    const int work_units = plan.tail_pieces > 1 ? plan.full_units + plan.tail_tiles() * plan.tail_pieces : units;
    p.pair_stores = work_units <= pairs ? 1 : 0;
    ProfScope ps(NQ_KCLASS_GEMM, stream, flops, bytes);
    cudaError_t e = nq::launch_gemm_bf16(splitx, bt, tm_w, tm_a, tm_alo, p, std::min(work_units, pairs), stream);
    if (e != cudaSuccess) return cuda_fail(e, "GEMM launch");
  } else {
    nq::GemmParams p;
    std::memset(&p, 0, sizeof(p));
    p.w = w->dev;
    p.n_tiles = w->n_tiles;
    p.kc_total = kc;
    p.N = w->n;
    p.glu = (w->flags & NQ_PACK_GLU) ? 1 : 0;
    p.n_out = out_width(w);
    p.M = static_cast<int>(m);
    p.bias = a.bias;
    p.epi = epilogue;
    p.y = a.y;
    p.y_dtype = y_dtype;
    p.ldy = a.ldy;
    p.splits = splits;
    p.cps = cps;
    p.grid_n = grid_n;
    p.grid_m = grid_m;
    p.partials = partials;
    p.ldp = ldp;
    p.ctl.status = ctx->status;
    p.ctl.wait_limit = g_wait_limit;
    ProfScope ps(NQ_KCLASS_GEMM, stream, flops, bytes);
    cudaError_t e = nq::launch_gemm(splitx ? nq::kGemmBt128SplitX : nq::kGemmBt128, tm_a, tm_alo, p,
                                    std::min(units, pairs), stream);
    if (e != cudaSuccess) return cuda_fail(e, "GEMM launch");
  }
  if (splits > 1) {
    nq::SplitkReduceParams r;
    r.partials = partials;
    r.splits = splits;
    r.M = static_cast<int>(m);
    r.ldp = ldp;
    r.n_out = out_width(w);
    r.glu = (w->flags & NQ_PACK_GLU) ? 1 : 0;
    r.bias = a.bias;
    r.epi = epilogue;
    r.y = a.y;
    r.y_dtype = y_dtype;
    r.ldy = a.ldy;
    ProfScope ps(NQ_KCLASS_REDUCE, stream, 0.0, static_cast<double>(splits) * m * ldp * 4);
    cudaError_t e = nq::launch_splitk_reduce(r, stream);
    if (e != cudaSuccess) return cuda_fail(e, "split-K reduce launch");
  }
  return NQ_OK;
}

// The tap-major copy of a conv weight for (c_in, kernel), built once on
// `stream` (dequantizing Q8_0 tiles into scratch first when the weight keeps
// no bf16 copy) and synchronized, so every stream may read it afterwards.
int ensure_tap_copy(const nq_weight *w, int64_t c_in, int kernel, cudaStream_t stream, const __nv_bfloat16 **out) {
  std::lock_guard<std::mutex> lk(g_tap_mu);
  if (w->tap && w->tap_cin == c_in && w->tap_k == kernel) {
    *out = w->tap;
    return NQ_OK;
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(stream, &cs);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
  if (cs != cudaStreamCaptureStatusNone)
    return fail(NQ_ERR_UNSUPPORTED,
                "nq_conv1d: the first call with a weight builds its tap-major copy and cannot run under stream "
                "capture; call it once before capturing");
  const int rows = w->n_tiles * nq::kPackRows;
  const int64_t k_pad = static_cast<int64_t>(w->kc) * nq::kPackK;
  const __nv_bfloat16 *src = w->bf16;
  __nv_bfloat16 *tmp = nullptr, *dst = nullptr;
  if (!src) {
    e = cudaMalloc(&tmp, static_cast<size_t>(rows) * k_pad * 2);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(conv weight dequantize scratch)");
    e = nq::launch_dequant_tiles(w->dev, w->n_tiles, w->kc, tmp, stream);
    if (e != cudaSuccess) {
      cudaFree(tmp);
      return cuda_fail(e, "weight dequantize launch");
    }
    src = tmp;
  }
  e = cudaMalloc(&dst, static_cast<size_t>(rows) * kernel * c_in * 2);
  if (e == cudaSuccess) e = nq::launch_conv_tap_weight(src, k_pad, rows, static_cast<int>(c_in), kernel, dst, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (tmp) cudaFree(tmp);
  if (e != cudaSuccess) {
    if (dst) cudaFree(dst);
    return cuda_fail(e, "conv weight tap-major copy");
  }
  if (w->tap) {  // a copy for another (c_in, kernel) view of the same weight
    e = cudaDeviceSynchronize();  // no launch in flight may still read it
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize(replace tap-major copy)");
    cudaFree(w->tap);
  }
  w->tap = dst;
  w->tap_cin = c_in;
  w->tap_k = kernel;
  *out = dst;
  return NQ_OK;
}

// The polyphase copy of a conv_transpose1d weight for `stride`, built once
// on `stream` from the weight's bf16 form and synchronized.
int ensure_poly_copy(const nq_weight *w, int64_t c_in, int64_t c_out, int kernel, int stride, cudaStream_t stream,
                     const __nv_bfloat16 **out) {
  std::lock_guard<std::mutex> lk(g_tap_mu);
  if (w->poly && w->poly_s == stride) {
    *out = w->poly;
    return NQ_OK;
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(stream, &cs);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
  if (cs != cudaStreamCaptureStatusNone)
    return fail(NQ_ERR_UNSUPPORTED,
                "nq_conv_transpose1d: the first call with a weight builds its polyphase copy and cannot run under "
                "stream capture; call it once before capturing");
  const int taps = (kernel + stride - 1) / stride;
  const int rows = static_cast<int>((c_out * stride + nq::kPackRows - 1) / nq::kPackRows) * nq::kPackRows;
  const int64_t k_pad = static_cast<int64_t>(w->kc) * nq::kPackK;
  __nv_bfloat16 *dst = nullptr;
  e = cudaMalloc(&dst, static_cast<size_t>(rows) * taps * c_in * 2);
  if (e == cudaSuccess)
    e = nq::launch_conv_poly_weight(w->bf16, k_pad, static_cast<int>(c_out), kernel, stride, static_cast<int>(c_in),
                                    taps, rows, dst, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) {
    if (dst) cudaFree(dst);
    return cuda_fail(e, "conv_transpose weight polyphase copy");
  }
  if (w->poly) {
    e = cudaDeviceSynchronize();  // no launch in flight may still read it
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize(replace polyphase copy)");
    cudaFree(w->poly);
  }
  w->poly = dst;
  w->poly_s = stride;
  *out = dst;
  return NQ_OK;
}

// Implicit-GEMM conv_transpose1d in polyphase form.  Output frame
// t = q s + r - padding (phase r = (t + padding) mod s) sums taps j = r + s i
// of input position q - i, so the whole transposed conv is one stride-1
// implicit GEMM over the token-major input: weight rows (co, r) with k =
// (tap i, channels), token m = input position q = q0 + m reading rows
// q - i (dilation -1), and an epilogue that scatters row (co, r) of token m
// to frame q s + r - padding.  No column buffer and no overlap-add pass.
int conv_transpose1d_implicit(DeviceCtx *ctx, const nq_weight *w, const void *x, int x_dtype, int64_t c_in,
                              int64_t t_in, int64_t ldx, int kernel, int stride, int padding, float x_leaky,
                              const float *bias, int epilogue, void *y, int y_dtype, int64_t ldy, int64_t t_out,
                              int64_t q0, int64_t m, cudaStream_t stream) {
  const int64_t c_out = w->n / kernel;
  const __nv_bfloat16 *wp = nullptr;
  int rc = ensure_poly_copy(w, c_in, c_out, kernel, stride, stream, &wp);
  if (rc) return rc;
  const bool splitx = x_dtype == NQ_F32;
  const int taps = (kernel + stride - 1) / stride;
  const int kc = static_cast<int>(taps * c_in / nq::kPackK);
  const int n_tiles = static_cast<int>((c_out * stride + nq::kPackRows - 1) / nq::kPackRows);
  const int ldp = n_tiles * nq::kPackRows;
  GemmPlan g;
  g.deq = true;
  g.cached = true;
  g.pairs = std::max(1, ctx->sm_count / 2);
  g.grid_n = (n_tiles + 1) / 2;
  const GemmPlan plan = plan_bf16(g, m, kc, ldp, false);
  const int bt = plan.bt;
  const size_t plane = align_up(static_cast<size_t>(t_in) * c_in * 2, 1024);
  const size_t tail_bytes = static_cast<size_t>(plan.tail_tiles()) * plan.tail_pieces * 2 * 16 * (bt / 4) * 32 * 4;
  if (kTailCounterBase + static_cast<size_t>(plan.tail_tiles()) * 2 * 16 > kCounterSlots)
    return fail(NQ_ERR_SHAPE, "tail split needs more counters than the workspace holds");
  Workspace *ws = nullptr;
  rc = get_workspace(ctx, stream, plane * (splitx ? 2 : 1) + tail_bytes, &ws, true);
  if (rc) return rc;
  __nv_bfloat16 *hi = reinterpret_cast<__nv_bfloat16 *>(ws->buf);
  __nv_bfloat16 *lo = splitx ? reinterpret_cast<__nv_bfloat16 *>(ws->buf + plane) : nullptr;
  float *tail_part = tail_bytes ? reinterpret_cast<float *>(ws->buf + plane * (splitx ? 2 : 1)) : nullptr;
  cudaError_t e = nq::launch_conv_tokens(x, x_dtype, ldx, static_cast<int>(c_in), static_cast<int>(t_in), x_leaky,
                                         hi, lo, stream);
  if (e != cudaSuccess) return cuda_fail(e, "conv_transpose input launch");
  CUtensorMap tm_w, tm_a, tm_alo;
  const int64_t kw = static_cast<int64_t>(kc) * nq::kPackK;
  rc = make_tmap(ctx, &tm_w, wp, kw, ldp, kw, nq::gemm_bf16_block_w() / 2);
  if (rc) return rc;
  rc = make_tmap(ctx, &tm_a, hi, c_in, t_in, c_in, nq::gemm_bf16_token_box(bt));
  if (rc) return rc;
  if (splitx) {
    rc = make_tmap(ctx, &tm_alo, lo, c_in, t_in, c_in, nq::gemm_bf16_token_box(bt));
    if (rc) return rc;
  } else {
    tm_alo = tm_a;
  }
  nq::GemmBf16Params p;
  std::memset(&p, 0, sizeof(p));
  p.N = c_out * stride;
  p.n_rows = ldp;
  p.n_out = p.N;
  p.M = static_cast<int>(m);
  p.kc_total = kc;
  p.bias = bias;
  p.epi = epilogue;
  p.y = y;
  p.y_dtype = y_dtype;
  p.ldy = ldy;
  p.splits = 1;
  p.cps = kc;
  p.grid_n = plan.grid_n;
  p.grid_m = plan.grid_m;
  p.full_units = plan.full_units;
  p.tail_pieces = plan.tail_pieces;
  p.tail_cps = plan.tail_cps;
  p.tail_part = tail_part;
  p.tail_cnt = ws->counters + kTailCounterBase;
  p.w_static = 1;
  p.conv_cpt = static_cast<int>(c_in / nq::kPackK);
  p.conv_dil = -1;
  p.conv_pad = static_cast<int>(-q0);
  p.y_cm = 1;
  p.poly_s = stride;
  p.poly_q0 = static_cast<int>(q0);
  p.poly_pad = padding;
  p.t_out = t_out;
  p.ctl.status = ctx->status;
  p.ctl.wait_limit = g_wait_limit;
  const int work_units = plan.tail_pieces > 1 ? plan.full_units + plan.tail_tiles() * plan.tail_pieces
                                              : plan.grid_m * plan.grid_n;
  const double flops = 2.0 * t_in * c_in * c_out * kernel;
  const double bytes = static_cast<double>(ldp) * kw * 2 + t_in * c_in * (splitx ? 4.0 : 2.0) +
                       c_out * t_out * (y_dtype == NQ_F32 ? 4.0 : 2.0) + (bias ? 4.0 * c_out : 0.0);
  ProfScope ps(NQ_KCLASS_GEMM, stream, flops, bytes);
  e = nq::launch_gemm_bf16(splitx, bt, tm_w, tm_a, tm_alo, p, std::min(work_units, plan.pairs), stream);
  if (e != cudaSuccess) return cuda_fail(e, "implicit conv_transpose GEMM launch");
  return NQ_OK;
}

// Implicit-GEMM conv1d (stride 1, channels in whole 64-wide k chunks): the
// input goes to token-major bf16 planes once (leaky ReLU applied), and the
// bf16 GEMM reads, for k chunk (tap j, channels c), the planes' rows shifted
// by j dilation - padding (zero outside the input), against the weight's
// tap-major copy; its epilogue writes the NCW output directly.  No im2col
// rows and no output transpose.  Split-K is not used (the tail split is).
int conv1d_implicit(DeviceCtx *ctx, const nq_weight *w, const void *x, int x_dtype, int64_t c_in, int64_t t_in,
                    int64_t ldx, int kernel, int padding, int dilation, float x_leaky, const float *bias, int epilogue,
                    void *y, int y_dtype, int64_t ldy, int64_t t_out, cudaStream_t stream) {
  const __nv_bfloat16 *wt = nullptr;
  int rc = ensure_tap_copy(w, c_in, kernel, stream, &wt);
  if (rc) return rc;
  const bool splitx = x_dtype == NQ_F32;
  const int kc = static_cast<int>(kernel * c_in / nq::kPackK);
  const int ldp = w->n_tiles * nq::kPackRows;
  GemmPlan g;
  g.deq = true;
  g.cached = true;
  g.pairs = std::max(1, ctx->sm_count / 2);
  g.grid_n = (w->n_tiles + 1) / 2;
  const GemmPlan plan = plan_bf16(g, t_out, kc, ldp, false);
  const int bt = plan.bt;
  const size_t plane = align_up(static_cast<size_t>(t_in) * c_in * 2, 1024);
  const size_t tail_bytes = static_cast<size_t>(plan.tail_tiles()) * plan.tail_pieces * 2 * 16 * (bt / 4) * 32 * 4;
  if (kTailCounterBase + static_cast<size_t>(plan.tail_tiles()) * 2 * 16 > kCounterSlots)
    return fail(NQ_ERR_SHAPE, "tail split needs more counters than the workspace holds");
  Workspace *ws = nullptr;
  rc = get_workspace(ctx, stream, plane * (splitx ? 2 : 1) + tail_bytes, &ws, true);
  if (rc) return rc;
  __nv_bfloat16 *hi = reinterpret_cast<__nv_bfloat16 *>(ws->buf);
  __nv_bfloat16 *lo = splitx ? reinterpret_cast<__nv_bfloat16 *>(ws->buf + plane) : nullptr;
  float *tail_part = tail_bytes ? reinterpret_cast<float *>(ws->buf + plane * (splitx ? 2 : 1)) : nullptr;
  cudaError_t e = nq::launch_conv_tokens(x, x_dtype, ldx, static_cast<int>(c_in), static_cast<int>(t_in), x_leaky,
                                         hi, lo, stream);
  if (e != cudaSuccess) return cuda_fail(e, "conv input launch");
  CUtensorMap tm_w, tm_a, tm_alo;
  rc = make_tmap(ctx, &tm_w, wt, static_cast<int64_t>(kc) * nq::kPackK, ldp, static_cast<int64_t>(kc) * nq::kPackK,
                 nq::gemm_bf16_block_w() / 2);
  if (rc) return rc;
  rc = make_tmap(ctx, &tm_a, hi, c_in, t_in, c_in, nq::gemm_bf16_token_box(bt));
  if (rc) return rc;
  if (splitx) {
    rc = make_tmap(ctx, &tm_alo, lo, c_in, t_in, c_in, nq::gemm_bf16_token_box(bt));
    if (rc) return rc;
  } else {
    tm_alo = tm_a;
  }
  nq::GemmBf16Params p;
  std::memset(&p, 0, sizeof(p));
  p.N = w->n;
  p.n_rows = ldp;
  p.n_out = w->n;
  p.M = static_cast<int>(t_out);
  p.kc_total = kc;
  p.bias = bias;
  p.epi = epilogue;
  p.y = y;
  p.y_dtype = y_dtype;
  p.ldy = ldy;
  p.splits = 1;
  p.cps = kc;
  p.grid_n = plan.grid_n;
  p.grid_m = plan.grid_m;
  p.full_units = plan.full_units;
  p.tail_pieces = plan.tail_pieces;
  p.tail_cps = plan.tail_cps;
  p.tail_part = tail_part;
  p.tail_cnt = ws->counters + kTailCounterBase;
  p.w_static = 1;
  p.conv_cpt = static_cast<int>(c_in / nq::kPackK);
  p.conv_dil = dilation;
  p.conv_pad = padding;
  p.y_cm = 1;
  p.ctl.status = ctx->status;
  p.ctl.wait_limit = g_wait_limit;
  const int work_units = plan.tail_pieces > 1 ? plan.full_units + plan.tail_tiles() * plan.tail_pieces
                                              : plan.grid_m * plan.grid_n;
  const double flops = 2.0 * t_out * w->n * c_in * kernel;
  const double bytes = static_cast<double>(ldp) * kc * nq::kPackK * 2 + t_in * c_in * (splitx ? 4.0 : 2.0) +
                       t_out * w->n * (y_dtype == NQ_F32 ? 4.0 : 2.0) + (bias ? 4.0 * w->n : 0.0);
  ProfScope ps(NQ_KCLASS_GEMM, stream, flops, bytes);
  e = nq::launch_gemm_bf16(splitx, bt, tm_w, tm_a, tm_alo, p, std::min(work_units, plan.pairs), stream);
  if (e != cudaSuccess) return cuda_fail(e, "implicit conv GEMM launch");
  return NQ_OK;
}

// QTiled semantics (NQ_MODE_QTILED weights): quantize the activation rows to
// Q8_0 once, then one int8 tensor-core launch per weight.
int run_qtiled(DeviceCtx *ctx, const LinearArgs *args, int nprob, const void *x, int x_dtype, int64_t m, int64_t ldx,
               int epilogue, int y_dtype, cudaStream_t stream) {
  const int kc = args[0].w->kc;
  for (int i = 1; i < nprob; ++i)
    if (args[i].w->kc != kc) return fail(NQ_ERR_SHAPE, "weights sharing x must share K");
  Workspace *ws = nullptr;
  int rc = get_workspace(ctx, stream, nq::qtiled_x_bytes(m, kc), &ws);
  if (rc) return rc;
  int8_t *xq = reinterpret_cast<int8_t *>(ws->buf);
  float *dx = reinterpret_cast<float *>(ws->buf + align_up(static_cast<size_t>(m) * kc * nq::kPackK, 256));
  cudaError_t e = nq::launch_qtiled_quantize(x, x_dtype, ldx, m, args[0].w->k, kc, xq, dx, stream);
  if (e != cudaSuccess) return cuda_fail(e, "activation quantize launch");
  for (int i = 0; i < nprob; ++i) {
    const nq_weight *w = args[i].w;
    nq::QtiledParams p;
    std::memset(&p, 0, sizeof(p));
    p.w = w->dev;
    p.n_tiles = w->n_tiles;
    p.kc = kc;
    p.N = w->n;
    p.M = static_cast<int>(m);
    p.xq = xq;
    p.dx = dx;
    p.bias = args[i].bias;
    p.epi = epilogue;
    p.y = args[i].y;
    p.y_dtype = y_dtype;
    p.ldy = args[i].ldy;
    double flops = 0, bytes = 0;
    linear_cost(&args[i], 1, m, x_dtype, y_dtype, &flops, &bytes);
    ProfScope ps(m <= 16 ? NQ_KCLASS_GEMV : NQ_KCLASS_GEMM, stream, flops, bytes);
    e = nq::launch_qtiled(p, stream);
    if (e != cudaSuccess) return cuda_fail(e, "QTiled GEMM launch");
  }
  return NQ_OK;
}

int linear_impl(const LinearArgs *args, int nprob, const void *x, int x_dtype, int64_t m, int64_t ldx, int epilogue,
                int y_dtype, void *stream) {
  for (int i = 0; i < nprob; ++i) {
    int rc = validate(args[i].w, x, x_dtype, m, ldx, epilogue, args[i].y, y_dtype, args[i].ldy);
    if (rc) return rc;
  }
  if (m == 0) return NQ_OK;
  DeviceCtx *ctx = nullptr;
  int dev = 0;
  int rc = current_ctx(&ctx, &dev);
  if (rc) return rc;
  for (int i = 0; i < nprob; ++i)
    if (args[i].w->device != dev)
      return fail(NQ_ERR_ARG, "weight lives on device %d, current device is %d", args[i].w->device, dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool qtiled = (args[0].w->flags & NQ_MODE_QTILED) != 0;
  for (int i = 1; i < nprob; ++i)
    if (((args[i].w->flags & NQ_MODE_QTILED) != 0) != qtiled)
      return fail(NQ_ERR_ARG, "weights sharing one call must all be NQ_MODE_QTILED or none");
  if (qtiled) return run_qtiled(ctx, args, nprob, x, x_dtype, m, ldx, epilogue, y_dtype, s);
  bool any_bf16_only = false;
  for (int i = 0; i < nprob; ++i) any_bf16_only = any_bf16_only || args[i].w->bf16_only;
  if (m <= 16 && !any_bf16_only) return run_gemv(ctx, args, nprob, x, x_dtype, m, ldx, epilogue, y_dtype, s);
  for (int i = 0; i < nprob; ++i) {
    rc = run_gemm(ctx, args[i], x, x_dtype, m, ldx, epilogue, y_dtype, s);
    if (rc) return rc;
  }
  return NQ_OK;
}

// ------------------------------------------------- static-scratch GEMV
// Scratch of nq_gemv_noalloc: the GEMV's unit partials, then the activation
// planes split_x writes when x is not read in place, then the work counter,
// in this module's own device memory (a file-scope device array), so a call
// needs no allocation.  One array per device, shared by every call on that
// device.
constexpr size_t kNoAllocPartialBytes = size_t(4) << 20;  // 4 MiB of unit partials
constexpr size_t kNoAllocXBytes = size_t(2) << 20;        // 2 MiB of bf16 activation planes
constexpr size_t kNoAllocBytes = kNoAllocPartialBytes + kNoAllocXBytes + 256;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mu;
unsigned char *g_noalloc_ptr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch for device `dev` (current), looked up
// once per device.
int noalloc_scratch(int dev, unsigned char **out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static GEMV scratch)");
    g_noalloc_ptr[dev] = static_cast<unsigned char *>(ptr);
  }
  *out = g_noalloc_ptr[dev];
  return NQ_OK;
}

}  // namespace

namespace nq {
int api_fail(int code, const std::string &msg) { return fail(code, "%s", msg.c_str()); }

std::atomic<long long> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int linear_launches(const nq_weight *w, int64_t m, int x_dtype, bool aligned) {
  if (!w || m <= 0) return 0;
  if (w->flags & NQ_MODE_QTILED) return 2;  // quantize x + the int8 GEMM
  if (m <= 16 && !w->bf16_only)  // GEMV + gemv_reduce (for up to three weights), after split_x unless x is read in place
    return x_dtype == NQ_BF16 && aligned && w->k % nq::kPackK == 0 ? 2 : 3;
  DeviceCtx *ctx = nullptr;
  int dev = 0;
  const int sm = current_ctx(&ctx, &dev) == NQ_OK ? ctx->sm_count : kSmCountB200;
  return plan_gemm(sm, w, m, x_dtype, x_dtype == NQ_BF16 && aligned).launches();
}

bool attention_tc(int Tp) { return g_attention_kernel == NQ_ATTENTION_TCGEN05 && Tp <= attention_tc_max_tp(); }

int layer_norm_rows(int mode, float *x, const void *u, float alpha, int rows, int D, const float *g1, const float *b1,
                    const float *g2, const float *b2, __nv_bfloat16 *h, float eps, cudaStream_t s) {
  // algorithmic bytes per row: x written (f32); x read unless kLnScale; u read
  // (f32 for kLnScale, else bf16); h written (bf16) unless the final norm_out
  // has no next LayerNorm
  const double per_row = 4.0 * D + (mode == enc::kLnScale ? 4.0 * D : 4.0 * D + 2.0 * D) +
                         (mode != enc::kLnResAddOut || g2 ? 2.0 * D : 0.0);
  ProfScope ps(NQ_KCLASS_NORM, s, 0.0, per_row * rows);
  const cudaError_t e = enc::ln_rows(mode, x, u, alpha, rows, D, g1, b1, g2, b2, h, eps, s);
  if (e != cudaSuccess) return cuda_fail(e, "ln_rows launch");
  return NQ_OK;
}

int relpos_bias(const __nv_bfloat16 *krel, const float *vmu, int nrel, int n_layers, int D, float *vrel,
                cudaStream_t s) {
  const cudaError_t e = launch_relpos_bias(krel, vmu, nrel, n_layers, D, vrel, s);
  if (e != cudaSuccess) return cuda_fail(e, "relpos_bias launch");
  return NQ_OK;
}

int relpos_attention(const __nv_bfloat16 *qkv, const __nv_bfloat16 *krel, int64_t ldr, const float *bias_u,
                     const float *bias_v, const float *vrel, const int *len, int B, int Tp, int H, int D,
                     __nv_bfloat16 *out, cudaStream_t s) {
  DeviceCtx *ctx = nullptr;
  int rc = current_ctx(&ctx, nullptr);
  if (rc) return rc;
  if (H <= 0 || D != H * 128 || Tp <= 0 || B <= 0 || ldr < D || ldr % 8)
    return fail(NQ_ERR_SHAPE, "attention shape B=%d Tp=%d H=%d D=%d ldr=%lld", B, Tp, H, D, (long long)ldr);
  const double tok = static_cast<double>(B) * Tp;
  ProfScope ps(NQ_KCLASS_ATTENTION, s, 6.0 * tok * Tp * D, (tok * 4.0 + 2.0 * Tp - 1.0) * D * 2.0);
  if (!attention_tc(Tp) || !vrel) {
    const cudaError_t e = enc::relpos_attention(qkv, krel, ldr, bias_u, bias_v, len, B, Tp, H, D, out, s);
    if (e != cudaSuccess) return cuda_fail(e, "relpos_attention launch");
    return NQ_OK;
  }
  CUtensorMap tm_qkv, tm_rel;
  rc = make_tmap(ctx, &tm_qkv, qkv, 3 * static_cast<int64_t>(D), static_cast<int64_t>(B) * Tp, 3 * static_cast<int64_t>(D), 64);
  if (rc) return rc;
  rc = make_tmap(ctx, &tm_rel, krel, D, 2 * static_cast<int64_t>(Tp) - 1, ldr, 64);
  if (rc) return rc;
  AttnTcParams p;
  p.qkv = qkv;
  p.vrel = vrel;
  p.len = len;
  p.out = out;
  p.B = B;
  p.Tp = Tp;
  p.D = D;
  p.rel_col0 = 0;
  p.sl2 = static_cast<float>(1.4426950408889634 / std::sqrt(128.0));
  p.ctl = DevCtl{ctx->status, g_wait_limit};
  const cudaError_t e = launch_relpos_attention_tc(tm_qkv, tm_rel, p, ctx->sm_count, s);
  if (e != cudaSuccess) return cuda_fail(e, "relpos_attention_tc launch");
  return NQ_OK;
}
}  // namespace nq

// ======================================================================= ABI
namespace {
int chain_add(nq_chain *c, const nq_weight *w, const void *x, const float *bias, int epilogue, void *y, int y_dtype,
              const float *res_in, float *res_out, const float *ln_g, const float *ln_b, float eps) {
  if (!c || !w || !x) return fail(NQ_ERR_ARG, "null argument");
  if (c->uploaded) return fail(NQ_ERR_UNSUPPORTED, "nq_chain: steps cannot be added after the first run");
  if (w->device != c->device) return fail(NQ_ERR_ARG, "weight lives on device %d, the chain on %d", w->device, c->device);
  if (w->bf16_only || (w->flags & NQ_MODE_QTILED))
    return fail(NQ_ERR_UNSUPPORTED, "nq_chain: Q8_0 weights with FbgemmBf16Op semantics only");
  if (static_cast<int64_t>(w->kc) * nq::kPackK > nq::kChainMaxK)
    return fail(NQ_ERR_SHAPE, "nq_chain: K = %lld exceeds %d", (long long)w->k, nq::kChainMaxK);
  if (reinterpret_cast<uintptr_t>(x) % 2) return fail(NQ_ERR_ARG, "nq_chain: x must be 2-byte aligned bf16");
  const bool resadd = res_out != nullptr;
  const bool glu_w = (w->flags & NQ_PACK_GLU) != 0;
  const bool glu_e = epilogue == NQ_EPI_GLU_SIGMOID || epilogue == NQ_EPI_GLU_SILU;
  if (epilogue < NQ_EPI_NONE || epilogue > NQ_EPI_RELU) return fail(NQ_ERR_ARG, "unknown epilogue %d", epilogue);
  if (glu_w != glu_e) return fail(NQ_ERR_ARG, "GLU epilogues need an NQ_PACK_GLU weight and vice versa");
  if (y_dtype != NQ_F32 && y_dtype != NQ_BF16) return fail(NQ_ERR_DTYPE, "y dtype %d unsupported", y_dtype);
  if (resadd) {
    if (!res_in || !ln_g) return fail(NQ_ERR_ARG, "nq_chain_gemv_resadd_ln: null residual or gamma");
    if (glu_w) return fail(NQ_ERR_ARG, "nq_chain_gemv_resadd_ln: GLU-packed weight");
    if (w->n > nq::kChainMaxLnN) return fail(NQ_ERR_SHAPE, "nq_chain_gemv_resadd_ln: N exceeds %d", nq::kChainMaxLnN);
    if (!(eps >= 0.f)) return fail(NQ_ERR_ARG, "nq_chain_gemv_resadd_ln: eps must be >= 0");
  } else if (!y) {
    return fail(NQ_ERR_ARG, "null output");
  }
  const int64_t n_out = glu_w ? w->n / 2 : w->n;
  using R = nq_chain::Range;
  const uintptr_t xa = reinterpret_cast<uintptr_t>(x), ya = reinterpret_cast<uintptr_t>(y);
  const R xr{xa, xa + static_cast<uintptr_t>(w->k) * 2};
  const R yr = y ? R{ya, ya + static_cast<uintptr_t>(n_out) * (y_dtype == NQ_F32 ? 4 : 2)} : R{};
  const R rr = resadd ? R{reinterpret_cast<uintptr_t>(res_out), reinterpret_cast<uintptr_t>(res_out) + w->n * 4} : R{};
  const R ri = resadd ? R{reinterpret_cast<uintptr_t>(res_in), reinterpret_cast<uintptr_t>(res_in) + w->n * 4} : R{};
  // Hazards inside one step: its input is read while other CTAs already write its outputs.
  if (xr.overlaps(yr) || xr.overlaps(rr)) return fail(NQ_ERR_UNSUPPORTED, "nq_chain: a step's input overlaps its output");
  if (resadd && ri.lo != rr.lo && ri.overlaps(rr))
    return fail(NQ_ERR_UNSUPPORTED, "nq_chain: res_in and res_out overlap without being the same row");
  int x_ln = 0;
  if (!c->steps.empty()) {
    const size_t ps = c->steps.size() - 1;
    const nq::ChainStep &pv = c->steps[ps];
    if (pv.res_out) {
      // The previous residual step's LayerNorm output is written while this
      // step runs: this step reads it computed on load, and must not write it.
      if (resadd) return fail(NQ_ERR_UNSUPPORTED, "nq_chain: two residual steps in a row");
      const R &lr = c->y_range[ps];
      if (pv.y && xa == lr.lo && w->k == pv.N) {
        x_ln = 1;
      } else if (xr.overlaps(lr)) {
        return fail(NQ_ERR_UNSUPPORTED, "nq_chain: the input reads part of the previous step's LayerNorm output");
      }
      if (yr.overlaps(lr) || yr.overlaps(c->res_range[ps]))
        return fail(NQ_ERR_UNSUPPORTED, "nq_chain: a step overwrites the previous step's residual or LayerNorm output");
    }
    for (size_t i = 0; i < c->steps.size(); ++i)
      if (!x_ln && xr.overlaps(c->y_range[i]) && c->steps[i].y_dtype != NQ_BF16)
        return fail(NQ_ERR_DTYPE, "nq_chain: the input reads an f32 output of step %zu", i);
  }
  nq::ChainStep st;
  std::memset(&st, 0, sizeof(st));
  st.w = w->dev;
  st.n_tiles = w->n_tiles;
  st.kc = w->kc;
  st.N = w->n;
  st.glu = glu_w ? 1 : 0;
  st.n_out = n_out;
  st.epi = epilogue;
  st.bias = bias;
  st.x_ln = x_ln;
  st.x = static_cast<const __nv_bfloat16 *>(x);
  st.K = static_cast<int>(w->k);
  st.res_in = res_in;
  st.res_out = res_out;
  st.ln_g = ln_g;
  st.ln_b = ln_b;
  st.ln_eps = eps;
  st.y = y;
  st.y_dtype = y_dtype;
  c->steps.push_back(st);
  c->x_range.push_back(xr);
  c->y_range.push_back(yr);
  c->res_range.push_back(rr);
  c->flops += 2.0 * w->n * w->k;
  c->bytes += w->n * (w->k / 32) * 34.0 + w->k * 2.0 + n_out * (y_dtype == NQ_F32 ? 4.0 : 2.0);
  return NQ_OK;
}

int chain_upload(nq_chain *c, DeviceCtx *ctx, cudaStream_t stream) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(stream, &cs);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
  if (cs != cudaStreamCaptureStatusNone)
    return fail(NQ_ERR_UNSUPPORTED, "nq_chain_run: the first run uploads the chain and cannot be captured");
  e = nq::chain_max_ctas(ctx->sm_count, &c->ctas);
  if (e != cudaSuccess) return cuda_fail(e, "chain occupancy");
  // A step with no more tiles than clusters splits each tile's k over a
  // cluster; larger steps give each tile to one CTA.  Owners go round-robin,
  // continuing from step to step.
  const int clusters = c->ctas / nq::kChainCluster;
  int rot_cl = 0, rot_cta = 0;
  for (auto &st : c->steps) {
    st.split = st.n_tiles <= clusters ? 1 : 0;
    if (st.split) {
      st.rot = rot_cl;
      rot_cl = (rot_cl + st.n_tiles) % clusters;
    } else {
      st.rot = rot_cta;
      rot_cta = (rot_cta + st.n_tiles) % c->ctas;
    }
  }
  const size_t n_steps = c->steps.size();
  c->counter_bytes = n_steps * sizeof(int);
  e = cudaMalloc(&c->d_counters, c->counter_bytes);
  if (e == cudaSuccess) e = cudaMemset(c->d_counters, 0, c->counter_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&c->d_steps, n_steps * sizeof(nq::ChainStep));
  if (e != cudaSuccess) return cuda_fail(e, "nq_chain_run: device buffers");
  e = cudaMemcpy(c->d_steps, c->steps.data(), n_steps * sizeof(nq::ChainStep), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "nq_chain_run: upload");
  {
    std::lock_guard<std::mutex> lk(ctx->mu);
    ctx->chain_counters[c->d_counters] = c->counter_bytes;
  }
  c->uploaded = true;
  return NQ_OK;
}
}  // namespace

extern "C" {

const char *nq_version(void) { return "nq8 0.1 sm_100a"; }

int nq_init(int device_ordinal) {
  if (device_ordinal < 0 || device_ordinal >= kMaxDevices) return fail(NQ_ERR_ARG, "bad device %d", device_ordinal);
  cudaError_t e = cudaSetDevice(device_ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  std::lock_guard<std::mutex> lk(g_init_mu);
  DeviceCtx &c = g_ctx[device_ordinal];
  if (c.ready) return NQ_OK;
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device_ordinal);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  if (prop.major != 10 || prop.minor != 0)
    return fail(NQ_ERR_UNSUPPORTED, "device %d is sm_%d%d; libnq8 is built for sm_100a (B200)", device_ordinal,
                prop.major, prop.minor);
  c.sm_count = prop.multiProcessorCount;
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || !fn || q != cudaDriverEntryPointSuccess)
    return fail(NQ_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  c.encode = reinterpret_cast<EncodeTiledFn>(fn);
  e = cudaMalloc(&c.status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(status)");
  e = cudaMemset(c.status, 0, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(status)");
  c.ready = true;
  return NQ_OK;
}

int nq_weight_from_q8_0(const void *blocks, int64_t n, int64_t k, int flags, nq_weight **out) {
  if (!blocks || !out) return fail(NQ_ERR_ARG, "null argument");
  int rc = check_weight_shape(n, k, flags);
  if (rc) return rc;
  return upload_packed(static_cast<const uint8_t *>(blocks), n, k, flags, out);
}

int nq_weight_from_f32(const float *wf, int64_t n, int64_t k, int flags, nq_weight **out) {
  if (!wf || !out) return fail(NQ_ERR_ARG, "null argument");
  if (k > 0 && k % 32 != 0 && !(flags & NQ_MODE_QTILED)) {
    // no Q8_0 form (blocks of 32 along K): a bf16-only weight
    int rc = check_weight_shape(n, (k + 31) / 32 * 32, flags);
    if (rc) return rc;
    for (int64_t i = 0; i < n * k; ++i)
      if (!std::isfinite(wf[i]))
        return fail(NQ_ERR_DTYPE, "nq_weight_from_f32: element [%lld, %lld] is not finite", (long long)(i / k),
                    (long long)(i % k));
    return upload_bf16_only(wf, n, k, flags, out);
  }
  int rc = check_weight_shape(n, k, flags);
  if (rc) return rc;
  std::vector<uint8_t> blocks(static_cast<size_t>(n) * (k / 32) * 34);
  nq::quantize_q8_0(wf, n, k, blocks.data());
  const int64_t bad = nq::q8_0_first_mismatch(wf, blocks.data(), n * k);
  if (bad < 0) return upload_packed(blocks.data(), n, k, flags, out);
  // Not a Q8_0 dequantization: keep it at bf16 precision, as the reference's
  // PackedMatrixBf16 does.  QTiled semantics need Q8_0 blocks.
  if (flags & NQ_MODE_QTILED)
    return fail(NQ_ERR_DTYPE,
                "nq_weight_from_f32: element [%lld, %lld] = %g is not a Q8_0 value; NQ_MODE_QTILED needs Q8_0 "
                "weights", (long long)(bad / k), (long long)(bad % k), static_cast<double>(wf[bad]));
  for (int64_t i = 0; i < n * k; ++i)
    if (!std::isfinite(wf[i]))
      return fail(NQ_ERR_DTYPE, "nq_weight_from_f32: element [%lld, %lld] is not finite", (long long)(i / k),
                  (long long)(i % k));
  return upload_bf16_only(wf, n, k, flags, out);
}

int nq_weight_from_gguf(const char *path, const char *tensor_name, int flags, nq_weight **out) {
  if (!path || !tensor_name || !out) return fail(NQ_ERR_ARG, "null argument");
  nq::GgufFile f;
  std::string err;
  int rc = f.open(path, &err);
  if (rc) return fail(rc, "%s", err.c_str());
  const nq::GgufTensor *t = f.find(tensor_name);
  if (!t) return fail(NQ_ERR_ARG, "tensor '%s' not found in %s", tensor_name, path);
  if (t->type != 8) return fail(NQ_ERR_DTYPE, "tensor '%s' has ggml type %u, expected Q8_0 (8)", tensor_name, t->type);
  if (t->dims.size() != 2) return fail(NQ_ERR_SHAPE, "tensor '%s' is %zu-D, expected 2-D", tensor_name, t->dims.size());
  const int64_t k = static_cast<int64_t>(t->dims[0]);
  const int64_t n = static_cast<int64_t>(t->dims[1]);
  rc = check_weight_shape(n, k, flags);
  if (rc) return rc;
  const size_t bytes = static_cast<size_t>(n) * (k / 32) * 34;
  const uint8_t *p = f.data(*t, bytes);
  if (!p) return fail(NQ_ERR_FORMAT, "tensor '%s' data lies beyond the end of the file", tensor_name);
  return upload_packed(p, n, k, flags, out);
}

int nq_gguf_tensor_info(const char *path, const char *tensor_name, int *ggml_type, int64_t *n, int64_t *k) {
  if (!path || !tensor_name) return fail(NQ_ERR_ARG, "null argument");
  nq::GgufFile f;
  std::string err;
  int rc = f.open(path, &err);
  if (rc) return fail(rc, "%s", err.c_str());
  const nq::GgufTensor *t = f.find(tensor_name);
  if (!t) return fail(NQ_ERR_ARG, "tensor '%s' not found in %s", tensor_name, path);
  if (ggml_type) *ggml_type = static_cast<int>(t->type);
  if (t->dims.size() != 2) return fail(NQ_ERR_SHAPE, "tensor '%s' is %zu-D, expected 2-D", tensor_name, t->dims.size());
  if (k) *k = static_cast<int64_t>(t->dims[0]);
  if (n) *n = static_cast<int64_t>(t->dims[1]);
  return NQ_OK;
}

int nq_weight_to_q8_0(const nq_weight *w, void *blocks_out) {
  if (!w || !blocks_out) return fail(NQ_ERR_ARG, "null argument");
  if (w->bf16_only) return fail(NQ_ERR_UNSUPPORTED, "a bf16-only weight has no Q8_0 blocks");
  std::vector<uint8_t> host(w->bytes);
  cudaError_t e = cudaMemcpy(host.data(), w->dev, w->bytes, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(weight readback)");
  nq::unpack_q8_0(host.data(), w->n, w->k, w->flags, static_cast<uint8_t *>(blocks_out));
  return NQ_OK;
}

int nq_weights_fuse(const nq_weight *const *ws, int count, int flags, nq_weight **out) {
  if (!ws || count <= 0 || !out) return fail(NQ_ERR_ARG, "null argument");
  int64_t k = -1, n_total = 0;
  for (int i = 0; i < count; ++i) {
    if (!ws[i]) return fail(NQ_ERR_ARG, "null weight %d", i);
    if (ws[i]->flags & NQ_PACK_GLU) return fail(NQ_ERR_UNSUPPORTED, "cannot fuse GLU-packed weights");
    if (ws[i]->bf16_only) return fail(NQ_ERR_UNSUPPORTED, "cannot fuse bf16-only weights");
    if (k < 0) k = ws[i]->k;
    if (ws[i]->k != k) return fail(NQ_ERR_SHAPE, "fused weights must share K");
    n_total += ws[i]->n;
  }
  int rc = check_weight_shape(n_total, k, flags);
  if (rc) return rc;
  const size_t row_bytes = static_cast<size_t>(k / 32) * 34;
  std::vector<uint8_t> blocks(static_cast<size_t>(n_total) * row_bytes);
  size_t off = 0;
  for (int i = 0; i < count; ++i) {
    rc = nq_weight_to_q8_0(ws[i], blocks.data() + off);
    if (rc) return rc;
    off += static_cast<size_t>(ws[i]->n) * row_bytes;
  }
  return upload_packed(blocks.data(), n_total, k, flags, out);
}

int nq_weight_shape(const nq_weight *w, int64_t *n, int64_t *k, int *flags) {
  if (!w) return fail(NQ_ERR_ARG, "null weight");
  if (n) *n = w->n;
  if (k) *k = w->k;
  if (flags) *flags = w->flags;
  return NQ_OK;
}

int nq_weight_keep_bf16(nq_weight *w, int keep) {
  if (!w) return fail(NQ_ERR_ARG, "null weight");
  int cur = 0;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (cur != w->device) return fail(NQ_ERR_ARG, "weight lives on device %d, current device is %d", w->device, cur);
  if (!keep) {
    if (w->bf16_only) return fail(NQ_ERR_UNSUPPORTED, "the bf16 copy is a bf16-only weight's only copy");
    if (w->bf16) {
      e = cudaDeviceSynchronize();  // no launch in flight may still read it
      if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize(drop bf16 copy)");
      cudaFree(w->bf16);
      w->bf16 = nullptr;
    }
    return NQ_OK;
  }
  if (w->bf16) return NQ_OK;
  const size_t bytes = static_cast<size_t>(w->n_tiles) * nq::kPackRows * w->kc * nq::kPackK * 2;
  __nv_bfloat16 *buf = nullptr;
  e = cudaMalloc(&buf, bytes);
  if (e != cudaSuccess) return fail(NQ_ERR_CUDA, "cudaMalloc(bf16 weight copy, %zu bytes): %s", bytes, cudaGetErrorString(e));
  cudaStream_t st = nullptr;
  e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = nq::launch_dequant_tiles(w->dev, w->n_tiles, w->kc, buf, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (st) cudaStreamDestroy(st);
  if (e != cudaSuccess) {
    cudaFree(buf);
    return cuda_fail(e, "dequantize bf16 weight copy");
  }
  w->bf16 = buf;
  return NQ_OK;
}

void nq_weight_free(nq_weight *w) {
  if (!w) return;
  int cur = 0;
  cudaGetDevice(&cur);
  if (cur != w->device) cudaSetDevice(w->device);
  if (w->bf16) cudaFree(w->bf16);
  if (w->dev) cudaFree(w->dev);
  if (w->tap) cudaFree(w->tap);
  if (w->poly) cudaFree(w->poly);
  if (cur != w->device) cudaSetDevice(cur);
  delete w;
}

int nq_linear(const nq_weight *w, const void *x, int x_dtype, int64_t m, int64_t ldx, const float *bias, int epilogue,
              void *y, int y_dtype, int64_t ldy, void *stream) {
  LinearArgs a{w, bias, y, ldy};
  return linear_impl(&a, 1, x, x_dtype, m, ldx, epilogue, y_dtype, stream);
}

int64_t nq_conv1d_out_len(int64_t t_in, int kernel, int stride, int padding, int dilation) {
  if (t_in < 1 || kernel < 1 || stride < 1 || padding < 0 || dilation < 1) return NQ_ERR_ARG;
  const int64_t span = static_cast<int64_t>(dilation) * (kernel - 1) + 1;
  if (t_in + 2 * padding < span) return NQ_ERR_SHAPE;
  return (t_in + 2 * padding - span) / stride + 1;
}

int64_t nq_conv_transpose1d_out_len(int64_t t_in, int kernel, int stride, int padding, int output_padding) {
  if (t_in < 1 || kernel < 1 || stride < 1 || padding < 0 || output_padding < 0) return NQ_ERR_ARG;
  const int64_t t = (t_in - 1) * stride - 2 * padding + kernel + output_padding;
  return t < 1 ? NQ_ERR_SHAPE : t;
}

int nq_conv1d(const nq_weight *w, const void *x, int x_dtype, int64_t c_in, int64_t t_in, int64_t ldx, int kernel,
              int stride, int padding, int dilation, float x_leaky, const float *bias, int epilogue, void *y,
              int y_dtype, int64_t ldy, void *stream) {
  if (!w || !x || !y) return fail(NQ_ERR_ARG, "null argument");
  if (x_dtype != NQ_F32 && x_dtype != NQ_BF16) return fail(NQ_ERR_DTYPE, "x dtype %d unsupported", x_dtype);
  if (y_dtype != NQ_F32 && y_dtype != NQ_BF16) return fail(NQ_ERR_DTYPE, "y dtype %d unsupported", y_dtype);
  if (w->flags & NQ_PACK_GLU) return fail(NQ_ERR_UNSUPPORTED, "nq_conv1d: GLU-packed weight");
  if (epilogue == NQ_EPI_GLU_SIGMOID || epilogue == NQ_EPI_GLU_SILU)
    return fail(NQ_ERR_UNSUPPORTED, "nq_conv1d: GLU epilogue");
  if (c_in < 1 || kernel < 1 || w->k != c_in * kernel)
    return fail(NQ_ERR_SHAPE, "nq_conv1d: weight K = %lld is not c_in (%lld) x kernel (%d)", (long long)w->k,
                (long long)c_in, kernel);
  if (ldx < t_in) return fail(NQ_ERR_SHAPE, "nq_conv1d: ldx < t_in");
  const int64_t t_out = nq_conv1d_out_len(t_in, kernel, stride, padding, dilation);
  if (t_out < 0) return fail(static_cast<int>(t_out), "nq_conv1d: no output frames (t_in %lld)", (long long)t_in);
  if (ldy < t_out) return fail(NQ_ERR_SHAPE, "nq_conv1d: ldy < output length %lld", (long long)t_out);
  if (t_out > (1 << 30) || c_in * t_in > (1LL << 40)) return fail(NQ_ERR_SHAPE, "nq_conv1d: too large");
  DeviceCtx *ctx = nullptr;
  int dev = 0;
  int rc = current_ctx(&ctx, &dev);
  if (rc) return rc;
  if (w->device != dev) return fail(NQ_ERR_ARG, "weight lives on device %d, current device is %d", w->device, dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (g_conv_path == NQ_CONV_AUTO && stride == 1 && c_in % nq::kPackK == 0 && t_out > 16 && !(w->flags & NQ_MODE_QTILED))
    return conv1d_implicit(ctx, w, x, x_dtype, c_in, t_in, ldx, kernel, padding, dilation, x_leaky, bias, epilogue, y,
                           y_dtype, ldy, t_out, s);
  // im2col rows in x's precision (f32 rows go through the GEMM's hi/lo path),
  // the GEMM's token-major output in y's.
  const int64_t k_pad = static_cast<int64_t>(w->kc) * nq::kPackK;
  const size_t esz = x_dtype == NQ_F32 ? 4 : 2, ysz = y_dtype == NQ_F32 ? 4 : 2;
  const size_t rows_bytes = align_up(static_cast<size_t>(t_out) * k_pad * esz, 256);
  const size_t out_bytes = align_up(static_cast<size_t>(t_out) * w->n * ysz, 256);
  Workspace *ws = nullptr;
  rc = get_workspace(ctx, s, rows_bytes + out_bytes, &ws, true);
  if (rc) return rc;
  void *rows = ws->buf;
  void *ytmp = ws->buf + rows_bytes;
  cudaError_t e = nq::launch_im2col(x, x_dtype, ldx, static_cast<int>(c_in), static_cast<int>(t_in), kernel, stride,
                                    padding, dilation, x_leaky, static_cast<int>(t_out), k_pad, x_dtype, rows, s);
  if (e != cudaSuccess) return cuda_fail(e, "im2col launch");
  LinearArgs a{w, bias, ytmp, w->n};
  rc = linear_impl(&a, 1, rows, x_dtype, t_out, k_pad, epilogue, y_dtype, stream);
  if (rc) return rc;
  e = nq::launch_transpose_out(ytmp, y_dtype, w->n, static_cast<int>(t_out), static_cast<int>(w->n), y, y_dtype, ldy,
                               s);
  if (e != cudaSuccess) return cuda_fail(e, "conv output transpose launch");
  return NQ_OK;
}

int nq_conv_transpose1d_weight(const float *w, int64_t c_in, int64_t c_out, int kernel, nq_weight **out) {
  if (!w || !out) return fail(NQ_ERR_ARG, "null argument");
  if (c_in < 1 || c_out < 1 || kernel < 1) return fail(NQ_ERR_SHAPE, "nq_conv_transpose1d_weight: bad shape");
  // [c_in][c_out][K] -> rows (co, j) of c_in: the GEMM weight [c_out * K, c_in]
  const int64_t n = c_out * kernel;
  std::vector<float> t(static_cast<size_t>(n) * c_in);
  for (int64_t ci = 0; ci < c_in; ++ci)
    for (int64_t r = 0; r < n; ++r) {
      const float v = w[ci * n + r];
      if (!std::isfinite(v)) return fail(NQ_ERR_DTYPE, "nq_conv_transpose1d_weight: non-finite element");
      t[r * c_in + ci] = v;
    }
  int rc = check_weight_shape(n, (c_in + 31) / 32 * 32, 0);
  if (rc) return rc;
  return upload_bf16_only(t.data(), n, c_in, 0, out);
}

int nq_conv_transpose1d(const nq_weight *w, const void *x, int x_dtype, int64_t c_in, int64_t t_in, int64_t ldx,
                        int kernel, int stride, int padding, int output_padding, float x_leaky, const float *bias,
                        int epilogue, void *y, int y_dtype, int64_t ldy, void *stream) {
  if (!w || !x || !y) return fail(NQ_ERR_ARG, "null argument");
  if (x_dtype != NQ_F32 && x_dtype != NQ_BF16) return fail(NQ_ERR_DTYPE, "x dtype %d unsupported", x_dtype);
  if (y_dtype != NQ_F32 && y_dtype != NQ_BF16) return fail(NQ_ERR_DTYPE, "y dtype %d unsupported", y_dtype);
  if (epilogue < NQ_EPI_NONE || epilogue > NQ_EPI_RELU || epilogue == NQ_EPI_GLU_SIGMOID ||
      epilogue == NQ_EPI_GLU_SILU)
    return fail(NQ_ERR_UNSUPPORTED, "nq_conv_transpose1d: epilogue %d", epilogue);
  if (kernel < 1 || w->k != c_in || w->n % kernel != 0 || (w->flags & NQ_PACK_GLU))
    return fail(NQ_ERR_SHAPE, "nq_conv_transpose1d: weight [%lld, %lld] is not [c_out * %d, c_in %lld]",
                (long long)w->n, (long long)w->k, kernel, (long long)c_in);
  if (ldx < t_in) return fail(NQ_ERR_SHAPE, "nq_conv_transpose1d: ldx < t_in");
  const int64_t t_out = nq_conv_transpose1d_out_len(t_in, kernel, stride, padding, output_padding);
  if (t_out < 0) return fail(static_cast<int>(t_out), "nq_conv_transpose1d: no output frames");
  if (ldy < t_out) return fail(NQ_ERR_SHAPE, "nq_conv_transpose1d: ldy < output length %lld", (long long)t_out);
  if (t_out > (1 << 30) || c_in * t_in > (1LL << 40)) return fail(NQ_ERR_SHAPE, "nq_conv_transpose1d: too large");
  DeviceCtx *ctx = nullptr;
  int dev = 0;
  int rc = current_ctx(&ctx, &dev);
  if (rc) return rc;
  if (w->device != dev) return fail(NQ_ERR_ARG, "weight lives on device %d, current device is %d", w->device, dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t c_out = w->n / kernel;
  // Polyphase implicit GEMM: input positions q in [q0, q1] reach an output
  // frame (t = q stride + r - padding in [0, t_out) for some phase r).
  auto floor_div = [](int64_t a, int64_t b) { return a >= 0 ? a / b : -((-a + b - 1) / b); };
  const int64_t q0 = floor_div(padding - (stride - 1), stride);
  const int64_t q1 = floor_div(t_out - 1 + padding, stride);
  const int64_t mq = q1 - q0 + 1;
  if (g_conv_path == NQ_CONV_AUTO && c_in % nq::kPackK == 0 && mq > 16 && w->bf16)
    return conv_transpose1d_implicit(ctx, w, x, x_dtype, c_in, t_in, ldx, kernel, stride, padding, x_leaky, bias,
                                     epilogue, y, y_dtype, ldy, t_out, q0, mq, s);
  const int64_t k_pad = static_cast<int64_t>(w->kc) * nq::kPackK;
  const size_t esz = x_dtype == NQ_F32 ? 4 : 2;
  const size_t rows_bytes = align_up(static_cast<size_t>(t_in) * k_pad * esz, 256);
  const size_t cols_bytes = align_up(static_cast<size_t>(t_in) * w->n * 4, 256);
  Workspace *ws = nullptr;
  rc = get_workspace(ctx, s, rows_bytes + cols_bytes, &ws, true);
  if (rc) return rc;
  void *rows = ws->buf;
  float *cols = reinterpret_cast<float *>(ws->buf + rows_bytes);
  // token-major input rows: the im2col of a 1-tap, stride-1 conv
  cudaError_t e = nq::launch_im2col(x, x_dtype, ldx, static_cast<int>(c_in), static_cast<int>(t_in), 1, 1, 0, 1,
                                    x_leaky, static_cast<int>(t_in), k_pad, x_dtype, rows, s);
  if (e != cudaSuccess) return cuda_fail(e, "conv_transpose input transpose launch");
  LinearArgs a{w, nullptr, cols, w->n};
  rc = linear_impl(&a, 1, rows, x_dtype, t_in, k_pad, NQ_EPI_NONE, NQ_F32, stream);
  if (rc) return rc;
  e = nq::launch_col2im(cols, w->n, static_cast<int>(t_in), static_cast<int>(c_out), kernel, stride, padding,
                        static_cast<int>(t_out), bias, epilogue, y, y_dtype, ldy, s);
  if (e != cudaSuccess) return cuda_fail(e, "col2im launch");
  return NQ_OK;
}

int nq_gemv_noalloc(const nq_weight *w, const void *x, int x_dtype, int64_t m, int64_t ldx, const float *bias,
                    int epilogue, void *y, int y_dtype, int64_t ldy, void *stream) {
  int rc = validate(w, x, x_dtype, m, ldx, epilogue, y, y_dtype, ldy);
  if (rc) return rc;
  if (m > 16) return fail(NQ_ERR_SHAPE, "nq_gemv_noalloc serves M <= 16 rows (got %lld)", (long long)m);
  if (w->flags & NQ_MODE_QTILED) return fail(NQ_ERR_UNSUPPORTED, "nq_gemv_noalloc: NQ_MODE_QTILED weight");
  if (w->bf16_only) return fail(NQ_ERR_UNSUPPORTED, "nq_gemv_noalloc: bf16-only weight");
  if (m == 0) return NQ_OK;
  DeviceCtx *ctx = nullptr;
  int dev = 0;
  rc = current_ctx(&ctx, &dev);
  if (rc) return rc;
  if (w->device != dev) return fail(NQ_ERR_ARG, "weight lives on device %d, current device is %d", w->device, dev);
  cudaStream_t stream_ = static_cast<cudaStream_t>(stream);
  // Same work split as nq_linear's GEMV, so both give the same sums.
  const int kc = w->kc;
  const nq::GemvPlan plan = nq::gemv_plan(ctx->sm_count, w->n_tiles, kc, static_cast<int>(m));
  const bool splitx = x_dtype == NQ_F32;
  const bool direct = gemv_x_direct(x, x_dtype, ldx, w->k);
  const int64_t k_pad = static_cast<int64_t>(kc) * nq::kPackK;
  const size_t plane = align_up(static_cast<size_t>(m) * k_pad * 2, 256);
  const size_t x_bytes = direct ? 0 : plane * (splitx ? 2 : 1);
  const size_t part_bytes = gemv_partial_bytes(plan, w->n_tiles, m);
  if (part_bytes > kNoAllocPartialBytes)
    return fail(NQ_ERR_SHAPE,
                "nq_gemv_noalloc: this weight (N=%lld, K=%lld) needs %zu bytes of split-K scratch; the static "
                "scratch holds %zu",
                (long long)w->n, (long long)w->k, part_bytes, kNoAllocPartialBytes);
  if (x_bytes > kNoAllocXBytes)
    return fail(NQ_ERR_SHAPE,
                "nq_gemv_noalloc: staging these activations (M=%lld, K=%lld) needs %zu bytes; the static scratch "
                "holds %zu",
                (long long)m, (long long)w->k, x_bytes, kNoAllocXBytes);
  unsigned char *scratch = nullptr;
  rc = noalloc_scratch(dev, &scratch);
  if (rc) return rc;
  unsigned char *xplanes = scratch + kNoAllocPartialBytes;
  // The work counter starts at zero (static storage) and every call's
  // gemv_reduce re-arms it.
  int *sched = reinterpret_cast<int *>(scratch + kNoAllocPartialBytes + kNoAllocXBytes);
  nq::GemvParams p;
  std::memset(&p, 0, sizeof(p));
  nq::GemvProblem &pr = p.prob[0];
  pr.w = w->dev;
  pr.n_tiles = w->n_tiles;
  pr.N = w->n;
  pr.glu = (w->flags & NQ_PACK_GLU) ? 1 : 0;
  pr.n_out = out_width(w);
  pr.bias = bias;
  pr.y = y;
  pr.ldy = ldy;
  pr.partials = reinterpret_cast<float *>(scratch);
  p.sched = sched;
  p.sm_count = ctx->sm_count;
  p.path = g_gemv_path;
  if (direct) {
    p.xh = static_cast<const __nv_bfloat16 *>(x);
    p.ldx = ldx;
  } else {
    __nv_bfloat16 *hi = reinterpret_cast<__nv_bfloat16 *>(xplanes);
    __nv_bfloat16 *lo = splitx ? reinterpret_cast<__nv_bfloat16 *>(xplanes + plane) : nullptr;
    cudaError_t e = nq::launch_split_x(x, x_dtype, ldx, m, w->k, k_pad, hi, lo, stream_);
    if (e != cudaSuccess) return cuda_fail(e, "split_x launch");
    p.xh = hi;
    p.xl = lo;
    p.ldx = k_pad;
  }
  p.M = static_cast<int>(m);
  p.epi = epilogue;
  p.y_dtype = y_dtype;
  p.nprob = 1;
  p.kc = kc;
  p.unit = plan.unit;
  p.upt = plan.upt;
  p.units = plan.units;
  p.ctas = plan.ctas;
  p.ctl.status = ctx->status;
  p.ctl.wait_limit = g_wait_limit;
  double flops = 0, bytes = 0;
  LinearArgs la{w, bias, y, ldy};
  linear_cost(&la, 1, m, x_dtype, y_dtype, &flops, &bytes);
  ProfScope ps(NQ_KCLASS_GEMV, stream_, flops, bytes);
  cudaError_t e = nq::launch_gemv(p, plan.ctas, stream_);
  if (e != cudaSuccess) {
    // The GEMV may have launched and bumped the shared work counter before
    // its reduce (which re-arms it) failed to launch: zero it on the stream.
    cudaMemsetAsync(sched, 0, sizeof(int), stream_);
    return cuda_fail(e, "GEMV launch");
  }
  return NQ_OK;
}

int nq_gemv_resadd_ln(const nq_weight *w, const void *x, int x_dtype, int64_t m, int64_t ldx, const float *bias,
                      const float *res_in, float *res_out, int64_t ld_res, const float *ln_gamma,
                      const float *ln_beta, float eps, void *norm_out, int out_dtype, int64_t ld_out, void *stream) {
  int rc = validate(w, x, x_dtype, m, ldx, NQ_EPI_NONE, norm_out, out_dtype, ld_out);
  if (rc) return rc;
  if (!res_in || !res_out || !ln_gamma) return fail(NQ_ERR_ARG, "nq_gemv_resadd_ln: null residual or gamma");
  if (m > 16) return fail(NQ_ERR_SHAPE, "nq_gemv_resadd_ln serves M <= 16 rows (got %lld)", (long long)m);
  if (w->flags & NQ_PACK_GLU) return fail(NQ_ERR_ARG, "nq_gemv_resadd_ln: GLU-packed weight");
  if (w->flags & NQ_MODE_QTILED) return fail(NQ_ERR_UNSUPPORTED, "nq_gemv_resadd_ln: NQ_MODE_QTILED weight");
  if (w->bf16_only) return fail(NQ_ERR_UNSUPPORTED, "nq_gemv_resadd_ln: bf16-only weight");
  if (w->n > nq::kGemvLnMaxN)
    return fail(NQ_ERR_SHAPE, "nq_gemv_resadd_ln: N = %lld exceeds %d", (long long)w->n, nq::kGemvLnMaxN);
  if (ld_res < w->n) return fail(NQ_ERR_SHAPE, "nq_gemv_resadd_ln: ld_res < N");
  if (!(eps >= 0.f)) return fail(NQ_ERR_ARG, "nq_gemv_resadd_ln: eps must be >= 0");
  if (m == 0) return NQ_OK;
  DeviceCtx *ctx = nullptr;
  int dev = 0;
  rc = current_ctx(&ctx, &dev);
  if (rc) return rc;
  if (w->device != dev) return fail(NQ_ERR_ARG, "weight lives on device %d, current device is %d", w->device, dev);
  LinearArgs a{w, bias, norm_out, ld_out};
  GemvResLn rl{res_in, res_out, ld_res, ln_gamma, ln_beta, eps};
  return run_gemv(ctx, &a, 1, x, x_dtype, m, ldx, NQ_EPI_NONE, out_dtype, static_cast<cudaStream_t>(stream), &rl);
}

int nq_chain_create(nq_chain **out) {
  if (!out) return fail(NQ_ERR_ARG, "null argument");
  DeviceCtx *ctx = nullptr;
  int dev = 0;
  int rc = current_ctx(&ctx, &dev);
  if (rc) return rc;
  nq_chain *c = new nq_chain;
  c->device = dev;
  *out = c;
  return NQ_OK;
}


int nq_chain_linear(nq_chain *c, const nq_weight *w, const void *x, const float *bias, int epilogue, void *y,
                    int y_dtype) {
  return chain_add(c, w, x, bias, epilogue, y, y_dtype, nullptr, nullptr, nullptr, nullptr, 0.f);
}

int nq_chain_gemv_resadd_ln(nq_chain *c, const nq_weight *w, const void *x, const float *bias, const float *res_in,
                            float *res_out, const float *ln_gamma, const float *ln_beta, float eps, void *norm_out) {
  if (!res_out) return fail(NQ_ERR_ARG, "nq_chain_gemv_resadd_ln: null residual output");
  return chain_add(c, w, x, bias, NQ_EPI_NONE, norm_out, NQ_BF16, res_in, res_out, ln_gamma, ln_beta, eps);
}

int nq_chain_steps(const nq_chain *c) { return c ? static_cast<int>(c->steps.size()) : NQ_ERR_ARG; }

int nq_chain_run(nq_chain *c, void *stream) {
  if (!c) return fail(NQ_ERR_ARG, "null chain");
  if (c->steps.empty()) return NQ_OK;
  DeviceCtx *ctx = nullptr;
  int dev = 0;
  int rc = current_ctx(&ctx, &dev);
  if (rc) return rc;
  if (dev != c->device) return fail(NQ_ERR_ARG, "the chain lives on device %d, current device is %d", c->device, dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!c->uploaded) {
    rc = chain_upload(c, ctx, s);
    if (rc) return rc;
  }
  nq::ChainParams p;
  p.steps = c->d_steps;
  p.n_steps = static_cast<int>(c->steps.size());
  p.ready = c->d_counters;
  p.ctl.status = ctx->status;
  p.ctl.wait_limit = g_wait_limit;
  ProfScope ps(NQ_KCLASS_GEMV, s, c->flops, c->bytes);
  cudaError_t e = nq::launch_chain(p, c->ctas, s);
  if (e != cudaSuccess) return cuda_fail(e, "decode chain launch");
  return NQ_OK;
}

void nq_chain_free(nq_chain *c) {
  if (!c) return;
  if (c->uploaded) {
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != c->device) cudaSetDevice(c->device);
    cudaDeviceSynchronize();  // no run may still read the step table or counters
    {
      std::lock_guard<std::mutex> lk(g_ctx[c->device].mu);
      g_ctx[c->device].chain_counters.erase(c->d_counters);
    }
    cudaFree(c->d_steps);
    cudaFree(c->d_counters);
    if (cur != c->device) cudaSetDevice(cur);
  }
  delete c;
}

int nq_matmul(const nq_weight *w, const void *a, int a_dtype, void *c, int c_dtype, int64_t m, void *stream) {
  if (!w) return fail(NQ_ERR_ARG, "null weight");
  return nq_linear(w, a, a_dtype, m, w->k, nullptr, NQ_EPI_NONE, c, c_dtype, w->n, stream);
}

int nq_matmul_bias(const nq_weight *w, const void *a, int a_dtype, const float *bias, void *c, int c_dtype, int64_t m,
                   void *stream) {
  if (!w) return fail(NQ_ERR_ARG, "null weight");
  return nq_linear(w, a, a_dtype, m, w->k, bias, NQ_EPI_NONE, c, c_dtype, w->n, stream);
}

int nq_matmul_bias_gelu(const nq_weight *w, const void *a, int a_dtype, const float *bias, void *c, int c_dtype,
                        int64_t m, void *stream) {
  if (!w) return fail(NQ_ERR_ARG, "null weight");
  return nq_linear(w, a, a_dtype, m, w->k, bias, NQ_EPI_GELU_ERF, c, c_dtype, w->n, stream);
}

int nq_gemv_splitk(const nq_weight *w, const void *x, int x_dtype, const float *bias, void *out, int out_dtype,
                   void *stream) {
  if (!w) return fail(NQ_ERR_ARG, "null weight");
  return nq_linear(w, x, x_dtype, 1, w->k, bias, NQ_EPI_NONE, out, out_dtype, w->n, stream);
}

int nq_gemv_glu_splitk(const nq_weight *w, const void *x, int x_dtype, const float *bias, void *out, int out_dtype,
                       void *stream) {
  if (!w) return fail(NQ_ERR_ARG, "null weight");
  return nq_linear(w, x, x_dtype, 1, w->k, bias, NQ_EPI_GLU_SILU, out, out_dtype, w->n / 2, stream);
}

int nq_gemv_qkv_splitk(const nq_weight *wq, const nq_weight *wk, const nq_weight *wv, const void *x, int x_dtype,
                       void *q, void *k, void *v, int out_dtype, void *stream) {
  if (!wq || !wk || !wv) return fail(NQ_ERR_ARG, "null weight");
  if (wq->k != wk->k || wq->k != wv->k) return fail(NQ_ERR_SHAPE, "Q/K/V weights must share K");
  LinearArgs a[3] = {{wq, nullptr, q, wq->n}, {wk, nullptr, k, wk->n}, {wv, nullptr, v, wv->n}};
  return linear_impl(a, 3, x, x_dtype, 1, wq->k, NQ_EPI_NONE, out_dtype, stream);
}

int nq_last_error(char *buf, int len) {
  const int n = static_cast<int>(t_err.size());
  if (buf && len > 0) {
    const int c = std::min(n, len - 1);
    std::memcpy(buf, t_err.data(), c);
    buf[c] = 0;
  }
  return n;
}

int nq_status(void *stream, int *bits) {
  DeviceCtx *ctx = nullptr;
  int rc = current_ctx(&ctx, nullptr);
  if (rc) return rc;
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  int v = 0;
  e = cudaMemcpy(&v, ctx->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(status)");
  if (bits) *bits = v;
  if (v) {
    cudaMemset(ctx->status, 0, sizeof(int));
    // A kernel that gave up may have left split-K counters armed: re-zero them.
    std::lock_guard<std::mutex> lk(ctx->mu);
    for (auto &kv : ctx->ws)
      if (kv.second.counters) cudaMemset(kv.second.counters, 0, kCounterSlots * sizeof(int));
    for (auto &kv : ctx->chain_counters) cudaMemset(kv.first, 0, kv.second);
    return fail(NQ_ERR_TIMEOUT, "device status 0x%x: a bounded wait in a kernel ran out", v);
  }
  return NQ_OK;
}

int nq_launch_counter(int64_t *count, int reset) {
  if (!count) return fail(NQ_ERR_ARG, "null count");
  *count = reset ? nq::g_launches.exchange(0) : nq::g_launches.load();
  return NQ_OK;
}

int nq_profile_enable(int on) {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  g_prof.on = on != 0;
  return NQ_OK;
}

int nq_profile_read(int kernel_class, int64_t *launches, double *total_ms, double *flops, double *bytes, int reset) {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  int64_t n = 0;
  double ms = 0, fl = 0, by = 0;
  for (const auto &r : g_prof.records) {
    if (r.kclass != kernel_class) continue;
    cudaError_t e = cudaEventSynchronize(r.stop);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventSynchronize(profile)");
    float t = 0.f;
    e = cudaEventElapsedTime(&t, r.start, r.stop);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventElapsedTime(profile)");
    ++n;
    ms += t;
    fl += r.flops;
    by += r.bytes;
  }
  if (launches) *launches = n;
  if (total_ms) *total_ms = ms;
  if (flops) *flops = fl;
  if (bytes) *bytes = by;
  if (reset) {
    std::vector<ProfRecord> keep;
    for (const auto &r : g_prof.records) {
      if (r.kclass != kernel_class) {
        keep.push_back(r);
        continue;
      }
      cudaEventSynchronize(r.stop);
      g_prof.pool.push_back(r.start);
      g_prof.pool.push_back(r.stop);
    }
    g_prof.records.swap(keep);
  }
  return NQ_OK;
}

int nq_set_gemm_path(int path) {
  if (path != NQ_GEMM_AUTO && path != NQ_GEMM_FUSED && path != NQ_GEMM_DEQUANT)
    return fail(NQ_ERR_ARG, "unknown GEMM path %d", path);
  g_gemm_path = path;
  return NQ_OK;
}

int nq_set_gemm_unit_tokens(int tokens) {
  if (tokens != 0 && !nq::gemm_bf16_unit_ok(tokens))
    return fail(NQ_ERR_ARG, "GEMM unit width %d (use 0, 64, 128 or 256)", tokens);
  g_gemm_unit_tokens = tokens;
  return NQ_OK;
}

int nq_set_gemm_tail_split(int mode) {
  if (mode < 0 || mode > 16) return fail(NQ_ERR_ARG, "tail split mode %d (0 auto, 1 off, 2..16 pieces)", mode);
  g_tail_split = mode;
  return NQ_OK;
}

int nq_set_gemv_path(int path) {
  if (path != NQ_GEMV_AUTO && path != NQ_GEMV_SPLIT && path != NQ_GEMV_CLUSTER)
    return fail(NQ_ERR_ARG, "GEMV path %d (0 auto, 1 split + reduce, 2 cluster)", path);
  g_gemv_path = path;
  return NQ_OK;
}

int nq_set_conv_path(int path) {
  if (path != NQ_CONV_AUTO && path != NQ_CONV_IM2COL)
    return fail(NQ_ERR_ARG, "conv path %d (0 auto, 1 im2col)", path);
  g_conv_path = path;
  return NQ_OK;
}

int nq_set_attention_kernel(int kernel) {
  if (kernel != NQ_ATTENTION_TCGEN05 && kernel != NQ_ATTENTION_MMA_SYNC)
    return fail(NQ_ERR_ARG, "attention kernel %d (0 tcgen05, 1 mma.sync)", kernel);
  g_attention_kernel = kernel;
  return NQ_OK;
}

int nq_set_wait_limit(int64_t cycles) {
  if (cycles <= 0) return fail(NQ_ERR_ARG, "wait limit must be positive");
  g_wait_limit = cycles;
  return NQ_OK;
}

int nq_debug_wait_timeout(void *stream) {
  DeviceCtx *ctx = nullptr;
  int rc = current_ctx(&ctx, nullptr);
  if (rc) return rc;
  nq::DevCtl ctl{ctx->status, g_wait_limit};
  cudaError_t e = nq::launch_wait_timeout_probe(ctl, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "probe launch");
  return NQ_OK;
}

}  // extern "C"
