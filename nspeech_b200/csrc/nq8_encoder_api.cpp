// nq8_encoder_api.cpp -- FastConformer encoder runner of libnq8 (C ABI in
// include/nq8.h).  Host orchestration of FastConformerEncoder::forward
// (src/parakeet/fast_conformer.rs:1072-1104, blocks :967-999) over the Q8_0
// kernels (nq_linear) and the glue kernels of nq8_encoder_kernels.cu.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/nq8.h"
#include "nq8_encoder.h"
#include "nq8_host.h"

namespace {

using nq::api_fail;

struct HostTensor {
  int type = 0;  // 0 f32, 8 Q8_0
  std::vector<int64_t> dims;
  std::vector<uint8_t> bytes;
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
  }
};

struct DevBuf {
  void *p = nullptr;
  size_t bytes = 0;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  // Grow to `want` bytes.  Work queued on `st` (the stream that uses the
  // buffer) may still read the old allocation: synchronize it before the free.
  int ensure(size_t want, cudaStream_t st = nullptr) {
    if (bytes >= want) return NQ_OK;
    if (p) {
      cudaError_t e = cudaStreamSynchronize(st);
      if (e != cudaSuccess)
        return api_fail(NQ_ERR_CUDA, std::string("cudaStreamSynchronize(arena growth): ") + cudaGetErrorString(e));
      cudaFree(p);
    }
    p = nullptr;
    bytes = 0;
    cudaError_t e = cudaMalloc(&p, want);
    if (e != cudaSuccess) return api_fail(NQ_ERR_CUDA, std::string("cudaMalloc(encoder arena): ") + cudaGetErrorString(e));
    bytes = want;
    return NQ_OK;
  }
  template <class T>
  T *as() const { return static_cast<T *>(p); }
};

struct Layer {
  nq_weight *ff1_w1 = nullptr, *ff1_w2 = nullptr, *ff2_w1 = nullptr, *ff2_w2 = nullptr;
  nq_weight *qkv = nullptr, *o = nullptr, *rel = nullptr, *pw1 = nullptr, *pw2 = nullptr;
  float *ff1_b1, *ff1_b2, *ff2_b1, *ff2_b2, *qkv_b, *o_b, *pw1_b, *pw2_b;
  float *bias_u, *bias_v, *dw_w, *dw_b, *bn_scale, *bn_shift;
  float *ln_ff1_g, *ln_ff1_b, *ln_mha_g, *ln_mha_b, *ln_conv_g, *ln_conv_b, *ln_ff2_g, *ln_ff2_b, *ln_out_g, *ln_out_b;
};

}  // namespace

// The buffers of one forward (sized for the largest batch seen), and the ring
// of pinned host slots through which each forward's segment lengths (4 x
// batch ints) travel, each slot reused only after its previous copy
// completed.
struct Arena {
  DevBuf x, h, t, u, u32, qkv, pos, krel, vrel, att, g, c, s1, s2a, s2b, s3a, s3b, flat, mel_in, out_buf;
  static constexpr int kLenSlots = 4;
  DevBuf lens[kLenSlots];
  int *lens_host[kLenSlots] = {nullptr, nullptr, nullptr, nullptr};
  cudaEvent_t lens_done[kLenSlots] = {nullptr, nullptr, nullptr, nullptr};
  int lens_cap = 0;
  int lens_next = 0;
  ~Arena() {
    for (int i = 0; i < kLenSlots; ++i) {
      if (lens_done[i]) {
        cudaEventSynchronize(lens_done[i]);
        cudaEventDestroy(lens_done[i]);
      }
      if (lens_host[i]) cudaFreeHost(lens_host[i]);
    }
  }
};

struct nq_encoder {
  nq_encoder_config cfg{};
  int device = 0;
  bool ready = false;
  std::map<std::string, HostTensor> staged;
  std::vector<void *> dev_allocs;  // f32 parameter vectors
  std::vector<nq_weight *> weights;
  std::vector<Layer> layers;
  // subsampling
  float *c0_w, *c0_b, *dw2_w, *dw2_b, *dw5_w, *dw5_b, *pw3_b, *pw6_b, *lin_b;
  nq_weight *pw3 = nullptr, *pw6 = nullptr, *lin = nullptr;
  // The layers' relative-key projections stacked along N ([n_layers * d, d]):
  // they depend only on the positions, so one GEMM per forward serves all
  // layers (krel holds [2T-1][n_layers * d]).
  nq_weight *rel_all = nullptr;
  // bias_v - bias_u of every layer, [n_layers][d] f32: with the stacked
  // relative keys it gives each layer's (v - u) . r table (relpos_bias).
  float *vmu_all = nullptr;
  float *zero_d = nullptr;  // [d] zeros: the mma.sync attention's u (already in q)
  // Activation arenas, one per stream (created on a stream's first forward):
  // forwards on one stream reuse its arena in stream order; forwards on
  // different streams have their own and may run concurrently.
  std::mutex arena_mu;
  std::map<cudaStream_t, std::unique_ptr<Arena>> arenas;

  // nq_encoder_forward_host_async: two device staging slots (mel in, output
  // out) used in turn, copies on their own streams ordered by events.
  struct HostSlot {
    DevBuf in, out;
    cudaEvent_t h2d_done = nullptr, comp_done = nullptr, d2h_done = nullptr;
    bool used = false;
  };
  HostSlot host_slots[2];
  cudaStream_t h2d_stream = nullptr, d2h_stream = nullptr;
  int host_next = 0;
  // Serializes nq_encoder_forward_host_async callers (slot choice, the lazy
  // stream creation and the enqueue of one call's copies and forward).
  std::mutex host_mu;

  ~nq_encoder() {
    if (h2d_stream) cudaStreamSynchronize(h2d_stream);
    if (d2h_stream) cudaStreamSynchronize(d2h_stream);
    for (auto &hs : host_slots)
      for (cudaEvent_t ev : {hs.h2d_done, hs.comp_done, hs.d2h_done})
        if (ev) cudaEventDestroy(ev);
    if (h2d_stream) cudaStreamDestroy(h2d_stream);
    if (d2h_stream) cudaStreamDestroy(d2h_stream);
    arenas.clear();
    for (auto *w : weights) nq_weight_free(w);
    for (auto *p : dev_allocs) cudaFree(p);
  }
};

namespace {

int check_cfg(const nq_encoder_config &c) {
  if (c.feat_in <= 0 || c.feat_in % 8) return api_fail(NQ_ERR_SHAPE, "feat_in must be a positive multiple of 8");
  if (c.d_model != 1024 && c.d_model != 512) return api_fail(NQ_ERR_UNSUPPORTED, "d_model must be 1024 or 512");
  if (c.n_heads <= 0 || c.d_model % c.n_heads || c.d_model / c.n_heads != 128)
    return api_fail(NQ_ERR_UNSUPPORTED, "head dim (d_model / n_heads) must be 128");
  if (c.ff_mult <= 0 || c.n_layers <= 0) return api_fail(NQ_ERR_SHAPE, "ff_mult and n_layers must be positive");
  if (c.conv_kernel <= 0 || c.conv_kernel % 2 == 0 || c.conv_kernel > 31)
    return api_fail(NQ_ERR_UNSUPPORTED, "conv_kernel must be odd and <= 31");
  if (c.sub_channels <= 0 || c.sub_channels % 32 || c.sub_channels > 1024)
    return api_fail(NQ_ERR_UNSUPPORTED, "sub_channels must be a multiple of 32, <= 1024");
  if ((c.sub_channels * (c.feat_in / 8)) % 32) return api_fail(NQ_ERR_SHAPE, "subsampling flatten dim must be a multiple of 32");
  return NQ_OK;
}

int sub_len(int L) { return L <= 0 ? 0 : (L - 1) / 2 + 1; }

const HostTensor *find(const nq_encoder *e, const std::string &name) {
  auto it = e->staged.find(name);
  return it == e->staged.end() ? nullptr : &it->second;
}

// Upload an f32 vector of `n` elements (or fill with `fill` when absent and
// `optional`).
int vec(nq_encoder *e, const std::string &name, int64_t n, bool optional, float fill, float **out) {
  const HostTensor *t = find(e, name);
  std::vector<float> host(n, fill);
  if (t) {
    if (t->type != 0) return api_fail(NQ_ERR_DTYPE, name + " must be F32");
    if (t->numel() != n) return api_fail(NQ_ERR_SHAPE, name + " has " + std::to_string(t->numel()) + " elements, expected " + std::to_string(n));
    std::memcpy(host.data(), t->bytes.data(), n * sizeof(float));
  } else if (!optional) {
    return api_fail(NQ_ERR_ARG, "missing tensor " + name);
  }
  void *p = nullptr;
  cudaError_t err = cudaMalloc(&p, n * sizeof(float));
  if (err != cudaSuccess) return api_fail(NQ_ERR_CUDA, "cudaMalloc(encoder parameter)");
  e->dev_allocs.push_back(p);
  err = cudaMemcpy(p, host.data(), n * sizeof(float), cudaMemcpyHostToDevice);
  if (err != cudaSuccess) return api_fail(NQ_ERR_CUDA, "cudaMemcpy(encoder parameter)");
  *out = static_cast<float *>(p);
  return NQ_OK;
}

// Host Q8_0 blocks of a [n, k] matrix (k = product of the inner dims).
int q8_blocks(nq_encoder *e, const std::string &name, int64_t n, int64_t k, std::vector<uint8_t> *blocks) {
  const HostTensor *t = find(e, name);
  if (!t) return api_fail(NQ_ERR_ARG, "missing tensor " + name);
  if (t->dims.empty() || t->dims[0] != n || t->numel() != n * k)
    return api_fail(NQ_ERR_SHAPE, name + " has the wrong shape (expected [" + std::to_string(n) + ", " + std::to_string(k) + "])");
  blocks->resize(static_cast<size_t>(n) * (k / 32) * 34);
  if (t->type == 8) {
    if (t->bytes.size() != blocks->size()) return api_fail(NQ_ERR_SHAPE, name + " Q8_0 byte size mismatch");
    std::memcpy(blocks->data(), t->bytes.data(), blocks->size());
  } else {
    nq::quantize_q8_0(reinterpret_cast<const float *>(t->bytes.data()), n, k, blocks->data());
  }
  return NQ_OK;
}

int matrix(nq_encoder *e, const std::string &name, int64_t n, int64_t k, int flags, nq_weight **out) {
  std::vector<uint8_t> b;
  int rc = q8_blocks(e, name, n, k, &b);
  if (rc) return rc;
  rc = nq_weight_from_q8_0(b.data(), n, k, flags, out);
  if (rc) return rc;
  e->weights.push_back(*out);
  return NQ_OK;
}

#define NQ_TRY(x)        \
  do {                   \
    int rc_ = (x);       \
    if (rc_) return rc_; \
  } while (0)

#define NQ_CUDA(x)                                                                                   \
  do {                                                                                               \
    cudaError_t e_ = (x);                                                                            \
    if (e_ != cudaSuccess) return api_fail(NQ_ERR_CUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
  } while (0)

int finalize(nq_encoder *e) {
  const auto &c = e->cfg;
  const int64_t d = c.d_model, ff = static_cast<int64_t>(c.d_model) * c.ff_mult, C = c.sub_channels;
  const int64_t flat = C * (c.feat_in / 8);
  const std::string sp = "encoder.subsampling.";
  NQ_TRY(vec(e, sp + "layers.0.weight", C * 9, false, 0.f, &e->c0_w));
  NQ_TRY(vec(e, sp + "layers.0.bias", C, true, 0.f, &e->c0_b));
  NQ_TRY(vec(e, sp + "layers.2.weight", C * 9, false, 0.f, &e->dw2_w));
  NQ_TRY(vec(e, sp + "layers.2.bias", C, true, 0.f, &e->dw2_b));
  NQ_TRY(matrix(e, sp + "layers.3.weight", C, C, 0, &e->pw3));
  NQ_TRY(vec(e, sp + "layers.3.bias", C, true, 0.f, &e->pw3_b));
  NQ_TRY(vec(e, sp + "layers.5.weight", C * 9, false, 0.f, &e->dw5_w));
  NQ_TRY(vec(e, sp + "layers.5.bias", C, true, 0.f, &e->dw5_b));
  NQ_TRY(matrix(e, sp + "layers.6.weight", C, C, 0, &e->pw6));
  NQ_TRY(vec(e, sp + "layers.6.bias", C, true, 0.f, &e->pw6_b));
  NQ_TRY(matrix(e, sp + "linear.weight", d, flat, 0, &e->lin));
  NQ_TRY(vec(e, sp + "linear.bias", d, true, 0.f, &e->lin_b));

  e->layers.resize(c.n_layers);
  for (int i = 0; i < c.n_layers; ++i) {
    Layer &L = e->layers[i];
    const std::string p = "encoder.layers." + std::to_string(i) + ".";
    NQ_TRY(matrix(e, p + "feed_forward1.linear1.weight", ff, d, 0, &L.ff1_w1));
    NQ_TRY(vec(e, p + "feed_forward1.linear1.bias", ff, true, 0.f, &L.ff1_b1));
    NQ_TRY(matrix(e, p + "feed_forward1.linear2.weight", d, ff, 0, &L.ff1_w2));
    NQ_TRY(vec(e, p + "feed_forward1.linear2.bias", d, true, 0.f, &L.ff1_b2));
    NQ_TRY(matrix(e, p + "feed_forward2.linear1.weight", ff, d, 0, &L.ff2_w1));
    NQ_TRY(vec(e, p + "feed_forward2.linear1.bias", ff, true, 0.f, &L.ff2_b1));
    NQ_TRY(matrix(e, p + "feed_forward2.linear2.weight", d, ff, 0, &L.ff2_w2));
    NQ_TRY(vec(e, p + "feed_forward2.linear2.bias", d, true, 0.f, &L.ff2_b2));
    // Fused Q/K/V: one [3d, d] weight and one [3d] bias.
    {
      std::vector<uint8_t> bq, bk, bv, all;
      NQ_TRY(q8_blocks(e, p + "self_attn.q_proj.weight", d, d, &bq));
      NQ_TRY(q8_blocks(e, p + "self_attn.k_proj.weight", d, d, &bk));
      NQ_TRY(q8_blocks(e, p + "self_attn.v_proj.weight", d, d, &bv));
      all.reserve(bq.size() * 3);
      all.insert(all.end(), bq.begin(), bq.end());
      all.insert(all.end(), bk.begin(), bk.end());
      all.insert(all.end(), bv.begin(), bv.end());
      NQ_TRY(nq_weight_from_q8_0(all.data(), 3 * d, d, 0, &L.qkv));
      e->weights.push_back(L.qkv);
      std::vector<float> b(3 * d, 0.f);
      const char *nm[3] = {"self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias"};
      for (int j = 0; j < 3; ++j) {
        const HostTensor *t = find(e, p + nm[j]);
        if (t) {
          if (t->type != 0 || t->numel() != d) return api_fail(NQ_ERR_SHAPE, p + nm[j] + " must be F32 [d]");
          std::memcpy(b.data() + j * d, t->bytes.data(), d * sizeof(float));
        }
      }
      void *pb = nullptr;
      NQ_CUDA(cudaMalloc(&pb, 3 * d * sizeof(float)));
      e->dev_allocs.push_back(pb);
      NQ_CUDA(cudaMemcpy(pb, b.data(), 3 * d * sizeof(float), cudaMemcpyHostToDevice));
      L.qkv_b = static_cast<float *>(pb);
    }
    NQ_TRY(matrix(e, p + "self_attn.o_proj.weight", d, d, 0, &L.o));
    NQ_TRY(vec(e, p + "self_attn.o_proj.bias", d, true, 0.f, &L.o_b));
    NQ_TRY(matrix(e, p + "self_attn.relative_k_proj.weight", d, d, 0, &L.rel));
    NQ_TRY(vec(e, p + "self_attn.bias_u", d, false, 0.f, &L.bias_u));
    NQ_TRY(vec(e, p + "self_attn.bias_v", d, false, 0.f, &L.bias_v));
    NQ_TRY(matrix(e, p + "conv.pointwise_conv1.weight", 2 * d, d, NQ_PACK_GLU, &L.pw1));
    NQ_TRY(vec(e, p + "conv.pointwise_conv1.bias", 2 * d, true, 0.f, &L.pw1_b));
    NQ_TRY(vec(e, p + "conv.depthwise_conv.weight", d * c.conv_kernel, false, 0.f, &L.dw_w));
    NQ_TRY(vec(e, p + "conv.depthwise_conv.bias", d, true, 0.f, &L.dw_b));
    {
      // Eval-mode BatchNorm folded to y = x * scale + shift (eps 1e-5, f32).
      std::vector<float> g(d, 1.f), bb(d, 0.f), mean(d, 0.f), var(d, 1.f);
      const char *nm[4] = {"conv.norm.weight", "conv.norm.bias", "conv.norm.running_mean", "conv.norm.running_var"};
      std::vector<float> *dst[4] = {&g, &bb, &mean, &var};
      for (int j = 0; j < 4; ++j) {
        const HostTensor *t = find(e, p + nm[j]);
        if (!t) continue;
        if (t->type != 0 || t->numel() != d) return api_fail(NQ_ERR_SHAPE, p + nm[j] + " must be F32 [d]");
        std::memcpy(dst[j]->data(), t->bytes.data(), d * sizeof(float));
      }
      std::vector<float> sc(d), sh(d);
      for (int64_t j = 0; j < d; ++j) {
        sc[j] = g[j] / std::sqrt(var[j] + 1e-5f);
        sh[j] = bb[j] - mean[j] * sc[j];
      }
      void *ps = nullptr, *ph = nullptr;
      NQ_CUDA(cudaMalloc(&ps, d * sizeof(float)));
      e->dev_allocs.push_back(ps);
      NQ_CUDA(cudaMalloc(&ph, d * sizeof(float)));
      e->dev_allocs.push_back(ph);
      NQ_CUDA(cudaMemcpy(ps, sc.data(), d * sizeof(float), cudaMemcpyHostToDevice));
      NQ_CUDA(cudaMemcpy(ph, sh.data(), d * sizeof(float), cudaMemcpyHostToDevice));
      L.bn_scale = static_cast<float *>(ps);
      L.bn_shift = static_cast<float *>(ph);
    }
    NQ_TRY(matrix(e, p + "conv.pointwise_conv2.weight", d, d, 0, &L.pw2));
    NQ_TRY(vec(e, p + "conv.pointwise_conv2.bias", d, true, 0.f, &L.pw2_b));
    const char *norms[5] = {"norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out"};
    float **gs[5] = {&L.ln_ff1_g, &L.ln_mha_g, &L.ln_conv_g, &L.ln_ff2_g, &L.ln_out_g};
    float **bs[5] = {&L.ln_ff1_b, &L.ln_mha_b, &L.ln_conv_b, &L.ln_ff2_b, &L.ln_out_b};
    for (int j = 0; j < 5; ++j) {
      NQ_TRY(vec(e, p + norms[j] + ".weight", d, true, 1.f, gs[j]));
      NQ_TRY(vec(e, p + norms[j] + ".bias", d, true, 0.f, bs[j]));
    }
  }
  // Every encoder GEMM runs the dequantize-once path for M >= 128 tokens:
  // keep each weight's bf16 copy (MatMul::PackedBf16 semantics) instead of
  // re-dequantizing it on every call.  Costs 2 bytes per weight element.
  {
    std::vector<const nq_weight *> rels;
    for (const Layer &L : e->layers) rels.push_back(L.rel);
    NQ_TRY(nq_weights_fuse(rels.data(), static_cast<int>(rels.size()), 0, &e->rel_all));
    e->weights.push_back(e->rel_all);
  }
  {
    // u moves into the q projection's bias (q + u comes out of the QKV GEMM,
    // rounded once); attention keeps v - u: (q + v) . r = (q + u) . r + (v - u) . r.
    std::vector<float> vmu(static_cast<size_t>(c.n_layers) * d), bu(d), bv(d), bq(3 * d);
    for (int i = 0; i < c.n_layers; ++i) {
      Layer &L = e->layers[i];
      NQ_CUDA(cudaMemcpy(bu.data(), L.bias_u, d * sizeof(float), cudaMemcpyDeviceToHost));
      NQ_CUDA(cudaMemcpy(bv.data(), L.bias_v, d * sizeof(float), cudaMemcpyDeviceToHost));
      NQ_CUDA(cudaMemcpy(bq.data(), L.qkv_b, 3 * d * sizeof(float), cudaMemcpyDeviceToHost));
      for (int64_t j = 0; j < d; ++j) {
        vmu[i * d + j] = bv[j] - bu[j];
        bq[j] += bu[j];
      }
      NQ_CUDA(cudaMemcpy(L.qkv_b, bq.data(), 3 * d * sizeof(float), cudaMemcpyHostToDevice));
    }
    void *pv = nullptr, *pz = nullptr;
    NQ_CUDA(cudaMalloc(&pv, vmu.size() * sizeof(float)));
    e->dev_allocs.push_back(pv);
    NQ_CUDA(cudaMemcpy(pv, vmu.data(), vmu.size() * sizeof(float), cudaMemcpyHostToDevice));
    e->vmu_all = static_cast<float *>(pv);
    NQ_CUDA(cudaMalloc(&pz, d * sizeof(float)));
    e->dev_allocs.push_back(pz);
    NQ_CUDA(cudaMemset(pz, 0, d * sizeof(float)));
    e->zero_d = static_cast<float *>(pz);
  }
  NQ_TRY(nq_weight_keep_bf16(e->pw3, 1));
  NQ_TRY(nq_weight_keep_bf16(e->pw6, 1));
  NQ_TRY(nq_weight_keep_bf16(e->lin, 1));
  NQ_TRY(nq_weight_keep_bf16(e->rel_all, 1));
  for (Layer &L : e->layers)
    for (nq_weight *w : {L.ff1_w1, L.ff1_w2, L.qkv, L.o, L.pw1, L.pw2, L.ff2_w1, L.ff2_w2})
      NQ_TRY(nq_weight_keep_bf16(w, 1));
  e->staged.clear();
  e->ready = true;
  return NQ_OK;
}

struct Shapes {
  int B, Tm, F, C, T1, F1, T2, F2, T3, F3, D, M;
};

Shapes shapes(const nq_encoder *e, int batch, int t_mel) {
  Shapes s;
  s.B = batch;
  s.Tm = t_mel;
  s.F = e->cfg.feat_in;
  s.C = e->cfg.sub_channels;
  s.T1 = sub_len(t_mel);
  s.F1 = sub_len(s.F);
  s.T2 = sub_len(s.T1);
  s.F2 = sub_len(s.F1);
  s.T3 = sub_len(s.T2);
  s.F3 = sub_len(s.F2);
  s.D = e->cfg.d_model;
  s.M = batch * s.T3;
  return s;
}

Arena *arena_for(nq_encoder *e, cudaStream_t st) {
  std::lock_guard<std::mutex> lk(e->arena_mu);
  std::unique_ptr<Arena> &a = e->arenas[st];
  if (!a) a.reset(new Arena());
  return a.get();
}

int ensure_arena(nq_encoder *e, Arena &A, const Shapes &s, cudaStream_t st) {
  const size_t M = s.M, D = s.D, ff = static_cast<size_t>(D) * e->cfg.ff_mult;
  const size_t P = 2 * static_cast<size_t>(s.T3) - 1;
  NQ_TRY(A.x.ensure(M * D * 4, st));
  NQ_TRY(A.h.ensure(M * D * 2, st));
  NQ_TRY(A.t.ensure(M * ff * 2, st));
  NQ_TRY(A.u.ensure(M * D * 2, st));
  NQ_TRY(A.u32.ensure(M * D * 4, st));
  NQ_TRY(A.qkv.ensure(M * 3 * D * 2, st));
  NQ_TRY(A.pos.ensure(P * D * 2, st));
  NQ_TRY(A.krel.ensure(P * D * e->cfg.n_layers * 2, st));
  if (nq::attention_tc(s.T3)) NQ_TRY(A.vrel.ensure(P * (D / 128) * e->cfg.n_layers * 4, st));
  NQ_TRY(A.att.ensure(M * D * 2, st));
  NQ_TRY(A.g.ensure(M * D * 2, st));
  NQ_TRY(A.c.ensure(M * D * 2, st));
  if (!nq::enc::conv0_dw_s2_supported(s.F, s.F1, s.C))
    NQ_TRY(A.s1.ensure(static_cast<size_t>(s.B) * s.T1 * s.F1 * s.C * 2, st));
  NQ_TRY(A.s2a.ensure(static_cast<size_t>(s.B) * s.T2 * s.F2 * s.C * 2, st));
  NQ_TRY(A.s2b.ensure(static_cast<size_t>(s.B) * s.T2 * s.F2 * s.C * 2, st));
  NQ_TRY(A.s3a.ensure(static_cast<size_t>(s.B) * s.T3 * s.F3 * s.C * 2, st));
  NQ_TRY(A.s3b.ensure(static_cast<size_t>(s.B) * s.T3 * s.F3 * s.C * 2, st));
  NQ_TRY(A.flat.ensure(static_cast<size_t>(s.B) * s.T3 * s.F3 * s.C * 2, st));
  if (A.lens_cap < s.B) {
    for (int i = 0; i < Arena::kLenSlots; ++i) {
      if (A.lens_done[i]) NQ_CUDA(cudaEventSynchronize(A.lens_done[i]));
      if (A.lens_host[i]) cudaFreeHost(A.lens_host[i]);
      NQ_CUDA(cudaMallocHost(&A.lens_host[i], static_cast<size_t>(4) * s.B * sizeof(int)));
      NQ_TRY(A.lens[i].ensure(static_cast<size_t>(4) * s.B * sizeof(int), st));
      if (!A.lens_done[i]) NQ_CUDA(cudaEventCreateWithFlags(&A.lens_done[i], cudaEventDisableTiming));
    }
    A.lens_cap = s.B;
  }
  return NQ_OK;
}

#define NQ_K(x) NQ_CUDA(x)

int forward(nq_encoder *e, const float *mel, const int32_t *lengths, int batch, int t_mel, float *out,
            int32_t *out_lengths, cudaStream_t st) {
  const Shapes s = shapes(e, batch, t_mel);
  Arena &A = *arena_for(e, st);
  NQ_TRY(ensure_arena(e, A, s, st));
  const int slot = A.lens_next;
  A.lens_next = (slot + 1) % Arena::kLenSlots;
  NQ_CUDA(cudaEventSynchronize(A.lens_done[slot]));  // its previous upload has been consumed
  int *lh = A.lens_host[slot];
  for (int b = 0; b < batch; ++b) {
    const int L0 = lengths ? lengths[b] : t_mel;
    if (L0 < 1 || L0 > t_mel) return api_fail(NQ_ERR_SHAPE, "segment length out of range [1, t_mel]");
    lh[b] = L0;
    lh[batch + b] = sub_len(L0);
    lh[2 * batch + b] = sub_len(lh[batch + b]);
    lh[3 * batch + b] = sub_len(lh[2 * batch + b]);
    if (out_lengths) out_lengths[b] = lh[3 * batch + b];
  }
  int *ld = A.lens[slot].as<int>();
  NQ_CUDA(cudaMemcpyAsync(ld, lh, static_cast<size_t>(4) * batch * sizeof(int), cudaMemcpyHostToDevice, st));
  NQ_CUDA(cudaEventRecord(A.lens_done[slot], st));
  const int *L0 = ld, *L1 = ld + batch, *L2 = ld + 2 * batch, *L3 = ld + 3 * batch;
  const auto &c = e->cfg;
  const int D = s.D, H = c.n_heads, FF = D * c.ff_mult, M = s.M, Tp = s.T3;
  void *stv = st;
  const float eps = 1e-5f;
  __nv_bfloat16 *h = A.h.as<__nv_bfloat16>(), *t = A.t.as<__nv_bfloat16>(), *u = A.u.as<__nv_bfloat16>();
  float *x = A.x.as<float>();

  // --- subsampling (fast_conformer.rs:172-188)
  if (nq::enc::conv0_dw_s2_supported(s.F, s.F1, s.C)) {
    NQ_K(nq::enc::conv0_dw_s2(mel, L0, L1, s.B, s.Tm, s.F, s.T1, s.F1, s.T2, s.F2, s.C, e->c0_w, e->c0_b, e->dw2_w,
                              e->dw2_b, A.s2a.as<__nv_bfloat16>(), st));
  } else {
    NQ_K(nq::enc::conv0_relu(mel, L0, s.B, s.Tm, s.F, s.T1, s.F1, s.C, e->c0_w, e->c0_b, A.s1.as<__nv_bfloat16>(), st));
    NQ_K(nq::enc::dwconv2d_s2(A.s1.as<__nv_bfloat16>(), L1, s.B, s.T1, s.F1, s.T2, s.F2, s.C, e->dw2_w, e->dw2_b,
                              A.s2a.as<__nv_bfloat16>(), st));
  }
  NQ_TRY(nq_linear(e->pw3, A.s2a.p, NQ_BF16, static_cast<int64_t>(s.B) * s.T2 * s.F2, s.C, e->pw3_b, NQ_EPI_RELU,
                   A.s2b.p, NQ_BF16, s.C, stv));
  NQ_K(nq::enc::dwconv2d_s2(A.s2b.as<__nv_bfloat16>(), L2, s.B, s.T2, s.F2, s.T3, s.F3, s.C, e->dw5_w, e->dw5_b,
                            A.s3a.as<__nv_bfloat16>(), st));
  NQ_TRY(nq_linear(e->pw6, A.s3a.p, NQ_BF16, static_cast<int64_t>(s.B) * s.T3 * s.F3, s.C, e->pw6_b, NQ_EPI_RELU,
                   A.s3b.p, NQ_BF16, s.C, stv));
  NQ_K(nq::enc::flatten_cf(A.s3b.as<__nv_bfloat16>(), M, s.F3, s.C, A.flat.as<__nv_bfloat16>(), st));
  NQ_TRY(nq_linear(e->lin, A.flat.p, NQ_BF16, M, static_cast<int64_t>(s.F3) * s.C, e->lin_b, NQ_EPI_NONE, A.u32.p,
                   NQ_F32, D, stv));
  const float alpha = c.scale_input ? std::sqrt(static_cast<float>(D)) : 1.0f;
  const Layer &L_0 = e->layers[0];
  NQ_TRY(nq::layer_norm_rows(nq::enc::kLnScale, x, A.u32.p, alpha, M, D, L_0.ln_ff1_g, L_0.ln_ff1_b, nullptr, nullptr, h,
                        eps, st));
  NQ_K(nq::enc::relpos(Tp, D, A.pos.as<__nv_bfloat16>(), st));
  // relative keys of every layer: krel[p][li * D + :] = pos[p] . W_rel(li)^T
  NQ_TRY(nq_linear(e->rel_all, A.pos.p, NQ_BF16, 2 * Tp - 1, D, nullptr, NQ_EPI_NONE, A.krel.p, NQ_BF16,
                   static_cast<int64_t>(c.n_layers) * D, stv));
  // (v - u) . r of every layer, head and relative row (tcgen05 attention)
  const bool att_tc = nq::attention_tc(Tp);
  if (att_tc) NQ_TRY(nq::relpos_bias(A.krel.as<__nv_bfloat16>(), e->vmu_all, 2 * Tp - 1, c.n_layers, D, A.vrel.as<float>(), st));

  for (int li = 0; li < c.n_layers; ++li) {
    const Layer &L = e->layers[li];
    // FF1 (x0.5) -> norm_self_att
    NQ_TRY(nq_linear(L.ff1_w1, h, NQ_BF16, M, D, L.ff1_b1, NQ_EPI_SILU, t, NQ_BF16, FF, stv));
    NQ_TRY(nq_linear(L.ff1_w2, t, NQ_BF16, M, FF, L.ff1_b2, NQ_EPI_NONE, u, NQ_BF16, D, stv));
    NQ_TRY(nq::layer_norm_rows(nq::enc::kLnResAdd, x, u, 0.5f, M, D, L.ln_mha_g, L.ln_mha_b, nullptr, nullptr, h, eps, st));
    // MHSA with relative positions -> norm_conv
    NQ_TRY(nq_linear(L.qkv, h, NQ_BF16, M, D, L.qkv_b, NQ_EPI_NONE, A.qkv.p, NQ_BF16, 3 * D, stv));
    NQ_TRY(nq::relpos_attention(A.qkv.as<__nv_bfloat16>(), A.krel.as<__nv_bfloat16>() + static_cast<size_t>(li) * D,
                                static_cast<int64_t>(c.n_layers) * D, e->zero_d, e->vmu_all + static_cast<size_t>(li) * D,
                                att_tc ? A.vrel.as<float>() + static_cast<size_t>(li) * H * (2 * Tp - 1) : nullptr,
                                L3, s.B, Tp, H, D, A.att.as<__nv_bfloat16>(), st));
    NQ_TRY(nq_linear(L.o, A.att.p, NQ_BF16, M, D, L.o_b, NQ_EPI_NONE, u, NQ_BF16, D, stv));
    NQ_TRY(nq::layer_norm_rows(nq::enc::kLnResAdd, x, u, 1.0f, M, D, L.ln_conv_g, L.ln_conv_b, nullptr, nullptr, h, eps, st));
    // Conv module -> norm_feed_forward2
    NQ_TRY(nq_linear(L.pw1, h, NQ_BF16, M, D, L.pw1_b, NQ_EPI_GLU_SIGMOID, A.g.p, NQ_BF16, D, stv));
    NQ_K(nq::enc::dwconv1d_bn_silu(A.g.as<__nv_bfloat16>(), L3, s.B, Tp, D, c.conv_kernel, L.dw_w, L.dw_b, L.bn_scale,
                                   L.bn_shift, A.c.as<__nv_bfloat16>(), st));
    NQ_TRY(nq_linear(L.pw2, A.c.p, NQ_BF16, M, D, L.pw2_b, NQ_EPI_NONE, u, NQ_BF16, D, stv));
    NQ_TRY(nq::layer_norm_rows(nq::enc::kLnResAdd, x, u, 1.0f, M, D, L.ln_ff2_g, L.ln_ff2_b, nullptr, nullptr, h, eps, st));
    // FF2 (x0.5) -> norm_out (-> next layer's norm_feed_forward1)
    NQ_TRY(nq_linear(L.ff2_w1, h, NQ_BF16, M, D, L.ff2_b1, NQ_EPI_SILU, t, NQ_BF16, FF, stv));
    NQ_TRY(nq_linear(L.ff2_w2, t, NQ_BF16, M, FF, L.ff2_b2, NQ_EPI_NONE, u, NQ_BF16, D, stv));
    const Layer *nx = li + 1 < c.n_layers ? &e->layers[li + 1] : nullptr;
    NQ_TRY(nq::layer_norm_rows(nq::enc::kLnResAddOut, x, u, 0.5f, M, D, L.ln_out_g, L.ln_out_b,
                          nx ? nx->ln_ff1_g : nullptr, nx ? nx->ln_ff1_b : nullptr, h, eps, st));
  }
  NQ_K(nq::enc::copy_masked(x, L3, s.B, Tp, D, out, st));
  return NQ_OK;
}

}  // namespace

// ======================================================================= ABI
extern "C" {

int nq_encoder_create(const nq_encoder_config *cfg, nq_encoder **out) {
  if (!cfg || !out) return api_fail(NQ_ERR_ARG, "null argument");
  NQ_TRY(check_cfg(*cfg));
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return api_fail(NQ_ERR_CUDA, "cudaGetDevice failed");
  std::unique_ptr<nq_encoder> e(new nq_encoder);
  e->cfg = *cfg;
  e->device = dev;
  *out = e.release();
  return NQ_OK;
}

int nq_encoder_set_tensor(nq_encoder *enc, const char *name, int ggml_type, const void *data, const int64_t *dims,
                          int n_dims) {
  if (!enc || !name || !data || (!dims && n_dims > 0)) return api_fail(NQ_ERR_ARG, "null argument");
  if (enc->ready) return api_fail(NQ_ERR_ARG, "encoder already finalized");
  if (ggml_type != 0 && ggml_type != 8) return api_fail(NQ_ERR_DTYPE, std::string(name) + ": only F32 (0) and Q8_0 (8)");
  if (n_dims < 1 || n_dims > 4) return api_fail(NQ_ERR_SHAPE, std::string(name) + ": 1 to 4 dims");
  HostTensor t;
  t.type = ggml_type;
  t.dims.assign(dims, dims + n_dims);
  const int64_t n = t.numel();
  if (n <= 0) return api_fail(NQ_ERR_SHAPE, std::string(name) + ": empty tensor");
  size_t bytes;
  if (ggml_type == 0) {
    bytes = static_cast<size_t>(n) * 4;
  } else {
    if (dims[n_dims - 1] % 32 && n_dims == 2) return api_fail(NQ_ERR_SHAPE, std::string(name) + ": inner dim % 32");
    if (n % 32) return api_fail(NQ_ERR_SHAPE, std::string(name) + ": Q8_0 element count % 32");
    bytes = static_cast<size_t>(n / 32) * 34;
  }
  t.bytes.assign(static_cast<const uint8_t *>(data), static_cast<const uint8_t *>(data) + bytes);
  enc->staged[name] = std::move(t);
  return NQ_OK;
}

int nq_encoder_load_gguf(nq_encoder *enc, const char *path) {
  if (!enc || !path) return api_fail(NQ_ERR_ARG, "null argument");
  nq::GgufFile f;
  std::string err;
  int rc = f.open(path, &err);
  if (rc) return api_fail(rc, err);
  int loaded = 0;
  for (const auto &t : f.tensors()) {
    if (t.name.compare(0, 8, "encoder.") != 0) continue;
    if (t.type != 0 && t.type != 8) return api_fail(NQ_ERR_DTYPE, t.name + ": only F32 and Q8_0 tensors are supported");
    std::vector<int64_t> dims(t.dims.rbegin(), t.dims.rend());  // GGUF ne0 is innermost
    int64_t n = 1;
    for (auto d : dims) n *= d;
    const size_t bytes = t.type == 0 ? static_cast<size_t>(n) * 4 : static_cast<size_t>(n / 32) * 34;
    const uint8_t *p = f.data(t, bytes);
    if (!p) return api_fail(NQ_ERR_FORMAT, t.name + ": data beyond the end of the file");
    rc = nq_encoder_set_tensor(enc, t.name.c_str(), static_cast<int>(t.type), p, dims.data(), static_cast<int>(dims.size()));
    if (rc) return rc;
    ++loaded;
  }
  if (!loaded) return api_fail(NQ_ERR_ARG, "no encoder.* tensors in the file");
  return NQ_OK;
}

int nq_encoder_finalize(nq_encoder *enc) {
  if (!enc) return api_fail(NQ_ERR_ARG, "null encoder");
  if (enc->ready) return NQ_OK;
  int cur = 0;
  cudaGetDevice(&cur);
  if (cur != enc->device) return api_fail(NQ_ERR_ARG, "encoder belongs to another device");
  return finalize(enc);
}

int nq_encoder_out_frames(int t_mel) { return sub_len(sub_len(sub_len(t_mel))); }

int nq_encoder_forward(nq_encoder *enc, const float *mel, const int32_t *lengths, int batch, int t_mel, float *out,
                       int32_t *out_lengths, void *stream) {
  if (!enc || !mel || !out) return api_fail(NQ_ERR_ARG, "null argument");
  if (!enc->ready) return api_fail(NQ_ERR_ARG, "encoder not finalized");
  if (batch < 1 || t_mel < 1) return api_fail(NQ_ERR_SHAPE, "batch and t_mel must be positive");
  return forward(enc, mel, lengths, batch, t_mel, out, out_lengths, static_cast<cudaStream_t>(stream));
}

int nq_encoder_forward_host(nq_encoder *enc, const float *mel_host, const int32_t *lengths, int batch, int t_mel,
                            float *out_host, int32_t *out_lengths, void *stream) {
  if (!enc || !mel_host || !out_host) return api_fail(NQ_ERR_ARG, "null argument");
  if (!enc->ready) return api_fail(NQ_ERR_ARG, "encoder not finalized");
  if (batch < 1 || t_mel < 1) return api_fail(NQ_ERR_SHAPE, "batch and t_mel must be positive");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t in_bytes = static_cast<size_t>(batch) * t_mel * enc->cfg.feat_in * sizeof(float);
  const size_t out_bytes = static_cast<size_t>(batch) * nq_encoder_out_frames(t_mel) * enc->cfg.d_model * sizeof(float);
  Arena &A = *arena_for(enc, st);
  NQ_TRY(A.mel_in.ensure(in_bytes, st));
  NQ_TRY(A.out_buf.ensure(out_bytes, st));
  NQ_CUDA(cudaMemcpyAsync(A.mel_in.p, mel_host, in_bytes, cudaMemcpyHostToDevice, st));
  NQ_TRY(forward(enc, A.mel_in.as<float>(), lengths, batch, t_mel, A.out_buf.as<float>(), out_lengths, st));
  NQ_CUDA(cudaMemcpyAsync(out_host, A.out_buf.p, out_bytes, cudaMemcpyDeviceToHost, st));
  NQ_CUDA(cudaStreamSynchronize(st));
  return NQ_OK;
}

int nq_encoder_forward_host_async(nq_encoder *enc, const float *mel_host, const int32_t *lengths, int batch, int t_mel,
                                  float *out_host, int32_t *out_lengths, void *stream) {
  if (!enc || !mel_host || !out_host) return api_fail(NQ_ERR_ARG, "null argument");
  if (!enc->ready) return api_fail(NQ_ERR_ARG, "encoder not finalized");
  if (batch < 1 || t_mel < 1) return api_fail(NQ_ERR_SHAPE, "batch and t_mel must be positive");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lk(enc->host_mu);
  if (!enc->h2d_stream) {
    NQ_CUDA(cudaStreamCreateWithFlags(&enc->h2d_stream, cudaStreamNonBlocking));
    NQ_CUDA(cudaStreamCreateWithFlags(&enc->d2h_stream, cudaStreamNonBlocking));
    for (auto &hs : enc->host_slots)
      for (cudaEvent_t *ev : {&hs.h2d_done, &hs.comp_done, &hs.d2h_done})
        NQ_CUDA(cudaEventCreateWithFlags(ev, cudaEventDisableTiming));
  }
  nq_encoder::HostSlot &hs = enc->host_slots[enc->host_next];
  enc->host_next ^= 1;
  const size_t in_bytes = static_cast<size_t>(batch) * t_mel * enc->cfg.feat_in * sizeof(float);
  const size_t out_bytes = static_cast<size_t>(batch) * nq_encoder_out_frames(t_mel) * enc->cfg.d_model * sizeof(float);
  if (hs.in.bytes < in_bytes || hs.out.bytes < out_bytes) {
    // growing a slot frees its buffers: let its previous use finish first
    if (hs.used) NQ_CUDA(cudaEventSynchronize(hs.d2h_done));
    NQ_TRY(hs.in.ensure(in_bytes, enc->d2h_stream));
    NQ_TRY(hs.out.ensure(out_bytes, enc->d2h_stream));
  }
  // The slot's previous forward must have consumed its input, and its
  // previous output must have left for the host, before they are overwritten.
  if (hs.used) NQ_CUDA(cudaStreamWaitEvent(enc->h2d_stream, hs.comp_done, 0));
  NQ_CUDA(cudaMemcpyAsync(hs.in.p, mel_host, in_bytes, cudaMemcpyHostToDevice, enc->h2d_stream));
  NQ_CUDA(cudaEventRecord(hs.h2d_done, enc->h2d_stream));
  NQ_CUDA(cudaStreamWaitEvent(st, hs.h2d_done, 0));
  if (hs.used) NQ_CUDA(cudaStreamWaitEvent(st, hs.d2h_done, 0));
  NQ_TRY(forward(enc, hs.in.as<float>(), lengths, batch, t_mel, hs.out.as<float>(), out_lengths, st));
  NQ_CUDA(cudaEventRecord(hs.comp_done, st));
  NQ_CUDA(cudaStreamWaitEvent(enc->d2h_stream, hs.comp_done, 0));
  NQ_CUDA(cudaMemcpyAsync(out_host, hs.out.p, out_bytes, cudaMemcpyDeviceToHost, enc->d2h_stream));
  NQ_CUDA(cudaEventRecord(hs.d2h_done, enc->d2h_stream));
  hs.used = true;
  return NQ_OK;
}

int nq_encoder_wait(nq_encoder *enc) {
  if (!enc) return api_fail(NQ_ERR_ARG, "null encoder");
  if (enc->h2d_stream) NQ_CUDA(cudaStreamSynchronize(enc->h2d_stream));
  if (enc->d2h_stream) NQ_CUDA(cudaStreamSynchronize(enc->d2h_stream));
  return NQ_OK;
}

int nq_encoder_launch_count(const nq_encoder *enc, int batch, int t_mel) {
  if (!enc) return api_fail(NQ_ERR_ARG, "null encoder");
  if (!enc->ready) return api_fail(NQ_ERR_ARG, "encoder not finalized");
  if (batch < 1 || t_mel < 1) return api_fail(NQ_ERR_SHAPE, "batch and t_mel must be positive");
  // Same kernel sequence as forward(): glue kernels plus the launches each
  // nq_linear call makes for its M (GEMV, or GEMM with its dequantize,
  // activation-staging and split-K reduction kernels).
  const Shapes s = shapes(enc, batch, t_mel);
  const int M = s.M, Tp = s.T3;
  auto lin = [&](const nq_weight *w, int64_t m, int64_t ldx) { return nq::linear_launches(w, m, NQ_BF16, ldx % 8 == 0); };
  // conv0 + dwconv (fused when supported), dwconv, flatten, scaled LN, relpos
  int n = nq::enc::conv0_dw_s2_supported(s.F, s.F1, s.C) ? 5 : 6;
  n += lin(enc->pw3, static_cast<int64_t>(s.B) * s.T2 * s.F2, s.C);
  n += lin(enc->pw6, static_cast<int64_t>(s.B) * s.T3 * s.F3, s.C);
  n += lin(enc->lin, M, static_cast<int64_t>(s.F3) * s.C);
  n += lin(enc->rel_all, 2 * Tp - 1, s.D);  // every layer's relative keys
  if (nq::attention_tc(Tp)) n += 1;          // their (v - u) . r table
  for (const Layer &L : enc->layers) {
    n += 6;  // 4 LN, attention, depthwise conv
    n += lin(L.ff1_w1, M, s.D) + lin(L.ff1_w2, M, s.D * enc->cfg.ff_mult) + lin(L.qkv, M, s.D) +
         lin(L.o, M, s.D) + lin(L.pw1, M, s.D) + lin(L.pw2, M, s.D) +
         lin(L.ff2_w1, M, s.D) + lin(L.ff2_w2, M, s.D * enc->cfg.ff_mult);
  }
  return n + 1;  // final masked copy
}

void nq_encoder_free(nq_encoder *enc) { delete enc; }

}  // extern "C"
