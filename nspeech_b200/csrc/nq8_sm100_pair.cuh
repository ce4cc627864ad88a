// nq8_sm100_pair.cuh -- sm_100a helpers shared by the GEMM kernels: CTA-pair
// (cluster of two) signalling, cta_group::2 TMEM / MMA / TMA forms, TMEM
// loads and stores, and the typed epilogue stores.
#pragma once
#include "nq8_common.cuh"

namespace nq {

// ---------------------------------------------------------------- cluster
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory variable in cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Arrive on a barrier of the peer CTA.  The peer's signals that the MMA
// issuer waits for (TMEM stores done, TMEM loads done) only order tcgen05
// operations: the signalling warp has already waited for its own tcgen05
// operations and fenced them (tcgen05.fence::before_thread_sync), so the
// issuer waits with the CTA-scope try_wait of mbar_wait.  A cluster-scope
// acquire on that wait measurably slows the issue loop.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Relaxed remote arrive: signals only that this thread's earlier tcgen05 work
// is done (ordered by tcgen05.fence::before_thread_sync), with no release of
// its ordinary memory writes -- the release form waits for the thread's
// epilogue stores to become visible to the cluster first.
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// ---------------------------------------------------------------- tcgen05 x2
__device__ __forceinline__ void tmem_alloc2(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D(256 x N, split over the pair's TMEM) (+)= A(TMEM, 128 rows per CTA) . B^T
// (B: N rows, half in each CTA's shared memory at the same offset).
__device__ __forceinline__ void umma2_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same with both operands in shared memory: A 128 rows per CTA, B N/2 rows
// per CTA, each at the same offset in both CTAs.
__device__ __forceinline__ void umma2_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the barrier at `bar` (same offset) in both CTAs of the pair
// when the pair MMAs issued so far by this thread have completed.
__device__ __forceinline__ void umma2_commit_both(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(static_cast<unsigned short>(0x3))
      : "memory");
}
// TMA 2-D load into this CTA's shared memory whose byte count completes on an
// mbarrier of either CTA of the pair (here: the leader's).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

constexpr int kEc = 16;  // epilogue chunk: tokens per lane per tcgen05.ld
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// ------------------------------------------------------------ epilogue math
template <int EPI>
__device__ __forceinline__ float act_t(float v) {
  if (EPI == kEpiSilu) return v * sigmoidf_(v);
  if (EPI == kEpiGeluErf) return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
  if (EPI == kEpiRelu) return fmaxf(v, 0.0f);
  return v;
}
template <typename T>
__device__ __forceinline__ void put(T *p, float v);
template <>
__device__ __forceinline__ void put<float>(float *p, float v) { *p = v; }
template <>
__device__ __forceinline__ void put<__nv_bfloat16>(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

// kEc tokens of one output feature column: y[tok0 + e][n] (ldy elements apart).
template <typename T, int EPI>
__device__ __forceinline__ void store_col(T *base, int64_t ldy, int valid, const float (&v)[kEc], float b) {
  if (valid >= kEc) {
#pragma unroll
    for (int e = 0; e < kEc; ++e) put<T>(base + e * ldy, act_t<EPI>(v[e] + b));
  } else {
#pragma unroll
    for (int e = 0; e < kEc; ++e)
      if (e < valid) put<T>(base + e * ldy, act_t<EPI>(v[e] + b));
  }
}
// GLU output for kEc tokens: (v + b) * act(gate), gate already biased.
template <typename T, int EPI>
__device__ __forceinline__ void store_glu(T *base, int64_t ldy, int valid, const float (&v)[kEc], float b,
                                          const float (&g)[kEc]) {
#pragma unroll
  for (int e = 0; e < kEc; ++e) {
    if (e < valid) {
      const float a = v[e] + b;
      put<T>(base + e * ldy, EPI == kEpiGluSigmoid ? a * sigmoidf_(g[e]) : a * (g[e] * sigmoidf_(g[e])));
    }
  }
}

// Runtime (epilogue, output dtype) dispatch of store_col / store_glu; `off`
// is the element offset of token 0 of the chunk in y.
__device__ __forceinline__ void store_act(int epi, int y_dtype, void *y, int64_t off, int64_t ldy, int valid,
                                          const float (&v)[kEc], float b) {
  float *yf = static_cast<float *>(y) + off;
  __nv_bfloat16 *yb = static_cast<__nv_bfloat16 *>(y) + off;
  switch (epi * 2 + y_dtype) {
    case kEpiNone * 2 + 0: store_col<float, kEpiNone>(yf, ldy, valid, v, b); break;
    case kEpiNone * 2 + 1: store_col<__nv_bfloat16, kEpiNone>(yb, ldy, valid, v, b); break;
    case kEpiSilu * 2 + 0: store_col<float, kEpiSilu>(yf, ldy, valid, v, b); break;
    case kEpiSilu * 2 + 1: store_col<__nv_bfloat16, kEpiSilu>(yb, ldy, valid, v, b); break;
    case kEpiGeluErf * 2 + 0: store_col<float, kEpiGeluErf>(yf, ldy, valid, v, b); break;
    case kEpiGeluErf * 2 + 1: store_col<__nv_bfloat16, kEpiGeluErf>(yb, ldy, valid, v, b); break;
    case kEpiRelu * 2 + 0: store_col<float, kEpiRelu>(yf, ldy, valid, v, b); break;
    default: store_col<__nv_bfloat16, kEpiRelu>(yb, ldy, valid, v, b); break;
  }
}
// bf16 output of kEc tokens from a warp whose lanes hold 32 consecutive
// output features (lane parity = feature parity, all 32 valid, all kEc tokens
// valid).  Lanes pair up through one shuffle per token pair so that every
// store writes two adjacent features (4 bytes): the even lane stores tokens
// [0, kEc/2), the odd lane tokens [kEc/2, kEc).  `pair_base` is the element
// offset of token 0 and the pair's even feature.  Half the store
// instructions of store_col, the same values.
template <int EPI>
__device__ __forceinline__ void store_pair_bf16(__nv_bfloat16 *pair_base, int64_t ldy, int lane, const float (&v)[kEc],
                                                float b) {
  float a[kEc];
#pragma unroll
  for (int e = 0; e < kEc; ++e) a[e] = act_t<EPI>(v[e] + b);
  const bool odd = lane & 1;
#pragma unroll
  for (int x = 0; x < kEc / 2; ++x) {
    const float send = odd ? a[x] : a[kEc / 2 + x];
    const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
    const float lo = odd ? recv : a[x];
    const float hi = odd ? a[kEc / 2 + x] : recv;
    const int tok = odd ? kEc / 2 + x : x;
    *reinterpret_cast<__nv_bfloat162 *>(pair_base + tok * ldy) = __floats2bfloat162_rn(lo, hi);
  }
}
__device__ __forceinline__ void store_pair_act(int epi, __nv_bfloat16 *pair_base, int64_t ldy, int lane,
                                               const float (&v)[kEc], float b) {
  switch (epi) {
    case kEpiSilu: store_pair_bf16<kEpiSilu>(pair_base, ldy, lane, v, b); break;
    case kEpiGeluErf: store_pair_bf16<kEpiGeluErf>(pair_base, ldy, lane, v, b); break;
    case kEpiRelu: store_pair_bf16<kEpiRelu>(pair_base, ldy, lane, v, b); break;
    default: store_pair_bf16<kEpiNone>(pair_base, ldy, lane, v, b); break;
  }
}

// kEc consecutive tokens of one output feature, contiguous in y (a row of a
// channel-major output): act(v + b), as 16-byte stores when `vec` (the run
// starts 16-byte aligned) and all kEc tokens are valid, else per element.
template <typename T, int EPI>
__device__ __forceinline__ void store_run(T *base, int valid, bool vec, const float (&v)[kEc], float b) {
  float a[kEc];
#pragma unroll
  for (int e = 0; e < kEc; ++e) a[e] = act_t<EPI>(v[e] + b);
  if (vec && valid >= kEc) {
    if constexpr (sizeof(T) == 4) {
#pragma unroll
      for (int e = 0; e < kEc; e += 4)
        *reinterpret_cast<float4 *>(reinterpret_cast<float *>(base) + e) = make_float4(a[e], a[e + 1], a[e + 2], a[e + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < kEc; e += 8)
        *reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(base) + e) =
            make_uint4(pack_bf16x2(a[e], a[e + 1]), pack_bf16x2(a[e + 2], a[e + 3]), pack_bf16x2(a[e + 4], a[e + 5]),
                       pack_bf16x2(a[e + 6], a[e + 7]));
    }
  } else {
#pragma unroll
    for (int e = 0; e < kEc; ++e)
      if (e < valid) put<T>(base + e, a[e]);
  }
}
__device__ __forceinline__ void store_run_act(int epi, int y_dtype, void *y, int64_t off, int valid, bool vec,
                                              const float (&v)[kEc], float b) {
  float *yf = static_cast<float *>(y) + off;
  __nv_bfloat16 *yb = static_cast<__nv_bfloat16 *>(y) + off;
  switch (epi * 2 + y_dtype) {
    case kEpiNone * 2 + 0: store_run<float, kEpiNone>(yf, valid, vec, v, b); break;
    case kEpiNone * 2 + 1: store_run<__nv_bfloat16, kEpiNone>(yb, valid, vec, v, b); break;
    case kEpiSilu * 2 + 0: store_run<float, kEpiSilu>(yf, valid, vec, v, b); break;
    case kEpiSilu * 2 + 1: store_run<__nv_bfloat16, kEpiSilu>(yb, valid, vec, v, b); break;
    case kEpiGeluErf * 2 + 0: store_run<float, kEpiGeluErf>(yf, valid, vec, v, b); break;
    case kEpiGeluErf * 2 + 1: store_run<__nv_bfloat16, kEpiGeluErf>(yb, valid, vec, v, b); break;
    case kEpiRelu * 2 + 0: store_run<float, kEpiRelu>(yf, valid, vec, v, b); break;
    default: store_run<__nv_bfloat16, kEpiRelu>(yb, valid, vec, v, b); break;
  }
}

// Channel-major output through lane quads.  A lane holds 64 contiguous bytes
// of its own output row as four 16-byte segments (act(v + b) of kEc f32
// tokens, or of 2 kEc bf16 tokens from two chunks); quad_transpose leaves lane
// 4g + s with segment s of rows 4g .. 4g + 3, so that store j of the warp
// writes 64 contiguous bytes of each of 8 rows (rows 4g + j) instead of 16
// bytes of each of 32 rows: a quarter of the cache lines per store.
template <int EPI>
__device__ __forceinline__ void act_segs_t(int y_dtype, const float (&v)[kEc], float b, uint4 &s0, uint4 &s1,
                                           uint4 &s2, uint4 &s3) {
  float a[kEc];
#pragma unroll
  for (int e = 0; e < kEc; ++e) a[e] = act_t<EPI>(v[e] + b);
  if (y_dtype == 0) {
    s0 = make_uint4(__float_as_uint(a[0]), __float_as_uint(a[1]), __float_as_uint(a[2]), __float_as_uint(a[3]));
    s1 = make_uint4(__float_as_uint(a[4]), __float_as_uint(a[5]), __float_as_uint(a[6]), __float_as_uint(a[7]));
    s2 = make_uint4(__float_as_uint(a[8]), __float_as_uint(a[9]), __float_as_uint(a[10]), __float_as_uint(a[11]));
    s3 = make_uint4(__float_as_uint(a[12]), __float_as_uint(a[13]), __float_as_uint(a[14]), __float_as_uint(a[15]));
  } else {  // two segments; s2, s3 untouched
    s0 = make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]), pack_bf16x2(a[4], a[5]), pack_bf16x2(a[6], a[7]));
    s1 = make_uint4(pack_bf16x2(a[8], a[9]), pack_bf16x2(a[10], a[11]), pack_bf16x2(a[12], a[13]),
                    pack_bf16x2(a[14], a[15]));
  }
}
__device__ __forceinline__ void act_segs(int epi, int y_dtype, const float (&v)[kEc], float b, uint4 &s0, uint4 &s1,
                                         uint4 &s2, uint4 &s3) {
  switch (epi) {
    case kEpiSilu: act_segs_t<kEpiSilu>(y_dtype, v, b, s0, s1, s2, s3); break;
    case kEpiGeluErf: act_segs_t<kEpiGeluErf>(y_dtype, v, b, s0, s1, s2, s3); break;
    case kEpiRelu: act_segs_t<kEpiRelu>(y_dtype, v, b, s0, s1, s2, s3); break;
    default: act_segs_t<kEpiNone>(y_dtype, v, b, s0, s1, s2, s3); break;
  }
}
__device__ __forceinline__ uint4 shfl_xor_u4(uint4 v, int d) {
  return make_uint4(__shfl_xor_sync(0xffffffffu, v.x, d), __shfl_xor_sync(0xffffffffu, v.y, d),
                    __shfl_xor_sync(0xffffffffu, v.z, d), __shfl_xor_sync(0xffffffffu, v.w, d));
}
// Lane s of each quad holds row s's segments a[0..3]; afterwards a[j] is
// segment s of row j of the quad.
__device__ __forceinline__ void quad_transpose(uint4 (&a)[4], int lane) {
  const bool b1 = (lane & 2) != 0;
  uint4 r0 = shfl_xor_u4(b1 ? a[0] : a[2], 2);
  uint4 r1 = shfl_xor_u4(b1 ? a[1] : a[3], 2);
  if (b1) {
    a[0] = r0;
    a[1] = r1;
  } else {
    a[2] = r0;
    a[3] = r1;
  }
  const bool b0 = (lane & 1) != 0;
  r0 = shfl_xor_u4(b0 ? a[0] : a[1], 1);
  r1 = shfl_xor_u4(b0 ? a[2] : a[3], 1);
  if (b0) {
    a[0] = r0;
    a[2] = r1;
  } else {
    a[1] = r0;
    a[3] = r1;
  }
}

__device__ __forceinline__ void store_glu_act(int epi, int y_dtype, void *y, int64_t off, int64_t ldy, int valid,
                                              const float (&v)[kEc], float b, const float (&g)[kEc]) {
  float *yf = static_cast<float *>(y) + off;
  __nv_bfloat16 *yb = static_cast<__nv_bfloat16 *>(y) + off;
  if (epi == kEpiGluSigmoid) {
    if (y_dtype == 0) store_glu<float, kEpiGluSigmoid>(yf, ldy, valid, v, b, g);
    else store_glu<__nv_bfloat16, kEpiGluSigmoid>(yb, ldy, valid, v, b, g);
  } else {
    if (y_dtype == 0) store_glu<float, kEpiGluSilu>(yf, ldy, valid, v, b, g);
    else store_glu<__nv_bfloat16, kEpiGluSilu>(yb, ldy, valid, v, b, g);
  }
}

}  // namespace nq
