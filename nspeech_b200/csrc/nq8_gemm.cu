// nq8_gemm.cu -- K1: persistent 2-SM tcgen05/TMEM Q8_0 GEMM for M > 16 (sm_100a).
//
// Replaces the tiled matmul family of the reference (Triton source
// kernels/moonshine_kernels.py:20-299, dispatched by triton_matmul*/enc_matmul*
// in src/triton_kernels.rs:170-309,1205-1289; CPU FbgemmBf16Op in
// src/fast_matmul.rs:138-167).
//
// Y[tok, n] = act(X[tok, :] . bf16(dequant(W[n, :])) + bias[n]).  Serves
// calls below ~128 tokens, where the weight bytes dominate (larger calls
// dequantize once and run K3, nq8_gemm_bf16.cu).  A cluster of two CTAs (an
// SM pair) computes transposed tiles D[256 weight rows x 192 tokens] with
// tcgen05.mma.cta_group::2: each CTA owns 128 weight rows (its TMEM lanes)
// and stages half of the token tile (96 rows).  The weights are operand A *in
// tensor memory*: dequantized in registers and written with tcgen05.st.  The
// pair walks a static list of work units (weight-row pair tile, token tile,
// k split); TMEM holds two accumulators, so the epilogue of unit j overlaps
// the main loop of unit j+1.  Per CTA:
//   warp 0      producer: per 64-wide k step, a bulk copy of its packed
//               weight tile (8.7 KB) into shared stage s (completes on its
//               own full_w[s]) and a TMA 2-D load of its 96 token rows (bf16,
//               128-byte swizzle; completes on the leader's full_b[s]).
//   warp 1      allocates 512 TMEM columns for the pair (D0, D1: 192 columns
//               each; 4 A stages of 32); in the leader, lane 0 issues
//               tcgen05.mma (M=256, N=192, K=16, kind::f16, A from TMEM) and
//               commits to empty_a / empty_b / accum_full of both CTAs
//               (multicast commit; no multicast loads anywhere).
//   warps 2-5   epilogue: tcgen05.ld (one weight row per lane, 16 tokens at a
//               time), bias + activation (GLU through shared memory), stores
//               contiguous along the output row across the warp, then arrive
//               on the leader's accum_empty; split-K writes raw partials for
//               splitk_reduce.
//   warps 6-21  dequant: the four warps of a TMEM lane quarter take turns by
//               k step (warp `sub` fills A stage `sub`): read the weight
//               chunk from shared memory, bf16(f32(d)*q) with packed f32x2
//               arithmetic, tcgen05.st 32x32b.x32, arrive on the leader's
//               full_a.
// f32 activations arrive as two bf16 planes (hi, lo): two MMAs per k step.
// Every mbarrier wait is bounded; on give-up the kernel records a status bit,
// drains, frees TMEM and returns.
#include "nq8_common.cuh"
#include "nq8_kernels.h"
#include "nq8_sm100_pair.cuh"

namespace nq {

constexpr int kBT = 192;       // tokens per pair unit (MMA N)
constexpr int kBTHalf = 96;    // token rows staged per CTA
constexpr int kAStages = 4;    // dequantized weight stages in TMEM
constexpr int kEpiWarps = 4;
constexpr int kConvWarps = 16;  // 4 per TMEM lane quarter, taking turns by k step
constexpr int kGemmThreads = 32 * (2 + kEpiWarps + kConvWarps);  // 704
constexpr int kEpiWarp0 = 2;
constexpr int kConvWarp0 = kEpiWarp0 + kEpiWarps;

template <bool SPLITX>
struct GemmCfg {
  // Shared-memory stages: this CTA's activation rows (TMA, 128-byte swizzle)
  // and its packed weight tile (bulk copy), deep enough to cover L2 latency.
  static constexpr int kStages = SPLITX ? 5 : 8;
  static constexpr int kBBytes = kBTHalf * kPackK * 2;  // 12 KB per activation plane per CTA
  static constexpr int kStageBytes = kBBytes * (SPLITX ? 2 : 1);
  static constexpr int kWOffset = kStages * kStageBytes;
  static constexpr int kGluOffset = kWOffset + kStages * kTileBytes;
  static constexpr int kGluBytes = 64 * kEc * 4;
  static constexpr int kBarOffset = kGluOffset + kGluBytes;
  static constexpr int kNumBars = 4 * kStages + 2 * kAStages + 4;
  static constexpr int kSmemBytes = 1024 /*align slack*/ + kBarOffset + kNumBars * 8 + 64;
  static constexpr uint32_t kIdesc = idesc_bf16_f32(256, kBT);
  static constexpr int kACol = 2 * kBT;  // D0 [0,192), D1 [192,384), A stages [384, 512)
  static constexpr int kTmemCols = 512;
  static_assert(kStageBytes % 1024 == 0, "swizzled stages must stay 1024-byte aligned");
  static_assert(kTileBytes % 16 == 0 && kGluOffset % 16 == 0, "bulk copies need 16-byte alignment");
  static_assert(kACol + kAStages * 32 <= kTmemCols, "TMEM budget");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// ---------------------------------------------------------------- dequant
struct WChunk64 {
  uint4 q[4];           // the 64 int8 of one row in a 64-wide k step
  unsigned short d[2];  // the row's two Q8_0 block scales (f16)
};

// Row `row` of a packed tile staged in shared memory: four 16-byte loads
// (consecutive rows in consecutive lanes: conflict-free) and the two scales.
__device__ __forceinline__ WChunk64 load_wchunk64(const uint8_t *tile, int row) {
  WChunk64 w;
#pragma unroll
  for (int c = 0; c < 4; ++c) w.q[c] = *reinterpret_cast<const uint4 *>(tile + qs_offset(row, c));
  w.d[0] = *reinterpret_cast<const unsigned short *>(tile + scale_offset(row, 0));
  w.d[1] = *reinterpret_cast<const unsigned short *>(tile + scale_offset(row, 1));
  return w;
}

// 64 elements -> 32 packed bf16x2 words in TMEM column order (k pairs).
__device__ __forceinline__ void dequant64(const WChunk64 &w, uint32_t (&r)[32]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float d = __half2float(__ushort_as_half(w.d[h]));
    const uint64_t dd = f2(d, d);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint4 v = w.q[2 * h + j];
      dequant8_bf16(v.x, v.y, dd, r + 16 * h + 8 * j);
      dequant8_bf16(v.z, v.w, dd, r + 16 * h + 8 * j + 4);
    }
  }
}

// ------------------------------------------------------------- work units
struct Unit {
  int ft, tt, split, kc0, nk;  // ft: weight-row pair tile (two 128-row packed tiles)
};
__device__ __forceinline__ Unit decode_unit(const GemmParams &p, int u) {
  Unit r;
  const int per_split = p.grid_n * p.grid_m;
  r.split = u / per_split;
  const int rem = u - r.split * per_split;
  r.tt = rem / p.grid_n;
  r.ft = rem - r.tt * p.grid_n;
  r.kc0 = r.split * p.cps;
  r.nk = max(min(r.kc0 + p.cps, p.kc_total) - r.kc0, 0);
  return r;
}

template <bool SPLITX>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_q8_sm100_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_alo,
                         const __grid_constant__ GemmParams p) {
  using C = GemmCfg<SPLITX>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: leader (issues the pair MMA), 1: peer
  const int cl = blockIdx.x >> 1;
  const int ncl = gridDim.x >> 1;
  const int n_units = p.grid_n * p.grid_m * p.splits;

  constexpr int kStages = C::kStages;
  auto stage_b = [&](int s) { return smem + s * C::kStageBytes; };
  auto stage_blo = [&](int s) { return smem + s * C::kStageBytes + C::kBBytes; };
  auto stage_w = [&](int s) { return smem + C::kWOffset + s * kTileBytes; };
  float *glu_s = reinterpret_cast<float *>(smem + C::kGluOffset);  // [kEc][64]
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOffset);
  // Shared-memory stages (kStages): activations and weights.
  auto full_b = [&](int s) { return smem_u32(&bars[s]); };                 // leader: both halves landed
  auto empty_b = [&](int s) { return smem_u32(&bars[kStages + s]); };      // pair MMA read the stage
  auto full_w = [&](int s) { return smem_u32(&bars[2 * kStages + s]); };   // weight tile landed
  auto empty_w = [&](int s) { return smem_u32(&bars[3 * kStages + s]); };  // converters read it
  // TMEM weight stages (kAStages).
  auto full_a = [&](int a) { return smem_u32(&bars[4 * kStages + a]); };             // leader: 8 warps stored
  auto empty_a = [&](int a) { return smem_u32(&bars[4 * kStages + kAStages + a]); };  // pair MMA read it
  auto accum_full = [&](int b) { return smem_u32(&bars[4 * kStages + 2 * kAStages + b]); };
  auto accum_empty = [&](int b) { return smem_u32(&bars[4 * kStages + 2 * kAStages + 2 + b]); };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(&bars[C::kNumBars]);
  // [0] abort (any role)  [2] epilogue gave up
  volatile int *flags = reinterpret_cast<volatile int *>(tmem_slot + 2);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_b(s), 1);   // leader producer's expect_tx (+ both halves' bytes)
      mbar_init(empty_b(s), 1);  // multicast commit
      mbar_init(full_w(s), 1);   // this CTA's producer (+ tile bytes)
      mbar_init(empty_w(s), 4);  // one converter warp per lane quarter
    }
    for (int a = 0; a < kAStages; ++a) {
      mbar_init(full_a(a), 8);   // one converter warp per lane quarter in each CTA
      mbar_init(empty_a(a), 1);  // multicast commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accum_full(b), 1);  // multicast commit
      mbar_init(accum_empty(b), 2 * kEpiWarps);
    }
    flags[0] = 0;
    flags[1] = 0;
    flags[2] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc2(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // both CTAs' barriers exist before anyone signals across the pair
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // barriers and TMEM are set up; now wait for the predecessor's data
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      prefetch_tmap(&tm_a);
      if (SPLITX) prefetch_tmap(&tm_alo);
      const uint64_t w_policy = policy_evict_last();  // weights are re-read by every token tile
      int g = 0;
      bool ok = true;
      for (int u = cl; u < n_units && ok; u += ncl) {
        const Unit un = decode_unit(p, u);
        const int row0 = un.tt * kBT + static_cast<int>(rank) * kBTHalf;
        const int tile = 2 * un.ft + static_cast<int>(rank);
        const uint8_t *wsrc = p.w + (static_cast<size_t>(tile) * p.kc_total + un.kc0) * kTileBytes;
        for (int i = 0; i < un.nk; ++i, ++g) {
          const int s = g % kStages;
          if (g >= kStages) {
            const uint32_t par = ((g / kStages) - 1) & 1;
            if (!mbar_wait(empty_b(s), par, p.ctl.wait_limit, flags) ||
                !mbar_wait(empty_w(s), par, p.ctl.wait_limit, flags)) {
              if (!flags[0]) report(p.ctl, flags, kDevTimeoutProducer);
              ok = false;
              break;
            }
          }
          if (flags[0]) {
            ok = false;
            break;
          }
          // The converters read weight stages with ordinary shared loads: order
          // those reads before the async-proxy copies that refill the stage.
          fence_proxy_async_smem();
          if (tile < p.n_tiles) {
            mbar_arrive_expect_tx(full_w(s), kTileBytes);
            bulk_load(smem_u32(stage_w(s)), wsrc + static_cast<size_t>(i) * kTileBytes, kTileBytes, full_w(s),
                      w_policy);
          } else {
            mbar_arrive(full_w(s));  // the pair's second tile lies beyond N: converters use zeros
          }
          if (rank == 0) mbar_arrive_expect_tx(full_b(s), 2 * C::kStageBytes);
          const uint32_t bar = map_rank(full_b(s), 0);
          tma_load_2d_pair(smem_u32(stage_b(s)), &tm_a, bar, (un.kc0 + i) * kPackK, row0);
          if (SPLITX) tma_load_2d_pair(smem_u32(stage_blo(s)), &tm_alo, bar, (un.kc0 + i) * kPackK, row0);
        }
      }
      // Drain: every copy issued into this CTA's shared memory has landed
      // (weights: full_w; activations: the leader's full_b, or the commit of
      // the MMA that read them).
      volatile int no_abort = 0;
      for (int s = 0; s < kStages && s < g; ++s) {
        const int last = s + kStages * ((g - 1 - s) / kStages);
        const uint32_t par = (last / kStages) & 1;
        bool done = mbar_wait(full_w(s), par, p.ctl.wait_limit, &no_abort);
        done = (rank == 0 ? mbar_wait(full_b(s), par, p.ctl.wait_limit, &no_abort)
                          : mbar_wait(empty_b(s), par, p.ctl.wait_limit, &no_abort)) && done;
        if (!done) atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ------------------------------------------------------- MMA (leader)
      int g = 0, j = 0;
      bool ok = true;
      for (int u = cl; u < n_units && ok; u += ncl, ++j) {
        const Unit un = decode_unit(p, u);
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(accum_empty(b), ((j >> 1) - 1) & 1, p.ctl.wait_limit, flags)) {
          if (!flags[0]) report(p.ctl, flags, kDevTimeoutMma);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * kBT;
        for (int i = 0; i < un.nk; ++i, ++g) {
          const int s = g % kStages;
          const int a = g % kAStages;
          if (!mbar_wait(full_a(a), (g / kAStages) & 1, p.ctl.wait_limit, flags) ||
              !mbar_wait(full_b(s), (g / kStages) & 1, p.ctl.wait_limit, flags)) {
            if (!flags[0]) report(p.ctl, flags, kDevTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_addr = smem_u32(stage_b(s));
          const uint32_t blo_addr = smem_u32(stage_blo(s));
          const uint32_t a_tmem = tmem_base + C::kACol + a * 32;
#pragma unroll
          for (int kk = 0; kk < kPackK / 16; ++kk) {
            umma2_bf16_ts(d_tmem, a_tmem + kk * 8, sw128_kmajor_desc(b_addr + kk * 32), C::kIdesc,
                          (i > 0 || kk > 0) ? 1u : 0u);
            if (SPLITX) umma2_bf16_ts(d_tmem, a_tmem + kk * 8, sw128_kmajor_desc(blo_addr + kk * 32), C::kIdesc, 1u);
          }
          umma2_commit_both(empty_a(a));
          umma2_commit_both(empty_b(s));
        }
        if (!ok) break;
        umma2_commit_both(accum_full(b));
      }
      if (!ok && g > 0) {
        // Aborted: the MMAs already issued must finish before TMEM is freed.
        volatile int no_abort = 0;
        const int last = g - 1;
        if (!mbar_wait(empty_a(last % kAStages), (last / kAStages) & 1, p.ctl.wait_limit, &no_abort))
          atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else if (warp < kConvWarp0) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int frow = 32 * q + lane;  // weight row within this CTA's tile == TMEM lane
    const uint32_t tlane = static_cast<uint32_t>(32 * q) << 16;
    int j = 0;
    for (int u = cl; u < n_units; u += ncl, ++j) {
      const Unit un = decode_unit(p, u);
      const int b = j & 1;
      const int tile = 2 * un.ft + static_cast<int>(rank);  // this CTA's 128-row packed tile
      bool ok = mbar_wait(accum_full(b), (j >> 1) & 1, p.ctl.wait_limit, flags);
      ok = __all_sync(0xffffffffu, ok);
      // The four epilogue warps share named barriers below, so they agree on
      // giving up before any of them leaves the loop.
      if (!ok && lane == 0) {
        flags[2] = 1;
        if (!flags[0]) report(p.ctl, flags, kDevTimeoutEpilogue);
      }
      named_bar_sync(1, 32 * kEpiWarps);
      const bool give_up = flags[2] != 0;
      named_bar_sync(1, 32 * kEpiWarps);
      if (give_up) break;
      tc_fence_after();
      const uint32_t trow = tmem_base + tlane + b * kBT;
      const int m0 = un.tt * kBT;
      // Token chunks past M hold padding: skip them (uniform across the
      // epilogue warps, which matters for the GLU named barriers).
      const int cols = min(kBT, ((p.M - m0 + kEc - 1) / kEc) * kEc);
      auto release_d = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) mbar_arrive(accum_empty(b));
          else mbar_arrive_remote(map_rank(accum_empty(b), 0));
        }
      };
      auto fetch = [&](int col, float (&v)[kEc]) {
        uint32_t r[kEc];
        __syncwarp();  // tcgen05.ld is warp-collective: reconverge first
        tmem_ld16(trow + col, r);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < kEc; ++e) v[e] = __uint_as_float(r[e]);
      };
      if (p.splits > 1) {
        // Raw partial sums, token-major [split][M][ldp]: per token the warp
        // writes 32 consecutive floats.  splitk_reduce sums them in order.
        const int64_t n = static_cast<int64_t>(tile) * kPackRows + frow;
        const bool nvalid = tile < p.n_tiles;
        float *part = p.partials + (static_cast<size_t>(un.split) * p.M + m0) * p.ldp + n;
        for (int col = 0; col < cols; col += kEc) {
          float v[kEc];
          fetch(col, v);
          const int valid = p.M - (m0 + col);
          if (!nvalid) continue;
#pragma unroll
          for (int e = 0; e < kEc; ++e)
            if (e < valid) part[static_cast<size_t>(col + e) * p.ldp] = v[e];
        }
        release_d();
        continue;
      }
      if (!p.glu) {
        const int64_t n = static_cast<int64_t>(tile) * kPackRows + frow;
        const bool nvalid = n < p.N;
        const float bn = (p.bias && nvalid) ? p.bias[n] : 0.f;
        for (int col = 0; col < cols; col += kEc) {
          float v[kEc];
          fetch(col, v);
          const int valid = p.M - (m0 + col);
          if (!nvalid) continue;
          const int64_t off = static_cast<int64_t>(m0 + col) * p.ldy + n;
          store_act(p.epi, p.y_dtype, p.y, off, p.ldy, valid, v, bn);
        }
      } else {
        // GLU tile: lanes [0, 64) value rows, [64, 128) their gate rows.  The
        // gate warps pass biased gates through shared memory ([token][row]:
        // conflict-free for both sides).
        const bool is_gate = frow >= 64;
        const int vrow = frow & 63;
        const int64_t jcol = static_cast<int64_t>(tile) * 64 + vrow;
        const bool jvalid = jcol < p.n_out;
        const float bv = (p.bias && jvalid) ? p.bias[is_gate ? p.n_out + jcol : jcol] : 0.f;
        for (int col = 0; col < cols; col += kEc) {
          float v[kEc];
          fetch(col, v);
          if (is_gate) {
#pragma unroll
            for (int e = 0; e < kEc; ++e) glu_s[e * 64 + vrow] = v[e] + bv;
          }
          named_bar_sync(1, 32 * kEpiWarps);
          const int valid = p.M - (m0 + col);
          if (!is_gate && jvalid) {
            float g[kEc];
#pragma unroll
            for (int e = 0; e < kEc; ++e) g[e] = glu_s[e * 64 + vrow];
            const int64_t off = static_cast<int64_t>(m0 + col) * p.ldy + jcol;
            store_glu_act(p.epi, p.y_dtype, p.y, off, p.ldy, valid, v, bv, g);
          }
          named_bar_sync(1, 32 * kEpiWarps);
        }
      }
      release_d();
    }
  } else {
    // ------------------------------------------------------------- dequant
    // Warp w: TMEM lane quarter q = w % 4 (weight rows 32q..32q+31 of this
    // CTA's tile); the four warps of a quarter take turns by k step: warp
    // `sub` dequantizes whole 64-wide steps g = sub (mod 4) into TMEM stage
    // `sub`, reading the weight tile from shared-memory stage g % kStages.
    static_assert(kAStages == kConvWarps / 4, "one TMEM stage per converter warp of a lane quarter");
    const int q = warp & 3;
    const int sub = (warp - kConvWarp0) >> 2;
    const int row = 32 * q + lane;
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + C::kACol + sub * 32;
    const uint32_t full_a_leader = map_rank(full_a(sub), 0);
    int G = 0;  // k steps of this CTA
    for (int u = cl; u < n_units; u += ncl) G += decode_unit(p, u).nk;
    int cu = cl, ci = 0;  // (unit, step) cursor of step g
    Unit cun = decode_unit(p, cu < n_units ? cu : 0);
    auto cursor_next = [&]() {
      if (++ci >= cun.nk) {
        ci = 0;
        cu += ncl;
        if (cu < n_units) cun = decode_unit(p, cu);
      }
    };
    for (int t = 0; t < sub && t < G; ++t) cursor_next();
    for (int g = sub; g < G; g += 4) {
      const int s = g % kStages;
      const bool tile_valid = 2 * cun.ft + static_cast<int>(rank) < p.n_tiles;
#pragma unroll 1
      for (int t = 0; t < 4; ++t) cursor_next();
      bool ok = mbar_wait(full_w(s), (g / kStages) & 1, p.ctl.wait_limit, flags);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0 && !flags[0]) report(p.ctl, flags, kDevTimeoutConsumer);
        break;
      }
      // A tile beyond N (the pair's second tile) arrives as a bare arrival:
      // its stage holds stale bytes, so zero scales are used instead.
      WChunk64 w = load_wchunk64(stage_w(s), row);
      if (!tile_valid) w.d[0] = w.d[1] = 0;
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_w(s));
      uint32_t r[32];
      dequant64(w, r);
      if (g >= kAStages) {
        ok = mbar_wait(empty_a(sub), ((g / kAStages) - 1) & 1, p.ctl.wait_limit, flags);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) {
          if (lane == 0 && !flags[0]) report(p.ctl, flags, kDevTimeoutConsumer);
          break;
        }
      }
      tc_fence_after();
      tmem_st32(taddr, r);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(full_a(sub));
        else mbar_arrive_remote(full_a_leader);
      }
    }
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // nobody leaves while the pair may still signal it
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc2(tmem_base, C::kTmemCols);
  }
}

int gemm_block_t(GemmVariant) { return kBT; }

size_t gemm_smem_bytes(GemmVariant v) {
  return v == kGemmBt128SplitX ? GemmCfg<true>::kSmemBytes : GemmCfg<false>::kSmemBytes;
}

template <bool SPLITX>
static cudaError_t launch_gemm_t(const CUtensorMap &a_hi, const CUtensorMap &a_lo, const GemmParams &p, int pairs,
                                 cudaStream_t stream) {
  using C = GemmCfg<SPLITX>;
  auto kern = gemm_q8_sm100_kernel<SPLITX>;
  static bool attr_set[64] = {false};  // once per device (the attribute is per-context state)
  static int max_pairs[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return e;
    int n = 0;
    cfg.gridDim = dim3(2 * 74);
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess) return e;
    if (n <= 0) return cudaErrorInvalidConfiguration;
    if (dev < 64) {
      attr_set[dev] = true;
      max_pairs[dev] = n;
    }
  }
  const int cap = dev < 64 ? max_pairs[dev] : 1;
  return launch_pdl(kern, dim3(2 * (pairs < cap ? pairs : cap)), dim3(kGemmThreads), C::kSmemBytes, stream, 2, a_hi,
                    a_lo, p);
}

cudaError_t launch_gemm(GemmVariant v, const CUtensorMap &a_hi, const CUtensorMap &a_lo, const GemmParams &p, int grid,
                        cudaStream_t stream) {
  return v == kGemmBt128SplitX ? launch_gemm_t<true>(a_hi, a_lo, p, grid, stream)
                               : launch_gemm_t<false>(a_hi, a_lo, p, grid, stream);
}

}  // namespace nq
