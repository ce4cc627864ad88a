// nq8_gemm_bf16.cu -- K3: persistent 2-SM tcgen05 bf16 x bf16 GEMM over a
// dequantized copy of a Q8_0 weight (sm_100a), for large token counts.
//
// Same contract as K1 (nq8_gemm.cu) and the reference's tiled matmul family
// (kernels/moonshine_kernels.py:20-299 via src/triton_kernels.rs:170-309,
// 1205-1289); the weight operand is bf16(f32(d) * q) computed once per call by
// dequant_tiles (nq8_aux.cu) -- the values the reference's FbgemmBf16Op
// multiplies (src/fast_matmul.rs:127-167, weights pre-dequantized to bf16).
// Dequantizing once instead of once per token tile is what makes the
// contraction tensor-bound rather than issue-bound when M is large.
//
// A cluster of two CTAs computes D[256 weight rows x 256 tokens] per work unit
// with tcgen05.mma.cta_group::2 (M=256, N=256, K=16, both operands in shared
// memory, 128-byte swizzle): CTA r holds weight rows 128r.. and token rows
// 128r.. of the unit.  TMEM holds two 256-column accumulators per CTA, so the
// epilogue of unit j overlaps the main loop of unit j+1.  Per CTA:
//   warp 0      producer: TMA 2-D loads of its weight rows [128 x 64 k] and
//               token rows [128 x 64 k] (hi and lo planes for f32 inputs)
//               into stage s; the bytes complete on the leader's full[s].
//   warp 1      allocates the pair's 512 TMEM columns; the leader's lane 0
//               issues the MMAs and commits to empty[s] / accum_full[b] of
//               both CTAs (multicast commit; no multicast loads anywhere).
//   warps 2-17  epilogue: warp w reads TMEM lane quarter w % 4 and a 64-token
//               column group; bias + activation (GLU through shared memory
//               between the value and gate warps of a column group); split-K
//               partials are raw f32 sums for splitk_reduce.
// Tail split: when the tiles leave the last round of pairs partly idle, the
// tiles of that round are cut into k pieces run by different pairs.  A piece
// stores its raw accumulator (L2-resident scratch) and bumps a counter per
// (tile, CTA, epilogue warp); the warp that arrives last sums the pieces in
// piece order and applies the epilogue.  Nothing waits for another CTA, so a
// grid that is only partly resident (another stream's kernels hold SMs)
// cannot deadlock, and the sums do not depend on arrival order.
// Every mbarrier wait is bounded; on give-up the kernel records a status bit,
// drains, frees TMEM and returns.
#include "nq8_common.cuh"
#include "nq8_kernels.h"
#include "nq8_sm100_pair.cuh"

namespace nq {
namespace {

constexpr int kPTDefault = 256;  // tokens per pair unit (MMA N) unless set otherwise
constexpr int kPW = 256;         // weight rows per pair unit (MMA M)
constexpr int kEpiW = 16;        // epilogue warps: 4 column groups x 4 lane quarters
constexpr int kThreads = 32 * (2 + kEpiW);  // 576
constexpr int kEpi0 = 2;
constexpr int kAgreeBar = 9;     // named barrier of all epilogue warps (1..8: GLU pairs)

// PT: tokens per pair unit: one MMA of N = PT per k slice (PT / 2 token rows
// per CTA), with two TMEM accumulators so the epilogue of one unit overlaps
// the next unit's main loop.  256 is the default; 128 and 64 give small-M
// calls more units.
template <bool SPLITX, int PT>
struct Cfg {
  static_assert(PT == 64 || PT == 128 || PT == 256, "unit widths 64, 128, 256");
  static constexpr int kPT = PT;
  static constexpr int kNB = 1;                      // MMAs (token sub-tiles) per k slice
  static constexpr int kMmaN = PT;                   // N of each MMA
  static constexpr int kSubRows = kMmaN / 2;         // token rows per CTA and sub-tile
  static constexpr int kAccBufs = 2;                 // TMEM accumulator buffers
  static constexpr int kColsPerWarp = PT / 4;        // tokens per epilogue warp (4 column groups)
  static_assert(kColsPerWarp % kEc == 0, "epilogue chunks");
  static constexpr int kStages = SPLITX ? (PT == 256 ? 4 : 6) : (PT == 256 ? 6 : 8);
  static constexpr int kABytes = 128 * kPackK * 2;          // 16 KB of weight rows
  static constexpr int kSubBytes = kSubRows * kPackK * 2;   // one token sub-tile of one plane
  static constexpr int kBBytes = kNB * kSubBytes;           // 4 / 8 / 16 KB per activation plane
  static constexpr int kStageBytes = kABytes + kBBytes * (SPLITX ? 2 : 1);
  static constexpr int kGluOffset = kStages * kStageBytes;
  static constexpr int kGluBytes = 8 * kEc * 32 * 4;    // 8 value/gate warp pairs
  static constexpr int kBarOffset = kGluOffset + kGluBytes;
  static constexpr int kNumBars = 2 * kStages + 4;
  static constexpr int kSmemBytes = 1024 /*align slack*/ + kBarOffset + kNumBars * 8 + 64;
  static constexpr uint32_t kIdesc = idesc_bf16_f32(kPW, kMmaN);
  static constexpr int kTmemCols = kAccBufs * PT;  // D0 [0, PT), D1 [PT, 2 PT)
  static_assert(kStageBytes % 1024 == 0 && kABytes % 1024 == 0 && kSubBytes % 1024 == 0, "swizzle alignment");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

struct Unit {
  int ft, tt, split, kc0, nk;
  int tail;    // tail tile index (tiles past full_units), or -1
  int piece;   // k piece of a tail tile
};
__device__ __forceinline__ int num_units(const GemmBf16Params &p) {
  const int tiles = p.grid_n * p.grid_m;
  return p.tail_pieces > 1 ? p.full_units + (tiles - p.full_units) * p.tail_pieces : tiles * p.splits;
}
__device__ __forceinline__ Unit decode_unit(const GemmBf16Params &p, int u) {
  Unit r;
  int tile;
  r.tail = -1;
  r.piece = 0;
  if (p.tail_pieces > 1 && u >= p.full_units) {
    const int w = u - p.full_units;
    r.tail = w / p.tail_pieces;
    r.piece = w - r.tail * p.tail_pieces;
    tile = p.full_units + r.tail;
    r.split = 0;
    r.kc0 = r.piece * p.tail_cps;
    r.nk = max(min(r.kc0 + p.tail_cps, p.kc_total) - r.kc0, 0);
  } else {
    const int per_split = p.grid_n * p.grid_m;
    r.split = u / per_split;
    tile = u - r.split * per_split;
    r.kc0 = r.split * p.cps;
    r.nk = max(min(r.kc0 + p.cps, p.kc_total) - r.kc0, 0);
  }
  r.tt = tile / p.grid_n;
  r.ft = tile - r.tt * p.grid_n;
  return r;
}

// CONV: the implicit conv1d form (shifted token rows per tap, channel-major
// output); compiled separately so that the plain GEMM carries none of it.
template <bool SPLITX, int PT, bool CONV>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_sm100_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                           const __grid_constant__ CUtensorMap tm_alo, const __grid_constant__ GemmBf16Params p) {
  using C = Cfg<SPLITX, PT>;
  constexpr int kStages = C::kStages;
  constexpr int kPT = C::kPT, kColsPerWarp = C::kColsPerWarp, kNB = C::kNB, kMmaN = C::kMmaN;
  constexpr int kSubRows = C::kSubRows, kAccBufs = C::kAccBufs;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: leader (issues the pair MMA), 1: peer
  const int cl = blockIdx.x >> 1;
  const int ncl = gridDim.x >> 1;
  const int n_units = num_units(p);

  auto stage_w = [&](int s) { return smem + s * C::kStageBytes; };
  auto stage_b = [&](int s) { return smem + s * C::kStageBytes + C::kABytes; };
  auto stage_blo = [&](int s) { return smem + s * C::kStageBytes + C::kABytes + C::kBBytes; };
  float *glu_s = reinterpret_cast<float *>(smem + C::kGluOffset);  // [8 pairs][kEc][32]
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOffset);
  auto full = [&](int s) { return smem_u32(&bars[s]); };            // leader: both CTAs' bytes landed
  auto empty = [&](int s) { return smem_u32(&bars[kStages + s]); }; // pair MMA read the stage
  auto accum_full = [&](int b) { return smem_u32(&bars[2 * kStages + b]); };
  auto accum_empty = [&](int b) { return smem_u32(&bars[2 * kStages + 2 + b]); };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(&bars[C::kNumBars]);
  // [0] abort (any role)  [1] epilogue gave up
  volatile int *flags = reinterpret_cast<volatile int *>(tmem_slot + 2);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full(s), 1);   // leader producer's expect_tx (+ both CTAs' bytes)
      mbar_init(empty(s), 1);  // multicast commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accum_full(b), 1);  // multicast commit
      mbar_init(accum_empty(b), 2 * kEpiW);
    }
    flags[0] = 0;
    flags[1] = 0;
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
  // A weight that no preceding kernel writes (a kept bf16 copy) streams its
  // first ring stages before the dependency wait, during the previous
  // kernel's tail; the token halves of those stages follow after the wait.
  int pre = 0;
  if (CONV && warp == 0 && lane == 0) {  // descriptors are launch parameters: fetch them before the wait
    prefetch_tmap(&tm_a);
    if (SPLITX) prefetch_tmap(&tm_alo);
  }
  if (warp == 0 && lane == 0 && p.w_static) {
    prefetch_tmap(&tm_w);
    for (int u = cl; u < n_units && pre < kStages; u += ncl) {
      const Unit un = decode_unit(p, u);
      const int wrow0 = un.ft * kPW + static_cast<int>(rank) * 128;
      for (int i = 0; i < un.nk && pre < kStages; ++i, ++pre) {
        if (rank == 0) mbar_arrive_expect_tx(full(pre), 2 * C::kStageBytes);
        tma_load_2d_pair(smem_u32(stage_w(pre)), &tm_w, map_rank(full(pre), 0), (un.kc0 + i) * kPackK, wrow0);
      }
    }
  }
  pdl_wait();  // barriers and TMEM are set up; now wait for the predecessor's data
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      prefetch_tmap(&tm_w);
      prefetch_tmap(&tm_a);
      if (SPLITX) prefetch_tmap(&tm_alo);
      int g = 0;
      bool ok = true;
      for (int u = cl; u < n_units && ok; u += ncl) {
        const Unit un = decode_unit(p, u);
        const int wrow0 = un.ft * kPW + static_cast<int>(rank) * 128;
        const int trow0 = un.tt * kPT + static_cast<int>(rank) * kSubRows;
        for (int i = 0; i < un.nk; ++i, ++g) {
          const int s = g % kStages;
          if (g >= kStages && !mbar_wait(empty(s), ((g / kStages) - 1) & 1, p.ctl.wait_limit, flags)) {
            if (!flags[0]) report(p.ctl, flags, kDevTimeoutProducer);
            ok = false;
            break;
          }
          if (flags[0]) {
            ok = false;
            break;
          }
          const uint32_t bar = map_rank(full(s), 0);
          const int kx = (un.kc0 + i) * kPackK;
          int ax = kx, arow = trow0;  // token operand coordinates
          if (CONV) {
            const int c = un.kc0 + i;
            const int tap = c / p.conv_cpt;
            ax = (c - tap * p.conv_cpt) * kPackK;
            arow = trow0 + tap * p.conv_dil - p.conv_pad;
          }
          // Weight rows past the matrix (odd tile count) and token rows past M
          // (conv: outside the input) are zero-filled by the TMA unit.
          if (g >= pre) {  // else its expect_tx and weight load were issued before the wait
            if (rank == 0) mbar_arrive_expect_tx(full(s), 2 * C::kStageBytes);
            tma_load_2d_pair(smem_u32(stage_w(s)), &tm_w, bar, kx, wrow0);
          }
#pragma unroll
          for (int t = 0; t < kNB; ++t) {  // token sub-tile t: unit tokens [t kMmaN, (t + 1) kMmaN)
            tma_load_2d_pair(smem_u32(stage_b(s)) + t * C::kSubBytes, &tm_a, bar, ax, arow + t * kMmaN);
            if (SPLITX)
              tma_load_2d_pair(smem_u32(stage_blo(s)) + t * C::kSubBytes, &tm_alo, bar, ax, arow + t * kMmaN);
          }
        }
      }
      // Drain: every copy into this CTA's shared memory has landed (the
      // leader's full barrier, or the commit of the MMA that read it).  Stages
      // whose weight half went out before the dependency wait count too.
      volatile int no_abort = 0;
      const int issued = g > pre ? g : pre;
      for (int s = 0; s < kStages && s < issued; ++s) {
        const int last = s + kStages * ((issued - 1 - s) / kStages);
        const bool done = rank == 0 ? mbar_wait(full(s), (last / kStages) & 1, p.ctl.wait_limit, &no_abort)
                                    : mbar_wait(empty(s), (last / kStages) & 1, p.ctl.wait_limit, &no_abort);
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
        const int b = kAccBufs == 2 ? (j & 1) : 0;
        const int jb = kAccBufs == 2 ? (j >> 1) : j;  // use count of buffer b before this unit
        if (j >= kAccBufs && !mbar_wait(accum_empty(b), (jb - 1) & 1, p.ctl.wait_limit, flags)) {
          if (!flags[0]) report(p.ctl, flags, kDevTimeoutMma);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * kPT;
        for (int i = 0; i < un.nk; ++i, ++g) {
          const int s = g % kStages;
          if (!mbar_wait(full(s), (g / kStages) & 1, p.ctl.wait_limit, flags)) {
            if (!flags[0]) report(p.ctl, flags, kDevTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stage_w(s));
          const uint32_t b_addr = smem_u32(stage_b(s));
          const uint32_t blo_addr = smem_u32(stage_blo(s));
#pragma unroll
          for (int kk = 0; kk < kPackK / 16; ++kk) {
            const uint64_t ad = sw128_kmajor_desc(a_addr + kk * 32);
#pragma unroll
            for (int t = 0; t < kNB; ++t) {  // sub-tile t accumulates into columns [t kMmaN, (t + 1) kMmaN)
              const uint32_t dt = d_tmem + t * kMmaN;
              const uint32_t boff = t * C::kSubBytes + kk * 32;
              umma2_bf16_ss(dt, ad, sw128_kmajor_desc(b_addr + boff), C::kIdesc, (i > 0 || kk > 0) ? 1u : 0u);
              if (SPLITX) umma2_bf16_ss(dt, ad, sw128_kmajor_desc(blo_addr + boff), C::kIdesc, 1u);
            }
          }
          umma2_commit_both(empty(s));
        }
        if (!ok) break;
        umma2_commit_both(accum_full(b));
      }
      if (!ok && g > 0) {
        // Aborted: the MMAs already issued must finish before TMEM is freed.
        volatile int no_abort = 0;
        const int last = g - 1;
        if (!mbar_wait(empty(last % kStages), (last / kStages) & 1, p.ctl.wait_limit, &no_abort))
          atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - kEpi0;  // 0..15
    const int q = warp & 3;      // TMEM lane quarter this warp may access
    const int cg = e >> 2;       // 64-token column group
    const int frow = 32 * q + lane;  // weight row within this CTA's 128 == TMEM lane
    const uint32_t tlane = static_cast<uint32_t>(32 * q) << 16;
    // GLU: value rows are lanes [0, 64) (quarters 0, 1), gate rows [64, 128)
    // (quarters 2, 3); warps (q, cg) and (q + 2, cg) form pair `pr`.
    const int pr = (q & 1) * 4 + cg;
    float *gbuf = glu_s + pr * (kEc * 32);
    // channel-major runs start at token multiples of kEc: 16-byte vector
    // stores when every row start is 16-byte aligned
    const int esz = p.y_dtype == 0 ? 4 : 2;
    const bool y_vec = CONV && (reinterpret_cast<uintptr_t>(p.y) & 15) == 0 && ((p.ldy * esz) & 15) == 0;
    int j = 0;
    for (int u = cl; u < n_units; u += ncl, ++j) {
      const Unit un = decode_unit(p, u);
      const int b = kAccBufs == 2 ? (j & 1) : 0;
      bool ok = mbar_wait(accum_full(b), (kAccBufs == 2 ? (j >> 1) : j) & 1, p.ctl.wait_limit, flags);
      ok = __all_sync(0xffffffffu, ok);
      // The GLU pairs share named barriers, so all epilogue warps agree on
      // giving up before any of them leaves the loop.
      if (!ok && lane == 0) {
        flags[1] = 1;
        if (!flags[0]) report(p.ctl, flags, kDevTimeoutEpilogue);
      }
      named_bar_sync(kAgreeBar, 32 * kEpiW);
      const bool give_up = flags[1] != 0;
      named_bar_sync(kAgreeBar, 32 * kEpiW);
      if (give_up) break;
      tc_fence_after();
      const uint32_t trow = tmem_base + tlane + b * kPT + cg * kColsPerWarp;
      const int m0 = un.tt * kPT + cg * kColsPerWarp;  // first token of this warp's columns
      const int cols = max(0, min(kColsPerWarp, ((p.M - m0 + kEc - 1) / kEc) * kEc));
      const int tile = 2 * un.ft + static_cast<int>(rank);
      const int64_t n = static_cast<int64_t>(tile) * kPackRows + frow;  // packed row
      auto fetch = [&](int col, float (&v)[kEc]) {
        uint32_t r[kEc];
        __syncwarp();  // tcgen05.ld is warp-collective: reconverge first
        tmem_ld16(trow + col, r);
        tmem_ld_wait();
#pragma unroll
        for (int x = 0; x < kEc; ++x) v[x] = __uint_as_float(r[x]);
      };
      // Channel-major output (y[n][ldy]) of this warp's columns; get(col, v)
      // yields chunk col's sums of the lane's own row (warp-uniform calls).
      // Whole, aligned groups of 64 bytes per row (16 f32 or 32 bf16 tokens)
      // go through quad_transpose: each store writes 64 bytes of 8 rows.
      // With 16 bf16 tokens per warp, lane pairs swap halves instead (32
      // bytes of 16 rows per store).  Partial groups store element runs.
      // Polyphase conv_transpose1d output of this lane's row (co, r): token
      // m goes to frame (poly_q0 + m) poly_s + r - poly_pad of channel co.
      auto emit_poly = [&](auto &&get, bool nvalid) {
        const int64_t co = n / p.poly_s;
        const int r = static_cast<int>(n - co * p.poly_s);
        const float b = (p.bias && nvalid) ? p.bias[co] : 0.f;
        for (int col = 0; col < cols; col += kEc) {
          float v[kEc];
          get(col, v);
          if (!nvalid) continue;
#pragma unroll
          for (int x = 0; x < kEc; ++x) {
            const int tok = m0 + col + x;
            const int64_t t = static_cast<int64_t>(p.poly_q0 + tok) * p.poly_s + r - p.poly_pad;
            if (tok < p.M && t >= 0 && t < p.t_out) {
              const float a = act_single(p.epi, v[x] + b);
              if (p.y_dtype == 0) static_cast<float *>(p.y)[co * p.ldy + t] = a;
              else static_cast<__nv_bfloat16 *>(p.y)[co * p.ldy + t] = __float2bfloat16_rn(a);
            }
          }
        }
      };
      auto emit_cm = [&](auto &&get, float b, bool nvalid) {
        const int gt = (p.y_dtype == 0 || kColsPerWarp < 2 * kEc) ? kEc : 2 * kEc;  // tokens per group
        const int64_t row_q = static_cast<int64_t>(tile) * kPackRows + 32 * q;  // row of lane 0
        if (row_q >= p.N) return;  // no output row in this lane quarter
        for (int col = 0; col < cols; col += gt) {
          const int valid = p.M - (m0 + col);
          if (y_vec && valid >= gt && col + gt <= cols) {
            uint4 a[4], unused0, unused1;
            float v[kEc];
            get(col, v);
            act_segs(p.epi, p.y_dtype, v, b, a[0], a[1], a[2], a[3]);
            if (gt == 2 * kEc) {
              get(col + kEc, v);
              act_segs(p.epi, p.y_dtype, v, b, a[2], a[3], unused0, unused1);
            }
            char *yb = static_cast<char *>(p.y);
            if (p.y_dtype == 0 || gt == 2 * kEc) {
              quad_transpose(a, lane);
              const int64_t tok = m0 + col + (lane & 3) * (16 / esz);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int64_t row = row_q + (lane & ~3) + j;
                if (row < p.N) *reinterpret_cast<uint4 *>(yb + (row * p.ldy + tok) * esz) = a[j];
              }
            } else {
              const bool odd = (lane & 1) != 0;
              const uint4 r = shfl_xor_u4(odd ? a[0] : a[1], 1);
              if (odd) a[0] = r;
              else a[1] = r;
              const int64_t tok = m0 + col + (lane & 1) * 8;
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const int64_t row = row_q + (lane & ~1) + j;
                if (row < p.N) *reinterpret_cast<uint4 *>(yb + (row * p.ldy + tok) * esz) = a[j];
              }
            }
          } else {
            for (int c2 = col; c2 < cols && c2 < col + gt; c2 += kEc) {
              float v[kEc];
              get(c2, v);
              if (nvalid)
                store_run_act(p.epi, p.y_dtype, p.y, n * p.ldy + m0 + c2, p.M - (m0 + c2), y_vec, v, b);
            }
          }
        }
      };
      if (un.tail >= 0) {
        // Tail piece: the raw accumulator goes to scratch and this warp
        // group's counter is bumped; the group that arrives last sums every
        // piece in piece order and runs the epilogue.  GLU value and gate
        // warps count together (the last of the two finishes both halves).
        const int grp = p.glu ? pr : e;
        const int expect = (p.glu ? 2 : 1) * p.tail_pieces;
        auto region = [&](int piece, int warp_e) {
          return p.tail_part + (((static_cast<size_t>(un.tail) * p.tail_pieces + piece) * 2 + rank) * kEpiW + warp_e) *
                                   (static_cast<size_t>(kColsPerWarp) * 32);
        };
        float *mine = region(un.piece, e);
        for (int col = 0; col < cols; col += kEc) {
          float v[kEc];
          fetch(col, v);
#pragma unroll
          for (int x = 0; x < kEc; ++x) __stcg(mine + (col + x) * 32 + lane, v[x]);
        }
        __threadfence();
        __syncwarp();
        int *cnt = p.tail_cnt + (un.tail * 2 + static_cast<int>(rank)) * kEpiW + grp;
        int old = 0;
        if (lane == 0) {
          old = atomicAdd(cnt, 1);
          __threadfence();
        }
        __syncwarp();
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == expect - 1) {
          if (lane == 0) *cnt = 0;  // every piece has counted: re-arm for the next call
          auto sum_pieces = [&](int warp_e, int col, float (&v)[kEc]) {
#pragma unroll
            for (int x = 0; x < kEc; ++x) v[x] = __ldcg(region(0, warp_e) + (col + x) * 32 + lane);
            for (int s2 = 1; s2 < p.tail_pieces; ++s2) {
              const float *r = region(s2, warp_e);
#pragma unroll
              for (int x = 0; x < kEc; ++x) v[x] += __ldcg(r + (col + x) * 32 + lane);
            }
          };
          if (!p.glu) {
            const bool nvalid = n < p.N;
            // (a polyphase bias is per output channel: emit_poly reads it)
            const float bn = (p.bias && nvalid && !(CONV && p.poly_s)) ? p.bias[n] : 0.f;
            if (CONV && p.poly_s) {
              emit_poly([&](int col, float(&v)[kEc]) { sum_pieces(e, col, v); }, nvalid);
            } else if (CONV) {
              emit_cm([&](int col, float(&v)[kEc]) { sum_pieces(e, col, v); }, bn, nvalid);
            } else {
              for (int col = 0; col < cols && nvalid; col += kEc) {
                float v[kEc];
                sum_pieces(e, col, v);
                const int valid = p.M - (m0 + col);
                store_act(p.epi, p.y_dtype, p.y, static_cast<int64_t>(m0 + col) * p.ldy + n, p.ldy, valid, v, bn);
              }
            }
          } else {
            // epilogue warp index of lane quarter qq in this column group
            // (warp w reads quarter w & 3; e = w - kEpi0)
            auto quarter_warp = [&](int qq) { return cg * 4 + ((qq - kEpi0) & 3); };
            const int ev = quarter_warp(q & 1), eg = quarter_warp((q & 1) + 2);  // value and gate warps
            const int64_t jcol = static_cast<int64_t>(tile) * 64 + (frow & 63);
            const bool jvalid = jcol < p.n_out;
            const float bv = (p.bias && jvalid) ? p.bias[jcol] : 0.f;
            const float bg = (p.bias && jvalid) ? p.bias[p.n_out + jcol] : 0.f;
            for (int col = 0; col < cols && jvalid; col += kEc) {
              float v[kEc], gv[kEc];
              sum_pieces(ev, col, v);
              sum_pieces(eg, col, gv);
#pragma unroll
              for (int x = 0; x < kEc; ++x) gv[x] += bg;
              const int valid = p.M - (m0 + col);
              store_glu_act(p.epi, p.y_dtype, p.y, static_cast<int64_t>(m0 + col) * p.ldy + jcol, p.ldy, valid, v,
                            bv, gv);
            }
          }
        }
      } else if (p.splits > 1) {
        const bool nvalid = n < p.n_rows;
        float *part = p.partials + (static_cast<size_t>(un.split) * p.M + m0) * p.n_rows + n;
        for (int col = 0; col < cols; col += kEc) {
          float v[kEc];
          fetch(col, v);
          const int valid = p.M - (m0 + col);
          if (!nvalid) continue;
#pragma unroll
          for (int x = 0; x < kEc; ++x)
            if (x < valid) part[static_cast<size_t>(col + x) * p.n_rows] = v[x];
        }
      } else if (CONV && p.poly_s) {
        emit_poly(fetch, n < p.N);
      } else if (CONV) {
        const bool nvalid = n < p.N;
        emit_cm(fetch, (p.bias && nvalid) ? p.bias[n] : 0.f, nvalid);
      } else if (!p.glu) {
        const bool nvalid = n < p.N;
        const float bn = (p.bias && nvalid) ? p.bias[n] : 0.f;
        // bf16 rows whose 32 features of this warp all exist: paired 4-byte
        // stores (half the store instructions for one shuffle per token pair;
        // they pay when the epilogue is exposed, and cost ~1% of a multi-round
        // call, where it overlaps the next unit's main loop)
        const bool paired = p.pair_stores && p.y_dtype == 1 && (p.ldy & 1) == 0 &&
                            (reinterpret_cast<uintptr_t>(p.y) & 3) == 0 &&
                            static_cast<int64_t>(tile) * kPackRows + 32 * q + 32 <= p.N;
        for (int col = 0; col < cols; col += kEc) {
          float v[kEc];
          fetch(col, v);
          const int valid = p.M - (m0 + col);
          if (paired && valid >= kEc) {
            store_pair_act(p.epi, static_cast<__nv_bfloat16 *>(p.y) + static_cast<int64_t>(m0 + col) * p.ldy + (n & ~1LL),
                           p.ldy, lane, v, bn);
            continue;
          }
          if (!nvalid) continue;
          store_act(p.epi, p.y_dtype, p.y, static_cast<int64_t>(m0 + col) * p.ldy + n, p.ldy, valid, v, bn);
        }
      } else {
        const bool is_gate = q >= 2;
        const int vrow = frow & 63;
        const int64_t jcol = static_cast<int64_t>(tile) * 64 + vrow;
        const bool jvalid = jcol < p.n_out;
        const float bv = (p.bias && jvalid) ? p.bias[is_gate ? p.n_out + jcol : jcol] : 0.f;
        for (int col = 0; col < cols; col += kEc) {
          float v[kEc];
          fetch(col, v);
          if (is_gate) {
#pragma unroll
            for (int x = 0; x < kEc; ++x) gbuf[x * 32 + lane] = v[x] + bv;
          }
          named_bar_sync(1 + pr, 64);
          if (!is_gate && jvalid) {
            float gv[kEc];
#pragma unroll
            for (int x = 0; x < kEc; ++x) gv[x] = gbuf[x * 32 + lane];
            const int valid = p.M - (m0 + col);
            store_glu_act(p.epi, p.y_dtype, p.y, static_cast<int64_t>(m0 + col) * p.ldy + jcol, p.ldy, valid, v,
                          bv, gv);
          }
          named_bar_sync(1 + pr, 64);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(accum_empty(b));
        else mbar_arrive_remote_relaxed(map_rank(accum_empty(b), 0));  // TMEM reads done; stores need no release
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

template <bool SPLITX, int PT, bool CONV>
cudaError_t launch_t(const CUtensorMap &w, const CUtensorMap &a_hi, const CUtensorMap &a_lo, const GemmBf16Params &p,
                     int pairs, cudaStream_t stream) {
  using C = Cfg<SPLITX, PT>;
  auto kern = gemm_bf16_sm100_kernel<SPLITX, PT, CONV>;
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
  cfg.blockDim = dim3(kThreads);
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
  return launch_pdl(kern, dim3(2 * (pairs < cap ? pairs : cap)), dim3(kThreads), C::kSmemBytes, stream, 2, w, a_hi,
                    a_lo, p);
}

}  // namespace

int gemm_bf16_block_t() { return kPTDefault; }
int gemm_bf16_block_w() { return kPW; }
bool gemm_bf16_unit_ok(int tokens) { return tokens == 64 || tokens == 128 || tokens == 256; }
int gemm_bf16_token_box(int unit_tokens) { return (unit_tokens < 256 ? unit_tokens : 256) / 2; }

cudaError_t launch_gemm_bf16(bool splitx, int unit_tokens, const CUtensorMap &w, const CUtensorMap &a_hi,
                             const CUtensorMap &a_lo, const GemmBf16Params &p, int pairs, cudaStream_t stream) {
  if (p.conv_cpt) {  // implicit conv1d: channel-major output, no GLU, no split-K
    if (!p.y_cm || p.glu || p.splits > 1) return cudaErrorInvalidValue;
    switch (unit_tokens * 2 + (splitx ? 1 : 0)) {
      case 512: return launch_t<false, 256, true>(w, a_hi, a_lo, p, pairs, stream);
      case 513: return launch_t<true, 256, true>(w, a_hi, a_lo, p, pairs, stream);
      case 256: return launch_t<false, 128, true>(w, a_hi, a_lo, p, pairs, stream);
      case 257: return launch_t<true, 128, true>(w, a_hi, a_lo, p, pairs, stream);
      case 128: return launch_t<false, 64, true>(w, a_hi, a_lo, p, pairs, stream);
      case 129: return launch_t<true, 64, true>(w, a_hi, a_lo, p, pairs, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  if (p.y_cm) return cudaErrorInvalidValue;
  switch (unit_tokens * 2 + (splitx ? 1 : 0)) {
    case 512: return launch_t<false, 256, false>(w, a_hi, a_lo, p, pairs, stream);
    case 513: return launch_t<true, 256, false>(w, a_hi, a_lo, p, pairs, stream);
    case 256: return launch_t<false, 128, false>(w, a_hi, a_lo, p, pairs, stream);
    case 257: return launch_t<true, 128, false>(w, a_hi, a_lo, p, pairs, stream);
    case 128: return launch_t<false, 64, false>(w, a_hi, a_lo, p, pairs, stream);
    case 129: return launch_t<true, 64, false>(w, a_hi, a_lo, p, pairs, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace nq
