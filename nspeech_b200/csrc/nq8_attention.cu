// nq8_attention.cu -- relative-position multi-head self-attention of the
// FastConformer encoder on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Math (MultiHeadSelfAttention::forward + rel_shift, src/parakeet/
// fast_conformer.rs:256-313, 407-425), per segment b and head h:
//   s[i][j] = ((q_i + u_h) . k_j + (q_i + v_h) . r[Tp-1 + j - i]) / sqrt(hd)
//   o_i     = softmax_j(s[i][:]) . V            (keys j >= len[b] masked)
// The reference builds the full [T, 2T-1] position matrix and shifts it
// (rel_shift); here the shift is an index: score (i, j) reads relative row
// Tp-1 + j - i of the band product.  Both score terms use one operand,
// bf16(q + u): (q + v) . r = (q + u) . r + (v - u) . r, and the last term is
// a per-relative-row number vrel[h][p] = (v_h - u_h) . r_p (f32, computed once
// per forward for all layers by relpos_bias_kernel).
//
// Persistent CTAs (one per SM): a work item is one (128 query rows, head,
// segment); CTA c takes items c, c + grid, ...  All tiles of a CTA's items
// form one sequence, so the loads and the S / band MMAs of an item's first
// tile overlap the previous item's last tile and epilogue.  320 threads:
//   warps 0-7  softmax: warp w owns TMEM lanes [32 (w % 4), +32) (query
//              rows) and keys [32 (w / 4), +32) of every 64-key tile; the two
//              warps of a row exchange row maxima through shared memory.
//   warp 8     TMA producers: lane 0 K, lane 1 V, lane 2 relative keys,
//              lane 3 Q, each waiting only on its own ring; owns the TMEM.
//   warp 9     MMA issuer (one elected thread).
// q arrives with u already added (the encoder folds u into the q projection's
// bias), so Q is an MMA operand straight from its TMA tile.
// TMEM (512 columns, f32):
//   [0, 128)   O accumulator                 (128 rows x hd)
//   [128, 256) S = (q+u) K^T, two 64-column buffers (tile tau in buffer tau % 2)
//   [256, 512) band = (q+u) R^T ring: 4 chunks of 64 relative rows.
// Tile t of an item needs relative rows [64t, 64t + 191) of the item's
// window (base row P0 = Tp - 1 - i0 - 127); its tile 0 computes chunks 0..2,
// tile t >= 1 only the new chunk t + 2, so every relative row is multiplied
// once per item (the reference's full [T, 2T-1] product costs twice the
// QK^T work; this costs the same as QK^T).  Each softmax thread loads the
// two 32-column ring chunks its row's diagonal band touches for its 32 keys,
// adds vrel, and shifts them by (31 - lane) in registers with a five-stage
// barrel shift (selects only), so band[i][jl - il + 127] lines up with its
// scores without a trip through shared memory.
// P = exp2(s - m) goes to shared memory as bf16 (K-major, 128-byte swizzle)
// and O += P V runs with V as an MN-major operand straight from its TMA tile.
// O is rescaled only when a row maximum grows by more than 2^8 (the
// exponentials stay <= 256; the final O / l is unchanged by the choice of
// reference maximum).  Items whose query rows all lie past the segment's
// length (padding) are written as zeros.
// Every wait is bounded (DevCtl); on give-up the roles record a kDev* bit,
// drain their copies and MMAs, free TMEM and return.  A softmax warp that
// gives up keeps stepping through its items without touching TMEM, so the
// named barriers it shares with the other softmax warps are always reached.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "nq8_attention.h"
#include "nq8_common.cuh"

namespace nq {
namespace {

constexpr int kHd = 128;       // head dimension
constexpr int kBQ = 128;       // query rows per CTA (TMEM lanes)
constexpr int kBK = 64;        // keys per tile
constexpr int kSoftWarps = 8;
constexpr int kSoftThreads = 32 * kSoftWarps;
constexpr int kProdWarp = kSoftWarps, kMmaWarp = kSoftWarps + 1;
constexpr int kThreads = 32 * (kSoftWarps + 2);  // 320
constexpr uint32_t kTile = 16384;  // [64 rows x 128 hd] bf16 as two 64-column SW128 boxes
constexpr uint32_t kBox = 8192;    // one [64 x 64] SW128 box

// Shared memory (offsets from the 1024-aligned base; SW128 regions 1024-aligned).
constexpr uint32_t kOffQ = 0;                  // [128 rows x 128] bf16(q + u): two 16 KB column halves
constexpr uint32_t kOffK = 32768;              // 2 slots
constexpr uint32_t kOffV = kOffK + 2 * kTile;  // 2 slots
constexpr int kRSlots = 3;                     // relative-key ring: tile 0 of an item takes three chunks
constexpr uint32_t kOffR = kOffV + 2 * kTile;
constexpr uint32_t kOffP = kOffR + kRSlots * kTile;  // [128 rows x 64 keys] bf16
constexpr int kStagePitch = 100;                     // floats per staging row (conflict-free)
constexpr uint32_t kOffStage = kOffP + kTile;        // output staging: one row per query row
constexpr uint32_t kOffRed = kOffStage + kBQ * kStagePitch * 4;
constexpr uint32_t kRedBytes = (2 * 2 + 2) * kBQ * 4;  // row maxima [tile parity][key half][row], sums [half][row]
constexpr uint32_t kOffBar = kOffRed + kRedBytes;
constexpr int kNumBars = 24;
constexpr uint32_t kOffVr = kOffBar + 256;     // vrel over an item's window (f32), sized per launch
constexpr uint32_t kSmemMax = 232448;
constexpr uint32_t kAlignSlack = 1024;

// TMEM columns.
constexpr uint32_t kTmO = 0;
constexpr uint32_t kTmS = 128;
constexpr uint32_t kTmBD = 256;
constexpr uint32_t kTmCols = 512;

// Barriers.
constexpr int kBarKFull = 0, kBarKEmpty = 2, kBarVFull = 4, kBarVEmpty = 6, kBarRFull = 8, kBarREmpty = 11;
constexpr int kBarSFull = 14, kBarSFree = 16, kBarPReady = 18, kBarPvDone = 19, kBarQFull = 20, kBarQFree = 21,
              kBarOFree = 22, kBarMmaDone = 23;
static_assert(kNumBars * 8 + 8 <= 256, "barrier block");

constexpr uint32_t kIdescS = idesc_bf16_f32(128, 64);                // K-major A and B
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, 64) | (1u << 16);  // B (V) MN-major

// Window of relative rows (floats of vrel) a CTA reads over `nt` key tiles:
// the band chunks of the last tile end at window column 64 nt + 128.
__host__ __device__ constexpr int vr_window(int nt) { return kBK * nt + 2 * kBK; }

// Shared-memory descriptor of an MN-major operand with the 128-byte swizzle:
// 64 MN elements per 128-byte row, one row per k, 8-row groups `sbo` apart.
// With N = 64 the operand is one swizzle atom wide, so the MN-atom stride is
// not used; it is set to the k-group stride as well.
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t saddr, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
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

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One work item: query rows [i0, i0 + 128) of head h in segment b, with nt
// key tiles (0: nothing to compute, rows written as zeros).
struct Item {
  int b, h, i0, L, nt;
};
__device__ __forceinline__ Item item_of(const AttnTcParams &p, int it) {
  const int nq = (p.Tp + kBQ - 1) / kBQ;
  const int heads = p.D / kHd;
  Item r;
  const int qt = it % nq;
  const int bh = it / nq;
  r.h = bh % heads;
  r.b = bh / heads;
  r.i0 = qt * kBQ;
  r.L = max(0, min(__ldg(p.len + r.b), p.Tp));
  r.nt = r.i0 < r.L ? (r.L + kBK - 1) / kBK : 0;
  return r;
}

__global__ void __launch_bounds__(kThreads, 1)
    relpos_attention_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_rel,
                               const __grid_constant__ AttnTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
  const uint32_t sbase = smem_u32(smem);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kOffBar);
  auto bar = [&](int i) { return smem_u32(&bars[i]); };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(&bars[kNumBars]);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  float *vr_s = reinterpret_cast<float *>(smem + kOffVr);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long lim = p.ctl.wait_limit;
  const int n_items = ((p.Tp + kBQ - 1) / kBQ) * (p.D / kHd) * p.B;
  const int Tp = p.Tp;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(kBarKFull + s), 1);
      mbar_init(bar(kBarKEmpty + s), 1);
      mbar_init(bar(kBarVFull + s), 1);
      mbar_init(bar(kBarVEmpty + s), 1);
      mbar_init(bar(kBarSFull + s), 1);
      mbar_init(bar(kBarSFree + s), kSoftThreads);
    }
    for (int s = 0; s < kRSlots; ++s) {
      mbar_init(bar(kBarRFull + s), 1);
      mbar_init(bar(kBarREmpty + s), 1);
    }
    mbar_init(bar(kBarPReady), kSoftThreads);
    mbar_init(bar(kBarPvDone), 1);
    mbar_init(bar(kBarQFull), 1);
    mbar_init(bar(kBarQFree), 1);
    mbar_init(bar(kBarOFree), kSoftThreads);
    mbar_init(bar(kBarMmaDone), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProdWarp) {
    tmem_alloc(smem_u32(tmem_slot), kTmCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // barriers and TMEM are set up; now wait for the predecessor's data
  pdl_trigger();

  if (warp == kProdWarp) {
    if (lane < 4) {
      // ------------------------------------------------------------ producers
      // Lane 0 K tiles, lane 1 V tiles, lane 2 relative-key chunks (0 .. nt + 1
      // of each item), lane 3 Q (one per item, once the previous item's last
      // S / band MMAs have read the buffer).
      const int which = lane;
      if (which == 0) {
        prefetch_tmap(&tm_qkv);
        prefetch_tmap(&tm_rel);
      }
      const int nslots = which == 2 ? kRSlots : which == 3 ? 1 : 2;
      const int full0 = which == 0 ? kBarKFull : which == 1 ? kBarVFull : which == 2 ? kBarRFull : kBarQFull;
      const int empty0 = which == 0 ? kBarKEmpty : which == 1 ? kBarVEmpty : which == 2 ? kBarREmpty : kBarQFree;
      const uint32_t slot0 = which == 0 ? kOffK : which == 1 ? kOffV : which == 2 ? kOffR : kOffQ;
      const CUtensorMap *map = which == 2 ? &tm_rel : &tm_qkv;
      int n = 0;  // loads issued
      bool ok = true;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
        const Item w = item_of(p, it);
        if (w.nt == 0) continue;
        const int row0 = w.b * Tp;
        const int P0 = Tp - 1 - w.i0 - (kBQ - 1);
        const int x = which == 0 ? p.D + w.h * kHd : which == 1 ? 2 * p.D + w.h * kHd
                    : which == 2 ? p.rel_col0 + w.h * kHd : w.h * kHd;
        const int count = which == 2 ? w.nt + 2 : which == 3 ? 1 : w.nt;
        for (int k = 0; k < count; ++k) {
          const int s = n % nslots;
          const int use = n / nslots;
          if (use > 0 && !mbar_wait(bar(empty0 + s), (use - 1) & 1, lim, abort_flag)) {
            if (!*abort_flag) report(p.ctl, abort_flag, kDevTimeoutProducer);
            ok = false;
            break;
          }
          if (*abort_flag) {
            ok = false;
            break;
          }
          const uint32_t full = bar(full0 + s);
          const uint32_t dst = sbase + slot0 + s * kTile;
          if (which == 3) {
            // Q rows [i0, i0 + 128): four [64 x 64] boxes (rows past the segment
            // belong to the next one or are zero-filled; their outputs are not stored)
            mbar_arrive_expect_tx(full, 2 * kTile);
#pragma unroll
            for (int half = 0; half < 2; ++half)
#pragma unroll
              for (int rh = 0; rh < 2; ++rh)
                tma_load_2d(dst + half * 16384 + rh * kBox, map, full, x + 64 * half, row0 + w.i0 + 64 * rh);
          } else {
            const int y = which == 2 ? P0 + kBK * k : row0 + k * kBK;
            mbar_arrive_expect_tx(full, kTile);
            tma_load_2d(dst, map, full, x, y);
            tma_load_2d(dst + kBox, map, full, x + 64, y);
          }
          ++n;
        }
      }
      // Drain: every copy this lane issued into shared memory has landed.
      volatile int no_abort = 0;
      for (int s = 0; s < nslots; ++s) {
        const int uses = n > s ? (n - 1 - s) / nslots + 1 : 0;
        if (uses > 0 && !mbar_wait(bar(full0 + s), (uses - 1) & 1, lim, &no_abort))
          atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA
      bool ok = true;
      bool issued = false;
      auto wait = [&](int i, int parity) -> bool {
        if (mbar_wait(bar(i), parity, lim, abort_flag)) return !*abort_flag;
        if (!*abort_flag) report(p.ctl, abort_flag, kDevTimeoutMma);
        return false;
      };
      const uint32_t qa = sbase + kOffQ;
      // O += P V of global tile tau (local tile t of the kq-th item with work):
      // P [128 x 64 keys] K-major, V [64 keys x 128 hd] MN-major.
      auto pv = [&](int tau, int t, int kq) -> bool {
        const int s = tau & 1;
        if (t == 0 && kq > 0 && !wait(kBarOFree, (kq - 1) & 1)) return false;  // previous item's O read
        if (!wait(kBarPReady, tau & 1) || !wait(kBarVFull + s, (tau >> 1) & 1)) return false;
        tc_fence_after();
        const uint32_t pa = sbase + kOffP, va = sbase + kOffV + s * kTile;
#pragma unroll
        for (int nh = 0; nh < 2; ++nh)
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_bf16(tmem + kTmO + 64 * nh, sw128_kmajor_desc(pa + kk * 32), sw128_mn_desc(va + nh * kBox + kk * 2048, 1024),
                      kIdescPV, (t > 0 || kk > 0) ? 1u : 0u);
        umma_commit(bar(kBarVEmpty + s));
        umma_commit(bar(kBarPvDone));
        return true;
      };
      // D[128 x 64] = Q[128 x 128] B[64 x 128]^T, both K-major SW128 tiles.
      auto qk = [&](uint32_t d, uint32_t bt) {
#pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk) {
          const uint32_t ko = (kk >> 2) * 16384 + (kk & 3) * 32, kb = (kk >> 2) * kBox + (kk & 3) * 32;
          umma_bf16(d, sw128_kmajor_desc(qa + ko), sw128_kmajor_desc(bt + kb), kIdescS, kk > 0 ? 1u : 0u);
        }
      };
      int tau = 0, ng = 0, kq = 0, g0 = 0;  // tiles, ring chunks consumed, items with work, chunk base
      int prev_tau = -1, prev_t = 0, prev_kq = 0;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
        const Item w = item_of(p, it);
        if (w.nt == 0) continue;
        // The previous item's last PV goes first: its epilogue (which waits
        // for it) then overlaps this item's first S / band MMAs, and nothing
        // here waits for this item's loads before it.
        if (prev_tau >= 0) {
          if (!(ok = pv(prev_tau, prev_t, prev_kq))) break;
          prev_tau = -1;
        }
        if (!(ok = wait(kBarQFull, kq & 1))) break;
        for (int t = 0; t < w.nt && ok; ++t, ++tau) {
          const int sb = tau & 1;
          // S buffer sb was last read by softmax tau - 2; a first tile also
          // overwrites ring chunks the previous tile (tau - 1) still reads.
          if (t == 0 && tau >= 1) {
            if (!(ok = wait(kBarSFree + ((tau - 1) & 1), ((tau - 1) >> 1) & 1))) break;
          } else if (tau >= 2) {
            if (!(ok = wait(kBarSFree + sb, ((tau >> 1) - 1) & 1))) break;
          }
          if (!(ok = wait(kBarKFull + sb, (tau >> 1) & 1))) break;
          tc_fence_after();
          qk(tmem + kTmS + 64 * sb, sbase + kOffK + sb * kTile);
          issued = true;
          umma_commit(bar(kBarKEmpty + sb));
          for (int c = (t == 0 ? 0 : t + 2); c < t + 3 && ok; ++c, ++ng) {
            const int rs = ng % kRSlots;
            if (!(ok = wait(kBarRFull + rs, (ng / kRSlots) & 1))) break;
            tc_fence_after();
            qk(tmem + kTmBD + 64 * ((g0 + c) & 3), sbase + kOffR + rs * kTile);
            umma_commit(bar(kBarREmpty + rs));
          }
          if (!ok) break;
          if (t == w.nt - 1) umma_commit(bar(kBarQFree));  // every MMA reading this Q is issued
          umma_commit(bar(kBarSFull + sb));
          if (prev_tau >= 0 && !(ok = pv(prev_tau, prev_t, prev_kq))) break;
          prev_tau = tau;
          prev_t = t;
          prev_kq = kq;
        }
        g0 += w.nt + 2;
        ++kq;
      }
      if (ok && prev_tau >= 0) pv(prev_tau, prev_t, prev_kq);
      // Every MMA issued by this thread completes before TMEM is freed.
      if (issued) {
        volatile int no_abort = 0;
        umma_commit(bar(kBarMmaDone));
        if (!mbar_wait(bar(kBarMmaDone), 0, lim, &no_abort)) atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else {
    // -------------------------------------------------------------- softmax
    const int q4 = warp & 3;             // TMEM lane quarter
    const int kh = warp >> 2;            // key half of every tile
    const int il = 32 * q4 + lane;       // query row within the item == TMEM lane
    const int pair_bar = 1 + q4;         // named barrier of warps q4 and q4 + 4
    const uint32_t tl = tmem + (static_cast<uint32_t>(32 * q4) << 16);
    float *red_max = reinterpret_cast<float *>(smem + kOffRed);  // [2][2][128]
    float *red_l = red_max + 4 * kBQ;                            // [2][128]
    float *stage_row = reinterpret_cast<float *>(smem + kOffStage) + il * kStagePitch;  // the row's output staging line
    const int nrel = 2 * Tp - 1;
    const float sl2 = p.sl2;
    bool dead = false;  // warp-uniform: a wait gave up; no TMEM access from here on
    auto wait_all = [&](int i_bar, int parity, int bit) -> bool {
      if (dead) return false;
      bool ok = mbar_wait(bar(i_bar), parity, lim, abort_flag) && !*abort_flag;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok && lane == 0 && !*abort_flag) report(p.ctl, abort_flag, bit);
      return ok;
    };
    int tau = 0, g0 = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      const Item w = item_of(p, it);
      const int i = w.i0 + il;
      const int row0 = w.b * Tp;
      // The previous item's vrel window and staged outputs are
      // no longer read by any softmax warp.
      named_bar_sync(5, kSoftThreads);
      if (w.nt == 0) {
        if (i < Tp) {
          uint4 *orow = reinterpret_cast<uint4 *>(p.out + (static_cast<int64_t>(row0) + i) * p.D + w.h * kHd + 64 * kh);
          for (int c8 = 0; c8 < 8; ++c8) orow[c8] = make_uint4(0u, 0u, 0u, 0u);
        }
        continue;
      }
      // vrel over the item's window: relative rows P0 + [0, W), zero outside the table.
      const int P0 = Tp - 1 - w.i0 - (kBQ - 1);
      const int W = vr_window(w.nt);
      const float *vrel = p.vrel + static_cast<int64_t>(w.h) * nrel;
      for (int x = threadIdx.x; x < W; x += kSoftThreads) {
        const int pr = P0 + x;
        vr_s[x] = (pr >= 0 && pr < nrel) ? __ldg(vrel + pr) : 0.f;
      }
      named_bar_sync(5, kSoftThreads);
      float m_use = -INFINITY, l_part = 0.f;
      for (int t = 0; t < w.nt; ++t, ++tau) {
        const int sb = tau & 1;
        float s[32];
        float tmax = -INFINITY;
        // Band chunks (32 columns) of this row: window chunks kc0 .. kc0 + 2
        // (ring chunk (2 g0 + kc) % 8); the key-half-0 thread reads the first
        // two, the key-half-1 thread the last two.
        const int kc0 = 2 * t + 3 - q4;
        const bool live = wait_all(kBarSFull + sb, (tau >> 1) & 1, kDevTimeoutConsumer);
        if (!live) dead = true;
        if (live) {
          tc_fence_after();
          // This thread's band values: window offsets (31 - lane) + 32 kh + jl,
          // inside the two 32-column chunks kcA, kcA + 1 (ring chunk
          // (2 g0 + kc) % 8), plus vrel of the same window columns.
          const int kcA = kc0 + kh;
          uint32_t a[64], rs[32];
          tmem_ld32(tl + kTmBD + 32 * ((2 * g0 + kcA) & 7), *reinterpret_cast<uint32_t(*)[32]>(a));
          tmem_ld32(tl + kTmBD + 32 * ((2 * g0 + kcA + 1) & 7), *reinterpret_cast<uint32_t(*)[32]>(a + 32));
          tmem_ld32(tl + kTmS + 64 * sb + 32 * kh, rs);
          tmem_ld_wait();
          tc_fence_before();
          mbar_arrive(bar(kBarSFree + sb));  // S buffer and this tile's ring reads are done
          float f[64];
          const float4 *vr4 = reinterpret_cast<const float4 *>(vr_s + 32 * kcA);  // same address in every lane
#pragma unroll
          for (int x = 0; x < 16; ++x) {
            const float4 b = vr4[x];
            f[4 * x] = __uint_as_float(a[4 * x]) + b.x;
            f[4 * x + 1] = __uint_as_float(a[4 * x + 1]) + b.y;
            f[4 * x + 2] = __uint_as_float(a[4 * x + 2]) + b.z;
            f[4 * x + 3] = __uint_as_float(a[4 * x + 3]) + b.w;
          }
          // rel_shift in registers: f[jl] <- f[jl + 31 - lane], a five-stage
          // barrel shift (selects only; register indices stay static).
          const int sh = 31 - lane;
#pragma unroll
          for (int i = 0; i < 48; ++i) f[i] = (sh & 16) ? f[i + 16] : f[i];
#pragma unroll
          for (int i = 0; i < 40; ++i) f[i] = (sh & 8) ? f[i + 8] : f[i];
#pragma unroll
          for (int i = 0; i < 36; ++i) f[i] = (sh & 4) ? f[i + 4] : f[i];
#pragma unroll
          for (int i = 0; i < 34; ++i) f[i] = (sh & 2) ? f[i + 2] : f[i];
#pragma unroll
          for (int i = 0; i < 32; ++i) f[i] = (sh & 1) ? f[i + 1] : f[i];
          const int jbase = t * kBK + 32 * kh;
#pragma unroll
          for (int jl = 0; jl < 32; ++jl) {
            float v = (__uint_as_float(rs[jl]) + f[jl]) * sl2;
            v = jbase + jl < w.L ? v : -INFINITY;
            s[jl] = v;
            tmax = fmaxf(tmax, v);
          }
        }
        // Row maximum over both key halves (the partner warp holds the other).
        float *rm = red_max + (tau & 1) * 2 * kBQ;
        rm[kh * kBQ + il] = tmax;
        named_bar_sync(pair_bar, 64);
        tmax = fmaxf(rm[kBQ + il], rm[il]);  // same order in both warps
        // Reference maximum: the first tile's, raised only when a row grows
        // by more than 8 (log2 units).  Both warps of a row decide alike.
        bool resc = false;
        float factor = 1.f;
        if (t == 0) {
          m_use = tmax;
        } else if (tmax > m_use + 8.f) {
          resc = true;
          factor = ex2(m_use - tmax);
          m_use = tmax;
        }
        // PV of the previous tile has finished: O is stable and the P buffer
        // is free (an item's first tile follows the previous item's epilogue,
        // which waited for it).
        if (t >= 1 && !wait_all(kBarPvDone, (tau - 1) & 1, kDevTimeoutConsumer)) dead = true;
        if (dead) continue;
        if (t >= 1) {
          tc_fence_after();
          if (__any_sync(0xffffffffu, resc)) {
#pragma unroll 1
            for (int x = 0; x < 2; ++x) {
              uint32_t o[32];
              tmem_ld32(tl + kTmO + 64 * kh + 32 * x, o);
              tmem_ld_wait();
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
              tmem_st32(tl + kTmO + 64 * kh + 32 * x, o);
            }
            tmem_st_wait();
          }
        }
        l_part *= factor;
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float p0 = ex2(s[2 * e] - m_use), p1 = ex2(s[2 * e + 1] - m_use);
          l_part += p0 + p1;
          pk[e] = pack_bf16x2(p0, p1);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4 *>(smem + kOffP + sw128_offset(il, 4 * kh + c)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar(kBarPReady));
      }
      // ---- item epilogue: O / l as bf16, through this row's staging line
      if (!wait_all(kBarPvDone, (tau - 1) & 1, kDevTimeoutEpilogue)) dead = true;
      red_l[kh * kBQ + il] = l_part;
      named_bar_sync(pair_bar, 64);
      if (!dead) {
        tc_fence_after();
        const float l_sum = red_l[il] + red_l[kBQ + il];  // same order in both warps
        const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
        uint32_t oa[32], ob[32];
        tmem_ld32(tl + kTmO + 64 * kh, oa);
        tmem_ld32(tl + kTmO + 64 * kh + 32, ob);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(bar(kBarOFree));  // the next item's first PV may overwrite O
        // This thread's 64 outputs (row il, columns [64 kh, +64)) as bf16 into
        // bytes [128 kh, +128) of its row's staging line, then the warp stores
        // its 32 rows 128 bytes at a time.
        uint4 *stage = reinterpret_cast<uint4 *>(stage_row) + 8 * kh;
        auto put = [&](int c, const uint32_t (&o)[32]) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            stage[c + q] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                                      pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                                      pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                                      pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
        };
        put(0, oa);
        put(4, ob);
        __syncwarp();
        const uint4 *wstage = reinterpret_cast<const uint4 *>(smem + kOffStage) + (32 * q4) * (kStagePitch / 4) + 8 * kh;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int r = 4 * k + (lane >> 3);  // row within the warp
          const int ri = w.i0 + 32 * q4 + r;
          if (ri < Tp)
            reinterpret_cast<uint4 *>(p.out + (static_cast<int64_t>(row0) + ri) * p.D + w.h * kHd + 64 * kh)[lane & 7] =
                wstage[r * (kStagePitch / 4) + (lane & 7)];
        }
      }
      g0 += w.nt + 2;
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kProdWarp) {
    tc_fence_after();
    __syncwarp();
    tmem_dealloc(tmem, kTmCols);
  }
}

// vrel[li][h][p] = (v - u)[li][h] . krel[p][li D + h hd : + hd], f32.
// One warp per (li, h) and relative row p; lanes read 4 consecutive bf16.
__global__ void __launch_bounds__(256) relpos_bias_kernel(const __nv_bfloat16 *__restrict__ krel,
                                                          const float *__restrict__ vmu, int nrel, int pairs, int D,
                                                          int64_t ldr, float *__restrict__ vrel) {
  pdl_wait();
  pdl_trigger();
  const int pr = blockIdx.x;
  const int pair = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (pair >= pairs) return;
  const int heads = D / kHd;
  const int li = pair / heads, h = pair - li * heads;
  const int64_t col = static_cast<int64_t>(li) * D + h * kHd + 4 * lane;
  const uint2 kr = *reinterpret_cast<const uint2 *>(krel + static_cast<int64_t>(pr) * ldr + col);
  const float4 w = *reinterpret_cast<const float4 *>(vmu + col);
  float acc = bf16_bits_to_f32(kr.x & 0xFFFFu) * w.x;
  acc = fmaf(bf16_bits_to_f32(kr.x >> 16), w.y, acc);
  acc = fmaf(bf16_bits_to_f32(kr.y & 0xFFFFu), w.z, acc);
  acc = fmaf(bf16_bits_to_f32(kr.y >> 16), w.w, acc);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) vrel[static_cast<int64_t>(pair) * nrel + pr] = acc;
}

}  // namespace

int attention_tc_max_tp() {
  // largest padded length whose vrel window fits next to the fixed buffers
  const int w_max = static_cast<int>((kSmemMax - kAlignSlack - kOffVr) / 4);
  return ((w_max - vr_window(0)) / kBK) * kBK;
}

size_t attention_tc_smem_bytes(int Tp) {
  const int nt = (Tp + kBK - 1) / kBK;
  return kOffVr + static_cast<size_t>(vr_window(nt)) * 4 + kAlignSlack;
}

cudaError_t launch_relpos_attention_tc(const CUtensorMap &tm_qkv, const CUtensorMap &tm_rel, const AttnTcParams &p,
                                       int sm_count, cudaStream_t stream) {
  if (p.D % kHd || p.Tp <= 0 || p.B <= 0 || p.Tp > attention_tc_max_tp() || !p.vrel) return cudaErrorInvalidValue;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(relpos_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemMax));
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const size_t smem = attention_tc_smem_bytes(p.Tp);
  const int items = ((p.Tp + kBQ - 1) / kBQ) * (p.D / kHd) * p.B;
  const int grid = items < sm_count ? items : sm_count;  // persistent: one CTA per SM
  return launch_pdl(relpos_attention_tc_kernel, dim3(grid), dim3(kThreads), smem, stream, 1, tm_qkv, tm_rel, p);
}

cudaError_t launch_relpos_bias(const __nv_bfloat16 *krel, const float *vmu, int nrel, int n_layers, int D,
                               float *vrel, cudaStream_t stream) {
  if (D % kHd || nrel <= 0 || n_layers <= 0) return cudaErrorInvalidValue;
  const int pairs = n_layers * (D / kHd);
  dim3 grid(nrel, (pairs + 7) / 8);
  return launch_pdl(relpos_bias_kernel, grid, dim3(256), 0, stream, 1, krel, vmu, nrel, pairs, D,
                    static_cast<int64_t>(n_layers) * D, vrel);
}

}  // namespace nq
