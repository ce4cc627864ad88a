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
// CTA = one (128 query rows, head, segment); 320 threads:
//   warps 0-7  softmax: warp w owns TMEM lanes [32 (w % 4), +32) (query
//              rows) and keys [32 (w / 4), +32) of every 64-key tile; the two
//              warps of a row exchange row maxima through shared memory.
//   warp 8     TMA producers: lane 0 Q and K, lane 1 V, lane 2 relative
//              keys, each waiting only on its own ring; owns the TMEM columns.
//   warp 9     MMA issuer (one elected thread).
// TMEM (512 columns, f32):
//   [0, 128)   O accumulator                 (128 rows x hd)
//   [128, 256) S = (q+u) K^T, two 64-column buffers (tile t in buffer t % 2)
//   [256, 512) band = (q+u) R^T ring: 4 chunks of 64 relative rows.
// Tile t needs relative rows [64t, 64t + 191) of the CTA's window (base row
// P0 = Tp - 1 - i0 - 127); tile 0 computes chunks 0..2, tile t >= 1 only the
// new chunk t + 2, so every relative row is multiplied once per CTA (the
// reference's full [T, 2T-1] product costs twice the QK^T work; this costs
// the same as QK^T).  Each softmax thread reads the 64 ring columns its
// diagonal band touches, adds vrel, parks them in its own shared-memory row
// and gathers band[i][jl - il + 127] for its 32 scores.
// P = exp2(s - m) goes to shared memory as bf16 (K-major, 128-byte swizzle)
// and O += P V runs with V as an MN-major operand straight from its TMA tile.
// O is rescaled only when a row maximum grows by more than 2^8 (the
// exponentials stay <= 256; the final O / l is unchanged by the choice of
// reference maximum).
// Every wait is bounded (DevCtl); on give-up the roles record a kDev* bit,
// drain their copies and MMAs, free TMEM and return.  A softmax warp that
// gives up keeps stepping through its tiles without touching TMEM, so the
// named barrier it shares with its partner warp is always reached.
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
constexpr uint32_t kOffR = kOffV + 2 * kTile;  // 2 slots of 64 relative rows
constexpr uint32_t kOffP = kOffR + 2 * kTile;  // [128 rows x 64 keys] bf16
constexpr int kParkPitch = 68;                 // floats per parked row (conflict-free)
constexpr uint32_t kOffPark = kOffP + kTile;   // one row per softmax thread
constexpr uint32_t kOffRed = kOffPark + kSoftThreads * kParkPitch * 4;
constexpr uint32_t kRedBytes = (2 * 2 + 2) * kBQ * 4;  // row maxima [tile parity][key half][row], sums [half][row]
constexpr uint32_t kOffBar = kOffRed + kRedBytes;
constexpr int kNumBars = 22;
constexpr uint32_t kOffVr = kOffBar + 256;     // vrel over the CTA's window (f32), sized per launch
constexpr uint32_t kSmemMax = 232448;
constexpr uint32_t kAlignSlack = 1024;

// TMEM columns.
constexpr uint32_t kTmO = 0;
constexpr uint32_t kTmS = 128;
constexpr uint32_t kTmBD = 256;
constexpr uint32_t kTmCols = 512;

// Barriers.
constexpr int kBarKFull = 0, kBarKEmpty = 2, kBarVFull = 4, kBarVEmpty = 6, kBarRFull = 8, kBarREmpty = 10;
constexpr int kBarSFull = 12, kBarSFree = 14, kBarPReady = 16, kBarPvDone = 17, kBarQFull = 18, kBarQReady = 19,
              kBarMmaDone = 20, kBarR2Full = 21;
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

// 32 TMEM words plus 32 vrel values -> this thread's parked row, floats
// [col, col + 32).  Plain shared-memory accesses (no asm memory clobber), so
// the compiler overlaps the broadcast vrel loads with the stores.
__device__ __forceinline__ void park32(float *row, int col, const uint32_t (&r)[32], const float *vr) {
  float4 *dst = reinterpret_cast<float4 *>(row + col);
  const float4 *src = reinterpret_cast<const float4 *>(vr);  // same address in every lane: broadcast
  float4 b[8];
#pragma unroll
  for (int x = 0; x < 8; ++x) b[x] = src[x];
#pragma unroll
  for (int x = 0; x < 8; ++x)
    dst[x] = make_float4(__uint_as_float(r[4 * x]) + b[x].x, __uint_as_float(r[4 * x + 1]) + b[x].y,
                         __uint_as_float(r[4 * x + 2]) + b[x].z, __uint_as_float(r[4 * x + 3]) + b[x].w);
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
  const int b = blockIdx.z;
  const int h = blockIdx.y;
  const int i0 = blockIdx.x * kBQ;
  const long long lim = p.ctl.wait_limit;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(kBarKFull + s), 1);
      mbar_init(bar(kBarKEmpty + s), 1);
      mbar_init(bar(kBarVFull + s), 1);
      mbar_init(bar(kBarVEmpty + s), 1);
      mbar_init(bar(kBarRFull + s), 1);
      mbar_init(bar(kBarREmpty + s), 1);
      mbar_init(bar(kBarSFull + s), 1);
      mbar_init(bar(kBarSFree + s), kSoftThreads);
    }
    mbar_init(bar(kBarPReady), kSoftThreads);
    mbar_init(bar(kBarPvDone), 1);
    mbar_init(bar(kBarQFull), 1);
    mbar_init(bar(kBarQReady), kSoftThreads);
    mbar_init(bar(kBarMmaDone), 1);
    mbar_init(bar(kBarR2Full), 1);
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

  const int Tp = p.Tp;
  const int L = max(0, min(p.len[b], Tp));
  const int nt = (L + kBK - 1) / kBK;
  const int row0 = b * Tp;                 // first qkv row of the segment
  const int P0 = Tp - 1 - i0 - (kBQ - 1);  // relative row of window column 0

  if (warp == kProdWarp) {
    if (lane < 3 && nt > 0) {
      // ------------------------------------------------------------ producers
      // One lane per ring, each waiting only on its own ring's slots: lane 0
      // Q and K, lane 1 V, lane 2 the relative keys.
      const int which = lane;
      if (which == 0) {
        prefetch_tmap(&tm_qkv);
        prefetch_tmap(&tm_rel);
        // Q rows [i0, i0 + 128): four [64 x 64] boxes (rows past the segment
        // belong to the next one or are zero-filled; their outputs are not stored)
        mbar_arrive_expect_tx(bar(kBarQFull), 2 * kTile);
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
          for (int rh = 0; rh < 2; ++rh)
            tma_load_2d(sbase + kOffQ + half * 16384 + rh * kBox, &tm_qkv, bar(kBarQFull), h * kHd + 64 * half,
                        row0 + i0 + 64 * rh);
      }
      const int full0 = which == 0 ? kBarKFull : which == 1 ? kBarVFull : kBarRFull;
      const uint32_t slot0 = which == 0 ? kOffK : which == 1 ? kOffV : kOffR;
      const CUtensorMap *map = which == 2 ? &tm_rel : &tm_qkv;
      const int x = which == 0 ? p.D + h * kHd : which == 1 ? 2 * p.D + h * kHd : p.rel_col0 + h * kHd;
      // K and V: tile k; relative keys: chunks 0, 1, then 3 .. nt + 1 through
      // the ring, and chunk 2 (tile 0's third) into the P buffer, which stays
      // unused until softmax 0 has waited for the MMA that reads it.
      const int count = which == 2 ? nt + 1 : nt;
      int n = 0;
      bool r2 = false;
      for (int k = 0; k < count; ++k) {
        if (which == 2 && k == 2 && !r2) {
          mbar_arrive_expect_tx(bar(kBarR2Full), kTile);
          tma_load_2d(sbase + kOffP, &tm_rel, bar(kBarR2Full), x, P0 + 2 * kBK);
          tma_load_2d(sbase + kOffP + kBox, &tm_rel, bar(kBarR2Full), x + 64, P0 + 2 * kBK);
          r2 = true;
        }
        const int y = which == 2 ? P0 + kBK * (k < 2 ? k : k + 1) : row0 + k * kBK;
        const int s = n & 1;
        const int use = n >> 1;
        if (use > 0 && !mbar_wait(bar(full0 + 2 + s), (use - 1) & 1, lim, abort_flag)) {
          if (!*abort_flag) report(p.ctl, abort_flag, kDevTimeoutProducer);
          break;
        }
        if (*abort_flag) break;
        const uint32_t full = bar(full0 + s);
        const uint32_t dst = sbase + slot0 + s * kTile;
        mbar_arrive_expect_tx(full, kTile);
        tma_load_2d(dst, map, full, x, y);
        tma_load_2d(dst + kBox, map, full, x + 64, y);
        ++n;
      }
      if (which == 2 && count == 2 && n == 2 && !r2) {  // nt == 1: chunk 2 after the loop
        mbar_arrive_expect_tx(bar(kBarR2Full), kTile);
        tma_load_2d(sbase + kOffP, &tm_rel, bar(kBarR2Full), x, P0 + 2 * kBK);
        tma_load_2d(sbase + kOffP + kBox, &tm_rel, bar(kBarR2Full), x + 64, P0 + 2 * kBK);
        r2 = true;
      }
      // Drain: every copy this lane issued into shared memory has landed.
      volatile int no_abort = 0;
      if (which == 0 && !mbar_wait(bar(kBarQFull), 0, lim, &no_abort)) atomicOr(p.ctl.status, kDevTimeoutDrain);
      if (r2 && !mbar_wait(bar(kBarR2Full), 0, lim, &no_abort)) atomicOr(p.ctl.status, kDevTimeoutDrain);
      for (int s = 0; s < 2; ++s) {
        const int uses = (n - s + 1) >> 1;
        if (uses > 0 && !mbar_wait(bar(full0 + s), (uses - 1) & 1, lim, &no_abort))
          atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0 && nt > 0) {
      // ------------------------------------------------------------ MMA
      bool ok = true;
      auto wait = [&](int i, int parity) -> bool {
        if (mbar_wait(bar(i), parity, lim, abort_flag)) return !*abort_flag;
        if (!*abort_flag) report(p.ctl, abort_flag, kDevTimeoutMma);
        return false;
      };
      const uint32_t qa = sbase + kOffQ;
      // O += P V_tau: P [128 x 64 keys] K-major, V [64 keys x 128 hd] MN-major.
      auto pv = [&](int tau) -> bool {
        const int s = tau & 1;
        if (!wait(kBarPReady, tau & 1) || !wait(kBarVFull + s, (tau >> 1) & 1)) return false;
        tc_fence_after();
        const uint32_t pa = sbase + kOffP, va = sbase + kOffV + s * kTile;
#pragma unroll
        for (int nh = 0; nh < 2; ++nh)
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_bf16(tmem + kTmO + 64 * nh, sw128_kmajor_desc(pa + kk * 32), sw128_mn_desc(va + nh * kBox + kk * 2048, 1024),
                      kIdescPV, (tau > 0 || kk > 0) ? 1u : 0u);
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
      ok = wait(kBarQReady, 0);
      tc_fence_after();
      int ng = 0;  // relative-key chunks consumed from the ring
      for (int t = 0; t < nt && ok; ++t) {
        const int sb = t & 1;
        // S buffer sb and ring chunk (t + 2) % 4 were last read by softmax t - 2.
        if (t >= 2 && !(ok = wait(kBarSFree + sb, ((t >> 1) - 1) & 1))) break;
        if (!(ok = wait(kBarKFull + sb, (t >> 1) & 1))) break;
        tc_fence_after();
        qk(tmem + kTmS + 64 * sb, sbase + kOffK + sb * kTile);
        umma_commit(bar(kBarKEmpty + sb));
        for (int g = (t == 0 ? 0 : t + 2); g < t + 3 && ok; ++g) {
          if (t == 0 && g == 2) {  // tile 0's third chunk sits in the P buffer
            if (!(ok = wait(kBarR2Full, 0))) break;
            tc_fence_after();
            qk(tmem + kTmBD + 64 * 2, sbase + kOffP);
            continue;
          }
          const int rs = ng & 1;
          if (!(ok = wait(kBarRFull + rs, (ng >> 1) & 1))) break;
          tc_fence_after();
          qk(tmem + kTmBD + 64 * (g & 3), sbase + kOffR + rs * kTile);
          umma_commit(bar(kBarREmpty + rs));
          ++ng;
        }
        if (!ok) break;
        umma_commit(bar(kBarSFull + sb));
        if (t >= 1) ok = pv(t - 1);
      }
      if (ok) pv(nt - 1);
      // Every MMA issued by this thread completes before TMEM is freed.
      volatile int no_abort = 0;
      umma_commit(bar(kBarMmaDone));
      if (!mbar_wait(bar(kBarMmaDone), 0, lim, &no_abort)) atomicOr(p.ctl.status, kDevTimeoutDrain);
    }
  } else {
    // -------------------------------------------------------------- softmax
    const int q4 = warp & 3;             // TMEM lane quarter
    const int kh = warp >> 2;            // key half of every tile
    const int il = 32 * q4 + lane;       // query row within the CTA == TMEM lane
    const int i = i0 + il;
    const int pair_bar = 1 + q4;         // named barrier of warps q4 and q4 + 4
    const uint32_t tl = tmem + (static_cast<uint32_t>(32 * q4) << 16);
    float *red_max = reinterpret_cast<float *>(smem + kOffRed);  // [2][2][128]
    float *red_l = red_max + 4 * kBQ;                            // [2][128]
    __nv_bfloat16 *orow = p.out + (static_cast<int64_t>(row0) + i) * p.D + h * kHd + 64 * kh;
    if (nt == 0) {
      if (i < Tp)
        for (int c8 = 0; c8 < 8; ++c8) reinterpret_cast<uint4 *>(orow)[c8] = make_uint4(0u, 0u, 0u, 0u);
    } else {
      // vrel over the window: relative rows P0 + [0, W), zero outside the table.
      const int W = vr_window(nt);
      const int nrel = 2 * Tp - 1;
      const float *vrel = p.vrel + static_cast<int64_t>(h) * nrel;
      for (int x = threadIdx.x; x < W; x += kSoftThreads) {
        const int pr = P0 + x;
        vr_s[x] = (pr >= 0 && pr < nrel) ? __ldg(vrel + pr) : 0.f;
      }
      // bf16(q + u) in place: this thread's row, columns [64 kh, 64 kh + 64).
      {
        float4 bu[16];
        const float4 *u4 = reinterpret_cast<const float4 *>(p.bias_u + h * kHd + 64 * kh);
#pragma unroll
        for (int x = 0; x < 16; ++x) bu[x] = __ldg(u4 + x);
        const bool okq = __all_sync(0xffffffffu, mbar_wait(bar(kBarQFull), 0, lim, abort_flag));
        if (okq) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint4 *a = reinterpret_cast<uint4 *>(smem + kOffQ + kh * 16384 + sw128_offset(il, c));
            const uint4 v = *a;
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float4 bb = bu[2 * c + (e >> 1)];
              const float b0 = (e & 1) ? bb.z : bb.x, b1 = (e & 1) ? bb.w : bb.y;
              o[e] = pack_bf16x2(bf16_bits_to_f32(w[e] & 0xFFFFu) + b0, bf16_bits_to_f32(w[e] >> 16) + b1);
            }
            *a = make_uint4(o[0], o[1], o[2], o[3]);
          }
        } else if (lane == 0 && !*abort_flag) {
          report(p.ctl, abort_flag, kDevTimeoutConsumer);
        }
        fence_proxy_async_smem();
      }
      named_bar_sync(5, kSoftThreads);  // vr_s written by every softmax thread
      mbar_arrive(bar(kBarQReady));
      float *park = reinterpret_cast<float *>(smem + kOffPark) + threadIdx.x * kParkPitch;
      const float sl2 = p.sl2;
      float m_use = -INFINITY, l_part = 0.f;
      bool dead = false;  // warp-uniform: a wait gave up; no TMEM access from here on
      auto wait_all = [&](int i_bar, int parity, int bit) -> bool {
        if (dead) return false;
        bool ok = mbar_wait(bar(i_bar), parity, lim, abort_flag) && !*abort_flag;
        ok = __all_sync(0xffffffffu, ok);
        if (!ok && lane == 0 && !*abort_flag) report(p.ctl, abort_flag, bit);
        return ok;
      };
      for (int t = 0; t < nt; ++t) {
        const int sb = t & 1;
        float s[32];
        float tmax = -INFINITY;
        if (wait_all(kBarSFull + sb, (t >> 1) & 1, kDevTimeoutConsumer)) {
          tc_fence_after();
          // Band chunks (32 columns) of this warp: window chunk kc (column
          // 32 kc) is ring chunk kc % 8; thread `lane` reads window offsets
          // 32 kc + (31 - lane) + jl.
          const int kc = 2 * t + 3 - q4 + kh;
          uint32_t ra[32], rb[32], rs[32];
          tmem_ld32(tl + kTmBD + 32 * (kc & 7), ra);
          tmem_ld32(tl + kTmBD + 32 * ((kc + 1) & 7), rb);
          tmem_ld32(tl + kTmS + 64 * sb + 32 * kh, rs);
          tmem_ld_wait();
          tc_fence_before();
          mbar_arrive(bar(kBarSFree + sb));  // S buffer and this tile's ring reads are done
          park32(park, 0, ra, vr_s + 32 * kc);
          park32(park, 32, rb, vr_s + 32 * (kc + 1));
          const int jbase = t * kBK + 32 * kh;
#pragma unroll
          for (int jl = 0; jl < 32; ++jl) {
            float v = (__uint_as_float(rs[jl]) + park[31 - lane + jl]) * sl2;
            v = jbase + jl < L ? v : -INFINITY;
            s[jl] = v;
            tmax = fmaxf(tmax, v);
          }
        } else {
          dead = true;
        }
        // Row maximum over both key halves (the partner warp holds the other).
        float *rm = red_max + (t & 1) * 2 * kBQ;
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
        // PV_{t-1} has finished: O is stable and the P buffer is free.
        if (t >= 1 && !wait_all(kBarPvDone, (t - 1) & 1, kDevTimeoutConsumer)) dead = true;
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
      if (!wait_all(kBarPvDone, (nt - 1) & 1, kDevTimeoutEpilogue)) dead = true;
      red_l[kh * kBQ + il] = l_part;
      named_bar_sync(pair_bar, 64);
      if (!dead) {
        tc_fence_after();
        const float l_sum = red_l[il] + red_l[kBQ + il];  // same order in both warps
        const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
        // This thread's 64 outputs (row il, columns [64 kh, +64)) as bf16 into
        // its own park row, then the warp stores its 32 rows 128 bytes at a time.
        uint4 *stage = reinterpret_cast<uint4 *>(park);
#pragma unroll 1
        for (int x = 0; x < 2; ++x) {
          uint32_t o[32];
          tmem_ld32(tl + kTmO + 64 * kh + 32 * x, o);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 4; ++c)
            stage[4 * x + c] = make_uint4(
                pack_bf16x2(__uint_as_float(o[8 * c + 0]) * inv, __uint_as_float(o[8 * c + 1]) * inv),
                pack_bf16x2(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv),
                pack_bf16x2(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv),
                pack_bf16x2(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv));
        }
        __syncwarp();
        const uint4 *wstage = reinterpret_cast<const uint4 *>(smem + kOffPark) + (32 * warp) * (kParkPitch / 4);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int r = 4 * k + (lane >> 3);  // row within the warp
          const int ri = i0 + 32 * q4 + r;
          if (ri < Tp)
            reinterpret_cast<uint4 *>(p.out + (static_cast<int64_t>(row0) + ri) * p.D + h * kHd + 64 * kh)[lane & 7] =
                wstage[r * (kParkPitch / 4) + (lane & 7)];
        }
      }
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
                                       int B, int H, cudaStream_t stream) {
  if (p.D != H * kHd || p.Tp <= 0 || B <= 0 || p.Tp > attention_tc_max_tp() || !p.vrel) return cudaErrorInvalidValue;
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
  dim3 grid((p.Tp + kBQ - 1) / kBQ, H, B);
  return launch_pdl(relpos_attention_tc_kernel, grid, dim3(kThreads), smem, stream, 1, tm_qkv, tm_rel, p);
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
