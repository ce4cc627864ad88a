// nq8_attention.cu -- relative-position multi-head self-attention of the
// FastConformer encoder on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Math (MultiHeadSelfAttention::forward + rel_shift, src/parakeet/
// fast_conformer.rs:256-313, 407-425), per segment b and head h:
//   s[i][j] = ((q_i + u_h) . k_j + (q_i + v_h) . r[Tp-1 + j - i]) / sqrt(hd)
//   o_i     = softmax_j(s[i][:]) . V            (keys j >= len[b] masked)
// The reference builds the full [T, 2T-1] position matrix and shifts it
// (rel_shift); here the shift is an index: score (i, j) reads relative row
// Tp-1 + j - i of the (q + v) R^T product.
//
// CTA = one (128 query rows, head, segment); 192 threads:
//   warps 0-3  softmax: thread = query row = TMEM lane (warp w owns lanes
//              [32w, 32w+32)); they also stage (q + u), (q + v) as bf16.
//   warp 4     TMA producer (K, V, relative-key tiles); owns the TMEM columns.
//   warp 5     MMA issuer (one elected thread).
// Key tiles of 64.  TMEM (512 columns, f32):
//   [0, 128)   O accumulator                 (128 rows x hd)
//   [128, 256) S = (q+u) K^T, two 64-column buffers (tile t in buffer t % 2)
//   [256, 512) BD = (q+v) R^T ring: 4 chunks of 64 relative rows.
// Tile t needs relative rows [64t, 64t + 191) of the CTA's window (base row
// P0 = Tp - 1 - i0 - 127); tile 0 computes chunks 0..2, tile t >= 1 only the
// new chunk t + 2, so every relative row is multiplied once per CTA (the
// reference's full [T, 2T-1] product costs twice the QK^T work; this costs
// the same as QK^T).  Each softmax thread reads the 96 ring columns its warp's
// diagonal band touches, parks them in its own shared-memory row and gathers
// BD[i][jl - il + 127] for its 64 scores.
// P = exp2(s - m) goes to shared memory as bf16 (K-major, 128-byte swizzle)
// and O += P V runs with V as an MN-major operand straight from its TMA tile.
// O is rescaled only when a row maximum grows by more than 2^8 (the
// exponentials stay <= 256; the final O / l is unchanged by the choice of
// reference maximum).
// Every wait is bounded (DevCtl); on give-up the roles record a kDev* bit,
// drain their copies and MMAs, free TMEM and return.
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
constexpr int kThreads = 192;  // 4 softmax warps, producer, MMA
constexpr uint32_t kTile = 16384;  // [64 rows x 128 hd] bf16 as two 64-column SW128 boxes
constexpr uint32_t kBox = 8192;    // one [64 x 64] SW128 box

// Shared memory (offsets from the 1024-aligned base; SW128 regions 1024-aligned).
constexpr uint32_t kOffQu = 0;                 // [128 rows x 128] (q + u): two 16 KB halves
constexpr uint32_t kOffQv = 32768;             // (q + v)
constexpr uint32_t kOffK = 65536;              // 2 slots
constexpr uint32_t kOffV = kOffK + 2 * kTile;  // 2 slots
constexpr uint32_t kOffR = kOffV + 2 * kTile;  // 2 slots of 64 relative rows
constexpr uint32_t kOffP = kOffR + 2 * kTile;  // [128 rows x 64 keys] bf16
constexpr int kParkPitch = 68;                 // floats per parked row (conflict-free)
constexpr uint32_t kOffPark = kOffP + kTile;
constexpr uint32_t kParkBytes = kBQ * kParkPitch * 4;
constexpr uint32_t kOffBar = kOffPark + kParkBytes;
constexpr int kNumBars = 20;
constexpr uint32_t kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "attention shared memory exceeds the sm_100 limit");

// TMEM columns.
constexpr uint32_t kTmO = 0;
constexpr uint32_t kTmS = 128;
constexpr uint32_t kTmBD = 256;
constexpr uint32_t kTmCols = 512;

// Barriers.
constexpr int kBarKFull = 0, kBarKEmpty = 2, kBarVFull = 4, kBarVEmpty = 6, kBarRFull = 8, kBarREmpty = 10;
constexpr int kBarSFull = 12, kBarSFree = 14, kBarPReady = 16, kBarPvDone = 17, kBarQReady = 18, kBarMmaDone = 19;

constexpr uint32_t kIdescS = idesc_bf16_f32(128, 64);                // K-major A and B
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, 64) | (1u << 16);  // B (V) MN-major

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

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// 32 TMEM words -> this thread's parked row, floats [col, col + 32).
__device__ __forceinline__ void park32(float *row, int col, const uint32_t (&r)[32]) {
  const uint32_t a = smem_u32(row + col);
#pragma unroll
  for (int x = 0; x < 8; ++x) st_shared_v4(a + 16 * x, r[4 * x], r[4 * x + 1], r[4 * x + 2], r[4 * x + 3]);
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
      mbar_init(bar(kBarSFree + s), kBQ);
    }
    mbar_init(bar(kBarPReady), kBQ);
    mbar_init(bar(kBarPvDone), 1);
    mbar_init(bar(kBarQReady), kBQ);
    mbar_init(bar(kBarMmaDone), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4) {
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

  if (warp == 4) {
    if (lane == 0 && nt > 0) {
      // ------------------------------------------------------------ producer
      prefetch_tmap(&tm_qkv);
      prefetch_tmap(&tm_rel);
      int n[3] = {0, 0, 0};  // loads issued: K, V, R
      const int full0[3] = {kBarKFull, kBarVFull, kBarRFull};
      const int empty0[3] = {kBarKEmpty, kBarVEmpty, kBarREmpty};
      const uint32_t slot0[3] = {kOffK, kOffV, kOffR};
      bool ok = true;
      // Load the next tile of ring `which` (0 K, 1 V, 2 R) from map rows
      // [y, y + 64), columns [x, x + 128).
      auto load = [&](int which, const CUtensorMap *map, int x, int y) -> bool {
        const int s = n[which] & 1;
        const int use = n[which] >> 1;
        if (use > 0 && !mbar_wait(bar(empty0[which] + s), (use - 1) & 1, lim, abort_flag)) {
          if (!*abort_flag) report(p.ctl, abort_flag, kDevTimeoutProducer);
          return false;
        }
        if (*abort_flag) return false;
        const uint32_t full = bar(full0[which] + s);
        const uint32_t dst = sbase + slot0[which] + s * kTile;
        mbar_arrive_expect_tx(full, kTile);
        tma_load_2d(dst, map, full, x, y);
        tma_load_2d(dst + kBox, map, full, x + 64, y);
        ++n[which];
        return true;
      };
      const int xk = p.D + h * kHd, xv = 2 * p.D + h * kHd, xr = p.rel_col0 + h * kHd;
      for (int t = 0; t < nt && ok; ++t) {
        ok = load(0, &tm_qkv, xk, row0 + t * kBK);
        for (int g = (t == 0 ? 0 : t + 2); g < t + 3 && ok; ++g) ok = load(2, &tm_rel, xr, P0 + kBK * g);
        if (ok && t >= 1) ok = load(1, &tm_qkv, xv, row0 + (t - 1) * kBK);
      }
      if (ok) load(1, &tm_qkv, xv, row0 + (nt - 1) * kBK);
      // Drain: every copy issued into this CTA's shared memory has landed.
      volatile int no_abort = 0;
      for (int w = 0; w < 3; ++w)
        for (int s = 0; s < 2; ++s) {
          const int uses = (n[w] - s + 1) >> 1;
          if (uses > 0 && !mbar_wait(bar(full0[w] + s), (uses - 1) & 1, lim, &no_abort))
            atomicOr(p.ctl.status, kDevTimeoutDrain);
        }
    }
  } else if (warp == 5) {
    if (lane == 0 && nt > 0) {
      // ------------------------------------------------------------ MMA
      bool ok = true;
      auto wait = [&](int i, int parity) -> bool {
        if (mbar_wait(bar(i), parity, lim, abort_flag)) return !*abort_flag;
        if (!*abort_flag) report(p.ctl, abort_flag, kDevTimeoutMma);
        return false;
      };
      const uint32_t qu = sbase + kOffQu, qv = sbase + kOffQv;
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
      // D[128 x 64] = A[128 x 128] B[64 x 128]^T, both K-major SW128 tiles.
      auto qk = [&](uint32_t d, uint32_t a, uint32_t bt) {
#pragma unroll
        for (int kk = 0; kk < kHd / 16; ++kk) {
          const uint32_t ko = (kk >> 2) * 16384 + (kk & 3) * 32, kb = (kk >> 2) * kBox + (kk & 3) * 32;
          umma_bf16(d, sw128_kmajor_desc(a + ko), sw128_kmajor_desc(bt + kb), kIdescS, kk > 0 ? 1u : 0u);
        }
      };
      ok = wait(kBarQReady, 0);
      tc_fence_after();
      int ng = 0;  // relative-key chunks consumed
      for (int t = 0; t < nt && ok; ++t) {
        const int sb = t & 1;
        // S buffer sb and ring chunk (t + 2) % 4 were last read by softmax t - 2.
        if (t >= 2 && !(ok = wait(kBarSFree + sb, ((t >> 1) - 1) & 1))) break;
        if (!(ok = wait(kBarKFull + sb, (t >> 1) & 1))) break;
        tc_fence_after();
        qk(tmem + kTmS + 64 * sb, qu, sbase + kOffK + sb * kTile);
        umma_commit(bar(kBarKEmpty + sb));
        for (int g = (t == 0 ? 0 : t + 2); g < t + 3 && ok; ++g, ++ng) {
          const int rs = ng & 1;
          if (!(ok = wait(kBarRFull + rs, (ng >> 1) & 1))) break;
          tc_fence_after();
          qk(tmem + kTmBD + 64 * (g & 3), qv, sbase + kOffR + rs * kTile);
          umma_commit(bar(kBarREmpty + rs));
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
    const int il = threadIdx.x;  // query row within the CTA == TMEM lane
    const int i = i0 + il;
    const uint32_t tl = tmem + (static_cast<uint32_t>(32 * warp) << 16);
    const int64_t ld = 3 * static_cast<int64_t>(p.D);
    // (q + u) and (q + v) rounded to bf16, K-major with the 128-byte swizzle.
    {
      const __nv_bfloat16 *src = p.qkv + (static_cast<int64_t>(row0) + i) * ld + h * kHd;
      const float *bu = p.bias_u + h * kHd;
      const float *bv = p.bias_v + h * kHd;
#pragma unroll 4
      for (int c8 = 0; c8 < kHd / 8; ++c8) {
        uint4 raw = make_uint4(0u, 0u, 0u, 0u);
        if (i < Tp) raw = __ldg(reinterpret_cast<const uint4 *>(src + c8 * 8));
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
        uint32_t pu[4], pv4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = c8 * 8 + 2 * e;
          const float q0 = bf16_bits_to_f32(w[e] & 0xFFFFu), q1 = bf16_bits_to_f32(w[e] >> 16);
          pu[e] = pack_bf16x2(q0 + __ldg(bu + c), q1 + __ldg(bu + c + 1));
          pv4[e] = pack_bf16x2(q0 + __ldg(bv + c), q1 + __ldg(bv + c + 1));
        }
        const uint32_t off = (c8 >> 3) * 16384 + sw128_offset(il, c8 & 7);
        st_shared_v4(sbase + kOffQu + off, pu[0], pu[1], pu[2], pu[3]);
        st_shared_v4(sbase + kOffQv + off, pv4[0], pv4[1], pv4[2], pv4[3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(bar(kBarQReady));
    }
    __nv_bfloat16 *orow = p.out + (static_cast<int64_t>(row0) + i) * p.D + h * kHd;
    if (nt == 0) {
      if (i < Tp)
        for (int c8 = 0; c8 < kHd / 8; ++c8) reinterpret_cast<uint4 *>(orow)[c8] = make_uint4(0u, 0u, 0u, 0u);
    } else {
      float *park = reinterpret_cast<float *>(smem + kOffPark) + il * kParkPitch;
      const float sl2 = p.sl2;
      float m_use = -INFINITY, l_sum = 0.f;
      bool alive = true;
      auto wait_all = [&](int i_bar, int parity, int bit) -> bool {
        bool ok = mbar_wait(bar(i_bar), parity, lim, abort_flag) && !*abort_flag;
        ok = __all_sync(0xffffffffu, ok);  // the warp proceeds (warp-collective TMEM access) or leaves together
        if (!ok && lane == 0 && !*abort_flag) report(p.ctl, abort_flag, bit);
        return ok;
      };
      for (int t = 0; t < nt; ++t) {
        const int sb = t & 1;
        if (!(alive = wait_all(kBarSFull + sb, (t >> 1) & 1, kDevTimeoutConsumer))) break;
        tc_fence_after();
        // Ring chunks (32 columns) of this warp's band: window offset
        // 64t + 96 - 32w; thread `lane` reads offsets (31 - lane) + jl.
        const int k0 = 2 * t + 3 - warp;
        float s[kBK];
        uint32_t ra[32], rb[32];
        tmem_ld32(tl + kTmBD + 32 * (k0 & 7), ra);
        tmem_ld32(tl + kTmBD + 32 * ((k0 + 1) & 7), rb);
        tmem_ld_wait();
        park32(park, 0, ra);
        park32(park, 32, rb);
        tmem_ld32(tl + kTmS + 64 * sb, ra);
        tmem_ld32(tl + kTmBD + 32 * ((k0 + 2) & 7), rb);
        tmem_ld_wait();
        const int jbase = t * kBK;
        float tmax = -INFINITY;
#pragma unroll
        for (int jl = 0; jl < 32; ++jl) {
          float v = (__uint_as_float(ra[jl]) + park[31 - lane + jl]) * sl2;
          v = jbase + jl < L ? v : -INFINITY;
          s[jl] = v;
          tmax = fmaxf(tmax, v);
        }
        park32(park, 0, rb);  // window offsets [64, 96) reuse parked columns [0, 32)
        tmem_ld32(tl + kTmS + 64 * sb + 32, ra);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(bar(kBarSFree + sb));  // S buffer and this tile's ring reads are done
#pragma unroll
        for (int jl = 32; jl < kBK; ++jl) {
          float v = (__uint_as_float(ra[jl - 32]) + park[(31 - lane + jl) & 63]) * sl2;
          v = jbase + jl < L ? v : -INFINITY;
          s[jl] = v;
          tmax = fmaxf(tmax, v);
        }
        // Reference maximum: the first tile's, raised only when a row grows
        // by more than 8 (log2 units).
        bool resc = false;
        float factor = 1.f;
        if (t == 0) {
          m_use = tmax;
        } else if (tmax > m_use + 8.f) {
          resc = true;
          factor = ex2(m_use - tmax);
          m_use = tmax;
        }
        if (t >= 1) {
          // PV_{t-1} has finished: O is stable and the P buffer is free.
          if (!(alive = wait_all(kBarPvDone, (t - 1) & 1, kDevTimeoutConsumer))) break;
          tc_fence_after();
          if (__any_sync(0xffffffffu, resc)) {
#pragma unroll 1
            for (int x = 0; x < kHd / 32; ++x) {
              uint32_t o[32];
              tmem_ld32(tl + kTmO + 32 * x, o);
              tmem_ld_wait();
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
              tmem_st32(tl + kTmO + 32 * x, o);
            }
            tmem_st_wait();
          }
        }
        l_sum *= factor;
        uint32_t pk[kBK / 2];
#pragma unroll
        for (int e = 0; e < kBK / 2; ++e) {
          const float p0 = ex2(s[2 * e] - m_use), p1 = ex2(s[2 * e + 1] - m_use);
          l_sum += p0 + p1;
          pk[e] = pack_bf16x2(p0, p1);
        }
#pragma unroll
        for (int c = 0; c < 8; ++c)
          st_shared_v4(sbase + kOffP + sw128_offset(il, c), pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar(kBarPReady));
      }
      if (alive && (alive = wait_all(kBarPvDone, (nt - 1) & 1, kDevTimeoutEpilogue))) {
        tc_fence_after();
        const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
#pragma unroll 1
        for (int x = 0; x < kHd / 32; ++x) {
          uint32_t o[32];
          tmem_ld32(tl + kTmO + 32 * x, o);
          tmem_ld_wait();
          if (i < Tp) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint4 v;
              v.x = pack_bf16x2(__uint_as_float(o[8 * c + 0]) * inv, __uint_as_float(o[8 * c + 1]) * inv);
              v.y = pack_bf16x2(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv);
              v.z = pack_bf16x2(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv);
              v.w = pack_bf16x2(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv);
              reinterpret_cast<uint4 *>(orow + 32 * x)[c] = v;
            }
          }
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    __syncwarp();
    tmem_dealloc(tmem, kTmCols);
  }
}

}  // namespace

size_t attention_tc_smem_bytes() { return kSmemBytes; }

cudaError_t launch_relpos_attention_tc(const CUtensorMap &tm_qkv, const CUtensorMap &tm_rel, const AttnTcParams &p,
                                       int B, int H, cudaStream_t stream) {
  if (p.D != H * kHd || p.Tp <= 0 || B <= 0) return cudaErrorInvalidValue;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(relpos_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  dim3 grid((p.Tp + kBQ - 1) / kBQ, H, B);
  return launch_pdl(relpos_attention_tc_kernel, grid, dim3(kThreads), kSmemBytes, stream, 1, tm_qkv, tm_rel, p);
}

}  // namespace nq
