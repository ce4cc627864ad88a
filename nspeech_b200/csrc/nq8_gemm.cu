// nq8_gemm.cu -- K1: persistent tcgen05/TMEM Q8_0 GEMM for M > 16 (sm_100a).
//
// Replaces the tiled matmul family of the reference (Triton source
// kernels/moonshine_kernels.py:20-299, dispatched by triton_matmul*/enc_matmul*
// in src/triton_kernels.rs:170-309,1205-1289; CPU FbgemmBf16Op in
// src/fast_matmul.rs:138-167).
//
// Y[tok, n] = act(X[tok, :] . bf16(dequant(W[n, :])) + bias[n]).  The tensor
// core computes transposed tiles D[128 weight rows x 128 tokens]: the weights
// are operand A *in tensor memory* (dequantized in registers, tcgen05.st), the
// activations operand B in shared memory (TMA), so dequantized weights never
// touch shared memory.  One CTA per SM walks a static list of work units
// (weight tile, token tile, k split); TMEM holds two accumulators so the
// epilogue of unit j overlaps the main loop of unit j+1.
//   warp 0      producer: TMA 2-D loads of activation tiles [128 tok x 64 k]
//               (bf16, 128-byte swizzle), ring of kStages, mbarrier full_b.
//   warp 1      allocates 512 TMEM columns (D0, D1, kStages A stages); lane 0
//               issues tcgen05.mma (M=128, N=128, K=16, kind::f16, A from
//               TMEM) and commits empty[s] per k step, accum_full[b] per unit.
//   warps 2-5   epilogue: tcgen05.ld (one weight row per lane, 32 tokens),
//               bias + activation (GLU through shared memory), stores that
//               are contiguous along the output row across the warp; split-K
//               partials with an arrival counter (last CTA sums in order).
//   warps 6-21  dequant: warp w owns TMEM lanes 32*(w%4).. (weight rows); the
//               four warps of a lane quarter take turns by 64-wide k step
//               (warp `sub` fills A stage `sub`): coalesced 16-byte loads of
//               the next turn prefetched across units, bf16(f32(d)*q) with
//               packed f32x2 arithmetic, tcgen05.st 32x32b.x32, arrive full_a.
// f32 activations arrive as two bf16 planes (hi, lo): two MMAs per k step.
// Every wait is bounded; on give-up the kernel records a status bit, drains
// in-flight copies and MMAs, frees TMEM and returns.  No cluster multicast.
#include "nq8_common.cuh"
#include "nq8_kernels.h"

namespace nq {

constexpr int kBT = 128;  // tokens per tile
constexpr int kStages = 4;
constexpr int kEpiWarps = 4;
constexpr int kConvWarps = 16;  // 4 per TMEM lane quarter, one 16-k chunk each
constexpr int kGemmThreads = 32 * (2 + kEpiWarps + kConvWarps);  // 704
constexpr int kEpiWarp0 = 2;
constexpr int kConvWarp0 = kEpiWarp0 + kEpiWarps;

template <bool SPLITX>
struct GemmCfg {
  static constexpr int kBBytes = kBT * kPackK * 2;  // 16 KB per activation plane
  static constexpr int kStageBytes = kBBytes * (SPLITX ? 2 : 1);
  static constexpr int kGluOffset = kStages * kStageBytes;
  static constexpr int kGluBytes = 64 * kBT * 4;
  static constexpr int kBarOffset = kGluOffset + kGluBytes;
  static constexpr int kSmemBytes = 1024 /*align slack*/ + kBarOffset + 512;
  static constexpr uint32_t kIdesc = idesc_bf16_f32(128, kBT);
  static constexpr int kACol = 2 * kBT;  // D0 [0,128), D1 [128,256), A stages [256, 384)
  static constexpr int kTmemCols = 512;
};

__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- dequant
__device__ __forceinline__ uint64_t f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_of(uint64_t v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  return pack_bf16x2(a, b);
}
// Eight int8 (two words) of one Q8_0 block -> four bf16x2 of bf16(f32(d) * q),
// exact like dequant4_bf16, with packed f32x2 subtract / multiply.
__device__ __forceinline__ void dequant8_bf16(uint32_t w0, uint32_t w1, uint64_t dd, uint32_t *out) {
  const uint32_t u0 = w0 ^ 0x80808080u, u1 = w1 ^ 0x80808080u;
  const uint64_t bias = f2(8388736.0f, 8388736.0f);
  uint64_t v[4];
  v[0] = f2(__uint_as_float(__byte_perm(u0, 0x4B000000u, 0x7440)), __uint_as_float(__byte_perm(u0, 0x4B000000u, 0x7441)));
  v[1] = f2(__uint_as_float(__byte_perm(u0, 0x4B000000u, 0x7442)), __uint_as_float(__byte_perm(u0, 0x4B000000u, 0x7443)));
  v[2] = f2(__uint_as_float(__byte_perm(u1, 0x4B000000u, 0x7440)), __uint_as_float(__byte_perm(u1, 0x4B000000u, 0x7441)));
  v[3] = f2(__uint_as_float(__byte_perm(u1, 0x4B000000u, 0x7442)), __uint_as_float(__byte_perm(u1, 0x4B000000u, 0x7443)));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint64_t q;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(q) : "l"(v[i]), "l"(bias));
    uint64_t s;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(s) : "l"(q), "l"(dd));
    out[i] = bf16x2_of(s);
  }
}

struct WChunk64 {
  uint4 q[4];            // the 64 int8 of one row in a 64-wide k step
  unsigned short d[2];   // the row's two Q8_0 block scales (f16)
};

// Row `row` of a packed tile: four coalesced 16-byte loads (32 consecutive
// rows per warp each) and the two 2-byte scales.
__device__ __forceinline__ WChunk64 load_wchunk64(const uint8_t *tile, int row) {
  WChunk64 w;
#pragma unroll
  for (int c = 0; c < 4; ++c) w.q[c] = __ldg(reinterpret_cast<const uint4 *>(tile + qs_offset(row, c)));
  w.d[0] = __ldg(reinterpret_cast<const unsigned short *>(tile + scale_offset(row, 0)));
  w.d[1] = __ldg(reinterpret_cast<const unsigned short *>(tile + scale_offset(row, 1)));
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

// ------------------------------------------------------------- work units
struct Unit {
  int ft, tt, split, kc0, nk;
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

// Epilogue chunk: kEc tokens per lane per tcgen05.ld (bounds live registers).
constexpr int kEc = 16;

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

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
template <typename T, int EPI>
__device__ __forceinline__ void store_glu(T *base, int64_t ldy, int valid, const float (&v)[kEc], float b,
                                          const float *gate) {
#pragma unroll
  for (int e = 0; e < kEc; ++e) {
    if (e < valid) {
      const float a = v[e] + b, g = gate[e];
      put<T>(base + e * ldy, EPI == kEpiGluSigmoid ? a * sigmoidf_(g) : a * (g * sigmoidf_(g)));
    }
  }
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
  const int n_units = p.grid_n * p.grid_m * p.splits;

  auto stage_b = [&](int s) { return smem + s * C::kStageBytes; };
  auto stage_blo = [&](int s) { return smem + s * C::kStageBytes + C::kBBytes; };
  float *glu_s = reinterpret_cast<float *>(smem + C::kGluOffset);  // [64][kBT]
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOffset);
  auto full_b = [&](int s) { return smem_u32(&bars[s]); };
  auto full_a = [&](int s) { return smem_u32(&bars[kStages + s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[2 * kStages + s]); };
  auto accum_full = [&](int b) { return smem_u32(&bars[3 * kStages + b]); };
  auto accum_empty = [&](int b) { return smem_u32(&bars[3 * kStages + 2 + b]); };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(&bars[3 * kStages + 4]);
  // [0] abort (any role)  [1] last split of a tile  [2] epilogue gave up
  volatile int *flags = reinterpret_cast<volatile int *>(&bars[3 * kStages + 5]);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_b(s), 1);
      mbar_init(full_a(s), 4);  // one converter warp per TMEM lane quarter fills a stage
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accum_full(b), 1);
      mbar_init(accum_empty(b), kEpiWarps);
    }
    flags[0] = 0;
    flags[1] = 0;
    flags[2] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      prefetch_tmap(&tm_a);
      if (SPLITX) prefetch_tmap(&tm_alo);
      int g = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const Unit un = decode_unit(p, u);
        for (int i = 0; i < un.nk; ++i, ++g) {
          const int s = g % kStages;
          if (g >= kStages && !mbar_wait(empty_bar(s), ((g / kStages) - 1) & 1, p.ctl.wait_limit, flags)) {
            if (!flags[0]) report(p.ctl, flags, kDevTimeoutProducer);
            ok = false;
            break;
          }
          if (flags[0]) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_b(s), C::kStageBytes);
          tma_load_2d(smem_u32(stage_b(s)), &tm_a, full_b(s), (un.kc0 + i) * kPackK, un.tt * kBT);
          if (SPLITX) tma_load_2d(smem_u32(stage_blo(s)), &tm_alo, full_b(s), (un.kc0 + i) * kPackK, un.tt * kBT);
        }
      }
      // Drain: the last load issued into each stage must have landed.
      volatile int no_abort = 0;
      for (int s = 0; s < kStages && s < g; ++s) {
        const int last = s + kStages * ((g - 1 - s) / kStages);
        if (!mbar_wait(full_b(s), (last / kStages) & 1, p.ctl.wait_limit, &no_abort))
          atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issue
      int g = 0, j = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++j) {
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
          const uint32_t par = (g / kStages) & 1;
          if (!mbar_wait(full_a(s), par, p.ctl.wait_limit, flags) || !mbar_wait(full_b(s), par, p.ctl.wait_limit, flags)) {
            if (!flags[0]) report(p.ctl, flags, kDevTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_addr = smem_u32(stage_b(s));
          const uint32_t blo_addr = smem_u32(stage_blo(s));
          const uint32_t a_tmem = tmem_base + C::kACol + s * 32;
#pragma unroll
          for (int kk = 0; kk < kPackK / 16; ++kk) {
            umma_bf16_ts(d_tmem, a_tmem + kk * 8, sw128_kmajor_desc(b_addr + kk * 32), C::kIdesc,
                         (i > 0 || kk > 0) ? 1u : 0u);
            if (SPLITX) umma_bf16_ts(d_tmem, a_tmem + kk * 8, sw128_kmajor_desc(blo_addr + kk * 32), C::kIdesc, 1u);
          }
          umma_commit(empty_bar(s));
        }
        if (!ok) break;
        umma_commit(accum_full(b));
      }
      if (!ok && g > 0) {
        // Aborted: the MMAs already issued must finish before TMEM is freed.
        volatile int no_abort = 0;
        const int last = g - 1;
        if (!mbar_wait(empty_bar(last % kStages), (last / kStages) & 1, p.ctl.wait_limit, &no_abort))
          atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else if (warp < kConvWarp0) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int frow = 32 * q + lane;  // weight row == TMEM lane
    const uint32_t tlane = static_cast<uint32_t>(32 * q) << 16;
    const int et = threadIdx.x - 32 * kEpiWarp0;  // 0..127
    int j = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++j) {
      const Unit un = decode_unit(p, u);
      const int b = j & 1;
      bool ok = mbar_wait(accum_full(b), (j >> 1) & 1, p.ctl.wait_limit, flags);
      ok = __all_sync(0xffffffffu, ok);
      // The four epilogue warps share named barriers below, so they agree on
      // giving up before any of them leaves the loop: a failed warp sets
      // flags[2], everyone reads it between two barriers.
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
      float *part = p.splits > 1
                        ? p.partials + ((static_cast<size_t>(un.split) * p.grid_m + un.tt) * p.grid_n + un.ft) * (128 * kBT)
                        : nullptr;
      if (p.splits > 1) {
        // Park this split's raw accumulators, release the TMEM buffer, then
        // let the last split of the tile finish it.
        for (int col = 0; col < kBT; col += kEc) {
          uint32_t r[kEc];
          tmem_ld16(trow + col, r);
          tmem_ld_wait();
          float4 *dst = reinterpret_cast<float4 *>(part + frow * kBT + col);
#pragma unroll
          for (int e = 0; e < kEc / 4; ++e)
            dst[e] = make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]),
                                 __uint_as_float(r[4 * e + 2]), __uint_as_float(r[4 * e + 3]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(accum_empty(b));
        __threadfence();
        named_bar_sync(1, 32 * kEpiWarps);
        if (et == 0) {
          const int prev = atomicAdd(&p.counters[un.tt * p.grid_n + un.ft], 1);
          flags[1] = (prev == p.splits - 1) ? 1 : 0;
        }
        named_bar_sync(1, 32 * kEpiWarps);
        const bool last = flags[1] != 0;
        named_bar_sync(1, 32 * kEpiWarps);  // everyone has read flags[1]
        if (!last) continue;
        __threadfence();
      }
      auto fetch = [&](int col, float (&v)[kEc]) {
        __syncwarp();  // tcgen05.ld is warp-collective: reconverge first
        if (p.splits == 1) {
          uint32_t r[kEc];
          tmem_ld16(trow + col, r);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < kEc; ++e) v[e] = __uint_as_float(r[e]);
        } else {
#pragma unroll
          for (int e = 0; e < kEc; ++e) v[e] = 0.f;
          for (int sp = 0; sp < p.splits; ++sp) {
            const float4 *src = reinterpret_cast<const float4 *>(
                p.partials + ((static_cast<size_t>(sp) * p.grid_m + un.tt) * p.grid_n + un.ft) * (128 * kBT) +
                frow * kBT + col);
#pragma unroll
            for (int e = 0; e < kEc / 4; ++e) {
              const float4 t = __ldcg(src + e);
              v[4 * e] += t.x;
              v[4 * e + 1] += t.y;
              v[4 * e + 2] += t.z;
              v[4 * e + 3] += t.w;
            }
          }
        }
      };
      if (!p.glu) {
        const int64_t n = static_cast<int64_t>(un.ft) * kPackRows + frow;
        const bool nvalid = n < p.N;
        const float bn = (p.bias && nvalid) ? p.bias[n] : 0.f;
        for (int col = 0; col < kBT; col += kEc) {
          float v[kEc];
          fetch(col, v);
          const int valid = p.M - (m0 + col);
          if (!nvalid || valid <= 0) continue;
          const int64_t off = static_cast<int64_t>(m0 + col) * p.ldy + n;
          const int sel = p.epi * 2 + p.y_dtype;
          switch (sel) {
            case kEpiNone * 2 + 0: store_col<float, kEpiNone>(static_cast<float *>(p.y) + off, p.ldy, valid, v, bn); break;
            case kEpiNone * 2 + 1: store_col<__nv_bfloat16, kEpiNone>(static_cast<__nv_bfloat16 *>(p.y) + off, p.ldy, valid, v, bn); break;
            case kEpiSilu * 2 + 0: store_col<float, kEpiSilu>(static_cast<float *>(p.y) + off, p.ldy, valid, v, bn); break;
            case kEpiSilu * 2 + 1: store_col<__nv_bfloat16, kEpiSilu>(static_cast<__nv_bfloat16 *>(p.y) + off, p.ldy, valid, v, bn); break;
            case kEpiGeluErf * 2 + 0: store_col<float, kEpiGeluErf>(static_cast<float *>(p.y) + off, p.ldy, valid, v, bn); break;
            case kEpiGeluErf * 2 + 1: store_col<__nv_bfloat16, kEpiGeluErf>(static_cast<__nv_bfloat16 *>(p.y) + off, p.ldy, valid, v, bn); break;
            case kEpiRelu * 2 + 0: store_col<float, kEpiRelu>(static_cast<float *>(p.y) + off, p.ldy, valid, v, bn); break;
            default: store_col<__nv_bfloat16, kEpiRelu>(static_cast<__nv_bfloat16 *>(p.y) + off, p.ldy, valid, v, bn); break;
          }
        }
      } else {
        // GLU tile: lanes [0, 64) value rows, [64, 128) their gate rows.
        const bool is_gate = frow >= 64;
        const int vrow = frow & 63;
        const int64_t jcol = static_cast<int64_t>(un.ft) * 64 + vrow;
        const bool jvalid = jcol < p.n_out;
        const float bv = (p.bias && jvalid) ? p.bias[is_gate ? p.n_out + jcol : jcol] : 0.f;
        for (int col = 0; col < kBT; col += kEc) {
          float v[kEc];
          fetch(col, v);
          if (is_gate) {
#pragma unroll
            for (int e = 0; e < kEc; ++e) glu_s[vrow * kBT + col + e] = v[e] + bv;
          }
          named_bar_sync(1, 32 * kEpiWarps);
          const int valid = p.M - (m0 + col);
          if (!is_gate && jvalid && valid > 0) {
            const int64_t off = static_cast<int64_t>(m0 + col) * p.ldy + jcol;
            const float *gate = glu_s + vrow * kBT + col;
            if (p.epi == kEpiGluSigmoid) {
              if (p.y_dtype == 0) store_glu<float, kEpiGluSigmoid>(static_cast<float *>(p.y) + off, p.ldy, valid, v, bv, gate);
              else store_glu<__nv_bfloat16, kEpiGluSigmoid>(static_cast<__nv_bfloat16 *>(p.y) + off, p.ldy, valid, v, bv, gate);
            } else {
              if (p.y_dtype == 0) store_glu<float, kEpiGluSilu>(static_cast<float *>(p.y) + off, p.ldy, valid, v, bv, gate);
              else store_glu<__nv_bfloat16, kEpiGluSilu>(static_cast<__nv_bfloat16 *>(p.y) + off, p.ldy, valid, v, bv, gate);
            }
          }
          named_bar_sync(1, 32 * kEpiWarps);
        }
      }
      if (p.splits > 1) {
        if (et == 0) p.counters[un.tt * p.grid_n + un.ft] = 0;  // re-armed for the next call
      } else {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(accum_empty(b));
      }
    }
  } else {
    // ------------------------------------------------------------- dequant
    // Warp w: TMEM lane quarter q = w % 4 (weight rows 32q..32q+31) and 16-k
    // chunk c of each 64-wide k step (columns 8c..8c+7 of the A stage).
    // Warp w: TMEM lane quarter q = w % 4 (weight rows 32q..32q+31); the four
    // warps of a quarter take turns by k step: warp `sub` dequantizes whole
    // 64-wide steps g = sub (mod 4) into A stage `sub` (kStages == 4), so the
    // per-step handshake is amortized over 64 elements and each warp has four
    // MMA steps of time for its loads, conversion and TMEM store.
    static_assert(kStages == kConvWarps / 4, "one A stage per converter warp of a lane quarter");
    const int q = warp & 3;
    const int sub = (warp - kConvWarp0) >> 2;
    const int row = 32 * q + lane;
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + C::kACol + sub * 32;
    int G = 0;  // k steps of this CTA
    for (int u = blockIdx.x; u < n_units; u += gridDim.x) G += decode_unit(p, u).nk;
    int cu = blockIdx.x, ci = 0;
    Unit cun = decode_unit(p, cu < n_units ? cu : 0);
    auto cursor_ptr = [&]() {
      return p.w + (static_cast<size_t>(cun.ft) * p.kc_total + cun.kc0 + ci) * kTileBytes;
    };
    auto cursor_next = [&]() {
      if (++ci >= cun.nk) {
        ci = 0;
        cu += gridDim.x;
        if (cu < n_units) cun = decode_unit(p, cu);
      }
    };
    auto cursor_skip4 = [&]() {
#pragma unroll
      for (int t = 0; t < 4; ++t) cursor_next();
    };
    for (int t = 0; t < sub && t < G; ++t) cursor_next();
    WChunk64 cur, nxt;
    if (sub < G) {
      cur = load_wchunk64(cursor_ptr(), row);
      cursor_skip4();
    }
    bool ok = true;
    for (int g = sub; g < G; g += 4) {
      if (g + 4 < G) {  // prefetch this warp's next step
        nxt = load_wchunk64(cursor_ptr(), row);
        cursor_skip4();
      }
      uint32_t r[32];
      dequant64(cur, r);
      if (g >= kStages) {
        bool w_ok = mbar_wait(empty_bar(sub), ((g / kStages) - 1) & 1, p.ctl.wait_limit, flags);
        w_ok = __all_sync(0xffffffffu, w_ok);
        if (!w_ok) {
          if (lane == 0 && !flags[0]) report(p.ctl, flags, kDevTimeoutConsumer);
          ok = false;
          break;
        }
      }
      tc_fence_after();
      tmem_st32(taddr, r);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(full_a(sub));
      cur = nxt;
    }
    (void)ok;
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

int gemm_block_t(GemmVariant) { return kBT; }

size_t gemm_smem_bytes(GemmVariant v) {
  return v == kGemmBt128SplitX ? GemmCfg<true>::kSmemBytes : GemmCfg<false>::kSmemBytes;
}

template <bool SPLITX>
static cudaError_t launch_gemm_t(const CUtensorMap &a_hi, const CUtensorMap &a_lo, const GemmParams &p, int grid,
                                 cudaStream_t stream) {
  using C = GemmCfg<SPLITX>;
  auto kern = gemm_q8_sm100_kernel<SPLITX>;
  static bool attr_set[64] = {false};  // once per device (the attribute is per-context state)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set[dev] = true;
  }
  kern<<<grid, kGemmThreads, C::kSmemBytes, stream>>>(a_hi, a_lo, p);
  return cudaGetLastError();
}

cudaError_t launch_gemm(GemmVariant v, const CUtensorMap &a_hi, const CUtensorMap &a_lo, const GemmParams &p, int grid,
                        cudaStream_t stream) {
  return v == kGemmBt128SplitX ? launch_gemm_t<true>(a_hi, a_lo, p, grid, stream)
                               : launch_gemm_t<false>(a_hi, a_lo, p, grid, stream);
}

}  // namespace nq
