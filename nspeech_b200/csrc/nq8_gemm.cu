// nq8_gemm.cu -- K1: tcgen05/TMEM Q8_0 GEMM for M > 16 (sm_100a).
//
// Replaces the tiled matmul family of the reference (Triton source
// kernels/moonshine_kernels.py:20-299, dispatched by triton_matmul*/enc_matmul*
// in src/triton_kernels.rs:170-309,1205-1289; CPU FbgemmBf16Op in
// src/fast_matmul.rs:138-167).
//
// C[M, N] = act(A[M, K] . bf16(dequant(W[N, K]))^T + bias), one 128 x BN tile
// per CTA (optionally split over K), 10 warps:
//   warp 0   producer: TMA 2-D load of the activation tile (bf16, 128-byte
//            swizzle) and one cp.async.bulk per 128-row packed weight tile
//            (int8 + f16 scales, raw) into stage s; mbarrier full[s] with tx.
//   warp 1   allocates BN TMEM columns; lane 0 issues tcgen05.mma
//            (M=128, N=BN, K=16, kind::f16, bf16 x bf16 -> f32 in TMEM) and
//            commits to empty[s] (stage reusable) and, at the end, accum.
//   warps 2-9 dequant: raw stage -> bf16(f32(d) * q) written into the
//            K-major SWIZZLE_128B operand layout the MMA reads, then
//            fence.proxy.async + arrive bready[s].  After the main loop they
//            run the epilogue: tcgen05.ld 32 lanes x 32 columns, bias,
//            SiLU / GELU-erf / GLU, f32 or bf16 stores.
// f32 activations arrive as two bf16 planes (hi, lo) and are issued as two
// MMAs per k step.  Every wait is bounded; on give-up the kernel records a
// status bit, drains in-flight copies and MMAs, frees TMEM and returns.
// No cluster multicast anywhere.
#include "nq8_common.cuh"
#include "nq8_kernels.h"

namespace nq {

constexpr int kGemmThreads = 320;
constexpr int kConvWarps = 8;
constexpr int kABytes = 128 * kPackK * 2;  // 16 KB

template <int BN, int STAGES, bool SPLITX>
struct GemmCfg {
  static constexpr int kPacks = BN / kPackRows;
  static constexpr int kBBytes = BN * kPackK * 2;
  static constexpr int kRawBytes = ((kPacks * kTileBytes + 1023) / 1024) * 1024;
  static constexpr int kStageBytes = kABytes * (SPLITX ? 2 : 1) + kBBytes + kRawBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kSmemBytes = 1024 /*align slack*/ + kBarOffset + 256;
  static constexpr uint32_t kIdesc = idesc_bf16_f32(128, BN);
  static constexpr int kTmemCols = BN;  // power of two >= 32
};

template <int BN, int STAGES, bool SPLITX>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_q8_sm100_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_alo,
                         const __grid_constant__ GemmParams p) {
  using C = GemmCfg<BN, STAGES, SPLITX>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment of the swizzled operand tiles.
  const uint32_t raw_u32 = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bx = blockIdx.x, by = blockIdx.y, bz = blockIdx.z;
  const int pack0 = bx * C::kPacks;
  const int valid_packs = min(C::kPacks, p.n_tiles - pack0);
  const int m0 = by * 128;
  const int kc0 = bz * p.cps;
  const int nk = max(min(kc0 + p.cps, p.kc_total) - kc0, 0);

  auto stage_a = [&](int s) { return smem + s * C::kStageBytes; };
  auto stage_alo = [&](int s) { return smem + s * C::kStageBytes + kABytes; };
  auto stage_b = [&](int s) { return smem + s * C::kStageBytes + kABytes * (SPLITX ? 2 : 1); };
  auto stage_raw = [&](int s) { return stage_b(s) + C::kBBytes; };
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kBarOffset);
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto bready_bar = [&](int s) { return smem_u32(&bars[STAGES + s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[2 * STAGES + s]); };
  const uint32_t accum_bar = smem_u32(&bars[3 * STAGES]);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(&bars[3 * STAGES + 1]);
  volatile int *flags = reinterpret_cast<volatile int *>(&bars[3 * STAGES + 2]);  // [0] abort [1] last [2] mma_done

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(bready_bar(s), kConvWarps);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(accum_bar, 1);
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
      const uint64_t pol = policy_evict_last();  // weight tiles are re-read by other M tiles
      const uint32_t tx = kABytes * (SPLITX ? 2 : 1) + valid_packs * kTileBytes;
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        if (i >= STAGES) {
          if (!mbar_wait(empty_bar(s), ((i / STAGES) - 1) & 1, p.ctl.wait_limit, flags)) {
            if (!flags[0]) report(p.ctl, flags, kDevTimeoutProducer);
            break;
          }
        }
        if (flags[0]) break;
        const int kc = kc0 + i;
        mbar_arrive_expect_tx(full_bar(s), tx);
        tma_load_2d(smem_u32(stage_a(s)), &tm_a, full_bar(s), kc * kPackK, m0);
        if (SPLITX) tma_load_2d(smem_u32(stage_alo(s)), &tm_alo, full_bar(s), kc * kPackK, m0);
        for (int pk = 0; pk < valid_packs; ++pk) {
          const uint8_t *src = p.w + (static_cast<size_t>(pack0 + pk) * p.kc_total + kc) * kTileBytes;
          bulk_load(smem_u32(stage_raw(s) + pk * kTileBytes), src, kTileBytes, full_bar(s), pol);
        }
        ++issued;
      }
      volatile int no_abort = 0;
      for (int s = 0; s < STAGES && s < issued; ++s) {
        const int last = s + STAGES * ((issued - 1 - s) / STAGES);
        if (!mbar_wait(full_bar(s), (last / STAGES) & 1, p.ctl.wait_limit, &no_abort))
          atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issue
      int done = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t par = (i / STAGES) & 1;
        if (!mbar_wait(bready_bar(s), par, p.ctl.wait_limit, flags) ||
            !mbar_wait(full_bar(s), par, p.ctl.wait_limit, flags)) {
          if (!flags[0]) report(p.ctl, flags, kDevTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(stage_a(s));
        const uint32_t alo_addr = smem_u32(stage_alo(s));
        const uint32_t b_addr = smem_u32(stage_b(s));
#pragma unroll
        for (int kk = 0; kk < kPackK / 16; ++kk) {
          const uint64_t bdesc = sw128_kmajor_desc(b_addr + kk * 32);
          umma_bf16(tmem_base, sw128_kmajor_desc(a_addr + kk * 32), bdesc, C::kIdesc,
                    (i > 0 || kk > 0) ? 1u : 0u);
          if (SPLITX) umma_bf16(tmem_base, sw128_kmajor_desc(alo_addr + kk * 32), bdesc, C::kIdesc, 1u);
        }
        umma_commit(empty_bar(s));
        ++done;
      }
      if (done == nk && nk > 0) {
        umma_commit(accum_bar);
      } else if (done > 0) {
        // Aborted: wait for the MMAs already issued before TMEM is released.
        volatile int no_abort = 0;
        const int last = done - 1;
        if (!mbar_wait(empty_bar(last % STAGES), (last / STAGES) & 1, p.ctl.wait_limit, &no_abort))
          atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else {
    // ----------------------------------------------------------- dequant
    const int ct = threadIdx.x - 64;  // 0..255
    constexpr int kIters = (BN * kPackK / 16) / (32 * kConvWarps);
    for (int i = 0; i < nk; ++i) {
      const int s = i % STAGES;
      bool ok = mbar_wait(full_bar(s), (i / STAGES) & 1, p.ctl.wait_limit, flags);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0 && !flags[0]) report(p.ctl, flags, kDevTimeoutConsumer);
        break;
      }
      const uint8_t *raw = stage_raw(s);
      uint8_t *bt = stage_b(s);
#pragma unroll
      for (int it = 0; it < kIters; ++it) {
        const int q = it * 32 * kConvWarps + ct;
        const int r = q >> 2;      // B row (output column n within the CTA tile)
        const int c = q & 3;       // 16-byte chunk of the 64-byte raw row
        const int pk = r >> 7;
        const int rr = r & 127;
        const uint8_t *tile = raw + pk * kTileBytes;
        const uint4 v = *reinterpret_cast<const uint4 *>(tile + rr * kPackK + c * 16);
        const float d = __half2float(*reinterpret_cast<const __half *>(tile + kTileQsBytes + rr * 4 + (c >> 1) * 2));
        uint4 o0, o1;
        dequant4_bf16(v.x, d, o0.x, o0.y);
        dequant4_bf16(v.y, d, o0.z, o0.w);
        dequant4_bf16(v.z, d, o1.x, o1.y);
        dequant4_bf16(v.w, d, o1.z, o1.w);
        *reinterpret_cast<uint4 *>(bt + sw128_offset(r, 2 * c)) = o0;
        *reinterpret_cast<uint4 *>(bt + sw128_offset(r, 2 * c + 1)) = o1;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bready_bar(s));
    }

    // ---------------------------------------------------------- epilogue
    const int sub = warp & 3;          // TMEM lane quarter this warp may read
    const int chalf = (warp - 2) >> 2;  // which half of the columns
    const int row = m0 + 32 * sub + lane;
    const uint32_t trow = tmem_base + (static_cast<uint32_t>(32 * sub) << 16);
    bool ok = (nk > 0) && !flags[0];
    if (ok) ok = mbar_wait(accum_bar, 0, p.ctl.wait_limit, flags);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && nk > 0 && lane == 0 && !flags[0]) report(p.ctl, flags, kDevTimeoutEpilogue);
    tc_fence_after();
    const int64_t n_base = static_cast<int64_t>(pack0) * kPackRows;
    float *part = nullptr;
    if (p.splits > 1)
      part = p.partials + ((static_cast<size_t>(bz) * p.grid_m + by) * p.grid_n + bx) * (128 * BN);

    // Phase 1 (split-K): every CTA parks its raw accumulators; the last one
    // to arrive for this tile sums all splits in index order.
    if (p.splits > 1) {
      if (ok) {
        for (int col = chalf * (BN / 2); col < (chalf + 1) * (BN / 2); col += 32) {
          uint32_t r[32];
          tmem_ld32(trow + col, r);
          tmem_ld_wait();
          float4 *dst = reinterpret_cast<float4 *>(part + (32 * sub + lane) * BN + col);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            dst[e] = make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]),
                                 __uint_as_float(r[4 * e + 2]), __uint_as_float(r[4 * e + 3]));
        }
      }
      __threadfence();
      named_bar_sync(1, 32 * kConvWarps);
      if (threadIdx.x == 64) {
        const int prev = atomicAdd(&p.counters[by * p.grid_n + bx], 1);
        flags[1] = (prev == p.splits - 1) ? 1 : 0;
      }
      named_bar_sync(1, 32 * kConvWarps);
      ok = ok && flags[1];
      if (flags[1]) __threadfence();
    }

    // Fetch 32 accumulator columns of this thread's row: TMEM, or the
    // ordered sum of the split partials.
    auto fetch = [&](int col, float (&v)[32]) {
      if (p.splits == 1) {
        uint32_t r[32];
        tmem_ld32(trow + col, r);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0.f;
        for (int sp = 0; sp < p.splits; ++sp) {
          const float4 *src = reinterpret_cast<const float4 *>(
              p.partials + ((static_cast<size_t>(sp) * p.grid_m + by) * p.grid_n + bx) * (128 * BN) +
              (32 * sub + lane) * BN + col);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float4 t = __ldcg(src + e);
            v[4 * e] += t.x;
            v[4 * e + 1] += t.y;
            v[4 * e + 2] += t.z;
            v[4 * e + 3] += t.w;
          }
        }
      }
    };

    if (ok) {
      if (!p.glu) {
        for (int col = chalf * (BN / 2); col < (chalf + 1) * (BN / 2); col += 32) {
          float v[32];
          fetch(col, v);
          if (row < p.M) {
            const int64_t n0 = n_base + col;
            if (p.y_dtype == 0 && n0 + 32 <= p.N && (p.ldy & 3) == 0) {
              float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.y) + row * p.ldy + n0);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                float t[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  float a = v[4 * e + u];
                  if (p.bias) a += p.bias[n0 + 4 * e + u];
                  t[u] = act_single(p.epi, a);
                }
                dst[e] = make_float4(t[0], t[1], t[2], t[3]);
              }
            } else if (p.y_dtype == 1 && n0 + 32 <= p.N && (p.ldy & 7) == 0) {
              uint4 *dst = reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(p.y) + row * p.ldy + n0);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                uint32_t w4[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  float a0 = v[8 * e + 2 * u], a1 = v[8 * e + 2 * u + 1];
                  if (p.bias) {
                    a0 += p.bias[n0 + 8 * e + 2 * u];
                    a1 += p.bias[n0 + 8 * e + 2 * u + 1];
                  }
                  w4[u] = pack_bf16x2(act_single(p.epi, a0), act_single(p.epi, a1));
                }
                dst[e] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
              }
            } else {
              for (int e = 0; e < 32; ++e) {
                const int64_t n = n0 + e;
                if (n < p.N) {
                  float a = v[e];
                  if (p.bias) a += p.bias[n];
                  store_out(p.y, p.y_dtype, row * p.ldy + n, act_single(p.epi, a));
                }
              }
            }
          }
        }
      } else {
        // GLU tiles: columns [0,64) value and [64,128) gate of each 128-column pack.
        for (int ci = chalf; ci < C::kPacks * 2; ci += 2) {
          const int pk = ci >> 1;
          const int cc = (ci & 1) * 32;
          float v[32], gt[32];
          fetch(pk * 128 + cc, v);
          fetch(pk * 128 + 64 + cc, gt);
          if (row < p.M) {
            const int64_t j0 = static_cast<int64_t>(pack0 + pk) * 64 + cc;
            for (int e = 0; e < 32; ++e) {
              const int64_t j = j0 + e;
              if (j < p.n_out) {
                float a = v[e], g = gt[e];
                if (p.bias) {
                  a += p.bias[j];
                  g += p.bias[p.n_out + j];
                }
                store_out(p.y, p.y_dtype, row * p.ldy + j, act_glu(p.epi, a, g));
              }
            }
          }
        }
      }
    }
    if (p.splits > 1 && flags[1] && threadIdx.x == 64) p.counters[by * p.grid_n + bx] = 0;
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::kTmemCols);
}

// Tile configurations compiled into the library.
using Cfg256 = GemmCfg<256, 3, false>;
using Cfg128 = GemmCfg<128, 4, false>;
using Cfg128X = GemmCfg<128, 3, true>;

int gemm_block_n(GemmVariant v) { return v == kGemmBn256 ? 256 : 128; }

size_t gemm_smem_bytes(GemmVariant v) {
  switch (v) {
    case kGemmBn256: return Cfg256::kSmemBytes;
    case kGemmBn128: return Cfg128::kSmemBytes;
    default: return Cfg128X::kSmemBytes;
  }
}

template <int BN, int STAGES, bool SPLITX>
static cudaError_t launch_gemm_t(const CUtensorMap &a_hi, const CUtensorMap &a_lo, const GemmParams &p,
                                 cudaStream_t stream) {
  using C = GemmCfg<BN, STAGES, SPLITX>;
  auto kern = gemm_q8_sm100_kernel<BN, STAGES, SPLITX>;
  static bool attr_set[64] = {false};  // once per device (the attribute is per-context state)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set[dev] = true;
  }
  dim3 grid(p.grid_n, p.grid_m, p.splits);
  kern<<<grid, kGemmThreads, C::kSmemBytes, stream>>>(a_hi, a_lo, p);
  return cudaGetLastError();
}

cudaError_t launch_gemm(GemmVariant v, const CUtensorMap &a_hi, const CUtensorMap &a_lo, const GemmParams &p,
                        cudaStream_t stream) {
  switch (v) {
    case kGemmBn256: return launch_gemm_t<256, 3, false>(a_hi, a_lo, p, stream);
    case kGemmBn128: return launch_gemm_t<128, 4, false>(a_hi, a_lo, p, stream);
    default: return launch_gemm_t<128, 3, true>(a_hi, a_lo, p, stream);
  }
}

}  // namespace nq
