// nq8_chain.cu -- decode chain: the dependent M = 1 Q8_0 GEMV steps of one
// decoder token (projections, GLU, residual add + LayerNorm) in one
// cooperative launch.
//
// The op-by-op form of a decoder token (src/moonshine/decoder.rs through
// DecoderBackend::gemv / gemv_resadd_ln, src/moonshine/gpu_decoder.rs:67-70,
// kernels/moonshine_kernels.py:1039-1146) is a chain where every call needs
// the previous call's whole output vector.  Per call that is a GEMV launch and
// a reduce launch (nq8_gemv.cu), each waiting for its predecessor; the
// dependent launches, not the weight bytes, set the time.  Here one
// persistent grid (one CTA per SM) runs the whole chain, with a single
// device-side dependency per step:
//   producer warp (lane 0): streams the weight chunks of this CTA's tiles of
//     every step, in step order, into a deep ring of shared-memory stages
//     (cp.async.bulk).  Weights do not depend on the data, so the ring fills
//     with later steps' chunks while earlier steps wait on their inputs.
//   16 consumer warps = 4 k groups x 4 row warps.  Tile T of step s belongs
//     to CTA (T + rot_s) mod grid, which computes all of it: chunk c of the
//     tile goes to k group c % 4, whose warp r owns rows [32r, 32r + 32)
//     (ldmatrix + dequantize to bf16(d*q) + mma.m16n8k16, the K2 consumer of
//     nq8_gemv.cu).  Per step with tiles on this CTA the consumers wait until
//     the previous step's tiles are all complete (a counter in global memory,
//     bounded wait) and stage the step's input vector in shared memory with
//     one batched read -- for an input that is the LayerNorm of the previous
//     step's residual row, the LayerNorm is computed here, in every CTA that
//     needs it.  At the end of a tile the four k groups' sums meet in shared
//     memory (added in group order), the epilogue (bias / activation / GLU,
//     or the residual add) writes the tile's outputs, and the tile is counted
//     complete.
// Results are deterministic (fixed chunk order per k group, fixed group
// order); they differ from the op-by-op calls, which cut k across CTAs, by
// f32 summation order only.
// Counters re-arm themselves: a step's counter is zeroed by the CTA that
// completes the next step (by then every CTA that waited on it has passed),
// the last step's by its own completer.  All CTAs are co-resident
// (cooperative launch) and every wait is bounded; a role that gives up sets
// the device status word, and every wait in every CTA stops when it sees a
// status bit.
#include "nq8_common.cuh"
#include "nq8_kernels.h"
#include "nq8_sm100_pair.cuh"

namespace nq {
namespace {

constexpr int kGroups = 4;                                 // k groups per CTA
constexpr int kRowWarps = 4;                               // 32 rows each: a 128-row tile
constexpr int kConsumerWarps = kGroups * kRowWarps;        // 16
constexpr int kConsumers = 32 * kConsumerWarps;            // 512
constexpr int kChainThreads = 32 + kConsumers;             // + producer warp
constexpr int kChainStages = 20;
constexpr int kLnPer = kChainMaxLnN / kConsumers;          // residual values per thread
constexpr int kXVecPer = kChainMaxK / 8 / kConsumers;      // 16-byte input vectors per thread
constexpr size_t kOffX = static_cast<size_t>(kChainStages) * kTileBytes;  // bf16 [kChainMaxK]
constexpr size_t kOffG = kOffX + kChainMaxK * 2;                           // f32 [kGroups][128] group sums
constexpr size_t kOffTot = kOffG + kGroups * kPackRows * 4;               // f32 [128] tile sums
constexpr size_t kOffRed = kOffTot + kPackRows * 4;                        // f32 [2][16] LayerNorm warp sums
constexpr size_t kOffBars = kOffRed + 2 * kConsumerWarps * 4;              // full, empty
constexpr size_t kOffPBar = kOffBars + 2 * kChainStages * 8;               // cluster partials barrier
constexpr size_t kOffPSlot = kOffPBar + 8;                                 // f32 [kCluster - 1][128]
constexpr size_t kOffFlags = kOffPSlot + (kChainCluster - 1) * kPackRows * 4;  // int [4] flags, int [16] votes
constexpr size_t kChainSmem = kOffFlags + (4 + kConsumerWarps) * 4;
constexpr int kConsumerBar = 1;  // named barrier of the consumer warps
// Drain limit: a CTA leaves only when its bulk copies have landed, which
// needs no other CTA, so it does not follow the (test-lowered) wait limit.
constexpr long long kDrainLimit = 1LL << 31;
static_assert(kChainMaxLnN % kConsumers == 0 && (kChainMaxK / 8) % kConsumers == 0, "staging split");

__device__ __forceinline__ bool status_set(const DevCtl &ctl) { return *static_cast<volatile int *>(ctl.status) != 0; }

// mbarrier wait bounded by ctl.wait_limit; also gives up when this CTA's
// abort flag or any device status bit is set.
__device__ __forceinline__ bool chain_wait(uint32_t bar, uint32_t parity, const DevCtl &ctl, volatile int *abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (*abort || status_set(ctl)) return false;
    if (clock64() - t0 > ctl.wait_limit) return false;
  }
}

__device__ __forceinline__ int ld_acquire(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until *cnt >= target (other CTAs' releases), bounded like chain_wait.
__device__ bool wait_count(const int *cnt, int target, const DevCtl &ctl, volatile int *abort) {
  long long t0 = 0;
  for (int it = 0;; ++it) {
    if (ld_acquire(cnt) >= target) return true;
    if (*abort || status_set(ctl)) return false;
    if (it == 0) {
      t0 = clock64();
    } else if (clock64() - t0 > ctl.wait_limit) {
      return false;
    }
    if (it > 256) __nanosleep(64);
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// c = -1152 * d exactly in f32, from the f16 bits of d (as nq8_gemv.cu).
__device__ __forceinline__ float neg1152(uint16_t d16) {
  float c;
  asm("{\n\t.reg .f16 dd, m;\n\tmov.b16 dd, %1;\n\tmov.b16 m, 0xE480;\n\tfma.rn.f32.f16 %0, dd, m, 0f00000000;\n\t}"
      : "=f"(c)
      : "h"(d16));
  return c;
}

// The first tile of step st this CTA works on, and the tile stride: split
// steps go to clusters (all ranks of a cluster on the same tile), the other
// steps to single CTAs.
__device__ __forceinline__ int first_tile(const ChainStep &st, int cta, int grid) {
  const int owner = st.split ? cta / kChainCluster : cta;
  const int owners = st.split ? grid / kChainCluster : grid;
  int t = (owner - st.rot) % owners;
  return t < 0 ? t + owners : t;
}
__device__ __forceinline__ int tile_stride(const ChainStep &st, int grid) {
  return st.split ? grid / kChainCluster : grid;
}

// try_wait with cluster-scope acquire: the arrivals are releases of other
// CTAs of the cluster, after their stores to this CTA's shared memory.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ bool wait_partials(uint32_t bar, uint32_t parity, const DevCtl &ctl, volatile int *abort) {
  long long t0 = 0;
  for (int it = 0;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort || status_set(ctl)) return false;
    if (it == 0) {
      t0 = clock64();
    } else if (clock64() - t0 > ctl.wait_limit) {
      return false;
    }
  }
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// LayerNorm of a residual step's row (f32 res_out[0, N)), mean and biased
// variance in f32 with fixed-order sums, into xs as bf16 (and gout when set).
// One batched read of the row per thread.
__device__ void ln_stage(const ChainStep &rs, __nv_bfloat16 *xs, float *red, __nv_bfloat16 *gout) {
  const int ct = threadIdx.x - 32, cw = ct >> 5, lane = ct & 31;
  const int N = static_cast<int>(rs.N);
  float v[kLnPer];
#pragma unroll
  for (int i = 0; i < kLnPer; ++i) {
    const int n = ct + i * kConsumers;
    v[i] = n < N ? __ldcg(rs.res_out + n) : 0.f;
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kLnPer; ++i) s += v[i];
  s = warp_sum(s);
  if (lane == 0) red[cw] = s;
  named_bar_sync(kConsumerBar, kConsumers);
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) tot += red[w];
  const float mean = tot / static_cast<float>(N);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kLnPer; ++i) {
    const int n = ct + i * kConsumers;
    const float d = n < N ? v[i] - mean : 0.f;
    q += d * d;
  }
  q = warp_sum(q);
  if (lane == 0) red[kConsumerWarps + cw] = q;
  named_bar_sync(kConsumerBar, kConsumers);
  float qt = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) qt += red[kConsumerWarps + w];
  const float rstd = rsqrtf(qt / static_cast<float>(N) + rs.ln_eps);
#pragma unroll
  for (int i = 0; i < kLnPer; ++i) {
    const int n = ct + i * kConsumers;
    if (n < N) {
      const __nv_bfloat16 o = __float2bfloat16_rn((v[i] - mean) * rstd * rs.ln_g[n] + (rs.ln_b ? rs.ln_b[n] : 0.f));
      xs[n] = o;
      if (gout) gout[n] = o;
    }
  }
}

// A plain input vector into xs: 16-byte loads when aligned, all issued
// before any is used.
__device__ void x_stage(const ChainStep &st, __nv_bfloat16 *xs) {
  const int ct = threadIdx.x - 32;
  if ((reinterpret_cast<uintptr_t>(st.x) & 15) == 0 && (st.K & 7) == 0) {
    const uint4 *src = reinterpret_cast<const uint4 *>(st.x);
    const int nv = st.K >> 3;
    uint4 v[kXVecPer];
#pragma unroll
    for (int i = 0; i < kXVecPer; ++i) {
      const int e = ct + i * kConsumers;
      v[i] = e < nv ? __ldcg(src + e) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < kXVecPer; ++i) {
      const int e = ct + i * kConsumers;
      if (e < nv) reinterpret_cast<uint4 *>(xs)[e] = v[i];
    }
  } else {
    const unsigned short *src = reinterpret_cast<const unsigned short *>(st.x);
    unsigned short *dst = reinterpret_cast<unsigned short *>(xs);
    for (int k = ct; k < st.K; k += kConsumers) dst[k] = __ldcg(src + k);
  }
}

__global__ void __launch_bounds__(kChainThreads, 1) chain_kernel(const __grid_constant__ ChainParams p) {
  constexpr int S = kChainStages;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *ring = smem;
  __nv_bfloat16 *xs = reinterpret_cast<__nv_bfloat16 *>(smem + kOffX);
  float *gsum = reinterpret_cast<float *>(smem + kOffG);
  float *tot = reinterpret_cast<float *>(smem + kOffTot);
  float *red = reinterpret_cast<float *>(smem + kOffRed);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kOffBars);
  uint64_t *pbar = reinterpret_cast<uint64_t *>(smem + kOffPBar);  // rank 0: the other ranks' partials landed
  float *pslot = reinterpret_cast<float *>(smem + kOffPSlot);      // rank 0: [rank - 1][128] partial tile sums
  const uint32_t rank = cluster_ctarank();
  // [0] abort (any role of this CTA)  [1] input ready  [2] tile count
  volatile int *flags = reinterpret_cast<volatile int *>(smem + kOffFlags);
  volatile int *vote = flags + 4;  // [16] per consumer warp: its part of the tile completed
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x, grid = gridDim.x;
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[S + s]); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), kRowWarps);  // the k group's four warps
    }
    mbar_init(smem_u32(pbar), (kChainCluster - 1) * kPackRows);  // one arrival per row of each other rank
    flags[0] = 0;
    fence_mbar_init();
  }
  __syncthreads();
  cluster_sync_all();  // every CTA's barriers exist before a remote arrive

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      const uint64_t pol = policy_evict_first();
      int s = 0, issued = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int si = 0; si < p.n_steps && ok; ++si) {
        const ChainStep &st = p.steps[si];
        const int c0 = st.split ? static_cast<int>(rank) : 0, cstep = st.split ? kChainCluster : 1;
        for (int T = first_tile(st, cta, grid); T < st.n_tiles && ok; T += tile_stride(st, grid)) {
          for (int ch = c0; ch < st.kc; ch += cstep) {
            const uint8_t *src = st.w + (static_cast<size_t>(T) * st.kc + ch) * kTileBytes;
            if (issued >= S && !chain_wait(empty_bar(s), ph ^ 1u, p.ctl, flags)) {
              if (!flags[0]) report(p.ctl, flags, kDevTimeoutProducer);
              ok = false;
              break;
            }
            // order the consumers' shared reads of the stage before the refill
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(full_bar(s), kTileBytes);
            bulk_load(smem_u32(ring + s * kTileBytes), src, kTileBytes, full_bar(s), pol);
            ++issued;
            if (++s == S) {
              s = 0;
              ph ^= 1u;
            }
          }
        }
      }
      // Drain: every issued copy has landed before the CTA leaves.
      volatile int no_abort = 0;
      for (int st = 0; st < S && st < issued; ++st) {
        const int last = st + S * ((issued - 1 - st) / S);
        if (!mbar_wait(full_bar(st), (last / S) & 1, kDrainLimit, &no_abort)) atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int ct = threadIdx.x - 32;
    const int cw = ct >> 5;          // 0..15
    const int grp = cw / kRowWarps;  // k group
    const int rw = cw % kRowWarps;   // rows [32 rw, 32 rw + 32) of the tile
    const int g4 = lane >> 2;
    const int c = lane & 3;
    const bool live = g4 == 0;  // row m = 0 of the 8-column operand (M = 1)
    uint32_t lofs[4], sofs[4][2];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      lofs[b] = qs_offset(32 * rw + 8 * b + (lane & 7), lane >> 3);
      sofs[b][0] = scale_offset(32 * rw + 8 * b + g4, 0);
      sofs[b][1] = scale_offset(32 * rw + 8 * b + g4, 1);
    }
    int q = 0;       // chunk sequence number of this CTA (stage q % S)
    int nsplit = 0;  // split tiles this CTA has worked on (rank 0: phase of pbar)
    bool ok = true;
    for (int si = 0; si < p.n_steps && ok; ++si) {
      const ChainStep &st = p.steps[si];
      int T = first_tile(st, cta, grid);
      if (T >= st.n_tiles) continue;  // no tile of this step here
      // The previous step's output is complete, then this step's input is
      // staged in shared memory (k beyond K zero).
      if (si > 0) {
        // One thread observes the completion (an acquire load); the CTA
        // barrier then orders every consumer's reads after it.
        if (ct == 0) {
          const bool got = wait_count(&p.ready[si - 1], p.steps[si - 1].n_tiles, p.ctl, flags);
          if (!got && !flags[0]) report(p.ctl, flags, kDevTimeoutConsumer);
          flags[1] = got ? 1 : 0;
        }
        named_bar_sync(kConsumerBar, kConsumers);
        ok = flags[1] != 0;
        if (!ok) break;
      }
      const int kpad = st.kc * kPackK;
      int kin;
      if (st.x_ln) {
        const ChainStep &rs = p.steps[si - 1];
        // the CTA of tile 0 also stores the LayerNorm output for later readers
        ln_stage(rs, xs, red, T == 0 && rank == 0 ? static_cast<__nv_bfloat16 *>(rs.y) : nullptr);
        kin = static_cast<int>(rs.N);
      } else {
        x_stage(st, xs);
        kin = st.K;
      }
      for (int k = kin + ct; k < kpad; k += kConsumers) xs[k] = __float2bfloat16_rn(0.f);
      named_bar_sync(kConsumerBar, kConsumers);
      const int c0 = st.split ? static_cast<int>(rank) : 0, cstep = st.split ? kChainCluster : 1;
      for (; T < st.n_tiles && ok; T += tile_stride(st, grid)) {
        float acc[2][4];
#pragma unroll
        for (int gi = 0; gi < 2; ++gi)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[gi][e] = 0.f;
        // A warp that gives up stops consuming but still reaches the tile's
        // barrier, where the warps vote and leave together (named barriers
        // have no time limit).
        bool wok = true;
        for (int ch = c0, idx = 0; ch < st.kc; ch += cstep, ++idx, ++q) {
          if (idx % kGroups != grp || !wok) continue;
          const int stg = q % S;
          bool got = chain_wait(full_bar(stg), (q / S) & 1, p.ctl, flags);
          got = __all_sync(0xffffffffu, got);
          if (!got) {
            if (lane == 0 && !flags[0]) report(p.ctl, flags, kDevTimeoutConsumer);
            wok = false;
            continue;
          }
          const uint8_t *sp = ring + stg * kTileBytes;
          const uint32_t sa = smem_u32(sp);
          uint32_t R[4][4];
#pragma unroll
          for (int b = 0; b < 4; ++b) ldsm_x4(sa + lofs[b], R[b]);
          uint16_t dv[4][2];
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            dv[b][0] = *reinterpret_cast<const uint16_t *>(sp + sofs[b][0]);
            dv[b][1] = *reinterpret_cast<const uint16_t *>(sp + sofs[b][1]);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(empty_bar(stg));
          uint2 xc[4];
#pragma unroll
          for (int qq = 0; qq < 4; ++qq)
            xc[qq] = live ? *reinterpret_cast<const uint2 *>(xs + ch * kPackK + 16 * qq + 4 * c) : make_uint2(0u, 0u);
#pragma unroll
          for (int gi = 0; gi < 2; ++gi) {
            const int ba = 2 * gi, bb = 2 * gi + 1;
            const float ca[2] = {neg1152(dv[ba][0]), neg1152(dv[ba][1])};
            const float cb[2] = {neg1152(dv[bb][0]), neg1152(dv[bb][1])};
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
              uint32_t a[4];
              dequant4_bf16_mix(R[ba][qq], dv[ba][qq >> 1], ca[qq >> 1], a[0], a[2]);
              dequant4_bf16_mix(R[bb][qq], dv[bb][qq >> 1], cb[qq >> 1], a[1], a[3]);
              mma_16816_bf16(acc[gi], a, xc[qq].x, xc[qq].y);
            }
          }
        }
        // this k group's sums of the warp's rows (column m = 0)
        if (c == 0) {
#pragma unroll
          for (int gi = 0; gi < 2; ++gi) {
            const int ra = 32 * rw + 16 * gi + g4;
            gsum[grp * kPackRows + ra] = acc[gi][0];
            gsum[grp * kPackRows + ra + 8] = acc[gi][2];
          }
        }
        if (lane == 0) vote[cw] = wok ? 1 : 0;
        named_bar_sync(kConsumerBar, kConsumers);
        bool all = true;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) all = all && vote[w] != 0;
        ok = all;
        if (!ok) break;  // every consumer warp read the same votes
        // tile T: thread r < 128 owns row r; this CTA's sum of the row
        float t = 0.f;
        if (ct < kPackRows) {
          t = gsum[ct];
#pragma unroll
          for (int g = 1; g < kGroups; ++g) t += gsum[g * kPackRows + ct];
        }
        if (st.split) {
          const int par = nsplit & 1;
          ++nsplit;
          if (rank != 0) {
            // hand the partial to rank 0 and go on; rank 0 finishes the tile
            // (each row's thread releases its own store with its arrival)
            if (ct < kPackRows) {
              st_cluster_f32(map_rank(smem_u32(&pslot[(rank - 1) * kPackRows + ct]), 0), t);
              mbar_arrive_remote(map_rank(smem_u32(pbar), 0));
            }
            continue;
          }
          if (ct < kPackRows && !wait_partials(smem_u32(pbar), par, p.ctl, flags) && !flags[0])
            report(p.ctl, flags, kDevTimeoutConsumer);
          named_bar_sync(kConsumerBar, kConsumers);
          if (flags[0]) {
            ok = false;
            break;
          }
          if (ct < kPackRows) {
#pragma unroll
            for (int rk = 1; rk < kChainCluster; ++rk) t += pslot[(rk - 1) * kPackRows + ct];
          }
        }
        // epilogue of tile T
        if (ct < kPackRows) {
          const int r = ct;
          const int64_t n = static_cast<int64_t>(T) * kPackRows + r;
          if (st.res_out) {
            if (n < st.N) {
              float a = t;
              if (st.bias) a += st.bias[n];
              a += st.res_in[n];
              st.res_out[n] = a;
            }
          } else if (st.glu) {
            tot[r] = t;
          } else if (n < st.N) {
            if (st.bias) t += st.bias[n];
            store_out(st.y, st.y_dtype, n, act_single(st.epi, t));
          }
        }
        if (st.glu) {
          named_bar_sync(kConsumerBar, kConsumers);
          const int64_t j = static_cast<int64_t>(T) * 64 + ct;
          if (ct < 64 && j < st.n_out) {
            float v = tot[ct], gt = tot[64 + ct];
            if (st.bias) {
              v += st.bias[j];
              gt += st.bias[st.n_out + j];
            }
            store_out(st.y, st.y_dtype, j, act_glu(st.epi, v, gt));
          }
        }
        // The tile's outputs are written: after the CTA barrier, one fence
        // (cumulative over the CTA's writes) and the count.
        named_bar_sync(kConsumerBar, kConsumers);
        if (ct == 0) {
          __threadfence();
          const int old = atomicAdd(&p.ready[si], 1);
          flags[2] = old;
          if (old == st.n_tiles - 1) {
            __threadfence();  // acquire: the other CTAs' outputs of this step are visible
            // Step complete.  Every CTA that waited on the previous step's
            // counter has passed it (its tiles of this step are done): re-arm.
            if (si > 0) atomicExch(&p.ready[si - 1], 0);
            if (si == p.n_steps - 1) atomicExch(&p.ready[si], 0);
          }
        }
        named_bar_sync(kConsumerBar, kConsumers);
        // The last step's LayerNorm output has no next step to write it.
        if (flags[2] == st.n_tiles - 1 && si == p.n_steps - 1 && st.res_out && st.y)
          ln_stage(st, xs, red, static_cast<__nv_bfloat16 *>(st.y));
      }
    }
  }
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while a peer may still signal it
}

}  // namespace

size_t chain_smem_bytes() { return kChainSmem; }
int chain_threads() { return kChainThreads; }

cudaError_t chain_max_ctas(int sm_count, int *ctas) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !attr_set[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kChainSmem));
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set[dev] = true;
  }
  (void)sm_count;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kChainCluster * 64);
  cfg.blockDim = dim3(kChainThreads);
  cfg.dynamicSmemBytes = kChainSmem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kChainCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, chain_kernel, &cfg);
  if (e != cudaSuccess) return e;
  *ctas = clusters * kChainCluster;
  return *ctas > 0 ? cudaSuccess : cudaErrorInvalidConfiguration;
}

cudaError_t launch_chain(const ChainParams &p, int ctas, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(kChainThreads);
  cfg.dynamicSmemBytes = kChainSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: they wait on one another
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = kChainCluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, chain_kernel, p);
  if (e == cudaSuccess) note_launch();
  return e;
}

}  // namespace nq
