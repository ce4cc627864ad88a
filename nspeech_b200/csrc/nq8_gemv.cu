// nq8_gemv.cu -- K2: persistent split-K Q8_0 GEMV / skinny GEMM (M <= 16).
//
// Replaces the split-K GEMV family of the reference (Triton source
// kernels/moonshine_kernels.py:1039-1276, dispatched by enc_gemv_splitk*,
// src/triton_kernels.rs:1036-1202) and the M=1 decoder projections of
// src/moonshine/decoder.rs.  HBM-bound: every weight byte is read once.
//
// Work: the weight tiles of up to three problems sharing x (fused Q/K/V) form
// one list; K is cut into `splits` ranges of cps 64-wide chunks.  CTA c owns
// split c % splits and walks tiles c / splits, + tgroups, ... (persistent:
// one continuous copy stream per CTA, so launch and prologue costs are paid
// once per CTA rather than per tile).  CTA = 1 producer warp + 8 consumer
// warps:
//   producer: cp.async.bulk of whole 8704-byte packed tiles into a ring of
//             kStages shared-memory slots, chunk after chunk across the CTA's
//             tiles; a proxy fence orders the consumers' shared reads of a
//             slot before the copy that refills it.
//   consumers: the CTA's activation slice [M][cps*64] is staged once (bf16,
//             hi + lo planes for f32 x, k order permuted to match the lanes'
//             weight bytes).  Warp w owns rows [16w, 16w+16) of each tile:
//             each lane loads 16 int8 of two rows, dequantizes them to
//             bf16(d*q) and issues mma.m16n8k16 with the weight as the 16-row
//             operand and the activations as the 8-column operand.
//   per tile: the accumulators go through shared memory; with split-K they
//             become f32 partials [split][tile][M][128] and the last CTA of a
//             tile (arrival counter) sums the splits in index order
//             (deterministic); then bias / activation / GLU and the store.
// Every wait is bounded; a consumer that gives up keeps taking part in the
// per-tile barriers (skipping work) until the CTA leaves together.
#include "nq8_common.cuh"
#include "nq8_kernels.h"

namespace nq {

constexpr int kGemvStages = 6;
constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvConsumers = 32 * kGemvConsumerWarps;
constexpr int kGemvThreads = 32 + kGemvConsumers;
constexpr int kAccPitch = 132;           // floats per row of the staged accumulator tile
constexpr int kGemvXStageBytes = 16384;  // activation slice budget (per plane set)
constexpr int kGemvBarEpi = 1;           // named barrier of the consumer warps

static __host__ __device__ inline int gemv_x_pitch(int cps) { return cps * kPackK * 2 + 8; }  // bytes

int gemv_max_cps(int m, bool splitx) {
  const int mrows = m <= 8 ? 8 : 16;
  return kGemvXStageBytes / (mrows * kPackK * 2 * (splitx ? 2 : 1));
}

size_t gemv_smem_bytes(int mrows, bool splitx, int cps) {
  size_t off = static_cast<size_t>(kGemvStages) * kTileBytes;                  // ring
  off += static_cast<size_t>(mrows) * gemv_x_pitch(cps) * (splitx ? 2 : 1);    // x planes
  off = (off + 15) & ~static_cast<size_t>(15);
  off += static_cast<size_t>(16) * kAccPitch * sizeof(float);                  // accumulator tile
  off += 2 * kGemvStages * sizeof(uint64_t) + 16;                              // barriers + flags
  return off;
}

template <int MT, bool SPLITX>
__global__ void __launch_bounds__(kGemvThreads) gemv_q8_kernel(const __grid_constant__ GemvParams p) {
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  constexpr int MROWS = 8 * MT;
  extern __shared__ __align__(128) uint8_t smem[];
  const int split = blockIdx.x % p.splits;
  const int tg0 = blockIdx.x / p.splits;
  const int t1 = p.prob[0].n_tiles, t2 = t1 + p.prob[1].n_tiles;
  const int total_tiles = t2 + (p.nprob > 2 ? p.prob[2].n_tiles : 0);
  const int kc0 = split * p.cps;
  const int nchunks = max(min(kc0 + p.cps, p.prob[0].kc_total) - kc0, 0);
  if (tg0 >= total_tiles || nchunks == 0) return;  // whole CTA, before any barrier is touched
  const int xpitch = gemv_x_pitch(p.cps);

  uint8_t *ring = smem;
  uint8_t *xs = smem + kGemvStages * kTileBytes;
  const int xplane = MROWS * xpitch;
  size_t off = static_cast<size_t>(kGemvStages) * kTileBytes + static_cast<size_t>(xplane) * (SPLITX ? 2 : 1);
  off = (off + 15) & ~static_cast<size_t>(15);
  float *acc_s = reinterpret_cast<float *>(smem + off);
  off += static_cast<size_t>(16) * kAccPitch * sizeof(float);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + off);
  // [0] abort (any role)  [1] last split of the current tile  [2] abort as sampled for this tile
  volatile int *flags = reinterpret_cast<volatile int *>(bars + 2 * kGemvStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[kGemvStages + s]); };
  auto tile_prob = [&](int T, int &local) {
    const int pi = (T >= t1) + (T >= t2);
    local = T - (pi == 0 ? 0 : (pi == 1 ? t1 : t2));
    return pi;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemvStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), kGemvConsumerWarps);
    }
    flags[0] = 0;
    flags[1] = 0;
    flags[2] = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      const uint64_t pol = policy_evict_first();
      int g = 0;
      bool ok = true;
      for (int T = tg0; T < total_tiles && ok; T += p.tgroups) {
        int tl = 0;
        const GemvProblem &pr = p.prob[tile_prob(T, tl)];
        const uint8_t *wbase = pr.w + (static_cast<size_t>(tl) * pr.kc_total + kc0) * kTileBytes;
        for (int i = 0; i < nchunks; ++i, ++g) {
          const int s = g % kGemvStages;
          if (g >= kGemvStages && !mbar_wait(empty_bar(s), ((g / kGemvStages) - 1) & 1, p.ctl.wait_limit, flags)) {
            if (!flags[0]) report(p.ctl, flags, kDevTimeoutProducer);
            ok = false;
            break;
          }
          if (flags[0]) {
            ok = false;
            break;
          }
          // The consumers read the slot with ordinary shared loads; order those
          // reads before the async-proxy bulk write that refills it.
          fence_proxy_async_smem();
          mbar_arrive_expect_tx(full_bar(s), kTileBytes);
          bulk_load(smem_u32(ring + s * kTileBytes), wbase + static_cast<size_t>(i) * kTileBytes, kTileBytes,
                    full_bar(s), pol);
        }
      }
      // Drain: every issued copy has landed before the CTA leaves.
      volatile int no_abort = 0;
      for (int s = 0; s < kGemvStages && s < g; ++s) {
        const int last = s + kGemvStages * ((g - 1 - s) / kGemvStages);
        if (!mbar_wait(full_bar(s), (last / kGemvStages) & 1, p.ctl.wait_limit, &no_abort))
          atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int ct = threadIdx.x - 32;
    const int cw = warp - 1;
    const int g4 = lane >> 2;
    const int c = lane & 3;
    const int M = p.M;
    // Stage the activation slice [MROWS][cps*64] once (bf16 hi [, lo] planes).
    {
      const int klen = p.cps * kPackK;
      const int64_t kbase = static_cast<int64_t>(kc0) * kPackK;
      for (int idx = ct; idx < MROWS * klen; idx += kGemvConsumers) {
        const int m = idx / klen;
        const int kk = idx - m * klen;
        const int64_t k = kbase + kk;
        float v = 0.f;
        if (m < M && k < p.K) {
          if (p.x_dtype == 0)
            v = static_cast<const float *>(p.x)[m * p.ldx + k];
          else
            v = __bfloat162float(static_cast<const __nv_bfloat16 *>(p.x)[m * p.ldx + k]);
        }
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        *reinterpret_cast<__nv_bfloat16 *>(xs + m * xpitch + kk * 2) = hi;
        if (SPLITX) {
          const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
          *reinterpret_cast<__nv_bfloat16 *>(xs + xplane + m * xpitch + kk * 2) = lo;
        }
      }
      named_bar_sync(kGemvBarEpi, kGemvConsumers);
    }
    const int row_a = 16 * cw + g4;
    const int row_b = row_a + 8;
    bool alive = true;  // this warp's waits have all succeeded
    int g = 0;
    for (int T = tg0; T < total_tiles; T += p.tgroups) {
      float acc[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mt][e] = 0.f;
      for (int i = 0; i < nchunks; ++i, ++g) {
        if (!alive) continue;  // keep g in step; no more waits after a give-up
        const int s = g % kGemvStages;
        bool ok = mbar_wait(full_bar(s), (g / kGemvStages) & 1, p.ctl.wait_limit, flags);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) {
          if (lane == 0 && !flags[0]) report(p.ctl, flags, kDevTimeoutConsumer);
          alive = false;
          continue;
        }
        const uint8_t *st = ring + s * kTileBytes;
        const uint4 qa = *reinterpret_cast<const uint4 *>(st + qs_offset(row_a, c));
        const uint4 qb = *reinterpret_cast<const uint4 *>(st + qs_offset(row_b, c));
        const float da = __half2float(*reinterpret_cast<const __half *>(st + scale_offset(row_a, c >> 1)));
        const float db = __half2float(*reinterpret_cast<const __half *>(st + scale_offset(row_b, c >> 1)));
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(s));

        // bf16(f32(d) * q), eight elements per call with packed f32x2 arithmetic
        uint32_t oa[8], ob[8];
        const uint64_t dda = f2(da, da), ddb = f2(db, db);
        dequant8_bf16(qa.x, qa.y, dda, oa);
        dequant8_bf16(qa.z, qa.w, dda, oa + 4);
        dequant8_bf16(qb.x, qb.y, ddb, ob);
        dequant8_bf16(qb.z, qb.w, ddb, ob + 4);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // A fragment of word j: rows (a, b) x k pairs (4j, 4j+1), (4j+2, 4j+3)
          const uint32_t a[4] = {oa[2 * j], ob[2 * j], oa[2 * j + 1], ob[2 * j + 1]};
          const int kk = i * kPackK + c * 16 + 4 * j;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const uint2 xv = *reinterpret_cast<const uint2 *>(xs + (mt * 8 + g4) * xpitch + kk * 2);
            mma_16816_bf16(acc[mt], a, xv.x, xv.y);
            if (SPLITX) {
              const uint2 xl = *reinterpret_cast<const uint2 *>(xs + xplane + (mt * 8 + g4) * xpitch + kk * 2);
              mma_16816_bf16(acc[mt], a, xl.x, xl.y);
            }
          }
        }
      }
      // ---------------------------------------------------- tile epilogue
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int m0 = mt * 8 + 2 * c;
        acc_s[m0 * kAccPitch + row_a] = acc[mt][0];
        acc_s[(m0 + 1) * kAccPitch + row_a] = acc[mt][1];
        acc_s[m0 * kAccPitch + row_a + 8] = acc[mt][2];
        acc_s[(m0 + 1) * kAccPitch + row_a + 8] = acc[mt][3];
      }
      // One consumer samples the abort flag (any role may raise it at any time)
      // so that all consumers take the same path through the barriers below.
      if (ct == 0) flags[2] = flags[0];
      named_bar_sync(kGemvBarEpi, kGemvConsumers);
      const bool abort = flags[2] != 0;
      int tl = 0;
      const GemvProblem &pr = p.prob[tile_prob(T, tl)];
      bool store = !abort;
      if (!abort && p.splits > 1) {
        // Partials hold the M live rows only: [split][tile][M][128] f32.
        const int elems = M * kPackRows;
        const size_t sstride = static_cast<size_t>(pr.n_tiles) * elems;
        float *part = pr.partials + split * sstride + static_cast<size_t>(tl) * elems;
        for (int idx = ct; idx < elems; idx += kGemvConsumers) part[idx] = acc_s[(idx >> 7) * kAccPitch + (idx & 127)];
        __threadfence();
        named_bar_sync(kGemvBarEpi, kGemvConsumers);
        if (ct == 0) {
          const int prev = atomicAdd(&pr.counters[tl], 1);
          flags[1] = (prev == p.splits - 1) ? 1 : 0;
        }
        named_bar_sync(kGemvBarEpi, kGemvConsumers);
        store = flags[1] != 0;
        if (store) {
          __threadfence();
          // Sum the splits in index order; eight loads are issued before their adds.
          for (int idx = ct; idx < elems; idx += kGemvConsumers) {
            const float *src = pr.partials + static_cast<size_t>(tl) * elems + idx;
            float sum = 0.f;
            int sp = 0;
            for (; sp + 8 <= p.splits; sp += 8) {
              float v[8];
#pragma unroll
              for (int u = 0; u < 8; ++u) v[u] = __ldcg(src + (sp + u) * sstride);
#pragma unroll
              for (int u = 0; u < 8; ++u) sum += v[u];
            }
            for (; sp < p.splits; ++sp) sum += __ldcg(src + sp * sstride);
            acc_s[(idx >> 7) * kAccPitch + (idx & 127)] = sum;
          }
          if (ct == 0) pr.counters[tl] = 0;  // re-armed for the next call on this stream
        }
        named_bar_sync(kGemvBarEpi, kGemvConsumers);
      }
      if (store) {
        if (pr.glu) {
          for (int idx = ct; idx < M * 64; idx += kGemvConsumers) {
            const int m = idx >> 6;
            const int r = idx & 63;
            const int64_t j = static_cast<int64_t>(tl) * 64 + r;
            if (j < pr.n_out) {
              float v = acc_s[m * kAccPitch + r];
              float gt = acc_s[m * kAccPitch + 64 + r];
              if (pr.bias) {
                v += pr.bias[j];
                gt += pr.bias[pr.n_out + j];
              }
              store_out(pr.y, p.y_dtype, m * pr.ldy + j, act_glu(p.epi, v, gt));
            }
          }
        } else {
          for (int idx = ct; idx < M * kPackRows; idx += kGemvConsumers) {
            const int m = idx >> 7;
            const int r = idx & 127;
            const int64_t j = static_cast<int64_t>(tl) * kPackRows + r;
            if (j < pr.N) {
              float v = acc_s[m * kAccPitch + r];
              if (pr.bias) v += pr.bias[j];
              store_out(pr.y, p.y_dtype, m * pr.ldy + j, act_single(p.epi, v));
            }
          }
        }
      }
      named_bar_sync(kGemvBarEpi, kGemvConsumers);  // acc_s and flags[1] free for the next tile
      if (abort) break;
    }
  }
  __syncthreads();
}

template <int MT, bool SPLITX>
static cudaError_t launch_gemv_t(const GemvParams &p, cudaStream_t stream) {
  const int cps_max = gemv_max_cps(8 * MT, SPLITX);
  if (p.cps > cps_max) return cudaErrorInvalidValue;
  const size_t smem = gemv_smem_bytes(8 * MT, SPLITX, p.cps);
  auto kern = gemv_q8_kernel<MT, SPLITX>;
  static bool attr_set[64] = {false};  // once per device, sized for the largest slice
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(gemv_smem_bytes(8 * MT, SPLITX, cps_max)));
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set[dev] = true;
  }
  return launch_pdl(kern, dim3(p.splits * p.tgroups), dim3(kGemvThreads), smem, stream, 1, p);
}

cudaError_t launch_gemv(const GemvParams &p, bool splitx, cudaStream_t stream) {
  if (p.M <= 8) return splitx ? launch_gemv_t<1, true>(p, stream) : launch_gemv_t<1, false>(p, stream);
  return splitx ? launch_gemv_t<2, true>(p, stream) : launch_gemv_t<2, false>(p, stream);
}

}  // namespace nq
