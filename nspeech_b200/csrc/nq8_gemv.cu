// nq8_gemv.cu -- K2: warp-specialised split-K Q8_0 GEMV / skinny GEMM (M <= 16).
//
// Replaces the split-K GEMV family of the reference (Triton source
// kernels/moonshine_kernels.py:1039-1276, dispatched by enc_gemv_splitk*,
// src/triton_kernels.rs:1036-1202) and the M=1 decoder projections of
// src/moonshine/decoder.rs.  Bandwidth-bound: every weight byte is read once.
//
// CTA = 1 producer warp + 8 consumer warps, one 128-row weight tile, a range of
// 64-wide K chunks (split-K over blockIdx.y, up to three weights over
// blockIdx.z for the fused Q/K/V call).
//   producer: cp.async.bulk of whole 8704-byte packed tiles into a ring of
//             kStages shared-memory slots, mbarrier full/empty handshake.
//   consumers: warp w owns rows [16w, 16w+16).  Each lane loads 16 int8 of two
//             rows, dequantizes them to bf16(d*q) in registers and issues
//             mma.m16n8k16 with the weight as the 16-row operand and the
//             activations (staged in shared memory, k order permuted to match
//             the lane's bytes) as the 8-column operand.  f32 activations
//             are split into bf16 hi + lo planes and issued as two MMAs.
//   split-K: f32 partial tiles in the workspace, an arrival counter per tile;
//             the last CTA sums the splits in index order (deterministic) and
//             runs the bias / activation / GLU epilogue.
#include "nq8_common.cuh"
#include "nq8_kernels.h"

namespace nq {

constexpr int kGemvStages = 6;
constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvThreads = 32 * (1 + kGemvConsumerWarps);
constexpr int kAccPitch = 132;  // floats per row of the staged accumulator tile
constexpr int kGemvMaxCps = 8;  // k chunks per split (bounds the staged activation slice)

static __host__ __device__ inline int gemv_x_pitch(int cps) { return cps * kPackK * 2 + 8; }

size_t gemv_smem_bytes(int mrows, bool splitx, int cps) {
  size_t off = static_cast<size_t>(kGemvStages) * kTileBytes;
  off += static_cast<size_t>(mrows) * gemv_x_pitch(cps) * (splitx ? 2 : 1);
  off = (off + 15) & ~static_cast<size_t>(15);
  off += 2 * kGemvStages * sizeof(uint64_t) + 16;
  size_t acc = static_cast<size_t>(16) * kAccPitch * sizeof(float);
  return off > acc ? off : acc;
}

template <int MT, bool SPLITX>
__global__ void __launch_bounds__(kGemvThreads) gemv_q8_kernel(const __grid_constant__ GemvParams p) {
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  constexpr int MROWS = 8 * MT;
  extern __shared__ __align__(128) uint8_t smem[];
  const GemvProblem &pr = p.prob[blockIdx.z];
  const int tile = blockIdx.x;
  if (tile >= pr.n_tiles) return;  // whole CTA, before any barrier is touched
  const int split = blockIdx.y;
  const int kc0 = split * p.cps;
  const int kc1 = min(kc0 + p.cps, pr.kc_total);
  const int nchunks = max(kc1 - kc0, 0);
  const int xpitch = gemv_x_pitch(p.cps);

  uint8_t *ring = smem;
  uint8_t *xs = smem + kGemvStages * kTileBytes;
  const int xplane = MROWS * xpitch;
  size_t off = static_cast<size_t>(kGemvStages) * kTileBytes + static_cast<size_t>(xplane) * (SPLITX ? 2 : 1);
  off = (off + 15) & ~static_cast<size_t>(15);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + off);
  volatile int *flags = reinterpret_cast<volatile int *>(bars + 2 * kGemvStages);
  float *acc_s = reinterpret_cast<float *>(smem);  // reuses the ring after the main loop

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[kGemvStages + s]); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemvStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), kGemvConsumerWarps);
    }
    flags[0] = 0;
    flags[1] = 0;
    fence_mbar_init();
  }
  __syncthreads();

  float acc[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[mt][e] = 0.f;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      const uint64_t pol = policy_evict_first();
      const uint8_t *wbase = pr.w + (static_cast<size_t>(tile) * pr.kc_total + kc0) * kTileBytes;
      int issued = 0;
      for (int i = 0; i < nchunks; ++i) {
        const int s = i % kGemvStages;
        if (i >= kGemvStages) {
          if (!mbar_wait(empty_bar(s), ((i / kGemvStages) - 1) & 1, p.ctl.wait_limit, flags)) {
            if (!flags[0]) report(p.ctl, flags, kDevTimeoutProducer);
            break;
          }
        }
        // The consumers read the stage with ordinary shared loads; order those
        // reads before the async-proxy bulk write that refills it.
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(full_bar(s), kTileBytes);
        bulk_load(smem_u32(ring + s * kTileBytes), wbase + static_cast<size_t>(i) * kTileBytes,
                  kTileBytes, full_bar(s), pol);
        ++issued;
      }
      // Drain: every issued copy must have landed before the CTA moves on.
      volatile int no_abort = 0;
      for (int s = 0; s < kGemvStages && s < issued; ++s) {
        const int last = s + kGemvStages * ((issued - 1 - s) / kGemvStages);
        if (!mbar_wait(full_bar(s), (last / kGemvStages) & 1, p.ctl.wait_limit, &no_abort))
          atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int ct = threadIdx.x - 32;
    const int cw = warp - 1;
    const int g = lane >> 2;
    const int c = lane & 3;
    // Stage activations [MROWS][cps*64] as bf16 (hi [, lo]) planes.
    const int klen = p.cps * kPackK;
    const int64_t kbase = static_cast<int64_t>(kc0) * kPackK;
    for (int idx = ct; idx < MROWS * klen; idx += 32 * kGemvConsumerWarps) {
      const int m = idx / klen;
      const int kk = idx - m * klen;
      const int64_t k = kbase + kk;
      float v = 0.f;
      if (m < p.M && k < p.K) {
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
    named_bar_sync(1, 32 * kGemvConsumerWarps);

    const int row_a = 16 * cw + g;
    const int row_b = row_a + 8;
    for (int i = 0; i < nchunks; ++i) {
      const int s = i % kGemvStages;
      bool ok = mbar_wait(full_bar(s), (i / kGemvStages) & 1, p.ctl.wait_limit, flags);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0 && !flags[0]) report(p.ctl, flags, kDevTimeoutConsumer);
        break;
      }
      const uint8_t *st = ring + s * kTileBytes;
      const uint4 qa = *reinterpret_cast<const uint4 *>(st + qs_offset(row_a, c));
      const uint4 qb = *reinterpret_cast<const uint4 *>(st + qs_offset(row_b, c));
      const float da = __half2float(*reinterpret_cast<const __half *>(st + scale_offset(row_a, c >> 1)));
      const float db = __half2float(*reinterpret_cast<const __half *>(st + scale_offset(row_b, c >> 1)));
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(s));

      const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w};
      const uint32_t wb[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t a[4];
        dequant4_bf16(wa[j], da, a[0], a[2]);
        dequant4_bf16(wb[j], db, a[1], a[3]);
        const int kk = i * kPackK + c * 16 + 4 * j;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const uint2 xv = *reinterpret_cast<const uint2 *>(xs + (mt * 8 + g) * xpitch + kk * 2);
          mma_16816_bf16(acc[mt], a, xv.x, xv.y);
          if (SPLITX) {
            const uint2 xl = *reinterpret_cast<const uint2 *>(xs + xplane + (mt * 8 + g) * xpitch + kk * 2);
            mma_16816_bf16(acc[mt], a, xl.x, xl.y);
          }
        }
      }
    }
  }
  __syncthreads();  // ring no longer in use: reuse it for the accumulator tile

  if (warp > 0) {
    const int cw = warp - 1;
    const int g = lane >> 2;
    const int c = lane & 3;
    const int row_a = 16 * cw + g;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int m0 = mt * 8 + 2 * c;
      acc_s[m0 * kAccPitch + row_a] = acc[mt][0];
      acc_s[(m0 + 1) * kAccPitch + row_a] = acc[mt][1];
      acc_s[m0 * kAccPitch + row_a + 8] = acc[mt][2];
      acc_s[(m0 + 1) * kAccPitch + row_a + 8] = acc[mt][3];
    }
  }
  __syncthreads();

  const int nth = blockDim.x;
  if (p.splits > 1) {
    // Partials hold the M live rows only: [split][tile][M][128] f32.
    const int elems = p.M * kPackRows;
    const size_t sstride = static_cast<size_t>(pr.n_tiles) * elems;
    float *part = pr.partials + split * sstride + static_cast<size_t>(tile) * elems;
    for (int idx = threadIdx.x; idx < elems; idx += nth) part[idx] = acc_s[(idx >> 7) * kAccPitch + (idx & 127)];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const int prev = atomicAdd(&pr.counters[tile], 1);
      flags[1] = (prev == p.splits - 1) ? 1 : 0;
    }
    __syncthreads();
    if (!flags[1]) return;  // uniform: not the last split of this tile
    __threadfence();
    // Sum the splits in index order; eight loads are issued before their adds.
    for (int idx = threadIdx.x; idx < elems; idx += nth) {
      const float *src = pr.partials + static_cast<size_t>(tile) * elems + idx;
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
    __syncthreads();
    if (threadIdx.x == 0) pr.counters[tile] = 0;  // re-armed for the next call on this stream
  }

  // ------------------------------------------------------------- epilogue
  const int M = p.M;
  if (pr.glu) {
    for (int idx = threadIdx.x; idx < MROWS * 64; idx += nth) {
      const int m = idx >> 6;
      const int r = idx & 63;
      const int64_t j = static_cast<int64_t>(tile) * 64 + r;
      if (m < M && j < pr.n_out) {
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
    for (int idx = threadIdx.x; idx < MROWS * kPackRows; idx += nth) {
      const int m = idx >> 7;
      const int r = idx & 127;
      const int64_t j = static_cast<int64_t>(tile) * kPackRows + r;
      if (m < M && j < pr.N) {
        float v = acc_s[m * kAccPitch + r];
        if (pr.bias) v += pr.bias[j];
        store_out(pr.y, p.y_dtype, m * pr.ldy + j, act_single(p.epi, v));
      }
    }
  }
}

template <int MT, bool SPLITX>
static cudaError_t launch_gemv_t(const GemvParams &p, int nprob, int grid_x, cudaStream_t stream) {
  const size_t smem = gemv_smem_bytes(8 * MT, SPLITX, p.cps);
  auto kern = gemv_q8_kernel<MT, SPLITX>;
  static bool attr_set[64] = {false};  // once per device, sized for the largest split (cps = 8)
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(gemv_smem_bytes(8 * MT, SPLITX, kGemvMaxCps)));
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set[dev] = true;
  }
  if (p.cps > kGemvMaxCps) return cudaErrorInvalidValue;
  dim3 grid(grid_x, p.splits, nprob);
  return launch_pdl(kern, grid, dim3(kGemvThreads), smem, stream, 1, p);
}

cudaError_t launch_gemv(const GemvParams &p, int nprob, int grid_x, bool splitx, cudaStream_t stream) {
  if (p.M <= 8) return splitx ? launch_gemv_t<1, true>(p, nprob, grid_x, stream) : launch_gemv_t<1, false>(p, nprob, grid_x, stream);
  return splitx ? launch_gemv_t<2, true>(p, nprob, grid_x, stream) : launch_gemv_t<2, false>(p, nprob, grid_x, stream);
}

}  // namespace nq
