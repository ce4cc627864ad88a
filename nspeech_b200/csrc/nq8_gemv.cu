// nq8_gemv.cu -- K2: dynamically scheduled Q8_0 GEMV / skinny GEMM (M <= 16).
//
// Replaces the split-K GEMV family of the reference (Triton source
// kernels/moonshine_kernels.py:1039-1276, dispatched by enc_gemv_splitk*,
// src/triton_kernels.rs:1036-1202) and the M=1 decoder projections of
// src/moonshine/decoder.rs.  HBM-bound: every weight byte is read once.
//
// Work: the weight tiles of up to three problems sharing x (fused Q/K/V) are
// cut into units of `unit` 64-wide k chunks (upt units per tile, tile-major).
// The cut is fixed by the shape, not by timing: unit j of a tile always owns
// the same k range and writes its f32 partial to slot j, and gemv_reduce
// (the next launch) sums each tile's slots in a fixed order, so results are
// reproducible bit for bit.  Which CTA computes a unit is dynamic: CTA c
// starts with unit c and then takes the next unit from a work counter, so
// CTAs that stream faster take more units (per-CTA HBM rates differ by tens
// of percent on B200).  CTA = 1 producer warp + 4 consumer warps:
//   producer: cp.async.bulk of whole 8704-byte packed chunks into a ring of
//             shared-memory stages, tagged with (unit, chunk); a proxy fence
//             orders the consumers' shared reads of a stage before the copy
//             that refills it.  The weights are constant, so the first unit
//             is fetched before the programmatic dependency wait and overlaps
//             the previous kernel's tail.
//   consumers: warp w owns rows [32w, 32w+32) of each tile as two 16-row
//             groups: ldmatrix hands each lane 16 int8 of four rows (four
//             bytes from each 16-byte k quarter; whole 128-byte rows per
//             matrix, so no bank conflicts), which it dequantizes to
//             bf16(d*q) and feeds to mma.m16n8k16 as the 16-row operand, with
//             the activations (bf16, the same k order, read from global / L1
//             one chunk ahead) as the 8-column operand.  At the
//             end of a unit each lane stores its accumulators to the unit's
//             partial slot and goes on with the next unit.
// gemv_reduce: one CTA per (tile, row of x) sums the tile's slots, applies
// bias / activation / GLU, stores the output and re-arms the work counter.
// Every wait is bounded; a role that gives up raises the CTA's abort flag and
// the others leave their loops at their next wait.
#include <algorithm>

#include "nq8_common.cuh"
#include "nq8_kernels.h"
#include "nq8_sm100_pair.cuh"

namespace nq {

constexpr int kGemvConsumerWarps = 4;
constexpr int kGemvConsumers = 32 * kGemvConsumerWarps;
constexpr int kGemvThreads = 32 + kGemvConsumers;  // producer warp, consumers
constexpr int kGemvCtasPerSm = 4;
constexpr int kGemvStages = 6;
constexpr int kGemvSlotsPerTile = 32;  // scheduling granularity target
constexpr size_t kGemvMetaOff = static_cast<size_t>(kGemvStages) * kTileBytes;     // int2 (unit, chunk) per stage
constexpr size_t kGemvBarOff = kGemvMetaOff + kGemvStages * 2 * sizeof(int);      // full, empty
constexpr size_t kGemvFlagOff = kGemvBarOff + 2 * kGemvStages * sizeof(uint64_t);  // abort flag
constexpr size_t kGemvSmemBytes = kGemvFlagOff + 16;

GemvPlan gemv_plan(int sm_count, int total_tiles, int kc, int m) {
  GemvPlan g;
  const int64_t slots = static_cast<int64_t>(kGemvCtasPerSm) * sm_count;
  // About kGemvSlotsPerTile units per tile (measured on B200 from 640 x 640
  // to 16384 x 16384: fewer, longer units leave a longer tail, more slots
  // cost partial traffic and a longer sum), at least two chunks.  The f32
  // partials of a unit (M x 128 x 4 bytes) are at most half its weight bytes
  // (2 x 8,704) for M <= 16 and stay in L2 until the sum reads them; longer
  // units for larger M cost more in lost parallelism (M = 16, K = 1024:
  // 12.2 us with 8-chunk units).
  (void)m;
  const int64_t u = std::max<int64_t>(2, (kc + kGemvSlotsPerTile - 1) / kGemvSlotsPerTile);
  g.unit = static_cast<int>(std::min<int64_t>(u, kc));
  g.upt = (kc + g.unit - 1) / g.unit;
  g.units = total_tiles * g.upt;
  g.ctas = static_cast<int>(std::min<int64_t>(slots, g.units));
  return g;
}

// Activation fragments of one 64-wide chunk for this lane (g, c): for each
// k quarter q the four bf16 at k = 16q + 4c .. +3 of its row (the k order of
// the weight words ldsm_x4 hands the lane), zero for rows beyond M.
template <int MT>
__device__ __forceinline__ void load_x_chunk(uint2 (&v)[MT][4], const __nv_bfloat16 *const (&xr)[MT],
                                             const bool (&live)[MT], int ch) {
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      v[mt][q] = live[mt] ? __ldg(reinterpret_cast<const uint2 *>(xr[mt] + static_cast<size_t>(ch) * kPackK + 16 * q))
                          : make_uint2(0u, 0u);
  }
}

// Four 8x8 b16 matrices from shared memory (lane i addresses row i % 8 of
// matrix i / 8); lane (g, c) receives 32 bits [g][2c, 2c+1] of each.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// c = -1152 * d exactly in f32, from the f16 bits of d (mixed-precision FMA).
__device__ __forceinline__ float neg1152(uint16_t d16) {
  float c;
  asm("{\n\t.reg .f16 dd, m;\n\tmov.b16 dd, %1;\n\tmov.b16 m, 0xE480;\n\tfma.rn.f32.f16 %0, dd, m, 0f00000000;\n\t}"
      : "=f"(c)
      : "h"(d16));
  return c;
}


// Resident CTAs per SM: 16 activation rows with hi + lo planes need more
// registers than four CTAs leave (the plan still sizes the grid for four;
// the dynamic unit schedule balances CTAs that start a wave later).
constexpr int gemv_min_ctas(int mt, bool splitx) { return mt == 2 && splitx ? 3 : kGemvCtasPerSm; }

template <int MT, bool SPLITX>
__global__ void __launch_bounds__(kGemvThreads, gemv_min_ctas(MT, SPLITX))
    gemv_q8_kernel(const __grid_constant__ GemvParams p) {
  constexpr int S = kGemvStages;
  // No dependency wait here: the producer's first unit only reads the
  // (constant) weights; every other access waits first.
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t smem[];
  const int kc = p.kc;
  const int t1 = p.prob[0].n_tiles, t2 = t1 + p.prob[1].n_tiles;

  uint8_t *ring = smem;
  volatile int *meta = reinterpret_cast<volatile int *>(smem + kGemvMetaOff);  // (unit, chunk) per stage
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kGemvBarOff);
  volatile int *flags = reinterpret_cast<volatile int *>(smem + kGemvFlagOff);  // [0] abort (any role)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[S + s]); };
  auto tile_prob = [&](int T, int &local) {
    const int pi = (T >= t1) + (T >= t2);
    local = T - (pi == 0 ? 0 : (pi == 1 ? t1 : t2));
    return pi;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), kGemvConsumerWarps);
    }
    flags[0] = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      const uint64_t pol = policy_evict_first();
      int s = 0, issued = 0;
      uint32_t ph = 0;  // (issued / S) & 1
      bool ok = true, waited = false;
      auto next_stage = [&](bool &good) {
        if (issued >= S && !mbar_wait(empty_bar(s), ph ^ 1u, p.ctl.wait_limit, flags)) {
          if (!flags[0]) report(p.ctl, flags, kDevTimeoutProducer);
          good = false;
        }
        if (flags[0]) good = false;
      };
      auto advance = [&]() {
        ++issued;
        if (++s == S) {
          s = 0;
          ph ^= 1u;
        }
      };
      int u = blockIdx.x;
      bool have_stage = false;  // a free stage is already waited for
      while (ok && u < p.units) {
        const int T = u / p.upt;
        const int c0 = (u - T * p.upt) * p.unit;
        const int c1 = min(c0 + p.unit, kc);
        int tl = 0;
        const GemvProblem &pr = p.prob[tile_prob(T, tl)];
        const uint8_t *src = pr.w + (static_cast<size_t>(tl) * kc + c0) * kTileBytes;
        for (int ch = c0; ch < c1; ++ch, src += kTileBytes) {
          if (!have_stage) next_stage(ok);
          have_stage = false;
          if (!ok) break;
          meta[2 * s] = u;
          meta[2 * s + 1] = ch;
          // The consumers read the stage with ordinary shared loads; order
          // those reads before the async-proxy bulk write that refills it.
          fence_proxy_async_smem();
          mbar_arrive_expect_tx(full_bar(s), kTileBytes);
          bulk_load(smem_u32(ring + s * kTileBytes), src, kTileBytes, full_bar(s), pol);
          advance();
        }
        if (!ok) break;
        if (!waited) {
          pdl_wait();  // the previous launch's gemv_reduce re-armed the work counter
          waited = true;
        }
        // Take the next unit only once a stage is free: a CTA holds at most
        // its ring of chunks beyond the unit being computed, which bounds the
        // imbalance when the work runs out.
        next_stage(ok);
        if (!ok) break;
        have_stage = true;
        u = p.ctas + atomicAdd(p.sched, 1);
      }
      if (ok) {
        // end marker: a stage whose phase completes with no copy
        if (!have_stage) next_stage(ok);
        if (ok) {
          meta[2 * s] = -1;
          mbar_arrive(full_bar(s));
          advance();
        }
      }
      // Drain: every issued copy has landed before the CTA leaves.
      volatile int no_abort = 0;
      for (int st = 0; st < S && st < issued; ++st) {
        const int last = st + S * ((issued - 1 - st) / S);
        if (!mbar_wait(full_bar(st), (last / S) & 1, p.ctl.wait_limit, &no_abort))
          atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    pdl_wait();  // predecessor kernel complete, its writes visible
    const int cw = warp - 1;
    const int g4 = lane >> 2;
    const int c = lane & 3;
    const int M = p.M;
    // Rows 32cw + 8b + g4 (b = 0..3): groups (b0, b1) and (b2, b3) are the
    // (row, row + 8) halves of the two 16-row MMA operands.  ldsm_x4 block b:
    // lane i addresses row 32cw + 8b + i % 8, k quarter i / 8.
    uint32_t lofs[4], sofs[4][2];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      lofs[b] = qs_offset(32 * cw + 8 * b + (lane & 7), lane >> 3);
      sofs[b][0] = scale_offset(32 * cw + 8 * b + g4, 0);
      sofs[b][1] = scale_offset(32 * cw + 8 * b + g4, 1);
    }
    const __nv_bfloat16 *xh[MT];
    const __nv_bfloat16 *xl[MT];
    bool live[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int m = mt * 8 + g4;
      live[mt] = m < M;
      xh[mt] = p.xh + static_cast<int64_t>(live[mt] ? m : 0) * p.ldx + 4 * c;
      xl[mt] = SPLITX ? p.xl + static_cast<int64_t>(live[mt] ? m : 0) * p.ldx + 4 * c : nullptr;
    }
    float acc[2][MT][4];
    uint2 xc[MT][4], xcl[MT][4];
    int s = 0, cur = -1, ch = 0, c_end = 0;
    uint32_t ph = 0;
    while (true) {
      const int st = s;
      const uint32_t par = ph;
      if (++s == S) {
        s = 0;
        ph ^= 1u;
      }
      bool ok = mbar_wait(full_bar(st), par, p.ctl.wait_limit, flags);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0 && !flags[0]) report(p.ctl, flags, kDevTimeoutConsumer);
        break;
      }
      if (cur < 0) {
        // first chunk of a unit (the stage's tag), or the end marker
        cur = meta[2 * st];
        if (cur < 0) break;
        ch = meta[2 * st + 1];
        const int T = cur / p.upt;
        c_end = min((cur - T * p.upt + 1) * p.unit, kc);
#pragma unroll
        for (int gi = 0; gi < 2; ++gi)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[gi][mt][e] = 0.f;
        load_x_chunk<MT>(xc, xh, live, ch);
        if (SPLITX) load_x_chunk<MT>(xcl, xl, live, ch);
      } else {
        ++ch;  // units are streamed chunk after chunk
      }
      const uint8_t *sp = ring + st * kTileBytes;
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
      if (lane == 0) mbar_arrive(empty_bar(st));
      const bool more = ch + 1 < c_end;
      // next chunk's activations, one chunk ahead of their use
      uint2 xn[MT][4], xnl[MT][4];
      if (more) {
        load_x_chunk<MT>(xn, xh, live, ch + 1);
        if (SPLITX) load_x_chunk<MT>(xnl, xl, live, ch + 1);
      }
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        const int ba = 2 * gi, bb = 2 * gi + 1;
        const float ca[2] = {neg1152(dv[ba][0]), neg1152(dv[ba][1])};
        const float cb[2] = {neg1152(dv[bb][0]), neg1152(dv[bb][1])};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          // bf16(f32(d) * q) of the lane's word in k quarter q (Q8_0 block q / 2)
          uint32_t a[4];
          dequant4_bf16_mix(R[ba][q], dv[ba][q >> 1], ca[q >> 1], a[0], a[2]);
          dequant4_bf16_mix(R[bb][q], dv[bb][q >> 1], cb[q >> 1], a[1], a[3]);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            mma_16816_bf16(acc[gi][mt], a, xc[mt][q].x, xc[mt][q].y);
            if (SPLITX) mma_16816_bf16(acc[gi][mt], a, xcl[mt][q].x, xcl[mt][q].y);
          }
        }
      }
      if (more) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            xc[mt][q] = xn[mt][q];
            if (SPLITX) xcl[mt][q] = xnl[mt][q];
          }
      } else {
        // end of the unit: its partial slot [j][M][ldp] of the problem
        const int T = cur / p.upt;
        const int j = cur - T * p.upt;
        int tl = 0;
        const GemvProblem &pr = p.prob[tile_prob(T, tl)];
        const size_t ldp = static_cast<size_t>(pr.n_tiles) * kPackRows;
        float *base = pr.partials + static_cast<size_t>(j) * M * ldp + static_cast<size_t>(tl) * kPackRows;
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
          const int ra = 32 * cw + 16 * gi + g4;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const int m0 = mt * 8 + 2 * c;
            if (m0 < M) {
              base[m0 * ldp + ra] = acc[gi][mt][0];
              base[m0 * ldp + ra + 8] = acc[gi][mt][2];
            }
            if (m0 + 1 < M) {
              base[(m0 + 1) * ldp + ra] = acc[gi][mt][1];
              base[(m0 + 1) * ldp + ra + 8] = acc[gi][mt][3];
            }
          }
        }
        cur = -1;
      }
    }
  }
  __syncthreads();
}

// Sum of a tile's unit partials for one row of x: warp w adds slots w, w+8,
// w+16, ... in order (each lane four outputs), then the eight warp sums are
// added in warp order -- a fixed order, so the result does not depend on
// which CTA computed which unit.  Then bias / activation / GLU and the store;
// the first CTA re-arms the GEMV's work counter for the next launch.
constexpr int kReduceWarps = 8;

__global__ void __launch_bounds__(32 * kReduceWarps) gemv_reduce_kernel(const __grid_constant__ GemvParams p) {
  pdl_wait();  // the GEMV's partials are complete and visible
  pdl_trigger();
  __shared__ float4 wsum[kReduceWarps][32];
  __shared__ float tot[kPackRows];
  const int T = blockIdx.x, m = blockIdx.y;
  const int t1 = p.prob[0].n_tiles, t2 = t1 + p.prob[1].n_tiles;
  const int pi = (T >= t1) + (T >= t2);
  const int tl = T - (pi == 0 ? 0 : (pi == 1 ? t1 : t2));
  const GemvProblem &pr = p.prob[pi];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t ldp = static_cast<size_t>(pr.n_tiles) * kPackRows;
  const size_t slot_stride = static_cast<size_t>(p.M) * ldp;
  const float *src = pr.partials + static_cast<size_t>(m) * ldp + static_cast<size_t>(tl) * kPackRows + lane * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j0 = warp; j0 < p.upt; j0 += 8 * kReduceWarps) {
    float4 v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int j = j0 + e * kReduceWarps;
      v[e] = j < p.upt ? __ldcg(reinterpret_cast<const float4 *>(src + j * slot_stride)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      acc.x += v[e].x;
      acc.y += v[e].y;
      acc.z += v[e].z;
      acc.w += v[e].w;
    }
  }
  wsum[warp][lane] = acc;
  __syncthreads();
  if (warp == 0) {
    float4 t = wsum[0][lane];
#pragma unroll
    for (int w = 1; w < kReduceWarps; ++w) {
      t.x += wsum[w][lane].x;
      t.y += wsum[w][lane].y;
      t.z += wsum[w][lane].z;
      t.w += wsum[w][lane].w;
    }
    reinterpret_cast<float4 *>(tot)[lane] = t;
  }
  __syncthreads();
  const int r = threadIdx.x;
  if (pr.glu) {
    const int64_t j = static_cast<int64_t>(tl) * 64 + r;
    if (r < 64 && j < pr.n_out) {
      float v = tot[r], gt = tot[64 + r];
      if (pr.bias) {
        v += pr.bias[j];
        gt += pr.bias[pr.n_out + j];
      }
      store_out(pr.y, p.y_dtype, m * pr.ldy + j, act_glu(p.epi, v, gt));
    }
  } else {
    const int64_t j = static_cast<int64_t>(tl) * kPackRows + r;
    if (r < kPackRows && j < pr.N) {
      float v = tot[r];
      if (pr.bias) v += pr.bias[j];
      store_out(pr.y, p.y_dtype, m * pr.ldy + j, act_single(p.epi, v));
    }
  }
  if (T == 0 && m == 0 && threadIdx.x == 0) p.sched[0] = 0;
}

// Decoder-step epilogue of the GEMV (the reference's split-K reduce +
// residual add + LayerNorm, kernels/moonshine_kernels.py:1109-1146, behind
// DecoderBackend::gemv_resadd_ln, src/moonshine/gpu_decoder.rs:67-70): one
// CTA per row of x.  Each output n of the row: y = sum of its unit partials in
// slot order + bias; res_out = res_in + y (f32, stored); then the row's mean
// and variance (fixed-order block sums) and out = (res_out - mean) * rstd *
// gamma + beta.  The first CTA re-arms the GEMV's work counter.
// 1024 threads: rows of up to 1024 outputs (the decoders' d_model) give each
// thread one output, whose unit partials it sums with 16 loads in flight --
// the call is a chain of dependent L2 round trips, so parallelism is what
// sets its latency.
constexpr int kLnThreads = 1024;
constexpr int kLnPerThread = kGemvLnMaxN / kLnThreads;

__device__ __forceinline__ float block_sum_fixed(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red is free (a previous sum has been read)
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kLnThreads / 32; ++w) t += red[w];
  return t;
}

__global__ void __launch_bounds__(kLnThreads) gemv_reduce_resadd_ln_kernel(const __grid_constant__ GemvParams p) {
  pdl_wait();  // the GEMV's partials are complete and visible
  pdl_trigger();
  __shared__ float red[kLnThreads / 32];
  const int m = blockIdx.x;
  const GemvProblem &pr = p.prob[0];
  const int N = static_cast<int>(pr.N);
  const size_t ldp = static_cast<size_t>(pr.n_tiles) * kPackRows;
  const size_t slot_stride = static_cast<size_t>(p.M) * ldp;
  const float *src = pr.partials + static_cast<size_t>(m) * ldp;
  const float *rin = p.res_in + static_cast<int64_t>(m) * p.ld_res;
  float *rout = p.res_out + static_cast<int64_t>(m) * p.ld_res;
  float v[kLnPerThread];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kLnPerThread; ++i) {
    const int n = threadIdx.x + i * kLnThreads;
    float a = 0.f;
    if (n < N) {
      // slots in index order, sixteen loads in flight
      const float *q = src + n;
      int j = 0;
      for (; j + 16 <= p.upt; j += 16) {
        float t[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) t[e] = __ldcg(q + (j + e) * slot_stride);
#pragma unroll
        for (int e = 0; e < 16; ++e) a += t[e];
      }
      if (j < p.upt) {
        float t[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) t[e] = j + e < p.upt ? __ldcg(q + (j + e) * slot_stride) : 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e)
          if (j + e < p.upt) a += t[e];
      }
      if (pr.bias) a += pr.bias[n];
      a += rin[n];
      rout[n] = a;
    }
    v[i] = a;
    sum += a;
  }
  const float mean = block_sum_fixed(sum, red) / static_cast<float>(N);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < kLnPerThread; ++i) {
    const int n = threadIdx.x + i * kLnThreads;
    const float dlt = n < N ? v[i] - mean : 0.f;
    sq += dlt * dlt;
  }
  const float rstd = rsqrtf(block_sum_fixed(sq, red) / static_cast<float>(N) + p.ln_eps);
#pragma unroll
  for (int i = 0; i < kLnPerThread; ++i) {
    const int n = threadIdx.x + i * kLnThreads;
    if (n < N)
      store_out(pr.y, p.y_dtype, m * pr.ldy + n, (v[i] - mean) * rstd * p.ln_g[n] + (p.ln_b ? p.ln_b[n] : 0.f));
  }
  if (m == 0 && threadIdx.x == 0) p.sched[0] = 0;
}

// ------------------------------------------------------- cluster form
// One launch per call for latency-bound shapes.  Tile T of the call (over
// all problems) belongs to a cluster of `cl` CTAs; rank r streams chunks
// r, r + cl, ... of the tile (the whole tile's k, so no unit partials leave
// the cluster) and runs the consumer above on them.  The ranks' 128-row
// partial sums meet in rank 0's shared memory through distributed shared
// memory, added in rank order; rank 0 applies bias / activation / GLU, or the
// residual add.  A residual call's LayerNorm needs whole rows: each cluster
// counts its tile on a device counter after storing its residual rows, and
// the cluster that counts last computes the LayerNorm of every row (mean and
// biased variance in f32, fixed-order sums) and re-arms the counter.  No
// wait depends on another CTA's progress except the cluster barriers, which
// every thread reaches.
constexpr int kGcStages = 5;
constexpr size_t kGcPartOff = static_cast<size_t>(kGcStages) * kTileBytes;  // f32 [16][128] this CTA's partial
constexpr size_t kGcRedOff = kGcPartOff + 16 * kPackRows * 4;                // f32 [8] block sums
constexpr size_t kGcBarOff = kGcRedOff + 32;
constexpr size_t kGcFlagOff = kGcBarOff + 2 * kGcStages * 8;
constexpr size_t kGcSmemBytes = kGcFlagOff + 16;
constexpr long long kGcDrainLimit = 1LL << 31;
static_assert(16 * kPackRows * 4 <= kGcStages * kTileBytes, "tile sums fit in the ring");

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Sum over the CTA's 160 threads in a fixed order (warp butterflies, then the
// five warp sums in warp order); every thread gets the result.
__device__ __forceinline__ float gc_block_sum(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();  // red is free
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kGemvThreads / 32; ++w) t += red[w];
  return t;
}

template <int MT, bool SPLITX>
__global__ void __launch_bounds__(kGemvThreads, gemv_min_ctas(MT, SPLITX))
    gemv_cluster_kernel(const __grid_constant__ GemvParams p, int cl) {
  constexpr int S = kGcStages;
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *ring = smem;
  float *part = reinterpret_cast<float *>(smem + kGcPartOff);  // [m][128]
  float *tot = reinterpret_cast<float *>(smem);                  // rank 0: [m][128] tile sums (ring space, free by then)
  float *red = reinterpret_cast<float *>(smem + kGcRedOff);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kGcBarOff);
  volatile int *flags = reinterpret_cast<volatile int *>(smem + kGcFlagOff);  // [0] abort [1] tile count
  const int kc = p.kc;
  const uint32_t rank = cluster_ctarank();
  const int T = blockIdx.x / cl;
  const int t1 = p.prob[0].n_tiles, t2 = t1 + p.prob[1].n_tiles;
  const int total_tiles = t2 + p.prob[2].n_tiles;
  const int pi = (T >= t1) + (T >= t2);
  const int tl = T - (pi == 0 ? 0 : (pi == 1 ? t1 : t2));
  const GemvProblem &pr = p.prob[pi];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_my = static_cast<int>(rank) < kc ? (kc - static_cast<int>(rank) + cl - 1) / cl : 0;
  auto full_bar = [&](int s) { return smem_u32(&bars[s]); };
  auto empty_bar = [&](int s) { return smem_u32(&bars[S + s]); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), kGemvConsumerWarps);
    }
    flags[0] = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      // producer: this rank's chunks of the tile (weights are constant: no
      // dependency wait before the copies)
      const uint64_t pol = policy_evict_first();
      int i = 0;
      for (; i < n_my; ++i) {
        const int s = i % S;
        if (i >= S && !mbar_wait(empty_bar(s), ((i / S) - 1) & 1, p.ctl.wait_limit, flags)) {
          if (!flags[0]) report(p.ctl, flags, kDevTimeoutProducer);
          break;
        }
        if (flags[0]) break;
        const int ch = static_cast<int>(rank) + i * cl;
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(full_bar(s), kTileBytes);
        bulk_load(smem_u32(ring + s * kTileBytes), pr.w + (static_cast<size_t>(tl) * kc + ch) * kTileBytes,
                  kTileBytes, full_bar(s), pol);
      }
      volatile int no_abort = 0;
      for (int st = 0; st < S && st < i; ++st) {
        const int last = st + S * ((i - 1 - st) / S);
        if (!mbar_wait(full_bar(st), (last / S) & 1, kGcDrainLimit, &no_abort))
          atomicOr(p.ctl.status, kDevTimeoutDrain);
      }
    }
  } else {
    pdl_wait();  // predecessor kernel complete, its writes visible
    const int cw = warp - 1;
    const int g4 = lane >> 2;
    const int c = lane & 3;
    const int M = p.M;
    uint32_t lofs[4], sofs[4][2];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      lofs[b] = qs_offset(32 * cw + 8 * b + (lane & 7), lane >> 3);
      sofs[b][0] = scale_offset(32 * cw + 8 * b + g4, 0);
      sofs[b][1] = scale_offset(32 * cw + 8 * b + g4, 1);
    }
    const __nv_bfloat16 *xh[MT];
    const __nv_bfloat16 *xl[MT];
    bool live[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int m = mt * 8 + g4;
      live[mt] = m < M;
      xh[mt] = p.xh + static_cast<int64_t>(live[mt] ? m : 0) * p.ldx + 4 * c;
      xl[mt] = SPLITX ? p.xl + static_cast<int64_t>(live[mt] ? m : 0) * p.ldx + 4 * c : nullptr;
    }
    float acc[2][MT][4];
#pragma unroll
    for (int gi = 0; gi < 2; ++gi)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[gi][mt][e] = 0.f;
    uint2 xc[MT][4], xcl[MT][4];
    if (n_my > 0) {
      load_x_chunk<MT>(xc, xh, live, static_cast<int>(rank));
      if (SPLITX) load_x_chunk<MT>(xcl, xl, live, static_cast<int>(rank));
    }
    for (int i = 0; i < n_my; ++i) {
      const int s = i % S;
      bool ok = mbar_wait(full_bar(s), (i / S) & 1, p.ctl.wait_limit, flags);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0 && !flags[0]) report(p.ctl, flags, kDevTimeoutConsumer);
        break;
      }
      const uint8_t *sp = ring + s * kTileBytes;
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
      if (lane == 0) mbar_arrive(empty_bar(s));
      // next chunk's activations, one chunk ahead of their use
      uint2 xn[MT][4], xnl[MT][4];
      const bool more = i + 1 < n_my;
      if (more) {
        load_x_chunk<MT>(xn, xh, live, static_cast<int>(rank) + (i + 1) * cl);
        if (SPLITX) load_x_chunk<MT>(xnl, xl, live, static_cast<int>(rank) + (i + 1) * cl);
      }
#pragma unroll
      for (int gi = 0; gi < 2; ++gi) {
        const int ba = 2 * gi, bb = 2 * gi + 1;
        const float ca[2] = {neg1152(dv[ba][0]), neg1152(dv[ba][1])};
        const float cb[2] = {neg1152(dv[bb][0]), neg1152(dv[bb][1])};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t a[4];
          dequant4_bf16_mix(R[ba][q], dv[ba][q >> 1], ca[q >> 1], a[0], a[2]);
          dequant4_bf16_mix(R[bb][q], dv[bb][q >> 1], cb[q >> 1], a[1], a[3]);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            mma_16816_bf16(acc[gi][mt], a, xc[mt][q].x, xc[mt][q].y);
            if (SPLITX) mma_16816_bf16(acc[gi][mt], a, xcl[mt][q].x, xcl[mt][q].y);
          }
        }
      }
      if (more) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            xc[mt][q] = xn[mt][q];
            if (SPLITX) xcl[mt][q] = xnl[mt][q];
          }
      }
    }
    // this rank's partial: part[m][row] (m < MT * 8; rows m >= M hold zeros)
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
      const int ra = 32 * cw + 16 * gi + g4;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int m0 = mt * 8 + 2 * c;
        part[m0 * kPackRows + ra] = acc[gi][mt][0];
        part[m0 * kPackRows + ra + 8] = acc[gi][mt][2];
        part[(m0 + 1) * kPackRows + ra] = acc[gi][mt][1];
        part[(m0 + 1) * kPackRows + ra + 8] = acc[gi][mt][3];
      }
    }
  }
  pdl_wait();  // every thread: the predecessor's writes are visible before the epilogue touches outputs
  __syncthreads();
  cluster_sync_all();  // every rank's partial is in place
  const int M = p.M;
  if (rank == 0) {
    for (int idx = threadIdx.x; idx < M * kPackRows; idx += kGemvThreads) {
      float v = part[idx];
      for (int k = 1; k < cl; ++k) v += ld_cluster_f32(map_rank(smem_u32(&part[idx]), static_cast<uint32_t>(k)));
      tot[idx] = v;
    }
  }
  cluster_sync_all();  // the peers' partials are read: they may leave
  if (rank != 0) return;
  if (!p.res_out) {
    if (pr.glu) {
      for (int idx = threadIdx.x; idx < M * 64; idx += kGemvThreads) {
        const int m = idx >> 6, r = idx & 63;
        const int64_t j = static_cast<int64_t>(tl) * 64 + r;
        if (j >= pr.n_out) continue;
        float v = tot[m * kPackRows + r], gt = tot[m * kPackRows + 64 + r];
        if (pr.bias) {
          v += pr.bias[j];
          gt += pr.bias[pr.n_out + j];
        }
        store_out(pr.y, p.y_dtype, m * pr.ldy + j, act_glu(p.epi, v, gt));
      }
    } else {
      for (int idx = threadIdx.x; idx < M * kPackRows; idx += kGemvThreads) {
        const int m = idx >> 7, r = idx & 127;
        const int64_t n = static_cast<int64_t>(tl) * kPackRows + r;
        if (n >= pr.N) continue;
        float v = tot[idx];
        if (pr.bias) v += pr.bias[n];
        store_out(pr.y, p.y_dtype, m * pr.ldy + n, act_single(p.epi, v));
      }
    }
    return;
  }
  // residual add of this tile's rows, then the tile count
  for (int idx = threadIdx.x; idx < M * kPackRows; idx += kGemvThreads) {
    const int m = idx >> 7, r = idx & 127;
    const int64_t n = static_cast<int64_t>(tl) * kPackRows + r;
    if (n >= pr.N) continue;
    float a = tot[idx];
    if (pr.bias) a += pr.bias[n];
    a += p.res_in[m * p.ld_res + n];
    p.res_out[m * p.ld_res + n] = a;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();  // this CTA's residual rows are visible before the count
    flags[1] = atomicAdd(&p.sched[1], 1);
    __threadfence();  // acquire: the other clusters' rows, when this is the last count
  }
  __syncthreads();
  if (flags[1] != total_tiles - 1) return;
  // last cluster: LayerNorm of every row (rows read once into registers in
  // pieces of 8 values per thread, so up to 1,280 wide rows take one read)
  const int N = static_cast<int>(pr.N);
  constexpr int kPer = 8;
  for (int m = 0; m < M; ++m) {
    const float *row = p.res_out + m * p.ld_res;
    float s = 0.f;
    for (int n0 = 0; n0 < N; n0 += kPer * kGemvThreads) {
      float v[kPer];
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int n = n0 + threadIdx.x + i * kGemvThreads;
        v[i] = n < N ? __ldcg(row + n) : 0.f;
      }
#pragma unroll
      for (int i = 0; i < kPer; ++i) s += v[i];
    }
    const float mean = gc_block_sum(s, red) / static_cast<float>(N);
    float q = 0.f;
    for (int n0 = 0; n0 < N; n0 += kPer * kGemvThreads) {
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        const int n = n0 + threadIdx.x + i * kGemvThreads;
        const float d = n < N ? __ldcg(row + n) - mean : 0.f;
        q += d * d;
      }
    }
    const float rstd = rsqrtf(gc_block_sum(q, red) / static_cast<float>(N) + p.ln_eps);
    for (int n = threadIdx.x; n < N; n += kGemvThreads)
      store_out(pr.y, p.y_dtype, m * pr.ldy + n,
                (__ldcg(row + n) - mean) * rstd * p.ln_g[n] + (p.ln_b ? p.ln_b[n] : 0.f));
  }
  if (threadIdx.x == 0) atomicExch(&p.sched[1], 0);  // every tile has counted: re-arm
}

template <int MT, bool SPLITX>
static cudaError_t launch_gemv_cluster_t(const GemvParams &p, int cl, cudaStream_t stream) {
  auto kern = gemv_cluster_kernel<MT, SPLITX>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !attr_set[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kGcSmemBytes));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set[dev] = true;
  }
  const int tiles = p.prob[0].n_tiles + p.prob[1].n_tiles + p.prob[2].n_tiles;
  return launch_pdl(kern, dim3(tiles * cl), dim3(kGemvThreads), kGcSmemBytes, stream, static_cast<unsigned>(cl), p,
                    cl);
}

template <int MT, bool SPLITX>
static cudaError_t launch_gemv_t(const GemvParams &p, int ctas, cudaStream_t stream) {
  auto kern = gemv_q8_kernel<MT, SPLITX>;
  static bool attr_set[64] = {false};  // once per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !attr_set[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kGemvSmemBytes));
    if (e != cudaSuccess) return e;
    if (dev < 64) attr_set[dev] = true;
  }
  return launch_pdl(kern, dim3(ctas), dim3(kGemvThreads), kGemvSmemBytes, stream, 1, p);
}

// AUTO takes the cluster form for plain calls of at most 8 rows whose CTAs
// get at most 5 k chunks (measured on B200: 640 x 640 3.2 vs 3.9 us,
// 640 -> 32,768 8.6 vs 9.7 us; at 8 chunks per CTA, 4096 x 4096, and with
// 16 rows the split form's dynamic schedule is faster).  A residual +
// LayerNorm call keeps the split form (its 1,024-thread LayerNorm launch is
// faster than one CTA's) unless CLUSTER is forced.
int gemv_cluster_size(int total_tiles, int kc, int sm_count, int path, bool resadd, int m) {
  if (path == 1 || (path != 2 && (resadd || m > 8))) return 0;
  const int slots = kGemvCtasPerSm * sm_count;
  const int max_chunks = path == 2 ? 8 : 5;
  for (int cl = 8; cl >= 1; cl >>= 1)
    if (cl <= kc && total_tiles * cl <= slots && (kc + cl - 1) / cl <= max_chunks) return cl;
  return 0;
}

cudaError_t launch_gemv(const GemvParams &p, int ctas, cudaStream_t stream) {
  const bool splitx = p.xl != nullptr;
  const int tiles = p.prob[0].n_tiles + p.prob[1].n_tiles + p.prob[2].n_tiles;
  const int cl = gemv_cluster_size(tiles, p.kc, p.sm_count, p.path, p.res_out != nullptr, p.M);
  if (cl > 0) {
    if (p.M <= 8)
      return splitx ? launch_gemv_cluster_t<1, true>(p, cl, stream) : launch_gemv_cluster_t<1, false>(p, cl, stream);
    return splitx ? launch_gemv_cluster_t<2, true>(p, cl, stream) : launch_gemv_cluster_t<2, false>(p, cl, stream);
  }
  cudaError_t e;
  if (p.M <= 8)
    e = splitx ? launch_gemv_t<1, true>(p, ctas, stream) : launch_gemv_t<1, false>(p, ctas, stream);
  else
    e = splitx ? launch_gemv_t<2, true>(p, ctas, stream) : launch_gemv_t<2, false>(p, ctas, stream);
  if (e != cudaSuccess) return e;
  if (p.res_out) return launch_pdl(gemv_reduce_resadd_ln_kernel, dim3(p.M), dim3(kLnThreads), 0, stream, 1, p);
  return launch_pdl(gemv_reduce_kernel, dim3(p.units / p.upt, p.M), dim3(32 * kReduceWarps), 0, stream, 1, p);
}

}  // namespace nq
