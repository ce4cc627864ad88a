// nq8_encoder_kernels.cu -- the non-GEMM kernels of the FastConformer encoder
// forward (src/parakeet/fast_conformer.rs:99-189, 214-494, 967-1104).  The
// Q8_0 contractions of the encoder run through nq_linear; these kernels are
// the glue between them.  Batches of padded segments: every kernel that mixes
// frames (convolutions, attention) reads frames >= the segment's own length as
// zero (keys: masked), so a padded batch reproduces per-segment results.
#include <algorithm>

#include "nq8_common.cuh"
#include "nq8_encoder.h"

namespace nq {
namespace enc {

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

// ------------------------------------------------------------ subsampling
// conv2d(1 -> C, 3x3, stride 2, pad 1) + bias + ReLU on the log-mel
// [B, T, F] (f32), output NHWC [B, T1, F1, C] bf16 (fast_conformer.rs:103-107,
// 176-177).  Frames t >= len0[b] read as zero.
// One block per output row (b, t1): the three input mel rows it needs are
// staged in shared memory (zero-padded on both axes, frames >= len0[b] zero),
// thread c computes channel c for every output frequency; each output row
// position is one contiguous C-wide store across the block.
constexpr int kMaxFeat = 512;
__global__ void conv0_relu_kernel(const float *__restrict__ mel, const int *__restrict__ len0, int T, int F,
                                  int T1, int F1, int C, const float *__restrict__ w, const float *__restrict__ bias,
                                  __nv_bfloat16 *__restrict__ out) {
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  __shared__ float rows[3][kMaxFeat + 2];  // column j holds frequency j - 1
  const int b = blockIdx.y;
  const int t1 = blockIdx.x;
  const int L = len0[b];
  for (int idx = threadIdx.x; idx < 3 * (F + 2); idx += blockDim.x) {
    const int dt = idx / (F + 2);
    const int j = idx - dt * (F + 2);
    const int t = 2 * t1 - 1 + dt;
    const int f = j - 1;
    float v = 0.f;
    if (t >= 0 && t < T && t < L && f >= 0 && f < F) v = mel[(static_cast<int64_t>(b) * T + t) * F + f];
    rows[dt][j] = v;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float wr[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) wr[i] = w[c * 9 + i];
    const float bc = bias[c];
    __nv_bfloat16 *o = out + (static_cast<int64_t>(b) * T1 + t1) * F1 * C + c;
    for (int f1 = 0; f1 < F1; ++f1) {
      float acc = bc;
#pragma unroll
      for (int dt = 0; dt < 3; ++dt)
#pragma unroll
        for (int df = 0; df < 3; ++df) acc += wr[dt * 3 + df] * rows[dt][2 * f1 + df];
      o[static_cast<int64_t>(f1) * C] = __float2bfloat16_rn(fmaxf(acc, 0.f));
    }
  }
}

// conv0 + the first depthwise conv of the subsampling stack in one pass:
//   out[b, t2, f2, c] = b2[c] + sum_{dt,df} w2[c][dt,df] * s1[2 t2 - 1 + dt][2 f2 - 1 + df][c]
//   s1[t1][f1][c]     = bf16(relu(b0[c] + sum_{dt,df} w0[c][dt,df] * mel[2 t1 - 1 + dt][2 f1 - 1 + df]))
// (fast_conformer.rs:172-180; s1 terms with t1 outside [0, len1) or f1 outside
// [0, F1) are zero, as in conv0_relu + dwconv2d_s2).  The s1 rows a tile of
// kCdTT output rows needs (2 kCdTT + 1) are computed into shared memory and
// never reach HBM.  conv0 runs on the tensor cores: a GEMM [positions x 16 taps
// (9 used)] x [16 x 64 channels] with mma.sync m16n8k16, the mel patches and
// weights split into bf16 hi + lo parts (x w = xh wh + xh wl + xl wh: f32-level
// accuracy).  The depthwise conv is f32 with packed f32x2 FMAs: each thread
// owns two channels and a 4 x 4 patch of outputs, so the 9 x 9 s1 tile it
// needs is read once and 32 independent accumulator chains keep the FMA pipe
// busy.  An s1 position holds kCdPos bf16 (64 channels + 8 pad), which makes
// both the fragment stores of the conv0 epilogue and the channel-contiguous
// loads of the depthwise conv free of bank conflicts.
// Block = (64 channels, kCdTT output rows, one segment), 8 warps.
constexpr int kCdTT = 4;   // output rows (t2) per block
constexpr int kCdCG = 64;  // channels per block
constexpr int kCdPos = kCdCG + 8;  // bf16 per s1 position in shared memory
constexpr int kCdRows1 = 2 * kCdTT + 1;
constexpr int kCdMelRows = 4 * kCdTT + 3;

// Padded mel row (16-byte multiple): column j holds frequency j - 1, with
// room for the last 16-position tile's patches.
__host__ __device__ constexpr int cd_mel_pitch(int F1) { return ((2 * (((F1 + 15) / 16) * 16) + 6 + 3) / 4) * 4; }
// s1 positions per row in shared memory: index 0 is the zero f1 = -1 guard,
// index f1 + 1 holds f1 for f1 < 16 ceil(F1 / 16) (zero from F1 on), which
// covers every column the 4-wide output patches read (8 ceil(F2 / 4) <= 16 ceil(F1 / 16)).
__host__ __device__ constexpr int cd_s1_cols(int F1) { return 1 + 16 * ((F1 + 15) / 16); }

size_t conv0_dw_smem_bytes(int F, int F1) {
  (void)F;
  return static_cast<size_t>(kCdMelRows) * cd_mel_pitch(F1) * sizeof(float) +
         static_cast<size_t>(kCdRows1) * cd_s1_cols(F1) * kCdPos * sizeof(__nv_bfloat16);
}

__device__ __forceinline__ uint32_t bf16x2_hi_lo(float a, float b, uint32_t &lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float2 hf = __bfloat1622float2(h);
  const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
  lo = *reinterpret_cast<const uint32_t *>(&l);
  return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// bf16(relu(v.lo)) in the low half, bf16(relu(v.hi)) in the high half
__device__ __forceinline__ uint32_t relu_bf16x2(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  uint32_t d;
  asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
// bf16x2 (low half = element 0) -> f32x2 (low word = element 0), exact
__device__ __forceinline__ uint64_t f32x2_of_bf16x2(uint32_t v) {
  return f2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

__global__ void __launch_bounds__(256) conv0_dw_s2_kernel(
    const float *__restrict__ mel, const int *__restrict__ len0, const int *__restrict__ len1, int T, int F, int T1,
    int F1, int T2, int F2, int C, const float *__restrict__ w0, const float *__restrict__ b0,
    const float *__restrict__ w2, const float *__restrict__ b2, __nv_bfloat16 *__restrict__ out) {
  extern __shared__ __align__(16) unsigned char cd_smem[];
  const int FP = cd_mel_pitch(F1);
  const int S1C = cd_s1_cols(F1);
  float *melS = reinterpret_cast<float *>(cd_smem);
  __nv_bfloat16 *s1S = reinterpret_cast<__nv_bfloat16 *>(cd_smem + static_cast<size_t>(kCdMelRows) * FP * sizeof(float));
  const int b = blockIdx.z;
  const int t2s = blockIdx.y * kCdTT;
  const int cg0 = blockIdx.x * kCdCG;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  // Weights and biases are never written by a kernel: fetch them before the
  // wait on the predecessor.  conv0 B fragments (col-major [tap][channel]):
  // b0 = taps (2 t4, 2 t4 + 1), b1 = taps (2 t4 + 8, 2 t4 + 9) of channel nt * 8 + g.
  uint32_t bh[8][2], bl[8][2];
  uint64_t bias0[8];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const float *wc = w0 + (cg0 + nt * 8 + g) * 9;
    const int k0 = 2 * t4, k2 = 2 * t4 + 8;
    bh[nt][0] = bf16x2_hi_lo(wc[k0], wc[k0 + 1], bl[nt][0]);
    bh[nt][1] = bf16x2_hi_lo(k2 < 9 ? wc[k2] : 0.f, 0.f, bl[nt][1]);  // tap 9 and beyond are padding
    bias0[nt] = f2(b0[cg0 + nt * 8 + 2 * t4], b0[cg0 + nt * 8 + 2 * t4 + 1]);
  }
  // depthwise weights of this thread's channel pair (cc, cc + 1)
  const int cc = cg0 + 2 * lane;
  uint64_t wv[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) wv[i] = f2(w2[cc * 9 + i], w2[(cc + 1) * 9 + i]);
  const uint64_t bias2 = f2(b2[cc], b2[cc + 1]);
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  const int L0 = len0[b], L1 = min(len1[b], T1);
  // 1. mel rows 4 t2s - 3 .. (zero outside [0, min(T, L0)) and the frequency range),
  //    one warp per row
  {
    const bool vec = (reinterpret_cast<uintptr_t>(mel) & 15) == 0 && (F & 3) == 0 && F + 1 <= FP;
    for (int r = warp; r < kCdMelRows; r += 8) {
      const int t = 4 * t2s - 3 + r;
      float *dst = melS + r * FP;
      const bool live = t >= 0 && t < T && t < L0;
      const float *src = mel + (static_cast<int64_t>(b) * T + (live ? t : 0)) * F;
      if (live && vec) {
        for (int f = 4 * lane; f < F; f += 128) {
          const float4 v = __ldg(reinterpret_cast<const float4 *>(src + f));
          dst[f + 1] = v.x;
          dst[f + 2] = v.y;
          dst[f + 3] = v.z;
          dst[f + 4] = v.w;
        }
        if (lane == 0) dst[0] = 0.f;
        for (int j = F + 1 + lane; j < FP; j += 32) dst[j] = 0.f;
      } else {
        for (int j = lane; j < FP; j += 32) dst[j] = live && j >= 1 && j <= F ? src[j - 1] : 0.f;
      }
    }
  }
  // zero guard position (f1 = -1) of every s1 row
  for (int idx = threadIdx.x; idx < kCdRows1 * (kCdCG / 2); idx += blockDim.x)
    reinterpret_cast<uint32_t *>(s1S + (idx / (kCdCG / 2)) * S1C * kCdPos)[idx % (kCdCG / 2)] = 0u;
  __syncthreads();
  // 2. conv0 on tensor cores, one 16-position x 64-channel tile per warp step
  {
    // this lane's tap offsets in the mel tile (taps 2t4, 2t4+1, 2t4+8, 2t4+9; -1 = padding)
    int off[4];
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      const int k = 2 * t4 + (x & 1) + 8 * (x >> 1);
      off[x] = k < 9 ? (k / 3) * FP + (k % 3) : -1;
    }
    const int mtr = (F1 + 15) / 16;  // 16-position tiles per s1 row
    for (int mt = warp; mt < kCdRows1 * mtr; mt += 8) {
      const int r1 = mt / mtr;
      const int f10 = (mt - r1 * mtr) * 16;
      const int t1 = 2 * t2s - 1 + r1;
      // this lane's C-fragment positions f10 + g (+ 8), channels nt * 8 + 2 t4 (+ 1)
      __nv_bfloat16 *dst = s1S + (r1 * S1C + f10 + g + 1) * kCdPos + 2 * t4;
      if (!(t1 >= 0 && t1 < L1)) {  // row outside the segment: zero for the depthwise conv
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          *reinterpret_cast<uint32_t *>(dst + nt * 8) = 0u;
          *reinterpret_cast<uint32_t *>(dst + 8 * kCdPos + nt * 8) = 0u;
        }
        continue;
      }
      // A fragments: rows g and g + 8 = positions f10 + g, f10 + g + 8 of row r1
      const float *base = melS + (2 * r1) * FP + 2 * (f10 + g);
      float xa[4], xb[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        xa[x] = off[x] >= 0 ? base[off[x]] : 0.f;
        xb[x] = off[x] >= 0 ? base[off[x] + 16] : 0.f;
      }
      uint32_t ah[4], al[4];
      ah[0] = bf16x2_hi_lo(xa[0], xa[1], al[0]);
      ah[1] = bf16x2_hi_lo(xb[0], xb[1], al[1]);
      ah[2] = bf16x2_hi_lo(xa[2], xa[3], al[2]);
      ah[3] = bf16x2_hi_lo(xb[2], xb[3], al[3]);
      const bool ok0 = f10 + g < F1, ok1 = f10 + g + 8 < F1;  // positions from F1 on stay zero
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        mma_16816_bf16(acc, ah, bh[nt][0], bh[nt][1]);
        mma_16816_bf16(acc, ah, bl[nt][0], bl[nt][1]);
        mma_16816_bf16(acc, al, bh[nt][0], bh[nt][1]);
        const uint32_t p0 = relu_bf16x2(add_f32x2(f2(acc[0], acc[1]), bias0[nt]));
        const uint32_t p1 = relu_bf16x2(add_f32x2(f2(acc[2], acc[3]), bias0[nt]));
        *reinterpret_cast<uint32_t *>(dst + nt * 8) = ok0 ? p0 : 0u;
        *reinterpret_cast<uint32_t *>(dst + 8 * kCdPos + nt * 8) = ok1 ? p1 : 0u;
      }
    }
  }
  __syncthreads();
  // 3. depthwise 3x3 stride 2 over the staged rows (zero rows / guard and pad
  //    positions stand in for the taps outside the segment): warp w takes the
  //    4-column output patches q = w, w + 8, ..., lane = channel pair
  {
    const int nq = (F2 + 3) / 4;
    for (int q = warp; q < nq; q += 8) {
      uint64_t acc[kCdTT][4];
#pragma unroll
      for (int r2 = 0; r2 < kCdTT; ++r2)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[r2][j] = bias2;
      // s1 row rr feeds output rows r2 with rr = 2 r2 + dt; columns 8q - 1 .. 8q + 7
      // (positions 8q .. 8q + 8) feed output columns 4q + j with column = 2 (4q + j) - 1 + df
#pragma unroll
      for (int rr = 0; rr < kCdRows1; ++rr) {
        const __nv_bfloat16 *row = s1S + (rr * S1C + 8 * q) * kCdPos + 2 * lane;
        uint64_t v[9];
#pragma unroll
        for (int c = 0; c < 9; ++c) v[c] = f32x2_of_bf16x2(*reinterpret_cast<const uint32_t *>(row + c * kCdPos));
#pragma unroll
        for (int r2 = 0; r2 < kCdTT; ++r2) {
          const int dt = rr - 2 * r2;
          if (dt < 0 || dt > 2) continue;
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int df = 0; df < 3; ++df) acc[r2][j] = fma_f32x2(wv[dt * 3 + df], v[2 * j + df], acc[r2][j]);
        }
      }
#pragma unroll
      for (int r2 = 0; r2 < kCdTT; ++r2) {
        const int t2 = t2s + r2;
        if (t2 >= T2) break;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int f2o = 4 * q + j;
          if (f2o >= F2) break;
          *reinterpret_cast<uint32_t *>(out + ((static_cast<int64_t>(b) * T2 + t2) * F2 + f2o) * C + cc) =
              bf16x2_of(acc[r2][j]);
        }
      }
    }
  }
}

// Depthwise 3x3 stride-2 conv (pad 1) over [B, Tin, Fin, C] bf16, taps with
// t outside [0, min(Tin, len)) or f outside [0, Fin) zero (fast_conformer.rs
// dwconv2d_s2).  Warp task = (2 output rows x 4 output columns, 64 channels):
// lane = channel pair, so every load is one 128-byte line of a position, the
// 5 x 9 input patch the task needs is read once (instead of 9 taps per output)
// and the eight outputs accumulate in independent packed f32x2 FMA chains, in
// the same tap order (dt, then df) as a per-output loop.
constexpr int kDwRows = 2, kDwCols = 4;

__global__ void __launch_bounds__(256) dwconv2d_s2_kernel(const __nv_bfloat16 *__restrict__ in,
                                                          const int *__restrict__ len_in, int Tin, int Fin, int Tout,
                                                          int Fout, int C, const float *__restrict__ w,
                                                          const float *__restrict__ bias,
                                                          __nv_bfloat16 *__restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.y * 64 + 2 * lane;
  uint64_t wv[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) wv[i] = f2(w[c * 9 + i], w[(c + 1) * 9 + i]);
  const uint64_t bv = f2(bias[c], bias[c + 1]);
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  const int b = blockIdx.z;
  const int nfq = (Fout + kDwCols - 1) / kDwCols;
  const int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int tr = task / nfq;
  const int fq = task - tr * nfq;
  const int to0 = kDwRows * tr, fo0 = kDwCols * fq;
  if (to0 >= Tout) return;
  const int L = min(len_in[b], Tin);
  uint64_t acc[kDwRows][kDwCols];
#pragma unroll
  for (int r = 0; r < kDwRows; ++r)
#pragma unroll
    for (int j = 0; j < kDwCols; ++j) acc[r][j] = bv;
  // input rows 2 to0 - 1 + rr (rr < 2 kDwRows + 1), columns 2 fo0 - 1 + cc (cc < 2 kDwCols + 1)
#pragma unroll
  for (int rr = 0; rr < 2 * kDwRows + 1; ++rr) {
    const int t = 2 * to0 - 1 + rr;
    if (t < 0 || t >= L) continue;  // zero row (warp-uniform)
    const __nv_bfloat16 *row = in + (static_cast<int64_t>(b) * Tin + t) * Fin * C + c;
    uint64_t v[2 * kDwCols + 1];
#pragma unroll
    for (int cc = 0; cc < 2 * kDwCols + 1; ++cc) {
      const int f = 2 * fo0 - 1 + cc;
      const uint32_t p = f >= 0 && f < Fin ? __ldg(reinterpret_cast<const unsigned int *>(row + static_cast<int64_t>(f) * C)) : 0u;
      v[cc] = f2(__uint_as_float(p << 16), __uint_as_float(p & 0xffff0000u));
    }
#pragma unroll
    for (int r = 0; r < kDwRows; ++r) {
      const int dt = rr - 2 * r;
      if (dt < 0 || dt > 2) continue;
#pragma unroll
      for (int j = 0; j < kDwCols; ++j)
#pragma unroll
        for (int df = 0; df < 3; ++df) {
          uint64_t d;
          asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(wv[dt * 3 + df]), "l"(v[2 * j + df]), "l"(acc[r][j]));
          acc[r][j] = d;
        }
    }
  }
#pragma unroll
  for (int r = 0; r < kDwRows; ++r) {
    const int to = to0 + r;
    if (to >= Tout) break;
#pragma unroll
    for (int j = 0; j < kDwCols; ++j) {
      const int fo = fo0 + j;
      if (fo >= Fout) break;
      *reinterpret_cast<uint32_t *>(out + ((static_cast<int64_t>(b) * Tout + to) * Fout + fo) * C + c) =
          bf16x2_of(acc[r][j]);
    }
  }
}

// Any C: one output per thread (the general fallback of the kernel above).
__global__ void dwconv2d_s2_any_kernel(const __nv_bfloat16 *__restrict__ in, const int *__restrict__ len_in, int Tin,
                                   int Fin, int Tout, int Fout, int C, const float *__restrict__ w,
                                   const float *__restrict__ bias, __nv_bfloat16 *__restrict__ out) {
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  const int b = blockIdx.z;
  const int to = blockIdx.y;
  const int L = len_in[b];
  for (int idx = threadIdx.x + blockIdx.x * blockDim.x; idx < Fout * C; idx += gridDim.x * blockDim.x) {
    const int fo = idx / C;
    const int c = idx - fo * C;
    float acc = bias[c];
#pragma unroll
    for (int dt = 0; dt < 3; ++dt) {
      const int t = 2 * to - 1 + dt;
      if (t < 0 || t >= Tin || t >= L) continue;
#pragma unroll
      for (int df = 0; df < 3; ++df) {
        const int f = 2 * fo - 1 + df;
        if (f < 0 || f >= Fin) continue;
        acc += w[c * 9 + dt * 3 + df] * bf(in[((static_cast<int64_t>(b) * Tin + t) * Fin + f) * C + c]);
      }
    }
    out[((static_cast<int64_t>(b) * Tout + to) * Fout + fo) * C + c] = __float2bfloat16_rn(acc);
  }
}

// NHWC [B*T, F, C] -> [B*T, C*F] (the reference flattens transpose(1,2) of
// NCHW, feature index c*F + f; fast_conformer.rs:184-186).
__global__ void flatten_cf_kernel(const __nv_bfloat16 *__restrict__ in, int rows, int F, int C,
                                  __nv_bfloat16 *__restrict__ out) {
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  const int r = blockIdx.x;
  for (int idx = threadIdx.x; idx < F * C; idx += blockDim.x) {
    const int c = idx / F;
    const int f = idx - c * F;
    out[static_cast<int64_t>(r) * F * C + idx] = in[(static_cast<int64_t>(r) * F + f) * C + c];
  }
}

// ---------------------------------------------------------- LayerNorm family
// One warp per row of D = 32 * 4 * kVec floats (D = 1024 -> kVec = 8).
// mode kLnScale:  x = alpha * u (u f32);            h1 = LN1(x)
// mode kLnResAdd: x = x + alpha * u (u bf16);       h1 = LN1(x)
// mode kLnResAddOut: x = LN1(x + alpha * u) (final norm_out, stored f32);
//                    h1 = LN2(x) if g2 != null (next layer's first norm)
// The grid is persistent (a few blocks per SM; each warp strides over the
// rows), and the LayerNorm parameters are staged once per block in shared
// memory before the dependency wait -- no kernel writes them.  A row then
// costs one global round trip (its x and u loads, issued together), not
// three (x/u, then gamma/beta of each LayerNorm after the reductions), and a
// warp issues the loads of its next row before the reductions of the current
// one, so that round trip overlaps the current row's work.
constexpr int kLnThreads = 256;
// Resident blocks per SM: a D = 1024 row in flight takes 48 registers per
// lane, and a warp holds one in flight beside the row it computes.
__host__ __device__ constexpr int ln_min_blocks(int kVec) { return kVec >= 8 ? 2 : 3; }
template <int kVec>
__global__ void __launch_bounds__(kLnThreads, ln_min_blocks(kVec))
    ln_row_kernel(int mode, float *__restrict__ x, const void *__restrict__ u, float alpha, int rows,
                  const float *__restrict__ g1, const float *__restrict__ b1, const float *__restrict__ g2,
                  const float *__restrict__ b2, __nv_bfloat16 *__restrict__ h, float eps) {
  constexpr int D = 32 * 4 * kVec;
  constexpr int kQ = D / 4;  // float4 per parameter vector
  extern __shared__ float4 ln_par[];  // g1 | b1 | g2 | b2, kQ float4 each (g2, b2 when given)
  {
    const int n = (g2 ? 4 : 2) * kQ;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int which = i / kQ;
      const float *src = which == 0 ? g1 : which == 1 ? b1 : which == 2 ? g2 : b2;
      ln_par[i] = reinterpret_cast<const float4 *>(src)[i - which * kQ];
    }
  }
  __syncthreads();
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  float4 ra[kVec];  // the x row (kLnScale: the f32 u row)
  uint2 rb[kVec];   // the bf16 u row (kLnResAdd, kLnResAddOut)
  auto load = [&](int r) {
    const int64_t off = static_cast<int64_t>(r) * D;
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
      const int col = (i * 32 + lane) * 4;
      if (mode == kLnScale) {
        ra[i] = *reinterpret_cast<const float4 *>(static_cast<const float *>(u) + off + col);
      } else {
        ra[i] = *reinterpret_cast<const float4 *>(x + off + col);
        rb[i] = *reinterpret_cast<const uint2 *>(static_cast<const __nv_bfloat16 *>(u) + off + col);
      }
    }
  };
  int warp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (warp < rows) load(warp);
  for (; warp < rows; warp += nwarps) {
    float *xr = x + static_cast<int64_t>(warp) * D;
    float v[kVec][4];
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      float uu[4];
      if (mode == kLnScale) {
        uu[0] = ra[i].x; uu[1] = ra[i].y; uu[2] = ra[i].z; uu[3] = ra[i].w;
      } else {
        a = ra[i];
        uu[0] = bf16_bits_to_f32(rb[i].x & 0xffffu); uu[1] = bf16_bits_to_f32(rb[i].x >> 16);
        uu[2] = bf16_bits_to_f32(rb[i].y & 0xffffu); uu[3] = bf16_bits_to_f32(rb[i].y >> 16);
      }
      v[i][0] = a.x + alpha * uu[0];
      v[i][1] = a.y + alpha * uu[1];
      v[i][2] = a.z + alpha * uu[2];
      v[i][3] = a.w + alpha * uu[3];
    }
    if (warp + nwarps < rows) load(warp + nwarps);  // next row: in flight during this row's work
    auto normalize = [&](const float4 *g, const float4 *bb) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < kVec; ++i) s += v[i][0] + v[i][1] + v[i][2] + v[i][3];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      const float mean = s * (1.0f / D);
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < kVec; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float dlt = v[i][e] - mean;
          q += dlt * dlt;
        }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
      const float rstd = rsqrtf(q * (1.0f / D) + eps);
#pragma unroll
      for (int i = 0; i < kVec; ++i) {
        const float4 gg = g[i * 32 + lane];
        const float4 bv = bb[i * 32 + lane];
        v[i][0] = (v[i][0] - mean) * rstd * gg.x + bv.x;
        v[i][1] = (v[i][1] - mean) * rstd * gg.y + bv.y;
        v[i][2] = (v[i][2] - mean) * rstd * gg.z + bv.z;
        v[i][3] = (v[i][3] - mean) * rstd * gg.w + bv.w;
      }
    };
    auto store_h = [&]() {
      __nv_bfloat16 *hr = h + static_cast<int64_t>(warp) * D;
#pragma unroll
      for (int i = 0; i < kVec; ++i) {
        const int col = (i * 32 + lane) * 4;
        *reinterpret_cast<uint2 *>(hr + col) = make_uint2(pack_bf16x2(v[i][0], v[i][1]), pack_bf16x2(v[i][2], v[i][3]));
      }
    };
    auto store_x = [&]() {
#pragma unroll
      for (int i = 0; i < kVec; ++i) {
        const int col = (i * 32 + lane) * 4;
        *reinterpret_cast<float4 *>(xr + col) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
      }
    };
    if (mode == kLnResAddOut) {
      normalize(ln_par, ln_par + kQ);
      store_x();
      if (g2) {
        normalize(ln_par + 2 * kQ, ln_par + 3 * kQ);
        store_h();
      }
    } else {
      store_x();
      normalize(ln_par, ln_par + kQ);
      store_h();
    }
  }
}

// --------------------------------------------------- conv module middle part
// Depthwise conv1d over time (kernel K, pad K/2, groups D) + bias, eval-mode
// BatchNorm folded to scale/shift, SiLU (fast_conformer.rs:486-488).
// in/out [B, Tp, D] bf16; input frames t >= len[b] count as zero.
// Thread = two adjacent channels (bf16x2: a warp moves 128 contiguous bytes
// per frame) sliding over a chunk of frames with the K input taps held in
// registers, so every input element is read once per chunk.
template <int K>
__global__ void __launch_bounds__(128) dwconv1d_bn_silu_kernel(
    const __nv_bfloat16 *__restrict__ in, const int *__restrict__ len, int Tp, int D, int t_chunk,
    const float *__restrict__ w, const float *__restrict__ bias, const float *__restrict__ bn_scale,
    const float *__restrict__ bn_shift, __nv_bfloat16 *__restrict__ out) {
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  const int b = blockIdx.z;
  const int L = min(len[b], Tp);
  const int c = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (c >= D) return;
  const int t0 = blockIdx.y * t_chunk;
  const int t1 = min(Tp, t0 + t_chunk);
  constexpr int pad = K / 2;
  float w0[K], w1[K];
#pragma unroll
  for (int i = 0; i < K; ++i) {
    w0[i] = w[c * K + i];
    w1[i] = w[(c + 1) * K + i];
  }
  const float b0 = bias[c], b1 = bias[c + 1];
  const float s0 = bn_scale[c], s1 = bn_scale[c + 1], h0 = bn_shift[c], h1 = bn_shift[c + 1];
  const __nv_bfloat162 *src = reinterpret_cast<const __nv_bfloat162 *>(in + static_cast<int64_t>(b) * Tp * D + c);
  __nv_bfloat162 *dst = reinterpret_cast<__nv_bfloat162 *>(out + static_cast<int64_t>(b) * Tp * D + c);
  const int dstride = D / 2;
  auto load = [&](int t) -> float2 {
    if (t < 0 || t >= L) return make_float2(0.f, 0.f);
    return __bfloat1622float2(src[static_cast<int64_t>(t) * dstride]);
  };
  // Four output frames per step; their four new input frames are loaded
  // together (x[i] = input frame t - pad + i).
  constexpr int kU = 4;
  float2 x[K - 1 + kU];
#pragma unroll
  for (int i = 0; i < K - 1; ++i) x[i] = load(t0 - pad + i);
  for (int t = t0; t < t1; t += kU) {
#pragma unroll
    for (int u = 0; u < kU; ++u) x[K - 1 + u] = load(t + pad + u);
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (t + u < t1) {
        float a0 = b0, a1 = b1;
#pragma unroll
        for (int i = 0; i < K; ++i) {
          a0 += w0[i] * x[u + i].x;
          a1 += w1[i] * x[u + i].y;
        }
        const float y0 = a0 * s0 + h0, y1 = a1 * s1 + h1;
        dst[static_cast<int64_t>(t + u) * dstride] = __floats2bfloat162_rn(y0 * sigmoidf_(y0), y1 * sigmoidf_(y1));
      }
    }
#pragma unroll
    for (int i = 0; i < K - 1; ++i) x[i] = x[i + kU];
  }
}

// Relative positional encoding of 2T-1 positions (fast_conformer.rs:69-97):
// row idx <-> relative position p = idx - (T-1); even columns
// sign(p) * sin(|p| / 10000^(2i/d)) with sign -1 for p > 0, odd columns cos.
__global__ void relpos_kernel(int T, int D, __nv_bfloat16 *__restrict__ pos) {
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  const int idx = blockIdx.x;
  const int p = idx - (T - 1);
  const float ap = fabsf(static_cast<float>(p));
  const float sign = p > 0 ? -1.f : 1.f;
  for (int i = threadIdx.x; i < D / 2; i += blockDim.x) {
    const float div = ap / powf(10000.0f, 2.0f * static_cast<float>(i) / static_cast<float>(D));
    pos[static_cast<int64_t>(idx) * D + 2 * i] = __float2bfloat16_rn(sign * sinf(div));
    pos[static_cast<int64_t>(idx) * D + 2 * i + 1] = __float2bfloat16_rn(cosf(div));
  }
}

// ------------------------------------------------- relative-position attention
// Flash-style MHSA with Transformer-XL relative positions
// (MultiHeadSelfAttention::forward + rel_shift, fast_conformer.rs:256-313,
// 407-425):
//   s[i][j] = ((q_i + u_h) . k_j + (q_i + v_h) . r[T-1 + j - i]) / sqrt(hd)
//   o_i = softmax_j(s[i][:]) . V          (keys j >= len masked)
// qkv [B*Tp, 3D] bf16 (q | k | v), krel [2Tp-1, D] bf16 with row stride ldr
// (the layers' relative projections are computed together, side by side),
// out [B*Tp, D] bf16.
// CTA = 8 warps x 16 query rows (128 rows), one head; key tiles of 64.  Each
// warp keeps its (q + u) and (q + v) A fragments in registers.  K and V tiles
// are double-buffered with cp.async; the relative rows live in a 256-row ring
// (a key tile needs 191 consecutive rows and the next tile 64 new ones), and
// each warp multiplies only the 80 relative rows its diagonal band touches
// (BD = Qv R^T, 16 x 80), parks them in shared memory and gathers
// BD[il][jl - il + 15] for its scores.  Legacy mma.sync m16n8k16.
constexpr int kHd = 128;
constexpr int kQT = 128;         // query rows per CTA
constexpr int kKT = 64;          // keys per tile
constexpr int kAWarps = kQT / 16;
constexpr int kRing = 256;       // relative rows kept (power of two)
constexpr int kBdCols = 80;      // relative rows per warp and tile
constexpr int kPitch = kHd + 8;  // bf16 elements per smem row (272 B): conflict-free ldmatrix
constexpr int kBdPitch = 84;     // floats per parked BD row

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// 16-byte global -> shared copy; src_bytes 0 writes zeros (rows out of range).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Rows [r0, r0 + nrows) x kHd of a [*, ld] bf16 matrix (column offset col0)
// into shared rows slot(r) with pitch kPitch; rows outside [0, rmax) are zero.
template <typename SlotFn>
__device__ __forceinline__ void load_rows_async(__nv_bfloat16 *dst, const __nv_bfloat16 *src, int64_t ld, int col0,
                                                int r0, int nrows, int rmax, SlotFn slot, int tid, int nthreads) {
  for (int idx = tid; idx < nrows * (kHd / 8); idx += nthreads) {
    const int r = idx / (kHd / 8);
    const int c8 = idx - r * (kHd / 8);
    const int gr = r0 + r;
    const bool ok = gr >= 0 && gr < rmax;
    const __nv_bfloat16 *g = src + static_cast<int64_t>(ok ? gr : 0) * ld + col0 + c8 * 8;
    cp_async16(smem_u32(dst + slot(r) * kPitch + c8 * 8), g, ok ? 16 : 0);
  }
}

__global__ void __launch_bounds__(32 * kAWarps, 1)
    relpos_attention_kernel(const __nv_bfloat16 *__restrict__ qkv, const __nv_bfloat16 *__restrict__ krel, int64_t ldr,
                            const float *__restrict__ bias_u, const float *__restrict__ bias_v,
                            const int *__restrict__ len, int Tp, int D, float scale, __nv_bfloat16 *__restrict__ out) {
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t sm[];
  __nv_bfloat16 *sK = reinterpret_cast<__nv_bfloat16 *>(sm);  // [2][kKT][kPitch]
  __nv_bfloat16 *sV = sK + 2 * kKT * kPitch;                   // [2][kKT][kPitch]
  __nv_bfloat16 *sR = sV + 2 * kKT * kPitch;                   // [kRing][kPitch]
  float *sBD = reinterpret_cast<float *>(sR + kRing * kPitch); // [kAWarps][16][kBdPitch]

  const int b = blockIdx.z;
  const int h = blockIdx.y;
  const int i0 = blockIdx.x * kQT;
  const int tid = threadIdx.x;
  const int nthr = blockDim.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int g = lane >> 2;
  const int t4 = lane & 3;
  const int L = min(len[b], Tp);
  const int64_t ld = 3 * static_cast<int64_t>(D);
  const __nv_bfloat16 *base = qkv + static_cast<int64_t>(b) * Tp * ld;
  const int wrow0 = warp * 16;  // CTA-local first query row of this warp
  const int ntiles = (L + kKT - 1) / kKT;
  // Relative row of CTA-window index 0 for key tile t: P0 + 64 t.
  const int P0 = Tp - 1 - i0 - (kQT - 1);
  auto ring = [](int p) { return p & (kRing - 1); };

  // Prefetch tile 0 (K, V, 192 relative rows) while the Q fragments load.
  if (ntiles > 0) {
    load_rows_async(sK, base, ld, D + h * kHd, 0, kKT, L, [](int r) { return r; }, tid, nthr);
    load_rows_async(sV, base, ld, 2 * D + h * kHd, 0, kKT, L, [](int r) { return r; }, tid, nthr);
    load_rows_async(sR, krel, ldr, h * kHd, P0, 192, 2 * Tp - 1, [&](int r) { return ring(P0 + r); }, tid, nthr);
  }
  cp_async_commit();

  // A fragments of (q + u) and (q + v) for this warp's 16 rows (m16n8k16 layout:
  // a0 (g, 2t4), a1 (g + 8, 2t4), a2 (g, 2t4 + 8), a3 (g + 8, 2t4 + 8) per 16-wide k slice).
  uint32_t au[kHd / 16][4], av[kHd / 16][4];
  {
    const int ra = i0 + wrow0 + g, rb = ra + 8;
#pragma unroll
    for (int kk = 0; kk < kHd / 16; ++kk) {
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        const int row = (x & 1) ? rb : ra;
        const int c = kk * 16 + 2 * t4 + 8 * (x >> 1);
        float q0 = 0.f, q1 = 0.f;
        if (row < Tp) {
          const __nv_bfloat162 q = *reinterpret_cast<const __nv_bfloat162 *>(base + static_cast<int64_t>(row) * ld + h * kHd + c);
          q0 = __low2float(q);
          q1 = __high2float(q);
        }
        au[kk][x] = pack_bf16x2(q0 + bias_u[h * kHd + c], q1 + bias_u[h * kHd + c + 1]);
        av[kk][x] = pack_bf16x2(q0 + bias_v[h * kHd + c], q1 + bias_v[h * kHd + c + 1]);
      }
    }
  }

  float o[kHd / 8][4];
#pragma unroll
  for (int n = 0; n < kHd / 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY};
  float lrow[2] = {0.f, 0.f};
  const float sl2 = scale * 1.4426950408889634f;  // softmax in base 2
  float *bd = sBD + warp * 16 * kBdPitch;
  // This warp's relative rows within the CTA window: [kQT - 16 - wrow0, + 80).
  const int wwin = kQT - 16 - wrow0;

  for (int t = 0; t < ntiles; ++t) {
    const int j0 = t * kKT;
    const int buf = t & 1;
    cp_async_wait_all();
    __syncthreads();  // tile t landed for everyone; tile t-1's buffers are free
    if (t + 1 < ntiles) {
      const int jn = j0 + kKT;
      __nv_bfloat16 *dk = sK + (buf ^ 1) * kKT * kPitch;
      __nv_bfloat16 *dv = sV + (buf ^ 1) * kKT * kPitch;
      load_rows_async(dk, base, ld, D + h * kHd, jn, kKT, L, [](int r) { return r; }, tid, nthr);
      load_rows_async(dv, base, ld, 2 * D + h * kHd, jn, kKT, L, [](int r) { return r; }, tid, nthr);
      const int pn = P0 + 192 + 64 * t;  // the 64 relative rows tile t + 1 adds
      load_rows_async(sR, krel, ldr, h * kHd, pn, 64, 2 * Tp - 1, [&](int r) { return ring(pn + r); }, tid, nthr);
    }
    cp_async_commit();
    const __nv_bfloat16 *cK = sK + buf * kKT * kPitch;
    const __nv_bfloat16 *cV = sV + buf * kKT * kPitch;
    const int pw = P0 + 64 * t + wwin;  // relative row of this warp's BD column 0

    // BD = Qv R^T over the warp's 80 relative rows, parked in shared memory.
    {
      float r[kBdCols / 8][4];
#pragma unroll
      for (int n = 0; n < kBdCols / 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) r[n][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < kHd / 16; ++kk) {
#pragma unroll
        for (int nb = 0; nb < kBdCols / 16; ++nb) {
          uint32_t b0, b1, b2, b3;
          const int q = lane >> 3, rr = lane & 7;
          const int pr = pw + nb * 16 + rr + 8 * (q >> 1);
          const int col = kk * 16 + 8 * (q & 1);
          ldsm_x4(smem_u32(sR + ring(pr) * kPitch + col), b0, b1, b2, b3);
          mma_16816_bf16(r[2 * nb], av[kk], b0, b1);
          mma_16816_bf16(r[2 * nb + 1], av[kk], b2, b3);
        }
      }
#pragma unroll
      for (int n = 0; n < kBdCols / 8; ++n) {
        *reinterpret_cast<float2 *>(bd + g * kBdPitch + n * 8 + 2 * t4) = make_float2(r[n][0], r[n][1]);
        *reinterpret_cast<float2 *>(bd + (g + 8) * kBdPitch + n * 8 + 2 * t4) = make_float2(r[n][2], r[n][3]);
      }
    }
    __syncwarp();

    // S = Qu K^T (16 x 64) + BD[il][jl - il + 15], scaled to base 2; keys >= len masked.
    float s[kKT / 8][4];
#pragma unroll
    for (int n = 0; n < kKT / 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kHd / 16; ++kk) {
#pragma unroll
      for (int nb = 0; nb < kKT / 16; ++nb) {
        uint32_t b0, b1, b2, b3;
        const int q = lane >> 3, rr = lane & 7;
        const int key = nb * 16 + rr + 8 * (q >> 1);
        const int col = kk * 16 + 8 * (q & 1);
        ldsm_x4(smem_u32(cK + key * kPitch + col), b0, b1, b2, b3);
        mma_16816_bf16(s[2 * nb], au[kk], b0, b1);
        mma_16816_bf16(s[2 * nb + 1], au[kk], b2, b3);
      }
    }
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < kKT / 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int rl = g + 8 * (e >> 1);          // row within the warp
        const int jl = n * 8 + 2 * t4 + (e & 1);  // key within the tile
        const float rel = bd[rl * kBdPitch + (jl - rl + 15)];
        float v = (s[n][e] + rel) * sl2;
        if (j0 + jl >= L) v = -INFINITY;
        s[n][e] = v;
        tmax[e >> 1] = fmaxf(tmax[e >> 1], v);
      }
    __syncwarp();  // bd reads done before the next tile parks
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      tmax[hh] = fmaxf(tmax[hh], __shfl_xor_sync(0xffffffffu, tmax[hh], 1));
      tmax[hh] = fmaxf(tmax[hh], __shfl_xor_sync(0xffffffffu, tmax[hh], 2));
    }
    float corr[2], tsum[2] = {0.f, 0.f};
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const float mnew = fmaxf(mrow[hh], tmax[hh]);
      corr[hh] = exp2f(mrow[hh] - mnew);
      mrow[hh] = mnew;
    }
    uint32_t pa[kKT / 16][4];
#pragma unroll
    for (int n = 0; n < kKT / 8; ++n) {
      const float p0 = exp2f(s[n][0] - mrow[0]);
      const float p1 = exp2f(s[n][1] - mrow[0]);
      const float p2 = exp2f(s[n][2] - mrow[1]);
      const float p3 = exp2f(s[n][3] - mrow[1]);
      tsum[0] += p0 + p1;
      tsum[1] += p2 + p3;
      const int kb = n >> 1;
      if ((n & 1) == 0) {
        pa[kb][0] = pack_bf16x2(p0, p1);
        pa[kb][1] = pack_bf16x2(p2, p3);
      } else {
        pa[kb][2] = pack_bf16x2(p0, p1);
        pa[kb][3] = pack_bf16x2(p2, p3);
      }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      tsum[hh] += __shfl_xor_sync(0xffffffffu, tsum[hh], 1);
      tsum[hh] += __shfl_xor_sync(0xffffffffu, tsum[hh], 2);
      lrow[hh] = lrow[hh] * corr[hh] + tsum[hh];
    }
#pragma unroll
    for (int n = 0; n < kHd / 8; ++n) {
      o[n][0] *= corr[0];
      o[n][1] *= corr[0];
      o[n][2] *= corr[1];
      o[n][3] *= corr[1];
    }
    // O += P V  (V [key][hd] -> transposed ldmatrix for the col-major operand)
#pragma unroll
    for (int kb = 0; kb < kKT / 16; ++kb) {
#pragma unroll
      for (int nb = 0; nb < kHd / 16; ++nb) {
        uint32_t b0, b1, b2, b3;
        const int q = lane >> 3, rr = lane & 7;
        const int key = kb * 16 + rr + 8 * (q & 1);
        const int col = nb * 16 + 8 * (q >> 1);
        ldsm_x4_t(smem_u32(cV + key * kPitch + col), b0, b1, b2, b3);
        mma_16816_bf16(o[2 * nb], pa[kb], b0, b1);
        mma_16816_bf16(o[2 * nb + 1], pa[kb], b2, b3);
      }
    }
  }
  cp_async_wait_all();  // nothing in flight at exit

  const float inv0 = lrow[0] > 0.f ? 1.f / lrow[0] : 0.f;
  const float inv1 = lrow[1] > 0.f ? 1.f / lrow[1] : 0.f;
  const int ia = i0 + wrow0 + g;
  const int ib = ia + 8;
  __nv_bfloat16 *ob = out + static_cast<int64_t>(b) * Tp * D + h * kHd;
#pragma unroll
  for (int n = 0; n < kHd / 8; ++n) {
    const int col = n * 8 + 2 * t4;
    if (ia < Tp)
      *reinterpret_cast<uint32_t *>(ob + static_cast<int64_t>(ia) * D + col) = pack_bf16x2(o[n][0] * inv0, o[n][1] * inv0);
    if (ib < Tp)
      *reinterpret_cast<uint32_t *>(ob + static_cast<int64_t>(ib) * D + col) = pack_bf16x2(o[n][2] * inv1, o[n][3] * inv1);
  }
}

__global__ void copy_masked_kernel(const float *__restrict__ x, const int *__restrict__ len, int Tp, int D,
                                   float *__restrict__ out) {
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  const int row = blockIdx.x;  // b * Tp + t
  const int b = row / Tp;
  const int t = row - b * Tp;
  const bool keep = t < len[b];
  const float4 *src = reinterpret_cast<const float4 *>(x + static_cast<int64_t>(row) * D);
  float4 *dst = reinterpret_cast<float4 *>(out + static_cast<int64_t>(row) * D);
  for (int i = threadIdx.x; i < D / 4; i += blockDim.x) dst[i] = keep ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
}

cudaError_t copy_masked(const float *x, const int *len, int B, int Tp, int D, float *out, cudaStream_t s) {
  if (B * Tp == 0) return cudaSuccess;
  return launch_pdl(copy_masked_kernel, dim3(B * Tp), dim3(256), 0, s, 1, x, len, Tp, D, out);
}

size_t attention_smem_bytes() {
  return static_cast<size_t>(4 * kKT + kRing) * kPitch * 2 + static_cast<size_t>(kAWarps) * 16 * kBdPitch * 4;
}

// ------------------------------------------------------------------ launches
cudaError_t conv0_relu(const float *mel, const int *len0, int B, int T, int F, int T1, int F1, int C, const float *w,
                       const float *bias, __nv_bfloat16 *out, cudaStream_t s) {
  if (F > kMaxFeat || 2 * (F1 - 1) + 2 > F + 1) return cudaErrorInvalidValue;
  dim3 grid(T1, B);
  return launch_pdl(conv0_relu_kernel, grid, dim3(C <= 1024 ? C : 1024), 0, s, 1, mel, len0, T, F, T1, F1, C, w, bias,
                    out);
}

bool conv0_dw_s2_supported(int F, int F1, int C) {
  return C % kCdCG == 0 && F <= kMaxFeat && conv0_dw_smem_bytes(F, F1) <= 160 * 1024;
}

cudaError_t conv0_dw_s2(const float *mel, const int *len0, const int *len1, int B, int T, int F, int T1, int F1, int T2,
                        int F2, int C, const float *w0, const float *b0, const float *w2, const float *b2,
                        __nv_bfloat16 *out, cudaStream_t s) {
  if (!conv0_dw_s2_supported(F, F1, C) || 2 * (F1 - 1) + 2 > F + 1) return cudaErrorInvalidValue;
  const size_t smem = conv0_dw_smem_bytes(F, F1);
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(conv0_dw_s2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  dim3 grid(C / kCdCG, (T2 + kCdTT - 1) / kCdTT, B);
  return launch_pdl(conv0_dw_s2_kernel, grid, dim3(256), smem, s, 1, mel, len0, len1, T, F, T1, F1, T2, F2, C, w0, b0,
                    w2, b2, out);
}

cudaError_t dwconv2d_s2(const __nv_bfloat16 *in, const int *len_in, int B, int Tin, int Fin, int Tout, int Fout, int C,
                        const float *w, const float *bias, __nv_bfloat16 *out, cudaStream_t s) {
  const int threads = 256;
  if (C % 64 == 0) {
    const int tasks = ((Tout + kDwRows - 1) / kDwRows) * ((Fout + kDwCols - 1) / kDwCols);
    dim3 grid((tasks + threads / 32 - 1) / (threads / 32), C / 64, B);
    return launch_pdl(dwconv2d_s2_kernel, grid, dim3(threads), 0, s, 1, in, len_in, Tin, Fin, Tout, Fout, C, w, bias,
                      out);
  }
  const int per = Fout * C;
  dim3 grid((per + threads - 1) / threads, Tout, B);
  return launch_pdl(dwconv2d_s2_any_kernel, grid, dim3(threads), 0, s, 1, in, len_in, Tin, Fin, Tout, Fout, C, w, bias,
                    out);
}

cudaError_t flatten_cf(const __nv_bfloat16 *in, int rows, int F, int C, __nv_bfloat16 *out, cudaStream_t s) {
  return launch_pdl(flatten_cf_kernel, dim3(rows), dim3(256), 0, s, 1, in, rows, F, C, out);
}

cudaError_t ln_rows(int mode, float *x, const void *u, float alpha, int rows, int D, const float *g1, const float *b1,
                    const float *g2, const float *b2, __nv_bfloat16 *h, float eps, cudaStream_t s) {
  if (D != 1024 && D != 512) return cudaErrorInvalidValue;
  if (rows <= 0) return cudaSuccess;
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!sms[dev]) {
    int n = 0;
    const cudaError_t e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    sms[dev] = n;
  }
  const int per_block = kLnThreads / 32;
  const int blocks = std::min((rows + per_block - 1) / per_block, sms[dev] * ln_min_blocks(D / 128));
  const size_t smem = static_cast<size_t>(g2 ? 4 : 2) * D * sizeof(float);
  if (D == 1024)
    return launch_pdl(ln_row_kernel<8>, dim3(blocks), dim3(kLnThreads), smem, s, 1, mode, x, u, alpha, rows, g1, b1,
                      g2, b2, h, eps);
  return launch_pdl(ln_row_kernel<4>, dim3(blocks), dim3(kLnThreads), smem, s, 1, mode, x, u, alpha, rows, g1, b1, g2,
                    b2, h, eps);
}

cudaError_t dwconv1d_bn_silu(const __nv_bfloat16 *in, const int *len, int B, int Tp, int D, int K, const float *w,
                             const float *bias, const float *bn_scale, const float *bn_shift, __nv_bfloat16 *out,
                             cudaStream_t s) {
  if (K < 1 || K > 31 || (D & 1)) return cudaErrorInvalidValue;
  constexpr int kThreads = 128;
  const int t_chunk = 32;
  dim3 grid((D / 2 + kThreads - 1) / kThreads, (Tp + t_chunk - 1) / t_chunk, B);
  switch (K) {
#define NQ_DW1D_CASE(k) \
  case k:                                                                                                      \
    return launch_pdl(dwconv1d_bn_silu_kernel<k>, grid, dim3(kThreads), 0, s, 1, in, len, Tp, D, t_chunk, w, bias, \
                      bn_scale, bn_shift, out);
    NQ_DW1D_CASE(1) NQ_DW1D_CASE(2) NQ_DW1D_CASE(3) NQ_DW1D_CASE(4) NQ_DW1D_CASE(5) NQ_DW1D_CASE(6)
    NQ_DW1D_CASE(7) NQ_DW1D_CASE(8) NQ_DW1D_CASE(9) NQ_DW1D_CASE(10) NQ_DW1D_CASE(11) NQ_DW1D_CASE(12)
    NQ_DW1D_CASE(13) NQ_DW1D_CASE(14) NQ_DW1D_CASE(15) NQ_DW1D_CASE(16) NQ_DW1D_CASE(17) NQ_DW1D_CASE(18)
    NQ_DW1D_CASE(19) NQ_DW1D_CASE(20) NQ_DW1D_CASE(21) NQ_DW1D_CASE(22) NQ_DW1D_CASE(23) NQ_DW1D_CASE(24)
    NQ_DW1D_CASE(25) NQ_DW1D_CASE(26) NQ_DW1D_CASE(27) NQ_DW1D_CASE(28) NQ_DW1D_CASE(29) NQ_DW1D_CASE(30)
    NQ_DW1D_CASE(31)
#undef NQ_DW1D_CASE
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t relpos(int T, int D, __nv_bfloat16 *pos, cudaStream_t s) {
  return launch_pdl(relpos_kernel, dim3(2 * T - 1), dim3(256), 0, s, 1, T, D, pos);
}

cudaError_t relpos_attention(const __nv_bfloat16 *qkv, const __nv_bfloat16 *krel, int64_t ldr, const float *bias_u,
                             const float *bias_v, const int *len, int B, int Tp, int H, int D, __nv_bfloat16 *out,
                             cudaStream_t s) {
  if (D / H != kHd) return cudaErrorInvalidValue;
  const size_t smem = attention_smem_bytes();
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(relpos_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  dim3 grid((Tp + kQT - 1) / kQT, H, B);
  return launch_pdl(relpos_attention_kernel, grid, dim3(32 * kAWarps), smem, s, 1, qkv, krel, ldr, bias_u, bias_v, len, Tp,
                    D, 1.0f / sqrtf(static_cast<float>(kHd)), out);
}

}  // namespace enc
}  // namespace nq
