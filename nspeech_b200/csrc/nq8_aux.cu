// nq8_aux.cu -- small helper kernels of the Q8_0 path.
#include "nq8_common.cuh"
#include "nq8_kernels.h"

namespace nq {

// hi[m, k] = bf16(x), lo[m, k] = bf16(x - hi); rows of k_pad, zero for k >= K.
// Four consecutive k per thread (8-byte stores).
__global__ void split_x_kernel(const void *__restrict__ x, int x_dtype, int64_t ldx, int64_t M, int64_t K,
                               int64_t k_pad, __nv_bfloat16 *__restrict__ hi, __nv_bfloat16 *__restrict__ lo) {
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  const int64_t quads = k_pad / 4;
  const int64_t total = M * quads;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = t / quads;
    const int64_t k = (t - m * quads) * 4;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int64_t kk = k + e;
      if (kk < K) {
        v[e] = x_dtype == 0 ? static_cast<const float *>(x)[m * ldx + kk]
                            : __bfloat162float(static_cast<const __nv_bfloat16 *>(x)[m * ldx + kk]);
      } else {
        v[e] = 0.f;
      }
    }
    const uint32_t h01 = pack_bf16x2(v[0], v[1]);
    const uint32_t h23 = pack_bf16x2(v[2], v[3]);
    *reinterpret_cast<uint2 *>(hi + m * k_pad + k) = make_uint2(h01, h23);
    if (lo) {
      const float r0 = v[0] - bf16_bits_to_f32(h01 & 0xffffu), r1 = v[1] - bf16_bits_to_f32(h01 >> 16);
      const float r2 = v[2] - bf16_bits_to_f32(h23 & 0xffffu), r3 = v[3] - bf16_bits_to_f32(h23 >> 16);
      *reinterpret_cast<uint2 *>(lo + m * k_pad + k) = make_uint2(pack_bf16x2(r0, r1), pack_bf16x2(r2, r3));
    }
  }
}

cudaError_t launch_split_x(const void *x, int x_dtype, int64_t ldx, int64_t M, int64_t K, int64_t k_pad,
                           __nv_bfloat16 *hi, __nv_bfloat16 *lo, cudaStream_t stream) {
  const int64_t total = M * (k_pad / 4);
  if (total == 0) return cudaSuccess;
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  return launch_pdl(split_x_kernel, dim3(blocks), dim3(256), 0, stream, 1, x, x_dtype, ldx, M, K, k_pad, hi, lo);
}

// One block per (k chunk, tile): 256 threads, thread t dequantizes Q8_0 block
// (t & 1) of row t / 2 (32 elements) and writes 64 contiguous bytes.
__global__ void __launch_bounds__(256) dequant_tiles_kernel(const uint8_t *__restrict__ w, int kc,
                                                           __nv_bfloat16 *__restrict__ out) {
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  const int c = blockIdx.x, tile = blockIdx.y;
  const uint8_t *t = w + (static_cast<size_t>(tile) * kc + c) * kTileBytes;
  const int r = threadIdx.x >> 1, h = threadIdx.x & 1;
  const uint4 q0 = __ldg(reinterpret_cast<const uint4 *>(t + qs_offset(r, 2 * h)));
  const uint4 q1 = __ldg(reinterpret_cast<const uint4 *>(t + qs_offset(r, 2 * h + 1)));
  const float d = __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short *>(t + scale_offset(r, h)))));
  uint32_t o[16];
  const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) dequant4_bf16(qw[i], d, o[2 * i], o[2 * i + 1]);
  const size_t ldk = static_cast<size_t>(kc) * kPackK;
  uint4 *dst = reinterpret_cast<uint4 *>(out + (static_cast<size_t>(tile) * kPackRows + r) * ldk + c * kPackK + h * 32);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
}

cudaError_t launch_dequant_tiles(const uint8_t *w, int n_tiles, int kc, __nv_bfloat16 *out, cudaStream_t stream) {
  if (n_tiles <= 0 || kc <= 0) return cudaSuccess;
  return launch_pdl(dequant_tiles_kernel, dim3(kc, n_tiles), dim3(256), 0, stream, 1, w, kc, out);
}

// Thread per (token, 4 consecutive output columns); the partial sums of the
// splits are added in split order, so the result does not depend on timing.
__global__ void splitk_reduce_kernel(SplitkReduceParams p) {
  pdl_wait();  // predecessor kernel complete, its writes visible
  pdl_trigger();
  const int64_t quads = (p.n_out + 3) / 4;
  const int64_t total = static_cast<int64_t>(p.M) * quads;
  const size_t split_stride = static_cast<size_t>(p.M) * p.ldp;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = t / quads;
    const int64_t j0 = (t - m * quads) * 4;
    const float *base = p.partials + static_cast<size_t>(m) * p.ldp;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int64_t j = j0 + e;
      if (j >= p.n_out) break;
      if (!p.glu) {
        float v = 0.f;
        for (int s = 0; s < p.splits; ++s) v += __ldcs(base + s * split_stride + j);
        if (p.bias) v += p.bias[j];
        store_out(p.y, p.y_dtype, m * p.ldy + j, act_single(p.epi, v));
      } else {
        const int64_t row = (j / 64) * kPackRows + (j % 64);
        float v = 0.f, g = 0.f;
        for (int s = 0; s < p.splits; ++s) {
          v += __ldcs(base + s * split_stride + row);
          g += __ldcs(base + s * split_stride + row + 64);
        }
        if (p.bias) {
          v += p.bias[j];
          g += p.bias[p.n_out + j];
        }
        store_out(p.y, p.y_dtype, m * p.ldy + j, act_glu(p.epi, v, g));
      }
    }
  }
}

cudaError_t launch_splitk_reduce(const SplitkReduceParams &p, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(p.M) * ((p.n_out + 3) / 4);
  if (total == 0) return cudaSuccess;
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(splitk_reduce_kernel, dim3(blocks), dim3(256), 0, stream, 1, p);
}

// Failure-detection probe: waits on an mbarrier that nothing arrives on,
// bounded by ctl.wait_limit, then records kDevTimeoutConsumer and returns.
__global__ void wait_timeout_probe_kernel(DevCtl ctl) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!mbar_wait(smem_u32(&bar), 0, ctl.wait_limit, &abort_flag)) report(ctl, &abort_flag, kDevTimeoutConsumer);
    // Complete the phase so the barrier is not left pending at exit.
    mbar_arrive(smem_u32(&bar));
  }
  __syncthreads();
}

cudaError_t launch_wait_timeout_probe(DevCtl ctl, cudaStream_t stream) {
  wait_timeout_probe_kernel<<<1, 32, 0, stream>>>(ctl);
  return launched();
}

}  // namespace nq
