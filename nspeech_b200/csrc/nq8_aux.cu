// nq8_aux.cu -- small helper kernels of the Q8_0 path.
#include "nq8_common.cuh"
#include "nq8_kernels.h"

namespace nq {

// hi[m, k] = bf16(x), lo[m, k] = bf16(x - hi); rows of k_pad, zero for k >= K.
// Four consecutive k per thread (8-byte stores).
__global__ void split_x_kernel(const void *__restrict__ x, int x_dtype, int64_t ldx, int64_t M, int64_t K,
                               int64_t k_pad, __nv_bfloat16 *__restrict__ hi, __nv_bfloat16 *__restrict__ lo) {
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
  split_x_kernel<<<blocks, 256, 0, stream>>>(x, x_dtype, ldx, M, K, k_pad, hi, lo);
  return cudaGetLastError();
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
  return cudaGetLastError();
}

}  // namespace nq
