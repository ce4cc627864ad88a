// nq8_common.cuh -- shared device helpers for the sm_100a Q8_0 kernels
// (packed weight layout: nq8_layout.h).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "nq8_layout.h"

namespace nq {

// Host side: count one kernel launch of this library (process-wide counter
// read by nq_launch_counter); `launched()` closes a <<<>>> launch with it.
void note_launch();
inline cudaError_t launched() {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) note_launch();
  return e;
}

// Programmatic dependent launch.  Kernels of this library start with
// pdl_wait() before their first global-memory access (and pdl_trigger()
// after it), so they may be launched with programmatic stream serialization:
// a launch then overlaps its launch latency and prologue with the tail of
// the previous kernel on the stream, and waits for that kernel's completion
// (and memory) before touching data.  A predecessor that never triggers
// completes first, as without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch `kern` with programmatic stream serialization (plus an optional
// cluster shape); counts the launch.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       unsigned cluster_x, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster_x > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    n = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<Args &&>(args)...);
  if (e == cudaSuccess) note_launch();
  return e;
}

// Device status bits (mirrors NQ_DEV_* in include/nq8.h).
constexpr int kDevTimeoutProducer = 0x1;
constexpr int kDevTimeoutConsumer = 0x2;
constexpr int kDevTimeoutMma = 0x4;
constexpr int kDevTimeoutEpilogue = 0x8;
constexpr int kDevTimeoutDrain = 0x10;

// Control block handed to every kernel: where to report, how long to wait.
struct DevCtl {
  int *status;           // device status word (OR of kDev* bits)
  long long wait_limit;  // cycles a bounded wait may spin before giving up
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or about `ns` nanoseconds pass, instead of spinning (a
// spinning waiter takes issue slots from the warps doing the work).
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Wait for the phase of parity `parity` to complete, for at most `limit`
// cycles, or until another role raised *abort.  Returns false on give-up; the
// caller then records its kDev* bit and unwinds (never traps).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, long long limit,
                                          volatile int *abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 200000u)) return true;  // <= ~0.2 ms asleep per try
    if (*abort) return false;
    if (clock64() - t0 > limit) return false;
  }
}

__device__ __forceinline__ void report(const DevCtl &ctl, volatile int *abort, int bit) {
  *abort = 1;
  atomicOr(ctl.status, bit);
}

// ------------------------------------------------------------- bulk copies
// 1-D bulk copy global -> shared (16-B aligned addresses, size % 16 == 0).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                          uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}
// 2-D tiled tensor copy global -> shared (no multicast).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (tensor core operand reads, bulk copies).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, bf16 inputs, f32 accumulate, one thread.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 lanes x 32 consecutive f32 columns: thread t gets lane (base lane + t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
      "[%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand stored with the
// 128-byte swizzle: rows of 128 B (64 bf16), 8-row atoms 1024 B apart.
// Bits: start>>4 [0,14), LBO>>4 [16,30) (unused for this layout),
// SBO>>4 [32,46), version 1 [46,48), layout SWIZZLE_128B = 2 [61,64).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: A, B bf16 (K-major),
// D f32, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4)                                   // D format f32
         | (1u << 7)                                 // A format bf16
         | (1u << 10)                                // B format bf16
         | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

// Byte offset of element (row, k) inside a K-major SWIZZLE_128B tile whose
// rows hold 64 bf16: the 16-B chunk index is XORed with (row % 8).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk16) {
  return row * 128u + ((chunk16 ^ (row & 7u)) << 4);
}

// ------------------------------------------------------------ conversions
// Four packed int8 -> four exact floats, by placing each byte (biased by 128)
// in the mantissa of 2^23 and subtracting 2^23 + 128.
__device__ __forceinline__ void s8x4_to_f32(uint32_t q4, float (&f)[4]) {
  const uint32_t u = q4 ^ 0x80808080u;
  f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)) - 8388736.0f;
  f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)) - 8388736.0f;
  f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)) - 8388736.0f;
  f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)) - 8388736.0f;
}
// Round two floats to bf16 (RNE) and pack: `lo` in bits [0,16).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b16) { return __uint_as_float(b16 << 16); }

// Four int8 of one Q8_0 block times its f16 scale d, rounded to bf16 exactly
// as bf16(f32(d) * q) (the product is exact in f32): two packed bf16x2.
__device__ __forceinline__ void dequant4_bf16(uint32_t q4, float d, uint32_t &p01, uint32_t &p23) {
  float f[4];
  s8x4_to_f32(q4, f);
  p01 = pack_bf16x2(f[0] * d, f[1] * d);
  p23 = pack_bf16x2(f[2] * d, f[3] * d);
}

// Packed f32x2 helpers and an eight-element Q8_0 dequantization with the
// same exact result as dequant4_bf16, in fewer instructions.
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


// Four int8 (one word) of one Q8_0 block -> two bf16x2 of bf16(f32(d) * q)
// with the mixed-precision FMA (f16 operands, f32 result): a byte u' = q + 128
// placed in the mantissa of f16 1024 gives the exact f16 value 1024 + u', and
// fma((1024 + u'), d, -1152 d) = q d exactly (-1152 d is exact in f32 for an
// f16 d; the sum needs at most 18 significant bits), so the single rounding
// is the final cvt to bf16.  d16: the f16 bits of d; c: -1152 * f32(d).
__device__ __forceinline__ void dequant4_bf16_mix(uint32_t w, uint16_t d16, float c, uint32_t &p01,
                                                  uint32_t &p23) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t h01 = __byte_perm(u, 0x64646464u, 0x4140);  // f16x2 (1024 + u'0, 1024 + u'1)
  const uint32_t h23 = __byte_perm(u, 0x64646464u, 0x4342);  // f16x2 (1024 + u'2, 1024 + u'3)
  float r0, r1, r2, r3;
  asm("{\n\t.reg .f16 a0, a1, a2, a3, dd;\n\t"
      "mov.b32 {a0, a1}, %4;\n\t"
      "mov.b32 {a2, a3}, %5;\n\t"
      "mov.b16 dd, %6;\n\t"
      "fma.rn.f32.f16 %0, a0, dd, %7;\n\t"
      "fma.rn.f32.f16 %1, a1, dd, %7;\n\t"
      "fma.rn.f32.f16 %2, a2, dd, %7;\n\t"
      "fma.rn.f32.f16 %3, a3, dd, %7;\n\t}"
      : "=f"(r0), "=f"(r1), "=f"(r2), "=f"(r3)
      : "r"(h01), "r"(h23), "h"(d16), "f"(c));
  p01 = pack_bf16x2(r0, r1);
  p23 = pack_bf16x2(r2, r3);
}

// Legacy warp-level MMA (used by the skinny GEMV where the tensor pipe is not
// the bound): D(16x8) += A(16x16) . B(16x8), bf16 in, f32 accumulate.
__device__ __forceinline__ void mma_16816_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ----------------------------------------------------------- epilogue math
enum Epi : int { kEpiNone = 0, kEpiSilu = 1, kEpiGeluErf = 2, kEpiGluSigmoid = 3, kEpiGluSilu = 4, kEpiRelu = 5 };

__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + __expf(-v)); }

// Non-GLU activation of a biased value.
__device__ __forceinline__ float act_single(int epi, float v) {
  if (epi == kEpiSilu) return v * sigmoidf_(v);
  if (epi == kEpiGeluErf) return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
  if (epi == kEpiRelu) return fmaxf(v, 0.0f);
  return v;
}
// GLU: value * act(gate).
__device__ __forceinline__ float act_glu(int epi, float value, float gate) {
  if (epi == kEpiGluSigmoid) return value * sigmoidf_(gate);
  return value * (gate * sigmoidf_(gate));
}

__device__ __forceinline__ void store_out(void *y, int y_dtype, int64_t idx, float v) {
  if (y_dtype == 0) {
    static_cast<float *>(y)[idx] = v;
  } else {
    static_cast<__nv_bfloat16 *>(y)[idx] = __float2bfloat16_rn(v);
  }
}

}  // namespace nq
