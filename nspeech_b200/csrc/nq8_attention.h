// nq8_attention.h -- launch interface of the tcgen05 relative-position
// attention (internal).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>

#include "nq8_common.cuh"

namespace nq {

// qkv [B * Tp, 3 D] bf16 (q | k | v) through tm_qkv (box 64 x 64, 128-byte
// swizzle); relative keys through tm_rel (rows 2 Tp - 1, this layer's columns
// from rel_col0; same box); out [B * Tp, D] bf16.
struct AttnTcParams {
  const __nv_bfloat16 *qkv;
  const float *bias_u;  // [D]
  const float *bias_v;  // [D]
  const int *len;       // [B] valid frames per segment
  __nv_bfloat16 *out;
  int Tp;
  int D;
  int rel_col0;
  float sl2;  // log2(e) / sqrt(head dim)
  DevCtl ctl;
};

size_t attention_tc_smem_bytes();
cudaError_t launch_relpos_attention_tc(const CUtensorMap &tm_qkv, const CUtensorMap &tm_rel, const AttnTcParams &p,
                                       int B, int H, cudaStream_t stream);

}  // namespace nq
