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
  const __nv_bfloat16 *qkv;  // q already holds q + u
  const float *vrel;    // [H][2 Tp - 1]: (v_h - u_h) . r_p of this layer (launch_relpos_bias)
  const int *len;       // [B] valid frames per segment
  __nv_bfloat16 *out;
  int B;
  int Tp;
  int D;
  int rel_col0;
  float sl2;  // log2(e) / sqrt(head dim)
  DevCtl ctl;
};

// Largest padded segment length (encoder frames) the kernel takes.
int attention_tc_max_tp();
size_t attention_tc_smem_bytes(int Tp);
// Persistent launch: min(work items, sm_count) CTAs, one per SM.
cudaError_t launch_relpos_attention_tc(const CUtensorMap &tm_qkv, const CUtensorMap &tm_rel, const AttnTcParams &p,
                                       int sm_count, cudaStream_t stream);
// vrel[li][h][p] = vmu[li][h hd : +hd] . krel[p][li D + h hd : +hd] for every
// layer li and head h; krel [nrel][n_layers D] bf16, vmu [n_layers][D] f32
// (bias_v - bias_u), vrel [n_layers][D / hd][nrel] f32.
cudaError_t launch_relpos_bias(const __nv_bfloat16 *krel, const float *vmu, int nrel, int n_layers, int D,
                               float *vrel, cudaStream_t stream);

}  // namespace nq
