// nq8_encoder.h -- launch interfaces of the encoder glue kernels (internal).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace nq {
namespace enc {

constexpr int kLnScale = 0;      // x = alpha * u (f32); h = LN1(x)
constexpr int kLnResAdd = 1;     // x += alpha * u (bf16); h = LN1(x)
constexpr int kLnResAddOut = 2;  // x = LN1(x + alpha * u); h = LN2(x) if LN2 given

cudaError_t conv0_relu(const float *mel, const int *len0, int B, int T, int F, int T1, int F1, int C, const float *w,
                       const float *bias, __nv_bfloat16 *out, cudaStream_t s);
// conv0_relu followed by the first dwconv2d_s2, without the intermediate in
// HBM (identical results); supported when C % 64 == 0 and the staged rows fit.
bool conv0_dw_s2_supported(int F, int F1, int C);
cudaError_t conv0_dw_s2(const float *mel, const int *len0, const int *len1, int B, int T, int F, int T1, int F1, int T2,
                        int F2, int C, const float *w0, const float *b0, const float *w2, const float *b2,
                        __nv_bfloat16 *out, cudaStream_t s);
cudaError_t dwconv2d_s2(const __nv_bfloat16 *in, const int *len_in, int B, int Tin, int Fin, int Tout, int Fout, int C,
                        const float *w, const float *bias, __nv_bfloat16 *out, cudaStream_t s);
cudaError_t flatten_cf(const __nv_bfloat16 *in, int rows, int F, int C, __nv_bfloat16 *out, cudaStream_t s);
cudaError_t ln_rows(int mode, float *x, const void *u, float alpha, int rows, int D, const float *g1, const float *b1,
                    const float *g2, const float *b2, __nv_bfloat16 *h, float eps, cudaStream_t s);
cudaError_t dwconv1d_bn_silu(const __nv_bfloat16 *in, const int *len, int B, int Tp, int D, int K, const float *w,
                             const float *bias, const float *bn_scale, const float *bn_shift, __nv_bfloat16 *out,
                             cudaStream_t s);
cudaError_t relpos(int T, int D, __nv_bfloat16 *pos, cudaStream_t s);
// krel: relative keys [2 Tp - 1] rows of stride ldr elements (this layer's D columns).
cudaError_t relpos_attention(const __nv_bfloat16 *qkv, const __nv_bfloat16 *krel, int64_t ldr, const float *bias_u,
                             const float *bias_v, const int *len, int B, int Tp, int H, int D, __nv_bfloat16 *out,
                             cudaStream_t s);
// out[b, t, :] = x[b, t, :] for t < len[b], else 0 (f32 rows of D).
cudaError_t copy_masked(const float *x, const int *len, int B, int Tp, int D, float *out, cudaStream_t s);

}  // namespace enc

// The encoder's attention on the kernel nq_set_attention_kernel selects: the
// tcgen05 kernel (nq8_attention.cu, tensor maps encoded on the current
// device) when attention_tc(Tp), else enc::relpos_attention; timed as
// NQ_KCLASS_ATTENTION when profiling.  The q columns of qkv hold q + u (the
// encoder folds u into the q projection's bias); the tcgen05 kernel takes
// vrel, this layer's [H][2 Tp - 1] table of (v - u) . r from relpos_bias, and
// enc::relpos_attention gets bias_u = 0 and bias_v = v - u.  Return NQ_*
// codes.
bool attention_tc(int Tp);
// enc::ln_rows, timed as NQ_KCLASS_NORM when profiling; returns an NQ_* code.
int layer_norm_rows(int mode, float *x, const void *u, float alpha, int rows, int D, const float *g1, const float *b1,
                    const float *g2, const float *b2, __nv_bfloat16 *h, float eps, cudaStream_t s);
int relpos_bias(const __nv_bfloat16 *krel, const float *vmu, int nrel, int n_layers, int D, float *vrel,
                cudaStream_t s);
int relpos_attention(const __nv_bfloat16 *qkv, const __nv_bfloat16 *krel, int64_t ldr, const float *bias_u,
                     const float *bias_v, const float *vrel, const int *len, int B, int Tp, int H, int D,
                     __nv_bfloat16 *out, cudaStream_t s);
}  // namespace nq
