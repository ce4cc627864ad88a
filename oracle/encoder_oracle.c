/*
 * encoder_oracle.c -- CPU restatement of the reference's Parakeet
 * FastConformer encoder forward, batch 1 (the reference never batches).
 *
 * TEST INFRASTRUCTURE ONLY (see nq8_oracle.c): used by tests/ and bench.py's
 * CPU-baseline leg; the shipped library never links or calls it.
 *
 * Follows src/parakeet/fast_conformer.rs (dropbox/nspeech):
 *   relative_positional_encoding   :69-97
 *   ConvSubsampling::forward        :172-188  (conv0+ReLU, dw+pw+ReLU, dw+pw+ReLU,
 *                                              flatten c*F+f, linear)
 *   FeedForward::forward            :206-211  (linear1, SiLU, linear2)
 *   MultiHeadSelfAttention::forward :256-313  (q,k,v, k_rel = pos . W_rel^T,
 *                                              (q+u)k^T + rel_shift((q+v)k_rel^T),
 *                                              / sqrt(hd), softmax, . v, o_proj)
 *   rel_shift                       :407-425  (result[i][j] = x[i][T-1+j-i])
 *   ConvModule::forward             :471-494  (pw1, GLU a*sigmoid(b), depthwise,
 *                                              BatchNorm eval, SiLU, pw2)
 *   FastConformerBlock::forward_with_pos :967-999 (macaron x0.5 residuals)
 *   FastConformerEncoder::forward   :1072-1104 (x * sqrt(d) when scale_input)
 * LayerNorm / BatchNorm eps 1e-5 (f32 VarBuilder, :934, :451).
 * All activations f32.  Linears: weight_mode 0 = fast_matmul semantics
 * (dequantized Q8_0 rounded to bf16, src/fast_matmul.rs:191-208), 1 = exact
 * dequantized f32 weights (candle Linear on dequantized tensors,
 * src/parakeet/transducer.rs:1841-1865).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int feat_in, d_model, n_heads, ff_mult, n_layers, conv_kernel, sub_channels, scale_input;
} oq_enc_cfg;

typedef struct {
    const uint8_t *ff1_w1, *ff1_w2, *ff2_w1, *ff2_w2, *q, *k, *v, *o, *rel, *pw1, *pw2;
    const float *ff1_b1, *ff1_b2, *ff2_b1, *ff2_b2, *q_b, *k_b, *v_b, *o_b, *pw1_b, *pw2_b;
    const float *bias_u, *bias_v, *dw_w, *dw_b, *bn_g, *bn_b, *bn_mean, *bn_var;
    const float *ln_g[5], *ln_b[5]; /* ff1, self_att, conv, ff2, out */
} oq_enc_layer;

typedef struct {
    const float *c0_w, *c0_b, *dw2_w, *dw2_b, *dw5_w, *dw5_b, *pw3_b, *pw6_b, *lin_b;
    const uint8_t *pw3, *pw6, *lin;
    const oq_enc_layer *layers;
} oq_enc_weights;

extern void oq_dequant_q8_0(const uint8_t *blocks, int64_t n_rows, int64_t k, float *w);
extern uint16_t oq_f32_to_bf16(float f);
extern float oq_bf16_to_f32(uint16_t b);

static int g_weight_mode = 0;

static float *dq(const uint8_t *blocks, int64_t n, int64_t k) {
    float *w = (float *)malloc(sizeof(float) * (size_t)(n * k));
    oq_dequant_q8_0(blocks, n, k, w);
    if (g_weight_mode == 0)
        for (int64_t i = 0; i < n * k; i++) w[i] = oq_bf16_to_f32(oq_f32_to_bf16(w[i]));
    return w;
}

/* y[m, n] = x[m, :] . W[n, :] + b[n] */
static void linear(const float *x, int64_t m, int64_t k, const uint8_t *wq, int64_t n, const float *b, float *y) {
    float *w = dq(wq, n, k);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < m; i++)
        for (int64_t j = 0; j < n; j++) {
            const float *xr = x + i * k, *wr = w + j * k;
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int64_t t = 0;
            for (; t + 8 <= k; t += 8)
                for (int e = 0; e < 8; e++) acc[e] += xr[t + e] * wr[t + e];
            float s = 0.f;
            for (int e = 0; e < 8; e++) s += acc[e];
            for (; t < k; t++) s += xr[t] * wr[t];
            y[i * n + j] = s + (b ? b[j] : 0.f);
        }
    free(w);
}

static float sigm(float v) { return 1.0f / (1.0f + expf(-v)); }

static void layernorm(const float *x, int64_t m, int64_t d, const float *g, const float *b, float *y) {
    for (int64_t i = 0; i < m; i++) {
        const float *xr = x + i * d;
        double s = 0;
        for (int64_t j = 0; j < d; j++) s += xr[j];
        float mean = (float)(s / d);
        double q = 0;
        for (int64_t j = 0; j < d; j++) q += (double)(xr[j] - mean) * (xr[j] - mean);
        float rstd = 1.0f / sqrtf((float)(q / d) + 1e-5f);
        for (int64_t j = 0; j < d; j++) y[i * d + j] = (xr[j] - mean) * rstd * g[j] + b[j];
    }
}

static int sub_len(int L) { return L <= 0 ? 0 : (L - 1) / 2 + 1; }

/* Depthwise 3x3 stride-2 pad-1 conv on [C][T][F] (NCHW, batch 1). */
static void dw3x3s2(const float *in, int C, int T, int F, const float *w, const float *b, float *out, int To, int Fo) {
#pragma omp parallel for schedule(static)
    for (int c = 0; c < C; c++)
        for (int t = 0; t < To; t++)
            for (int f = 0; f < Fo; f++) {
                float acc = b[c];
                for (int dt = 0; dt < 3; dt++) {
                    int ti = 2 * t - 1 + dt;
                    if (ti < 0 || ti >= T) continue;
                    for (int df = 0; df < 3; df++) {
                        int fi = 2 * f - 1 + df;
                        if (fi < 0 || fi >= F) continue;
                        acc += w[c * 9 + dt * 3 + df] * in[((size_t)c * T + ti) * F + fi];
                    }
                }
                out[((size_t)c * To + t) * Fo + f] = acc;
            }
}

/* Pointwise conv (1x1) C->C + ReLU on NCHW [C][P]: y[co][p] = relu(sum_ci W[co][ci] x[ci][p] + b). */
static void pw_relu(const float *in, int C, int P, const uint8_t *wq, const float *b, float *out) {
    /* transpose to [P][C], linear, transpose back */
    float *xt = (float *)malloc(sizeof(float) * (size_t)P * C);
    float *yt = (float *)malloc(sizeof(float) * (size_t)P * C);
    for (int c = 0; c < C; c++)
        for (int p = 0; p < P; p++) xt[(size_t)p * C + c] = in[(size_t)c * P + p];
    linear(xt, P, C, wq, C, b, yt);
    for (int c = 0; c < C; c++)
        for (int p = 0; p < P; p++) {
            float v = yt[(size_t)p * C + c];
            out[(size_t)c * P + p] = v > 0.f ? v : 0.f;
        }
    free(xt);
    free(yt);
}

void oq_encoder_set_weight_mode(int mode) { g_weight_mode = mode; }

/* mel [t_mel][feat_in] -> out [T3][d_model]; returns T3. */
int oq_encoder_forward(const oq_enc_cfg *cfg, const oq_enc_weights *W, const float *mel, int t_mel, float *out) {
    const int F = cfg->feat_in, C = cfg->sub_channels, D = cfg->d_model, H = cfg->n_heads;
    const int hd = D / H, FF = D * cfg->ff_mult, K = cfg->conv_kernel;
    const int T1 = sub_len(t_mel), F1 = sub_len(F), T2 = sub_len(T1), F2 = sub_len(F1), T3 = sub_len(T2), F3 = sub_len(F2);
    /* ---- subsampling */
    float *a1 = (float *)calloc((size_t)C * T1 * F1, sizeof(float));
#pragma omp parallel for schedule(static)
    for (int c = 0; c < C; c++)
        for (int t = 0; t < T1; t++)
            for (int f = 0; f < F1; f++) {
                float acc = W->c0_b[c];
                for (int dt = 0; dt < 3; dt++) {
                    int ti = 2 * t - 1 + dt;
                    if (ti < 0 || ti >= t_mel) continue;
                    for (int df = 0; df < 3; df++) {
                        int fi = 2 * f - 1 + df;
                        if (fi < 0 || fi >= F) continue;
                        acc += W->c0_w[c * 9 + dt * 3 + df] * mel[(size_t)ti * F + fi];
                    }
                }
                a1[((size_t)c * T1 + t) * F1 + f] = acc > 0.f ? acc : 0.f;
            }
    float *a2 = (float *)malloc(sizeof(float) * (size_t)C * T2 * F2);
    dw3x3s2(a1, C, T1, F1, W->dw2_w, W->dw2_b, a2, T2, F2);
    float *a3 = (float *)malloc(sizeof(float) * (size_t)C * T2 * F2);
    pw_relu(a2, C, T2 * F2, W->pw3, W->pw3_b, a3);
    float *a4 = (float *)malloc(sizeof(float) * (size_t)C * T3 * F3);
    dw3x3s2(a3, C, T2, F2, W->dw5_w, W->dw5_b, a4, T3, F3);
    float *a5 = (float *)malloc(sizeof(float) * (size_t)C * T3 * F3);
    pw_relu(a4, C, T3 * F3, W->pw6, W->pw6_b, a5);
    float *flat = (float *)malloc(sizeof(float) * (size_t)T3 * C * F3);
    for (int t = 0; t < T3; t++)
        for (int c = 0; c < C; c++)
            for (int f = 0; f < F3; f++) flat[(size_t)t * C * F3 + c * F3 + f] = a5[((size_t)c * T3 + t) * F3 + f];
    float *x = (float *)malloc(sizeof(float) * (size_t)T3 * D);
    linear(flat, T3, (int64_t)C * F3, W->lin, D, W->lin_b, x);
    free(a1); free(a2); free(a3); free(a4); free(a5); free(flat);
    if (cfg->scale_input) {
        float s = (float)sqrt((double)D);
        for (int64_t i = 0; i < (int64_t)T3 * D; i++) x[i] *= s;
    }
    /* ---- relative positions [2T-1][D] */
    const int P = 2 * T3 - 1;
    float *pos = (float *)malloc(sizeof(float) * (size_t)P * D);
    for (int idx = 0; idx < P; idx++) {
        int p = idx - (T3 - 1);
        float ap = fabsf((float)p), sign = p > 0 ? -1.f : 1.f;
        for (int i = 0; i < D / 2; i++) {
            float div = ap / powf(10000.0f, 2.0f * (float)i / (float)D);
            pos[(size_t)idx * D + 2 * i] = sign * sinf(div);
            pos[(size_t)idx * D + 2 * i + 1] = cosf(div);
        }
    }
    float *h = (float *)malloc(sizeof(float) * (size_t)T3 * D);
    float *tt = (float *)malloc(sizeof(float) * (size_t)T3 * FF);
    float *u = (float *)malloc(sizeof(float) * (size_t)T3 * D);
    float *q = (float *)malloc(sizeof(float) * (size_t)T3 * D);
    float *kk = (float *)malloc(sizeof(float) * (size_t)T3 * D);
    float *vv = (float *)malloc(sizeof(float) * (size_t)T3 * D);
    float *kr = (float *)malloc(sizeof(float) * (size_t)P * D);
    float *ctx = (float *)malloc(sizeof(float) * (size_t)T3 * D);
    float *g2 = (float *)malloc(sizeof(float) * (size_t)T3 * 2 * D);
    float *gl = (float *)malloc(sizeof(float) * (size_t)T3 * D);
    float *cv = (float *)malloc(sizeof(float) * (size_t)T3 * D);
    const float inv_scale = 1.0f / (float)sqrt((double)hd);

    for (int li = 0; li < cfg->n_layers; li++) {
        const oq_enc_layer *L = &W->layers[li];
        /* FF1 */
        layernorm(x, T3, D, L->ln_g[0], L->ln_b[0], h);
        linear(h, T3, D, L->ff1_w1, FF, L->ff1_b1, tt);
        for (int64_t i = 0; i < (int64_t)T3 * FF; i++) tt[i] = tt[i] * sigm(tt[i]);
        linear(tt, T3, FF, L->ff1_w2, D, L->ff1_b2, u);
        for (int64_t i = 0; i < (int64_t)T3 * D; i++) x[i] += 0.5f * u[i];
        /* MHSA */
        layernorm(x, T3, D, L->ln_g[1], L->ln_b[1], h);
        linear(h, T3, D, L->q, D, L->q_b, q);
        linear(h, T3, D, L->k, D, L->k_b, kk);
        linear(h, T3, D, L->v, D, L->v_b, vv);
        linear(pos, P, D, L->rel, D, NULL, kr);
#pragma omp parallel for schedule(static)
        for (int hh = 0; hh < H; hh++) {
            float *sc = (float *)malloc(sizeof(float) * (size_t)T3);
            for (int i = 0; i < T3; i++) {
                const float *qi = q + (size_t)i * D + hh * hd;
                float mx = -INFINITY;
                for (int j = 0; j < T3; j++) {
                    const float *kj = kk + (size_t)j * D + hh * hd;
                    const float *rj = kr + (size_t)(T3 - 1 + j - i) * D + hh * hd;
                    float ac = 0.f, bd = 0.f;
                    for (int e = 0; e < hd; e++) {
                        ac += (qi[e] + L->bias_u[hh * hd + e]) * kj[e];
                        bd += (qi[e] + L->bias_v[hh * hd + e]) * rj[e];
                    }
                    sc[j] = (ac + bd) * inv_scale;
                    if (sc[j] > mx) mx = sc[j];
                }
                float sum = 0.f;
                for (int j = 0; j < T3; j++) {
                    sc[j] = expf(sc[j] - mx);
                    sum += sc[j];
                }
                for (int e = 0; e < hd; e++) {
                    float acc = 0.f;
                    for (int j = 0; j < T3; j++) acc += sc[j] * vv[(size_t)j * D + hh * hd + e];
                    ctx[(size_t)i * D + hh * hd + e] = acc / sum;
                }
            }
            free(sc);
        }
        linear(ctx, T3, D, L->o, D, L->o_b, u);
        for (int64_t i = 0; i < (int64_t)T3 * D; i++) x[i] += u[i];
        /* Conv module */
        layernorm(x, T3, D, L->ln_g[2], L->ln_b[2], h);
        linear(h, T3, D, L->pw1, 2 * D, L->pw1_b, g2);
        for (int t = 0; t < T3; t++)
            for (int c = 0; c < D; c++)
                gl[(size_t)t * D + c] = g2[(size_t)t * 2 * D + c] * sigm(g2[(size_t)t * 2 * D + D + c]);
        for (int t = 0; t < T3; t++)
            for (int c = 0; c < D; c++) {
                float acc = L->dw_b[c];
                for (int i = 0; i < K; i++) {
                    int ts = t - K / 2 + i;
                    if (ts < 0 || ts >= T3) continue;
                    acc += L->dw_w[c * K + i] * gl[(size_t)ts * D + c];
                }
                float y = (acc - L->bn_mean[c]) / sqrtf(L->bn_var[c] + 1e-5f) * L->bn_g[c] + L->bn_b[c];
                cv[(size_t)t * D + c] = y * sigm(y);
            }
        linear(cv, T3, D, L->pw2, D, L->pw2_b, u);
        for (int64_t i = 0; i < (int64_t)T3 * D; i++) x[i] += u[i];
        /* FF2 */
        layernorm(x, T3, D, L->ln_g[3], L->ln_b[3], h);
        linear(h, T3, D, L->ff2_w1, FF, L->ff2_b1, tt);
        for (int64_t i = 0; i < (int64_t)T3 * FF; i++) tt[i] = tt[i] * sigm(tt[i]);
        linear(tt, T3, FF, L->ff2_w2, D, L->ff2_b2, u);
        for (int64_t i = 0; i < (int64_t)T3 * D; i++) x[i] += 0.5f * u[i];
        layernorm(x, T3, D, L->ln_g[4], L->ln_b[4], h);
        memcpy(x, h, sizeof(float) * (size_t)T3 * D);
    }
    memcpy(out, x, sizeof(float) * (size_t)T3 * D);
    free(x); free(pos); free(h); free(tt); free(u); free(q); free(kk); free(vv); free(kr); free(ctx);
    free(g2); free(gl); free(cv);
    return T3;
}
