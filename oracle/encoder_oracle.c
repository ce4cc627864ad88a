/*
 * encoder_oracle.c -- CPU restatement of the reference's Parakeet
 * FastConformer encoder forward, batch 1 (the reference never batches).
 *
 * TEST INFRASTRUCTURE AND CPU BASELINE ONLY (see nq8_oracle.c): used by
 * tests/ as the checker and by bench.py's CPU-baseline and reference legs;
 * the shipped library never links or calls it.
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
 * (dequantized Q8_0 rounded to bf16 and packed once, src/fast_matmul.rs:
 * 191-208, multiplied by fbgemm_cpu.c's FbgemmBf16Op restatement), 1 = exact
 * dequantized f32 weights (candle Linear on dequantized tensors,
 * src/parakeet/transducer.rs:1841-1865).
 *
 * A model is prepared once (every linear packed, as the reference packs at
 * load time) and run many times; attention runs as blocked f32 GEMMs per
 * (head, 32-query block), as candle's matmuls do in the reference.
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

typedef struct ofb_mat ofb_mat;
extern ofb_mat *ofb_pack_q8_0(const uint8_t *blocks, int64_t n, int64_t k, int bf16);
extern ofb_mat *ofb_pack_f32_kn(const float *b, int64_t k, int64_t n, int64_t ldb);
extern ofb_mat *ofb_pack_f32_nk_strided(const float *b, int64_t n, int64_t k, int64_t ldb);
extern void ofb_free(ofb_mat *m);
extern void ofb_linear(const ofb_mat *mat, const float *x, int64_t m, int64_t ldx, const float *bias, float *y,
                       int64_t ldy);
extern void ofb_linear_serial(const ofb_mat *mat, const float *x, int64_t m, int64_t ldx, const float *bias,
                              float *y, int64_t ldy);

typedef struct {
    ofb_mat *ff1_w1, *ff1_w2, *ff2_w1, *ff2_w2, *q, *k, *v, *o, *rel, *pw1, *pw2;
} oq_enc_layer_mats;

typedef struct {
    oq_enc_cfg cfg;
    oq_enc_weights W;        /* the caller's arrays (kept alive by the caller) */
    oq_enc_layer *layers;    /* copy of the caller's layer table */
    ofb_mat *pw3, *pw6, *lin;
    oq_enc_layer_mats *mats; /* packed linears per layer */
} oq_enc_model;

static int g_weight_mode = 0;

static float sigm(float v) { return 1.0f / (1.0f + expf(-v)); }

static void layernorm(const float *x, int64_t m, int64_t d, const float *g, const float *b, float *y) {
#pragma omp parallel for schedule(static)
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
static void pw_relu(const float *in, int C, int P, const ofb_mat *w, const float *b, float *out) {
    float *xt = (float *)malloc(sizeof(float) * (size_t)P * C);
    float *yt = (float *)malloc(sizeof(float) * (size_t)P * C);
#pragma omp parallel for schedule(static)
    for (int p = 0; p < P; p++)
        for (int c = 0; c < C; c++) xt[(size_t)p * C + c] = in[(size_t)c * P + p];
    ofb_linear(w, xt, P, C, b, yt, C);
#pragma omp parallel for schedule(static)
    for (int c = 0; c < C; c++)
        for (int p = 0; p < P; p++) {
            float v = yt[(size_t)p * C + c];
            out[(size_t)c * P + p] = v > 0.f ? v : 0.f;
        }
    free(xt);
    free(yt);
}

void oq_encoder_set_weight_mode(int mode) { g_weight_mode = mode; }

/* Pack every linear of the model once (bf16 for weight_mode 0, f32 for 1). */
oq_enc_model *oq_encoder_prepare(const oq_enc_cfg *cfg, const oq_enc_weights *W, int weight_mode) {
    const int C = cfg->sub_channels, D = cfg->d_model, FF = D * cfg->ff_mult;
    const int F3 = sub_len(sub_len(sub_len(cfg->feat_in)));
    const int bf = weight_mode == 0;
    oq_enc_model *m = (oq_enc_model *)calloc(1, sizeof(oq_enc_model));
    m->cfg = *cfg;
    m->W = *W;
    m->layers = (oq_enc_layer *)malloc(sizeof(oq_enc_layer) * (size_t)cfg->n_layers);
    memcpy(m->layers, W->layers, sizeof(oq_enc_layer) * (size_t)cfg->n_layers);
    m->W.layers = m->layers;
    m->pw3 = ofb_pack_q8_0(W->pw3, C, C, bf);
    m->pw6 = ofb_pack_q8_0(W->pw6, C, C, bf);
    m->lin = ofb_pack_q8_0(W->lin, D, (int64_t)C * F3, bf);
    m->mats = (oq_enc_layer_mats *)calloc((size_t)cfg->n_layers, sizeof(oq_enc_layer_mats));
    for (int li = 0; li < cfg->n_layers; li++) {
        const oq_enc_layer *L = &m->layers[li];
        oq_enc_layer_mats *M = &m->mats[li];
        M->ff1_w1 = ofb_pack_q8_0(L->ff1_w1, FF, D, bf);
        M->ff1_w2 = ofb_pack_q8_0(L->ff1_w2, D, FF, bf);
        M->ff2_w1 = ofb_pack_q8_0(L->ff2_w1, FF, D, bf);
        M->ff2_w2 = ofb_pack_q8_0(L->ff2_w2, D, FF, bf);
        M->q = ofb_pack_q8_0(L->q, D, D, bf);
        M->k = ofb_pack_q8_0(L->k, D, D, bf);
        M->v = ofb_pack_q8_0(L->v, D, D, bf);
        M->o = ofb_pack_q8_0(L->o, D, D, bf);
        M->rel = ofb_pack_q8_0(L->rel, D, D, bf);
        M->pw1 = ofb_pack_q8_0(L->pw1, 2 * D, D, bf);
        M->pw2 = ofb_pack_q8_0(L->pw2, D, D, bf);
    }
    return m;
}

void oq_encoder_release(oq_enc_model *m) {
    if (!m) return;
    for (int li = 0; li < m->cfg.n_layers; li++) {
        oq_enc_layer_mats *M = &m->mats[li];
        ofb_mat *all[] = {M->ff1_w1, M->ff1_w2, M->ff2_w1, M->ff2_w2, M->q, M->k, M->v, M->o, M->rel, M->pw1, M->pw2};
        for (size_t i = 0; i < sizeof(all) / sizeof(all[0]); i++) ofb_free(all[i]);
    }
    ofb_free(m->pw3);
    ofb_free(m->pw6);
    ofb_free(m->lin);
    free(m->mats);
    free(m->layers);
    free(m);
}

#define QB 32 /* query rows per attention task */

/* Rel-pos MHSA core for one layer: ctx[T][D] from q, k, v [T][D] and kr [P][D]. */
static void attention(const oq_enc_layer *L, int T, int D, int H, const float *q, const float *kk, const float *vv,
                      const float *kr, float *ctx) {
    const int hd = D / H, P = 2 * T - 1;
    const float inv_scale = 1.0f / (float)sqrt((double)hd);
    ofb_mat **kp = (ofb_mat **)calloc((size_t)H, sizeof(ofb_mat *));
    ofb_mat **rp = (ofb_mat **)calloc((size_t)H, sizeof(ofb_mat *));
    ofb_mat **vp = (ofb_mat **)calloc((size_t)H, sizeof(ofb_mat *));
#pragma omp parallel for schedule(static)
    for (int h = 0; h < H; h++) {
        kp[h] = ofb_pack_f32_nk_strided(kk + h * hd, T, hd, D); /* AC: N = keys, K = hd */
        rp[h] = ofb_pack_f32_nk_strided(kr + h * hd, P, hd, D); /* BD: N = rel positions */
        vp[h] = ofb_pack_f32_kn(vv + h * hd, T, hd, D);         /* PV: N = hd, K = keys */
    }
    const int nb = (T + QB - 1) / QB;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int h = 0; h < H; h++)
        for (int b = 0; b < nb; b++) {
            const int i0 = b * QB, rows = T - i0 < QB ? T - i0 : QB;
            float *qu = (float *)malloc(sizeof(float) * QB * hd);
            float *qv = (float *)malloc(sizeof(float) * QB * hd);
            float *ac = (float *)malloc(sizeof(float) * QB * (size_t)T);
            float *bd = (float *)malloc(sizeof(float) * QB * (size_t)P);
            float *o = (float *)malloc(sizeof(float) * QB * hd);
            float sums[QB];
            for (int r = 0; r < rows; r++)
                for (int e = 0; e < hd; e++) {
                    float x = q[(size_t)(i0 + r) * D + h * hd + e];
                    qu[r * hd + e] = x + L->bias_u[h * hd + e];
                    qv[r * hd + e] = x + L->bias_v[h * hd + e];
                }
            ofb_linear_serial(kp[h], qu, rows, hd, NULL, ac, T);
            ofb_linear_serial(rp[h], qv, rows, hd, NULL, bd, P);
            for (int r = 0; r < rows; r++) {
                const int i = i0 + r;
                float *s = ac + (size_t)r * T;
                const float *br = bd + (size_t)r * P;
                float mx = -INFINITY;
                for (int j = 0; j < T; j++) {
                    s[j] = (s[j] + br[T - 1 + j - i]) * inv_scale;
                    if (s[j] > mx) mx = s[j];
                }
                float sum = 0.f;
                for (int j = 0; j < T; j++) {
                    s[j] = expf(s[j] - mx);
                    sum += s[j];
                }
                sums[r] = sum;
            }
            ofb_linear_serial(vp[h], ac, rows, T, NULL, o, hd);
            for (int r = 0; r < rows; r++)
                for (int e = 0; e < hd; e++) ctx[(size_t)(i0 + r) * D + h * hd + e] = o[r * hd + e] / sums[r];
            free(qu);
            free(qv);
            free(ac);
            free(bd);
            free(o);
        }
    for (int h = 0; h < H; h++) {
        ofb_free(kp[h]);
        ofb_free(rp[h]);
        ofb_free(vp[h]);
    }
    free(kp);
    free(rp);
    free(vp);
}

/* mel [t_mel][feat_in] -> out [T3][d_model]; returns T3. */
int oq_encoder_run(const oq_enc_model *model, const float *mel, int t_mel, float *out) {
    const oq_enc_cfg *cfg = &model->cfg;
    const oq_enc_weights *W = &model->W;
    const int F = cfg->feat_in, C = cfg->sub_channels, D = cfg->d_model, H = cfg->n_heads;
    const int FF = D * cfg->ff_mult, K = cfg->conv_kernel;
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
    pw_relu(a2, C, T2 * F2, model->pw3, W->pw3_b, a3);
    float *a4 = (float *)malloc(sizeof(float) * (size_t)C * T3 * F3);
    dw3x3s2(a3, C, T2, F2, W->dw5_w, W->dw5_b, a4, T3, F3);
    float *a5 = (float *)malloc(sizeof(float) * (size_t)C * T3 * F3);
    pw_relu(a4, C, T3 * F3, model->pw6, W->pw6_b, a5);
    float *flat = (float *)malloc(sizeof(float) * (size_t)T3 * C * F3);
    for (int t = 0; t < T3; t++)
        for (int c = 0; c < C; c++)
            for (int f = 0; f < F3; f++) flat[(size_t)t * C * F3 + c * F3 + f] = a5[((size_t)c * T3 + t) * F3 + f];
    float *x = (float *)malloc(sizeof(float) * (size_t)T3 * D);
    ofb_linear(model->lin, flat, T3, (int64_t)C * F3, W->lin_b, x, D);
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
    const int64_t TD = (int64_t)T3 * D, TF = (int64_t)T3 * FF;

    for (int li = 0; li < cfg->n_layers; li++) {
        const oq_enc_layer *L = &model->layers[li];
        const oq_enc_layer_mats *M = &model->mats[li];
        /* FF1 */
        layernorm(x, T3, D, L->ln_g[0], L->ln_b[0], h);
        ofb_linear(M->ff1_w1, h, T3, D, L->ff1_b1, tt, FF);
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < TF; i++) tt[i] = tt[i] * sigm(tt[i]);
        ofb_linear(M->ff1_w2, tt, T3, FF, L->ff1_b2, u, D);
        for (int64_t i = 0; i < TD; i++) x[i] += 0.5f * u[i];
        /* MHSA */
        layernorm(x, T3, D, L->ln_g[1], L->ln_b[1], h);
        ofb_linear(M->q, h, T3, D, L->q_b, q, D);
        ofb_linear(M->k, h, T3, D, L->k_b, kk, D);
        ofb_linear(M->v, h, T3, D, L->v_b, vv, D);
        ofb_linear(M->rel, pos, P, D, NULL, kr, D);
        attention(L, T3, D, H, q, kk, vv, kr, ctx);
        ofb_linear(M->o, ctx, T3, D, L->o_b, u, D);
        for (int64_t i = 0; i < TD; i++) x[i] += u[i];
        /* Conv module */
        layernorm(x, T3, D, L->ln_g[2], L->ln_b[2], h);
        ofb_linear(M->pw1, h, T3, D, L->pw1_b, g2, 2 * D);
#pragma omp parallel for schedule(static)
        for (int t = 0; t < T3; t++)
            for (int c = 0; c < D; c++)
                gl[(size_t)t * D + c] = g2[(size_t)t * 2 * D + c] * sigm(g2[(size_t)t * 2 * D + D + c]);
#pragma omp parallel for schedule(static)
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
        ofb_linear(M->pw2, cv, T3, D, L->pw2_b, u, D);
        for (int64_t i = 0; i < TD; i++) x[i] += u[i];
        /* FF2 */
        layernorm(x, T3, D, L->ln_g[3], L->ln_b[3], h);
        ofb_linear(M->ff2_w1, h, T3, D, L->ff2_b1, tt, FF);
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < TF; i++) tt[i] = tt[i] * sigm(tt[i]);
        ofb_linear(M->ff2_w2, tt, T3, FF, L->ff2_b2, u, D);
        for (int64_t i = 0; i < TD; i++) x[i] += 0.5f * u[i];
        layernorm(x, T3, D, L->ln_g[4], L->ln_b[4], h);
        memcpy(x, h, sizeof(float) * (size_t)TD);
    }
    memcpy(out, x, sizeof(float) * (size_t)TD);
    free(x); free(pos); free(h); free(tt); free(u); free(q); free(kk); free(vv); free(kr); free(ctx);
    free(g2); free(gl); free(cv);
    return T3;
}

/* One-shot form: prepare (weight mode of oq_encoder_set_weight_mode), run, release. */
int oq_encoder_forward(const oq_enc_cfg *cfg, const oq_enc_weights *W, const float *mel, int t_mel, float *out) {
    oq_enc_model *m = oq_encoder_prepare(cfg, W, g_weight_mode);
    int t3 = oq_encoder_run(m, mel, t_mel, out);
    oq_encoder_release(m);
    return t3;
}
