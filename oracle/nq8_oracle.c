/*
 * nq8_oracle.c -- CPU restatement of the reference's GGUF Q8_0 matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this file.  It is imported by tests/, by __graft_entry__.smoke() as the
 * checker, and by bench.py's CPU-baseline leg.  The CUDA product path must
 * never route through it.
 *
 * What it restates (paths relative to the dropbox/nspeech source tree):
 *   - Q8_0 block format: 34 bytes = f16 scale d, then 32 int8 qs
 *     (gguf-py constants.py GGML_QUANT_SIZES Q8_0 = (32, 2 + 32)).
 *   - Q8_0 quantize, as used by tools/quantize-parakeet/src/main.rs:108
 *     (candle QTensor::quantize, which follows ggml-quants.c
 *     quantize_row_q8_0_ref; gguf-py quants.py:378-393 is the bit-exact
 *     Python restatement this oracle is pinned against).
 *   - Q8_0 dequantize: w = f32(d) * q (gguf-py quants.py:396-401; called at
 *     src/moonshine/encoder.rs:33, src/parakeet/transducer.rs:1865).
 *   - FbgemmBf16Op (src/fast_matmul.rs:138-167, packing at :191-208):
 *     y[m,n] = sum_k x_f32[m,k] * f32(bf16(dequant(W)[n,k])), f32 accumulate.
 *     fbgemm-rs is an un-vendored git dependency (branch main, no lockfile);
 *     its bf16 rounding mode and summation order are not visible, so this
 *     oracle ASSUMES round-to-nearest-even packing and k-sequential fmaf
 *     accumulation.  Parity for this semantic is therefore "unpinned" at the
 *     fbgemm boundary; tests use the f64 exact product as tolerance anchor.
 *   - QTiledOp (src/fast_matmul.rs:30-62, 71-125): activations quantized per
 *     32 to Q8_0 (from_float, :42), then per-block integer dot times
 *     d_w * d_x (vec_dot, :57).  candle's vec_dot association order is not
 *     visible (un-vendored candle-core, branch windows); this oracle uses
 *     sumf += ((float)sumi * d_w) * d_x, block-sequential.
 *   - Exact reference: y = x . dequant(W)^T in f64 (tolerance anchor).
 *   - Epilogues from the call sites: bias (QLinear::forward,
 *     src/parakeet/quantized_layers.rs:31-38), SiLU (fast_conformer.rs:207),
 *     GELU-erf (moonshine/encoder.rs:105), GLU-sigmoid a*sigmoid(b)
 *     (fast_conformer.rs:479-484), GLU-SiLU x*silu(gate)
 *     (moonshine/decoder.rs:403-410), gate in the second half in both.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OQ_QK 32
#define OQ_BLOCK_BYTES 34

/* ---------------------------------------------------------------- f16 / bf16 */

/* IEEE binary16 round-to-nearest-even, with subnormals, overflow to inf.
 * Matches numpy's float32 -> float16 cast used by gguf-py quants.py:391. */
uint16_t oq_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) return (uint16_t)(sign | (a > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 -> inf */
    if (a < 0x38800000u) {                                   /* below 2^-14 */
        if (a < 0x33000000u) return (uint16_t)sign;          /* below 2^-25 -> 0 */
        uint32_t e = a >> 23;
        uint32_t m = (a & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126u - e; /* 14..24 */
        uint32_t r = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = a - 0x38000000u;
    uint32_t rem = r & 0x1fffu;
    r >>= 13;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
}

float oq_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else { /* subnormal: normalise */
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; sh++; }
            m &= 0x3ffu;
            x = sign | ((uint32_t)(113 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* bfloat16 round-to-nearest-even (NaN stays NaN). */
uint16_t oq_f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

float oq_bf16_to_f32(uint16_t b) {
    uint32_t x = (uint32_t)b << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static float bf16_round(float f) { return oq_bf16_to_f32(oq_f32_to_bf16(f)); }

/* ------------------------------------------------------------------ Q8_0 */

/* Quantize rows of length k (k % 32 == 0) into GGUF Q8_0 blocks.
 * ggml quantize_row_q8_0_ref / gguf-py quants.py:381-393:
 *   d = amax / 127; id = d ? 1/d : 0; q = roundf(x * id) (half away from 0);
 *   d stored as f16 (RNE). */
void oq_quantize_q8_0(const float *x, int64_t n_rows, int64_t k, uint8_t *out) {
    int64_t nb = n_rows * (k / OQ_QK);
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; b++) {
        const float *xb = x + b * OQ_QK;
        uint8_t *ob = out + b * OQ_BLOCK_BYTES;
        float amax = 0.0f;
        for (int j = 0; j < OQ_QK; j++) {
            float v = fabsf(xb[j]);
            if (v > amax) amax = v;
        }
        float d = amax / 127.0f;
        float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t dh = oq_f32_to_f16(d);
        memcpy(ob, &dh, 2);
        for (int j = 0; j < OQ_QK; j++) {
            float q = roundf(xb[j] * id);
            ob[2 + j] = (uint8_t)(int8_t)q;
        }
    }
}

/* w[n,k] = f32(d) * q (row-major [n_rows, k]). */
void oq_dequant_q8_0(const uint8_t *blocks, int64_t n_rows, int64_t k, float *w) {
    int64_t nb = n_rows * (k / OQ_QK);
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t *ib = blocks + b * OQ_BLOCK_BYTES;
        uint16_t dh;
        memcpy(&dh, ib, 2);
        float d = oq_f16_to_f32(dh);
        for (int j = 0; j < OQ_QK; j++) w[b * OQ_QK + j] = d * (float)(int8_t)ib[2 + j];
    }
}

/* Transposed dequant to [k, n_rows] row-major: the semantics the GPU encoders
 * expect from q8_dequant::dequant_2d (call sites src/moonshine/gpu_encoder.rs:
 * 181-185, used as [in, out] at :197-205). */
void oq_dequant_q8_0_t(const uint8_t *blocks, int64_t n_rows, int64_t k, float *wt) {
    int64_t kb = k / OQ_QK;
    for (int64_t n = 0; n < n_rows; n++)
        for (int64_t b = 0; b < kb; b++) {
            const uint8_t *ib = blocks + (n * kb + b) * OQ_BLOCK_BYTES;
            uint16_t dh;
            memcpy(&dh, ib, 2);
            float d = oq_f16_to_f32(dh);
            for (int j = 0; j < OQ_QK; j++)
                wt[(b * OQ_QK + j) * n_rows + n] = d * (float)(int8_t)ib[2 + j];
        }
}

/* fbgemm-rs PackedMatrixBf16::from_transposed stand-in: element-wise bf16
 * (RNE assumed) of the dequantized [n, k] weight, kept [n, k]. */
void oq_pack_bf16(const float *w, int64_t count, uint16_t *out) {
    for (int64_t i = 0; i < count; i++) out[i] = oq_f32_to_bf16(w[i]);
}

/* --------------------------------------------------------------- epilogues */

enum {
    OQ_EPI_NONE = 0,
    OQ_EPI_SILU = 1,
    OQ_EPI_GELU_ERF = 2,
    OQ_EPI_GLU_SIGMOID = 3,
    OQ_EPI_GLU_SILU = 4,
    OQ_EPI_RELU = 5,
};

static double sigmoid_d(double v) { return 1.0 / (1.0 + exp(-v)); }

/* Apply bias then activation to a raw product y[m, n] (f64), writing
 * out[m, n_out]; n_out = n/2 for the GLU forms (first half times act(second
 * half)), else n. */
void oq_epilogue_f64(const double *y, int64_t m, int64_t n, const float *bias, int epi,
                     double *out) {
    int glu = (epi == OQ_EPI_GLU_SIGMOID || epi == OQ_EPI_GLU_SILU);
    int64_t n_out = glu ? n / 2 : n;
    for (int64_t i = 0; i < m; i++) {
        const double *yr = y + i * n;
        double *orow = out + i * n_out;
        for (int64_t j = 0; j < n_out; j++) {
            double a = yr[j] + (bias ? (double)bias[j] : 0.0);
            if (!glu) {
                if (epi == OQ_EPI_SILU) a = a * sigmoid_d(a);
                else if (epi == OQ_EPI_GELU_ERF) a = 0.5 * a * (1.0 + erf(a / sqrt(2.0)));
                else if (epi == OQ_EPI_RELU) a = a > 0.0 ? a : 0.0;
                orow[j] = a;
            } else {
                double g = yr[j + n_out] + (bias ? (double)bias[j + n_out] : 0.0);
                orow[j] = epi == OQ_EPI_GLU_SIGMOID ? a * sigmoid_d(g) : a * (g * sigmoid_d(g));
            }
        }
    }
}

/* ----------------------------------------------------------------- matmuls */

/* REF_FBGEMM_BF16: y = x . bf16(dequant(W))^T, f32, k-sequential fmaf. */
void oq_matmul_fbgemm_bf16(const float *x, int64_t m, int64_t k, const uint8_t *blocks,
                           int64_t n, float *y) {
    float *wb = (float *)malloc(sizeof(float) * (size_t)(n * k));
    oq_dequant_q8_0(blocks, n, k, wb);
    for (int64_t i = 0; i < n * k; i++) wb[i] = bf16_round(wb[i]);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < m; i++)
        for (int64_t j = 0; j < n; j++) {
            const float *xr = x + i * k;
            const float *wr = wb + j * k;
            float acc = 0.0f;
            for (int64_t t = 0; t < k; t++) acc = fmaf(xr[t], wr[t], acc);
            y[i * n + j] = acc;
        }
    free(wb);
}

/* REF_QTILED: quantize x rows to Q8_0, integer dot per block, f32 scale. */
void oq_matmul_qtiled(const float *x, int64_t m, int64_t k, const uint8_t *blocks, int64_t n,
                      float *y) {
    int64_t kb = k / OQ_QK;
    uint8_t *xq = (uint8_t *)malloc((size_t)(m * kb * OQ_BLOCK_BYTES));
    oq_quantize_q8_0(x, m, k, xq);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < m; i++)
        for (int64_t j = 0; j < n; j++) {
            float sumf = 0.0f;
            for (int64_t b = 0; b < kb; b++) {
                const uint8_t *wbk = blocks + (j * kb + b) * OQ_BLOCK_BYTES;
                const uint8_t *xbk = xq + (i * kb + b) * OQ_BLOCK_BYTES;
                int32_t sumi = 0;
                for (int t = 0; t < OQ_QK; t++)
                    sumi += (int32_t)(int8_t)wbk[2 + t] * (int32_t)(int8_t)xbk[2 + t];
                uint16_t dw, dx;
                memcpy(&dw, wbk, 2);
                memcpy(&dx, xbk, 2);
                sumf += ((float)sumi * oq_f16_to_f32(dw)) * oq_f16_to_f32(dx);
            }
            y[i * n + j] = sumf;
        }
    free(xq);
}

/* REF_EXACT: y = x . dequant(W)^T in f64. */
void oq_matmul_exact_f64(const float *x, int64_t m, int64_t k, const uint8_t *blocks, int64_t n,
                         double *y) {
    float *w = (float *)malloc(sizeof(float) * (size_t)(n * k));
    oq_dequant_q8_0(blocks, n, k, w);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < m; i++)
        for (int64_t j = 0; j < n; j++) {
            const float *xr = x + i * k;
            const float *wr = w + j * k;
            double acc = 0.0;
            for (int64_t t = 0; t < k; t++) acc += (double)xr[t] * (double)wr[t];
            y[i * n + j] = acc;
        }
    free(w);
}

/* ------------------------------------------------------------------ metric */

/* max_{m,n} |y - yref| / max(|yref|, tau * rms(yref[m, :])). */
double oq_max_rel_err(const float *y, const double *yref, int64_t m, int64_t n, double tau) {
    double worst = 0.0;
    for (int64_t i = 0; i < m; i++) {
        double ss = 0.0;
        for (int64_t j = 0; j < n; j++) ss += yref[i * n + j] * yref[i * n + j];
        double rms = n ? sqrt(ss / (double)n) : 0.0;
        for (int64_t j = 0; j < n; j++) {
            double r = yref[i * n + j];
            double den = fabs(r) > tau * rms ? fabs(r) : tau * rms;
            double e = fabs((double)y[i * n + j] - r);
            double rel;
            if (den > 0.0) rel = e / den;
            else rel = e > 0.0 ? INFINITY : 0.0;
            if (isnan(y[i * n + j])) rel = INFINITY;
            if (rel > worst) worst = rel;
        }
    }
    return worst;
}

/* ----------------------------------------------------------------- seeded RNG
 * xoshiro256** seeded by splitmix64; normals by Box-Muller in double.
 * The same generator feeds every test and benchmark input, so inputs are
 * identical wherever this file is compiled. */

typedef struct { uint64_t s[4]; } oq_rng;

static uint64_t splitmix64(uint64_t *x) {
    uint64_t z = (*x += 0x9e3779b97f4a7c15ull);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

static uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

static uint64_t rng_next(oq_rng *r) {
    uint64_t *s = r->s;
    uint64_t result = rotl(s[1] * 5, 7) * 9;
    uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return result;
}

static void rng_seed(oq_rng *r, uint64_t seed) {
    uint64_t x = seed;
    for (int i = 0; i < 4; i++) r->s[i] = splitmix64(&x);
}

/* Fill out[0..count) with N(mean, std) as f32. */
void oq_fill_normal(uint64_t seed, float *out, int64_t count, float mean, float std) {
    oq_rng r;
    rng_seed(&r, seed);
    const double two_pi = 6.283185307179586476925286766559;
    for (int64_t i = 0; i < count; i += 2) {
        double u1 = ((double)(rng_next(&r) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
        double u2 = (double)(rng_next(&r) >> 11) * (1.0 / 9007199254740992.0);
        double rad = sqrt(-2.0 * log(u1));
        out[i] = (float)((double)mean + (double)std * rad * cos(two_pi * u2));
        if (i + 1 < count) out[i + 1] = (float)((double)mean + (double)std * rad * sin(two_pi * u2));
    }
}

/* Fill out[0..count) with U[lo, hi) as f32. */
void oq_fill_uniform(uint64_t seed, float *out, int64_t count, float lo, float hi) {
    oq_rng r;
    rng_seed(&r, seed);
    for (int64_t i = 0; i < count; i++) {
        double u = (double)(rng_next(&r) >> 11) * (1.0 / 9007199254740992.0);
        out[i] = (float)((double)lo + ((double)hi - (double)lo) * u);
    }
}
