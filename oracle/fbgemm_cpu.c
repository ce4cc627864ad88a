/*
 * fbgemm_cpu.c -- CPU restatement of the reference's executing Q8_0 matmul,
 * FbgemmBf16Op (src/fast_matmul.rs:138-167), with the performance structure
 * the reference relies on.
 *
 * TEST INFRASTRUCTURE AND CPU BASELINE ONLY.  Used by the encoder oracle
 * (encoder_oracle.c), by tests/ and by bench.py's CPU-baseline and reference
 * legs.  The shipped library never links, loads or calls it.
 *
 * What it restates:
 *   - MatMul::from_tensor (src/fast_matmul.rs:191-208): the Q8_0 weight is
 *     dequantized (w = f32(d) * q) and packed ONCE to bf16
 *     (PackedMatrixBf16::from_transposed, :202).  Rounding is RNE (assumed:
 *     the fbgemm-rs source is not vendored; torch's float->bfloat16 cast
 *     gives the same bits, checked in tests/test_oracle.py).
 *   - FbgemmBf16Op::cpu_fwd (:138-167) -> fbgemm_rs::sgemm_bf16_simple: f32
 *     activations times the bf16 weights widened to f32 in registers, f32
 *     FMA accumulation.  Every output is the k-sequential chain
 *     acc = fma(x[k], w[k], acc) from acc = 0, so results are bit-identical to
 *     oq_matmul_fbgemm_bf16 (the scalar oracle) whatever the ISA or threads.
 *   - The parallel split follows tiled_matmul_inner (:45-61): 128-column
 *     tiles of the output run in parallel (OpenMP), here also split into
 *     48-row blocks so that small-N shapes use every core.
 *
 * Packed layout: 64-column panels, [panel][k][32 words].  bf16 word w of a
 * k row holds column (w < 16 ? w : 16 + w) in its low half and the column 16
 * further in its high half, so a 512-bit load yields four 16-column f32
 * vectors with one shift and one mask each (no shuffles).  Columns past N are
 * zero.  f32 panels ([panel][k][64]) carry exact dequantized weights (candle
 * Linear on dequantized tensors, the Parakeet Linux path of
 * src/parakeet/transducer.rs:1841-1865) and attention operands.
 */
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

extern void oq_dequant_q8_0(const uint8_t *blocks, int64_t n_rows, int64_t k, float *w);
extern uint16_t oq_f32_to_bf16(float f);

#define OFB_NP 64 /* columns per panel */
#define OFB_ROWS 48 /* rows per parallel task */

typedef struct {
    int64_t n, k;
    int bf16;     /* 1: bf16 words [panel][k][32]; 0: f32 [panel][k][64] */
    int64_t panels;
    void *data;
} ofb_mat;

static int g_isa = -1; /* 512: AVX-512F, 256: AVX2+FMA */

int ofb_isa(void) {
    if (g_isa < 0) {
        __builtin_cpu_init();
        g_isa = __builtin_cpu_supports("avx512f") ? 512 : 256;
    }
    return g_isa;
}

/* Force the AVX2 kernels (tests check both give identical bits). */
void ofb_force_isa(int isa) { g_isa = isa == 512 && __builtin_cpu_supports("avx512f") ? 512 : 256; }

void ofb_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int ofb_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Column held by the low half of word w of a 64-column bf16 panel row. */
static inline int word_col(int w) { return w < 16 ? w : w + 16; }

static ofb_mat *alloc_mat(int64_t n, int64_t k, int bf16) {
    ofb_mat *m = (ofb_mat *)calloc(1, sizeof(ofb_mat));
    m->n = n;
    m->k = k;
    m->bf16 = bf16;
    m->panels = (n + OFB_NP - 1) / OFB_NP;
    size_t bytes = (size_t)m->panels * (size_t)k * OFB_NP * (bf16 ? 2 : 4);
    m->data = aligned_alloc(64, (bytes + 63) / 64 * 64);
    memset(m->data, 0, bytes);
    return m;
}

/* Pack a row-major [n, k] f32 matrix (W[n][k]: output column n, reduction k). */
ofb_mat *ofb_pack_f32_nk(const float *w, int64_t n, int64_t k, int bf16) {
    ofb_mat *m = alloc_mat(n, k, bf16);
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < m->panels; p++) {
        for (int64_t kk = 0; kk < k; kk++) {
            if (bf16) {
                uint32_t *row = (uint32_t *)m->data + ((size_t)p * k + kk) * 32;
                for (int wd = 0; wd < 32; wd++) {
                    int64_t c0 = p * OFB_NP + word_col(wd), c1 = c0 + 16;
                    uint32_t lo = c0 < n ? oq_f32_to_bf16(w[c0 * k + kk]) : 0;
                    uint32_t hi = c1 < n ? oq_f32_to_bf16(w[c1 * k + kk]) : 0;
                    row[wd] = lo | (hi << 16);
                }
            } else {
                float *row = (float *)m->data + ((size_t)p * k + kk) * OFB_NP;
                for (int c = 0; c < OFB_NP; c++) {
                    int64_t col = p * OFB_NP + c;
                    row[c] = col < n ? w[col * k + kk] : 0.f;
                }
            }
        }
    }
    return m;
}

/* Q8_0 blocks [n, k/32 * 34] -> packed matrix (bf16 != 0: RNE bf16 of the
 * dequantized value, the fast_matmul packing; 0: exact f32). */
ofb_mat *ofb_pack_q8_0(const uint8_t *blocks, int64_t n, int64_t k, int bf16) {
    float *w = (float *)malloc(sizeof(float) * (size_t)n * (size_t)k);
    oq_dequant_q8_0(blocks, n, k, w);
    ofb_mat *m = ofb_pack_f32_nk(w, n, k, bf16);
    free(w);
    return m;
}

void ofb_free(ofb_mat *m) {
    if (!m) return;
    free(m->data);
    free(m);
}

int64_t ofb_rows(const ofb_mat *m) { return m->n; }

/* ------------------------------------------------------------ AVX-512 */
#define MR512 6

__attribute__((target("avx512f"))) static void mk512(int rows, int64_t K, const float *const *a, const void *panel,
                                                      int bf16, float *c, int64_t ldc, int cols, const float *bias) {
    __m512 acc[MR512][4];
    for (int r = 0; r < MR512; r++)
        for (int j = 0; j < 4; j++) acc[r][j] = _mm512_setzero_ps();
    const __m512i mask_hi = _mm512_set1_epi32((int)0xffff0000u);
    for (int64_t k = 0; k < K; k++) {
        __m512 w0, w1, w2, w3;
        if (bf16) {
            const uint32_t *row = (const uint32_t *)panel + k * 32;
            __m512i z0 = _mm512_loadu_si512((const void *)row);
            __m512i z1 = _mm512_loadu_si512((const void *)(row + 16));
            w0 = _mm512_castsi512_ps(_mm512_slli_epi32(z0, 16));
            w1 = _mm512_castsi512_ps(_mm512_and_si512(z0, mask_hi));
            w2 = _mm512_castsi512_ps(_mm512_slli_epi32(z1, 16));
            w3 = _mm512_castsi512_ps(_mm512_and_si512(z1, mask_hi));
        } else {
            const float *row = (const float *)panel + k * OFB_NP;
            w0 = _mm512_loadu_ps(row);
            w1 = _mm512_loadu_ps(row + 16);
            w2 = _mm512_loadu_ps(row + 32);
            w3 = _mm512_loadu_ps(row + 48);
        }
#pragma GCC unroll 6
        for (int r = 0; r < MR512; r++) {
            __m512 x = _mm512_set1_ps(a[r][k]);
            acc[r][0] = _mm512_fmadd_ps(x, w0, acc[r][0]);
            acc[r][1] = _mm512_fmadd_ps(x, w1, acc[r][1]);
            acc[r][2] = _mm512_fmadd_ps(x, w2, acc[r][2]);
            acc[r][3] = _mm512_fmadd_ps(x, w3, acc[r][3]);
        }
    }
    for (int r = 0; r < rows; r++) {
        float out[64];
        _mm512_storeu_ps(out, acc[r][0]);
        _mm512_storeu_ps(out + 16, acc[r][1]);
        _mm512_storeu_ps(out + 32, acc[r][2]);
        _mm512_storeu_ps(out + 48, acc[r][3]);
        for (int j = 0; j < cols; j++) c[r * ldc + j] = bias ? out[j] + bias[j] : out[j];
    }
}

/* ------------------------------------------------------- AVX2 + FMA */
#define MR256 3

/* 32 columns of a panel (half h): lanes of the 8-word loads map to columns
 * (w, w + 16) for bf16 words, plain columns for f32. */
__attribute__((target("avx2,fma"))) static void mk256(int rows, int64_t K, const float *const *a, const void *panel,
                                                       int bf16, int half, float *c, int64_t ldc, int cols,
                                                       const float *bias) {
    __m256 acc[MR256][4];
    for (int r = 0; r < MR256; r++)
        for (int j = 0; j < 4; j++) acc[r][j] = _mm256_setzero_ps();
    const __m256i mask_hi = _mm256_set1_epi32((int)0xffff0000u);
    for (int64_t k = 0; k < K; k++) {
        __m256 w[4];
        if (bf16) {
            /* half 0: words 0..15 -> columns 0..31; half 1: words 16..31 -> 32..63 */
            const uint32_t *row = (const uint32_t *)panel + k * 32 + half * 16;
            __m256i z0 = _mm256_loadu_si256((const __m256i *)row);
            __m256i z1 = _mm256_loadu_si256((const __m256i *)(row + 8));
            w[0] = _mm256_castsi256_ps(_mm256_slli_epi32(z0, 16));  /* cols 0..7 */
            w[1] = _mm256_castsi256_ps(_mm256_slli_epi32(z1, 16));  /* cols 8..15 */
            w[2] = _mm256_castsi256_ps(_mm256_and_si256(z0, mask_hi)); /* cols 16..23 */
            w[3] = _mm256_castsi256_ps(_mm256_and_si256(z1, mask_hi)); /* cols 24..31 */
        } else {
            const float *row = (const float *)panel + k * OFB_NP + half * 32;
            for (int j = 0; j < 4; j++) w[j] = _mm256_loadu_ps(row + 8 * j);
        }
        for (int r = 0; r < MR256; r++) {
            __m256 x = _mm256_set1_ps(a[r][k]);
            for (int j = 0; j < 4; j++) acc[r][j] = _mm256_fmadd_ps(x, w[j], acc[r][j]);
        }
    }
    for (int r = 0; r < rows; r++) {
        float out[32];
        for (int j = 0; j < 4; j++) _mm256_storeu_ps(out + 8 * j, acc[r][j]);
        for (int j = 0; j < cols; j++) c[r * ldc + j] = bias ? out[j] + bias[j] : out[j];
    }
}

/* One task: rows [r0, r1) x panel p. */
static void run_block(const ofb_mat *m, const float *x, int64_t ldx, int64_t r0, int64_t r1, int64_t p,
                      const float *bias, float *y, int64_t ldy) {
    const int isa = ofb_isa();
    const int64_t K = m->k;
    const void *panel = m->bf16 ? (const void *)((const uint32_t *)m->data + (size_t)p * K * 32)
                                : (const void *)((const float *)m->data + (size_t)p * K * OFB_NP);
    const int64_t c0 = p * OFB_NP;
    const int cols = (int)(m->n - c0 < OFB_NP ? m->n - c0 : OFB_NP);
    const int mr = isa == 512 ? MR512 : MR256;
    for (int64_t r = r0; r < r1; r += mr) {
        int rows = (int)(r1 - r < mr ? r1 - r : mr);
        const float *a[MR512];
        for (int i = 0; i < mr; i++) a[i] = x + (r + (i < rows ? i : rows - 1)) * ldx;
        if (isa == 512) {
            mk512(rows, K, a, panel, m->bf16, y + r * ldy + c0, ldy, cols, bias ? bias + c0 : NULL);
        } else {
            for (int h = 0; h < 2; h++) {
                int hc = cols - 32 * h;
                if (hc <= 0) break;
                mk256(rows, K, a, panel, m->bf16, h, y + r * ldy + c0 + 32 * h, ldy, hc > 32 ? 32 : hc,
                      bias ? bias + c0 + 32 * h : NULL);
            }
        }
    }
}

/* y[i, :n] = x[i, :k] . W^T (+ bias), i < m.  Parallel over (row block,
 * 128-column tile) unless already inside a parallel region. */
void ofb_linear(const ofb_mat *mat, const float *x, int64_t m, int64_t ldx, const float *bias, float *y,
                int64_t ldy) {
    const int64_t rb = (m + OFB_ROWS - 1) / OFB_ROWS;
    const int64_t tiles = (mat->panels + 1) / 2;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
    for (int64_t i = 0; i < rb; i++)
        for (int64_t t = 0; t < tiles; t++) {
            int64_t r0 = i * OFB_ROWS, r1 = r0 + OFB_ROWS < m ? r0 + OFB_ROWS : m;
            for (int64_t p = 2 * t; p < 2 * t + 2 && p < mat->panels; p++) run_block(mat, x, ldx, r0, r1, p, bias, y, ldy);
        }
}

/* Single-threaded form for callers that parallelise around it. */
void ofb_linear_serial(const ofb_mat *mat, const float *x, int64_t m, int64_t ldx, const float *bias, float *y,
                       int64_t ldy) {
    for (int64_t p = 0; p < mat->panels; p++) run_block(mat, x, ldx, 0, m, p, bias, y, ldy);
}

/* Pack B given as [k][n] (row stride ldb) into f32 panels (no transpose
 * needed: a panel row is 64 consecutive columns of one k). */
ofb_mat *ofb_pack_f32_kn(const float *b, int64_t k, int64_t n, int64_t ldb) {
    ofb_mat *m = alloc_mat(n, k, 0);
    for (int64_t p = 0; p < m->panels; p++)
        for (int64_t kk = 0; kk < k; kk++) {
            float *row = (float *)m->data + ((size_t)p * k + kk) * OFB_NP;
            for (int c = 0; c < OFB_NP; c++) {
                int64_t col = p * OFB_NP + c;
                row[c] = col < n ? b[kk * ldb + col] : 0.f;
            }
        }
    return m;
}

/* Pack B given as [n][k] rows of stride ldb (a strided view, e.g. one head's
 * slice of a [T, D] matrix) into f32 panels. */
ofb_mat *ofb_pack_f32_nk_strided(const float *b, int64_t n, int64_t k, int64_t ldb) {
    ofb_mat *m = alloc_mat(n, k, 0);
    for (int64_t p = 0; p < m->panels; p++)
        for (int64_t kk = 0; kk < k; kk++) {
            float *row = (float *)m->data + ((size_t)p * k + kk) * OFB_NP;
            for (int c = 0; c < OFB_NP; c++) {
                int64_t col = p * OFB_NP + c;
                row[c] = col < n ? b[col * ldb + kk] : 0.f;
            }
        }
    return m;
}

/* Test entry: y = x . bf16(dequant(W))^T through the packed kernels. */
void ofb_matmul_q8_0(const float *x, int64_t m, int64_t k, const uint8_t *blocks, int64_t n, int bf16, float *y) {
    ofb_mat *w = ofb_pack_q8_0(blocks, n, k, bf16);
    ofb_linear(w, x, m, k, NULL, y, n);
    ofb_free(w);
}
