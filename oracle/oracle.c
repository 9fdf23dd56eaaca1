/*
 * oracle.c - CPU restatement of hedone21/llm.rs's x86_64 CPU path (the
 * batch-1 Llama token loop).  TEST INFRASTRUCTURE: used only by tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg, never by the
 * shipped CUDA library.  See oracle.h for what pins it and what does not.
 *
 * Built with -O3 -fopenmp -ffp-contract=off: Rust does not contract a*b+c into
 * an FMA, so neither may this file.  Every loop that sums floats keeps the
 * reference's sequential order.  libm (expf, sinf, cosf, powf, sqrtf) stands in
 * for Rust std's calls into the same platform libm.
 */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>
#if defined(__AVX2__)
#include <immintrin.h>
#endif

#include "../llm.rs_b200/csrc/llmrs_synth.h"

static int g_threads = 0;

void orc_set_threads(int n) { g_threads = n; if (n > 0) omp_set_num_threads(n); }
int orc_get_threads(void) { return g_threads > 0 ? g_threads : omp_get_max_threads(); }

/* ------------------------------------------------------------------------ */
/* Q8_0 activation quantiser: src/backend/cpu.rs:663-745, x86 branch 724-743. */
void orc_quantize_row_q8_0(const float *x, int k, int8_t *q, float *s)
{
    int nb = k / 32; /* trailing k%32 elements are ignored, as zip() truncates at cpu.rs:665-668 */
    for (int b = 0; b < nb; b++) {
        const float *src = x + (size_t)b * 32;
        int8_t *dst = q + (size_t)b * 32;
        float max_abs = 0.0f;
        for (int i = 0; i < 32; i++) {
            float a = fabsf(src[i]);
            if (a > max_abs)
                max_abs = a;
        }
        if (max_abs == 0.0f) {
            s[b] = 0.0f;
            memset(dst, 0, 32);
        } else {
            float scale = max_abs / 127.0f;
            s[b] = scale;
            float inv = 1.0f / scale;
            for (int i = 0; i < 32; i++) {
                float v = roundf(src[i] * inv); /* f32::round: half away from zero */
                if (v != v)
                    v = 0.0f; /* `as i8` maps NaN to 0 */
                if (v < -127.0f)
                    v = -127.0f;
                if (v > 127.0f)
                    v = 127.0f;
                dst[i] = (int8_t)v;
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Q4 weight quantiser: src/core/tensor.rs:102-167 (planar: nibbles then f32 scales). */
void orc_quantize_q4(const float *w, size_t n, uint8_t *qs, float *scales)
{
    size_t nblocks = (n + 31) / 32;
    size_t out = 0;
    for (size_t b = 0; b < nblocks; b++) {
        size_t base = b * 32;
        size_t len = n - base < 32 ? n - base : 32;
        float max_abs = 0.0f;
        for (size_t i = 0; i < len; i++) {
            float a = fabsf(w[base + i]);
            max_abs = fmaxf(max_abs, a); /* fold(0.0, acc.max(|x|)) */
        }
        float scale = max_abs / 7.0f;
        scales[b] = scale;
        size_t pairs = (len + 1) / 2;
        if (scale == 0.0f) {
            for (size_t p = 0; p < pairs; p++)
                qs[out++] = 0x88;
        } else {
            float inv = 1.0f / scale;
            for (size_t p = 0; p < pairs; p++) {
                float v0 = w[base + 2 * p];
                float v1 = (2 * p + 1 < len) ? w[base + 2 * p + 1] : 0.0f;
                float f0 = v0 * inv + 8.5f;
                float f1 = v1 * inv + 8.5f;
                f0 = f0 < 0.0f ? 0.0f : (f0 > 15.0f ? 15.0f : f0);
                f1 = f1 < 0.0f ? 0.0f : (f1 > 15.0f ? 15.0f : f1);
                uint8_t q0 = (f0 != f0) ? 0 : (uint8_t)f0; /* `as u8` truncates; NaN -> 0 */
                uint8_t q1 = (f1 != f1) ? 0 : (uint8_t)f1;
                qs[out++] = (uint8_t)(q0 | (q1 << 4));
            }
        }
    }
}

/* dequantise: (q-8)*scale, src/test/opencl.rs:182-235 */
void orc_dequantize_q4(const uint8_t *qs, const float *scales, size_t n, float *out)
{
    for (size_t i = 0; i < (n + 1) / 2; i++) {
        float s = scales[(i * 2) / 32];
        out[2 * i] = ((float)(qs[i] & 0x0F) - 8.0f) * s;
        if (2 * i + 1 < n)
            out[2 * i + 1] = ((float)(qs[i] >> 4) - 8.0f) * s;
    }
}

/* ------------------------------------------------------------------------ */
/* Q4 x Q8 block kernel: src/backend/cpu.rs:888-941 (kernel_avx2).
 *
 * Per row j: total = 0; for each block b in order:
 *   scale = sw[j,b] * sa[b]  (f32)
 *   isum  = sum_i (nibble_i - 8) * q8_i   (exact int32)
 *   total += (float)isum * scale          (mul, then add; no FMA)
 *
 * The activation is prepared once per row of A: codes are re-ordered so that
 * the 16 low nibbles of a block line up with the even elements and the 16
 * high nibbles with the odd ones, and 8*sum(q8) per block is precomputed, so
 * the inner loop needs no unpacking.  The integer result is the same. */
typedef struct {
    int8_t *perm; /* [nb][32]: even elements, then odd elements */
    int32_t *corr; /* [nb]: 8 * sum of the block's codes */
    float *s;
    int8_t *q;
    int nb;
} orc_act;

static void orc_act_prepare(orc_act *A, const float *a, int k)
{
    A->nb = k / 32;
    orc_quantize_row_q8_0(a, k, A->q, A->s);
    for (int b = 0; b < A->nb; b++) {
        const int8_t *src = A->q + (size_t)b * 32;
        int8_t *dst = A->perm + (size_t)b * 32;
        int32_t sum = 0;
        for (int i = 0; i < 16; i++) {
            dst[i] = src[2 * i];
            dst[16 + i] = src[2 * i + 1];
        }
        for (int i = 0; i < 32; i++)
            sum += src[i];
        A->corr[b] = 8 * sum;
    }
}

static inline int32_t orc_block_q4(const uint8_t *w16, const int8_t *perm32, int32_t corr)
{
#if defined(__AVX2__)
    __m128i raw = _mm_loadu_si128((const __m128i *)w16);
    __m128i m = _mm_set1_epi8(0x0F);
    __m256i w = _mm256_set_m128i(_mm_and_si128(_mm_srli_epi16(raw, 4), m), _mm_and_si128(raw, m));
    __m256i a = _mm256_loadu_si256((const __m256i *)perm32);
    __m256i p = _mm256_madd_epi16(_mm256_maddubs_epi16(w, a), _mm256_set1_epi16(1));
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(p), _mm256_extracti128_si256(p, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
    return _mm_cvtsi128_si32(s) - corr;
#else
    int32_t sum = 0;
    for (int i = 0; i < 16; i++)
        sum += (int32_t)(w16[i] & 0x0F) * perm32[i] + (int32_t)(w16[i] >> 4) * perm32[16 + i];
    return sum - corr;
#endif
}

static float orc_row_q4(const uint8_t *qrow, const float *srow, const orc_act *A)
{
    float total = 0.0f;
    for (int b = 0; b < A->nb; b++) {
        float scale = srow[b] * A->s[b];
        int32_t isum = orc_block_q4(qrow + (size_t)b * 16, A->perm + (size_t)b * 32, A->corr[b]);
        total += (float)isum * scale;
    }
    return total;
}

static inline int32_t orc_block_q8(const int8_t *w32, const int8_t *a32)
{
    int32_t sum = 0;
    for (int i = 0; i < 32; i++)
        sum += (int32_t)w32[i] * a32[i];
    return sum;
}

/* Q8_0-weight analogue of the Q4 kernel (the reference has no Q8_0 weight
 * path; this follows kernel_avx2's accumulation with int8 weights). */
static float orc_row_q8(const int8_t *wrow, const float *srow, const orc_act *A)
{
    float total = 0.0f;
    for (int b = 0; b < A->nb; b++) {
        float scale = srow[b] * A->s[b];
        int32_t isum = orc_block_q8(wrow + (size_t)b * 32, A->q + (size_t)b * 32);
        total += (float)isum * scale;
    }
    return total;
}

static void orc_act_alloc(orc_act *A, int k)
{
    int nb = k / 32;
    A->perm = (int8_t *)malloc((size_t)k + 32);
    A->q = (int8_t *)malloc((size_t)k + 32);
    A->corr = (int32_t *)malloc(sizeof(int32_t) * (size_t)(nb + 1));
    A->s = (float *)malloc(sizeof(float) * (size_t)(nb + 1));
    A->nb = nb;
}

static void orc_act_free(orc_act *A)
{
    free(A->perm);
    free(A->q);
    free(A->corr);
    free(A->s);
}

/* CpuBackend::matmul_transposed, Q4 branch: src/backend/cpu.rs:31-111.
 * m==1: one quantise, rows in parallel chunks of 512 (cpu.rs:76-89);
 * m>1: per-row quantise (cpu.rs:90-110).  Both give the same per-row math. */
void orc_matmul_transposed_q4(const float *a, int m, int k, const uint8_t *qs, const float *sw, int n, float *c)
{
    orc_act A;
    orc_act_alloc(&A, k);
    int nb = k / 32;
    for (int i = 0; i < m; i++) {
        orc_act_prepare(&A, a + (size_t)i * k, k);
        int nchunks = (n + 511) / 512;
#pragma omp parallel for schedule(dynamic, 1)
        for (int ch = 0; ch < nchunks; ch++) {
            int j1 = (ch + 1) * 512 < n ? (ch + 1) * 512 : n;
            for (int j = ch * 512; j < j1; j++)
                c[(size_t)i * n + j] = orc_row_q4(qs + (size_t)j * (k / 2), sw + (size_t)j * nb, &A);
        }
    }
    orc_act_free(&A);
}

void orc_matmul_transposed_q8w(const float *a, int m, int k, const int8_t *qw, const float *sw, int n, float *c)
{
    orc_act A;
    orc_act_alloc(&A, k);
    int nb = k / 32;
    for (int i = 0; i < m; i++) {
        orc_act_prepare(&A, a + (size_t)i * k, k);
        int nchunks = (n + 511) / 512;
#pragma omp parallel for schedule(dynamic, 1)
        for (int ch = 0; ch < nchunks; ch++) {
            int j1 = (ch + 1) * 512 < n ? (ch + 1) * 512 : n;
            for (int j = ch * 512; j < j1; j++)
                c[(size_t)i * n + j] = orc_row_q8(qw + (size_t)j * k, sw + (size_t)j * nb, &A);
        }
    }
    orc_act_free(&A);
}

/* x86 simd_dot_f32 is a plain sequential sum: src/backend/cpu.rs:546-549 */
static inline float orc_dot(const float *a, const float *b, int n)
{
    float sum = 0.0f;
    for (int i = 0; i < n; i++)
        sum += a[i] * b[i];
    return sum;
}

/* f32 branch of matmul_transposed: src/backend/cpu.rs:113-146 */
void orc_matmul_transposed_f32(const float *a, int m, int k, const float *b, int n, float *c)
{
#pragma omp parallel for collapse(2) schedule(static)
    for (int i = 0; i < m; i++)
        for (int j = 0; j < n; j++)
            c[(size_t)i * n + j] = orc_dot(a + (size_t)i * k, b + (size_t)j * k, k);
}

/* CpuBackend::matmul (SAXPY, skipping zero multipliers): src/backend/cpu.rs:157-224 */
void orc_matmul_f32(const float *a, int m, int k, const float *b, int n, float *c)
{
#pragma omp parallel for schedule(static)
    for (int i = 0; i < m; i++) {
        float *row = c + (size_t)i * n;
        for (int j = 0; j < n; j++)
            row[j] = 0.0f;
        for (int p = 0; p < k; p++) {
            float val = a[(size_t)i * k + p];
            if (val == 0.0f)
                continue;
            const float *brow = b + (size_t)p * n;
            for (int j = 0; j < n; j++)
                row[j] += val * brow[j]; /* simd_saxpy x86: y += alpha*x, cpu.rs:620-625 */
        }
    }
}

/* CpuBackend::matmul_slice: src/backend/cpu.rs:230-269 */
void orc_matmul_slice(const float *a, int m, int k, const float *other, int rows, float *c)
{
#pragma omp parallel for collapse(2) schedule(static)
    for (int i = 0; i < m; i++)
        for (int j = 0; j < rows; j++)
            c[(size_t)i * rows + j] = orc_dot(a + (size_t)i * k, other + (size_t)j * k, k);
}

/* src/backend/cpu.rs:274-296 */
void orc_add_assign(float *a, const float *b, size_t n)
{
    for (size_t i = 0; i < n; i++)
        a[i] += b[i];
}

/* src/backend/cpu.rs:298-324 (and the host loop src/core/layer.rs:75-80) */
void orc_silu_mul(float *gate, const float *up, size_t n)
{
    for (size_t i = 0; i < n; i++) {
        float g = gate[i];
        float silu = g / (1.0f + expf(-g));
        gate[i] = silu * up[i];
    }
}

/* src/backend/cpu.rs:326-357; chunk i of head_dim values gets pos = start_pos + i */
void orc_rope_inplace(float *x, int rows, int head_dim, int start_pos, float theta_base)
{
    int mid = head_dim / 2;
    for (int i = 0; i < rows; i++) {
        float *chunk = x + (size_t)i * head_dim;
        int pos = start_pos + i;
        for (int j = 0; j < mid; j++) {
            float freq_idx = ((float)j * 2.0f) / (float)head_dim;
            float theta = 1.0f / powf(theta_base, freq_idx);
            float m_theta = (float)pos * theta;
            float sn = sinf(m_theta), cs = cosf(m_theta);
            float re = chunk[j], im = chunk[j + mid];
            chunk[j] = re * cs - im * sn;
            chunk[j + mid] = re * sn + im * cs;
        }
    }
}

/* src/backend/cpu.rs:359-393 */
void orc_rms_norm(const float *x, const float *w, float *y, int rows, int cols, float eps)
{
    for (int r = 0; r < rows; r++) {
        const float *in = x + (size_t)r * cols;
        float *out = y + (size_t)r * cols;
        float ss = 0.0f;
        for (int i = 0; i < cols; i++)
            ss = ss + in[i] * in[i];
        float rms = sqrtf(ss / (float)cols + eps);
        float scale = 1.0f / rms;
        for (int i = 0; i < cols; i++)
            out[i] = in[i] * scale * w[i];
    }
}

/* src/backend/cpu.rs:395-423 */
void orc_softmax(const float *x, float *y, int rows, int cols)
{
    for (int r = 0; r < rows; r++) {
        const float *in = x + (size_t)r * cols;
        float *out = y + (size_t)r * cols;
        float max_val = -3.40282347e+38f; /* f32::MIN */
        for (int j = 0; j < cols; j++)
            max_val = fmaxf(max_val, in[j]);
        float sum = 0.0f;
        for (int j = 0; j < cols; j++) {
            float e = expf(in[j] - max_val);
            out[j] = e;
            sum += e;
        }
        float inv = 1.0f / sum;
        for (int j = 0; j < cols; j++)
            out[j] *= inv;
    }
}

/* src/backend/cpu.rs:425-435 */
void orc_scale(const float *x, float *y, size_t n, float value)
{
    for (size_t i = 0; i < n; i++)
        y[i] = x[i] * value;
}

int orc_argmax(const float *v, int n)
{
    int best = 0;
    for (int i = 1; i < n; i++)
        if (v[i] > v[best])
            best = i; /* ties keep the lowest index */
    return best;
}

/* Next-token sampling, src/main.rs:192-305 restated (u: the draw the reference
 * takes from rng.random::<f32>()).  *margin: how far the walk's running r was
 * from zero around the pick (small = the draw sits on a boundary). */
typedef struct {
    float p;
    int i;
} orc_cand;

static int orc_cand_cmp(const void *a, const void *b)
{
    const orc_cand *x = (const orc_cand *)a, *y = (const orc_cand *)b;
    if (x->p > y->p)
        return -1;
    if (x->p < y->p)
        return 1;
    return x->i < y->i ? -1 : (x->i > y->i); /* the reference's unstable sort leaves ties unordered */
}

int orc_sample(const float *logits, int V, const int *recent, int n_recent, float penalty, float temperature,
               float top_p, float u, float *margin)
{
    float *l = (float *)malloc((size_t)V * 4), *p = (float *)malloc((size_t)V * 4);
    memcpy(l, logits, (size_t)V * 4);
    if (penalty > 1.0f) /* src/main.rs:192-214: each distinct id of the window once */
        for (int j = 0; j < n_recent; j++) {
            int id = recent[j], first = id >= 0 && id < V;
            for (int k = 0; k < j && first; k++)
                first = recent[k] != id;
            if (first)
                l[id] = l[id] < 0.0f ? l[id] * penalty : l[id] / penalty;
        }
    if (fabsf(temperature - 1.0f) > 1e-6f) /* src/main.rs:216-222 */
        for (int i = 0; i < V; i++)
            l[i] /= temperature;
    float mx = -FLT_MAX; /* src/main.rs:230-240 */
    for (int i = 0; i < V; i++)
        mx = fmaxf(mx, l[i]);
    for (int i = 0; i < V; i++)
        p[i] = expf(l[i] - mx);
    float sum = 0.0f;
    for (int i = 0; i < V; i++)
        sum += p[i];
    for (int i = 0; i < V; i++)
        p[i] /= sum;
    int tok = 0;
    float mg = INFINITY;
    if (top_p < 1.0f) { /* src/main.rs:246-292 */
        orc_cand *c = (orc_cand *)malloc((size_t)V * sizeof(orc_cand));
        int n = 0;
        for (int i = 0; i < V; i++)
            if (p[i] > 1e-5f)
                c[n++] = (orc_cand){p[i], i};
        if (n == 0)
            for (int i = 0; i < V; i++)
                c[n++] = (orc_cand){p[i], i};
        qsort(c, (size_t)n, sizeof(orc_cand), orc_cand_cmp);
        float cum = 0.0f;
        int cut = n - 1;
        for (int i = 0; i < n; i++) {
            cum += c[i].p;
            if (cum > top_p) {
                cut = i;
                break;
            }
        }
        float total = 0.0f;
        for (int i = 0; i <= cut; i++)
            total += c[i].p;
        float r = u * total;
        tok = c[0].i;
        for (int i = 0; i <= cut; i++) {
            const float before = r;
            r -= c[i].p;
            if (r <= 0.0f) {
                tok = c[i].i;
                mg = fminf(before, -r);
                break;
            }
        }
        free(c);
    } else { /* src/main.rs:293-305 */
        float r = u;
        for (int i = 0; i < V; i++) {
            const float before = r;
            r -= p[i];
            if (r <= 0.0f) {
                tok = i;
                mg = fminf(before, -r);
                break;
            }
        }
    }
    if (margin)
        *margin = mg;
    free(l);
    free(p);
    return tok;
}

float orc_top2_margin(const float *v, int n)
{
    int b = orc_argmax(v, n);
    float second = -INFINITY;
    for (int i = 0; i < n; i++)
        if (i != b && v[i] > second)
            second = v[i];
    return v[b] - second;
}

/* ------------------------------------------------------------------------ */
/* synthetic generator wrappers                                              */
uint16_t orc_f32_to_f16(float f) { return llmrs_f32_to_f16(f); }
float orc_f16_to_f32(uint16_t h) { return llmrs_f16_to_f32(h); }

uint32_t orc_synth_token(uint64_t seed, uint64_t i, uint32_t vocab)
{
    uint64_t st = llmrs_stream(seed, LLMRS_GLOBAL_LAYER, LLMRS_T_TOKENS, LLMRS_SUB_F32);
    return (uint32_t)(llmrs_draw(st, i) % vocab);
}

void orc_synth_q4(uint64_t seed, uint32_t layer, uint32_t tensor, size_t n, size_t k, uint8_t *qs, float *scales)
{
    uint64_t sc = llmrs_stream(seed, layer, tensor, LLMRS_SUB_Q4CODES);
    uint64_t ss = llmrs_stream(seed, layer, tensor, LLMRS_SUB_SCALES);
    size_t nbytes = n * k / 2, nsc = n * k / 32;
#pragma omp parallel for schedule(static)
    for (size_t j = 0; j < nbytes; j++)
        qs[j] = llmrs_synth_q4_byte(sc, j);
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < nsc; i++)
        scales[i] = llmrs_f16_to_f32(llmrs_synth_scale_f16(ss, i));
}

void orc_synth_q8(uint64_t seed, uint32_t layer, uint32_t tensor, size_t n, size_t k, int8_t *qw, float *scales)
{
    uint64_t sc = llmrs_stream(seed, layer, tensor, LLMRS_SUB_Q8CODES);
    uint64_t ss = llmrs_stream(seed, layer, tensor, LLMRS_SUB_SCALES);
    size_t ncodes = n * k, nsc = n * k / 32;
#pragma omp parallel for schedule(static)
    for (size_t j = 0; j < ncodes; j++)
        qw[j] = llmrs_synth_q8_code(sc, j);
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < nsc; i++)
        scales[i] = llmrs_f16_to_f32(llmrs_synth_scale_f16(ss, i));
}

void orc_synth_normal(uint64_t seed, uint32_t layer, uint32_t tensor, size_t n, float mu, float sd, float *out)
{
    uint64_t st = llmrs_stream(seed, layer, tensor, LLMRS_SUB_F32);
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++)
        out[i] = llmrs_normal_ms(st, i, mu, sd);
}

/* ------------------------------------------------------------------------ */
/* model: src/core/{model,layer,loader}.rs                                   */
typedef struct {
    uint8_t *q4;  /* Q4: [n][k/2] nibbles (planar, src/core/tensor.rs:129-131) */
    int8_t *q8;   /* Q8_0: [n][k] codes */
    float *s;     /* [n][k/32] f32 scales */
    size_t n, k;
} orc_lin;

typedef struct {
    orc_lin q, k, v, o, gate_up, down;
    float *attn_norm, *mlp_norm;
    float *kc; /* [cache_heads][max_seq][D]            (src/core/layer.rs:114-128) */
    float *vc; /* [cache_heads][D][max_seq] transposed */
} orc_layer;

struct orc_model {
    orc_config c;
    int expand; /* 1: K/V weights and cache expanded to n_heads (src/core/loader.rs:62-98) */
    int cache_heads;
    orc_layer *L;
    float *embed, *final_norm;
    orc_lin lm_head;
    float *trace; /* optional: [2*n_layers+1][hidden] residuals entering each RMSNorm (last row) */
};

static void lin_alloc(orc_lin *l, size_t n, size_t k, int fmt)
{
    l->n = n;
    l->k = k;
    l->q4 = fmt == 0 ? (uint8_t *)malloc(n * k / 2) : NULL;
    l->q8 = fmt == 1 ? (int8_t *)malloc(n * k) : NULL;
    l->s = (float *)malloc(sizeof(float) * n * k / 32);
}

static void lin_free(orc_lin *l)
{
    free(l->q4);
    free(l->q8);
    free(l->s);
}

static void lin_forward(const orc_lin *l, const float *x, int m, float *y)
{
    if (l->q4)
        orc_matmul_transposed_q4(x, m, (int)l->k, l->q4, l->s, (int)l->n, y);
    else
        orc_matmul_transposed_q8w(x, m, (int)l->k, l->q8, l->s, (int)l->n, y);
}

orc_model *orc_model_create(const orc_config *cfg, int expand_gqa)
{
    orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
    m->c = *cfg;
    m->expand = expand_gqa;
    const orc_config *c = cfg;
    int D = c->head_dim, H = c->hidden;
    int kvh = expand_gqa ? c->n_heads : c->n_kv_heads;
    m->cache_heads = kvh;
    m->L = (orc_layer *)calloc((size_t)c->n_layers, sizeof(orc_layer));
    for (int i = 0; i < c->n_layers; i++) {
        orc_layer *L = &m->L[i];
        lin_alloc(&L->q, (size_t)c->n_heads * D, H, c->weight_format);
        lin_alloc(&L->k, (size_t)kvh * D, H, c->weight_format);
        lin_alloc(&L->v, (size_t)kvh * D, H, c->weight_format);
        lin_alloc(&L->o, H, (size_t)c->n_heads * D, c->weight_format);
        lin_alloc(&L->gate_up, (size_t)2 * c->ffn, H, c->weight_format);
        lin_alloc(&L->down, H, c->ffn, c->weight_format);
        L->attn_norm = (float *)malloc(sizeof(float) * H);
        L->mlp_norm = (float *)malloc(sizeof(float) * H);
        L->kc = (float *)calloc((size_t)kvh * c->max_seq * D, sizeof(float));
        L->vc = (float *)calloc((size_t)kvh * c->max_seq * D, sizeof(float));
    }
    m->embed = (float *)malloc(sizeof(float) * (size_t)c->vocab * H);
    m->final_norm = (float *)malloc(sizeof(float) * H);
    lin_alloc(&m->lm_head, c->vocab, H, c->tied_embeddings ? 0 : c->weight_format);
    return m;
}

void orc_model_destroy(orc_model *m)
{
    if (!m)
        return;
    for (int i = 0; i < m->c.n_layers; i++) {
        orc_layer *L = &m->L[i];
        lin_free(&L->q);
        lin_free(&L->k);
        lin_free(&L->v);
        lin_free(&L->o);
        lin_free(&L->gate_up);
        lin_free(&L->down);
        free(L->attn_norm);
        free(L->mlp_norm);
        free(L->kc);
        free(L->vc);
    }
    free(m->L);
    free(m->embed);
    free(m->final_norm);
    lin_free(&m->lm_head);
    free(m);
}

static void synth_lin(orc_lin *l, uint64_t seed, uint32_t layer, uint32_t tensor, size_t n, size_t k, size_t row0)
{
    if (l->q4)
        orc_synth_q4(seed, layer, tensor, n, k, l->q4 + row0 * k / 2, l->s + row0 * k / 32);
    else
        orc_synth_q8(seed, layer, tensor, n, k, l->q8 + row0 * k, l->s + row0 * k / 32);
}

/* GQA row replication of src/core/loader.rs:62-98: each KV head's D rows are
 * repeated n_rep times in place (the source occupies the first n_kv*D rows). */
static void expand_rows(orc_lin *l, int n_kv, int n_rep, int D)
{
    size_t k = l->k;
    size_t rowb = l->q4 ? k / 2 : k, rows_s = k / 32;
    uint8_t *cb = l->q4 ? l->q4 : (uint8_t *)l->q8;
    for (int g = n_kv - 1; g >= 0; g--)
        for (int r = n_rep - 1; r >= 0; r--) {
            size_t dst = (size_t)(g * n_rep + r) * D, src = (size_t)g * D;
            memmove(cb + dst * rowb, cb + src * rowb, (size_t)D * rowb);
            memmove(l->s + dst * rows_s, l->s + src * rows_s, sizeof(float) * (size_t)D * rows_s);
        }
}

void orc_model_init_synthetic(orc_model *m, uint64_t seed)
{
    const orc_config *c = &m->c;
    int D = c->head_dim, H = c->hidden, F = c->ffn;
    int n_rep = c->n_heads / c->n_kv_heads;
    for (int i = 0; i < c->n_layers; i++) {
        orc_layer *L = &m->L[i];
        synth_lin(&L->q, seed, i, LLMRS_T_Q, (size_t)c->n_heads * D, H, 0);
        synth_lin(&L->k, seed, i, LLMRS_T_K, (size_t)c->n_kv_heads * D, H, 0);
        synth_lin(&L->v, seed, i, LLMRS_T_V, (size_t)c->n_kv_heads * D, H, 0);
        if (m->expand && n_rep > 1) {
            expand_rows(&L->k, c->n_kv_heads, n_rep, D);
            expand_rows(&L->v, c->n_kv_heads, n_rep, D);
        }
        synth_lin(&L->o, seed, i, LLMRS_T_O, H, (size_t)c->n_heads * D, 0);
        /* gate rows first, then up rows: src/core/loader.rs:128-147 */
        synth_lin(&L->gate_up, seed, i, LLMRS_T_GATE, F, H, 0);
        synth_lin(&L->gate_up, seed, i, LLMRS_T_UP, F, H, F);
        synth_lin(&L->down, seed, i, LLMRS_T_DOWN, H, F, 0);
        orc_synth_normal(seed, i, LLMRS_T_ATTN_NORM, H, 1.0f, 0.02f, L->attn_norm);
        orc_synth_normal(seed, i, LLMRS_T_MLP_NORM, H, 1.0f, 0.02f, L->mlp_norm);
    }
    orc_synth_normal(seed, LLMRS_GLOBAL_LAYER, LLMRS_T_EMBED, (size_t)c->vocab * H, 1.0f, 0.02f, m->embed);
    orc_synth_normal(seed, LLMRS_GLOBAL_LAYER, LLMRS_T_FINAL_NORM, H, 1.0f, 0.02f, m->final_norm);
    if (c->tied_embeddings) /* src/core/loader.rs:186-190 */
        orc_quantize_q4(m->embed, (size_t)c->vocab * H, m->lm_head.q4, m->lm_head.s);
    else
        synth_lin(&m->lm_head, seed, LLMRS_GLOBAL_LAYER, LLMRS_T_LM_HEAD, c->vocab, H, 0);
}

void orc_model_kv_fill_synthetic(orc_model *m, uint64_t seed, int n_pos)
{
    const orc_config *c = &m->c;
    int D = c->head_dim, S = c->max_seq;
    int n_rep = m->expand ? c->n_heads / c->n_kv_heads : 1;
    for (int i = 0; i < c->n_layers; i++) {
        orc_layer *L = &m->L[i];
        uint64_t sk = llmrs_stream(seed, i, LLMRS_T_KCACHE, LLMRS_SUB_F32);
        uint64_t sv = llmrs_stream(seed, i, LLMRS_T_VCACHE, LLMRS_SUB_F32);
#pragma omp parallel for collapse(2) schedule(static)
        for (int h = 0; h < m->cache_heads; h++)
            for (int t = 0; t < n_pos; t++) {
                int g = h / n_rep;
                for (int d = 0; d < D; d++) {
                    uint64_t idx = llmrs_kv_index(g, t, d, D);
                    L->kc[((size_t)h * S + t) * D + d] = llmrs_normal(sk, idx);
                    L->vc[((size_t)h * D + d) * S + t] = llmrs_normal(sv, idx);
                }
            }
    }
}

/* LlamaAttention::forward: src/core/layer.rs:175-333 */
static void attention(orc_model *m, orc_layer *L, const float *x, int seq, int start_pos, float *out)
{
    const orc_config *c = &m->c;
    int D = c->head_dim, Hq = c->n_heads, S = c->max_seq;
    int qdim = Hq * D, kvdim = m->cache_heads * D;
    int n_rep_cache = Hq / m->cache_heads;
    int total = start_pos + seq;
    float *q_all = (float *)malloc(sizeof(float) * (size_t)seq * qdim);
    float *k_all = (float *)malloc(sizeof(float) * (size_t)seq * kvdim);
    float *v_all = (float *)malloc(sizeof(float) * (size_t)seq * kvdim);
    float *ctx = (float *)calloc((size_t)seq * qdim, sizeof(float));
    lin_forward(&L->q, x, seq, q_all);
    lin_forward(&L->k, x, seq, k_all);
    lin_forward(&L->v, x, seq, v_all);

    /* RoPE on K and the cache append (layer.rs:216-246).  With expansion every
     * head owns a cache; natively a KV head's cache is shared by n_rep query
     * heads and is written once, before any of them reads it. */
#pragma omp parallel for schedule(static)
    for (int g = 0; g < m->cache_heads; g++) {
        float *kh = (float *)malloc(sizeof(float) * (size_t)seq * D);
        for (int i = 0; i < seq; i++)
            memcpy(kh + (size_t)i * D, k_all + (size_t)i * kvdim + (size_t)g * D, sizeof(float) * D);
        orc_rope_inplace(kh, seq, D, start_pos, c->rope_theta);
        for (int i = 0; i < seq; i++) {
            int pos = start_pos + i;
            memcpy(L->kc + ((size_t)g * S + pos) * D, kh + (size_t)i * D, sizeof(float) * D);
            for (int d = 0; d < D; d++)
                L->vc[((size_t)g * D + d) * S + pos] = v_all[(size_t)i * kvdim + (size_t)g * D + d];
        }
        free(kh);
    }

#pragma omp parallel for schedule(dynamic, 1)
    for (int h = 0; h < Hq; h++) {
        int g = h / n_rep_cache;
        float *qh = (float *)malloc(sizeof(float) * (size_t)seq * D);
        float *sc = (float *)malloc(sizeof(float) * (size_t)seq * total);
        float *pr = (float *)malloc(sizeof(float) * (size_t)seq * total);
        for (int i = 0; i < seq; i++)
            memcpy(qh + (size_t)i * D, q_all + (size_t)i * qdim + (size_t)h * D, sizeof(float) * D);
        orc_rope_inplace(qh, seq, D, start_pos, c->rope_theta);
        const float *kslice = L->kc + (size_t)g * S * D;
        for (int i = 0; i < seq; i++)
            for (int t = 0; t < total; t++)
                sc[(size_t)i * total + t] = orc_dot(qh + (size_t)i * D, kslice + (size_t)t * D, D);
        float inv_sqrt = 1.0f / sqrtf((float)D);
        orc_scale(sc, sc, (size_t)seq * total, inv_sqrt);
        if (seq > 1)
            for (int i = 0; i < seq; i++)
                for (int t = 0; t < total; t++)
                    if (t > start_pos + i)
                        sc[(size_t)i * total + t] = -INFINITY;
        orc_softmax(sc, pr, seq, total);
        const float *vbase = L->vc + (size_t)g * D * S;
        if (seq == 1) {
            for (int d = 0; d < D; d++) { /* layer.rs:276-299 */
                float sum = 0.0f;
                const float *vrow = vbase + (size_t)d * S;
                for (int t = 0; t < total; t++)
                    sum += pr[t] * vrow[t];
                ctx[(size_t)h * D + d] = sum;
            }
        } else {
            /* layer.rs:300-326: gather V history, then CpuBackend::matmul (SAXPY) */
            for (int i = 0; i < seq; i++) {
                float *row = ctx + (size_t)i * qdim + (size_t)h * D;
                for (int p = 0; p < total; p++) {
                    float val = pr[(size_t)i * total + p];
                    if (val == 0.0f)
                        continue;
                    for (int d = 0; d < D; d++)
                        row[d] += val * vbase[(size_t)d * S + p];
                }
            }
        }
        free(qh);
        free(sc);
        free(pr);
    }
    lin_forward(&L->o, ctx, seq, out);
    free(q_all);
    free(k_all);
    free(v_all);
    free(ctx);
}

/* LlamaMLP::forward: src/core/layer.rs:37-97 */
static void mlp(orc_model *m, orc_layer *L, const float *x, int seq, float *out)
{
    int F = m->c.ffn;
    float *fused = (float *)malloc(sizeof(float) * (size_t)seq * 2 * F);
    float *act = (float *)malloc(sizeof(float) * (size_t)seq * F);
    lin_forward(&L->gate_up, x, seq, fused);
    for (int i = 0; i < seq; i++) {
        const float *g = fused + (size_t)i * 2 * F, *u = g + F;
        float *d = act + (size_t)i * F;
        for (int j = 0; j < F; j++) {
            float gv = g[j];
            float silu = gv / (1.0f + expf(-gv));
            d[j] = silu * u[j];
        }
    }
    lin_forward(&L->down, act, seq, out);
    free(fused);
    free(act);
}

/* LlamaModel::forward (src/core/model.rs:17-49) + LlamaBlock::forward
 * (src/core/layer.rs:373-406).  The LM head is applied to the last row only:
 * rows are independent in matmul_transposed, so its logits equal the last row
 * of the reference's all-rows LM head (model.rs:47). */
int orc_model_forward_embeds(orc_model *m, const float *xin, int n, int start_pos, float *logits_last)
{
    const orc_config *c = &m->c;
    int H = c->hidden;
    if (n <= 0 || start_pos + n > c->max_seq)
        return -1;
    size_t sz = sizeof(float) * (size_t)n * H;
    float *x = (float *)malloc(sz), *hn = (float *)malloc(sz), *a = (float *)malloc(sz), *f = (float *)malloc(sz);
    memcpy(x, xin, sz);
    const size_t last = (size_t)(n - 1) * H;
    for (int l = 0; l < c->n_layers; l++) {
        orc_layer *L = &m->L[l];
        if (m->trace)
            memcpy(m->trace + (size_t)(2 * l) * H, x + last, sizeof(float) * H);
        orc_rms_norm(x, L->attn_norm, hn, n, H, c->rms_eps);
        attention(m, L, hn, n, start_pos, a);
        orc_add_assign(a, x, (size_t)n * H); /* attn_out += x */
        if (m->trace)
            memcpy(m->trace + (size_t)(2 * l + 1) * H, a + last, sizeof(float) * H);
        orc_rms_norm(a, L->mlp_norm, hn, n, H, c->rms_eps);
        mlp(m, L, hn, n, f);
        orc_add_assign(f, a, (size_t)n * H); /* mlp_out += h */
        float *t = x;
        x = f;
        f = t;
    }
    if (m->trace)
        memcpy(m->trace + (size_t)(2 * c->n_layers) * H, x + last, sizeof(float) * H);
    orc_rms_norm(x + last, m->final_norm, hn, 1, H, c->rms_eps);
    lin_forward(&m->lm_head, hn, 1, logits_last);
    free(x);
    free(hn);
    free(a);
    free(f);
    return 0;
}

/* embedding gather: src/main.rs:159-171 */
int orc_model_forward(orc_model *m, const int *ids, int n, int start_pos, float *logits_last)
{
    int H = m->c.hidden;
    float *x = (float *)malloc(sizeof(float) * (size_t)n * H);
    for (int i = 0; i < n; i++) {
        if (ids[i] < 0 || ids[i] >= m->c.vocab) {
            free(x);
            return -2;
        }
        memcpy(x + (size_t)i * H, m->embed + (size_t)ids[i] * H, sizeof(float) * H);
    }
    int rc = orc_model_forward_embeds(m, x, n, start_pos, logits_last);
    free(x);
    return rc;
}

int orc_model_tensor(orc_model *m, int layer, int which, void **qs, void **scales, size_t *n_rows, size_t *k)
{
    orc_lin *l = NULL;
    float *vec = NULL;
    size_t vn = 0;
    if (which == ORC_W_EMBED) {
        *qs = m->embed;
        *scales = NULL;
        *n_rows = (size_t)m->c.vocab;
        *k = (size_t)m->c.hidden;
        return 0;
    }
    if (which == ORC_W_FINAL_NORM) {
        vec = m->final_norm;
        vn = (size_t)m->c.hidden;
    } else if (which == ORC_W_LM_HEAD) {
        l = &m->lm_head;
    } else {
        if (layer < 0 || layer >= m->c.n_layers)
            return -1;
        orc_layer *L = &m->L[layer];
        switch (which) {
        case ORC_W_Q: l = &L->q; break;
        case ORC_W_K: l = &L->k; break;
        case ORC_W_V: l = &L->v; break;
        case ORC_W_O: l = &L->o; break;
        case ORC_W_GATE_UP: l = &L->gate_up; break;
        case ORC_W_DOWN: l = &L->down; break;
        case ORC_W_ATTN_NORM: vec = L->attn_norm; vn = (size_t)m->c.hidden; break;
        case ORC_W_MLP_NORM: vec = L->mlp_norm; vn = (size_t)m->c.hidden; break;
        default: return -1;
        }
    }
    if (vec) {
        *qs = vec;
        *scales = NULL;
        *n_rows = 1;
        *k = vn;
        return 0;
    }
    *qs = l->q4 ? (void *)l->q4 : (void *)l->q8;
    *scales = l->s;
    *n_rows = l->n;
    *k = l->k;
    return 0;
}

void orc_model_set_trace(orc_model *m, float *buf) { m->trace = buf; }

float *orc_model_kcache(orc_model *m, int layer) { return m->L[layer].kc; }
float *orc_model_vcache(orc_model *m, int layer) { return m->L[layer].vc; }
size_t orc_model_cache_heads(orc_model *m) { return (size_t)m->cache_heads; }
