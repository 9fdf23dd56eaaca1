// ops.cu - the remaining Backend-trait operations (src/backend.rs:20-39) as
// sm_100a kernels on device f32 buffers, plus the bit-exact quantisers and the
// synthetic-weight generators.
//
// These are the op-level drop-ins; the decode step itself fuses them into the
// GEMV prologues/epilogues and the attention kernel.  Reductions that the
// reference performs sequentially (dot products, RMSNorm sum of squares,
// softmax sum) are sequential per thread here where the op is small enough
// (matmul/matmul_slice) and fixed-order tree reductions otherwise; every
// product/sum the reference rounds separately is rounded separately here
// (__fmul_rn/__fadd_rn), so no FMA contraction changes results.
#include <cuda_fp16.h>

#include "common.cuh"
#include "llmrs_synth.h"
#include "ops.cuh"

namespace llmrs {

namespace {

constexpr int EW_THREADS = 256;

inline int ew_grid(size_t n)
{
    size_t g = (n + EW_THREADS - 1) / EW_THREADS;
    return (int)(g > 65535 * 8 ? 65535 * 8 : (g < 1 ? 1 : g));
}

__global__ void add_assign_kernel(float *a, const float *b, size_t n)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        a[i] = __fadd_rn(a[i], b[i]);
}

// src/backend/cpu.rs:316-323: silu = g / (1 + exp(-g)); g = silu * u
__global__ void silu_mul_kernel(float *g, const float *u, size_t n)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float x = g[i];
        const float s = __fdiv_rn(x, __fadd_rn(1.0f, expf(-x)));
        g[i] = __fmul_rn(s, u[i]);
    }
}

__global__ void scale_kernel(const float *x, float *y, size_t n, float v)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __fmul_rn(x[i], v);
}

__global__ void copy_kernel(const float *x, float *y, size_t n)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = x[i];
}

// src/backend/cpu.rs:326-357 (theta computed on the device with CUDA's powf,
// sinf, cosf; the decode step instead uses a table built with the host libm)
__global__ void rope_kernel(float *x, int rows, int head_dim, int start_pos, float theta_base)
{
    const int mid = head_dim / 2;
    const size_t total = (size_t)rows * mid;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const int i = (int)(e / mid), j = (int)(e % mid);
        float *chunk = x + (size_t)i * head_dim;
        const float freq = __fdiv_rn((float)j * 2.0f, (float)head_dim);
        const float theta = __fdiv_rn(1.0f, powf(theta_base, freq));
        const float m = __fmul_rn((float)(start_pos + i), theta);
        const float sn = sinf(m), cs = cosf(m);
        const float re = chunk[j], im = chunk[j + mid];
        chunk[j] = __fsub_rn(__fmul_rn(re, cs), __fmul_rn(im, sn));
        chunk[j + mid] = __fadd_rn(__fmul_rn(re, sn), __fmul_rn(im, cs));
    }
}

// src/backend/cpu.rs:359-393, one CTA per row, fixed-order tree reduction
__global__ void rms_norm_kernel(const float *x, const float *w, float *y, int cols, float eps)
{
    __shared__ float red[32];
    const float *in = x + (size_t)blockIdx.x * cols;
    float *out = y + (size_t)blockIdx.x * cols;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < cols; i += blockDim.x)
        ss = __fadd_rn(ss, __fmul_rn(in[i], in[i]));
    ss = warp_sum(ss);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (lane == 0)
        red[warp] = ss;
    __syncthreads();
    float tot = red[0];
    for (int k = 1; k < nw; k++)
        tot = __fadd_rn(tot, red[k]);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)cols), eps));
    const float scale = __fdiv_rn(1.0f, rms);
    for (int i = threadIdx.x; i < cols; i += blockDim.x)
        out[i] = __fmul_rn(__fmul_rn(in[i], scale), w[i]);
}

// src/backend/cpu.rs:395-423, one CTA per row
__global__ void softmax_kernel(const float *x, float *y, int cols)
{
    __shared__ float red[32];
    __shared__ float bcast;
    const float *in = x + (size_t)blockIdx.x * cols;
    float *out = y + (size_t)blockIdx.x * cols;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float m = -3.40282347e+38f; // f32::MIN
    for (int i = threadIdx.x; i < cols; i += blockDim.x)
        m = fmaxf(m, in[i]);
    m = warp_max(m);
    if (lane == 0)
        red[warp] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = red[0];
        for (int k = 1; k < nw; k++)
            t = fmaxf(t, red[k]);
        bcast = t;
    }
    __syncthreads();
    m = bcast;
    float s = 0.0f;
    for (int i = threadIdx.x; i < cols; i += blockDim.x) {
        const float e = expf(__fsub_rn(in[i], m));
        out[i] = e;
        s = __fadd_rn(s, e);
    }
    s = warp_sum(s);
    __syncthreads();
    if (lane == 0)
        red[warp] = s;
    __syncthreads();
    float tot = red[0];
    for (int k = 1; k < nw; k++)
        tot = __fadd_rn(tot, red[k]);
    const float inv = __fdiv_rn(1.0f, tot);
    for (int i = threadIdx.x; i < cols; i += blockDim.x)
        out[i] = __fmul_rn(out[i], inv);
}

// Backend::matmul_transposed (f32) / matmul_slice: thread per output,
// sequential dot exactly as the x86 simd_dot_f32 (src/backend/cpu.rs:546-549)
__global__ void matmul_t_kernel(const float *a, const float *b, float *c, int m, int k, int n)
{
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y;
    if (j >= n || i >= m)
        return;
    const float *ar = a + (size_t)i * k, *br = b + (size_t)j * k;
    float s = 0.0f;
    for (int p = 0; p < k; p++)
        s = __fadd_rn(s, __fmul_rn(ar[p], br[p]));
    c[(size_t)i * n + j] = s;
}

// Backend::matmul: SAXPY order, zero multipliers skipped (src/backend/cpu.rs:203-221)
__global__ void matmul_kernel(const float *a, const float *b, float *c, int m, int k, int n)
{
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const int i = blockIdx.y;
    if (j >= n || i >= m)
        return;
    const float *ar = a + (size_t)i * k;
    float s = 0.0f;
    for (int p = 0; p < k; p++) {
        const float v = ar[p];
        if (v == 0.0f)
            continue;
        s = __fadd_rn(s, __fmul_rn(v, b[(size_t)p * n + j]));
    }
    c[(size_t)i * n + j] = s;
}

// quantize_row_q8_0 (src/backend/cpu.rs:724-743): one warp per 32-block
__global__ void quantize_q8_kernel(const float *x, int8_t *q, float *s, size_t nblocks)
{
    const size_t b = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (b >= nblocks)
        return;
    const float v = x[b * 32 + lane];
    const float amax = warp_max(fabsf(v));
    int qv = 0;
    float scale = 0.0f;
    if (amax != 0.0f) {
        scale = __fdiv_rn(amax, 127.0f);
        const float inv = __fdiv_rn(1.0f, scale);
        float r = roundf(__fmul_rn(v, inv));
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        qv = (r != r) ? 0 : (int)r;
    }
    q[b * 32 + lane] = (int8_t)qv;
    if (lane == 0)
        s[b] = scale;
}

// Tensor::quantize_q4 (src/core/tensor.rs:102-167): thread per block of 32
__global__ void quantize_q4_kernel(const float *w, size_t n, uint8_t *qs, float *scales)
{
    const size_t nblocks = (n + 31) / 32;
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nblocks; b += (size_t)gridDim.x * blockDim.x) {
        const size_t base = b * 32;
        const int len = (int)(n - base < 32 ? n - base : 32);
        float amax = 0.0f;
        for (int i = 0; i < len; i++)
            amax = fmaxf(amax, fabsf(w[base + i]));
        const float scale = __fdiv_rn(amax, 7.0f);
        scales[b] = scale;
        const int pairs = (len + 1) / 2;
        uint8_t *out = qs + b * 16;
        if (scale == 0.0f) {
            for (int p = 0; p < pairs; p++)
                out[p] = 0x88;
        } else {
            const float inv = __fdiv_rn(1.0f, scale);
            for (int p = 0; p < pairs; p++) {
                const float v0 = w[base + 2 * p];
                const float v1 = (2 * p + 1 < len) ? w[base + 2 * p + 1] : 0.0f;
                float f0 = __fadd_rn(__fmul_rn(v0, inv), 8.5f);
                float f1 = __fadd_rn(__fmul_rn(v1, inv), 8.5f);
                f0 = f0 < 0.0f ? 0.0f : (f0 > 15.0f ? 15.0f : f0);
                f1 = f1 < 0.0f ? 0.0f : (f1 > 15.0f ? 15.0f : f1);
                const uint32_t q0 = (f0 != f0) ? 0u : (uint32_t)f0;
                const uint32_t q1 = (f1 != f1) ? 0u : (uint32_t)f1;
                out[p] = (uint8_t)(q0 | (q1 << 4));
            }
        }
    }
}

// ------------------------------------------------------- synthetic generators
// Quantised weight rows [row0, row0+nrows) x columns [col0, col0+ncols) of a
// logical [N][K] synthetic tensor, written to dst rows dst_row(r) of a
// [.][ncols] destination.  The destination row map supports the interleaved
// gate/up layout (dst row = 2*r + parity) and QKV concatenation (offset).
__global__ void synth_q4_kernel(uint64_t sc, uint64_t ss, int K, int row0, int nrows, int col0, int ncols,
                                uint8_t *dst_w, __half *dst_s16, float *dst_s32, int dst_row_mul, int dst_row_add)
{
    const size_t rowbytes = (size_t)ncols / 2;
    const size_t total = (size_t)nrows * rowbytes;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / rowbytes);
        const size_t cb = e % rowbytes;
        const uint64_t j = (uint64_t)(row0 + r) * (K / 2) + col0 / 2 + cb;
        const size_t drow = (size_t)r * dst_row_mul + dst_row_add;
        dst_w[drow * rowbytes + cb] = llmrs_synth_q4_byte(sc, j);
    }
    const size_t nbr = (size_t)ncols / 32;
    const size_t tsc = (size_t)nrows * nbr;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < tsc; e += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / nbr);
        const size_t bb = e % nbr;
        const uint64_t i = (uint64_t)(row0 + r) * (K / 32) + col0 / 32 + bb;
        const size_t drow = (size_t)r * dst_row_mul + dst_row_add;
        const uint16_t h = llmrs_synth_scale_f16(ss, i);
        if (dst_s16)
            dst_s16[drow * nbr + bb] = __ushort_as_half(h);
        else
            dst_s32[drow * nbr + bb] = llmrs_f16_to_f32(h);
    }
}

__global__ void synth_q8_kernel(uint64_t sc, uint64_t ss, int K, int row0, int nrows, int col0, int ncols,
                                int8_t *dst_w, __half *dst_s16, float *dst_s32, int dst_row_mul, int dst_row_add)
{
    const size_t total = (size_t)nrows * ncols;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / ncols);
        const size_t c = e % ncols;
        const uint64_t j = (uint64_t)(row0 + r) * K + col0 + c;
        const size_t drow = (size_t)r * dst_row_mul + dst_row_add;
        dst_w[drow * ncols + c] = llmrs_synth_q8_code(sc, j);
    }
    const size_t nbr = (size_t)ncols / 32;
    const size_t tsc = (size_t)nrows * nbr;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < tsc; e += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(e / nbr);
        const size_t bb = e % nbr;
        const uint64_t i = (uint64_t)(row0 + r) * (K / 32) + col0 / 32 + bb;
        const size_t drow = (size_t)r * dst_row_mul + dst_row_add;
        const uint16_t h = llmrs_synth_scale_f16(ss, i);
        if (dst_s16)
            dst_s16[drow * nbr + bb] = __ushort_as_half(h);
        else
            dst_s32[drow * nbr + bb] = llmrs_f16_to_f32(h);
    }
}

__global__ void synth_normal_kernel(uint64_t st, size_t n, float mu, float sd, float *out)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = llmrs_normal_ms(st, i, mu, sd);
}

// KV pre-fill for kv heads [h0, h0+nh) of a layer: cache [nh][S][D]
__global__ void synth_kv_kernel(uint64_t sk, uint64_t sv, int h0, int nh, int n_pos, int S, int D, float *kc,
                                float *vc)
{
    const size_t total = (size_t)nh * n_pos * D;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const int d = (int)(e % D);
        const int t = (int)((e / D) % n_pos);
        const int h = (int)(e / ((size_t)D * n_pos));
        const uint64_t idx = llmrs_kv_index((uint32_t)(h0 + h), (uint32_t)t, (uint32_t)d, (uint32_t)D);
        const size_t o = ((size_t)h * S + t) * D + d;
        kc[o] = llmrs_normal(sk, idx);
        vc[o] = llmrs_normal(sv, idx);
    }
}

__global__ void f32_to_f16_scales_kernel(const float *src, __half *dst, size_t n, uint32_t *inexact)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const uint16_t h = llmrs_f32_to_f16(src[i]);
        if (llmrs_f16_to_f32(h) != src[i])
            atomicOr(inexact, 1u);
        dst[i] = __ushort_as_half(h);
    }
}

// bf16 -> f32 (the top 16 bits of the f32: exact, as half::bf16::to_f32,
// src/core/loader.rs:37-41)
__global__ void bf16_to_f32_kernel(const uint16_t *src, float *dst, size_t n)
{
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = __uint_as_float((uint32_t)src[i] << 16);
}

} // namespace

// ------------------------------------------------------------ host launchers
int op_bf16_to_f32(cudaStream_t s, const uint16_t *src, float *dst, size_t n)
{
    if (n == 0)
        return LLMRS_OK;
    bf16_to_f32_kernel<<<ew_grid(n), EW_THREADS, 0, s>>>(src, dst, n);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int op_add_assign(cudaStream_t s, float *a, const float *b, size_t n)
{
    add_assign_kernel<<<ew_grid(n), EW_THREADS, 0, s>>>(a, b, n);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int op_silu_mul(cudaStream_t s, float *g, const float *u, size_t n)
{
    silu_mul_kernel<<<ew_grid(n), EW_THREADS, 0, s>>>(g, u, n);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int op_scale(cudaStream_t s, const float *x, float *y, size_t n, float v)
{
    scale_kernel<<<ew_grid(n), EW_THREADS, 0, s>>>(x, y, n, v);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int op_copy(cudaStream_t s, const float *x, float *y, size_t n)
{
    copy_kernel<<<ew_grid(n), EW_THREADS, 0, s>>>(x, y, n);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int op_rope(cudaStream_t s, float *x, int rows, int head_dim, int start_pos, float theta)
{
    LLMRS_CHECK_ARG(head_dim > 0 && head_dim % 2 == 0, "rope: head_dim %d must be even", head_dim);
    rope_kernel<<<ew_grid((size_t)rows * head_dim / 2), EW_THREADS, 0, s>>>(x, rows, head_dim, start_pos, theta);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int op_rms_norm(cudaStream_t s, const float *x, const float *w, float *y, int rows, int cols, float eps)
{
    rms_norm_kernel<<<rows, 256, 0, s>>>(x, w, y, cols, eps);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int op_softmax(cudaStream_t s, const float *x, float *y, int rows, int cols)
{
    softmax_kernel<<<rows, 256, 0, s>>>(x, y, cols);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int op_matmul_t(cudaStream_t s, const float *a, const float *b, float *c, int m, int k, int n)
{
    matmul_t_kernel<<<dim3((n + 127) / 128, m), 128, 0, s>>>(a, b, c, m, k, n);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int op_matmul(cudaStream_t s, const float *a, const float *b, float *c, int m, int k, int n)
{
    matmul_kernel<<<dim3((n + 127) / 128, m), 128, 0, s>>>(a, b, c, m, k, n);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int op_quantize_q8(cudaStream_t s, const float *x, int8_t *q, float *sc, size_t nblocks)
{
    if (nblocks == 0)
        return LLMRS_OK;
    const size_t threads = nblocks * 32;
    quantize_q8_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, q, sc, nblocks);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int op_quantize_q4(cudaStream_t s, const float *w, size_t n, uint8_t *qs, float *scales)
{
    if (n == 0)
        return LLMRS_OK;
    quantize_q4_kernel<<<ew_grid((n + 31) / 32), EW_THREADS, 0, s>>>(w, n, qs, scales);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int synth_quant(cudaStream_t s, int wf, uint64_t seed, uint32_t layer, uint32_t tensor, int K, int row0, int nrows,
                int col0, int ncols, void *dst_w, void *dst_s, int st, int dst_row_mul, int dst_row_add)
{
    const uint64_t ss = llmrs_stream(seed, layer, tensor, LLMRS_SUB_SCALES);
    __half *s16 = st == 0 ? reinterpret_cast<__half *>(dst_s) : nullptr;
    float *s32 = st == 1 ? reinterpret_cast<float *>(dst_s) : nullptr;
    const size_t work = (size_t)nrows * ncols / (wf == 0 ? 2 : 1);
    if (wf == 0) {
        const uint64_t sc = llmrs_stream(seed, layer, tensor, LLMRS_SUB_Q4CODES);
        synth_q4_kernel<<<ew_grid(work), EW_THREADS, 0, s>>>(sc, ss, K, row0, nrows, col0, ncols,
                                                             reinterpret_cast<uint8_t *>(dst_w), s16, s32,
                                                             dst_row_mul, dst_row_add);
    } else {
        const uint64_t sc = llmrs_stream(seed, layer, tensor, LLMRS_SUB_Q8CODES);
        synth_q8_kernel<<<ew_grid(work), EW_THREADS, 0, s>>>(sc, ss, K, row0, nrows, col0, ncols,
                                                             reinterpret_cast<int8_t *>(dst_w), s16, s32,
                                                             dst_row_mul, dst_row_add);
    }
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int synth_normal(cudaStream_t s, uint64_t seed, uint32_t layer, uint32_t tensor, size_t n, float mu, float sd,
                 float *out)
{
    const uint64_t st = llmrs_stream(seed, layer, tensor, LLMRS_SUB_F32);
    synth_normal_kernel<<<ew_grid(n), EW_THREADS, 0, s>>>(st, n, mu, sd, out);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int synth_kv(cudaStream_t s, uint64_t seed, uint32_t layer, int h0, int nh, int n_pos, int S, int D, float *kc,
             float *vc)
{
    const uint64_t sk = llmrs_stream(seed, layer, LLMRS_T_KCACHE, LLMRS_SUB_F32);
    const uint64_t sv = llmrs_stream(seed, layer, LLMRS_T_VCACHE, LLMRS_SUB_F32);
    synth_kv_kernel<<<ew_grid((size_t)nh * n_pos * D), EW_THREADS, 0, s>>>(sk, sv, h0, nh, n_pos, S, D, kc, vc);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int scales_to_f16(cudaStream_t s, const float *src, void *dst, size_t n, uint32_t *d_flag)
{
    f32_to_f16_scales_kernel<<<ew_grid(n), EW_THREADS, 0, s>>>(src, reinterpret_cast<__half *>(dst), n, d_flag);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

} // namespace llmrs
