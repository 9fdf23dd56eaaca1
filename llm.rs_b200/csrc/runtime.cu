// runtime.cu - context, device-resident model and the C ABI (include/llmrs_cuda.h).
//
// The model keeps every weight in the reference's block formats in one HBM
// arena (Q4_0 nibbles / Q8_0 codes + block scales), a position-major fp32 KV
// cache per layer, and a small set of activation buffers.  One decode step is
// 5 kernels per layer + the LM head (see enqueue_step) and is captured once as
// a CUDA graph; programmatic dependent launch lets each GEMV start streaming
// its weights while the previous kernel finishes.
#include <cuda_fp16.h>
#include <math.h>
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "prefill.cuh"
#include "sample.cuh"
#include "llmrs_synth.h"
#include "ops.cuh"

// ------------------------------------------------------------------ errors
namespace llmrs {

static thread_local char g_err[1024] = "";

void set_error(const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int fail(int code, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int num_sms(int device)
{
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
        n = 148;
    return n;
}

} // namespace llmrs

using namespace llmrs;

struct llmrs_ctx {
    int device = 0;
    int sms = 148;
    cudaStream_t own = nullptr;
    cudaStream_t stream = nullptr;
    uint32_t *d_err = nullptr; // op-level device error word
    void *scratch = nullptr;   // op-level scratch (attention split partials), grown on demand
    size_t scratch_bytes = 0;
};

namespace {

struct QW {
    uint8_t *w = nullptr; // codes
    void *s = nullptr;    // scales
    int n = 0, k = 0;
    int st = 0;           // LLMRS_F16 / LLMRS_F32
    GemvPlan plan;        // launch geometry + tensor maps (weights never move)
};

struct LayerW {
    QW qkv, o, gate_up, down;
    PrefillWeights p_qkv, p_o, p_gate_up, p_down; // tensor maps of the M>1 (prefill) path
    float *attn_norm = nullptr, *mlp_norm = nullptr;
    float *kc = nullptr, *vc = nullptr;
};

struct Arena {
    uint8_t *base = nullptr;
    size_t size = 0, used = 0;
    void *take(size_t bytes)
    {
        size_t off = (used + 255) & ~size_t(255);
        if (off + bytes > size)
            return nullptr;
        used = off + bytes;
        return base + off;
    }
};

inline size_t wbytes(int wf, size_t n, size_t k) { return wf == 0 ? n * k / 2 : n * k; }

int check_cfg(const llmrs_config *c)
{
    LLMRS_CHECK_ARG(c, "config is NULL");
    LLMRS_CHECK_ARG(c->n_layers > 0 && c->hidden > 0 && c->n_heads > 0 && c->n_kv_heads > 0 && c->head_dim > 0 &&
                        c->ffn > 0 && c->vocab > 0 && c->max_seq > 0,
                    "config: all sizes must be positive");
    LLMRS_CHECK_ARG(c->n_heads % c->n_kv_heads == 0, "config: n_heads %d not a multiple of n_kv_heads %d",
                    c->n_heads, c->n_kv_heads);
    LLMRS_CHECK_ARG(c->hidden % 32 == 0 && c->ffn % 32 == 0 && (c->n_heads * c->head_dim) % 32 == 0,
                    "config: hidden, ffn and n_heads*head_dim must be multiples of 32");
    LLMRS_CHECK_ARG(c->head_dim == 64 || c->head_dim == 128, "config: head_dim %d not supported (64 or 128)",
                    c->head_dim);
    const int nrep = c->n_heads / c->n_kv_heads;
    LLMRS_CHECK_ARG(nrep == 4 || nrep == 8, "config: n_heads/n_kv_heads = %d not supported (4 or 8)", nrep);
    LLMRS_CHECK_ARG(c->weight_format == LLMRS_WFMT_Q4_0 || c->weight_format == LLMRS_WFMT_Q8_0,
                    "config: weight_format %d unknown", c->weight_format);
    LLMRS_CHECK_ARG(!c->tied_embeddings || c->weight_format == LLMRS_WFMT_Q4_0,
                    "config: tied embeddings require Q4_0 (quantize_q4 of the embedding)");
    LLMRS_CHECK_ARG(c->scale_dtype == LLMRS_F16 || c->scale_dtype == LLMRS_F32, "config: scale_dtype %d unknown",
                    c->scale_dtype);
    const int T = c->tp_size > 0 ? c->tp_size : 1;
    LLMRS_CHECK_ARG(T == 1 || T == 2 || T == 4 || T == 8, "config: tp_size %d not 1, 2, 4 or 8", c->tp_size);
    LLMRS_CHECK_ARG(c->tp_rank >= 0 && c->tp_rank < T, "config: tp_rank %d outside [0,%d)", c->tp_rank, T);
    LLMRS_CHECK_ARG(c->n_kv_heads % T == 0 && c->vocab % T == 0 && (c->ffn / T) % 32 == 0 &&
                        (c->n_heads / T * c->head_dim) % 32 == 0,
                    "config: n_kv_heads, vocab, ffn/32 and n_heads*head_dim/32 must split over tp_size %d", T);
    LLMRS_CHECK_ARG(T == 1 || !c->tied_embeddings || (c->vocab / T) % 1 == 0, "config: bad vocab shard");
    return LLMRS_OK;
}

} // namespace

struct llmrs_model {
    llmrs_ctx *ctx = nullptr;
    llmrs_config cfg{};
    int wf = 0, st = 0;
    // Hq, Hkv, F: this rank's shard (the whole model for one GPU); V: full vocab,
    // Vl: this rank's LM-head rows
    int D = 0, Hq = 0, Hkv = 0, H = 0, F = 0, V = 0, Vl = 0, S = 0;
    int T = 1, rank = 0;
    Arena arena;
    std::vector<LayerW> layers;
    float *embed = nullptr, *final_norm = nullptr;
    QW lm_head;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    // activations
    float *x = nullptr, *qkv = nullptr, *ctxv = nullptr, *act = nullptr, *logits = nullptr, *part = nullptr;
    float *x1 = nullptr; // tensor parallel: second residual buffer (o_proj all-reduce target)
    // tensor parallel: communication region (own cudaMalloc, shared over IPC) and links
    void *tp_region = nullptr;
    size_t tp_bytes = 0, tp_off_o = 0, tp_off_d = 0, tp_off_keys = 0, tp_off_cnt = 0;
    TpLink *d_tp = nullptr;
    bool tp_connected = false;
    unsigned int *att_counter = nullptr;
    unsigned long long peer_ns = 5000000000ull; // tensor parallel: longest wait for another rank
    StepState *state = nullptr;
    int *token_log = nullptr;
    int log_cap = 0;
    int n_splits = 1;
    int kernels_per_step = 0;
    // graph of one decode step (and a copy that records a device timeline)
    cudaGraphExec_t graph = nullptr;
    cudaGraphExec_t graph_traced = nullptr;
    unsigned long long *d_trace = nullptr; // TRACE_MARKS marks per kernel
    // pinned host staging
    int *h_stage = nullptr; // 13 slots of 4 ints (token, pos) for H2D; [60..61]: next token, err
    int h_stage_n = 0;
    uint32_t *d_flag = nullptr;
    // prefill on the tensor cores: row buffers for chunks of up to pf_rows rows
    int pf_rows = 0;
    int pf_weights = -1; // -1: not checked, 0: some linear is off the tensor-core path, 1: ready
    void *pf_buf = nullptr;
    float *pf_x = nullptr, *pf_qkv = nullptr, *pf_ctx = nullptr, *pf_act = nullptr;
    int *pf_ids = nullptr;
    void *pf_acts = nullptr;
    void *pf_bf16 = nullptr; // bf16 copies of every linear (the bf16 prefill GEMM)
    int pf_bf = 0;
};

// ================================================================== C ABI
extern "C" {

const char *llmrs_last_error(void) { return g_err; }

const char *llmrs_version(void) { return "llmrs-b200 0.1 (sm_100a)"; }

const char *llmrs_backend_name(void) { return "Cuda"; }

int llmrs_device_count(int *count)
{
    LLMRS_CHECK_ARG(count, "count is NULL");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        *count = 0;
        return fail(LLMRS_ECUDA, "cudaGetDeviceCount: %s", cudaGetErrorString(e));
    }
    *count = n;
    return LLMRS_OK;
}

int llmrs_ctx_create(int device, llmrs_ctx **out)
{
    LLMRS_CHECK_ARG(out, "out is NULL");
    *out = nullptr;
    int n = 0;
    LLMRS_CUDA_TRY(cudaGetDeviceCount(&n));
    LLMRS_CHECK_ARG(device >= 0 && device < n, "device %d out of range (%d devices)", device, n);
    LLMRS_CUDA_TRY(cudaSetDevice(device));
    cudaDeviceProp prop;
    LLMRS_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(LLMRS_ENOTSUP, "device %d is sm_%d%d; this library is built for sm_100a (B200)", device,
                    prop.major, prop.minor);
    llmrs_ctx *c = new llmrs_ctx();
    c->device = device;
    c->sms = num_sms(device);
    cudaError_t e = cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking);
    if (e == cudaSuccess)
        e = cudaMalloc(&c->d_err, sizeof(uint32_t));
    if (e == cudaSuccess)
        e = cudaMemset(c->d_err, 0, sizeof(uint32_t));
    if (e != cudaSuccess) {
        delete c;
        return fail(LLMRS_ECUDA, "context set-up: %s", cudaGetErrorString(e));
    }
    c->stream = c->own;
    int rc = gemv_prepare();
    if (rc == LLMRS_OK)
        rc = attention_prepare();
    if (rc == LLMRS_OK)
        rc = prefill_prepare();
    if (rc != LLMRS_OK) {
        cudaFree(c->d_err);
        cudaStreamDestroy(c->own);
        delete c;
        return rc;
    }
    *out = c;
    return LLMRS_OK;
}

int llmrs_ctx_destroy(llmrs_ctx *ctx)
{
    if (!ctx)
        return LLMRS_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->scratch)
        cudaFree(ctx->scratch);
    if (ctx->d_err)
        cudaFree(ctx->d_err);
    if (ctx->own)
        cudaStreamDestroy(ctx->own);
    delete ctx;
    return LLMRS_OK;
}

int llmrs_ctx_set_stream(llmrs_ctx *ctx, void *s)
{
    LLMRS_CHECK_ARG(ctx, "ctx is NULL");
    ctx->stream = s ? reinterpret_cast<cudaStream_t>(s) : ctx->own;
    return LLMRS_OK;
}

int llmrs_ctx_device(llmrs_ctx *ctx, int *device)
{
    LLMRS_CHECK_ARG(ctx && device, "NULL argument");
    *device = ctx->device;
    return LLMRS_OK;
}

int llmrs_malloc(llmrs_ctx *ctx, size_t bytes, void **d_ptr)
{
    LLMRS_CHECK_ARG(ctx && d_ptr, "NULL argument");
    cudaSetDevice(ctx->device);
    cudaError_t e = cudaMalloc(d_ptr, bytes ? bytes : 16);
    if (e != cudaSuccess)
        return fail(LLMRS_ENOMEM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    return LLMRS_OK;
}

int llmrs_free(llmrs_ctx *ctx, void *d_ptr)
{
    LLMRS_CHECK_ARG(ctx, "ctx is NULL");
    if (!d_ptr)
        return LLMRS_OK;
    cudaSetDevice(ctx->device);
    LLMRS_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    LLMRS_CUDA_TRY(cudaFree(d_ptr));
    return LLMRS_OK;
}

int llmrs_h2d(llmrs_ctx *ctx, void *d_dst, const void *h_src, size_t bytes)
{
    LLMRS_CHECK_ARG(ctx && (bytes == 0 || (d_dst && h_src)), "NULL argument");
    LLMRS_CUDA_TRY(cudaMemcpyAsync(d_dst, h_src, bytes, cudaMemcpyHostToDevice, ctx->stream));
    return LLMRS_OK;
}

int llmrs_d2h(llmrs_ctx *ctx, void *h_dst, const void *d_src, size_t bytes)
{
    LLMRS_CHECK_ARG(ctx && (bytes == 0 || (h_dst && d_src)), "NULL argument");
    LLMRS_CUDA_TRY(cudaMemcpyAsync(h_dst, d_src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
    LLMRS_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    return LLMRS_OK;
}

int llmrs_d2d(llmrs_ctx *ctx, void *d_dst, const void *d_src, size_t bytes)
{
    LLMRS_CHECK_ARG(ctx && (bytes == 0 || (d_dst && d_src)), "NULL argument");
    LLMRS_CUDA_TRY(cudaMemcpyAsync(d_dst, d_src, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
    return LLMRS_OK;
}

int llmrs_memset(llmrs_ctx *ctx, void *d_dst, int value, size_t bytes)
{
    LLMRS_CHECK_ARG(ctx && (bytes == 0 || d_dst), "NULL argument");
    LLMRS_CUDA_TRY(cudaMemsetAsync(d_dst, value, bytes, ctx->stream));
    return LLMRS_OK;
}

static int ctx_check_err(llmrs_ctx *ctx)
{
    uint32_t e = 0;
    LLMRS_CUDA_TRY(cudaMemcpy(&e, ctx->d_err, sizeof(e), cudaMemcpyDeviceToHost));
    if (e) {
        cudaMemset(ctx->d_err, 0, sizeof(uint32_t));
        return fail(e == DEV_ERR_MBAR_TIMEOUT || e == DEV_ERR_PEER_TIMEOUT ? LLMRS_ETIMEDOUT : LLMRS_EDEVICE,
                    "device error word %u", e);
    }
    return LLMRS_OK;
}

int llmrs_sync(llmrs_ctx *ctx)
{
    LLMRS_CHECK_ARG(ctx, "ctx is NULL");
    LLMRS_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    return ctx_check_err(ctx);
}

// ---------------------------------------------------------------- ops
static int ctx_scratch(llmrs_ctx *ctx, size_t bytes, void **out);

static int gemv_op(llmrs_ctx *ctx, int wf, const float *a, const void *w, const void *scales, int st, float *c,
                   int m, int k, int n)
{
    LLMRS_CHECK_ARG(ctx && a && w && scales && c, "NULL argument");
    LLMRS_CHECK_ARG(m >= 1 && k >= 32 && k % 32 == 0 && n >= 1, "matmul_transposed: m=%d k=%d n=%d (k must be a multiple of 32)", m, k, n);
    LLMRS_CHECK_ARG(st == LLMRS_F16 || st == LLMRS_F32, "scale_dtype %d unknown", st);
    LLMRS_CHECK_ARG(!((uintptr_t)a & 15), "matmul_transposed: activation pointer must be 16-byte aligned");
    // rows of A are independent (the m>1 path quantises each row, src/backend/cpu.rs:90-110)
    if (m >= PREFILL_MIN_ROWS) {
        PrefillWeights pw;
        LLMRS_TRY(prefill_weights_init(&pw, w, scales, n, k, wf, st));
        if (pw.ok) { // tensor cores: per-row Q8_0 quantise, then one GEMM over all rows
            const int bf = prefill_use_bf16() && n % 4 == 0;
            const size_t ab = (prefill_acts_bytes(m, k) + 1023) & ~size_t(1023);
            void *scr = nullptr;
            LLMRS_TRY(ctx_scratch(ctx, ab + (bf ? prefill_bf16_bytes(n, k) : 0), &scr));
            if (bf) // this call's bf16 copy of the weights
                LLMRS_TRY(prefill_weights_to_bf16(&pw, w, scales, reinterpret_cast<uint8_t *>(scr) + ab, ctx->stream));
            PrefillActs acts;
            LLMRS_TRY(prefill_acts_init(&acts, scr, m, k, wf, bf));
            LLMRS_TRY(prefill_quantize(a, k, nullptr, 0.0f, acts, ctx->d_err, ctx->stream));
            return prefill_gemm(pw, acts, PEPI_STORE, c, n, nullptr, 0, ctx->d_err, ctx->sms, ctx->stream);
        }
    }
    GemvPlan plan;
    LLMRS_TRY(gemv_plan(&plan, w, scales, n, k, wf, st, false, ctx->sms));
    for (int i = 0; i < m; i++) {
        GemvParams p{};
        p.w = reinterpret_cast<const uint8_t *>(w);
        p.scales = scales;
        p.N = n;
        p.K = k;
        p.x = a + (size_t)i * k;
        p.y = c + (size_t)i * n;
        p.err = ctx->d_err;
        LLMRS_TRY(gemv_launch(plan, p, PRO_F32, EPI_STORE, ctx->stream, false));
    }
    return LLMRS_OK;
}

int llmrs_matmul_transposed_q4(llmrs_ctx *ctx, const float *d_a, const uint8_t *d_qs, const void *d_scales,
                               int scale_dtype, float *d_c, int m, int k, int n)
{
    return gemv_op(ctx, 0, d_a, d_qs, d_scales, scale_dtype, d_c, m, k, n);
}

int llmrs_matmul_transposed_q8(llmrs_ctx *ctx, const float *d_a, const int8_t *d_qw, const void *d_scales,
                               int scale_dtype, float *d_c, int m, int k, int n)
{
    return gemv_op(ctx, 1, d_a, d_qw, d_scales, scale_dtype, d_c, m, k, n);
}

int llmrs_matmul_transposed_f32(llmrs_ctx *ctx, const float *d_a, const float *d_b, float *d_c, int m, int k, int n)
{
    LLMRS_CHECK_ARG(ctx && d_a && d_b && d_c && m > 0 && k > 0 && n > 0, "matmul_transposed_f32: bad arguments");
    return op_matmul_t(ctx->stream, d_a, d_b, d_c, m, k, n);
}

int llmrs_matmul(llmrs_ctx *ctx, const float *d_a, const float *d_b, float *d_c, int m, int k, int n)
{
    LLMRS_CHECK_ARG(ctx && d_a && d_b && d_c && m > 0 && k > 0 && n > 0, "matmul: bad arguments");
    return op_matmul(ctx->stream, d_a, d_b, d_c, m, k, n);
}

int llmrs_matmul_slice(llmrs_ctx *ctx, const float *d_a, const float *d_other, float *d_c, int m, int rows, int cols)
{
    LLMRS_CHECK_ARG(ctx && d_a && d_other && d_c && m > 0 && rows > 0 && cols > 0, "matmul_slice: bad arguments");
    return op_matmul_t(ctx->stream, d_a, d_other, d_c, m, cols, rows);
}

int llmrs_add_assign(llmrs_ctx *ctx, float *d_a, const float *d_b, size_t n)
{
    LLMRS_CHECK_ARG(ctx && (n == 0 || (d_a && d_b)), "add_assign: bad arguments");
    return n ? op_add_assign(ctx->stream, d_a, d_b, n) : LLMRS_OK;
}

int llmrs_silu_mul(llmrs_ctx *ctx, float *d_gate, const float *d_up, size_t n)
{
    LLMRS_CHECK_ARG(ctx && (n == 0 || (d_gate && d_up)), "silu_mul: bad arguments");
    return n ? op_silu_mul(ctx->stream, d_gate, d_up, n) : LLMRS_OK;
}

int llmrs_rope_inplace(llmrs_ctx *ctx, float *d_x, int rows, int head_dim, int start_pos, float theta_base)
{
    LLMRS_CHECK_ARG(ctx && d_x && rows >= 0 && head_dim > 0 && start_pos >= 0, "rope_inplace: bad arguments");
    return rows ? op_rope(ctx->stream, d_x, rows, head_dim, start_pos, theta_base) : LLMRS_OK;
}

int llmrs_rms_norm(llmrs_ctx *ctx, const float *d_x, const float *d_w, float *d_y, int rows, int cols, float eps)
{
    LLMRS_CHECK_ARG(ctx && d_x && d_w && d_y && rows >= 0 && cols > 0, "rms_norm: bad arguments");
    return rows ? op_rms_norm(ctx->stream, d_x, d_w, d_y, rows, cols, eps) : LLMRS_OK;
}

int llmrs_softmax(llmrs_ctx *ctx, const float *d_x, float *d_y, int rows, int cols)
{
    LLMRS_CHECK_ARG(ctx && d_x && d_y && rows >= 0 && cols > 0, "softmax: bad arguments");
    return rows ? op_softmax(ctx->stream, d_x, d_y, rows, cols) : LLMRS_OK;
}

int llmrs_scale(llmrs_ctx *ctx, const float *d_x, float *d_y, size_t n, float value)
{
    LLMRS_CHECK_ARG(ctx && (n == 0 || (d_x && d_y)), "scale: bad arguments");
    return n ? op_scale(ctx->stream, d_x, d_y, n, value) : LLMRS_OK;
}

int llmrs_copy_from(llmrs_ctx *ctx, const float *d_src, float *d_dst, size_t n)
{
    LLMRS_CHECK_ARG(ctx && (n == 0 || (d_src && d_dst)), "copy_from: bad arguments");
    return n ? op_copy(ctx->stream, d_src, d_dst, n) : LLMRS_OK;
}

static int ctx_scratch(llmrs_ctx *ctx, size_t bytes, void **out)
{
    if (ctx->scratch_bytes < bytes) {
        LLMRS_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
        if (ctx->scratch)
            cudaFree(ctx->scratch);
        ctx->scratch = nullptr;
        ctx->scratch_bytes = 0;
        cudaError_t e = cudaMalloc(&ctx->scratch, bytes);
        if (e != cudaSuccess)
            return fail(LLMRS_ENOMEM, "scratch of %zu bytes: %s", bytes, cudaGetErrorString(e));
        ctx->scratch_bytes = bytes;
    }
    *out = ctx->scratch;
    return LLMRS_OK;
}

int llmrs_attention_decode(llmrs_ctx *ctx, const float *d_qkv, float *d_kcache, float *d_vcache,
                           const float *d_rope_cos, const float *d_rope_sin, float *d_out, int n_heads,
                           int n_kv_heads, int head_dim, int max_seq, int pos)
{
    LLMRS_CHECK_ARG(ctx && d_qkv && d_kcache && d_vcache && d_rope_cos && d_rope_sin && d_out, "NULL argument");
    LLMRS_CHECK_ARG(n_kv_heads > 0 && n_heads > 0 && n_heads % n_kv_heads == 0, "bad head counts %d/%d", n_heads,
                    n_kv_heads);
    LLMRS_CHECK_ARG(max_seq > 0 && pos >= 0 && pos < max_seq, "position %d outside [0,%d)", pos, max_seq);
    AttnParams a{};
    a.n_heads = n_heads;
    a.n_kv = n_kv_heads;
    a.head_dim = head_dim;
    a.max_seq = max_seq;
    a.n_splits = attention_default_splits(n_kv_heads);
    a.pos_fixed = pos;
    a.qkv = d_qkv;
    a.kc = d_kcache;
    a.vc = d_vcache;
    a.rope_cos = d_rope_cos;
    a.rope_sin = d_rope_sin;
    a.ctx = d_out;
    a.err = ctx->d_err;
    a.inv_sqrt_d = 1.0f / sqrtf((float)head_dim);
    const size_t part = attention_partials_floats(n_heads, head_dim, a.n_splits) * 4;
    void *scr = nullptr;
    LLMRS_TRY(ctx_scratch(ctx, part + (size_t)n_kv_heads * 4 + 256, &scr));
    a.part = reinterpret_cast<float *>(scr);
    a.counter = reinterpret_cast<unsigned int *>(reinterpret_cast<uint8_t *>(scr) + ((part + 255) & ~size_t(255)));
    LLMRS_CUDA_TRY(cudaMemsetAsync(a.counter, 0, (size_t)n_kv_heads * 4, ctx->stream));
    return attention_decode_launch(a, ctx->stream, false);
}

int llmrs_attention_prefill(llmrs_ctx *ctx, float *d_qkv, float *d_kcache, float *d_vcache, const float *d_rope_cos,
                            const float *d_rope_sin, float *d_out, int n_rows, int n_heads, int n_kv_heads,
                            int head_dim, int max_seq, int start_pos)
{
    LLMRS_CHECK_ARG(ctx && d_qkv && d_kcache && d_vcache && d_rope_cos && d_rope_sin && d_out, "NULL argument");
    LLMRS_CHECK_ARG(n_kv_heads > 0 && n_heads > 0 && n_heads % n_kv_heads == 0, "bad head counts %d/%d", n_heads,
                    n_kv_heads);
    LLMRS_CHECK_ARG(n_rows > 0 && start_pos >= 0 && max_seq > 0 && start_pos + n_rows <= max_seq,
                    "rows [%d, %d) outside [0,%d)", start_pos, start_pos + n_rows, max_seq);
    LLMRS_TRY(prefill_rope_append(d_qkv, d_kcache, d_vcache, d_rope_cos, d_rope_sin, n_rows, start_pos, n_heads,
                                  n_kv_heads, head_dim, max_seq, ctx->stream));
    return prefill_attention(d_qkv, d_kcache, d_vcache, d_out, n_rows, start_pos, n_heads, n_kv_heads, head_dim,
                             max_seq, 1.0f / sqrtf((float)head_dim), ctx->stream);
}

int llmrs_sample(llmrs_ctx *ctx, const float *d_logits, int vocab, const int *h_recent, int n_recent,
                 float repeat_penalty, float temperature, float top_p, float u, int *h_token)
{
    LLMRS_CHECK_ARG(ctx && d_logits && h_token && vocab > 0, "sample: bad arguments");
    void *scr = nullptr;
    LLMRS_TRY(ctx_scratch(ctx, sample_scratch_bytes(vocab), &scr));
    return sample_launch(d_logits, vocab, h_recent, n_recent, repeat_penalty, temperature, top_p, u, scr, h_token,
                         ctx->stream);
}

int llmrs_quantize_row_q8_0(llmrs_ctx *ctx, const float *d_x, int8_t *d_q, float *d_s, int rows, int k)
{
    LLMRS_CHECK_ARG(ctx && d_x && d_q && d_s && rows >= 0 && k > 0 && k % 32 == 0,
                    "quantize_row_q8_0: bad arguments (k=%d must be a multiple of 32)", k);
    return op_quantize_q8(ctx->stream, d_x, d_q, d_s, (size_t)rows * (k / 32));
}

int llmrs_rms_norm_quantize_q8_0(llmrs_ctx *ctx, const float *d_x, const float *d_w, int8_t *d_q, float *d_s, int k,
                                 float eps)
{
    LLMRS_CHECK_ARG(ctx, "NULL context");
    LLMRS_TRY(gemv_norm_quantize(d_x, d_w, k, eps, d_q, d_s, ctx->d_err, ctx->stream));
    return LLMRS_OK;
}

int llmrs_quantize_q4(llmrs_ctx *ctx, const float *d_w, size_t n, uint8_t *d_qs, float *d_scales)
{
    LLMRS_CHECK_ARG(ctx && (n == 0 || (d_w && d_qs && d_scales)), "quantize_q4: bad arguments");
    return op_quantize_q4(ctx->stream, d_w, n, d_qs, d_scales);
}

// ---------------------------------------------------------------- model
int llmrs_rope_table(int head_dim, int n_pos, float theta_base, float *h_cos, float *h_sin)
{
    LLMRS_CHECK_ARG(head_dim > 0 && head_dim % 2 == 0 && n_pos >= 0 && h_cos && h_sin, "rope_table: bad arguments");
    const int mid = head_dim / 2;
    for (int pos = 0; pos < n_pos; pos++)
        for (int j = 0; j < mid; j++) {
            // src/backend/cpu.rs:346-349, each operation rounded to f32
            volatile float freq_idx = ((float)j * 2.0f) / (float)head_dim;
            volatile float theta = 1.0f / powf(theta_base, freq_idx);
            volatile float m_theta = (float)pos * theta;
            h_sin[(size_t)pos * mid + j] = sinf(m_theta);
            h_cos[(size_t)pos * mid + j] = cosf(m_theta);
        }
    return LLMRS_OK;
}

static void model_free(llmrs_model *m)
{
    if (!m)
        return;
    if (m->graph)
        cudaGraphExecDestroy(m->graph);
    if (m->graph_traced)
        cudaGraphExecDestroy(m->graph_traced);
    if (m->arena.base)
        cudaFree(m->arena.base);
    if (m->tp_region)
        cudaFree(m->tp_region);
    if (m->pf_buf)
        cudaFree(m->pf_buf);
    if (m->pf_bf16)
        cudaFree(m->pf_bf16);
    if (m->h_stage)
        cudaFreeHost(m->h_stage);
    delete m;
}

int llmrs_model_create(llmrs_ctx *ctx, const llmrs_config *cfg, llmrs_model **out)
{
    LLMRS_CHECK_ARG(ctx && out, "NULL argument");
    *out = nullptr;
    LLMRS_TRY(check_cfg(cfg));
    LLMRS_CUDA_TRY(cudaSetDevice(ctx->device));
    llmrs_model *m = new llmrs_model();
    m->ctx = ctx;
    m->cfg = *cfg;
    m->wf = cfg->weight_format;
    m->st = cfg->scale_dtype;
    m->T = cfg->tp_size > 0 ? cfg->tp_size : 1;
    m->rank = cfg->tp_rank;
    m->cfg.tp_size = m->T;
    m->D = cfg->head_dim;
    m->Hq = cfg->n_heads / m->T;
    m->Hkv = cfg->n_kv_heads / m->T;
    m->H = cfg->hidden;
    m->F = cfg->ffn / m->T;
    m->V = cfg->vocab;
    m->Vl = cfg->vocab / m->T;
    m->S = cfg->max_seq;
    m->n_splits = attention_default_splits(m->Hkv);
    m->log_cap = 1 << 16;
    const int D = m->D, H = m->H, F = m->F, V = m->V, Vl = m->Vl, S = m->S;
    const size_t qkv_rows = (size_t)(m->Hq + 2 * m->Hkv) * D;
    const size_t qdim = (size_t)m->Hq * D;
    const int wf = m->wf;
    // arena size (scales always reserve 4 bytes so either dtype fits)
    auto qsize = [&](size_t n, size_t k) { return wbytes(wf, n, k) + n * k / 32 * 4 + 512; };
    size_t total = 0;
    for (int l = 0; l < cfg->n_layers; l++) {
        total += qsize(qkv_rows, H) + qsize(H, qdim) + qsize(2 * (size_t)F, H) + qsize(H, F);
        total += 2 * (size_t)H * 4 + 512;
        total += 2 * (size_t)m->Hkv * S * D * 4 + 512;
    }
    total += (size_t)V * H * 4 + 256;                                       // embed
    total += (size_t)H * 4 + 256;                                           // final norm
    total += (cfg->tied_embeddings ? (size_t)Vl * H / 2 : wbytes(wf, Vl, H)) + (size_t)Vl * H / 32 * 4 + 512;
    total += 2 * (size_t)S * D / 2 * 4 + 512;                              // rope
    total += ((size_t)2 * H + qkv_rows + qdim + F + Vl) * 4 + 6 * 256;       // activations
    total += sizeof(TpLink) + 256;
    total += attention_partials_floats(m->Hq, D, m->n_splits) * 4 + 256;
    total += (size_t)m->Hkv * 4 + sizeof(StepState) + (size_t)m->log_cap * 4 + 1024;
    total += (size_t)TRACE_MARKS * (5 * cfg->n_layers + 8) * 8 + 256; // timeline marks
    cudaError_t e = cudaMalloc(&m->arena.base, total);
    if (e != cudaSuccess) {
        model_free(m);
        return fail(LLMRS_ENOMEM, "model arena of %zu bytes: %s", total, cudaGetErrorString(e));
    }
    m->arena.size = total;
    Arena &A = m->arena;
    auto mkq = [&](QW &q, size_t n, size_t k, int st) {
        q.n = (int)n;
        q.k = (int)k;
        q.st = st;
        q.w = (uint8_t *)A.take(wbytes(wf, n, k));
        q.s = A.take(n * k / 32 * 4);
    };
    m->layers.resize(cfg->n_layers);
    for (auto &L : m->layers) {
        mkq(L.qkv, qkv_rows, H, m->st);
        mkq(L.o, H, qdim, m->st);
        mkq(L.gate_up, 2 * (size_t)F, H, m->st);
        mkq(L.down, H, F, m->st);
        L.attn_norm = (float *)A.take((size_t)H * 4);
        L.mlp_norm = (float *)A.take((size_t)H * 4);
        L.kc = (float *)A.take((size_t)m->Hkv * S * D * 4);
        L.vc = (float *)A.take((size_t)m->Hkv * S * D * 4);
    }
    m->embed = (float *)A.take((size_t)V * H * 4);
    m->final_norm = (float *)A.take((size_t)H * 4);
    if (cfg->tied_embeddings) {
        m->lm_head.n = Vl;
        m->lm_head.k = H;
        m->lm_head.st = LLMRS_F32;
        m->lm_head.w = (uint8_t *)A.take((size_t)Vl * H / 2);
        m->lm_head.s = A.take((size_t)Vl * H / 32 * 4);
    } else {
        mkq(m->lm_head, Vl, H, m->st);
    }
    m->rope_cos = (float *)A.take((size_t)S * D / 2 * 4);
    m->rope_sin = (float *)A.take((size_t)S * D / 2 * 4);
    m->x = (float *)A.take((size_t)H * 4);
    m->qkv = (float *)A.take(qkv_rows * 4);
    m->ctxv = (float *)A.take(qdim * 4);
    m->act = (float *)A.take((size_t)F * 4);
    m->logits = (float *)A.take((size_t)Vl * 4);
    m->x1 = (float *)A.take((size_t)H * 4);
    m->d_tp = (TpLink *)A.take(sizeof(TpLink));
    m->part = (float *)A.take(attention_partials_floats(m->Hq, D, m->n_splits) * 4);
    m->att_counter = (unsigned int *)A.take((size_t)m->Hkv * 4);
    m->state = (StepState *)A.take(sizeof(StepState));
    m->token_log = (int *)A.take((size_t)m->log_cap * 4);
    m->d_trace = (unsigned long long *)A.take((size_t)TRACE_MARKS * (5 * cfg->n_layers + 8) * 8);
    if (!m->token_log || !m->d_trace || !m->d_tp) {
        model_free(m);
        return fail(LLMRS_ENOMEM, "model arena layout overflow");
    }
    {
        const int sms = ctx->sms;
        int rc = LLMRS_OK;
        for (auto &L : m->layers) {
            if (rc == LLMRS_OK)
                rc = gemv_plan(&L.qkv.plan, L.qkv.w, L.qkv.s, L.qkv.n, L.qkv.k, wf, L.qkv.st, false, sms);
            if (rc == LLMRS_OK)
                rc = gemv_plan(&L.o.plan, L.o.w, L.o.s, L.o.n, L.o.k, wf, L.o.st, false, sms);
            if (rc == LLMRS_OK)
                rc = gemv_plan(&L.gate_up.plan, L.gate_up.w, L.gate_up.s, L.gate_up.n, L.gate_up.k, wf, L.gate_up.st,
                               true, sms);
            if (rc == LLMRS_OK)
                rc = gemv_plan(&L.down.plan, L.down.w, L.down.s, L.down.n, L.down.k, wf, L.down.st, false, sms);
        }
        if (rc == LLMRS_OK)
            rc = gemv_plan(&m->lm_head.plan, m->lm_head.w, m->lm_head.s, m->lm_head.n, m->lm_head.k,
                           cfg->tied_embeddings ? 0 : wf, m->lm_head.st, false, sms);
        if (rc != LLMRS_OK) {
            model_free(m);
            return rc;
        }
    }
    cudaStream_t s = ctx->stream;
    e = cudaMemsetAsync(m->arena.base, 0, total, s);
    // RoPE table from the host libm (bit-exact with the reference)
    std::vector<float> hc((size_t)S * D / 2), hs((size_t)S * D / 2);
    llmrs_rope_table(D, S, cfg->rope_theta, hc.data(), hs.data());
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->rope_cos, hc.data(), hc.size() * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->rope_sin, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaHostAlloc((void **)&m->h_stage, 64 * sizeof(int), cudaHostAllocDefault);
    if (e == cudaSuccess) {
        StepState st0{};
        st0.log_cap = m->log_cap;
        e = cudaMemcpyAsync(m->state, &st0, sizeof(st0), cudaMemcpyHostToDevice, s);
    }
    if (e == cudaSuccess && m->T > 1) {
        // communication region: partials [T][H] for o_proj and down_proj, keys [T], counters
        auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
        m->tp_off_o = 0;
        m->tp_off_d = up((size_t)m->T * H * 8);
        m->tp_off_keys = m->tp_off_d + up((size_t)m->T * H * 8);
        m->tp_off_cnt = m->tp_off_keys + up((size_t)m->T * 8);
        m->tp_bytes = m->tp_off_cnt + up((size_t)TP_CNT_N * 8);
        e = cudaMalloc(&m->tp_region, m->tp_bytes);
        if (e == cudaSuccess)
            e = cudaMemsetAsync(m->tp_region, 0, m->tp_bytes, s);
    }
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        model_free(m);
        return fail(LLMRS_ECUDA, "model set-up: %s", cudaGetErrorString(e));
    }
    m->kernels_per_step = 5 * cfg->n_layers + 1;
    *out = m;
    return LLMRS_OK;
}

int llmrs_model_destroy(llmrs_model *m)
{
    if (!m)
        return LLMRS_OK;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    model_free(m);
    return LLMRS_OK;
}

static int finish_sync(llmrs_model *m)
{
    LLMRS_CUDA_TRY(cudaStreamSynchronize(m->ctx->stream));
    return LLMRS_OK;
}

// weights changed: the prefill path's bf16 copies are rebuilt on next use
static void prefill_invalidate(llmrs_model *m)
{
    if (m->pf_bf16) {
        cudaStreamSynchronize(m->ctx->stream);
        cudaFree(m->pf_bf16);
    }
    m->pf_bf16 = nullptr;
    m->pf_bf = 0;
    m->pf_weights = -1;
}

int llmrs_model_init_synthetic(llmrs_model *m, uint64_t seed)
{
    LLMRS_CHECK_ARG(m, "model is NULL");
    prefill_invalidate(m);
    LLMRS_CHECK_ARG(m->st == LLMRS_F16 || m->st == LLMRS_F32, "bad scale dtype");
    cudaSetDevice(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    const int D = m->D, H = m->H, F = m->F, V = m->V, Vl = m->Vl, r = m->rank;
    const int qd = m->Hq * D, kd = m->Hkv * D; // this rank's rows
    const int QD = qd * m->T, FF = F * m->T;   // full o_proj / down_proj input widths
    for (int l = 0; l < m->cfg.n_layers; l++) {
        LayerW &L = m->layers[l];
        // fused QKV rows: q | k | v (native GQA); rank r: its heads' rows
        LLMRS_TRY(synth_quant(s, m->wf, seed, l, LLMRS_T_Q, H, r * qd, qd, 0, H, L.qkv.w, L.qkv.s, L.qkv.st, 1, 0));
        LLMRS_TRY(synth_quant(s, m->wf, seed, l, LLMRS_T_K, H, r * kd, kd, 0, H, L.qkv.w, L.qkv.s, L.qkv.st, 1, qd));
        LLMRS_TRY(synth_quant(s, m->wf, seed, l, LLMRS_T_V, H, r * kd, kd, 0, H, L.qkv.w, L.qkv.s, L.qkv.st, 1,
                              qd + kd));
        // o_proj: all rows, the input columns of this rank's heads
        LLMRS_TRY(synth_quant(s, m->wf, seed, l, LLMRS_T_O, QD, 0, H, r * qd, qd, L.o.w, L.o.s, L.o.st, 1, 0));
        // gate/up interleaved: device row 2i = gate i, 2i+1 = up i (this rank's FFN rows)
        LLMRS_TRY(synth_quant(s, m->wf, seed, l, LLMRS_T_GATE, H, r * F, F, 0, H, L.gate_up.w, L.gate_up.s,
                              L.gate_up.st, 2, 0));
        LLMRS_TRY(synth_quant(s, m->wf, seed, l, LLMRS_T_UP, H, r * F, F, 0, H, L.gate_up.w, L.gate_up.s,
                              L.gate_up.st, 2, 1));
        // down_proj: all rows, this rank's FFN columns
        LLMRS_TRY(synth_quant(s, m->wf, seed, l, LLMRS_T_DOWN, FF, 0, H, r * F, F, L.down.w, L.down.s, L.down.st, 1,
                              0));
        LLMRS_TRY(synth_normal(s, seed, l, LLMRS_T_ATTN_NORM, H, 1.0f, 0.02f, L.attn_norm));
        LLMRS_TRY(synth_normal(s, seed, l, LLMRS_T_MLP_NORM, H, 1.0f, 0.02f, L.mlp_norm));
    }
    LLMRS_TRY(synth_normal(s, seed, LLMRS_GLOBAL_LAYER, LLMRS_T_EMBED, (size_t)V * H, 1.0f, 0.02f, m->embed));
    LLMRS_TRY(synth_normal(s, seed, LLMRS_GLOBAL_LAYER, LLMRS_T_FINAL_NORM, H, 1.0f, 0.02f, m->final_norm));
    if (m->cfg.tied_embeddings)
        LLMRS_TRY(op_quantize_q4(s, m->embed + (size_t)r * Vl * H, (size_t)Vl * H, m->lm_head.w,
                                 (float *)m->lm_head.s));
    else
        LLMRS_TRY(synth_quant(s, m->wf, seed, LLMRS_GLOBAL_LAYER, LLMRS_T_LM_HEAD, H, r * Vl, Vl, 0, H, m->lm_head.w,
                              m->lm_head.s, m->lm_head.st, 1, 0));
    return finish_sync(m);
}

// Where a weight tensor of the reference layout goes in this rank's model:
// rows [row0, row0 + n) x columns [col0, col0 + k) of the caller's full
// [.][src_k] tensor land in rows add, add + mul, ... of the device tensor q
// (q | k | v fused rows, gate / up interleaved, tensor-parallel shards).
struct WeightSeg {
    QW *q;
    size_t n, k;
    int mul, add;
    size_t src_k, row0, col0;
};

static int weight_segs(llmrs_model *m, int layer, int which, WeightSeg *seg, int *nseg)
{
    const size_t T = (size_t)m->T, r = (size_t)m->rank, D = m->D, H = m->H, F = m->F, Vl = m->Vl;
    const size_t qd = (size_t)m->Hq * D, kd = (size_t)m->Hkv * D;
    *nseg = 1;
    if (which == LLMRS_W_LM_HEAD) {
        seg[0] = {&m->lm_head, Vl, H, 1, 0, H, r * Vl, 0};
        return LLMRS_OK;
    }
    LLMRS_CHECK_ARG(layer >= 0 && layer < m->cfg.n_layers, "layer %d out of range", layer);
    LayerW &L = m->layers[layer];
    switch (which) {
    case LLMRS_W_Q: seg[0] = {&L.qkv, qd, H, 1, 0, H, r * qd, 0}; break;
    case LLMRS_W_K: seg[0] = {&L.qkv, kd, H, 1, (int)qd, H, r * kd, 0}; break;
    case LLMRS_W_V: seg[0] = {&L.qkv, kd, H, 1, (int)(qd + kd), H, r * kd, 0}; break;
    case LLMRS_W_O: seg[0] = {&L.o, H, qd, 1, 0, qd * T, 0, r * qd}; break;
    case LLMRS_W_GATE_UP: // the reference's fused layout: gate rows [0, ffn), then up rows [ffn, 2 ffn)
        seg[0] = {&L.gate_up, F, H, 2, 0, H, r * F, 0};
        seg[1] = {&L.gate_up, F, H, 2, 1, H, F * T + r * F, 0};
        *nseg = 2;
        break;
    case LLMRS_W_GATE: seg[0] = {&L.gate_up, F, H, 2, 0, H, r * F, 0}; break;
    case LLMRS_W_UP: seg[0] = {&L.gate_up, F, H, 2, 1, H, r * F, 0}; break;
    case LLMRS_W_DOWN: seg[0] = {&L.down, H, F, 1, 0, F * T, 0, r * F}; break;
    default: return fail(LLMRS_EINVAL, "weight id %d is not a quantised linear", which);
    }
    return LLMRS_OK;
}

// f32 block scales [n][k/32] on the device into q's rows (add, add + mul, ...):
// as they are, or as f16 when q stores f16 (every scale must then be exact)
static int place_scales(llmrs_model *m, const WeightSeg &g, const float *d_s)
{
    cudaStream_t s = m->ctx->stream;
    const size_t nb = g.k / 32;
    if (g.q->st == LLMRS_F32) {
        LLMRS_CUDA_TRY(cudaMemcpy2DAsync((uint8_t *)g.q->s + (size_t)g.add * nb * 4, nb * 4 * g.mul, d_s, nb * 4,
                                         nb * 4, g.n, cudaMemcpyDeviceToDevice, s));
        return LLMRS_OK;
    }
    uint32_t *flag = m->ctx->d_err; // reuse the op error word as the inexact flag
    LLMRS_CUDA_TRY(cudaMemsetAsync(flag, 0, 4, s));
    __half *h16 = nullptr;
    LLMRS_CUDA_TRY(cudaMallocAsync((void **)&h16, g.n * nb * 2 + 16, s));
    LLMRS_TRY(scales_to_f16(s, d_s, h16, g.n * nb, flag));
    LLMRS_CUDA_TRY(cudaMemcpy2DAsync((uint8_t *)g.q->s + (size_t)g.add * nb * 2, nb * 2 * g.mul, h16, nb * 2, nb * 2,
                                     g.n, cudaMemcpyDeviceToDevice, s));
    LLMRS_CUDA_TRY(cudaFreeAsync(h16, s));
    uint32_t inexact = 0;
    LLMRS_CUDA_TRY(cudaMemcpyAsync(&inexact, flag, 4, cudaMemcpyDeviceToHost, s));
    LLMRS_CUDA_TRY(cudaStreamSynchronize(s));
    LLMRS_CUDA_TRY(cudaMemsetAsync(flag, 0, 4, s));
    if (inexact)
        return fail(LLMRS_EINVAL, "a block scale is not exactly representable in f16; create the model with "
                                  "scale_dtype = LLMRS_F32");
    return LLMRS_OK;
}

// quantised host tensor (reference layout, f32 scales) -> one segment
static int upload_quant(llmrs_model *m, const WeightSeg &g, int wf, const void *h_codes, const float *h_scales)
{
    cudaStream_t s = m->ctx->stream;
    const size_t rb = wbytes(wf, 1, g.k), src_rb = wbytes(wf, 1, g.src_k);
    const size_t nb = g.k / 32, src_nb = g.src_k / 32;
    const uint8_t *c = (const uint8_t *)h_codes + g.row0 * src_rb + wbytes(wf, 1, g.col0);
    const float *sc = h_scales + g.row0 * src_nb + g.col0 / 32;
    LLMRS_CUDA_TRY(cudaMemcpy2DAsync(g.q->w + (size_t)g.add * rb, rb * g.mul, c, src_rb, rb, g.n,
                                     cudaMemcpyHostToDevice, s));
    float *tmp = nullptr;
    LLMRS_CUDA_TRY(cudaMallocAsync((void **)&tmp, g.n * nb * 4 + 16, s));
    LLMRS_CUDA_TRY(cudaMemcpy2DAsync(tmp, nb * 4, sc, src_nb * 4, nb * 4, g.n, cudaMemcpyHostToDevice, s));
    const int rc = place_scales(m, g, tmp);
    cudaFreeAsync(tmp, s);
    return rc;
}

// rows of a raw f32 / bf16 host tensor, the slice [row0, +n) x [col0, +k) of
// [.][src_k], as f32 on the device (the caller frees *out with cudaFreeAsync)
static int stage_raw(llmrs_model *m, const void *h, int dtype, size_t src_k, size_t row0, size_t col0, size_t n,
                     size_t k, float **out)
{
    cudaStream_t s = m->ctx->stream;
    const size_t es = dtype == LLMRS_BF16 ? 2 : 4;
    void *raw = nullptr;
    LLMRS_CUDA_TRY(cudaMallocAsync(&raw, n * k * es + 16, s));
    LLMRS_CUDA_TRY(cudaMemcpy2DAsync(raw, k * es, (const uint8_t *)h + (row0 * src_k + col0) * es, src_k * es, k * es,
                                     n, cudaMemcpyHostToDevice, s));
    if (dtype == LLMRS_F32) {
        *out = (float *)raw;
        return LLMRS_OK;
    }
    float *f = nullptr;
    LLMRS_CUDA_TRY(cudaMallocAsync((void **)&f, n * k * 4 + 16, s));
    LLMRS_TRY(op_bf16_to_f32(s, (const uint16_t *)raw, f, n * k));
    LLMRS_CUDA_TRY(cudaFreeAsync(raw, s));
    *out = f;
    return LLMRS_OK;
}

// raw f32 / bf16 host weights -> quantised (quantize_q4, src/core/tensor.rs:102-167,
// or the Q8_0 block quantiser for Q8_0 models) into one segment
static int load_quant(llmrs_model *m, const WeightSeg &g, int wf, const void *h, int dtype)
{
    cudaStream_t s = m->ctx->stream;
    float *f = nullptr;
    LLMRS_TRY(stage_raw(m, h, dtype, g.src_k, g.row0, g.col0, g.n, g.k, &f));
    const size_t rb = wbytes(wf, 1, g.k), nb = g.k / 32;
    uint8_t *codes = nullptr;
    float *sc = nullptr;
    LLMRS_CUDA_TRY(cudaMallocAsync((void **)&codes, g.n * rb + 16, s));
    LLMRS_CUDA_TRY(cudaMallocAsync((void **)&sc, g.n * nb * 4 + 16, s));
    // blocks of 32 never straddle a row (k % 32 == 0), so quantising the slice
    // gives the slice of the full tensor's quantisation
    int rc = wf == 0 ? op_quantize_q4(s, f, g.n * g.k, codes, sc)
                     : op_quantize_q8(s, f, reinterpret_cast<int8_t *>(codes), sc, g.n * nb);
    if (rc == LLMRS_OK) {
        cudaError_t e = cudaMemcpy2DAsync(g.q->w + (size_t)g.add * rb, rb * g.mul, codes, rb, rb, g.n,
                                          cudaMemcpyDeviceToDevice, s);
        rc = e == cudaSuccess ? place_scales(m, g, sc) : fail(LLMRS_ECUDA, "weight copy: %s", cudaGetErrorString(e));
    }
    cudaFreeAsync(f, s);
    cudaFreeAsync(codes, s);
    cudaFreeAsync(sc, s);
    return rc;
}

// f32 / bf16 host vector or matrix -> an f32 device tensor (norms, embedding);
// the tied LM head is then re-derived from this rank's embedding rows
static int load_f32(llmrs_model *m, int layer, int which, const void *h, int dtype)
{
    cudaStream_t s = m->ctx->stream;
    const size_t H = m->H, V = m->V, Vl = m->Vl, r = m->rank;
    float *dst = nullptr;
    size_t n = H;
    switch (which) {
    case LLMRS_W_ATTN_NORM: dst = m->layers[layer].attn_norm; break;
    case LLMRS_W_MLP_NORM: dst = m->layers[layer].mlp_norm; break;
    case LLMRS_W_FINAL_NORM: dst = m->final_norm; break;
    case LLMRS_W_EMBED: dst = m->embed; n = V * H; break;
    default: return fail(LLMRS_EINVAL, "weight id %d is not an f32 tensor", which);
    }
    if (dtype == LLMRS_F32 && h) {
        LLMRS_CUDA_TRY(cudaMemcpyAsync(dst, h, n * 4, cudaMemcpyHostToDevice, s));
    } else {
        float *f = nullptr;
        LLMRS_TRY(stage_raw(m, h, dtype, n, 0, 0, 1, n, &f));
        LLMRS_CUDA_TRY(cudaMemcpyAsync(dst, f, n * 4, cudaMemcpyDeviceToDevice, s));
        LLMRS_CUDA_TRY(cudaFreeAsync(f, s));
    }
    if (which == LLMRS_W_EMBED && m->cfg.tied_embeddings) // src/core/loader.rs:186-190
        LLMRS_TRY(op_quantize_q4(s, m->embed + r * Vl * H, Vl * H, m->lm_head.w, (float *)m->lm_head.s));
    return LLMRS_OK;
}

static bool is_f32_weight(int which)
{
    return which == LLMRS_W_ATTN_NORM || which == LLMRS_W_MLP_NORM || which == LLMRS_W_EMBED ||
           which == LLMRS_W_FINAL_NORM;
}

int llmrs_model_set_weight(llmrs_model *m, int layer, int which, const void *h_codes, const float *h_scales)
{
    if (m)
        prefill_invalidate(m);
    LLMRS_CHECK_ARG(m && h_codes, "NULL argument");
    cudaSetDevice(m->ctx->device);
    const bool global = which == LLMRS_W_EMBED || which == LLMRS_W_FINAL_NORM || which == LLMRS_W_LM_HEAD;
    LLMRS_CHECK_ARG(global || (layer >= 0 && layer < m->cfg.n_layers), "layer %d out of range", layer);
    if (is_f32_weight(which)) {
        LLMRS_TRY(load_f32(m, layer, which, h_codes, LLMRS_F32));
        return finish_sync(m);
    }
    LLMRS_CHECK_ARG(h_scales, "quantised tensor needs scales");
    if (which == LLMRS_W_LM_HEAD && m->cfg.tied_embeddings)
        return LLMRS_OK; // derived from the embedding
    WeightSeg seg[2];
    int nseg = 0;
    LLMRS_TRY(weight_segs(m, layer, which, seg, &nseg));
    for (int i = 0; i < nseg; i++)
        LLMRS_TRY(upload_quant(m, seg[i], m->wf, h_codes, h_scales));
    return finish_sync(m);
}

int llmrs_model_load_weight(llmrs_model *m, int layer, int which, const void *h_data, int dtype)
{
    if (m)
        prefill_invalidate(m);
    LLMRS_CHECK_ARG(m && h_data, "NULL argument");
    LLMRS_CHECK_ARG(dtype == LLMRS_F32 || dtype == LLMRS_BF16, "dtype %d is neither LLMRS_F32 nor LLMRS_BF16", dtype);
    cudaSetDevice(m->ctx->device);
    const bool global = which == LLMRS_W_EMBED || which == LLMRS_W_FINAL_NORM || which == LLMRS_W_LM_HEAD;
    LLMRS_CHECK_ARG(global || (layer >= 0 && layer < m->cfg.n_layers), "layer %d out of range", layer);
    if (is_f32_weight(which)) {
        LLMRS_TRY(load_f32(m, layer, which, h_data, dtype));
        return finish_sync(m);
    }
    if (which == LLMRS_W_LM_HEAD && m->cfg.tied_embeddings)
        return LLMRS_OK; // derived from the embedding
    WeightSeg seg[2];
    int nseg = 0;
    LLMRS_TRY(weight_segs(m, layer, which, seg, &nseg));
    for (int i = 0; i < nseg; i++)
        LLMRS_TRY(load_quant(m, seg[i], m->wf, h_data, dtype));
    return finish_sync(m);
}

int llmrs_kv_fill(llmrs_model *m, int layer, const float *h_k, const float *h_v, int n_pos)
{
    LLMRS_CHECK_ARG(m && h_k && h_v, "NULL argument");
    LLMRS_CHECK_ARG(layer >= 0 && layer < m->cfg.n_layers, "layer %d out of range", layer);
    LLMRS_CHECK_ARG(n_pos >= 0 && n_pos <= m->S, "n_pos %d exceeds max_seq %d", n_pos, m->S);
    if (n_pos == 0)
        return LLMRS_OK;
    cudaSetDevice(m->ctx->device);
    const size_t row = (size_t)n_pos * m->D * 4, pitch = (size_t)m->S * m->D * 4;
    cudaStream_t s = m->ctx->stream;
    LLMRS_CUDA_TRY(cudaMemcpy2DAsync(m->layers[layer].kc, pitch, h_k, row, row, m->Hkv, cudaMemcpyHostToDevice, s));
    LLMRS_CUDA_TRY(cudaMemcpy2DAsync(m->layers[layer].vc, pitch, h_v, row, row, m->Hkv, cudaMemcpyHostToDevice, s));
    return finish_sync(m);
}

int llmrs_kv_read(llmrs_model *m, int layer, float *h_k, float *h_v, int n_pos)
{
    LLMRS_CHECK_ARG(m && h_k && h_v, "NULL argument");
    LLMRS_CHECK_ARG(layer >= 0 && layer < m->cfg.n_layers, "layer %d out of range", layer);
    LLMRS_CHECK_ARG(n_pos >= 0 && n_pos <= m->S, "n_pos %d exceeds max_seq %d", n_pos, m->S);
    if (n_pos == 0)
        return LLMRS_OK;
    cudaSetDevice(m->ctx->device);
    const size_t row = (size_t)n_pos * m->D * 4, pitch = (size_t)m->S * m->D * 4;
    cudaStream_t s = m->ctx->stream;
    LLMRS_CUDA_TRY(cudaMemcpy2DAsync(h_k, row, m->layers[layer].kc, pitch, row, m->Hkv, cudaMemcpyDeviceToHost, s));
    LLMRS_CUDA_TRY(cudaMemcpy2DAsync(h_v, row, m->layers[layer].vc, pitch, row, m->Hkv, cudaMemcpyDeviceToHost, s));
    return finish_sync(m);
}

int llmrs_kv_fill_synthetic(llmrs_model *m, uint64_t seed, int n_pos)
{
    LLMRS_CHECK_ARG(m, "model is NULL");
    LLMRS_CHECK_ARG(n_pos >= 0 && n_pos <= m->S, "n_pos %d exceeds max_seq %d", n_pos, m->S);
    if (n_pos == 0)
        return LLMRS_OK;
    cudaSetDevice(m->ctx->device);
    for (int l = 0; l < m->cfg.n_layers; l++)
        LLMRS_TRY(synth_kv(m->ctx->stream, seed, l, m->rank * m->Hkv, m->Hkv, n_pos, m->S, m->D, m->layers[l].kc,
                           m->layers[l].vc));
    return finish_sync(m);
}

// One decode step (src/core/model.rs:17-49 for a 1-token chunk).  The first
// kernel launches without programmatic overlap, so the step's position and
// token are settled before any kernel of the step runs; every later kernel
// overlaps its weight prefetch with its predecessor.
struct KernelTimer {
    std::vector<cudaEvent_t> ev;
    std::vector<int> kind;
    int cap = 0;
    int mark(cudaStream_t s, int k)
    {
        if ((int)kind.size() >= cap)
            return LLMRS_OK;
        cudaEvent_t e;
        LLMRS_CUDA_TRY(cudaEventCreate(&e));
        LLMRS_CUDA_TRY(cudaEventRecord(e, s));
        ev.push_back(e);
        kind.push_back(k);
        return LLMRS_OK;
    }
};

// One op of a decode step: a GEMV over a weight matrix (with its prologue /
// epilogue variant) or decode attention.
enum HostOpKind : int { OP_GEMV = 0, OP_ATTN = 1 };
struct HostOp {
    int kind = OP_GEMV;
    int trace_kind = 0; // KERNEL kind of profile_decode / trace_decode
    const QW *q = nullptr;
    GemvParams g{};
    int pro = PRO_F32, epi = EPI_STORE;
    AttnParams a{};
};

// The decode step (src/core/model.rs:17-49 for a 1-token chunk) as an op list.
static void build_ops(llmrs_model *m, std::vector<HostOp> &ops, unsigned long long *trace)
{
    ops.clear();
    int slot = 0;
    const int H = m->H, F = m->F;
    const int qkv_rows = (m->Hq + 2 * m->Hkv) * m->D;
    uint32_t *err = &m->state->err;
    // Tensor parallel: o_proj and down_proj write partial sums to every rank
    // (EPI_PARTIAL); the next GEMV's prologue waits for all of them and forms
    // x = sum + x (PRO_AR_NORM).  The residual stream alternates between x
    // (after down_proj) and x1 (after o_proj) so no CTA overwrites the value
    // another CTA still reads.
    const bool tp = m->T > 1;
    const int L_n = m->cfg.n_layers;
    auto ar_in = [&](GemvParams &g, int kind, int index, const QW &producer, const float *x_in, float *x_out) {
        g.tp = m->d_tp;
        g.state = m->state;
        g.ar_kind = kind;
        g.ar_index = index;
        g.ar_per_step = L_n;
        g.x = x_in;
        g.x_out = x_out;
    };
    auto push_gemv = [&](int tkind, const QW &q, const GemvParams &g, int pro, int epi) {
        HostOp o;
        o.kind = OP_GEMV;
        o.trace_kind = tkind;
        o.q = &q;
        o.g = g;
        o.g.trace = trace;
        o.g.trace_slot = slot++;
        o.g.peer_ns = m->peer_ns;
        o.pro = pro;
        o.epi = epi;
        ops.push_back(o);
    };
    for (int l = 0; l < L_n; l++) {
        LayerW &L = m->layers[l];
        // (1) input RMSNorm + Q8_0 + fused QKV projection (layer 0: embedding gather, src/main.rs:159-171)
        GemvParams p{};
        p.err = err;
        p.eps = m->cfg.rms_eps;
        p.w = L.qkv.w;
        p.scales = L.qkv.s;
        p.N = qkv_rows;
        p.K = H;
        p.x = m->x;
        p.norm_w = L.attn_norm;
        p.y = m->qkv;
        p.state = m->state;
        int pro = PRO_NORM;
        if (l == 0) {
            pro = PRO_EMBED_NORM;
            p.embed = m->embed;
            p.vocab = m->V;
            p.x_out = m->x;
        } else if (tp) {
            pro = PRO_AR_NORM;
            ar_in(p, TP_CNT_DOWN, l - 1, m->layers[l - 1].down, m->x1, m->x);
        }
        push_gemv(0, L.qkv, p, pro, EPI_STORE);
        // (2) RoPE + KV append + attention (src/core/layer.rs:175-333)
        HostOp at;
        at.kind = OP_ATTN;
        at.trace_kind = 1;
        AttnParams &a = at.a;
        a.qkv = m->qkv;
        a.kc = L.kc;
        a.vc = L.vc;
        a.rope_cos = m->rope_cos;
        a.rope_sin = m->rope_sin;
        a.ctx = m->ctxv;
        a.part = m->part;
        a.counter = m->att_counter;
        a.state = m->state;
        a.err = err;
        a.n_heads = m->Hq;
        a.n_kv = m->Hkv;
        a.head_dim = m->D;
        a.max_seq = m->S;
        a.n_splits = m->n_splits;
        a.inv_sqrt_d = 1.0f / sqrtf((float)m->D);
        a.trace = trace;
        a.trace_slot = slot++;
        ops.push_back(at);
        // (3) o_proj + residual (src/core/layer.rs:332, 386)
        GemvParams o{};
        o.err = err;
        o.w = L.o.w;
        o.scales = L.o.s;
        o.N = H;
        o.K = m->Hq * m->D;
        o.x = m->ctxv;
        o.y = m->x;
        o.residual = m->x;
        if (tp) { // producer of exchange (o, l): its tag comes from the step's epoch
            o.tp = m->d_tp;
            o.state = m->state;
            o.ar_kind = TP_CNT_O;
            o.ar_index = l;
            o.ar_per_step = L_n;
        }
        push_gemv(2, L.o, o, PRO_F32, tp ? EPI_PARTIAL : EPI_RESIDUAL);
        // (4) post RMSNorm + gate_up + SiLU*up (src/core/layer.rs:37-89)
        GemvParams g{};
        g.err = err;
        g.eps = m->cfg.rms_eps;
        g.w = L.gate_up.w;
        g.scales = L.gate_up.s;
        g.N = 2 * F;
        g.K = H;
        g.x = m->x;
        g.norm_w = L.mlp_norm;
        g.y = m->act;
        if (tp)
            ar_in(g, TP_CNT_O, l, L.o, m->x, m->x1);
        push_gemv(3, L.gate_up, g, tp ? PRO_AR_NORM : PRO_NORM, EPI_SILU);
        // (5) down + residual (src/core/layer.rs:96, 403)
        GemvParams d{};
        d.err = err;
        d.w = L.down.w;
        d.scales = L.down.s;
        d.N = H;
        d.K = F;
        d.x = m->act;
        d.y = m->x;
        d.residual = m->x;
        if (tp) {
            d.tp = m->d_tp;
            d.state = m->state;
            d.ar_kind = TP_CNT_DOWN;
            d.ar_index = l;
            d.ar_per_step = L_n;
        }
        push_gemv(4, L.down, d, PRO_F32, tp ? EPI_PARTIAL : EPI_RESIDUAL);
    }
    // final RMSNorm + LM head + greedy argmax (src/core/model.rs:39-47, src/main.rs:185-190)
    GemvParams h{};
    h.err = err;
    h.eps = m->cfg.rms_eps;
    h.w = m->lm_head.w;
    h.scales = m->lm_head.s;
    h.N = m->Vl;
    h.K = H;
    h.x = m->x;
    h.norm_w = m->final_norm;
    h.y = m->logits;
    h.state = m->state;
    h.token_log = m->token_log;
    int hpro = PRO_NORM;
    if (tp) {
        hpro = PRO_AR_NORM;
        ar_in(h, TP_CNT_DOWN, L_n - 1, m->layers[L_n - 1].down, m->x1, m->x);
        h.row_offset = m->rank * m->Vl;
    }
    push_gemv(5, m->lm_head, h, hpro, EPI_ARGMAX);
}

// one kernel per op; every kernel but the step's first starts under
// programmatic dependent launch
static int enqueue_step(llmrs_model *m, cudaStream_t s, KernelTimer *kt = nullptr, unsigned long long *trace = nullptr)
{
    // with a timer every kernel is bracketed by events and launched without
    // programmatic overlap, so each event pair times exactly one kernel
    const bool overlap = kt == nullptr;
    std::vector<HostOp> ops;
    build_ops(m, ops, trace);
    for (size_t i = 0; i < ops.size(); i++) {
        const HostOp &o = ops[i];
        if (kt)
            LLMRS_TRY(kt->mark(s, o.trace_kind));
        if (o.kind == OP_GEMV)
            LLMRS_TRY(gemv_launch(o.q->plan, o.g, o.pro, o.epi, s, overlap && i != 0));
        else
            LLMRS_TRY(attention_decode_launch(o.a, s, overlap));
        if (kt)
            LLMRS_TRY(kt->mark(s, -1));
    }
    return LLMRS_OK;
}

static int capture_step(llmrs_model *m, cudaGraphExec_t *out, unsigned long long *trace)
{
    cudaStream_t s = m->ctx->stream;
    cudaGraph_t g = nullptr;
    LLMRS_CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(m, s, nullptr, trace);
    cudaError_t e = cudaStreamEndCapture(s, &g);
    if (rc != LLMRS_OK) {
        if (g)
            cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess)
        return fail(LLMRS_ECUDA, "graph capture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
        *out = nullptr;
        return fail(LLMRS_ECUDA, "graph instantiate: %s", cudaGetErrorString(e));
    }
    return LLMRS_OK;
}

static int ensure_graph(llmrs_model *m)
{
    if (m->T > 1 && !m->tp_connected)
        return fail(LLMRS_EINVAL, "tensor-parallel model (rank %d of %d) is not connected to its peers", m->rank,
                    m->T);
    if (m->graph)
        return LLMRS_OK;
    return capture_step(m, &m->graph, nullptr);
}

static int check_state_err(llmrs_model *m, uint32_t e)
{
    if (!e)
        return LLMRS_OK;
    cudaMemsetAsync(&m->state->err, 0, 4, m->ctx->stream);
    cudaStreamSynchronize(m->ctx->stream);
    if (e == DEV_ERR_MBAR_TIMEOUT || e == DEV_ERR_PEER_TIMEOUT)
        return fail(LLMRS_ETIMEDOUT, "decode step: device wait timed out (code %u)", e);
    return fail(LLMRS_EDEVICE, "decode step: device error word %u (%s)", e,
                e == DEV_ERR_BAD_TOKEN ? "token id out of range" : (e == DEV_ERR_BAD_POS ? "position out of range" : "?"));
}

// stage token/pos into the step state (8 bytes H2D from pinned memory)
static int set_token_pos(llmrs_model *m, int token, int pos, int slot)
{
    int *hs = m->h_stage + 4 * slot;
    hs[0] = token;
    hs[1] = pos;
    LLMRS_CUDA_TRY(cudaMemcpyAsync(m->state, hs, 2 * sizeof(int), cudaMemcpyHostToDevice, m->ctx->stream));
    return LLMRS_OK;
}

int llmrs_decode_step(llmrs_model *m, int token, int pos, float *h_logits, int *h_argmax)
{
    LLMRS_CHECK_ARG(m, "model is NULL");
    LLMRS_CHECK_ARG(token >= 0 && token < m->V, "token %d out of range [0,%d)", token, m->V);
    LLMRS_CHECK_ARG(pos >= 0 && pos < m->S, "position %d out of range [0,%d)", pos, m->S);
    cudaSetDevice(m->ctx->device);
    LLMRS_TRY(ensure_graph(m));
    cudaStream_t s = m->ctx->stream;
    LLMRS_TRY(set_token_pos(m, token, pos, 0));
    LLMRS_CUDA_TRY(cudaGraphLaunch(m->graph, s));
    int *out = m->h_stage + 60;
    LLMRS_CUDA_TRY(cudaMemcpyAsync(out, &m->state->token, sizeof(int), cudaMemcpyDeviceToHost, s));
    LLMRS_CUDA_TRY(cudaMemcpyAsync(out + 1, &m->state->err, sizeof(int), cudaMemcpyDeviceToHost, s));
    if (h_logits)
        LLMRS_CUDA_TRY(cudaMemcpyAsync(h_logits, m->logits, (size_t)m->Vl * 4, cudaMemcpyDeviceToHost, s));
    LLMRS_CUDA_TRY(cudaStreamSynchronize(s));
    LLMRS_TRY(check_state_err(m, (uint32_t)out[1]));
    if (h_argmax)
        *h_argmax = out[0];
    return LLMRS_OK;
}

int llmrs_generate(llmrs_model *m, int token, int pos, int n_steps, int *h_tokens_out)
{
    LLMRS_CHECK_ARG(m && h_tokens_out, "NULL argument");
    LLMRS_CHECK_ARG(n_steps >= 0 && n_steps <= m->log_cap, "n_steps %d out of range", n_steps);
    LLMRS_CHECK_ARG(token >= 0 && token < m->V, "token %d out of range", token);
    LLMRS_CHECK_ARG(pos >= 0 && pos + n_steps <= m->S, "positions [%d,%d) exceed max_seq %d", pos, pos + n_steps, m->S);
    if (n_steps == 0)
        return LLMRS_OK;
    cudaSetDevice(m->ctx->device);
    LLMRS_TRY(ensure_graph(m));
    cudaStream_t s = m->ctx->stream;
    LLMRS_TRY(set_token_pos(m, token, pos, 0));
    LLMRS_CUDA_TRY(cudaMemsetAsync(&m->state->n_log, 0, sizeof(int), s));
    for (int i = 0; i < n_steps; i++)
        LLMRS_CUDA_TRY(cudaGraphLaunch(m->graph, s));
    int *out = m->h_stage + 60;
    LLMRS_CUDA_TRY(cudaMemcpyAsync(out + 1, &m->state->err, sizeof(int), cudaMemcpyDeviceToHost, s));
    LLMRS_CUDA_TRY(cudaMemcpyAsync(h_tokens_out, m->token_log, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, s));
    LLMRS_CUDA_TRY(cudaStreamSynchronize(s));
    return check_state_err(m, (uint32_t)out[1]);
}

// ------------------------------------------------------------ prefill (M>1)
constexpr int PF_CHUNK = 512; // rows per tensor-core prefill chunk

// tensor maps of every linear for the M>1 path; false if one is off it
static int prefill_weights_ready(llmrs_model *m, bool *ready)
{
    if (m->pf_weights < 0) {
        int ok = m->T == 1 ? 1 : 0;
        for (int l = 0; ok && l < m->cfg.n_layers; l++) {
            LayerW &L = m->layers[l];
            const QW *q[4] = {&L.qkv, &L.o, &L.gate_up, &L.down};
            PrefillWeights *pw[4] = {&L.p_qkv, &L.p_o, &L.p_gate_up, &L.p_down};
            for (int i = 0; i < 4 && ok; i++) {
                LLMRS_TRY(prefill_weights_init(pw[i], q[i]->w, q[i]->s, q[i]->n, q[i]->k, m->wf, q[i]->st));
                ok = pw[i]->ok;
            }
        }
        if (ok && prefill_use_bf16()) { // one buffer holds every linear's bf16 copy
            size_t total = 0;
            for (int l = 0; l < m->cfg.n_layers; l++) {
                LayerW &L = m->layers[l];
                const QW *q[4] = {&L.qkv, &L.o, &L.gate_up, &L.down};
                for (int i = 0; i < 4; i++)
                    total += prefill_bf16_bytes(q[i]->n, q[i]->k);
            }
            // The copy is an optimisation: when it does not fit (or exceeds
            // LLMRS_PREFILL_BF16_MAX_MB), the int8 tensor-core GEMM reads the
            // Q8_0 / Q4_0 storage directly, with the same exact results.
            const char *cap_env = getenv("LLMRS_PREFILL_BF16_MAX_MB");
            const size_t cap = cap_env ? (size_t)atol(cap_env) << 20 : ~(size_t)0;
            cudaError_t e = total <= cap ? cudaMalloc(&m->pf_bf16, total) : cudaErrorMemoryAllocation;
            if (e != cudaSuccess) {
                cudaGetLastError(); // clear the failed allocation's error state
                m->pf_bf16 = nullptr;
                m->pf_bf = 0;
                m->pf_weights = ok;
                *ready = m->pf_weights == 1;
                return LLMRS_OK;
            }
            uint8_t *b = reinterpret_cast<uint8_t *>(m->pf_bf16);
            for (int l = 0; l < m->cfg.n_layers; l++) {
                LayerW &L = m->layers[l];
                const QW *q[4] = {&L.qkv, &L.o, &L.gate_up, &L.down};
                PrefillWeights *pw[4] = {&L.p_qkv, &L.p_o, &L.p_gate_up, &L.p_down};
                for (int i = 0; i < 4; i++) {
                    LLMRS_TRY(prefill_weights_to_bf16(pw[i], q[i]->w, q[i]->s, b, m->ctx->stream));
                    b += prefill_bf16_bytes(q[i]->n, q[i]->k);
                }
            }
            m->pf_bf = 1;
        }
        m->pf_weights = ok;
    }
    *ready = m->pf_weights == 1;
    return LLMRS_OK;
}

static int prefill_buffers(llmrs_model *m, int rows)
{
    if (m->pf_rows >= rows)
        return LLMRS_OK;
    if (m->pf_buf)
        cudaFree(m->pf_buf);
    m->pf_buf = nullptr;
    m->pf_rows = 0;
    const int H = m->H, QD = m->Hq * m->D, NQKV = (m->Hq + 2 * m->Hkv) * m->D, F = m->F;
    const int kmax = std::max(std::max(H, QD), F);
    auto up = [](size_t b) { return (b + 1023) & ~size_t(1023); };
    const size_t bx = up((size_t)rows * H * 4), bq = up((size_t)rows * NQKV * 4), bc = up((size_t)rows * QD * 4),
                 ba = up((size_t)rows * F * 4), bi = up((size_t)m->S * 4), bacts = up(prefill_acts_bytes(rows, kmax));
    uint8_t *b = nullptr;
    cudaError_t e = cudaMalloc(&b, bx + bq + bc + ba + bi + bacts);
    if (e != cudaSuccess)
        return fail(LLMRS_ENOMEM, "prefill buffers for %d rows: %s", rows, cudaGetErrorString(e));
    m->pf_buf = b;
    m->pf_x = reinterpret_cast<float *>(b);
    m->pf_qkv = reinterpret_cast<float *>(b + bx);
    m->pf_ctx = reinterpret_cast<float *>(b + bx + bq);
    m->pf_act = reinterpret_cast<float *>(b + bx + bq + bc);
    m->pf_ids = reinterpret_cast<int *>(b + bx + bq + bc + ba);
    m->pf_acts = b + bx + bq + bc + ba + bi;
    m->pf_rows = rows;
    return LLMRS_OK;
}

// Rows start .. start+n-1 through every layer as M = n contractions
// (src/core/model.rs:17-49 with src/core/layer.rs:160-406 for seq = n): per
// row RMSNorm + Q8_0, tensor-core QKV, RoPE + KV append, causal attention,
// o_proj + residual, RMSNorm + gate_up + SiLU*up, down + residual.  Leaves the
// residual stream of every row in pf_x.
static int prefill_chunk(llmrs_model *m, const int *d_ids, int n, int start)
{
    cudaStream_t s = m->ctx->stream;
    uint32_t *err = &m->state->err;
    const int H = m->H, D = m->D, Hq = m->Hq, Hkv = m->Hkv, F = m->F, QD = Hq * D, NQKV = (Hq + 2 * Hkv) * D;
    const int sms = m->ctx->sms;
    LLMRS_TRY(prefill_embed(m->embed, d_ids, m->pf_x, n, H, m->V, err, s));
    PrefillActs aH, aQ, aF; // one buffer, three row widths (used one after another)
    LLMRS_TRY(prefill_acts_init(&aH, m->pf_acts, n, H, m->wf, m->pf_bf));
    LLMRS_TRY(prefill_acts_init(&aQ, m->pf_acts, n, QD, m->wf, m->pf_bf));
    LLMRS_TRY(prefill_acts_init(&aF, m->pf_acts, n, F, m->wf, m->pf_bf));
    const float eps = m->cfg.rms_eps, inv_sqrt_d = 1.0f / sqrtf((float)D);
    for (int l = 0; l < m->cfg.n_layers; l++) {
        LayerW &L = m->layers[l];
        LLMRS_TRY(prefill_quantize(m->pf_x, H, L.attn_norm, eps, aH, err, s));
        LLMRS_TRY(prefill_gemm(L.p_qkv, aH, PEPI_STORE, m->pf_qkv, NQKV, nullptr, 0, err, sms, s));
        LLMRS_TRY(prefill_rope_append(m->pf_qkv, L.kc, L.vc, m->rope_cos, m->rope_sin, n, start, Hq, Hkv, D, m->S, s));
        LLMRS_TRY(prefill_attention(m->pf_qkv, L.kc, L.vc, m->pf_ctx, n, start, Hq, Hkv, D, m->S, inv_sqrt_d, s));
        LLMRS_TRY(prefill_quantize(m->pf_ctx, QD, nullptr, 0.0f, aQ, err, s));
        LLMRS_TRY(prefill_gemm(L.p_o, aQ, PEPI_RESIDUAL, m->pf_x, H, m->pf_x, H, err, sms, s));
        LLMRS_TRY(prefill_quantize(m->pf_x, H, L.mlp_norm, eps, aH, err, s));
        LLMRS_TRY(prefill_gemm(L.p_gate_up, aH, PEPI_SILU, m->pf_act, F, nullptr, 0, err, sms, s));
        LLMRS_TRY(prefill_quantize(m->pf_act, F, nullptr, 0.0f, aF, err, s));
        LLMRS_TRY(prefill_gemm(L.p_down, aF, PEPI_RESIDUAL, m->pf_x, H, m->pf_x, H, err, sms, s));
    }
    return LLMRS_OK;
}

// final RMSNorm + LM head + argmax of one residual row (the batch-1 kernel):
// the decode state then holds the next token at position pos + 1
static int prefill_head(llmrs_model *m, const float *x_row, int token, int pos)
{
    LLMRS_TRY(set_token_pos(m, token, pos, 0));
    GemvParams h{};
    h.err = &m->state->err;
    h.eps = m->cfg.rms_eps;
    h.w = m->lm_head.w;
    h.scales = m->lm_head.s;
    h.N = m->Vl;
    h.K = m->H;
    h.x = x_row;
    h.norm_w = m->final_norm;
    h.y = m->logits;
    h.state = m->state;
    h.token_log = m->token_log;
    return gemv_launch(m->lm_head.plan, h, PRO_NORM, EPI_ARGMAX, m->ctx->stream, false);
}

// the ids already in pf_ids: every chunk, then the LM head on the last row
static int prefill_rows(llmrs_model *m, int n, int start_pos, int last_id)
{
    for (int c0 = 0; c0 < n; c0 += PF_CHUNK) {
        const int rows = std::min(PF_CHUNK, n - c0);
        LLMRS_TRY(prefill_chunk(m, m->pf_ids + c0, rows, start_pos + c0));
        if (c0 + rows == n)
            LLMRS_TRY(prefill_head(m, m->pf_x + (size_t)(rows - 1) * m->H, last_id, start_pos + n - 1));
    }
    return LLMRS_OK;
}

int llmrs_model_time_prefill(llmrs_model *m, const int *h_ids, int n, int start_pos, int iters, float *ms_out)
{
    LLMRS_CHECK_ARG(m && h_ids && ms_out && iters > 0, "bad arguments");
    LLMRS_CHECK_ARG(n >= 1 && start_pos >= 0 && start_pos + n <= m->S, "prefill of %d tokens at %d exceeds max_seq %d",
                    n, start_pos, m->S);
    for (int i = 0; i < n; i++)
        LLMRS_CHECK_ARG(h_ids[i] >= 0 && h_ids[i] < m->V, "token id %d at %d out of range", h_ids[i], i);
    cudaSetDevice(m->ctx->device);
    LLMRS_TRY(ensure_graph(m));
    bool tc = false;
    if (n >= PREFILL_MIN_ROWS)
        LLMRS_TRY(prefill_weights_ready(m, &tc));
    if (!tc)
        return fail(LLMRS_ENOTSUP, "this model/prompt does not take the tensor-core prefill path");
    cudaStream_t s = m->ctx->stream;
    LLMRS_TRY(prefill_buffers(m, std::min(n, PF_CHUNK)));
    LLMRS_CUDA_TRY(cudaMemcpyAsync(m->pf_ids, h_ids, (size_t)n * 4, cudaMemcpyHostToDevice, s));
    cudaEvent_t e0, e1;
    LLMRS_CUDA_TRY(cudaEventCreate(&e0));
    LLMRS_CUDA_TRY(cudaEventCreate(&e1));
    int rc = LLMRS_OK;
    cudaEventRecord(e0, s);
    for (int i = 0; i < iters && rc == LLMRS_OK; i++)
        rc = prefill_rows(m, n, start_pos, h_ids[n - 1]);
    cudaEventRecord(e1, s);
    cudaError_t e = cudaEventSynchronize(e1);
    float ms = 0.0f;
    if (e == cudaSuccess)
        e = cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (rc != LLMRS_OK)
        return rc;
    if (e != cudaSuccess)
        return fail(LLMRS_ECUDA, "prefill timing: %s", cudaGetErrorString(e));
    *ms_out = ms / iters;
    uint32_t err = 0;
    LLMRS_CUDA_TRY(cudaMemcpy(&err, &m->state->err, 4, cudaMemcpyDeviceToHost));
    return check_state_err(m, err);
}

int llmrs_prefill(llmrs_model *m, const int *h_ids, int n, int start_pos, float *h_logits, int *h_argmax)
{
    LLMRS_CHECK_ARG(m && h_ids, "NULL argument");
    LLMRS_CHECK_ARG(n >= 1 && start_pos >= 0 && start_pos + n <= m->S, "prefill of %d tokens at %d exceeds max_seq %d",
                    n, start_pos, m->S);
    for (int i = 0; i < n; i++)
        LLMRS_CHECK_ARG(h_ids[i] >= 0 && h_ids[i] < m->V, "token id %d at %d out of range", h_ids[i], i);
    cudaSetDevice(m->ctx->device);
    LLMRS_TRY(ensure_graph(m));
    cudaStream_t s = m->ctx->stream;
    bool tc = false;
    if (n >= PREFILL_MIN_ROWS)
        LLMRS_TRY(prefill_weights_ready(m, &tc));
    if (tc) {
        LLMRS_TRY(prefill_buffers(m, std::min(n, PF_CHUNK)));
        LLMRS_CUDA_TRY(cudaMemcpyAsync(m->pf_ids, h_ids, (size_t)n * 4, cudaMemcpyHostToDevice, s));
        LLMRS_TRY(prefill_rows(m, n, start_pos, h_ids[n - 1]));
    }
    // Otherwise (tensor parallel, short prompts, a linear whose K is not a
    // multiple of 256): rows of a
    // prefill chunk are causal and row-independent in every contraction
    // (src/backend/cpu.rs:90-110, src/core/layer.rs:260-269), so the chunk
    // runs as n consecutive single-row steps over the same cache.
    for (int i = 0; !tc && i < n; i++) {
        if (i % 12 == 0 && i > 0)
            LLMRS_CUDA_TRY(cudaStreamSynchronize(s)); // recycle the 12 pinned staging slots
        LLMRS_TRY(set_token_pos(m, h_ids[i], start_pos + i, 1 + (i % 12)));
        LLMRS_CUDA_TRY(cudaGraphLaunch(m->graph, s));
    }
    int *out = m->h_stage + 60;
    LLMRS_CUDA_TRY(cudaMemcpyAsync(out, &m->state->token, sizeof(int), cudaMemcpyDeviceToHost, s));
    LLMRS_CUDA_TRY(cudaMemcpyAsync(out + 1, &m->state->err, sizeof(int), cudaMemcpyDeviceToHost, s));
    if (h_logits)
        LLMRS_CUDA_TRY(cudaMemcpyAsync(h_logits, m->logits, (size_t)m->Vl * 4, cudaMemcpyDeviceToHost, s));
    LLMRS_CUDA_TRY(cudaStreamSynchronize(s));
    LLMRS_TRY(check_state_err(m, (uint32_t)out[1]));
    if (h_argmax)
        *h_argmax = out[0];
    return LLMRS_OK;
}

int llmrs_model_sample(llmrs_model *m, const int *h_recent, int n_recent, float repeat_penalty, float temperature,
                       float top_p, float u, int *h_token)
{
    LLMRS_CHECK_ARG(m && h_token, "NULL argument");
    LLMRS_CHECK_ARG(m->T == 1, "sample: a tensor-parallel model holds a vocabulary shard per rank");
    cudaSetDevice(m->ctx->device);
    return llmrs_sample(m->ctx, m->logits, m->V, h_recent, n_recent, repeat_penalty, temperature, top_p, u, h_token);
}

int llmrs_model_logits(llmrs_model *m, float *h_logits)
{
    LLMRS_CHECK_ARG(m && h_logits, "NULL argument");
    cudaSetDevice(m->ctx->device);
    LLMRS_CUDA_TRY(cudaMemcpyAsync(h_logits, m->logits, (size_t)m->Vl * 4, cudaMemcpyDeviceToHost, m->ctx->stream));
    return finish_sync(m);
}

int llmrs_model_decode_kernel_count(llmrs_model *m, int *count)
{
    LLMRS_CHECK_ARG(m && count, "NULL argument");
    *count = m->kernels_per_step;
    return LLMRS_OK;
}

int llmrs_model_profile_decode(llmrs_model *m, int token, int pos, float *ms_out, int *kind_out, int *n)
{
    LLMRS_CHECK_ARG(m && ms_out && kind_out && n && *n > 0, "bad arguments");
    LLMRS_CHECK_ARG(token >= 0 && token < m->V && pos >= 0 && pos < m->S, "token/position out of range");
    LLMRS_CHECK_ARG(m->T == 1 || m->tp_connected, "tensor-parallel model is not connected to its peers");
    cudaSetDevice(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    KernelTimer kt;
    kt.cap = 2 * (*n);
    LLMRS_TRY(set_token_pos(m, token, pos, 0));
    int rc = enqueue_step(m, s, &kt);
    cudaError_t e = cudaStreamSynchronize(s);
    int cnt = 0;
    for (size_t i = 0; i + 1 < kt.ev.size(); i += 2) {
        float ms = 0;
        if (e == cudaSuccess)
            e = cudaEventElapsedTime(&ms, kt.ev[i], kt.ev[i + 1]);
        if (cnt < *n) {
            ms_out[cnt] = ms;
            kind_out[cnt] = kt.kind[i];
            cnt++;
        }
    }
    for (auto ev : kt.ev)
        cudaEventDestroy(ev);
    *n = cnt;
    LLMRS_TRY(rc);
    if (e != cudaSuccess)
        return fail(LLMRS_ECUDA, "profile: %s", cudaGetErrorString(e));
    uint32_t err = 0;
    LLMRS_CUDA_TRY(cudaMemcpy(&err, &m->state->err, 4, cudaMemcpyDeviceToHost));
    return check_state_err(m, err);
}

int llmrs_model_trace_decode(llmrs_model *m, int token, int pos, unsigned long long *h_marks, int *kinds, int *n)
{
    LLMRS_CHECK_ARG(m, "model is NULL");
    LLMRS_CHECK_ARG(m->T == 1 || m->tp_connected, "tensor-parallel model is not connected to its peers");
    LLMRS_CHECK_ARG(m && h_marks && kinds && n, "NULL argument");
    LLMRS_CHECK_ARG(token >= 0 && token < m->V && pos >= 0 && pos < m->S, "token/position out of range");
    const int nk = m->kernels_per_step;
    LLMRS_CHECK_ARG(*n >= nk, "marks buffer holds %d kernels, the step launches %d", *n, nk);
    cudaSetDevice(m->ctx->device);
    if (!m->graph_traced)
        LLMRS_TRY(capture_step(m, &m->graph_traced, m->d_trace));
    cudaStream_t s = m->ctx->stream;
    std::vector<unsigned long long> init((size_t)TRACE_MARKS * nk);
    for (int i = 0; i < nk; i++) {
        init[TRACE_MARKS * i] = ~0ull;     // min marks
        init[TRACE_MARKS * i + 1] = ~0ull;
        init[TRACE_MARKS * i + 2] = 0ull;  // max marks
        init[TRACE_MARKS * i + 3] = 0ull;
    }
    LLMRS_CUDA_TRY(cudaMemcpyAsync(m->d_trace, init.data(), init.size() * 8, cudaMemcpyHostToDevice, s));
    LLMRS_TRY(set_token_pos(m, token, pos, 0));
    LLMRS_CUDA_TRY(cudaGraphLaunch(m->graph_traced, s));
    LLMRS_CUDA_TRY(cudaMemcpyAsync(h_marks, m->d_trace, init.size() * 8, cudaMemcpyDeviceToHost, s));
    LLMRS_CUDA_TRY(cudaStreamSynchronize(s));
    for (int l = 0; l < m->cfg.n_layers; l++)
        for (int k = 0; k < 5; k++)
            kinds[5 * l + k] = k;
    kinds[nk - 1] = 5;
    *n = nk;
    uint32_t err = 0;
    LLMRS_CUDA_TRY(cudaMemcpy(&err, &m->state->err, 4, cudaMemcpyDeviceToHost));
    return check_state_err(m, err);
}

int llmrs_time_gemv(llmrs_ctx *ctx, int weight_format, int scale_dtype, const void *const *h_codes,
                    const void *const *h_scales, int copies, const float *d_x, float *d_y, int n, int k, int reps,
                    float *us_per_launch)
{
    LLMRS_CHECK_ARG(ctx && h_codes && h_scales && d_x && d_y && us_per_launch, "NULL argument");
    LLMRS_CHECK_ARG(copies > 0 && copies <= 4096 && reps > 0 && n > 0 && k > 0, "bad sizes");
    LLMRS_CHECK_ARG(weight_format == LLMRS_WFMT_Q4_0 || weight_format == LLMRS_WFMT_Q8_0, "bad weight format");
    LLMRS_CHECK_ARG(scale_dtype == LLMRS_F16 || scale_dtype == LLMRS_F32, "bad scale dtype");
    cudaSetDevice(ctx->device);
    std::vector<GemvPlan> plans((size_t)copies);
    for (int i = 0; i < copies; i++) {
        LLMRS_CHECK_ARG(h_codes[i] && h_scales[i], "NULL weight copy %d", i);
        LLMRS_TRY(gemv_plan(&plans[i], h_codes[i], h_scales[i], n, k, weight_format, scale_dtype, false, ctx->sms));
    }
    cudaStream_t s = ctx->stream;
    // one graph: every copy once, back to back, each launch overlapping its predecessor's tail
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    LLMRS_CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    int rc = LLMRS_OK;
    for (int i = 0; i < copies && rc == LLMRS_OK; i++) {
        GemvParams p{};
        p.w = reinterpret_cast<const uint8_t *>(h_codes[i]);
        p.scales = h_scales[i];
        p.N = n;
        p.K = k;
        p.x = d_x;
        p.y = d_y;
        p.err = ctx->d_err;
        rc = gemv_launch(plans[i], p, PRO_F32, EPI_STORE, s, i > 0);
    }
    cudaError_t e = cudaStreamEndCapture(s, &g);
    if (rc != LLMRS_OK) {
        if (g)
            cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess)
        return fail(LLMRS_ECUDA, "gemv timing capture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess)
        return fail(LLMRS_ECUDA, "gemv timing graph: %s", cudaGetErrorString(e));
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    float ms = 0.0f;
    e = cudaGraphLaunch(ge, s); // warm-up
    if (e == cudaSuccess)
        e = cudaEventCreate(&e0);
    if (e == cudaSuccess)
        e = cudaEventCreate(&e1);
    if (e == cudaSuccess)
        e = cudaEventRecord(e0, s);
    for (int r = 0; r < reps && e == cudaSuccess; r++)
        e = cudaGraphLaunch(ge, s);
    if (e == cudaSuccess)
        e = cudaEventRecord(e1, s);
    if (e == cudaSuccess)
        e = cudaEventSynchronize(e1);
    if (e == cudaSuccess)
        e = cudaEventElapsedTime(&ms, e0, e1);
    if (e0)
        cudaEventDestroy(e0);
    if (e1)
        cudaEventDestroy(e1);
    cudaGraphExecDestroy(ge);
    if (e != cudaSuccess)
        return fail(LLMRS_ECUDA, "gemv timing: %s", cudaGetErrorString(e));
    *us_per_launch = ms * 1000.0f / (float)((size_t)reps * copies);
    return ctx_check_err(ctx);
}

int llmrs_model_time_decode(llmrs_model *m, int token, int pos, int iters, float *ms_total)
{
    LLMRS_CHECK_ARG(m && ms_total && iters > 0, "bad arguments");
    LLMRS_CHECK_ARG(token >= 0 && token < m->V && pos >= 0 && pos + iters <= m->S, "token/position out of range");
    cudaSetDevice(m->ctx->device);
    LLMRS_TRY(ensure_graph(m));
    cudaStream_t s = m->ctx->stream;
    cudaEvent_t e0, e1;
    LLMRS_CUDA_TRY(cudaEventCreate(&e0));
    LLMRS_CUDA_TRY(cudaEventCreate(&e1));
    LLMRS_TRY(set_token_pos(m, token, pos, 0));
    LLMRS_CUDA_TRY(cudaMemsetAsync(&m->state->n_log, 0, sizeof(int), s));
    LLMRS_CUDA_TRY(cudaEventRecord(e0, s));
    for (int i = 0; i < iters; i++)
        LLMRS_CUDA_TRY(cudaGraphLaunch(m->graph, s));
    LLMRS_CUDA_TRY(cudaEventRecord(e1, s));
    LLMRS_CUDA_TRY(cudaEventSynchronize(e1));
    float ms = 0;
    LLMRS_CUDA_TRY(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *ms_total = ms;
    int *out = m->h_stage + 60;
    LLMRS_CUDA_TRY(cudaMemcpy(out + 1, &m->state->err, sizeof(int), cudaMemcpyDeviceToHost));
    return check_state_err(m, (uint32_t)out[1]);
}

// ------------------------------------------------------------ tensor parallel
int llmrs_model_tp_region(llmrs_model *m, void **d_region, size_t *bytes)
{
    LLMRS_CHECK_ARG(m && d_region && bytes, "NULL argument");
    LLMRS_CHECK_ARG(m->T > 1, "model is not tensor parallel (tp_size 1)");
    *d_region = m->tp_region;
    *bytes = m->tp_bytes;
    return LLMRS_OK;
}

int llmrs_model_tp_connect(llmrs_model *m, void *const *regions)
{
    LLMRS_CHECK_ARG(m && regions, "NULL argument");
    LLMRS_CHECK_ARG(m->T > 1, "model is not tensor parallel (tp_size 1)");
    LLMRS_CHECK_ARG(regions[m->rank] == m->tp_region, "regions[%d] must be this rank's own region", m->rank);
    TpLink h{};
    h.rank = m->rank;
    h.size = m->T;
    for (int q = 0; q < m->T; q++) {
        LLMRS_CHECK_ARG(regions[q] != nullptr, "region of rank %d is NULL", q);
        uint8_t *b = reinterpret_cast<uint8_t *>(regions[q]);
        h.ar[TP_CNT_O][q] = reinterpret_cast<unsigned long long *>(b + m->tp_off_o);
        h.ar[TP_CNT_DOWN][q] = reinterpret_cast<unsigned long long *>(b + m->tp_off_d);
        h.keys[q] = reinterpret_cast<unsigned long long *>(b + m->tp_off_keys);
        h.cnt[q] = reinterpret_cast<unsigned long long *>(b + m->tp_off_cnt);
    }
    cudaSetDevice(m->ctx->device);
    LLMRS_CUDA_TRY(cudaMemcpyAsync(m->d_tp, &h, sizeof(h), cudaMemcpyHostToDevice, m->ctx->stream));
    LLMRS_TRY(finish_sync(m));
    m->tp_connected = true;
    return LLMRS_OK;
}

int llmrs_model_set_peer_timeout(llmrs_model *m, int timeout_ms)
{
    LLMRS_CHECK_ARG(m, "model is NULL");
    LLMRS_CHECK_ARG(timeout_ms >= 1 && timeout_ms <= 600000, "peer timeout %d ms outside [1, 600000]", timeout_ms);
    cudaSetDevice(m->ctx->device);
    LLMRS_TRY(finish_sync(m));
    m->peer_ns = (unsigned long long)timeout_ms * 1000000ull;
    // the step graphs hold the old limit: rebuild them on next use
    if (m->graph)
        cudaGraphExecDestroy(m->graph);
    if (m->graph_traced)
        cudaGraphExecDestroy(m->graph_traced);
    m->graph = m->graph_traced = nullptr;
    return LLMRS_OK;
}

int llmrs_model_tp_epoch(llmrs_model *m, unsigned long long *epoch)
{
    LLMRS_CHECK_ARG(m && epoch, "NULL argument");
    cudaSetDevice(m->ctx->device);
    LLMRS_TRY(finish_sync(m));
    LLMRS_CUDA_TRY(cudaMemcpy(epoch, &m->state->epoch, sizeof(*epoch), cudaMemcpyDeviceToHost));
    return LLMRS_OK;
}

int llmrs_model_tp_resync(llmrs_model *m, unsigned long long epoch)
{
    LLMRS_CHECK_ARG(m, "model is NULL");
    LLMRS_CHECK_ARG(m->T > 1 && m->tp_connected, "tensor-parallel model is not connected to its peers");
    cudaSetDevice(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    LLMRS_TRY(finish_sync(m));
    // exchange tags derive from the epoch, so after this every rank tags the
    // same step alike and a stale word never matches; this rank's arrival
    // counters are what `epoch` completed steps leave behind
    unsigned long long cnt[TP_CNT_N] = {};
    cnt[TP_CNT_KEY] = epoch * (unsigned long long)m->T;
    uint8_t *own = reinterpret_cast<uint8_t *>(m->tp_region);
    LLMRS_CUDA_TRY(cudaMemcpyAsync(own + m->tp_off_cnt, cnt, sizeof(cnt), cudaMemcpyHostToDevice, s));
    LLMRS_CUDA_TRY(cudaMemcpyAsync(&m->state->epoch, &epoch, sizeof(epoch), cudaMemcpyHostToDevice, s));
    LLMRS_CUDA_TRY(cudaMemsetAsync(&m->state->key, 0, sizeof(m->state->key), s));
    LLMRS_CUDA_TRY(cudaMemsetAsync(&m->state->done, 0, sizeof(m->state->done), s));
    LLMRS_CUDA_TRY(cudaMemsetAsync(&m->state->err, 0, sizeof(m->state->err), s));
    return finish_sync(m);
}

int llmrs_ipc_get_handle(const void *d_ptr, void *handle_out)
{
    LLMRS_CHECK_ARG(d_ptr && handle_out, "NULL argument");
    static_assert(sizeof(cudaIpcMemHandle_t) == LLMRS_IPC_HANDLE_BYTES, "IPC handle size");
    cudaIpcMemHandle_t h;
    LLMRS_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void *>(d_ptr)));
    memcpy(handle_out, &h, sizeof(h));
    return LLMRS_OK;
}

int llmrs_ipc_open_handle(int device, const void *handle, void **d_ptr_out)
{
    LLMRS_CHECK_ARG(handle && d_ptr_out, "NULL argument");
    LLMRS_CUDA_TRY(cudaSetDevice(device));
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    LLMRS_CUDA_TRY(cudaIpcOpenMemHandle(d_ptr_out, h, cudaIpcMemLazyEnablePeerAccess));
    return LLMRS_OK;
}

int llmrs_ipc_close_handle(int device, void *d_ptr)
{
    LLMRS_CHECK_ARG(d_ptr, "NULL argument");
    LLMRS_CUDA_TRY(cudaSetDevice(device));
    LLMRS_CUDA_TRY(cudaIpcCloseMemHandle(d_ptr));
    return LLMRS_OK;
}

} // extern "C"
