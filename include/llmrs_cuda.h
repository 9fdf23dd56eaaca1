/*
 * llmrs_cuda.h - C ABI of the B200 (sm_100a) CUDA backend for hedone21/llm.rs.
 *
 * This is the drop-in boundary for the batch-1 Llama token loop.  The op-level
 * entry points replace the methods of the reference's `trait Backend`
 * (src/backend.rs:15-40) on device-resident f32 buffers; the model-level entry
 * points replace the per-op token loop of src/core/model.rs:17-49 /
 * src/core/layer.rs:373-406 with fused, device-resident decode steps (the
 * reference's OpenCL backend crossed the host/device boundary at every op,
 * src/backend/opencl.rs:325-345).
 *
 * Conventions
 *   - Every function returns LLMRS_OK (0) or an LLMRS_E* code; the text of the
 *     last error on the calling thread is available from llmrs_last_error().
 *     (The reference panics instead, e.g. assert_eq! at src/backend/cpu.rs:37;
 *     a Rust shim turns a nonzero status back into a panic.)
 *   - Pointers named d_* (and all op arguments) are device pointers obtained
 *     from llmrs_malloc; h_* are host pointers owned by the caller.
 *   - Work is stream-ordered on the context's stream and asynchronous until
 *     llmrs_d2h / llmrs_sync.  A context is not thread-safe.
 *   - Q4 weights use the reference's planar layout (src/core/tensor.rs:102-167):
 *     nibbles [n][k/2] (byte i: element 2i low nibble, 2i+1 high nibble), then
 *     block scales [n][k/32] as f32 (scale_dtype LLMRS_F32) or as f16 when every
 *     scale is exactly representable (LLMRS_F16, 18 bytes per 32 weights).
 *     Q8_0 weights: int8 codes [n][k] and block scales [n][k/32].
 *     k must be a multiple of 32 (the reference silently drops a k%32 tail,
 *     src/backend/cpu.rs:665-668; this library rejects it with LLMRS_EINVAL).
 */
#ifndef LLMRS_CUDA_H
#define LLMRS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default) /* the library builds with -fvisibility=hidden */
#endif

/* ---- status codes ---- */
#define LLMRS_OK 0
#define LLMRS_EINVAL 1     /* bad argument / shape */
#define LLMRS_ENOMEM 2     /* device allocation failed */
#define LLMRS_ECUDA 3      /* CUDA runtime/driver error */
#define LLMRS_ETIMEDOUT 4  /* a bounded device-side wait ran out (peer or pipeline) */
#define LLMRS_ENOTSUP 5    /* configuration not supported */
#define LLMRS_ENCCL 6      /* NCCL error */
#define LLMRS_EDEVICE 7    /* device-side error word set (bad token id, bad position) */

/* ---- dtypes: block scales (LLMRS_F16 / LLMRS_F32); raw checkpoint tensors
 *      of llmrs_model_load_weight (LLMRS_F32 / LLMRS_BF16) ---- */
#define LLMRS_F16 0
#define LLMRS_F32 1
#define LLMRS_BF16 2

/* ---- weight formats ---- */
#define LLMRS_WFMT_Q4_0 0
#define LLMRS_WFMT_Q8_0 1

typedef struct llmrs_ctx llmrs_ctx;
typedef struct llmrs_model llmrs_model;

/* ======================================================================
 * Library / context  (replaces the OpenCL global ProQue + scratch pool,
 * src/backend/opencl.rs:8-90)
 * ====================================================================== */
const char *llmrs_last_error(void);
const char *llmrs_version(void);
int llmrs_device_count(int *count);
int llmrs_ctx_create(int device, llmrs_ctx **out);
int llmrs_ctx_destroy(llmrs_ctx *ctx);
/* optional: run on a caller-owned cudaStream_t (NULL restores the context's own stream) */
int llmrs_ctx_set_stream(llmrs_ctx *ctx, void *cuda_stream);
int llmrs_malloc(llmrs_ctx *ctx, size_t bytes, void **d_ptr);
int llmrs_free(llmrs_ctx *ctx, void *d_ptr);
/* host<->device copies (Tensor::to_device, src/core/tensor.rs:218-291) */
int llmrs_h2d(llmrs_ctx *ctx, void *d_dst, const void *h_src, size_t bytes);
int llmrs_d2h(llmrs_ctx *ctx, void *h_dst, const void *d_src, size_t bytes);
int llmrs_d2d(llmrs_ctx *ctx, void *d_dst, const void *d_src, size_t bytes);
int llmrs_memset(llmrs_ctx *ctx, void *d_dst, int value, size_t bytes);
int llmrs_sync(llmrs_ctx *ctx);
/* Backend::device / Backend::name (src/backend.rs:17-18): "Cuda" and the device ordinal */
const char *llmrs_backend_name(void);
int llmrs_ctx_device(llmrs_ctx *ctx, int *device);

/* ======================================================================
 * Backend trait operations (src/backend.rs:20-39), device f32 buffers
 * ====================================================================== */
/* Backend::matmul_transposed, Q4 weights: C[m,n] = A[m,k] . W[n,k]^T with the
 * Q8_0 activation quantisation of src/backend/cpu.rs:31-111 (per row of A) */
int llmrs_matmul_transposed_q4(llmrs_ctx *ctx, const float *d_a, const uint8_t *d_qs, const void *d_scales,
                               int scale_dtype, float *d_c, int m, int k, int n);
/* same contraction with Q8_0 weights (int8 codes + block scales) */
int llmrs_matmul_transposed_q8(llmrs_ctx *ctx, const float *d_a, const int8_t *d_qw, const void *d_scales,
                               int scale_dtype, float *d_c, int m, int k, int n);
/* Backend::matmul_transposed, f32 weights B[n,k] (src/backend/cpu.rs:113-146) */
int llmrs_matmul_transposed_f32(llmrs_ctx *ctx, const float *d_a, const float *d_b, float *d_c, int m, int k,
                                int n);
/* Backend::matmul: C[m,n] = A[m,k] . B[k,n] (src/backend/cpu.rs:157-224) */
int llmrs_matmul(llmrs_ctx *ctx, const float *d_a, const float *d_b, float *d_c, int m, int k, int n);
/* Backend::matmul_slice: C[m,rows] = A[m,cols] . Other[rows,cols]^T (src/backend/cpu.rs:230-269) */
int llmrs_matmul_slice(llmrs_ctx *ctx, const float *d_a, const float *d_other, float *d_c, int m, int rows,
                       int cols);
/* Backend::add_assign: a += b (src/backend/cpu.rs:274-296) */
int llmrs_add_assign(llmrs_ctx *ctx, float *d_a, const float *d_b, size_t n);
/* Backend::silu_mul: gate = silu(gate) * up (src/backend/cpu.rs:298-324) */
int llmrs_silu_mul(llmrs_ctx *ctx, float *d_gate, const float *d_up, size_t n);
/* Backend::rope_inplace: rotate-half RoPE over rows of head_dim; row i uses
 * position start_pos + i (src/backend/cpu.rs:326-357; the reference fixes
 * theta_base = 500000) */
int llmrs_rope_inplace(llmrs_ctx *ctx, float *d_x, int rows, int head_dim, int start_pos, float theta_base);
/* Backend::rms_norm (src/backend/cpu.rs:359-393) */
int llmrs_rms_norm(llmrs_ctx *ctx, const float *d_x, const float *d_w, float *d_y, int rows, int cols,
                   float eps);
/* Backend::softmax over the last dimension (src/backend/cpu.rs:395-423) */
int llmrs_softmax(llmrs_ctx *ctx, const float *d_x, float *d_y, int rows, int cols);
/* Backend::scale: y = x * value (src/backend/cpu.rs:425-435) */
int llmrs_scale(llmrs_ctx *ctx, const float *d_x, float *d_y, size_t n, float value);
/* Backend::copy_from (src/backend/cpu.rs:437-446) */
int llmrs_copy_from(llmrs_ctx *ctx, const float *d_src, float *d_dst, size_t n);

/* Fused decode attention for one token at position pos over a device KV cache
 * (the per-head loop of src/core/layer.rs:175-333 for seq == 1, native GQA):
 * RoPE(q), RoPE(k_new) with the caller's [max_seq][head_dim/2] cos/sin tables
 * (llmrs_rope_table), append k_new / v_new at pos, softmax(q.k / sqrt(D)) over
 * positions [0, pos], out = P.V.  d_qkv = q [n_heads*D] | k [n_kv*D] | v [n_kv*D];
 * caches [n_kv][max_seq][D] f32 (position-major).  Split partials live in
 * scratch memory owned by the context (allocated on first use). */
int llmrs_attention_decode(llmrs_ctx *ctx, const float *d_qkv, float *d_kcache, float *d_vcache,
                           const float *d_rope_cos, const float *d_rope_sin, float *d_out, int n_heads,
                           int n_kv_heads, int head_dim, int max_seq, int pos);

/* The same decode attention for callers that cannot allocate device memory
 * (their memory belongs to another allocator that must account for every byte,
 * or they must not allocate after start-up, or they cannot create an llmrs_ctx).
 * No counterpart in the reference: it adds no op, only a way to call this one.
 * Runs on the caller's cuda_stream (NULL = legacy default stream) on the current
 * device; the caller passes every input and output.  Split partials and tickets
 * use a fixed array linked into the library (2 MiB + 1 KiB, held by every GPU
 * that loads the library until exit): n_heads * splits * (head_dim + 2) floats
 * must fit in 2 MiB and n_kv_heads <= 128, else LLMRS_EINVAL.  Nothing is
 * allocated: no cudaMalloc/cudaFree.  The first call on a device resolves the
 * array's device address and sets kernel attributes; make that first call before
 * any stream capture.  All calls share the one array: calls that overlap on the
 * GPU (other streams, other host threads) race and must be serialised by the
 * caller.  Bounded device waits that time out set *d_err (optional device word;
 * NULL keeps the status inside the library, unreported). */
int llmrs_attention_decode_noalloc(void *cuda_stream, const float *d_qkv, float *d_kcache, float *d_vcache,
                                   const float *d_rope_cos, const float *d_rope_sin, float *d_out, int n_heads,
                                   int n_kv_heads, int head_dim, int max_seq, int pos, unsigned int *d_err);

/* Fused causal attention for n_rows consecutive tokens at positions
 * start_pos .. start_pos+n_rows-1 (the per-head loop of src/core/layer.rs:175-333
 * for seq_len > 1, native GQA): RoPE of every row's q (in place in d_qkv) and k,
 * k / v appended to the caches, then row i attends to positions
 * [0, start_pos + i] (the causal mask of src/core/layer.rs:260-269).
 * d_qkv rows [n_rows][(n_heads + 2*n_kv_heads)*head_dim] (q | k | v);
 * d_out rows [n_rows][n_heads*head_dim]. */
int llmrs_attention_prefill(llmrs_ctx *ctx, float *d_qkv, float *d_kcache, float *d_vcache, const float *d_rope_cos,
                            const float *d_rope_sin, float *d_out, int n_rows, int n_heads, int n_kv_heads,
                            int head_dim, int max_seq, int start_pos);

/* Next-token sampling of src/main.rs:192-305 on the device, over d_logits[vocab]:
 * repetition penalty (when repeat_penalty > 1) on each distinct id of
 * h_recent[n_recent] (the caller passes the last penalty_window ids, at most
 * 4096), temperature, softmax, then top-p (top_p < 1) or roulette selection.
 * u in [0, 1) is the uniform draw the reference takes from rng.random::<f32>()
 * (an OS-seeded generator there; the caller's draw here, so runs repeat).
 * Probabilities agree with the reference to rounding; ties in p go to the lower
 * id.  Blocks until *h_token is written. */
int llmrs_sample(llmrs_ctx *ctx, const float *d_logits, int vocab, const int *h_recent, int n_recent,
                 float repeat_penalty, float temperature, float top_p, float u, int *h_token);

/* CpuBackend::quantize_row_q8_0 (src/backend/cpu.rs:663-745) for rows of k
 * values: codes [rows][k] and f32 scales [rows][k/32]; bit-exact */
int llmrs_quantize_row_q8_0(llmrs_ctx *ctx, const float *d_x, int8_t *d_q, float *d_s, int rows, int k);
/* CpuBackend::rms_norm then quantize_row_q8_0 of one row of k values
 * (src/backend/cpu.rs:359-393, 724-743) exactly as the decode GEMVs' fused
 * prologue computes them (its thread count and reduction tree; the sum of
 * squares is tree-ordered, so a value within rounding of a Q8_0 boundary can
 * take the neighbouring code): codes [k], f32 scales [k/32].  For parity
 * checks of that prologue; d_x, d_w and d_q 16-byte aligned, k <= 38912. */
int llmrs_rms_norm_quantize_q8_0(llmrs_ctx *ctx, const float *d_x, const float *d_w, int8_t *d_q, float *d_s, int k,
                                 float eps);
/* Tensor::quantize_q4 (src/core/tensor.rs:102-167): n values -> planar nibbles
 * [(n+1)/2] and f32 scales [(n+31)/32]; bit-exact */
int llmrs_quantize_q4(llmrs_ctx *ctx, const float *d_w, size_t n, uint8_t *d_qs, float *d_scales);

/* ======================================================================
 * Model: device-resident weights + KV cache, fused decode step
 * (LlamaModel src/core/model.rs, LlamaBlock/Attention/MLP src/core/layer.rs,
 *  Loader layout decisions src/core/loader.rs:62-198)
 * ====================================================================== */
typedef struct {
    int n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab;
    int max_seq;        /* KV capacity (the reference hard-codes 2048, src/core/loader.rs:162-166) */
    float rms_eps;      /* LlamaConfig::rms_norm_eps */
    float rope_theta;   /* LlamaConfig::rope_theta (500000) */
    int weight_format;  /* LLMRS_WFMT_Q4_0 or LLMRS_WFMT_Q8_0 */
    int tied_embeddings;/* LM head = quantize_q4(embed_tokens), src/core/loader.rs:186-190 */
    int scale_dtype;    /* LLMRS_F16: 18 B per 32 Q4 weights, every scale must be exactly
                           representable (synthetic models); LLMRS_F32: the reference's own
                           f32 scales (20 B per 32), e.g. for quantize_q4 of real checkpoints */
    int tp_rank;        /* tensor parallel: this process's rank (0 for one GPU) */
    int tp_size;        /* ranks (1, 2, 4 or 8; 0 = 1).  Rank r holds query/KV heads
                           [r*n/tp, (r+1)*n/tp), FFN rows [r*ffn/tp, ...), the matching
                           o_proj / down_proj input columns and LM-head rows
                           [r*vocab/tp, ...); o_proj and down_proj outputs are summed
                           across ranks over NVLink.  No counterpart in the reference
                           (CPU / OpenCL, one device). */
} llmrs_config;

/* which-codes for llmrs_model_set_weight */
#define LLMRS_W_Q 0          /* [n_heads*D][hidden]            quantised */
#define LLMRS_W_K 1          /* [n_kv_heads*D][hidden]         quantised (native GQA, not expanded) */
#define LLMRS_W_V 2          /* [n_kv_heads*D][hidden]         quantised */
#define LLMRS_W_O 3          /* [hidden][n_heads*D]            quantised */
#define LLMRS_W_GATE_UP 4    /* [2*ffn][hidden] gate rows then up rows (src/core/loader.rs:128-147) */
#define LLMRS_W_DOWN 5       /* [hidden][ffn]                  quantised */
#define LLMRS_W_ATTN_NORM 6  /* [hidden] f32 */
#define LLMRS_W_MLP_NORM 7   /* [hidden] f32 */
#define LLMRS_W_EMBED 8      /* [vocab][hidden] f32 */
#define LLMRS_W_FINAL_NORM 9 /* [hidden] f32 */
#define LLMRS_W_LM_HEAD 10   /* [vocab][hidden] quantised (ignored when tied) */
#define LLMRS_W_GATE 11      /* [ffn][hidden] quantised: gate_proj alone (the gate rows of LLMRS_W_GATE_UP) */
#define LLMRS_W_UP 12        /* [ffn][hidden] quantised: up_proj alone (the up rows of LLMRS_W_GATE_UP) */

int llmrs_model_create(llmrs_ctx *ctx, const llmrs_config *cfg, llmrs_model **out);
int llmrs_model_destroy(llmrs_model *model);
/* random-init every weight from `seed` with the documented synthetic recipe */
int llmrs_model_init_synthetic(llmrs_model *model, uint64_t seed);
/* upload one tensor in the reference layout (quantised: h_codes + h_scales as
 * f32; f32 tensors: h_codes is float*, h_scales NULL), always the whole,
 * unsharded tensor of the shapes listed with the which-codes: a tensor-parallel
 * rank takes its own shard (its heads' rows of q/k/v, its columns of o_proj and
 * down_proj, its FFN rows of gate/up, its vocab rows of the LM head; the full
 * embedding and norms).  For the tied 1B head the LM head is re-derived on the
 * device with quantize_q4 of the embedding. */
int llmrs_model_set_weight(llmrs_model *model, int layer, int which, const void *h_codes, const float *h_scales);
/* Load one checkpoint tensor as the reference's loader reads it
 * (src/core/loader.rs:25-46 read_tensor: f32 or bf16, row-major [rows][cols],
 * the layout of the safetensors file; dtype LLMRS_F32 or LLMRS_BF16), whole and
 * unsharded as for llmrs_model_set_weight.  On the device: bf16 -> f32 (exact),
 * then for the linears quantize_q4 (src/core/tensor.rs:102-167, f32 block
 * scales; Q8_0 models: the Q8_0 block quantiser), with the loader's layout
 * decisions: K/V kept at n_kv_heads rows (the reference replicates them per
 * query head, loader.rs:62-98, which quantises to identical rows), gate and up
 * accepted fused (LLMRS_W_GATE_UP, loader.rs:128-147) or as LLMRS_W_GATE /
 * LLMRS_W_UP, and the tied LM head quantised from the embedding
 * (loader.rs:186-190).  Quantize_q4 scales are rarely exact in f16: checkpoint
 * models use scale_dtype LLMRS_F32 (else LLMRS_EINVAL). */
int llmrs_model_load_weight(llmrs_model *model, int layer, int which, const void *h_data, int dtype);
/* KV cache: h_k/h_v [n_kv_heads][n_pos][head_dim] f32 written at positions [0,n_pos) */
int llmrs_kv_fill(llmrs_model *model, int layer, const float *h_k, const float *h_v, int n_pos);
int llmrs_kv_fill_synthetic(llmrs_model *model, uint64_t seed, int n_pos);
int llmrs_kv_read(llmrs_model *model, int layer, float *h_k, float *h_v, int n_pos);
/* one decode step: token at position pos (KV [0,pos) must be valid).  Writes the
 * next greedy token to *h_argmax and, if h_logits is non-NULL, the [vocab]
 * logits.  Synchronous. */
int llmrs_decode_step(llmrs_model *model, int token, int pos, float *h_logits, int *h_argmax);
/* greedy loop on the device: n_steps decode steps starting from (token, pos),
 * each step feeding its argmax to the next; tokens_out[i] = argmax of step i.
 * Runs as CUDA-graph replays with no host round trip between steps. */
int llmrs_generate(llmrs_model *model, int token, int pos, int n_steps, int *h_tokens_out);
/* prefill n prompt tokens at positions [start_pos, start_pos+n) (src/main.rs:134-138
 * chunk, the m>1 path of src/backend/cpu.rs:90-110); writes the last row's
 * logits / argmax like llmrs_decode_step.  On one GPU, n >= 8 rows with every
 * linear's K a multiple of 256 run as M = n contractions on the tensor cores
 * (chunks of 512 rows; the LM head on the last row only, the row the caller
 * reads at src/main.rs:185-190); otherwise as n single-row steps. */
int llmrs_prefill(llmrs_model *model, const int *h_ids, int n, int start_pos, float *h_logits, int *h_argmax);
/* device time (CUDA events) of one tensor-core prefill of h_ids, averaged over
 * iters back-to-back prefills with the ids already on the device;
 * LLMRS_ENOTSUP when the prompt/model takes the single-row path */
int llmrs_model_time_prefill(llmrs_model *model, const int *h_ids, int n, int start_pos, int iters, float *ms_out);
/* llmrs_sample over the model's last decode/prefill logits (one GPU) */
int llmrs_model_sample(llmrs_model *model, const int *h_recent, int n_recent, float repeat_penalty, float temperature,
                       float top_p, float u, int *h_token);
/* read the last decode/prefill logits (device resident) into h_logits[vocab] */
int llmrs_model_logits(llmrs_model *model, float *h_logits);
/* host-only helper: the RoPE cos/sin table the decode step uses, [n_pos][head_dim/2]
 * each, computed with the host libm exactly as src/backend/cpu.rs:345-349 does */
int llmrs_rope_table(int head_dim, int n_pos, float theta_base, float *h_cos, float *h_sin);
/* model-level stats: number of kernels the decode step launches */
int llmrs_model_decode_kernel_count(llmrs_model *model, int *count);
/* run one decode step kernel by kernel (no graph, no programmatic overlap)
 * with a CUDA event pair around every kernel on the model's stream; writes
 * each kernel's duration (ms) to ms_out[i] and its kind to kind_out[i]
 * (0 QKV GEMV, 1 attention, 2 o_proj GEMV, 3 gate_up GEMV, 4 down GEMV,
 * 5 LM head GEMV) for i < *n (in: capacity, out: kernels run) */
int llmrs_model_profile_decode(llmrs_model *model, int token, int pos, float *ms_out, int *kind_out, int *n);
/* run one decode step through a traced copy of the step graph (same launches,
 * same programmatic overlap) and return a device timeline: for kernel i,
 * h_marks[4i] = first CTA start, [4i+1] = first CTA past its wait on the previous
 * kernel, [4i+2] = last CTA done with its activation prologue, [4i+3] = last CTA
 * end (globaltimer ns); kinds[i] as in profile_decode.
 * *n: in = capacity (kernels), out = kernels of the step */
int llmrs_model_trace_decode(llmrs_model *model, int token, int pos, unsigned long long *h_marks, int *kinds, int *n);
/* Device time per launch of the batch-1 GEMV of llmrs_matmul_transposed_q4/_q8
 * (m = 1): the `copies` weight matrices [n][k] (h_codes[i] / h_scales[i]: device
 * pointers, the layout of llmrs_matmul_transposed_q4) are multiplied with d_x[k]
 * into d_y[n] back to back as one CUDA graph, each launch overlapping its
 * predecessor's tail as consecutive GEMVs of a decode step do; the graph is
 * replayed `reps` times after one warm-up replay.  Copies that together exceed
 * the L2 make every launch stream its weights from HBM.  A measurement helper
 * (the reference's bench binary, src/bench/main.rs, times its ops on the host). */
int llmrs_time_gemv(llmrs_ctx *ctx, int weight_format, int scale_dtype, const void *const *h_codes,
                    const void *const *h_scales, int copies, const float *d_x, float *d_y, int n, int k, int reps,
                    float *us_per_launch);
/* time `iters` device-resident decode steps (graph replays) with CUDA events
 * on the model's stream; *ms_total = elapsed ms; the KV position advances */
int llmrs_model_time_decode(llmrs_model *model, int token, int pos, int iters, float *ms_total);

/* ---- tensor parallel (one process per GPU; no counterpart in the reference) ----
 * Each rank's model owns a communication region (partial sums of o_proj and
 * down_proj from every rank, LM-head argmax keys, arrival counters).  Ranks
 * exchange IPC handles of their regions (any host channel), open the others'
 * and connect; decode calls then run on all ranks in the same order with the
 * same token/position, every rank gets the same greedy token, and logits are
 * the rank's vocab shard (vocab/tp floats).  A peer that stops answering makes
 * the waiting kernels give up after the peer timeout (5 s unless set) and the
 * step return LLMRS_ETIMEDOUT; the context stays usable, and the ranks resume
 * with llmrs_model_tp_resync. */
#define LLMRS_IPC_HANDLE_BYTES 64
/* the region of this rank (device pointer and size) */
int llmrs_model_tp_region(llmrs_model *model, void **d_region, size_t *bytes);
/* regions[q] = rank q's region as mapped in this process (regions[rank] = own) */
int llmrs_model_tp_connect(llmrs_model *model, void *const *regions);
/* CUDA IPC of a cudaMalloc'ed region: handle out (LLMRS_IPC_HANDLE_BYTES) */
int llmrs_ipc_get_handle(const void *d_ptr, void *handle_out);
/* map another process's region on `device` (peer access over NVLink) */
int llmrs_ipc_open_handle(int device, const void *handle, void **d_ptr_out);
int llmrs_ipc_close_handle(int device, void *d_ptr);
/* the longest a decode-step kernel waits for another rank's partial sums or
 * argmax key before the step fails with LLMRS_ETIMEDOUT (default 5000 ms;
 * 1 .. 600000); the step graph is rebuilt on its next launch */
int llmrs_model_set_peer_timeout(llmrs_model *model, int timeout_ms);
/* decode steps this rank has completed (the count its exchange tags derive
 * from; ranks that ran the same steps agree) */
int llmrs_model_tp_epoch(llmrs_model *model, unsigned long long *epoch);
/* After a step that timed out on some rank (ranks then disagree on the step
 * count): every rank calls this with the same epoch (e.g. the maximum of
 * llmrs_model_tp_epoch over the ranks), while no rank has a step running
 * (a host barrier before and after).  Clears the device error word and sets
 * this rank's step count and arrival counters so the next step's exchanges
 * match on every rank.  No counterpart in the reference (one device). */
int llmrs_model_tp_resync(llmrs_model *model, unsigned long long epoch);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif /* LLMRS_CUDA_H */
