/*
 * oracle.h - CPU restatement of hedone21/llm.rs's x86_64 CPU path for the
 * batch-1 Llama token loop.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg use it, as the checker and as the timed CPU reference arm.
 *
 * Parity status.  The reference is Rust and cannot be compiled in this image
 * (no cargo/rustc, dependencies not vendored), so there is no reference binary
 * to pin against.  Pinned by the reference's own known-answer and property
 * tests (tests/test_oracle_*.py): RMSNorm [1,2,3,4] known answer
 * (src/test/cpu.rs:197-212), softmax sum/order (src/test/cpu.rs:214-227), RoPE
 * pair magnitude (src/test/cpu.rs:229-245), the Q4 dequantisation identity
 * (src/test/opencl.rs:182-258), attention causality and KV update
 * (src/core/layer.rs:430-489), naive matmul agreement (src/test/cpu.rs:103-160).
 * Parity unpinned: the Q8_0 activation quantiser, the Q4xQ8 block kernel and
 * the full-model logits have no reference golden vectors; for them the oracle
 * is a line-by-line restatement of the cited reference code.
 */
#ifndef LLMRS_ORACLE_H
#define LLMRS_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Backend-trait operations (src/backend/cpu.rs) ---- */
void orc_set_threads(int n);
int orc_get_threads(void);
void orc_quantize_row_q8_0(const float *x, int k, int8_t *q, float *s);
void orc_quantize_q4(const float *w, size_t n, uint8_t *qs, float *scales);
void orc_matmul_transposed_q4(const float *a, int m, int k, const uint8_t *qs, const float *sw, int n, float *c);
void orc_matmul_transposed_q8w(const float *a, int m, int k, const int8_t *qw, const float *sw, int n, float *c);
void orc_matmul_transposed_f32(const float *a, int m, int k, const float *b, int n, float *c);
void orc_matmul_f32(const float *a, int m, int k, const float *b, int n, float *c);
void orc_matmul_slice(const float *a, int m, int k, const float *other, int rows, float *c);
void orc_add_assign(float *a, const float *b, size_t n);
void orc_silu_mul(float *gate, const float *up, size_t n);
void orc_rope_inplace(float *x, int rows, int head_dim, int start_pos, float theta_base);
void orc_rms_norm(const float *x, const float *w, float *y, int rows, int cols, float eps);
void orc_softmax(const float *x, float *y, int rows, int cols);
void orc_scale(const float *x, float *y, size_t n, float value);
void orc_dequantize_q4(const uint8_t *qs, const float *scales, size_t n, float *out);

/* ---- model (src/core/{model,layer,loader}.rs) ---- */
typedef struct {
    int n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab;
    int max_seq;
    float rms_eps, rope_theta;
    int weight_format; /* 0 = Q4_0, 1 = Q8_0 */
    int tied_embeddings;
} orc_config;

typedef struct orc_model orc_model;

orc_model *orc_model_create(const orc_config *cfg, int expand_gqa);
void orc_model_destroy(orc_model *m);
void orc_model_init_synthetic(orc_model *m, uint64_t seed);
void orc_model_kv_fill_synthetic(orc_model *m, uint64_t seed, int n_pos);
/* forward of a chunk of n tokens at start_pos; writes the logits of the last row */
int orc_model_forward(orc_model *m, const int *ids, int n, int start_pos, float *logits_last);
/* forward from caller-provided embeddings [n][hidden] (used by layer-level tests) */
int orc_model_forward_embeds(orc_model *m, const float *x, int n, int start_pos, float *logits_last);
/* record, in every later forward, the last row's residual stream entering each
 * RMSNorm into buf[2*n_layers+1][hidden]: [2l] before layer l's attention norm,
 * [2l+1] before its MLP norm, [2L] before the final norm (NULL stops) */
void orc_model_set_trace(orc_model *m, float *buf);
/* raw access for tests and uploads (reference layouts) */
int orc_model_tensor(orc_model *m, int layer, int which, void **qs, void **scales, size_t *n_rows, size_t *k);
float *orc_model_kcache(orc_model *m, int layer);
float *orc_model_vcache(orc_model *m, int layer);
size_t orc_model_cache_heads(orc_model *m);

int orc_argmax(const float *v, int n);
int orc_sample(const float *logits, int V, const int *recent, int n_recent, float penalty, float temperature,
               float top_p, float u, float *margin);
float orc_top2_margin(const float *v, int n);

/* synthetic generator helpers exposed for tests */
void orc_synth_q4(uint64_t seed, uint32_t layer, uint32_t tensor, size_t n, size_t k, uint8_t *qs, float *scales);
void orc_synth_q8(uint64_t seed, uint32_t layer, uint32_t tensor, size_t n, size_t k, int8_t *qw, float *scales);
void orc_synth_normal(uint64_t seed, uint32_t layer, uint32_t tensor, size_t n, float mu, float sd, float *out);
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);
uint32_t orc_synth_token(uint64_t seed, uint64_t i, uint32_t vocab);

/* which-codes for orc_model_tensor (and the device library's weight API) */
enum {
    ORC_W_Q = 0, ORC_W_K = 1, ORC_W_V = 2, ORC_W_O = 3, ORC_W_GATE_UP = 4, ORC_W_DOWN = 5,
    ORC_W_ATTN_NORM = 6, ORC_W_MLP_NORM = 7, ORC_W_EMBED = 8, ORC_W_FINAL_NORM = 9, ORC_W_LM_HEAD = 10
};

#ifdef __cplusplus
}
#endif
#endif
