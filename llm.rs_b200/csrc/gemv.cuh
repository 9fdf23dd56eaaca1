// gemv.cuh - batch-1 quantised matrix-vector product (decode hot path).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace llmrs {

// activation prologues
enum GemvPro : int {
    PRO_F32 = 0,        // x [K] f32 -> Q8_0
    PRO_NORM = 1,       // RMSNorm(x, norm_w) -> Q8_0
    PRO_EMBED_NORM = 2, // x = embed[*token] (CTA 0 stores it to x_out) -> RMSNorm -> Q8_0
    PRO_Q8 = 3,         // pre-quantised codes xq [K] + scales xs [K/32]
};

// output epilogues
enum GemvEpi : int {
    EPI_STORE = 0,    // y[row] = acc
    EPI_RESIDUAL = 1, // y[row] = acc + residual[row]   (y may alias residual)
    EPI_SILU = 2,     // rows (2i, 2i+1) = (gate_i, up_i): y[i] = silu(gate_i) * up_i
    EPI_ARGMAX = 3,   // y[row] = acc; greedy argmax over all rows -> step state
};

struct StepState {
    int token;               // input token of the current decode step
    int pos;                 // its position
    unsigned long long key;  // argmax key of the step being computed
    unsigned int done;       // LM-head CTA completion counter
    unsigned int err;        // device error word (DEV_ERR_*)
    int n_log;               // tokens appended to the log so far
    int log_cap;             // capacity of the token log
    int pad;
};

struct GemvParams {
    const uint8_t *w;      // Q4: [N][K/2] nibbles; Q8: [N][K] codes
    const void *scales;    // [N][K/32] f16 or f32
    int N, K;
    // prologue inputs
    const float *x;
    const float *norm_w;
    float eps;
    const float *embed;
    int vocab;
    float *x_out;
    const int8_t *xq;
    const float *xs;
    // epilogue
    float *y;
    const float *residual;
    StepState *state;      // EPI_ARGMAX / PRO_EMBED_NORM
    int *token_log;        // EPI_ARGMAX: appended greedy tokens
    uint32_t *err;         // device error word
    int n_stages;
};

// Launch the fast (TMA-pipelined) kernel when the shape allows it (K % 256 == 0,
// N even, 16-byte aligned operands); otherwise a simple row-per-thread kernel
// with identical arithmetic.  wf: 0 = Q4_0, 1 = Q8_0; st: 0 = f16 scales, 1 = f32.
int gemv_launch(const GemvParams &p, int wf, int st, int pro, int epi, cudaStream_t stream, bool pdl,
                int max_ctas);
// bytes of dynamic shared memory the fast kernel uses for this shape (0 = fallback)
size_t gemv_smem_bytes(int wf, int st, int K, int *stages);
bool gemv_fast_ok(const GemvParams &p, int wf, int st);
// set kernel attributes (dynamic smem limits) for every variant on the current device;
// called once per context, outside any stream capture
int gemv_prepare(void);

} // namespace llmrs
