// gemv.cuh - batch-1 quantised matrix-vector product (decode hot path).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace llmrs {

// activation prologues
enum GemvPro : int {
    PRO_F32 = 0,        // x [K] f32 -> Q8_0
    PRO_NORM = 1,       // RMSNorm(x, norm_w) -> Q8_0
    PRO_EMBED_NORM = 2, // x = embed[*token] (CTA 0 stores it to x_out) -> RMSNorm -> Q8_0
    PRO_Q8 = 3,         // pre-quantised codes xq [K] + scales xs [K/32]
    PRO_AR_NORM = 4,    // tensor parallel: x = (sum of every rank's partial) + x (CTA 0 stores it to
                        // x_out) once all partials arrived -> RMSNorm -> Q8_0
};

// output epilogues
enum GemvEpi : int {
    EPI_STORE = 0,    // y[row] = acc
    EPI_RESIDUAL = 1, // y[row] = acc + residual[row]   (y may alias residual)
    EPI_SILU = 2,     // rows (2i, 2i+1) = (gate_i, up_i): y[i] = silu(gate_i) * up_i
    EPI_ARGMAX = 3,   // y[row] = acc; greedy argmax over all rows -> step state
    EPI_PARTIAL = 4,  // tensor parallel: acc -> every rank's partial buffer, then count the CTA in
};

// Tensor-parallel links of one rank: pointers into every rank's communication
// region (this rank's own included), mapped over NVLink.
constexpr int TP_MAX = 8;
enum TpCounter : int { TP_CNT_O = 0, TP_CNT_DOWN = 1, TP_CNT_KEY = 2, TP_CNT_N = 4 };
struct TpLink {
    int rank = 0, size = 1;
    // [o / down][rank q]: q's receive buffer [size][N] of 64-bit words (tag << 32 | f32 bits),
    // block r written by rank r; a word is valid once it carries the exchange's tag
    unsigned long long *ar[2][TP_MAX] = {};
    unsigned long long *cnt[TP_MAX] = {}; // [rank q]: q's arrival counters [TP_CNT_N]
    unsigned long long *keys[TP_MAX] = {}; // [rank q]: q's argmax key slots [size]
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
    unsigned long long epoch; // decode steps completed (tensor-parallel counter targets)
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
    int n_stages;          // set by gemv_launch from the plan
    int n_pre;             // stages streamed before the activation is requested (set by gemv_launch)
    int box_rows;
    int rows_per_cta;
    unsigned long long *trace; // optional timeline marks, 3 per kernel (see trace_start)
    int trace_slot;
    // tensor parallel (EPI_PARTIAL, PRO_AR_NORM, EPI_ARGMAX over a vocab shard)
    const TpLink *tp;      // nullptr: one GPU
    int ar_kind;           // TP_CNT_O / TP_CNT_DOWN
    int ar_index;          // all-reduce instance within the step (layer)
    int ar_per_step;       // instances of this kind per step
    int row_offset;        // EPI_ARGMAX: global index of local row 0
    unsigned long long peer_ns; // longest wait for another rank's data (0: 5 s)
    int pro, epi;          // GemvPro / GemvEpi of this launch (set by gemv_launch)
};

// Launch geometry + TMA descriptors of one weight matrix, built once per weight.
// Each CTA owns rows [i*rows_per_cta, (i+1)*rows_per_cta) and streams them as
// tiles of box_rows rows x 32 blocks with 2-D tensor-map copies.
struct GemvPlan {
    CUtensorMap tw;    // codes: [N rows][K/2 or K bytes] viewed as u32 elements
    CUtensorMap ts;    // scales: [N rows][K/32] f16 or f32
    int fast = 0;      // 0: shape needs the simple fallback kernel
    int wf = 0, st = 0, N = 0, K = 0;
    int box_rows = 0, rows_per_cta = 0, grid = 0, stages = 0;
    size_t smem = 0;
};

// wf: 0 = Q4_0, 1 = Q8_0; st: 0 = f16 scales, 1 = f32.  pairs: row pairs must
// stay in one tile (SiLU epilogue over interleaved gate/up rows).
int gemv_plan(GemvPlan *plan, const void *w, const void *scales, int N, int K, int wf, int st, bool pairs,
              int sms);
// p.w / p.scales / p.N / p.K must match the plan
int gemv_launch(const GemvPlan &plan, const GemvParams &p, int pro, int epi, cudaStream_t stream, bool pdl);
// set kernel attributes (dynamic smem limits) for every variant on the current device;
// called once per context, outside any stream capture
int gemv_prepare(void);
// one row's RMSNorm + Q8_0 exactly as the GEMV prologue computes it (codes [K], scales [K/32])
int gemv_norm_quantize(const float *x, const float *w, int K, float eps, int8_t *q, float *s, uint32_t *err,
                       cudaStream_t stream);
// CTAs a launch of this plan uses
int gemv_grid(const GemvPlan &plan);
// weight stages a GEMV streams before its activation loads are issued
// (LLMRS_GEMV_PREFETCH, default 0)
int gemv_prefetch_stages(void);
// cuTensorMapEncodeTiled from the driver (nullptr if unavailable)
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

} // namespace llmrs
