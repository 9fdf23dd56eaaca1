// step.cuh - the whole decode step as one persistent kernel (host interface).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "attention.cuh"
#include "gemv.cuh"

namespace llmrs {

enum StepOpKind : int { OP_GEMV = 0, OP_ATTN = 1 };

// One op of the decode step, as the persistent kernel reads it from device
// memory.  GEMV: tw/ts, g (n_stages, box_rows, rows_per_cta filled in), pro,
// epi, wf, st.  Attention: a (tk encoded with STEP_ATTN_ROWS-row boxes).
// wait_op: the op whose output (all CTAs) this op reads; -1 for none (the
// first op, or an all-reduce prologue that waits on the ranks' counters).
struct alignas(64) StepOp {
    CUtensorMap tw, ts;
    GemvParams g;
    AttnParams a;
    int kind, pro, epi, wf, st, wait_op;
};

constexpr int STEP_ATTN_ROWS = 16; // cached positions per ring stage in the attention op

// Shared memory the kernel needs for models of this shape (0 if no
// instantiation covers it); *stages: ring depth.
size_t step_smem_bytes(int wf, int st, int lm_st, int D, int nrep, int tp, int kmax, int *stages);
// set kernel attributes on the current device (once, outside capture)
int step_prepare(void);
// one decode step over n_ops ops on `grid` co-resident CTAs (cooperative
// launch); trace (optional): TRACE_MARKS timeline marks per op, the layout of
// the one-kernel-per-op timeline
int step_launch(int wf, int st, int lm_st, int D, int nrep, int tp, int kmax, int stages, size_t smem, int grid,
                const StepOp *d_ops, int n_ops, unsigned long long *d_done, const StepState *state, uint32_t *err,
                unsigned long long *trace, cudaStream_t stream);

} // namespace llmrs
