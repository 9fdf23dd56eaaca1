// ops.cuh - launchers for the op-level kernels and the synthetic generators.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace llmrs {

int op_add_assign(cudaStream_t s, float *a, const float *b, size_t n);
int op_silu_mul(cudaStream_t s, float *g, const float *u, size_t n);
int op_scale(cudaStream_t s, const float *x, float *y, size_t n, float v);
int op_copy(cudaStream_t s, const float *x, float *y, size_t n);
int op_rope(cudaStream_t s, float *x, int rows, int head_dim, int start_pos, float theta);
int op_rms_norm(cudaStream_t s, const float *x, const float *w, float *y, int rows, int cols, float eps);
int op_softmax(cudaStream_t s, const float *x, float *y, int rows, int cols);
int op_matmul_t(cudaStream_t s, const float *a, const float *b, float *c, int m, int k, int n);
int op_matmul(cudaStream_t s, const float *a, const float *b, float *c, int m, int k, int n);
int op_quantize_q8(cudaStream_t s, const float *x, int8_t *q, float *sc, size_t nblocks);
int op_quantize_q4(cudaStream_t s, const float *w, size_t n, uint8_t *qs, float *scales);
int op_bf16_to_f32(cudaStream_t s, const uint16_t *src, float *dst, size_t n);

// synthetic quantised tensor: rows [row0,row0+nrows) x cols [col0,col0+ncols)
// of the logical [.][K] tensor; destination row of source row r is
// r*dst_row_mul + dst_row_add; st 0 = f16 scales, 1 = f32
int synth_quant(cudaStream_t s, int wf, uint64_t seed, uint32_t layer, uint32_t tensor, int K, int row0, int nrows,
                int col0, int ncols, void *dst_w, void *dst_s, int st, int dst_row_mul, int dst_row_add);
int synth_normal(cudaStream_t s, uint64_t seed, uint32_t layer, uint32_t tensor, size_t n, float mu, float sd,
                 float *out);
int synth_kv(cudaStream_t s, uint64_t seed, uint32_t layer, int h0, int nh, int n_pos, int S, int D, float *kc,
             float *vc);
// f32 -> f16 block scales; *d_flag |= 1 if any scale is not exactly representable
int scales_to_f16(cudaStream_t s, const float *src, void *dst, size_t n, uint32_t *d_flag);

} // namespace llmrs
