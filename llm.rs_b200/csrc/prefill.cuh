// prefill.cuh - the M>1 (prefill) path: Q8_0 rows of activations times
// Q8_0/Q4_0 weights on the tcgen05 tensor cores, plus the per-row kernels
// around it (RMSNorm + Q8_0 quantise, RoPE + KV append, causal attention).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemv.cuh"

namespace llmrs {

constexpr int PG_TILE = 128;      // weight rows (MMA M, TMEM lanes) and token rows (MMA N, TMEM columns) per tile
constexpr int PG_KSTAGE = 256;    // K elements (8 Q8_0 blocks) per pipeline stage
constexpr int PREFILL_MIN_ROWS = 8; // from this many rows on, M>1 contractions use the tensor cores

// Q8_0 activation rows as the GEMM reads them.  q: [Mpad][K] int8 codes (Q4
// models: every 32-block in the even|odd element order of the nibble planes);
// s: [K/32][Mpad] f32 block scales (block-major, so a tile's scales are one
// box); c: [K/32][Mpad] int32 conversion bias per block (see prefill.cu).
struct PrefillActs {
    int8_t *q = nullptr;
    float *s = nullptr;
    int *c = nullptr;
    int M = 0, Mpad = 0, K = 0, wf = 0;
    int bf16 = 0;         // 1: codes stored as bf16 [Mpad][K] (natural order) for the bf16 tensor-core GEMM
    CUtensorMap tq, ts, tc;
};

// bytes of device memory one PrefillActs of (M, K) needs (either code type)
size_t prefill_acts_bytes(int M, int K);
// carve a PrefillActs out of buf (prefill_acts_bytes(M, K) bytes, 1024-aligned)
int prefill_acts_init(PrefillActs *a, void *buf, int M, int K, int wf, int bf16 = 0);

// weight-side tensor maps of one linear (weights never move)
struct PrefillWeights {
    CUtensorMap tw, ts;
    int wf = 0, st = 0, N = 0, K = 0;
    int ok = 0; // 0: shape not supported by the tensor-core path
    // bf16 copy for the bf16 tensor-core GEMM: codes (Q4: nibble - 8) as bf16
    // [N][K] and scales as f32 block-major [K/32][N]
    void *wbf = nullptr;
    float *sbf = nullptr;
    CUtensorMap tw16, ts16;
    int bf16 = 0;
};
int prefill_weights_init(PrefillWeights *w, const void *codes, const void *scales, int N, int K, int wf, int st);
// bytes the bf16 copy of an (N, K) linear takes
size_t prefill_bf16_bytes(int N, int K);
// fill the bf16 copy into buf (prefill_bf16_bytes(N, K) bytes, 1024-aligned) and
// set its tensor maps
int prefill_weights_to_bf16(PrefillWeights *w, const void *codes, const void *scales, void *buf,
                            cudaStream_t stream);
// which GEMM serves M>1 rows: 1 = bf16 operands (exact integer sums in f32
// accumulators), 0 = int8 operands (LLMRS_PREFILL_BF16 overrides)
int prefill_use_bf16(void);

// x rows [M][ldx] -> (RMSNorm with norm_w when non-null) -> Q8_0 rows in a
int prefill_quantize(const float *x, int ldx, const float *norm_w, float eps, PrefillActs &a, uint32_t *err,
                     cudaStream_t stream);

enum PrefillEpi : int { PEPI_STORE = 0, PEPI_RESIDUAL = 1, PEPI_SILU = 2 };
// y[m][n] (row stride ldy) = sum over blocks of A row m . W row n, block order
// and rounding of src/backend/cpu.rs:888-941; RESIDUAL adds residual[m][n]
// (stride ldr; may alias y); SILU writes silu(row 2i) * row 2i+1 to y[m][i].
int prefill_gemm(const PrefillWeights &w, const PrefillActs &a, int epi, float *y, int ldy, const float *residual,
                 int ldr, uint32_t *err, int sms, cudaStream_t stream);
// set kernel attributes on the current device (once per context)
int prefill_prepare(void);

// rows m of qkv [M][(Hq+2Hkv)*D]: RoPE of q and k at position start+m (in
// place for q), k and v appended to the caches [Hkv][S][D]
int prefill_rope_append(float *qkv, float *kc, float *vc, const float *rope_cos, const float *rope_sin, int M,
                        int start, int Hq, int Hkv, int D, int S, cudaStream_t stream);
// causal attention of rows m (position start+m) over cache positions
// 0..start+m; ctx [M][Hq*D]
int prefill_attention(const float *qkv, const float *kc, const float *vc, float *ctx, int M, int start, int Hq,
                      int Hkv, int D, int S, float inv_sqrt_d, cudaStream_t stream);
// x[m] = embed[ids[m]] (ids on the device)
int prefill_embed(const float *embed, const int *ids, float *x, int M, int H, int V, uint32_t *err,
                  cudaStream_t stream);

} // namespace llmrs
