// attention.cuh - decode attention over the device-resident KV cache.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "gemv.cuh"

namespace llmrs {

struct AttnParams {
    CUtensorMap tk;          // K cache as [D/32 segments][rows][32 floats], 128B-swizzled boxes (set at launch)
    const float *qkv;        // q [Hq*D] | k [Hkv*D] | v [Hkv*D], pre-RoPE (fused QKV GEMV output)
    float *kc, *vc;          // KV cache [Hkv][S][D] f32, position-major
    const float *rope_cos;   // [S][D/2]
    const float *rope_sin;   // [S][D/2]
    float *ctx;              // [Hq*D] attention output (context)
    float *part;             // split partials [Hq][n_splits][D + 2]
    unsigned int *counter;   // [Hkv] split completion tickets (left at 0)
    const StepState *state;  // decode position (nullptr: use pos_fixed)
    int pos_fixed;
    uint32_t *err;
    unsigned long long *trace; // optional timeline (see GemvParams)
    int trace_slot;
    int n_heads, n_kv, head_dim, max_seq, n_splits;
    int early;               // K/V chunks per warp requested before the dependency wait (set at launch)
    float inv_sqrt_d;        // 1 / sqrt(D), as src/core/layer.rs:258 computes it
};

int attention_decode_launch(const AttnParams &p, cudaStream_t stream, bool pdl);
int attention_default_splits(int n_kv);
// set kernel attributes on the current device (once per context, outside capture)
int attention_prepare(void);
size_t attention_partials_floats(int n_heads, int head_dim, int n_splits);
// tensor map of a K cache [rows][D] as swizzled boxes of box_rows rows (see attention.cu)
int encode_k_map(CUtensorMap *map, const float *kc, int rows, int D, int box_rows);

} // namespace llmrs
