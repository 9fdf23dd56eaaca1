// prefetch.cuh - L2 prefetch of the next decode-step kernel's first bytes.
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace llmrs {

__device__ __forceinline__ void prefetch_next_cta(const NextPrefetch &pf, int j);

// Called by one thread of CTA j (of ncur) of the current kernel after its own
// bulk copies are requested (they stay ahead in the memory queues); covers the
// next kernel's CTAs j, j + ncur, ...
__device__ __forceinline__ void issue_next_prefetch(const NextPrefetch &pf, int j, int ncur)
{
    if (pf.kind == PF_NONE)
        return;
    for (; j < pf.ncta; j += ncur)
        prefetch_next_cta(pf, j);
}

__device__ __forceinline__ void prefetch_next_cta(const NextPrefetch &pf, int j)
{
    if (pf.kind == PF_ROWS) {
        const size_t a0 = (size_t)j * pf.a_stride, b0 = (size_t)j * pf.b_stride;
        if (a0 < pf.a_end)
            prefetch_l2_range(pf.a + a0, min(pf.a_bytes, pf.a_end - a0));
        if (pf.b && b0 < pf.b_end)
            prefetch_l2_range(pf.b + b0, min(pf.b_bytes, pf.b_end - b0));
        return;
    }
    // PF_KV: the cached rows [t0, t1) of split s of KV head g, as the
    // attention kernel splits them
    const int s = j % pf.n_splits, g = j / pf.n_splits;
    const int pos = pf.state ? pf.state->pos : 0;
    if (pos <= 0 || pos >= pf.max_seq)
        return;
    const int t0 = (int)(((long long)s * pos) / pf.n_splits);
    const int t1 = (int)(((long long)(s + 1) * pos) / pf.n_splits);
    const size_t row = (size_t)pf.head_dim * 4;
    const size_t off = ((size_t)g * pf.max_seq + t0) * row;
    const size_t n = min((size_t)(t1 - t0) * row, pf.kv_bytes);
    prefetch_l2_range(reinterpret_cast<const uint8_t *>(pf.kc) + off, n);
    prefetch_l2_range(reinterpret_cast<const uint8_t *>(pf.vc) + off, n);
}

} // namespace llmrs
