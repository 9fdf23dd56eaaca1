// sample.cu - device-side sampling of the next token (src/main.rs:192-305):
// repetition penalty over the recent ids, temperature, softmax, then top-p
// (nucleus) or plain roulette selection with a caller-supplied uniform draw.
//
// Reference order of operations, restated:
//   1. for each distinct id in the recent window: l = l < 0 ? l * penalty : l / penalty
//      (only when penalty > 1)
//   2. if |temperature - 1| > 1e-6: l /= temperature
//   3. m = max l (from f32::MIN); e = exp(l - m); s = sum e; p = e / s
//   4a. top_p < 1: candidates p > 1e-5 (all if none), sorted by p descending;
//       cutoff = first i with running sum > top_p (else the last); total = sum of
//       candidates 0..=cutoff; r = u * total; walk r -= p, pick the first with
//       r <= 0 (else candidate 0)
//   4b. otherwise: r = u; walk every id in order, r -= p, pick the first with
//       r <= 0 (else id 0)
// The reference draws u from an OS-seeded generator (rand::rng()); here the
// caller supplies it, so runs are reproducible.  The sum in step 3 is a tree
// here and CUDA's expf differs from libm's by an ulp at times, so
// probabilities agree to rounding; the walk can pick a neighbour only when
// the draw falls within that rounding of a cumulative boundary.  Ties in p
// (unordered by the reference's unstable sort) go to the lower id.
#include <cuda_runtime.h>
#include <float.h>
#include <math.h>
#include <stdint.h>

#include "common.cuh"
#include "sample.cuh"

namespace llmrs {

namespace {

constexpr int SM_THREADS = 1024;
constexpr int SM_CAND_SMEM = 4096; // candidates sorted in shared memory; more go through global memory

struct SampleState {
    float max_l, sum_e;
    unsigned int n_cand;
    int token;
};

__device__ __forceinline__ float block_reduce_max(float v, float *red)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_max(v);
    if (lane == 0)
        red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < (int)(blockDim.x >> 5) ? red[lane] : -FLT_MAX;
        v = warp_max(v);
        if (lane == 0)
            red[32] = v;
    }
    __syncthreads();
    const float r = red[32];
    __syncthreads();
    return r;
}

__device__ __forceinline__ float block_reduce_sum(float v, float *red)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    if (lane == 0)
        red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
        v = warp_sum(v);
        if (lane == 0)
            red[32] = v;
    }
    __syncthreads();
    const float r = red[32];
    __syncthreads();
    return r;
}

// steps 1-3 (+ candidate compaction for top-p): one CTA over the vocabulary
__global__ void __launch_bounds__(SM_THREADS) sample_probs_kernel(const float *logits, int V, const int *recent,
                                                                  int n_recent, float penalty, float temperature,
                                                                  float top_p, float *probs, float2 *cand,
                                                                  SampleState *st)
{
    __shared__ float red[33];
    for (int i = threadIdx.x; i < V; i += blockDim.x)
        probs[i] = logits[i];
    __syncthreads();
    if (penalty > 1.0f)
        for (int j = threadIdx.x; j < n_recent; j += blockDim.x) {
            const int id = recent[j];
            bool first = id >= 0 && id < V;
            for (int k = 0; k < j && first; k++)
                first = recent[k] != id; // each distinct id once (a set, like the reference)
            if (first) {
                const float s = probs[id];
                probs[id] = s < 0.0f ? __fmul_rn(s, penalty) : __fdiv_rn(s, penalty);
            }
        }
    __syncthreads();
    const bool scale = fabsf(temperature - 1.0f) > 1e-6f;
    float mx = -FLT_MAX;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        float l = probs[i];
        if (scale) {
            l = __fdiv_rn(l, temperature);
            probs[i] = l;
        }
        mx = fmaxf(mx, l);
    }
    mx = block_reduce_max(mx, red);
    float s = 0.0f;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float e = expf(__fsub_rn(probs[i], mx));
        probs[i] = e;
        s = __fadd_rn(s, e);
    }
    s = block_reduce_sum(s, red);
    if (threadIdx.x == 0) {
        st->max_l = mx;
        st->sum_e = s;
        st->n_cand = 0u;
        st->token = 0;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float p = __fdiv_rn(probs[i], s);
        probs[i] = p;
        if (top_p < 1.0f && p > 1e-5f) {
            const unsigned int k = atomicAdd(&st->n_cand, 1u);
            cand[k] = make_float2(p, __int_as_float(i));
        }
    }
}

// descending p, ties to the lower id
__device__ __forceinline__ bool cand_before(float2 a, float2 b)
{
    return a.x > b.x || (a.x == b.x && __float_as_int(a.y) < __float_as_int(b.y));
}

// the nucleus walk over sorted candidates (one thread)
__device__ __forceinline__ int nucleus_pick(const float2 *c, int n, float top_p, float u)
{
    float cum = 0.0f;
    int cut = n - 1;
    for (int i = 0; i < n; i++) {
        cum = __fadd_rn(cum, c[i].x);
        if (cum > top_p) {
            cut = i;
            break;
        }
    }
    float total = 0.0f;
    for (int i = 0; i <= cut; i++)
        total = __fadd_rn(total, c[i].x);
    float r = __fmul_rn(u, total);
    int tok = __float_as_int(c[0].y);
    for (int i = 0; i <= cut; i++) {
        r = __fsub_rn(r, c[i].x);
        if (r <= 0.0f) {
            tok = __float_as_int(c[i].y);
            break;
        }
    }
    return tok;
}

// top-p with <= SM_CAND_SMEM candidates: bitonic sort in shared memory, then the walk
__global__ void __launch_bounds__(SM_THREADS) sample_nucleus_kernel(const float2 *cand, const SampleState *st_in,
                                                                    float top_p, float u, SampleState *st)
{
    __shared__ float2 c[SM_CAND_SMEM];
    const int n = (int)st_in->n_cand;
    int np = 1;
    while (np < n)
        np <<= 1;
    for (int i = threadIdx.x; i < np; i += blockDim.x)
        c[i] = i < n ? cand[i] : make_float2(-1.0f, __int_as_float(0x7fffffff));
    __syncthreads();
    for (int k = 2; k <= np; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < np; i += blockDim.x) {
                const int l = i ^ j;
                if (l > i) {
                    const bool up = (i & k) == 0; // this run sorts in "before" order
                    const float2 a = c[i], b = c[l];
                    if (up ? cand_before(b, a) : cand_before(a, b)) {
                        c[i] = b;
                        c[l] = a;
                    }
                }
            }
            __syncthreads();
        }
    if (threadIdx.x == 0)
        st->token = nucleus_pick(c, n, top_p, u);
}

// one compare-exchange step of a bitonic sort over np (power of two) global entries
__global__ void sample_bitonic_step(float2 *c, int np, int j, int k)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= np)
        return;
    const int l = i ^ j;
    if (l > i) {
        const bool up = (i & k) == 0;
        const float2 a = c[i], b = c[l];
        if (up ? cand_before(b, a) : cand_before(a, b)) {
            c[i] = b;
            c[l] = a;
        }
    }
}

__global__ void sample_pad_kernel(float2 *c, const float *probs, int n, int np, int all)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= np)
        return;
    if (all && i < n)
        c[i] = make_float2(probs[i], __int_as_float(i));
    else if (i >= n)
        c[i] = make_float2(-1.0f, __int_as_float(0x7fffffff));
}

__global__ void sample_walk_kernel(const float2 *c, int n, float top_p, float u, SampleState *st)
{
    st->token = nucleus_pick(c, n, top_p, u);
}

// plain roulette: chunk sums, the chunk where the running draw crosses zero,
// then the walk inside it
__global__ void __launch_bounds__(SM_THREADS) sample_roulette_kernel(const float *probs, int V, float u,
                                                                     SampleState *st)
{
    __shared__ float part[SM_THREADS];
    __shared__ int s_chunk;
    __shared__ float s_r;
    const int per = (V + blockDim.x - 1) / blockDim.x;
    const int i0 = threadIdx.x * per, i1 = min(V, i0 + per);
    float s = 0.0f;
    for (int i = i0; i < i1; i++)
        s = __fadd_rn(s, probs[i]);
    part[threadIdx.x] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float r = u;
        int ch = -1;
        for (int t = 0; t < (int)blockDim.x; t++) {
            if (__fsub_rn(r, part[t]) <= 0.0f) {
                ch = t;
                break;
            }
            r = __fsub_rn(r, part[t]);
        }
        s_chunk = ch;
        s_r = r;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int tok = 0;
        const int ch = s_chunk;
        if (ch >= 0) {
            float r = s_r;
            const int a = ch * per, b = min(V, a + per);
            tok = b - 1;
            for (int i = a; i < b; i++) {
                r = __fsub_rn(r, probs[i]);
                if (r <= 0.0f) {
                    tok = i;
                    break;
                }
            }
        }
        st->token = tok;
    }
}

} // namespace

size_t sample_scratch_bytes(int V)
{
    int np = 1;
    while (np < V)
        np <<= 1;
    return ((size_t)V * 4 + 255) / 256 * 256 + (size_t)np * 8 + 256 + (size_t)SAMPLE_MAX_RECENT * 4;
}

int sample_launch(const float *d_logits, int V, const int *h_recent, int n_recent, float penalty, float temperature,
                  float top_p, float u, void *scratch, int *h_token, cudaStream_t stream)
{
    LLMRS_CHECK_ARG(d_logits && V > 0 && scratch && h_token, "sample: bad arguments");
    LLMRS_CHECK_ARG(n_recent >= 0 && n_recent <= SAMPLE_MAX_RECENT && (n_recent == 0 || h_recent),
                    "sample: %d recent ids (at most %d)", n_recent, SAMPLE_MAX_RECENT);
    LLMRS_CHECK_ARG(temperature > 0.0f && u >= 0.0f && u < 1.0f, "sample: temperature must be > 0, u in [0, 1)");
    int np = 1;
    while (np < V)
        np <<= 1;
    uint8_t *b = reinterpret_cast<uint8_t *>(scratch);
    float *probs = reinterpret_cast<float *>(b);
    float2 *cand = reinterpret_cast<float2 *>(b + ((size_t)V * 4 + 255) / 256 * 256);
    SampleState *st = reinterpret_cast<SampleState *>(reinterpret_cast<uint8_t *>(cand) + (size_t)np * 8);
    int *recent = reinterpret_cast<int *>(reinterpret_cast<uint8_t *>(st) + 256);
    if (n_recent)
        LLMRS_CUDA_TRY(cudaMemcpyAsync(recent, h_recent, (size_t)n_recent * 4, cudaMemcpyHostToDevice, stream));
    sample_probs_kernel<<<1, SM_THREADS, 0, stream>>>(d_logits, V, recent, n_recent, penalty, temperature, top_p, probs,
                                                     cand, st);
    LLMRS_CUDA_TRY(cudaGetLastError());
    if (top_p < 1.0f) {
        SampleState h{};
        LLMRS_CUDA_TRY(cudaMemcpyAsync(&h, st, sizeof(h), cudaMemcpyDeviceToHost, stream));
        LLMRS_CUDA_TRY(cudaStreamSynchronize(stream));
        int n = (int)h.n_cand;
        if (n >= 1 && n <= SM_CAND_SMEM) {
            sample_nucleus_kernel<<<1, SM_THREADS, 0, stream>>>(cand, st, top_p, u, st);
        } else { // many (or no) candidates: sort in global memory
            const int all = n == 0;
            if (all)
                n = V; // every probability is a candidate, like the reference
            int npn = 1;
            while (npn < n)
                npn <<= 1;
            const int thr = 256, blocks = (npn + thr - 1) / thr;
            sample_pad_kernel<<<blocks, thr, 0, stream>>>(cand, probs, n, npn, all);
            for (int k = 2; k <= npn; k <<= 1)
                for (int j = k >> 1; j > 0; j >>= 1)
                    sample_bitonic_step<<<blocks, thr, 0, stream>>>(cand, npn, j, k);
            sample_walk_kernel<<<1, 1, 0, stream>>>(cand, n, top_p, u, st);
        }
    } else {
        sample_roulette_kernel<<<1, SM_THREADS, 0, stream>>>(probs, V, u, st);
    }
    LLMRS_CUDA_TRY(cudaGetLastError());
    LLMRS_CUDA_TRY(cudaMemcpyAsync(h_token, &st->token, sizeof(int), cudaMemcpyDeviceToHost, stream));
    LLMRS_CUDA_TRY(cudaStreamSynchronize(stream));
    return LLMRS_OK;
}

} // namespace llmrs
