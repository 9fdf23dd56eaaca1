// attention.cu - batch-1 decode attention over the device KV cache (sm_100a).
//
// Replaces the per-head host loop of src/core/layer.rs:175-333 for seq == 1:
//   RoPE(q), RoPE(k_new) (src/backend/cpu.rs:326-357, table-driven, bit-exact),
//   append k_new / v_new at `pos` (src/core/layer.rs:219-246),
//   scores = (q . k_t) * (1/sqrt(D)), softmax, ctx = sum_t p_t v_t
//   (src/core/layer.rs:248-299).
// Native GQA: one CTA serves the n_rep query heads of a KV head, so every K/V
// row is read from HBM once (the reference replicates K/V per query head,
// src/core/loader.rs:62-98; the values are identical).
//
// Split-K (flash-decoding): grid = n_splits x n_kv.  A producer warp streams
// 32-position K and V tiles of its split into a shared-memory ring with bulk
// TMA copies; the cache rows it reads were written by earlier steps, so it
// starts before griddepcontrol.wait (the first kernel of every decode step is
// launched without programmatic overlap, so `pos` is stable for the whole
// step).  Four consumer warps take 8 positions of each tile, reduce the
// q.k partial dots with a transposing butterfly (31 shuffles per 32 dots),
// run an online softmax and accumulate V.  Split partials (m, l, acc) go to
// global memory; the last CTA of each KV head merges them in split order.
#include <mutex>

#include "attention.cuh"
#include "common.cuh"

namespace llmrs {

namespace {

constexpr int TILE = 32;   // positions per stage
constexpr int CWARPS = 4;  // consumer warps
// 3 stages for n_rep 4 (keeps ~106 KB so a PDL-prefetching GEMV CTA fits beside it); 2 for n_rep 8
template <int NREP>
struct AttnStages {
    static constexpr int value = NREP >= 8 ? 2 : 3;
};
constexpr int ATHREADS = (CWARPS + 1) * 32;

// v[j] holds lane-partial sums of 32 dot products; on return lane i holds the
// full sum of dot product i.
__device__ __forceinline__ float butterfly32(float (&v)[32], int lane)
{
#pragma unroll
    for (int w = 16; w >= 1; w >>= 1) {
        const bool upper = (lane & w) != 0;
#pragma unroll
        for (int j = 0; j < w; j++) {
            const float send = upper ? v[j] : v[j + w];
            const float keep = upper ? v[j + w] : v[j];
            v[j] = keep + __shfl_xor_sync(0xffffffffu, send, w);
        }
    }
    return v[0];
}

// rotate-half RoPE of one head held DL values per lane (lane l: dims l*DL..),
// exact reference arithmetic: x[j]*cos - x[j+mid]*sin ; x[j]*sin + x[j+mid]*cos
template <int D>
__device__ __forceinline__ void rope_lane(float (&x)[D / 32], int lane, const float *cosr, const float *sinr)
{
    constexpr int DL = D / 32;
    float other[DL];
#pragma unroll
    for (int k = 0; k < DL; k++)
        other[k] = __shfl_xor_sync(0xffffffffu, x[k], 16);
    const bool upper = lane >= 16;
#pragma unroll
    for (int k = 0; k < DL; k++) {
        const int j = (lane & 15) * DL + k; // frequency index 0..D/2-1
        const float c = cosr[j], s = sinr[j];
        if (!upper)
            x[k] = __fsub_rn(__fmul_rn(x[k], c), __fmul_rn(other[k], s));
        else
            x[k] = __fadd_rn(__fmul_rn(other[k], s), __fmul_rn(x[k], c));
    }
}

template <int D, int NREP>
__global__ void __launch_bounds__(ATHREADS) attn_decode_kernel(const AttnParams p)
{
    static_assert(NREP == 4 || NREP == 8, "n_rep must be 4 or 8");
    constexpr int NSTAGE = AttnStages<NREP>::value;
    constexpr int DL = D / 32;
    constexpr int G = 32 / NREP;          // positions per butterfly
    constexpr int NFLY = 8 / G;           // butterflies per warp per tile (8 positions)
    constexpr int ROWB = D * 4;           // bytes per cache row
    constexpr int STAGE = 2 * TILE * ROWB;
    extern __shared__ __align__(128) uint8_t smem[];
    float *kv_stage = reinterpret_cast<float *>(smem);
    float *knew = reinterpret_cast<float *>(smem + NSTAGE * STAGE);
    float *vnew = knew + D;
    float *wm = vnew + D;                       // [CWARPS][NREP]
    float *wl = wm + CWARPS * NREP;             // [CWARPS][NREP]
    float *wacc = wl + CWARPS * NREP;           // [CWARPS][NREP][D]
    uint64_t *full = reinterpret_cast<uint64_t *>(wacc + CWARPS * NREP * D);
    uint64_t *empty = full + NSTAGE;
    __shared__ unsigned int s_last;

    griddep_launch_dependents();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, g = blockIdx.y;
    const int pos = p.state ? p.state->pos : p.pos_fixed;
    const bool pos_ok = pos >= 0 && pos < p.max_seq;
    const int Lc = pos_ok ? pos : 0;           // cached positions [0, pos)
    const int t0 = (int)(((long long)split * Lc) / p.n_splits);
    const int t1 = (int)(((long long)(split + 1) * Lc) / p.n_splits);
    const int ntiles = (t1 - t0 + TILE - 1) / TILE;
    const bool owner = split == p.n_splits - 1;
    const float *kbase = p.kc + (size_t)g * p.max_seq * D;
    const float *vbase = p.vc + (size_t)g * p.max_seq * D;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NSTAGE; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CWARPS);
        }
        fence_mbar_init();
        trace_start(p.trace, p.trace_slot);
    }
    __syncthreads();

    if (warp == CWARPS) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            for (int it = 0; it < ntiles; it++) {
                const int s = it % NSTAGE;
                if (it >= NSTAGE && !mbar_wait(&empty[s], ((it / NSTAGE) - 1) & 1, p.err))
                    return;
                const int ta = t0 + it * TILE;
                const int rows = min(TILE, t1 - ta);
                mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * rows * ROWB));
                uint8_t *st = smem + (size_t)s * STAGE;
                bulk_g2s(st, kbase + (size_t)ta * D, (uint32_t)(rows * ROWB), &full[s], pol);
                bulk_g2s(st + TILE * ROWB, vbase + (size_t)ta * D, (uint32_t)(rows * ROWB), &full[s], pol);
            }
        }
        return;
    }

    // ------------------------------------------------------------ consumers
    griddep_wait();
    if (threadIdx.x == 0)
        trace_go(p.trace, p.trace_slot);
    if (!pos_ok) {
        if (threadIdx.x == 0)
            atomicCAS(p.err, 0u, (uint32_t)DEV_ERR_BAD_POS);
    }
    const float *cosr = p.rope_cos + (size_t)(pos_ok ? pos : 0) * (D / 2);
    const float *sinr = p.rope_sin + (size_t)(pos_ok ? pos : 0) * (D / 2);
    float q[NREP][DL];
#pragma unroll
    for (int h = 0; h < NREP; h++) {
        const float *qh = p.qkv + (size_t)(g * NREP + h) * D + lane * DL;
#pragma unroll
        for (int k = 0; k < DL; k++)
            q[h][k] = qh[k];
        rope_lane<D>(q[h], lane, cosr, sinr);
    }
    if (owner && warp == 0) {
        float kk[DL], vv[DL];
        const float *kn = p.qkv + (size_t)p.n_heads * D + (size_t)g * D + lane * DL;
        const float *vn = p.qkv + (size_t)(p.n_heads + p.n_kv) * D + (size_t)g * D + lane * DL;
#pragma unroll
        for (int k = 0; k < DL; k++) {
            kk[k] = kn[k];
            vv[k] = vn[k];
        }
        rope_lane<D>(kk, lane, cosr, sinr);
#pragma unroll
        for (int k = 0; k < DL; k++) {
            knew[lane * DL + k] = kk[k];
            vnew[lane * DL + k] = vv[k];
            if (pos_ok) {
                p.kc[((size_t)g * p.max_seq + pos) * D + lane * DL + k] = kk[k];
                p.vc[((size_t)g * p.max_seq + pos) * D + lane * DL + k] = vv[k];
            }
        }
    }
    named_bar_sync(1, CWARPS * 32);

    const int myh = lane % NREP; // head whose softmax state this lane tracks
    float m_run = -INFINITY, l_run = 0.0f;
    float acc[NREP][DL];
#pragma unroll
    for (int h = 0; h < NREP; h++)
#pragma unroll
        for (int k = 0; k < DL; k++)
            acc[h][k] = 0.0f;

    // one tile step over 8 positions held at krow(pp)/vrow(pp); valid(pp) masks
    auto process = [&](const float *kt, const float *vt, int nvalid) {
        float sc[NFLY];
#pragma unroll
        for (int b = 0; b < NFLY; b++) {
            float v[32];
#pragma unroll
            for (int pp = 0; pp < G; pp++) {
                const int pl = b * G + pp;
                float kr[DL];
#pragma unroll
                for (int k = 0; k < DL; k++)
                    kr[k] = pl < nvalid ? kt[pl * D + lane * DL + k] : 0.0f;
#pragma unroll
                for (int h = 0; h < NREP; h++) {
                    float d = 0.0f;
#pragma unroll
                    for (int k = 0; k < DL; k++)
                        d = fmaf(q[h][k], kr[k], d);
                    v[pp * NREP + h] = d;
                }
            }
            const float s = butterfly32(v, lane) * p.inv_sqrt_d;
            const int pl = b * G + lane / NREP;
            sc[b] = pl < nvalid ? s : -INFINITY;
        }
        // per-head max over this warp's 8 positions
        float tmax = sc[0];
#pragma unroll
        for (int b = 1; b < NFLY; b++)
            tmax = fmaxf(tmax, sc[b]);
#pragma unroll
        for (int o = NREP; o < 32; o <<= 1)
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
        const float m_new = fmaxf(m_run, tmax);
        const float corr = (m_run == -INFINITY) ? 0.0f : expf(m_run - m_new);
        float pr[NFLY];
        float psum = 0.0f;
#pragma unroll
        for (int b = 0; b < NFLY; b++) {
            pr[b] = (sc[b] == -INFINITY) ? 0.0f : expf(sc[b] - m_new);
            psum += pr[b];
        }
#pragma unroll
        for (int o = NREP; o < 32; o <<= 1)
            psum += __shfl_xor_sync(0xffffffffu, psum, o);
        l_run = l_run * corr + psum;
        m_run = m_new;
        // rescale and accumulate V for every head
#pragma unroll
        for (int h = 0; h < NREP; h++) {
            const float ch = __shfl_sync(0xffffffffu, corr, h);
#pragma unroll
            for (int k = 0; k < DL; k++)
                acc[h][k] *= ch;
        }
#pragma unroll
        for (int b = 0; b < NFLY; b++) {
#pragma unroll
            for (int pp = 0; pp < G; pp++) {
                const int pl = b * G + pp;
                if (pl < nvalid) {
                    float vr[DL];
#pragma unroll
                    for (int k = 0; k < DL; k++)
                        vr[k] = vt[pl * D + lane * DL + k];
#pragma unroll
                    for (int h = 0; h < NREP; h++) {
                        const float ph = __shfl_sync(0xffffffffu, pr[b], pp * NREP + h);
#pragma unroll
                        for (int k = 0; k < DL; k++)
                            acc[h][k] = fmaf(ph, vr[k], acc[h][k]);
                    }
                }
            }
        }
    };

    bool ok = true;
    for (int it = 0; it < ntiles; it++) {
        const int s = it % NSTAGE;
        if (ok && !mbar_wait(&full[s], (it / NSTAGE) & 1, p.err))
            ok = false;
        const int rows = min(TILE, t1 - (t0 + it * TILE));
        const float *st = kv_stage + (size_t)s * (STAGE / 4);
        const int nvalid = max(0, min(8, rows - warp * 8));
        if (nvalid > 0)
            process(st + warp * 8 * D, st + TILE * D + warp * 8 * D, nvalid);
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&empty[s]);
    }
    if (owner && warp == 0 && pos_ok)
        process(knew, vnew, 1);

    // merge the warps of this CTA
    if (lane < NREP) {
        wm[warp * NREP + lane] = m_run;
        wl[warp * NREP + lane] = l_run;
    }
#pragma unroll
    for (int h = 0; h < NREP; h++)
#pragma unroll
        for (int k = 0; k < DL; k++)
            wacc[(warp * NREP + h) * D + lane * DL + k] = acc[h][k];
    named_bar_sync(1, CWARPS * 32);
    const int ctid = threadIdx.x;
    const int PS = D + 2;
    for (int e = ctid; e < NREP * D; e += CWARPS * 32) {
        const int h = e / D, d = e % D;
        float M = -INFINITY;
        for (int w = 0; w < CWARPS; w++)
            M = fmaxf(M, wm[w * NREP + h]);
        float a = 0.0f, l = 0.0f;
        for (int w = 0; w < CWARPS; w++) {
            const float mw = wm[w * NREP + h];
            const float f = (mw == -INFINITY) ? 0.0f : expf(mw - M);
            a += wacc[(w * NREP + h) * D + d] * f;
            l += wl[w * NREP + h] * f;
        }
        float *dst = p.part + ((size_t)(g * NREP + h) * p.n_splits + split) * PS;
        dst[d] = a;
        if (d == 0) {
            dst[D] = M;
            dst[D + 1] = l;
        }
    }
    __threadfence();
    named_bar_sync(1, CWARPS * 32);
    if (ctid == 0)
        s_last = (atomicAdd(&p.counter[g], 1u) == (unsigned)(p.n_splits - 1)) ? 1u : 0u;
    named_bar_sync(1, CWARPS * 32);
    if (ctid == 0)
        trace_end(p.trace, p.trace_slot);
    if (!s_last)
        return;
    __threadfence();
    // Last CTA of this KV head: merge the splits in split order.  First every
    // (head, split) max / sum is fetched in parallel and turned into weights
    // in shared memory; then each output element sums its split partials with
    // all loads in flight together.
    float *wsplit = wacc; // reuse: [NREP][n_splits] weights, then [NREP] totals
    float *ltot = wacc + NREP * p.n_splits;
    for (int e = ctid; e < NREP * p.n_splits; e += CWARPS * 32) {
        const int h = e / p.n_splits, s = e % p.n_splits;
        const float *src = p.part + ((size_t)(g * NREP + h) * p.n_splits + s) * PS;
        wsplit[e] = __ldcg(src + D);               // m_s
        ltot[NREP + e] = __ldcg(src + D + 1);      // l_s
    }
    named_bar_sync(1, CWARPS * 32);
    if (ctid < NREP) {
        const int h = ctid;
        float M = -INFINITY;
        for (int s = 0; s < p.n_splits; s++)
            M = fmaxf(M, wsplit[h * p.n_splits + s]);
        float l = 0.0f;
        for (int s = 0; s < p.n_splits; s++) {
            const float ms = wsplit[h * p.n_splits + s];
            const float f = (ms == -INFINITY) ? 0.0f : expf(ms - M);
            l += ltot[NREP + h * p.n_splits + s] * f;
            wsplit[h * p.n_splits + s] = f;
        }
        ltot[h] = l;
    }
    named_bar_sync(1, CWARPS * 32);
    for (int e = ctid; e < NREP * D; e += CWARPS * 32) {
        const int h = e / D, d = e % D;
        const float *src = p.part + (size_t)(g * NREP + h) * p.n_splits * PS + d;
        float a = 0.0f;
        int s = 0;
        for (; s + 8 <= p.n_splits; s += 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; u++)
                v[u] = __ldcg(src + (size_t)(s + u) * PS);
#pragma unroll
            for (int u = 0; u < 8; u++)
                a += v[u] * wsplit[h * p.n_splits + s + u];
        }
        for (; s < p.n_splits; s++)
            a += __ldcg(src + (size_t)s * PS) * wsplit[h * p.n_splits + s];
        p.ctx[(size_t)(g * NREP + h) * D + d] = a / ltot[h];
    }
    if (ctid == 0) {
        p.counter[g] = 0u;
        trace_end(p.trace, p.trace_slot);
    }
}

template <int D, int NREP>
constexpr size_t attn_smem_bytes()
{
    return (size_t)AttnStages<NREP>::value * (2 * TILE * D * 4) +
           (size_t)(2 * D + 2 * CWARPS * NREP + CWARPS * NREP * D) * 4 + 2 * AttnStages<NREP>::value * 8;
}

template <int D, int NREP>
int launch_attn(const AttnParams &p, cudaStream_t stream, bool pdl)
{
    const size_t smem = attn_smem_bytes<D, NREP>();
    LLMRS_CUDA_TRY(launch(attn_decode_kernel<D, NREP>, dim3(p.n_splits, p.n_kv), dim3(ATHREADS), smem, stream, pdl, p));
    return LLMRS_OK;
}

template <int D, int NREP>
cudaError_t prepare_attn()
{
    return cudaFuncSetAttribute(attn_decode_kernel<D, NREP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)attn_smem_bytes<D, NREP>());
}

} // namespace

int attention_prepare(void)
{
    cudaError_t e = prepare_attn<128, 4>();
    if (e == cudaSuccess)
        e = prepare_attn<128, 8>();
    if (e == cudaSuccess)
        e = prepare_attn<64, 4>();
    if (e == cudaSuccess)
        e = prepare_attn<64, 8>();
    if (e != cudaSuccess)
        return fail(LLMRS_ECUDA, "attention kernel attributes: %s", cudaGetErrorString(e));
    return LLMRS_OK;
}

int attention_default_splits(int n_kv)
{
    int s = (144 + n_kv - 1) / n_kv;
    return s < 1 ? 1 : (s > 32 ? 32 : s);
}

size_t attention_partials_floats(int n_heads, int head_dim, int n_splits)
{
    return (size_t)n_heads * n_splits * (head_dim + 2);
}

int attention_decode_launch(const AttnParams &p, cudaStream_t stream, bool pdl)
{
    LLMRS_CHECK_ARG(p.n_kv > 0 && p.n_heads % p.n_kv == 0, "attention: n_heads %d not a multiple of n_kv %d",
                    p.n_heads, p.n_kv);
    const int nrep = p.n_heads / p.n_kv;
    if (p.head_dim == 128 && nrep == 4)
        return launch_attn<128, 4>(p, stream, pdl);
    if (p.head_dim == 128 && nrep == 8)
        return launch_attn<128, 8>(p, stream, pdl);
    if (p.head_dim == 64 && nrep == 4)
        return launch_attn<64, 4>(p, stream, pdl);
    if (p.head_dim == 64 && nrep == 8)
        return launch_attn<64, 8>(p, stream, pdl);
    return fail(LLMRS_ENOTSUP, "attention: head_dim %d with n_rep %d not supported", p.head_dim, nrep);
}

// ----------------------------------------------------------------------------
// Allocation-free variant.  Some callers cannot allocate device memory: their
// device memory belongs to another allocator that must account for every byte
// (a serving runtime's pre-reserved pool), or they must not allocate after
// start-up, or they cannot create an llmrs_ctx (which allocates).  For them
// the split partials, the KV-head tickets and an error word live in this fixed
// array, linked into the library: every GPU that loads the library holds it
// until the process exits.
constexpr size_t NOALLOC_HEADER = 1024;                        // tickets + error word
constexpr size_t NOALLOC_BYTES = NOALLOC_HEADER + (2u << 20);  // + 2 MiB of split partials
constexpr int NOALLOC_MAX_KV = 128;                            // tickets that fit the header
static __device__ __align__(256) unsigned char g_attn_scratch[NOALLOC_BYTES];

namespace {
std::mutex g_noalloc_mu;
unsigned char *g_noalloc_ptr[256];   // device address of g_attn_scratch, per device
bool g_noalloc_ready[256];

// Once per device, with that device current: resolve the array's device
// address (the host-side name is only a stand-in) and set kernel attributes.
int noalloc_setup(int device, unsigned char **out)
{
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (device < 0 || device >= 256)
        return fail(LLMRS_EINVAL, "device ordinal %d out of range", device);
    if (!g_noalloc_ready[device]) {
        unsigned char *ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress((void **)&ptr, g_attn_scratch);
        if (e != cudaSuccess)
            return fail(LLMRS_ECUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
        LLMRS_TRY(attention_prepare());
        g_noalloc_ptr[device] = ptr;
        g_noalloc_ready[device] = true;
    }
    *out = g_noalloc_ptr[device];
    return LLMRS_OK;
}
} // namespace

} // namespace llmrs

using namespace llmrs;

extern "C" int llmrs_attention_decode_noalloc(void *cuda_stream, const float *d_qkv, float *d_kcache,
                                              float *d_vcache, const float *d_rope_cos, const float *d_rope_sin,
                                              float *d_out, int n_heads, int n_kv_heads, int head_dim, int max_seq,
                                              int pos, unsigned int *d_err)
{
    LLMRS_CHECK_ARG(d_qkv && d_kcache && d_vcache && d_rope_cos && d_rope_sin && d_out, "NULL argument");
    LLMRS_CHECK_ARG(n_kv_heads > 0 && n_heads > 0 && n_heads % n_kv_heads == 0, "bad head counts %d/%d", n_heads,
                    n_kv_heads);
    LLMRS_CHECK_ARG(max_seq > 0 && pos >= 0 && pos < max_seq, "position %d outside [0,%d)", pos, max_seq);
    const int n_splits = attention_default_splits(n_kv_heads);
    const size_t part_bytes = attention_partials_floats(n_heads, head_dim, n_splits) * sizeof(float);
    LLMRS_CHECK_ARG(n_kv_heads <= NOALLOC_MAX_KV,
                    "attention_decode_noalloc: %d KV heads exceed the fixed scratch limit of %d", n_kv_heads,
                    NOALLOC_MAX_KV);
    LLMRS_CHECK_ARG(part_bytes <= NOALLOC_BYTES - NOALLOC_HEADER,
                    "attention_decode_noalloc: %zu bytes of split partials exceed the fixed scratch of %zu bytes "
                    "(%d heads x %d splits x head_dim %d)",
                    part_bytes, (size_t)(NOALLOC_BYTES - NOALLOC_HEADER), n_heads, n_splits, head_dim);
    int device = 0;
    LLMRS_CUDA_TRY(cudaGetDevice(&device));
    unsigned char *scratch = nullptr;
    LLMRS_TRY(noalloc_setup(device, &scratch));
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(cuda_stream);
    unsigned int *tickets = reinterpret_cast<unsigned int *>(scratch);
    unsigned int *own_err = tickets + NOALLOC_MAX_KV;
    // tickets must start at zero (a previous call that was cut short may have left counts)
    LLMRS_CUDA_TRY(cudaMemsetAsync(tickets, 0, (size_t)(NOALLOC_MAX_KV + 1) * sizeof(unsigned int), stream));
    AttnParams a{};
    a.n_heads = n_heads;
    a.n_kv = n_kv_heads;
    a.head_dim = head_dim;
    a.max_seq = max_seq;
    a.n_splits = n_splits;
    a.pos_fixed = pos;
    a.qkv = d_qkv;
    a.kc = d_kcache;
    a.vc = d_vcache;
    a.rope_cos = d_rope_cos;
    a.rope_sin = d_rope_sin;
    a.ctx = d_out;
    a.err = d_err ? d_err : own_err;
    a.inv_sqrt_d = 1.0f / sqrtf((float)head_dim);
    a.part = reinterpret_cast<float *>(scratch + NOALLOC_HEADER);
    a.counter = tickets;
    return attention_decode_launch(a, stream, false);
}

