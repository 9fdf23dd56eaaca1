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
// Split-K (flash-decoding): grid = n_splits x n_kv, one CTA per SM.  Each of
// the CTA's 12 (D = 128) or 16 (D = 64) warps owns every NW-th 8-position
// chunk of the split and a private 2-slot shared-memory ring that its lane 0
// fills with bulk copies of K and V rows; the cached rows were written by
// earlier steps, so the first two chunks per warp are requested before
// griddepcontrol.wait (the first kernel of every decode step is launched
// without programmatic overlap, so `pos` is stable for the whole step).  A
// warp reduces the q.k partial dots of a chunk with a transposing butterfly
// (31 shuffles per 32 dots), runs an online softmax and accumulates V; the
// warps of a CTA merge through shared memory, split partials (m, l, acc) go
// to global memory, and the last CTA of each KV head merges them in split
// order.
#include <stdlib.h>
#include <mutex>

#include "attention.cuh"
#include "attention_core.cuh"
#include "common.cuh"

namespace llmrs {

namespace {

constexpr int CH = 8; // positions per chunk: one warp's unit of work

// Phase marks for an instrumented build (no-ops here): 0 entry, 1 q staged,
// 2 first chunk landed, 3 chunk loop done, 4 warps merged, 5 ticket taken,
// 6 split merge done, 7 last warp's loop done.
#ifndef LLMRS_ATTN_MARK
#define LLMRS_ATTN_MARK(ev)
#define LLMRS_ATTN_MARK_MAX(ev)
#endif

// Consumer warps per CTA.  Each warp owns a private 2-slot ring of CH-position
// K|V chunks (loaded by its own lane 0 with bulk copies, one mbarrier per
// slot), so warps never wait on each other until the end-of-split merge and
// a slot's barrier is only ever awaited by the warp that consumed its
// previous phase (no parity aliasing).  The ring fills the shared memory:
// 12 warps x 2 x 8 KB at D = 128, 16 x 2 x 4 KB at D = 64.
template <int D>
struct AttnWarps {
    static constexpr int value = D >= 128 ? 12 : 16;
};

template <int D, int NREP>
struct AttnLayout {
    static constexpr int NW = AttnWarps<D>::value;
    static constexpr int ROWB = D * 4;           // bytes per cache row
    static constexpr int KBYTES = CH * ROWB;     // swizzled K box (multiple of 1024)
    static constexpr int SLOT = 2 * KBYTES;      // K box, then CH plain V rows
    static constexpr int RING = 2 * SLOT;        // per warp
    static constexpr int QS = D + 4;             // padded q row: NREP heads in distinct banks
    static constexpr size_t q_off = (size_t)NW * RING;                        // [NREP][QS]
    static constexpr size_t probs_off = q_off + (size_t)NREP * QS * 4;        // [NW][CH*NREP]
    static constexpr size_t wm_off = probs_off + (size_t)NW * CH * NREP * 4; // [NW][NREP]
    static constexpr size_t wl_off = wm_off + (size_t)NW * NREP * 4;        // [NW][NREP]
    static constexpr size_t fw_off = wl_off + (size_t)NW * NREP * 4;        // [NW][NREP]
    static constexpr size_t tot_off = fw_off + (size_t)NW * NREP * 4;       // [2][NREP]
    static constexpr size_t bar_off = (tot_off + 2 * NREP * 4 + 7) / 8 * 8; // [NW][2]
    static constexpr size_t merge_bar_off = bar_off + (size_t)NW * 2 * 8;
    static constexpr size_t bytes = merge_bar_off + 8 + 1024; // + 1024-byte alignment slack
    static_assert(NREP * D * 4 <= RING, "a warp's partial accumulator must fit its ring");
    static_assert(KBYTES % 1024 == 0 && CH == 8, "swizzled K boxes must stay 1024-byte aligned");
};

template <int D, int NREP>
__global__ void __launch_bounds__(AttnWarps<D>::value * 32, 1) attn_decode_kernel(const __grid_constant__ AttnParams p)
{
    static_assert(NREP == 4 || NREP == 8, "n_rep must be 4 or 8");
    using Lay = AttnLayout<D, NREP>;
    constexpr int NW = Lay::NW;
    constexpr int NT = NW * 32;
    constexpr int DL = D / 32;
    constexpr int ROWB = Lay::ROWB;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    float *q_s = reinterpret_cast<float *>(smem + Lay::q_off);
    float *wm = reinterpret_cast<float *>(smem + Lay::wm_off);
    float *wl = reinterpret_cast<float *>(smem + Lay::wl_off);
    float *fw = reinterpret_cast<float *>(smem + Lay::fw_off);
    float *tot = reinterpret_cast<float *>(smem + Lay::tot_off);
    __shared__ unsigned int s_last;

    griddep_launch_dependents();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = blockIdx.x, g = blockIdx.y;
    LLMRS_ATTN_MARK(0);
    // `pos` was written by the previous step's last kernel, which finished
    // before this step's first (non-overlapped) kernel began
    const int pos = p.state ? p.state->pos : p.pos_fixed;
    const bool pos_ok = pos >= 0 && pos < p.max_seq;
    const int Lc = pos_ok ? pos : 0;           // cached positions [0, pos)
    const int t0 = (int)(((long long)split * Lc) / p.n_splits);
    const int t1 = (int)(((long long)(split + 1) * Lc) / p.n_splits);
    const int nch = (t1 - t0 + CH - 1) / CH;
    const int mine = warp < nch ? (nch - warp + NW - 1) / NW : 0; // chunks warp, warp+NW, ...
    const bool owner = split == p.n_splits - 1;
    const float *vbase = p.vc + (size_t)g * p.max_seq * D;
    uint8_t *ring = smem + (size_t)warp * Lay::RING;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + Lay::bar_off) + warp * 2;
    uint64_t *merge_bar = reinterpret_cast<uint64_t *>(smem + Lay::merge_bar_off);
    float *probs = reinterpret_cast<float *>(smem + Lay::probs_off) + warp * CH * NREP;

    auto issue = [&](int j, uint64_t pol) { // chunk j of this warp into slot j & 1 (lane 0)
        const int ta = t0 + (warp + j * NW) * CH;
        const int rows = min(CH, t1 - ta);
        uint64_t *bar = &full[j & 1];
        uint8_t *dst = ring + (j & 1) * Lay::SLOT;
        // the K box always moves CH rows (rows past the split are ignored;
        // past the end of the cache they read as zero)
        mbar_arrive_expect_tx(bar, (uint32_t)(Lay::KBYTES + rows * ROWB));
        tma_load_3d(dst, &p.tk, 0, g * p.max_seq + ta, 0, bar, pol);
        bulk_g2s(dst + Lay::KBYTES, vbase + (size_t)ta * D, (uint32_t)(rows * ROWB), bar, pol);
    };
    if (lane == 0) {
        mbar_init(&full[0], 1);
        mbar_init(&full[1], 1);
        if (threadIdx.x == 0) {
            mbar_init(merge_bar, 1);
            trace_start(p.trace, p.trace_slot);
        }
        fence_mbar_init();
        // K/V rows of the cached positions [0, pos) were written by earlier
        // steps, not by the kernel this one may overlap: the first chunks
        // stream before the dependency wait
        for (int j = 0; j < p.early && j < 2 && j < mine; j++)
            issue(j, policy_evict_first());
    }

    griddep_wait();
    if (threadIdx.x == 0) {
        trace_go(p.trace, p.trace_slot);
        if (!pos_ok)
            atomicCAS(p.err, 0u, (uint32_t)DEV_ERR_BAD_POS);
    }
    // The few small loads (q, the new k/v, the RoPE row) are issued before
    // the K/V stream: queued behind it they would wait for most of it.
    const float *cosr = p.rope_cos + (size_t)Lc * (D / 2);
    const float *sinr = p.rope_sin + (size_t)Lc * (D / 2);
    const bool appender = owner && warp == 0;
    float qv[DL], kk[DL], vv[DL], rc[DL], rs[DL];
    if (warp < NREP || appender)
        rope_table_lane<D>(rc, rs, lane, cosr, sinr);
    if (warp < NREP) {
        const float *qh = p.qkv + (size_t)(g * NREP + warp) * D + lane * DL;
#pragma unroll
        for (int k = 0; k < DL; k++)
            qv[k] = qh[k];
    }
    if (appender) {
        const float *kn = p.qkv + (size_t)p.n_heads * D + (size_t)g * D + lane * DL;
        const float *vn = p.qkv + (size_t)(p.n_heads + p.n_kv) * D + (size_t)g * D + lane * DL;
#pragma unroll
        for (int k = 0; k < DL; k++) {
            kk[k] = kn[k];
            vv[k] = vn[k];
        }
    }
    __syncthreads(); // small loads issued; barriers initialised
    if (lane == 0) {
        const uint64_t pol = policy_evict_first();
        for (int j = p.early < 0 ? 0 : p.early; j < 2 && j < mine; j++)
            issue(j, pol);
    }
    __syncwarp();
    if (warp < NREP) { // RoPE(q) of head `warp` into shared memory
        rope_lane<D>(qv, lane, rc, rs);
#pragma unroll
        for (int k = 0; k < DL; k++)
            q_s[warp * Lay::QS + lane * DL + k] = qv[k];
    }
    if (appender) { // RoPE the new key, append k/v at `pos`
        rope_lane<D>(kk, lane, rc, rs);
        if (pos_ok) {
#pragma unroll
            for (int k = 0; k < DL; k++) {
                p.kc[((size_t)g * p.max_seq + pos) * D + lane * DL + k] = kk[k];
                p.vc[((size_t)g * p.max_seq + pos) * D + lane * DL + k] = vv[k];
            }
        }
    }
    __syncthreads(); // q_s complete
    LLMRS_ATTN_MARK(1);
    if (threadIdx.x == 0)
        trace_ready(p.trace, p.trace_slot);

    float m_run = -INFINITY, l_run = 0.0f; // softmax state of head lane % NREP
    float acc[NREP][DL];
#pragma unroll
    for (int h = 0; h < NREP; h++)
#pragma unroll
        for (int k = 0; k < DL; k++)
            acc[h][k] = 0.0f;

    bool ok = true;
    for (int j = 0; j < mine; j++) {
        const int slot = j & 1;
        if (ok && !mbar_wait(&full[slot], (uint32_t)((j >> 1) & 1), p.err))
            ok = false;
        if (j == 0)
            LLMRS_ATTN_MARK(2);
        if (ok) {
            const int rows = min(CH, t1 - (t0 + (warp + j * NW) * CH));
            const float *st = reinterpret_cast<const float *>(ring + slot * Lay::SLOT);
            attn_chunk<D, NREP, CH>(st, 0, st + Lay::KBYTES / 4, rows, q_s, Lay::QS, probs, p.inv_sqrt_d, m_run,
                                    l_run, acc, lane);
        }
        if (ok && lane == 0 && j + 2 < mine) {
            fence_proxy_async_smem(); // this warp's reads of the slot precede the refill
            issue(j + 2, policy_evict_first());
        }
    }
    LLMRS_ATTN_MARK(3);
    LLMRS_ATTN_MARK_MAX(7);
    if (appender && pos_ok) {
        // the new position, staged as plain rows in this warp's (now idle) first slot
        float *st = reinterpret_cast<float *>(ring);
#pragma unroll
        for (int k = 0; k < DL; k++) {
            st[lane * DL + k] = kk[k];
            st[D + lane * DL + k] = vv[k];
        }
        __syncwarp();
        attn_new_position<D, NREP>(st, st + D, q_s, Lay::QS, p.inv_sqrt_d, m_run, l_run, acc, lane);
        __syncwarp();
    }

    // merge the warps of this CTA: warp partials at the start of each ring
    float *wacc = reinterpret_cast<float *>(ring);
    if (lane < NREP) {
        wm[warp * NREP + lane] = m_run;
        wl[warp * NREP + lane] = l_run;
    }
#pragma unroll
    for (int h = 0; h < NREP; h++)
#pragma unroll
        for (int k = 0; k < DL; k++)
            wacc[h * D + lane * DL + k] = acc[h][k];
    __syncthreads();
    LLMRS_ATTN_MARK(4);
    const int ctid = threadIdx.x;
    if (ctid < NREP) {
        const int h = ctid;
        float M = -INFINITY;
        for (int w = 0; w < NW; w++)
            M = fmaxf(M, wm[w * NREP + h]);
        float l = 0.0f;
        for (int w = 0; w < NW; w++) {
            const float mw = wm[w * NREP + h];
            const float f = (mw == -INFINITY) ? 0.0f : expf(mw - M);
            fw[w * NREP + h] = f;
            l += wl[w * NREP + h] * f;
        }
        tot[h] = M;
        tot[NREP + h] = l;
    }
    __syncthreads();
    const int PS = D + 2;
    for (int e = ctid; e < NREP * D; e += NT) {
        const int h = e / D, d = e % D;
        float a = 0.0f;
#pragma unroll 4
        for (int w = 0; w < NW; w++)
            a += reinterpret_cast<const float *>(smem + (size_t)w * Lay::RING)[h * D + d] * fw[w * NREP + h];
        float *dst = p.part + ((size_t)(g * NREP + h) * p.n_splits + split) * PS;
        dst[d] = a;
        if (d == 0) {
            dst[D] = tot[h];
            dst[D + 1] = tot[NREP + h];
        }
    }
    __threadfence();
    __syncthreads();
    if (ctid == 0)
        s_last = (atomicAdd(&p.counter[g], 1u) == (unsigned)(p.n_splits - 1)) ? 1u : 0u;
    __syncthreads();
    LLMRS_ATTN_MARK(5);
    if (ctid == 0)
        trace_end(p.trace, p.trace_slot);
    if (!s_last)
        return;
    __threadfence();
    // Last CTA of this KV head: one bulk copy brings every split partial of
    // its NREP heads ([NREP][n_splits][D + 2], contiguous) into shared memory
    // (the ring is idle now); the splits are then merged in split order.
    const int ns = p.n_splits;
    float *pm = reinterpret_cast<float *>(smem); // [NREP][ns][PS]
    float *wsplit = pm + NREP * ns * PS;         // [NREP][ns] split weights
    float *ltot = wsplit + NREP * ns;            // [NREP] softmax denominators
    if (ctid == 0) {
        // the partials were written through the generic proxy by other CTAs
        asm volatile("fence.proxy.async.global;" ::: "memory");
        const uint32_t bytes = (uint32_t)(NREP * ns * PS * 4);
        mbar_arrive_expect_tx(merge_bar, bytes);
        bulk_g2s(pm, p.part + (size_t)g * NREP * ns * PS, bytes, merge_bar, policy_evict_first());
    }
    const bool got = mbar_wait(merge_bar, 0, p.err);
    if (warp < NREP && got) { // head `warp`: max over splits, weights, denominator
        const int h = warp;
        float M = -INFINITY;
        for (int sp = lane; sp < ns; sp += 32)
            M = fmaxf(M, pm[(h * ns + sp) * PS + D]);
        M = warp_max(M);
        float l = 0.0f;
        for (int sp = lane; sp < ns; sp += 32) {
            const float ms = pm[(h * ns + sp) * PS + D];
            const float f = (ms == -INFINITY) ? 0.0f : expf(ms - M);
            wsplit[h * ns + sp] = f;
            l += pm[(h * ns + sp) * PS + D + 1] * f;
        }
        l = warp_sum(l);
        if (lane == 0)
            ltot[h] = l;
    }
    __syncthreads();
    for (int e = ctid; e < NREP * D && got; e += NT) {
        const int h = e / D, d = e % D;
        const float *src = pm + (size_t)h * ns * PS + d;
        float a = 0.0f;
        for (int sp = 0; sp < ns; sp++)
            a += src[(size_t)sp * PS] * wsplit[h * ns + sp];
        p.ctx[(size_t)(g * NREP + h) * D + d] = a / ltot[h];
    }
    if (ctid == 0) {
        p.counter[g] = 0u;
        trace_end(p.trace, p.trace_slot);
    }
    __syncthreads();
    LLMRS_ATTN_MARK(6);
}

} // namespace

// K cache [n_kv * max_seq rows][D] viewed as (x: 32 floats of a 128-byte
// segment, y: row, z: segment), boxes of box_rows rows x every segment, swizzled
int encode_k_map(CUtensorMap *map, const float *kc, int rows, int D, int box_rows)
{
    auto fn = tensor_map_encoder();
    if (!fn)
        return fail(LLMRS_ECUDA, "cuTensorMapEncodeTiled unavailable");
    LLMRS_CHECK_ARG(((uintptr_t)kc & 15) == 0, "attention: K cache not 16-byte aligned");
    cuuint64_t dims[3] = {32, (cuuint64_t)rows, (cuuint64_t)(D / 32)};
    cuuint64_t strides[2] = {(cuuint64_t)D * 4, 128};
    cuuint32_t box[3] = {32, (cuuint32_t)box_rows, (cuuint32_t)(D / 32)};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(kc), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(LLMRS_ECUDA, "cuTensorMapEncodeTiled (K cache) failed (%d)", (int)r);
    return LLMRS_OK;
}

namespace {

template <int D, int NREP>
int launch_attn(const AttnParams &p, cudaStream_t stream, bool pdl)
{
    using Lay = AttnLayout<D, NREP>;
    LLMRS_CUDA_TRY(launch(attn_decode_kernel<D, NREP>, dim3(p.n_splits, p.n_kv), dim3(Lay::NW * 32), Lay::bytes,
                          stream, pdl, p));
    return LLMRS_OK;
}

template <int D, int NREP>
cudaError_t prepare_attn()
{
    return cudaFuncSetAttribute(attn_decode_kernel<D, NREP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)AttnLayout<D, NREP>::bytes);
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

// chunks per warp issued before the dependency wait (LLMRS_ATTN_EARLY, 0..2)
static int attn_early(void)
{
    static const int n = [] {
        const char *e = getenv("LLMRS_ATTN_EARLY");
        const int v = e ? atoi(e) : 1;
        return v < 0 ? 0 : (v > 2 ? 2 : v);
    }();
    return n;
}

int attention_decode_launch(const AttnParams &p0, cudaStream_t stream, bool pdl)
{
    AttnParams p = p0;
    p.early = attn_early();
    LLMRS_CHECK_ARG(p.n_kv > 0 && p.n_heads % p.n_kv == 0, "attention: n_heads %d not a multiple of n_kv %d",
                    p.n_heads, p.n_kv);
    const int nrep = p.n_heads / p.n_kv;
    const bool known = (p.head_dim == 128 || p.head_dim == 64) && (nrep == 4 || nrep == 8);
    if (!known)
        return fail(LLMRS_ENOTSUP, "attention: head_dim %d with n_rep %d not supported", p.head_dim, nrep);
    LLMRS_CHECK_ARG(((uintptr_t)p.vc & 15) == 0, "attention: V cache not 16-byte aligned");
    LLMRS_CHECK_ARG(p.n_splits >= 1 && p.n_splits <= 32, "attention: %d splits outside [1, 32]", p.n_splits);
    AttnParams q = p;
    LLMRS_TRY(encode_k_map(&q.tk, p.kc, p.n_kv * p.max_seq, p.head_dim, CH));
    if (p.head_dim == 128 && nrep == 4)
        return launch_attn<128, 4>(q, stream, pdl);
    if (p.head_dim == 128 && nrep == 8)
        return launch_attn<128, 8>(q, stream, pdl);
    if (p.head_dim == 64 && nrep == 4)
        return launch_attn<64, 4>(q, stream, pdl);
    if (p.head_dim == 64 && nrep == 8)
        return launch_attn<64, 8>(q, stream, pdl);
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

