// step.cu - one decode step (every layer + LM head) as a single persistent
// kernel on sm_100a.
//
// One CTA per SM for the whole step.  The CTA's producer warp walks the op
// list (QKV GEMV, attention, o_proj, gate_up, down per layer, then the LM
// head) and streams each op's share of weights (TMA tensor-map boxes) or
// K/V rows into one shared-memory ring, running ahead across op boundaries:
// weights do not depend on activations, so the HBM stream does not stop while
// the consumers wait for an op's input.  The 16 consumer warps walk the same
// list; before an op that reads the previous op's output they wait until
// every CTA has counted itself done with that op (a global counter per op,
// release / acquire at GPU scope, bounded), which replaces the kernel
// boundary and its launch gap.  Each op's consumer code is the one the
// one-kernel-per-op path uses (gemv_core.cuh, attention_core.cuh), so results
// are identical to it.
//
// Ring ownership: during a GEMV, warp group g owns stages g, g+4; during
// attention, warps 2s and 2s+1 own stage s (16 positions, 8 each).  Every
// consumer thread tracks the phase parity of every stage across ops (the
// per-op use counts are known on both sides), so a stage's barrier is only
// ever awaited one phase ahead of its completion.
//
// Activations written by other CTAs are read through L2 (ld.global.cg), since
// an SM's L1 is not coherent with other SMs' stores within one kernel.
#include <cstdlib>
#include <mutex>

#include "attention_core.cuh"
#include "gemv_core.cuh"
#include "step.cuh"

namespace llmrs {

namespace {

constexpr int R = STEP_ATTN_ROWS;
// dynamic shared memory cap: 227 KB per block minus the kernel's static arrays
constexpr size_t STEP_SMEM_MAX = 220 * 1024;

struct StepLayout {
    size_t ring, act, acts, actc, tb, link, tree, red, qs, probs, wm, wl, fw, ml, kn, vn, flag, bars, total;
};

__host__ __device__ inline size_t step_stage_bytes(int wf, int st)
{
    return align_up((size_t)TR * CB * wbytes_per_block(wf) + (size_t)TR * CB * sbytes(st), 1024);
}

// offsets from a 1024-byte aligned base; [act, ...) doubles as the attention
// op's warp-merge tree and split-merge scratch
__host__ __device__ inline StepLayout step_layout(size_t stage_bytes, int S, int kmax, int D, int nrep)
{
    StepLayout L;
    L.ring = 0;
    L.act = (size_t)S * stage_bytes;
    L.tree = L.act;
    L.acts = L.act + (size_t)kmax;
    L.actc = L.acts + (size_t)kmax / 32 * 4;
    L.tb = align_up(L.actc + (size_t)kmax / 32 * 4, 16);
    L.link = L.tb + (size_t)NW * RPW * TBS * 4;
    size_t end = L.link + (size_t)NW * RPW * 4;
    const size_t tree_end = L.tree + (size_t)(NW / 2) * nrep * D * 4;
    end = end > tree_end ? end : tree_end;
    L.red = align_up(end, 16);
    L.qs = align_up(L.red + 16 * 4, 16);
    L.probs = align_up(L.qs + (size_t)nrep * (D + 4) * 4, 16);
    L.wm = L.probs + (size_t)NW * 8 * nrep * 4;
    L.wl = L.wm + (size_t)NW * nrep * 4;
    L.fw = L.wl + (size_t)NW * nrep * 4;
    L.ml = L.fw + (size_t)NW * nrep * 4;
    L.kn = align_up(L.ml + (size_t)2 * nrep * 4, 16);
    L.vn = L.kn + (size_t)D * 4;
    L.flag = L.vn + (size_t)D * 4;
    L.bars = align_up(L.flag + 16, 8);
    L.total = L.bars + (size_t)(2 * S + NW) * 8 + 1024; // + base alignment slack
    return L;
}

// warp-cooperative copy of one op's parameters (global -> shared memory)
__device__ __forceinline__ void copy_op(StepOp *dst, const StepOp *src, int lane)
{
    static_assert(sizeof(StepOp) % 16 == 0, "16-byte units");
    const int4 *s4 = reinterpret_cast<const int4 *>(src);
    int4 *d4 = reinterpret_cast<int4 *>(dst);
    for (int k = lane; k < (int)(sizeof(StepOp) / 16); k += 32)
        d4[k] = __ldg(s4 + k);
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *m)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// wait until every CTA has counted itself done with an op (bounded: 2 s, then
// DEV_ERR_STEP_TIMEOUT; later waits of the step then return at once)
__device__ __forceinline__ void wait_done(const unsigned long long *c, unsigned long long target, uint32_t *err)
{
    if (ld_acquire_gpu(c) >= target)
        return;
    if (*reinterpret_cast<volatile uint32_t *>(err) != 0)
        return;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        __nanosleep(32);
        if (ld_acquire_gpu(c) >= target)
            return;
        if (globaltimer_ns() - t0 > 2000000000ull) {
            atomicCAS(err, 0u, (uint32_t)DEV_ERR_STEP_TIMEOUT);
            return;
        }
    }
}

struct AttnSplit {
    bool active, pos_ok, owner;
    int split, g, pos, t0, t1, nchunks;
};

__device__ __forceinline__ AttnSplit attn_split(const AttnParams &a, int cta, int pos)
{
    AttnSplit s;
    s.active = cta < a.n_kv * a.n_splits;
    s.split = cta % a.n_splits;
    s.g = cta / a.n_splits;
    s.pos = pos;
    s.pos_ok = pos >= 0 && pos < a.max_seq;
    const int Lc = s.pos_ok ? pos : 0;
    s.t0 = (int)(((long long)s.split * Lc) / a.n_splits);
    s.t1 = (int)(((long long)(s.split + 1) * Lc) / a.n_splits);
    s.nchunks = s.active ? (s.t1 - s.t0 + R - 1) / R : 0;
    s.owner = s.active && s.split == a.n_splits - 1;
    return s;
}

// attention op, producer side: this CTA's cached K/V rows, R positions per stage
template <int D>
__device__ __forceinline__ bool attn_produce(const AttnParams &a, const CUtensorMap *tk, const AttnSplit &sp,
                                             const GemvSmem &sm, uint32_t &fill_par, uint32_t &filled, uint64_t pol,
                                             uint32_t *err, InFlight &q)
{
    constexpr int ROWB = D * 4, KB = R * ROWB;
    for (int u = 0; u < sp.nchunks; u++) {
        const int s = u % sm.S;
        const uint32_t bit = 1u << s;
        if ((filled & bit) && !mbar_wait(&sm.empty[s], (fill_par & bit) ? 0u : 1u, err))
            return false;
        if (!inflight_admit(q, sm.full, err))
            return false;
        const int ta = sp.t0 + u * R;
        const int rows = min(R, sp.t1 - ta);
        uint8_t *st = sm.ring + (size_t)s * sm.stage_bytes;
        // the K box always moves R rows (rows past the split are ignored)
        mbar_arrive_expect_tx(&sm.full[s], (uint32_t)(KB + rows * ROWB));
        tma_load_3d(st, tk, 0, sp.g * a.max_seq + ta, 0, &sm.full[s], pol);
        bulk_g2s(st + KB, a.vc + ((size_t)sp.g * a.max_seq + ta) * D, (uint32_t)(rows * ROWB), &sm.full[s], pol);
        inflight_push(q, s);
        fill_par ^= bit;
        filled |= bit;
    }
    return true;
}

// attention op, consumer side (all consumer warps of an active CTA)
template <int D, int NREP>
__device__ __forceinline__ void attn_consume(const AttnParams &a, const AttnSplit &sp, const GemvSmem &sm, const StepLayout &L,
                             uint8_t *smem, uint32_t &cpar, int ctid, uint32_t *err, unsigned long long *ready_mark)
{
    constexpr int DL = D / 32, QS = D + 4, PS = D + 2;
    const int warp = ctid >> 5, lane = ctid & 31;
    float *q_s = reinterpret_cast<float *>(smem + L.qs);
    float *kn = reinterpret_cast<float *>(smem + L.kn);
    float *vn = reinterpret_cast<float *>(smem + L.vn);
    float *wm = reinterpret_cast<float *>(smem + L.wm);
    float *wl = reinterpret_cast<float *>(smem + L.wl);
    float *fw = reinterpret_cast<float *>(smem + L.fw);
    float *ml = reinterpret_cast<float *>(smem + L.ml);
    float *tree = reinterpret_cast<float *>(smem + L.tree);
    unsigned int *flag = reinterpret_cast<unsigned int *>(smem + L.flag);
    const int ns = a.n_splits, g = sp.g;

    // RoPE of q (warps < NREP, one head each) and of the new key (the owner
    // split's warp 0, which also appends k/v at pos)
    const int Lc = sp.pos_ok ? sp.pos : 0;
    const float *cosr = a.rope_cos + (size_t)Lc * (D / 2);
    const float *sinr = a.rope_sin + (size_t)Lc * (D / 2);
    const bool appender = sp.owner && warp == 0;
    float qv[DL], kk[DL], vv[DL], rc[DL], rs[DL];
    if (warp < NREP || appender)
        rope_table_lane<D>(rc, rs, lane, cosr, sinr);
    if (warp < NREP) {
        const float *qh = a.qkv + (size_t)(g * NREP + warp) * D + lane * DL;
#pragma unroll
        for (int k = 0; k < DL; k++)
            qv[k] = __ldcg(qh + k);
        rope_lane<D>(qv, lane, rc, rs);
#pragma unroll
        for (int k = 0; k < DL; k++)
            q_s[warp * QS + lane * DL + k] = qv[k];
    }
    if (appender) {
        const float *kp = a.qkv + (size_t)a.n_heads * D + (size_t)g * D + lane * DL;
        const float *vp = a.qkv + (size_t)(a.n_heads + a.n_kv) * D + (size_t)g * D + lane * DL;
#pragma unroll
        for (int k = 0; k < DL; k++) {
            kk[k] = __ldcg(kp + k);
            vv[k] = __ldcg(vp + k);
        }
        rope_lane<D>(kk, lane, rc, rs);
#pragma unroll
        for (int k = 0; k < DL; k++) {
            kn[lane * DL + k] = kk[k];
            vn[lane * DL + k] = vv[k];
            if (sp.pos_ok) {
                a.kc[((size_t)g * a.max_seq + sp.pos) * D + lane * DL + k] = kk[k];
                a.vc[((size_t)g * a.max_seq + sp.pos) * D + lane * DL + k] = vv[k];
            }
        }
    }
    if (ctid == 0 && !sp.pos_ok)
        atomicCAS(err, 0u, (uint32_t)DEV_ERR_BAD_POS);
    named_bar_sync(1, PRO_THREADS);
    if (ready_mark && ctid == 0)
        atomicMax(ready_mark, (unsigned long long)globaltimer_ns());

    float m_run = -INFINITY, l_run = 0.0f;
    float acc[NREP][DL];
#pragma unroll
    for (int h = 0; h < NREP; h++)
#pragma unroll
        for (int k = 0; k < DL; k++)
            acc[h][k] = 0.0f;
    if (warp < 2 * sm.S) {
        const int s = warp >> 1, half = warp & 1;
        uint32_t par = (cpar >> s) & 1u;
        float *probs = reinterpret_cast<float *>(smem + L.probs) + warp * 8 * NREP;
        for (int u = s; u < sp.nchunks; u += sm.S) {
            if (!mbar_wait(&sm.full[s], par, err))
                break;
            par ^= 1u;
            const int rows = min(R, sp.t1 - (sp.t0 + u * R));
            const int nvalid = max(0, min(8, rows - half * 8));
            const float *st = reinterpret_cast<const float *>(sm.ring + (size_t)s * sm.stage_bytes);
            if (nvalid > 0)
                attn_chunk<D, NREP, R>(st, half * 8, st + R * D + half * 8 * D, nvalid, q_s, QS, probs,
                                       a.inv_sqrt_d, m_run, l_run, acc, lane);
            __syncwarp();
            if (lane == 0)
                mbar_arrive_n(&sm.empty[s], WPG / 2); // the stage's two warps release it together
        }
    }
    if (appender && sp.pos_ok)
        attn_new_position<D, NREP>(kn, vn, q_s, QS, a.inv_sqrt_d, m_run, l_run, acc, lane);
    for (int s = 0; s < sm.S; s++) {
        const int uses = sp.nchunks > s ? (sp.nchunks - 1 - s) / sm.S + 1 : 0;
        cpar ^= (uint32_t)(uses & 1) << s;
    }

    // merge the warps: common max per head, then a fixed pairwise tree
    if (lane < NREP) {
        wm[warp * NREP + lane] = m_run;
        wl[warp * NREP + lane] = l_run;
    }
    named_bar_sync(1, PRO_THREADS);
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
        ml[h] = M;
        ml[NREP + h] = l;
    }
    named_bar_sync(1, PRO_THREADS);
#pragma unroll
    for (int h = 0; h < NREP; h++) {
        const float f = fw[warp * NREP + h];
#pragma unroll
        for (int k = 0; k < DL; k++)
            acc[h][k] *= f;
    }
    for (int hn = NW / 2; hn >= 1; hn >>= 1) {
        if (warp >= hn && warp < 2 * hn)
#pragma unroll
            for (int h = 0; h < NREP; h++)
#pragma unroll
                for (int k = 0; k < DL; k++)
                    tree[((warp - hn) * NREP + h) * D + lane * DL + k] = acc[h][k];
        named_bar_sync(1, PRO_THREADS);
        if (warp < hn)
#pragma unroll
            for (int h = 0; h < NREP; h++)
#pragma unroll
                for (int k = 0; k < DL; k++)
                    acc[h][k] += tree[(warp * NREP + h) * D + lane * DL + k];
        named_bar_sync(1, PRO_THREADS);
    }
    if (warp == 0) {
#pragma unroll
        for (int h = 0; h < NREP; h++) {
            float *dst = a.part + ((size_t)(g * NREP + h) * ns + sp.split) * PS;
#pragma unroll
            for (int k = 0; k < DL; k++)
                dst[lane * DL + k] = acc[h][k];
            if (lane == 0) {
                dst[D] = ml[h];
                dst[D + 1] = ml[NREP + h];
            }
        }
    }
    // the last CTA of this KV head merges the splits in split order
    named_bar_sync(1, PRO_THREADS);
    if (ctid == 0) {
        __threadfence();
        flag[0] = (atomicAdd(&a.counter[g], 1u) == (unsigned)(ns - 1)) ? 1u : 0u;
    }
    named_bar_sync(1, PRO_THREADS);
    if (!flag[0])
        return;
    __threadfence();
    float *mm = tree;              // [NREP][ns] split maxima, then weights
    float *ll = tree + NREP * ns;  // [NREP][ns] split sums
    float *ltot = ll + NREP * ns;  // [NREP]
    for (int e = ctid; e < NREP * ns; e += PRO_THREADS) {
        const int h = e / ns, s = e % ns;
        const float *src = a.part + ((size_t)(g * NREP + h) * ns + s) * PS;
        mm[e] = __ldcg(src + D);
        ll[e] = __ldcg(src + D + 1);
    }
    named_bar_sync(1, PRO_THREADS);
    if (warp < NREP) {
        const int h = warp;
        float M = -INFINITY;
        for (int s = lane; s < ns; s += 32)
            M = fmaxf(M, mm[h * ns + s]);
        M = warp_max(M);
        float l = 0.0f;
        for (int s = lane; s < ns; s += 32) {
            const float ms = mm[h * ns + s];
            const float f = (ms == -INFINITY) ? 0.0f : expf(ms - M);
            mm[h * ns + s] = f;
            l += ll[h * ns + s] * f;
        }
        l = warp_sum(l);
        if (lane == 0)
            ltot[h] = l;
    }
    named_bar_sync(1, PRO_THREADS);
    for (int e = ctid; e < NREP * D; e += PRO_THREADS) {
        const int h = e / D, d = e % D;
        const float *src = a.part + (size_t)(g * NREP + h) * ns * PS + d;
        float v = 0.0f;
        for (int s = 0; s < ns; s++)
            v += __ldcg(src + (size_t)s * PS) * mm[h * ns + s];
        a.ctx[(size_t)(g * NREP + h) * D + d] = v / ltot[h];
    }
    if (ctid == 0)
        a.counter[g] = 0u;
}

__device__ __forceinline__ GemvSmem step_gemv_smem(uint8_t *smem, const StepLayout &L, size_t stage_bytes, int S,
                                                   int wf)
{
    GemvSmem sm;
    sm.ring = smem + L.ring;
    sm.stage_bytes = stage_bytes;
    sm.scale_off = (size_t)TR * CB * wbytes_per_block(wf);
    sm.S = S;
    sm.full = reinterpret_cast<uint64_t *>(smem + L.bars);
    sm.empty = sm.full + S;
    sm.link = sm.empty + S;
    sm.issued = nullptr;
    sm.act = reinterpret_cast<uint32_t *>(smem + L.act);
    sm.act_s = reinterpret_cast<float *>(smem + L.acts);
    sm.act_c = reinterpret_cast<int *>(smem + L.actc);
    sm.tbuf = reinterpret_cast<float *>(smem + L.tb);
    sm.linkbuf = reinterpret_cast<float *>(smem + L.link);
    sm.red = reinterpret_cast<float *>(smem + L.red);
    return sm;
}

// Each GEMV variant runs as its own (non-inlined) function that builds its
// shared-memory view and work split itself: inlined into one switch, the
// variants shared one register allocation and spilled in their hot loops.
// Scalars in, two parity words through pointers, once per op.
template <int W, int S_, int P, int E>
__device__ __noinline__ void gemv_op(const StepOp *op, uint8_t *smem, const StepLayout *L, size_t stage_bytes, int S,
                                     uint32_t *cpar, uint32_t *lpar, int ctid, unsigned long long *ready_mark)
{
    GemvSmem sm = step_gemv_smem(smem, *L, stage_bytes, S, W);
    sm.ready_mark = ready_mark;
    const GemvWork w = gemv_work(op->g, blockIdx.x);
    uint32_t c = *cpar, l = *lpar;
    gemv_consume<W, S_, P, E>(op->g, w, sm, c, l, ctid);
    *cpar = c;
    *lpar = l;
}

#define LLMRS_STEP_GEMV_CASE(W, S_, P, E)                                                                      \
    case P * 8 + E:                                                                                            \
        gemv_op<W, S_, P, E>(&op, smem, &L, stage_bytes, S, &cpar, &lpar, ctid, ready_mark);                   \
        return true;

// GEMV op, consumer side: the layers' (WF, ST) or the LM head's (Q4, LMST);
// only the variants a one-GPU (TP = 0) or tensor-parallel (TP = 1) step uses,
// to keep the kernel's code (and its instruction-cache footprint) small
template <int WF, int ST, int LMST, int TP>
__device__ __forceinline__ bool step_gemv_consume(const StepOp &op, uint8_t *smem, const StepLayout &L,
                                                  size_t stage_bytes, int S, uint32_t &cpar, uint32_t &lpar, int ctid,
                                                  unsigned long long *ready_mark)
{
    const int key = op.pro * 8 + op.epi;
    if (op.wf == WF && op.st == ST) {
        if (TP == 0) {
            switch (key) {
                LLMRS_STEP_GEMV_CASE(WF, ST, PRO_EMBED_NORM, EPI_STORE)
                LLMRS_STEP_GEMV_CASE(WF, ST, PRO_NORM, EPI_STORE)
                LLMRS_STEP_GEMV_CASE(WF, ST, PRO_F32, EPI_RESIDUAL)
                LLMRS_STEP_GEMV_CASE(WF, ST, PRO_NORM, EPI_SILU)
                LLMRS_STEP_GEMV_CASE(WF, ST, PRO_NORM, EPI_ARGMAX)
            default:
                break;
            }
        } else {
            switch (key) {
                LLMRS_STEP_GEMV_CASE(WF, ST, PRO_EMBED_NORM, EPI_STORE)
                LLMRS_STEP_GEMV_CASE(WF, ST, PRO_F32, EPI_PARTIAL)
                LLMRS_STEP_GEMV_CASE(WF, ST, PRO_AR_NORM, EPI_STORE)
                LLMRS_STEP_GEMV_CASE(WF, ST, PRO_AR_NORM, EPI_SILU)
                LLMRS_STEP_GEMV_CASE(WF, ST, PRO_AR_NORM, EPI_ARGMAX)
            default:
                break;
            }
        }
    }
    if (!(WF == 0 && ST == LMST) && op.wf == 0 && op.st == LMST) {
        switch (key) {
            LLMRS_STEP_GEMV_CASE(0, LMST, TP ? PRO_AR_NORM : PRO_NORM, EPI_ARGMAX)
        default:
            break;
        }
    }
    return false;
}
#undef LLMRS_STEP_GEMV_CASE

template <int WF, int ST, int LMST, int D, int NREP, int TP>
__global__ void __launch_bounds__(NTHREADS, 1)
    decode_step_kernel(const StepOp *__restrict__ ops, int n_ops, unsigned long long *done, const StepState *state,
                       uint32_t *err, int kmax, int S, unsigned long long *trace, int inflight)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    constexpr size_t SB1 = (size_t)TR * CB * wbytes_per_block(WF) + (size_t)TR * CB * sbytes(ST);
    constexpr size_t SB2 = (size_t)TR * CB * wbytes_per_block(0) + (size_t)TR * CB * sbytes(LMST);
    // Kernel-wide constants live in shared memory, not in registers held across
    // the op loop: the ops' own code needs the registers.
    __shared__ StepLayout L;
    __shared__ size_t s_stage_bytes;
    __shared__ int s_pos;
    __shared__ unsigned long long s_target;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        s_stage_bytes = align_up(SB1 > SB2 ? SB1 : SB2, 1024);
        L = step_layout(s_stage_bytes, S, kmax, D, NREP);
        // the step's position and epoch are settled before the kernel starts
        // (host write or the previous step's LM head); the LM head of this
        // step changes them only after every CTA is past its last use of them
        s_pos = __ldcg(&state->pos);
        // done[n_ops] counts this kernel's launches (decode steps may also run
        // one kernel per op, which leaves these counters alone)
        s_target = (__ldcg(&done[n_ops]) + 1) * (unsigned long long)gridDim.x;
        uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bars);
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&full[S + s], WPG); // empty: released by a warp group (or two attention warps)
        }
        for (int i = 0; i < NW; i++)
            mbar_init(&full[2 * S + i], 1); // GEMV running-sum links
        fence_mbar_init();
    }
    __syncthreads();

    // Both roles read each op's parameters from a shared-memory copy made one
    // op ahead (global loads on every use cost latency and registers); TMA
    // descriptors stay in global memory, prefetched one op ahead.
    __shared__ __align__(64) StepOp s_pop[2], s_cop[2];
    if (warp == NW) {
        // ------------------------------------------------------------ producer
        copy_op(&s_pop[0], &ops[0], lane);
        uint32_t fill_par = 0, filled = 0;
        const uint64_t pol = policy_evict_first();
        InFlight q;
        q.cap = inflight;
        for (int i = 0; i < n_ops; i++) {
            if (i + 1 < n_ops) {
                copy_op(&s_pop[(i + 1) & 1], &ops[i + 1], lane);
                if (lane == 0) { // the next op's descriptors into the TMA unit's cache
                    const StepOp &nx = ops[i + 1];
                    prefetch_tensormap(&nx.tw);
                    prefetch_tensormap(&nx.ts);
                    prefetch_tensormap(&nx.a.tk);
                }
            }
            __syncwarp();
            bool ok = true;
            if (lane == 0) {
                const StepOp &op = s_pop[i & 1];
                const StepOp &og = ops[i]; // descriptors
                if (op.kind == OP_GEMV) {
                    const GemvSmem sm = step_gemv_smem(smem, L, s_stage_bytes, S, op.wf);
                    const GemvWork w = gemv_work(op.g, blockIdx.x);
                    if (op.wf == WF && op.st == ST)
                        ok = gemv_produce<WF, ST>(&og.tw, &og.ts, op.g, w, sm, fill_par, filled, pol, -1, q);
                    else
                        ok = gemv_produce<0, LMST>(&og.tw, &og.ts, op.g, w, sm, fill_par, filled, pol, -1, q);
                } else {
                    const GemvSmem sm = step_gemv_smem(smem, L, s_stage_bytes, S, 0);
                    ok = attn_produce<D>(op.a, &og.a.tk, attn_split(op.a, blockIdx.x, s_pos), sm, fill_par, filled,
                                         pol, err, q);
                }
            }
            if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0))
                break;
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    const int ctid = threadIdx.x;
    uint32_t cpar = 0, lpar = 0;
    if (warp == 0)
        copy_op(&s_cop[0], &ops[0], lane);
    named_bar_sync(1, PRO_THREADS);
    for (int i = 0; i < n_ops; i++) {
        const StepOp &op = s_cop[i & 1];
        if (warp == NW - 1 && i + 1 < n_ops) // ready for the next op (its buffer's last reader finished op i-1)
            copy_op(&s_cop[(i + 1) & 1], &ops[i + 1], lane);
        if (trace && ctid == 0)
            atomicMin(&trace[TRACE_MARKS * i], (unsigned long long)globaltimer_ns());
        if (op.wait_op >= 0) {
            if (ctid == 0)
                wait_done(done + op.wait_op, s_target, err);
            named_bar_sync(1, PRO_THREADS);
        }
        if (trace && ctid == 0) // op timeline: first CTA past the input wait, last CTA
            atomicMin(&trace[TRACE_MARKS * i + 1], (unsigned long long)globaltimer_ns()); // done with its prologue, last CTA done
        if (op.kind == OP_GEMV) {
            if (!step_gemv_consume<WF, ST, LMST, TP>(op, smem, L, s_stage_bytes, S, cpar, lpar, ctid,
                                                     trace ? &trace[TRACE_MARKS * i + 2] : nullptr) &&
                ctid == 0)
                atomicCAS(err, 0u, (uint32_t)DEV_ERR_BAD_OP);
        } else {
            const GemvSmem sm = step_gemv_smem(smem, L, s_stage_bytes, S, 0);
            const AttnSplit sp = attn_split(op.a, blockIdx.x, s_pos);
            if (sp.active)
                attn_consume<D, NREP>(op.a, sp, sm, L, smem, cpar, ctid, err,
                                      trace ? &trace[TRACE_MARKS * i + 2] : nullptr);
        }
        // this CTA's share of op i is stored: count it in
        named_bar_sync(1, PRO_THREADS);
        if (ctid == 0) {
            __threadfence();
            const unsigned long long prev = atomicAdd(done + i, 1ull);
            if (i == n_ops - 1 && prev + 1 == s_target) // the last CTA out: every CTA has read the launch count
                atomicAdd(done + n_ops, 1ull);
            if (trace)
                atomicMax(&trace[TRACE_MARKS * i + 3], (unsigned long long)globaltimer_ns());
        }
    }
}

// the model shapes the kernel is built for: (weights, scales, LM-head scales, D, n_rep)
// the model shapes the kernel is built for: (weights, scales, LM-head scales, D, n_rep, tensor parallel)
#define LLMRS_STEP_VARIANTS(X)                                                                                 \
    X(0, 0, 0, 128, 4, 0) X(0, 0, 0, 128, 8, 0) X(0, 0, 1, 64, 4, 0) X(0, 0, 0, 64, 4, 0)                    \
    X(0, 1, 1, 64, 4, 0) X(1, 0, 0, 64, 4, 0) X(1, 0, 0, 128, 4, 0) X(0, 0, 0, 128, 4, 1)                    \
    X(0, 0, 0, 128, 8, 1) X(0, 0, 1, 64, 4, 1)

} // namespace

size_t step_smem_bytes(int wf, int st, int lm_st, int D, int nrep, int tp, int kmax, int *stages)
{
    bool known = false;
#define LLMRS_STEP_KNOWN(W, S_, LM, DD, NR, TP)                                                                \
    if (wf == W && st == S_ && lm_st == LM && D == DD && nrep == NR && tp == TP)                               \
        known = true;
    LLMRS_STEP_VARIANTS(LLMRS_STEP_KNOWN)
#undef LLMRS_STEP_KNOWN
    if (!known)
        return 0;
    const size_t a = step_stage_bytes(wf, st), b = step_stage_bytes(0, lm_st);
    const size_t sb = a > b ? a : b;
    for (int S = 8; S >= 4; S -= 4) {
        const size_t t = step_layout(sb, S, kmax, D, nrep).total;
        if (t <= STEP_SMEM_MAX) {
            *stages = S;
            return t;
        }
    }
    return 0;
}

// stages a CTA's producer keeps requested but not landed (LLMRS_STEP_INFLIGHT,
// default 0 = unbounded)
static int step_inflight(void)
{
    static const int n = [] {
        const char *e = getenv("LLMRS_STEP_INFLIGHT");
        const int v = e ? atoi(e) : 0;
        return v < 0 ? 0 : (v > 8 ? 8 : v);
    }();
    return n;
}

int step_prepare(void)
{
    cudaError_t e = cudaSuccess;
#define LLMRS_STEP_PREP(W, S_, LM, DD, NR, TP)                                                                 \
    if (e == cudaSuccess)                                                                                      \
        e = cudaFuncSetAttribute(decode_step_kernel<W, S_, LM, DD, NR, TP>,                                    \
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)STEP_SMEM_MAX);
    LLMRS_STEP_VARIANTS(LLMRS_STEP_PREP)
#undef LLMRS_STEP_PREP
    if (e != cudaSuccess)
        return fail(LLMRS_ECUDA, "decode-step kernel attributes: %s", cudaGetErrorString(e));
    return LLMRS_OK;
}

int step_launch(int wf, int st, int lm_st, int D, int nrep, int tp, int kmax, int stages, size_t smem, int grid,
                const StepOp *d_ops, int n_ops, unsigned long long *d_done, const StepState *state, uint32_t *err,
                unsigned long long *trace, cudaStream_t stream)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NTHREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative; // every CTA resident at once, or the launch fails
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
#define LLMRS_STEP_LAUNCH(W, S_, LM, DD, NR, TP)                                                               \
    if (wf == W && st == S_ && lm_st == LM && D == DD && nrep == NR && tp == TP) {                            \
        LLMRS_CUDA_TRY(cudaLaunchKernelEx(&cfg, decode_step_kernel<W, S_, LM, DD, NR, TP>, d_ops, n_ops, d_done, \
                                          state, err, kmax, stages, trace, step_inflight()));                                          \
        return LLMRS_OK;                                                                                       \
    }
    LLMRS_STEP_VARIANTS(LLMRS_STEP_LAUNCH)
#undef LLMRS_STEP_LAUNCH
    return fail(LLMRS_ENOTSUP, "decode-step kernel not built for this model shape");
}

} // namespace llmrs
