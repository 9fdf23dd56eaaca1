// gemv.cu - Q4_0 / Q8_0 weight x Q8_0 activation matrix-vector product for
// batch-1 decode on B200 (sm_100a).
//
// Arithmetic (bit-exact with src/backend/cpu.rs:888-941, kernel_avx2):
//   per output row j:  acc = 0; for blocks b = 0..K/32-1 in order:
//       scale = sw[j,b] * sa[b]                 (f32 multiply)
//       isum  = sum_i (w_i - 8) * q8_i          (exact int32; Q8_0 weights: w_i * q8_i)
//       acc   = acc + (float)isum * scale       (f32 multiply, then f32 add; never FMA)
// The activation is quantised to Q8_0 in the kernel's prologue exactly as
// CpuBackend::quantize_row_q8_0 does (src/backend/cpu.rs:724-743).
//
// Work split.  Each CTA owns rows [i*rows_per_cta, (i+1)*rows_per_cta), cut
// into tiles of box_rows (<= 32) rows; a tile is processed in chunks of 32
// blocks (1024 weights).  One (tile, chunk) pair is one pipeline stage.
//
// Data movement.  A producer thread streams each stage with two 2-D
// tensor-map TMA copies straight from the reference's planar layout (a box of
// rows x 512 bytes of nibbles, or x 1024 bytes of int8 codes, and a box of
// rows x 32 block scales) into a ring of shared-memory stages.
//
// Compute.  16 consumer warps form 4 groups; group g owns tiles g, g+4, ...
// and ring stages g, g+4, ...  Within a stage, lane l of a warp handles block
// l for the warp's 8 rows (dp4a products times the two scales); the products
// are transposed through shared memory so that 4 lanes per row add the 32
// block products in order (8 each, passed lane to lane).  A row's running sum
// stays in registers from chunk to chunk, so the reference's sequential order
// holds while four tiles are computed at once.
//
// The prologue (RMSNorm where fused, Q8_0 quantisation) runs once per CTA in
// shared memory.  Activation loads are issued before the weight stream (loads
// queued behind bulk copies wait for them, L2 hits included).  With
// programmatic dependent launch the CTA starts while the previous kernel
// finishes; consumers call griddepcontrol.wait before touching activations.
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "gemv.cuh"

// Optional phase tracing (cycle counters around pipeline waits); compiled out
// unless a tracing build defines LLMRS_GEMV_TRACE and provides the hooks.
#ifndef LLMRS_GEMV_TRACE
#define LLMRS_TRACE_BEGIN(slot)
#define LLMRS_TRACE_END(slot)
#define LLMRS_TRACE_FLUSH(role)
#define LLMRS_TRACE_PROLOG
#endif

namespace llmrs {

namespace {

constexpr int NG = 4;                    // consumer warp groups (one pipeline stage each)
constexpr int WPG = 4;                   // warps per group
constexpr int RPW = 8;                   // tile rows per warp (WPG * RPW = 32)
constexpr int NW = NG * WPG;             // consumer warps
constexpr int NTHREADS = (NW + 1) * 32;  // + producer warp
constexpr int TR = 32;                   // max rows per tile
constexpr int CB = 32;                   // blocks per chunk (1024 weights), one per lane
constexpr int TBS = 36;                  // transpose row stride (floats): 16-byte aligned, conflict-free
constexpr size_t SMEM_BUDGET = 200 * 1024; // one CTA per SM (544 threads): use most of the SM's shared memory
constexpr int MAX_STAGES = 8;
constexpr int PRO_THREADS = NW * 32;

__host__ __device__ constexpr int wbytes_per_block(int wf) { return wf == 0 ? 16 : 32; }
__host__ __device__ constexpr int sbytes(int st) { return st == 0 ? 2 : 4; }
__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) & ~(a - 1); }

struct SmemLayout {
    size_t stage_bytes, scale_off, act_off, acts_off, actc_off, tb_off, link_off, bar_off, red_off, total;
};

// offsets are relative to a 128-byte aligned base
__host__ __device__ inline SmemLayout smem_layout(int wf, int st, int K, int stages)
{
    SmemLayout L;
    const int nb = K / 32;
    L.scale_off = (size_t)TR * CB * wbytes_per_block(wf);
    L.stage_bytes = align_up(L.scale_off + (size_t)TR * CB * sbytes(st), 128);
    L.act_off = L.stage_bytes * stages;
    L.acts_off = L.act_off + (size_t)nb * 32;
    L.actc_off = align_up(L.acts_off + (size_t)nb * 4, 16);
    L.tb_off = align_up(L.actc_off + (size_t)nb * 4, 16);
    L.link_off = L.tb_off + (size_t)NW * RPW * TBS * 4;
    L.bar_off = align_up(L.link_off + (size_t)NW * RPW * 4, 16);
    L.red_off = L.bar_off + (size_t)(2 * stages + NW + 1) * 8; // full, empty, link, activation-issued
    L.total = align_up(L.red_off + 16 * 4, 16) + 128; // + slack to align the base
    return L;
}

// ------------------------------------------------------------- activation
// Quantise one 32-value block held by one thread (bit-exact Q8_0) and pack it
// for the weight format: Q4 order puts the even elements of every 8 in words
// 0-3 and the odd ones in words 4-7 (matching low / high nibbles), Q8 keeps
// the natural order.
template <int WF>
__device__ __forceinline__ void quantize_pack(const float (&v)[32], uint32_t *dst_words, float *dst_s, int *dst_c)
{
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; i++)
        amax = fmaxf(amax, fabsf(v[i]));
    float scale = 0.0f, inv = 0.0f;
    if (amax != 0.0f) {
        scale = __fdiv_rn(amax, 127.0f);
        inv = __fdiv_rn(1.0f, scale);
    }
    int q[32];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 32; i++) {
        float r = roundf(__fmul_rn(v[i], inv));
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        q[i] = (amax == 0.0f || r != r) ? 0 : (int)r;
        sum += q[i];
    }
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        uint32_t x = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int e = WF == 0 ? (j < 4 ? 8 * j + 2 * k : 8 * (j - 4) + 2 * k + 1) : 4 * j + k;
            x |= (uint32_t)(q[e] & 0xFF) << (8 * k);
        }
        w[j] = x;
    }
    reinterpret_cast<uint4 *>(dst_words)[0] = make_uint4(w[0], w[1], w[2], w[3]);
    reinterpret_cast<uint4 *>(dst_words)[1] = make_uint4(w[4], w[5], w[6], w[7]);
    *dst_s = scale;
    *dst_c = WF == 0 ? -8 * sum : 0;
}

// 32 floats through L2 only (data other GPUs wrote into this GPU's memory)
__device__ __forceinline__ void load32_cg(const float *src, float (&v)[32])
{
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const float4 t = __ldcg(reinterpret_cast<const float4 *>(src) + j);
        v[4 * j] = t.x;
        v[4 * j + 1] = t.y;
        v[4 * j + 2] = t.z;
        v[4 * j + 3] = t.w;
    }
}

__device__ __forceinline__ void load32(const float *src, float (&v)[32])
{
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float4 f = s4[i];
        v[4 * i] = f.x;
        v[4 * i + 1] = f.y;
        v[4 * i + 2] = f.z;
        v[4 * i + 3] = f.w;
    }
}

// Fill the shared-memory activation (codes, scales, corrections).  One thread
// per 32-block; `nthr` threads with ids `tid` take part; `bar` is a named
// barrier id covering exactly those threads.
// Tell the producer that this warp's activation loads are in flight (one
// arrival per warp).  Loads issued after a stream of bulk weight copies queue
// behind it, even when they hit L2, so the producer holds the stream until the
// activation (a few KB that every CTA needs first) has been requested.
__device__ __forceinline__ void signal_issued(uint64_t *issued, int tid)
{
    if (issued) {
        __syncwarp();
        if ((tid & 31) == 0)
            mbar_arrive(issued);
    }
}

template <int WF>
__device__ __forceinline__ void pack_q8_block(const uint4 c0, const uint4 c1, uint32_t *dst, int *dst_c)
{
    const uint32_t in[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    int q[32], sum = 0;
#pragma unroll
    for (int i = 0; i < 32; i++) {
        q[i] = (int)(int8_t)(in[i >> 2] >> (8 * (i & 3)));
        sum += q[i];
    }
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        uint32_t x = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int e = WF == 0 ? (j < 4 ? 8 * j + 2 * k : 8 * (j - 4) + 2 * k + 1) : 4 * j + k;
            x |= (uint32_t)(q[e] & 0xFF) << (8 * k);
        }
        w[j] = x;
    }
    reinterpret_cast<uint4 *>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
    reinterpret_cast<uint4 *>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
    *dst_c = WF == 0 ? -8 * sum : 0;
}

// Activation prologue: thread t handles blocks t, t + nthr, ...; the first
// block's loads are issued before signal_issued, later blocks (K > 32 * nthr)
// load as they go.
template <int WF, int PRO>
__device__ void load_activation(const GemvParams &p, uint32_t *act, float *act_s, int *act_c, float *red, int tid,
                                int nthr, int bar, uint64_t *issued)
{
    const int K = p.K, nb = K >> 5;
    const bool has = tid < nb;
    if (PRO == PRO_Q8) {
        uint4 c0 = make_uint4(0, 0, 0, 0), c1 = c0;
        float xs = 0.0f;
        if (has) {
            c0 = reinterpret_cast<const uint4 *>(p.xq + (size_t)tid * 32)[0];
            c1 = reinterpret_cast<const uint4 *>(p.xq + (size_t)tid * 32)[1];
            xs = p.xs[tid];
        }
        signal_issued(issued, tid);
        if (has) {
            pack_q8_block<WF>(c0, c1, act + (size_t)tid * 8, act_c + tid);
            act_s[tid] = xs;
        }
        for (int b = tid + nthr; b < nb; b += nthr) {
            const uint4 d0 = reinterpret_cast<const uint4 *>(p.xq + (size_t)b * 32)[0];
            const uint4 d1 = reinterpret_cast<const uint4 *>(p.xq + (size_t)b * 32)[1];
            pack_q8_block<WF>(d0, d1, act + (size_t)b * 8, act_c + b);
            act_s[b] = p.xs[b];
        }
        return;
    }
    constexpr bool NORM = PRO == PRO_NORM || PRO == PRO_EMBED_NORM || PRO == PRO_AR_NORM;
    constexpr bool AR = PRO == PRO_AR_NORM;
    const float *x = p.x;
    if (PRO == PRO_EMBED_NORM) {
        int tok = p.state->token;
        if (tok < 0 || tok >= p.vocab) {
            if (tid == 0)
                atomicCAS(p.err, 0u, (uint32_t)DEV_ERR_BAD_TOKEN);
            tok = 0;
        }
        x = p.embed + (size_t)tok * K;
    }
    const float *part = nullptr; // AR: this rank's receive buffer [size][K]
    int nparts = 0;
    if (AR) {
        // the weight stream need not wait for the other ranks
        signal_issued(issued, tid);
        const TpLink *tp = p.tp;
        if (tid == 0) {
            const unsigned long long target =
                ((unsigned long long)p.state->epoch * p.ar_per_step + p.ar_index + 1) * (unsigned long long)p.ar_arrivals;
            wait_counter(tp->cnt[tp->rank] + p.ar_kind, target, p.err);
        }
        named_bar_sync(bar, nthr);
        part = tp->ar[p.ar_kind][tp->rank];
        nparts = tp->size;
    }
    // block b of the input: x, or (AR) the ranks' partial sums in rank order, then + x
    auto load_x = [&](int b, float (&u)[32]) {
        load32(x + (size_t)b * 32, u);
        if (AR) {
            float t[32];
            load32_cg(part + (size_t)b * 32, t);
            for (int q = 1; q < nparts; q++) {
                float w[32];
                load32_cg(part + (size_t)q * K + (size_t)b * 32, w);
#pragma unroll
                for (int i = 0; i < 32; i++)
                    t[i] = __fadd_rn(t[i], w[i]);
            }
#pragma unroll
            for (int i = 0; i < 32; i++)
                u[i] = __fadd_rn(t[i], u[i]);
        }
    };
    float v[32], wn[32];
    if (has) {
        load_x(tid, v);
        if (NORM)
            load32(p.norm_w + (size_t)tid * 32, wn);
    }
    if (!AR)
        signal_issued(issued, tid);
    if ((PRO == PRO_EMBED_NORM || AR) && blockIdx.x == 0) { // the residual stream's new value
        if (has)
#pragma unroll
            for (int i = 0; i < 32; i++)
                p.x_out[(size_t)tid * 32 + i] = v[i];
        for (int b = tid + nthr; b < nb; b += nthr) {
            float u[32];
            load_x(b, u);
            for (int i = 0; i < 32; i++)
                p.x_out[(size_t)b * 32 + i] = u[i];
        }
    }
    float scale = 1.0f;
    if (NORM) {
        // sum of squares in a fixed order (per thread, then a fixed tree)
        float ss = 0.0f;
        if (has)
#pragma unroll
            for (int i = 0; i < 32; i++)
                ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
        for (int b = tid + nthr; b < nb; b += nthr) {
            float u[32];
            load_x(b, u);
#pragma unroll
            for (int i = 0; i < 32; i++)
                ss = __fadd_rn(ss, __fmul_rn(u[i], u[i]));
        }
        ss = warp_sum(ss);
        const int warp = tid >> 5;
        if ((tid & 31) == 0)
            red[warp] = ss;
        named_bar_sync(bar, nthr);
        float tot = red[0];
        for (int w = 1; w < nthr / 32; w++)
            tot = __fadd_rn(tot, red[w]);
        const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), p.eps));
        scale = __fdiv_rn(1.0f, rms);
    }
    if (has) {
        if (NORM)
#pragma unroll
            for (int i = 0; i < 32; i++)
                v[i] = __fmul_rn(__fmul_rn(v[i], scale), wn[i]);
        quantize_pack<WF>(v, act + (size_t)tid * 8, act_s + tid, act_c + tid);
    }
    for (int b = tid + nthr; b < nb; b += nthr) {
        float u[32];
        load_x(b, u);
        if (NORM) {
            float un[32];
            load32(p.norm_w + (size_t)b * 32, un);
#pragma unroll
            for (int i = 0; i < 32; i++)
                u[i] = __fmul_rn(__fmul_rn(u[i], scale), un[i]);
        }
        quantize_pack<WF>(u, act + (size_t)b * 8, act_s + b, act_c + b);
    }
}

// Tensor parallel: this CTA's partial rows are in every rank's buffer; count
// the CTA in on every rank.  The barrier orders every thread's stores before
// thread 0's system-scope fence (cumulativity), which orders them before the
// counter increments the other ranks acquire.
__device__ __forceinline__ void partial_signal(const GemvParams &p, int tid, int nthr, int bar)
{
    named_bar_sync(bar, nthr);
    if (tid == 0) {
        __threadfence_system();
        for (int q = 0; q < p.tp->size; q++)
            atomicAdd_system(p.tp->cnt[q] + p.ar_kind, 1ull);
    }
}

__device__ __forceinline__ void partial_store(const GemvParams &p, int row, float acc)
{
    const size_t off = (size_t)p.tp->rank * p.N + row;
    for (int q = 0; q < p.tp->size; q++)
        p.tp->ar[p.ar_kind][q][off] = acc;
}

// ------------------------------------------------------------- block dots
__device__ __forceinline__ int dot_block_q4(const uint4 wv, const uint4 ae, const uint4 ao, int acc)
{
    const uint32_t m = 0x0F0F0F0Fu;
    acc = __dp4a((int)(wv.x & m), (int)ae.x, acc);
    acc = __dp4a((int)((wv.x >> 4) & m), (int)ao.x, acc);
    acc = __dp4a((int)(wv.y & m), (int)ae.y, acc);
    acc = __dp4a((int)((wv.y >> 4) & m), (int)ao.y, acc);
    acc = __dp4a((int)(wv.z & m), (int)ae.z, acc);
    acc = __dp4a((int)((wv.z >> 4) & m), (int)ao.z, acc);
    acc = __dp4a((int)(wv.w & m), (int)ae.w, acc);
    acc = __dp4a((int)((wv.w >> 4) & m), (int)ao.w, acc);
    return acc;
}

__device__ __forceinline__ int dot_block_q8(const uint4 w0, const uint4 w1, const uint4 a0, const uint4 a1, int acc)
{
    acc = __dp4a((int)w0.x, (int)a0.x, acc);
    acc = __dp4a((int)w0.y, (int)a0.y, acc);
    acc = __dp4a((int)w0.z, (int)a0.z, acc);
    acc = __dp4a((int)w0.w, (int)a0.w, acc);
    acc = __dp4a((int)w1.x, (int)a1.x, acc);
    acc = __dp4a((int)w1.y, (int)a1.y, acc);
    acc = __dp4a((int)w1.z, (int)a1.z, acc);
    acc = __dp4a((int)w1.w, (int)a1.w, acc);
    return acc;
}

template <int ST>
__device__ __forceinline__ float load_scale(const uint8_t *base, int idx)
{
    if (ST == 0)
        return __half2float(reinterpret_cast<const __half *>(base)[idx]);
    return reinterpret_cast<const float *>(base)[idx];
}

// 2-D tensor-map TMA load of a box at (x, y) into shared memory
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                            uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Publish the step's greedy token: CTA max -> global atomicMax; the last CTA
// writes the token, logs it and advances the decode position.
__device__ void argmax_finalize(const GemvParams &p, unsigned long long key, int tid, int nthr, int bar)
{
    __shared__ unsigned long long s_key[32];
    const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
    }
    if (lane == 0)
        s_key[warp] = key;
    named_bar_sync(bar, nthr);
    if (tid == 0) {
        unsigned long long k = s_key[0];
        for (int w = 1; w < nthr / 32; w++)
            k = s_key[w] > k ? s_key[w] : k;
        atomicMax(&p.state->key, k);
        __threadfence();
        const unsigned int ticket = atomicAdd(&p.state->done, 1u);
        if (ticket == gridDim.x - 1) {
            __threadfence();
            unsigned long long best = atomicAdd(&p.state->key, 0ull);
            StepState *st = p.state;
            const unsigned long long epoch = st->epoch;
            if (p.tp && p.tp->size > 1) { // every rank holds a vocab shard: exchange the best keys
                const TpLink *tp = p.tp;
                for (int q = 0; q < tp->size; q++)
                    tp->keys[q][tp->rank] = best;
                __threadfence_system();
                for (int q = 0; q < tp->size; q++)
                    atomicAdd_system(tp->cnt[q] + TP_CNT_KEY, 1ull);
                if (wait_counter(tp->cnt[tp->rank] + TP_CNT_KEY, (epoch + 1) * (unsigned long long)tp->size, p.err))
                    for (int q = 0; q < tp->size; q++) {
                        const unsigned long long k = __ldcg(tp->keys[tp->rank] + q);
                        best = k > best ? k : best;
                    }
            }
            const int tok = (int)argmax_key_index(best);
            const int n = st->n_log;
            if (p.token_log && n < st->log_cap)
                p.token_log[n] = tok;
            st->n_log = n + 1;
            st->token = tok;
            st->pos = st->pos + 1;
            st->key = 0ull;
            st->done = 0u;
            st->epoch = epoch + 1;
            __threadfence();
        }
    }
}

template <int WF, int ST, int PRO, int EPI>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap ts, const GemvParams p)
{
    constexpr int WB = wbytes_per_block(WF);
    constexpr int W_ROW = CB * WB;       // bytes of one row of a chunk (512 / 1024)
    constexpr int S_ROW = CB * sbytes(ST);
    extern __shared__ __align__(128) uint8_t smem_raw[];

    griddep_launch_dependents();
    LLMRS_TRACE_PROLOG

    uint8_t *smem = smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u);
    const int S = p.n_stages;
    const int K = p.K, nb = K >> 5;
    const int nchunks = (nb + CB - 1) / CB;
    const SmemLayout L = smem_layout(WF, ST, K, S);
    uint32_t *act = reinterpret_cast<uint32_t *>(smem + L.act_off);
    float *act_s = reinterpret_cast<float *>(smem + L.acts_off);
    int *act_c = reinterpret_cast<int *>(smem + L.actc_off);
    float *tbuf = reinterpret_cast<float *>(smem + L.tb_off);
    float *linkbuf = reinterpret_cast<float *>(smem + L.link_off);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar_off);
    uint64_t *empty = full + S;
    uint64_t *link = empty + S;   // link[w]: warp w hands its rows' running sums on
    uint64_t *issued = link + NW; // every consumer warp has requested its activation
    float *red = reinterpret_cast<float *>(smem + L.red_off);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // TPS tile sets are worked on at once (4 when the CTA has >= 4 tiles, else
    // 2 or 1); the GT = NG / TPS groups of a set take its (tile, chunk) steps
    // u = 0, 1, ... in turn, group q of the set taking u = q, q + GT, ...  With
    // GT = 1 a row's running sum stays in registers; with GT > 1 it is handed
    // from group to group through shared memory (one mbarrier per warp), which
    // keeps the reference's block order while GT chunks are computed at once.
    // Group g also owns ring stages g, g + NG, ...: a stage barrier is only
    // awaited by the group that consumed its previous phase.
    const int SPG = S / NG; // stages per group
    const int B = p.box_rows;
    const int r0 = blockIdx.x * p.rows_per_cta;
    const int r1 = min(p.N, r0 + p.rows_per_cta);
    const int ntiles = (r1 - r0 + B - 1) / B;
    const int TPS_rt = ntiles >= NG ? NG : (ntiles >= 2 ? 2 : 1);
    const int GT_rt = NG / TPS_rt;
    auto group_iters = [&](int g) {
        const int set = g % TPS_rt, q = g / TPS_rt;
        const int nset = ntiles > set ? (ntiles - 1 - set) / TPS_rt + 1 : 0;
        const int U = nset * nchunks;
        return U > q ? (U - 1 - q) / GT_rt + 1 : 0;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], WPG); // released by the group's warps
        }
        for (int w = 0; w < NW; w++)
            mbar_init(&link[w], 1);
        mbar_init(issued, NW);
        fence_mbar_init();
        trace_start(p.trace, p.trace_slot);
    }
    __syncthreads();

    if (warp == NW) {
        // ------------------------------------------------------------ producer
        // Weights do not depend on the previous kernel: the first n_pre stages
        // stream right away, the rest once the consumers have requested the
        // activation (queued behind the weight stream it would arrive last).
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            const uint32_t stage_tx = (uint32_t)(B * (W_ROW + S_ROW)); // whole boxes (OOB is zero-filled)
            const int pre = min(p.n_pre, S);
            // One thread issues every stage, so its loop is kept free of
            // divisions: per group, the step's chunk and tile advance by GT.
            int gi[NG], gc[NG], gt[NG];
#pragma unroll
            for (int g = 0; g < NG; g++) {
                gi[g] = group_iters(g);
                gc[g] = g / TPS_rt; // first step u = q: chunk u % nchunks of tile set g % TPS_rt
                gt[g] = g % TPS_rt;
                while (gc[g] >= nchunks) {
                    gc[g] -= nchunks;
                    gt[g] += TPS_rt;
                }
            }
            const int spg_shift = SPG == 2 ? 1 : 0; // stages are 4 or 8: SPG is 1 or 2
            int issued_n = 0;
            for (int k = 0; k < gi[0]; k++) { // group 0 has the most steps
                const int slot = k & (SPG - 1), use = k >> spg_shift;
#pragma unroll
                for (int g = 0; g < NG; g++) {
                    if (k >= gi[g])
                        continue;
                    if (issued_n++ == pre && !mbar_wait(issued, 0, p.err))
                        return;
                    const int s = g + NG * slot;
                    LLMRS_TRACE_BEGIN(0);
                    if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, p.err))
                        return;
                    LLMRS_TRACE_END(0);
                    const int y = r0 + gt[g] * B, c = gc[g];
                    uint8_t *st = smem + (size_t)s * L.stage_bytes;
                    mbar_arrive_expect_tx(&full[s], stage_tx);
                    tma_load_2d(st, &tw, c * (W_ROW / 4), y, &full[s], pol);
                    tma_load_2d(st + L.scale_off, &ts, c * CB, y, &full[s], pol);
                    gc[g] += GT_rt;
                    while (gc[g] >= nchunks) {
                        gc[g] -= nchunks;
                        gt[g] += TPS_rt;
                    }
                }
            }
            LLMRS_TRACE_FLUSH(1);
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    LLMRS_TRACE_BEGIN(1);
    griddep_wait();
    LLMRS_TRACE_END(1);
    LLMRS_TRACE_BEGIN(2);
    const int ctid = threadIdx.x;
    if (ctid == 0)
        trace_go(p.trace, p.trace_slot);
    load_activation<WF, PRO>(p, act, act_s, act_c, red, ctid, PRO_THREADS, 1, issued);
    named_bar_sync(1, PRO_THREADS);
    if (ctid == 0)
        trace_ready(p.trace, p.trace_slot);
    LLMRS_TRACE_END(2);

    // warp (grp, wq): group grp = warp / WPG takes every chunk of tiles grp,
    // grp + NG, ...; wq = warp % WPG takes tile rows wq*RPW .. +RPW-1.  Lane l =
    // block l of the chunk.
    const int grp = warp / WPG, wq = warp % WPG;
    float *tb = tbuf + (size_t)warp * RPW * TBS;
    // transposed roles: lane j sums row ri = j % RPW over blocks seg*8 .. seg*8+7
    const int ri = lane % RPW, seg = lane / RPW;
    unsigned long long best = 0ull;
    bool ok = true;
    // the step loop, specialised for the number of groups per tile set
    auto steps = [&](auto gt_tag) {
    constexpr int GT = decltype(gt_tag)::value;
    constexpr int TPS = NG / GT;
    float acc = 0.0f; // running sum of row ri (complete in the segment-3 lanes)
    const int tset = grp % TPS, q = grp / TPS;
    const int prevw = (tset + TPS * ((q + GT - 1) % GT)) * WPG + wq; // previous step's warp
    const int my_iters = group_iters(grp);
    int c = q, tile = tset; // this group's first step u = q
    while (c >= nchunks) {
        c -= nchunks;
        tile += TPS;
    }
    for (int k = 0; k < my_iters; k++) {
        if (k > 0) { // next step: u += GT
            c += GT;
            while (c >= nchunks) {
                c -= nchunks;
                tile += TPS;
            }
        }
        const int s = grp + NG * (k & (SPG - 1));
        const int u = k * GT + q;
        const int trow0 = r0 + tile * B;
        const int rows = min(B, r1 - trow0);
        const int nbc = min(CB, nb - c * CB);
        LLMRS_TRACE_BEGIN(3);
        if (ok && !mbar_wait(&full[s], (uint32_t)((SPG == 2 ? k >> 1 : k) & 1), p.err))
            ok = false;
        LLMRS_TRACE_END(3);
        LLMRS_TRACE_BEGIN(4);
        const uint8_t *st = smem + (size_t)s * L.stage_bytes;
        float t[RPW];
        {
            const int b = c * CB + min(lane, nbc - 1);
            const uint4 a0 = reinterpret_cast<const uint4 *>(act)[2 * b];
            const uint4 a1 = reinterpret_cast<const uint4 *>(act)[2 * b + 1];
            const float sa = act_s[b];
            const int cz = act_c[b];
#pragma unroll
            for (int i = 0; i < RPW; i++) {
                const int lr = wq * RPW + i;
                const uint8_t *wrow = st + (size_t)lr * W_ROW;
                int isum;
                if (WF == 0) {
                    const uint4 wv = *reinterpret_cast<const uint4 *>(wrow + lane * 16);
                    isum = dot_block_q4(wv, a0, a1, cz);
                } else {
                    const uint4 *wp = reinterpret_cast<const uint4 *>(wrow + lane * 32);
                    isum = dot_block_q8(wp[0], wp[1], a0, a1, cz);
                }
                const float sw = load_scale<ST>(st + L.scale_off + (size_t)lr * S_ROW, lane);
                t[i] = __fmul_rn((float)isum, __fmul_rn(sw, sa));
            }
        }
        // products are in registers: hand the stage back to the producer
        __syncwarp();
        if (lane == 0)
            mbar_arrive(&empty[s]);
        // transpose: lane j then holds row ri's products for blocks seg*8 .. +7
#pragma unroll
        for (int i = 0; i < RPW; i++)
            tb[i * TBS + lane] = t[i];
        __syncwarp();
        const float4 v0 = *reinterpret_cast<const float4 *>(tb + ri * TBS + seg * 8);
        const float4 v1 = *reinterpret_cast<const float4 *>(tb + ri * TBS + seg * 8 + 4);
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        if (GT == 1) { // the running sum moves from the segment-3 lane to the segment-0 lane
            const float carry = __shfl_sync(0xffffffffu, acc, 3 * RPW + ri);
            acc = (c > 0 && seg == 0) ? carry : 0.0f;
        } else { // ... or arrives from the previous step's warp
            acc = 0.0f;
            if (u > 0) {
                const int kp = q > 0 ? k : k - 1; // that warp's step index
                if (ok && !mbar_wait(&link[prevw], (uint32_t)(kp & 1), p.err))
                    ok = false;
                if (c > 0 && seg == 0)
                    acc = linkbuf[prevw * RPW + ri];
            }
        }
        // add the chunk's blocks in order: segment 0 first, then 1, 2, 3
        const bool live_row = wq * RPW + ri < rows;
#pragma unroll
        for (int sg = 0; sg < 4; sg++) {
            if (sg > 0) {
                const float prev = __shfl_up_sync(0xffffffffu, acc, RPW);
                if (seg == sg)
                    acc = prev;
            }
            if (seg == sg && live_row) {
#pragma unroll
                for (int k = 0; k < 8; k++)
                    if (sg * 8 + k < nbc)
                        acc = __fadd_rn(acc, v[k]);
            }
        }
        if (GT > 1) {
            __syncwarp();
            if (seg == 3)
                linkbuf[warp * RPW + ri] = acc;
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&link[warp]);
        }
        LLMRS_TRACE_END(4);
        if (c == nchunks - 1) {
            // ---- epilogue: lanes of segment 3 hold the complete rows
            const int row = trow0 + wq * RPW + ri;
            const bool valid = seg == 3 && live_row;
            if (EPI == EPI_STORE) {
                if (valid)
                    p.y[row] = acc;
            } else if (EPI == EPI_RESIDUAL) {
                if (valid)
                    p.y[row] = __fadd_rn(acc, p.residual[row]);
            } else if (EPI == EPI_SILU) {
                const float up = __shfl_down_sync(0xffffffffu, acc, 1);
                if (valid && (row & 1) == 0) {
                    const float silu = __fdiv_rn(acc, __fadd_rn(1.0f, expf(-acc)));
                    p.y[row >> 1] = __fmul_rn(silu, up);
                }
            } else if (EPI == EPI_ARGMAX) {
                if (valid) {
                    if (p.y)
                        p.y[row] = acc;
                    const unsigned long long k = argmax_key(acc, (uint32_t)(row + p.row_offset));
                    best = k > best ? k : best;
                }
            } else if (EPI == EPI_PARTIAL) {
                if (valid)
                    partial_store(p, row, acc);
            }
        }
    }
    };
    if (GT_rt == 1)
        steps(std::integral_constant<int, 1>{});
    else if (GT_rt == 2)
        steps(std::integral_constant<int, 2>{});
    else
        steps(std::integral_constant<int, 4>{});
    if (EPI == EPI_PARTIAL)
        partial_signal(p, ctid, PRO_THREADS, 1);
    if (EPI == EPI_ARGMAX)
        argmax_finalize(p, best, ctid, PRO_THREADS, 1);
    LLMRS_TRACE_FLUSH(0);
    if (ctid == 0)
        trace_end(p.trace, p.trace_slot);
}

// ------------------------------------------------------------------ fallback
// One thread per output row, same arithmetic; activation quantised into smem.
constexpr int SIMPLE_THREADS = 256;

template <int WF, int ST, int PRO, int EPI>
__global__ void __launch_bounds__(SIMPLE_THREADS) gemv_simple_kernel(const GemvParams p)
{
    extern __shared__ __align__(16) uint8_t smem[];
    griddep_launch_dependents();
    const int K = p.K, nb = K >> 5;
    uint32_t *act = reinterpret_cast<uint32_t *>(smem);
    float *act_s = reinterpret_cast<float *>(smem + (size_t)nb * 32);
    int *act_c = reinterpret_cast<int *>(act_s + nb);
    float *red = reinterpret_cast<float *>(act_c + nb);
    griddep_wait();
    load_activation<WF, PRO>(p, act, act_s, act_c, red, threadIdx.x, SIMPLE_THREADS, 1, nullptr);
    named_bar_sync(1, SIMPLE_THREADS);
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    unsigned long long best = 0ull;
    float row_acc = 0.0f;
    if (row < p.N) {
        const uint8_t *sb = reinterpret_cast<const uint8_t *>(p.scales) + (size_t)row * nb * sbytes(ST);
        float acc = 0.0f;
        for (int b = 0; b < nb; b++) {
            int isum;
            const uint4 a0 = reinterpret_cast<const uint4 *>(act)[2 * b];
            const uint4 a1 = reinterpret_cast<const uint4 *>(act)[2 * b + 1];
            if (WF == 0) {
                const uint8_t *wp = p.w + (size_t)row * (K / 2) + (size_t)b * 16;
                uint4 wv;
                wv.x = wp[0] | (wp[1] << 8) | (wp[2] << 16) | ((uint32_t)wp[3] << 24);
                wv.y = wp[4] | (wp[5] << 8) | (wp[6] << 16) | ((uint32_t)wp[7] << 24);
                wv.z = wp[8] | (wp[9] << 8) | (wp[10] << 16) | ((uint32_t)wp[11] << 24);
                wv.w = wp[12] | (wp[13] << 8) | (wp[14] << 16) | ((uint32_t)wp[15] << 24);
                isum = dot_block_q4(wv, a0, a1, act_c[b]);
            } else {
                const uint8_t *wp = p.w + (size_t)row * K + (size_t)b * 32;
                uint4 w0, w1;
                uint32_t *ww0 = &w0.x, *ww1 = &w1.x;
                for (int i = 0; i < 4; i++) {
                    ww0[i] = wp[4 * i] | (wp[4 * i + 1] << 8) | (wp[4 * i + 2] << 16) | ((uint32_t)wp[4 * i + 3] << 24);
                    ww1[i] = wp[16 + 4 * i] | (wp[16 + 4 * i + 1] << 8) | (wp[16 + 4 * i + 2] << 16) |
                             ((uint32_t)wp[16 + 4 * i + 3] << 24);
                }
                isum = dot_block_q8(w0, w1, a0, a1, act_c[b]);
            }
            const float sw = load_scale<ST>(sb, b);
            acc = __fadd_rn(acc, __fmul_rn((float)isum, __fmul_rn(sw, act_s[b])));
        }
        row_acc = acc;
        if (EPI == EPI_STORE) {
            p.y[row] = acc;
        } else if (EPI == EPI_RESIDUAL) {
            p.y[row] = __fadd_rn(acc, p.residual[row]);
        } else if (EPI == EPI_ARGMAX) {
            if (p.y)
                p.y[row] = acc;
            best = argmax_key(acc, (uint32_t)(row + p.row_offset));
        } else if (EPI == EPI_PARTIAL) {
            partial_store(p, row, acc);
        }
    }
    if (EPI == EPI_PARTIAL)
        partial_signal(p, threadIdx.x, SIMPLE_THREADS, 1);
    if (EPI == EPI_SILU) {
        // rows (2i, 2i+1) are threads (2i, 2i+1) of this block
        __shared__ float rows_acc[SIMPLE_THREADS];
        rows_acc[threadIdx.x] = row_acc;
        __syncthreads();
        if (row < p.N && (row & 1) == 0 && row + 1 < p.N) {
            const float g = row_acc, up = rows_acc[threadIdx.x + 1];
            const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
            p.y[row >> 1] = __fmul_rn(silu, up);
        }
    }
    if (EPI == EPI_ARGMAX)
        argmax_finalize(p, best, threadIdx.x, SIMPLE_THREADS, 1);
}

constexpr int SIMPLE_SMEM_MAX = 200 * 1024;

template <int WF, int ST, int PRO, int EPI>
cudaError_t prepare_one()
{
    cudaError_t e = cudaFuncSetAttribute(gemv_tma_kernel<WF, ST, PRO, EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BUDGET + 2048);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemv_simple_kernel<WF, ST, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 SIMPLE_SMEM_MAX);
    return e;
}

template <int WF, int ST, int PRO, int EPI>
int launch_one(const GemvPlan &plan, const GemvParams &p0, cudaStream_t stream, bool pdl)
{
    GemvParams p = p0;
    if (plan.fast) {
        p.n_stages = plan.stages;
        p.n_pre = gemv_prefetch_stages();
        p.box_rows = plan.box_rows;
        p.rows_per_cta = plan.rows_per_cta;
        LLMRS_CUDA_TRY(launch(gemv_tma_kernel<WF, ST, PRO, EPI>, dim3(plan.grid), dim3(NTHREADS), plan.smem, stream,
                              pdl, plan.tw, plan.ts, p));
    } else {
        const int nb = p.K / 32;
        size_t smem = (size_t)nb * 40 + 64;
        LLMRS_CHECK_ARG(smem <= (size_t)SIMPLE_SMEM_MAX, "gemv: K=%d too large", p.K);
        int grid = (p.N + SIMPLE_THREADS - 1) / SIMPLE_THREADS;
        LLMRS_CUDA_TRY(
            launch(gemv_simple_kernel<WF, ST, PRO, EPI>, dim3(grid), dim3(SIMPLE_THREADS), smem, stream, pdl, p));
    }
    return LLMRS_OK;
}

} // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

namespace {

// 2-D map over `rows` rows of `row_bytes` bytes viewed as `elem`-byte elements
int encode_2d(CUtensorMap *map, const void *base, int elem, size_t row_bytes, int rows, int box_x, int box_y,
              CUtensorMapSwizzle swizzle)
{
    auto fn = tensor_map_encoder();
    if (!fn)
        return fail(LLMRS_ECUDA, "cuTensorMapEncodeTiled unavailable");
    const CUtensorMapDataType dt = elem == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT32;
    cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / elem), (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_y};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(LLMRS_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return LLMRS_OK;
}

} // namespace

static size_t smem_bytes_for(int wf, int st, int K, int *stages)
{
    int best = 0;
    for (int s = MAX_STAGES; s >= NG; s -= NG) { // each warp group owns stages/NG of them
        if (smem_layout(wf, st, K, s).total <= SMEM_BUDGET) {
            best = s;
            break;
        }
    }
    if (stages)
        *stages = best;
    return best ? smem_layout(wf, st, K, best).total : 0;
}

int gemv_plan(GemvPlan *plan, const void *w, const void *scales, int N, int K, int wf, int st, bool pairs, int sms)
{
    LLMRS_CHECK_ARG(plan && w && scales, "gemv_plan: NULL argument");
    LLMRS_CHECK_ARG(K > 0 && K % 32 == 0, "gemv: K=%d must be a positive multiple of 32", K);
    LLMRS_CHECK_ARG(N > 0, "gemv: N=%d must be positive", N);
    LLMRS_CHECK_ARG(!pairs || N % 2 == 0, "gemv: paired rows need an even row count");
    *plan = GemvPlan();
    plan->wf = wf;
    plan->st = st;
    plan->N = N;
    plan->K = K;
    const bool aligned = !((uintptr_t)w & 15) && !((uintptr_t)scales & 15);
    int stages = 0;
    const size_t smem = smem_bytes_for(wf, st, K, &stages);
    if (K % 256 != 0 || !aligned || smem == 0 || N < 2)
        return LLMRS_OK; // simple kernel
    // rows per CTA so that the grid covers the SMs once, in tiles of <= 32 rows
    int rc = (N + sms - 1) / sms;
    if (pairs)
        rc += rc & 1;
    const int ntiles = (rc + TR - 1) / TR;
    int box = (rc + ntiles - 1) / ntiles;
    if (pairs)
        box += box & 1;
    plan->box_rows = box;
    plan->rows_per_cta = ntiles * box;
    plan->grid = (N + plan->rows_per_cta - 1) / plan->rows_per_cta;
    plan->stages = stages;
    plan->smem = smem;
    const size_t wrow = wf == 0 ? (size_t)K / 2 : (size_t)K;
    // codes: boxes of box rows x 512 (Q4) / 1024 (Q8) bytes
    LLMRS_TRY(encode_2d(&plan->tw, w, 4, wrow, N, CB * wbytes_per_block(wf) / 4, box, CU_TENSOR_MAP_SWIZZLE_NONE));
    LLMRS_TRY(encode_2d(&plan->ts, scales, sbytes(st), (size_t)(K / 32) * sbytes(st), N, CB, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE));
    plan->fast = 1;
    return LLMRS_OK;
}

// every (weight format, scale dtype, prologue, epilogue) the op-level API and the decode step use
#define LLMRS_GEMV_VARIANTS(X)                                                                             \
    X(0, 0, PRO_F32, EPI_STORE) X(0, 0, PRO_NORM, EPI_STORE) X(0, 0, PRO_EMBED_NORM, EPI_STORE)            \
    X(0, 0, PRO_F32, EPI_RESIDUAL) X(0, 0, PRO_NORM, EPI_SILU) X(0, 0, PRO_NORM, EPI_ARGMAX)               \
    X(0, 1, PRO_F32, EPI_STORE) X(0, 1, PRO_NORM, EPI_STORE) X(0, 1, PRO_EMBED_NORM, EPI_STORE)            \
    X(0, 1, PRO_F32, EPI_RESIDUAL) X(0, 1, PRO_NORM, EPI_SILU) X(0, 1, PRO_NORM, EPI_ARGMAX)               \
    X(1, 0, PRO_F32, EPI_STORE) X(1, 0, PRO_NORM, EPI_STORE) X(1, 0, PRO_EMBED_NORM, EPI_STORE)            \
    X(1, 0, PRO_F32, EPI_RESIDUAL) X(1, 0, PRO_NORM, EPI_SILU) X(1, 0, PRO_NORM, EPI_ARGMAX)               \
    X(1, 1, PRO_F32, EPI_STORE) X(1, 1, PRO_NORM, EPI_STORE) X(1, 1, PRO_EMBED_NORM, EPI_STORE)            \
    X(1, 1, PRO_F32, EPI_RESIDUAL) X(1, 1, PRO_NORM, EPI_SILU) X(1, 1, PRO_NORM, EPI_ARGMAX)               \
    X(0, 0, PRO_Q8, EPI_RESIDUAL) X(0, 1, PRO_Q8, EPI_RESIDUAL) X(1, 0, PRO_Q8, EPI_RESIDUAL)             \
    X(1, 1, PRO_Q8, EPI_RESIDUAL)                                                                          \
    X(0, 0, PRO_F32, EPI_PARTIAL) X(0, 0, PRO_AR_NORM, EPI_STORE) X(0, 0, PRO_AR_NORM, EPI_SILU)           \
    X(0, 0, PRO_AR_NORM, EPI_ARGMAX) X(0, 1, PRO_F32, EPI_PARTIAL) X(0, 1, PRO_AR_NORM, EPI_STORE)         \
    X(0, 1, PRO_AR_NORM, EPI_SILU) X(0, 1, PRO_AR_NORM, EPI_ARGMAX) X(1, 0, PRO_F32, EPI_PARTIAL)          \
    X(1, 0, PRO_AR_NORM, EPI_STORE) X(1, 0, PRO_AR_NORM, EPI_SILU) X(1, 0, PRO_AR_NORM, EPI_ARGMAX)        \
    X(1, 1, PRO_F32, EPI_PARTIAL) X(1, 1, PRO_AR_NORM, EPI_STORE) X(1, 1, PRO_AR_NORM, EPI_SILU)           \
    X(1, 1, PRO_AR_NORM, EPI_ARGMAX)

int gemv_launch(const GemvPlan &plan, const GemvParams &p, int pro, int epi, cudaStream_t stream, bool pdl)
{
    LLMRS_CHECK_ARG(p.N == plan.N && p.K == plan.K, "gemv: params do not match the plan");
    LLMRS_CHECK_ARG(epi != EPI_SILU || p.N % 2 == 0, "gemv: SiLU epilogue needs an even row count");
    const int wf = plan.wf, st = plan.st;
#define LLMRS_GEMV_CASE(WF, ST, PRO, EPI)                                                                   \
    if (wf == WF && st == ST && pro == PRO && epi == EPI)                                                  \
        return launch_one<WF, ST, PRO, EPI>(plan, p, stream, pdl);
    LLMRS_GEMV_VARIANTS(LLMRS_GEMV_CASE)
#undef LLMRS_GEMV_CASE
    return fail(LLMRS_ENOTSUP, "gemv: unsupported variant wf=%d st=%d pro=%d epi=%d", wf, st, pro, epi);
}

int gemv_grid(const GemvPlan &plan)
{
    return plan.fast ? plan.grid : (plan.N + SIMPLE_THREADS - 1) / SIMPLE_THREADS;
}

int gemv_prefetch_stages(void)
{
    static const int n = [] {
        const char *e = getenv("LLMRS_GEMV_PREFETCH");
        const int v = e ? atoi(e) : 0;
        return v < 0 ? 0 : v;
    }();
    return n;
}

int gemv_prepare(void)
{
    cudaError_t e = cudaSuccess;
#define LLMRS_GEMV_PREP(WF, ST, PRO, EPI)                                                                   \
    if (e == cudaSuccess)                                                                                  \
        e = prepare_one<WF, ST, PRO, EPI>();
    LLMRS_GEMV_VARIANTS(LLMRS_GEMV_PREP)
#undef LLMRS_GEMV_PREP
    if (e != cudaSuccess)
        return fail(LLMRS_ECUDA, "gemv kernel attributes: %s", cudaGetErrorString(e));
    return LLMRS_OK;
}

} // namespace llmrs
