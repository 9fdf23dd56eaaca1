// gemv_core.cuh - device side of the batch-1 Q4_0 / Q8_0 GEMV: shared-memory
// layout, activation prologue, block dots, the producer (weight stream) and
// the consumer (dp4a products, in-order row sums, epilogues), used by
// gemv.cu.  Arithmetic: see gemv.cu.
#pragma once

#include <cudaTypedefs.h>
#include <cuda_fp16.h>

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
constexpr int NSUM = 2;                  // summer warps: in-order row sums when groups share a tile
constexpr int NTHREADS = (NW + NSUM + 1) * 32; // + summers + producer warp
constexpr int TR = 32;                   // max rows per tile
constexpr int CB = 32;                   // blocks per chunk (1024 weights), one per lane
constexpr int TBS = 36;                  // transpose row stride (floats): 16-byte aligned, conflict-free
constexpr int PSLOTS = 8;                // product slots [TR rows][TBS] shared by the tile sets of a CTA
constexpr size_t SMEM_BUDGET = 224 * 1024; // one CTA per SM: use most of the SM's shared memory
constexpr int MAX_STAGES = 8;
constexpr int PRO_THREADS = NW * 32;

__host__ __device__ constexpr int wbytes_per_block(int wf) { return wf == 0 ? 16 : 32; }
__host__ __device__ constexpr int sbytes(int st) { return st == 0 ? 2 : 4; }
__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) & ~(a - 1); }

struct SmemLayout {
    size_t stage_bytes, scale_off, act_off, acts_off, actc_off, tb_off, bar_off, red_off, total;
};

// bytes of the region that holds either the per-warp transpose buffers (one
// group per tile) or the product slots (groups sharing a tile): a CTA uses one
__host__ __device__ constexpr size_t tb_region_bytes()
{
    return (size_t)NW * RPW * TBS * 4 > (size_t)PSLOTS * TR * TBS * 4 ? (size_t)NW * RPW * TBS * 4
                                                                     : (size_t)PSLOTS * TR * TBS * 4;
}

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
    L.bar_off = align_up(L.tb_off + tb_region_bytes(), 16);
    // full, empty, activation-issued, product full / empty, summers' argmax key
    L.red_off = L.bar_off + (size_t)(2 * stages + 1 + 2 * PSLOTS + 1) * 8;
    L.total = align_up(L.red_off + 16 * 4, 16) + 128; // + slack to align the base
    return L;
}

// ------------------------------------------------------------- activation
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

// Quantise one 32-value block held by 8 consecutive lanes (4 values each,
// lane j of the group: elements 4j .. 4j+3) to Q8_0 exactly like
// quantize_row_q8_0, and store its 8 packed words (one per lane), its scale
// and (Q4) the -8*sum(q) offset.
template <int WF>
__device__ __forceinline__ void quantize_block8(const float (&v)[4], int j, bool live, uint32_t *dst_words,
                                                float *dst_s, int *dst_c)
{
    float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1)
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o, 8));
    float scale = 0.0f, inv = 0.0f;
    if (amax != 0.0f) {
        scale = __fdiv_rn(amax, 127.0f);
        inv = __fdiv_rn(1.0f, scale);
    }
    int q[4];
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float r = roundf(__fmul_rn(v[i], inv));
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        q[i] = (amax == 0.0f || r != r) ? 0 : (int)r;
        sum += q[i];
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1)
        sum += __shfl_xor_sync(0xffffffffu, sum, o, 8);
    if (WF == 0) {
        // Q4 order: word k (k < 4) = elements 8k, 8k+2, 8k+4, 8k+6; word 4+k =
        // 8k+1, 8k+3, 8k+5, 8k+7 -- lanes 2k and 2k+1 hold group k
        const uint32_t ev = (uint32_t)(q[0] & 0xFF) | (uint32_t)(q[2] & 0xFF) << 8;
        const uint32_t od = (uint32_t)(q[1] & 0xFF) | (uint32_t)(q[3] & 0xFF) << 8;
        const uint32_t pev = __shfl_xor_sync(0xffffffffu, ev, 1, 8);
        const uint32_t pod = __shfl_xor_sync(0xffffffffu, od, 1, 8);
        if (!live)
            return;
        if ((j & 1) == 0)
            dst_words[j >> 1] = ev | pev << 16;
        else
            dst_words[4 + (j >> 1)] = pod | od << 16;
    } else if (live) {
        dst_words[j] = (uint32_t)(q[0] & 0xFF) | (uint32_t)(q[1] & 0xFF) << 8 | (uint32_t)(q[2] & 0xFF) << 16 |
                       (uint32_t)(q[3] & 0xFF) << 24;
    }
    if (live && j == 0) {
        *dst_s = scale;
        *dst_c = WF == 0 ? -8 * sum : 0;
    }
}

// Activation prologue over nthr threads (whole warps): a 32-value block is
// handled by 8 consecutive lanes, 4 values each, so every warp load is a
// coalesced 512-byte row and the per-block chains are 4 deep.  Warp w takes
// blocks 4*(r*nwarps + w) .. +3 in round r.  The first rounds' loads are all
// issued at once and stay in registers (across the RMSNorm reduction where
// fused): 4 rounds with a norm (x and its weights), 8 without; later rounds
// (larger K) load as they go.

// tag of a tensor-parallel exchange (kind, index) in this step: nonzero and
// different for every exchange of a kind until 2^32 of them
__device__ __forceinline__ uint32_t ar_tag(const GemvParams &p)
{
    return (uint32_t)(p.state->epoch * (unsigned long long)p.ar_per_step + (unsigned long long)p.ar_index + 1ull);
}

__device__ __forceinline__ ulonglong2 ld_volatile_u64x2(const unsigned long long *a)
{
    ulonglong2 v;
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(a) : "memory");
    return v;
}

__device__ __forceinline__ void st_volatile_u64(unsigned long long *a, unsigned long long v)
{
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}

// Tensor parallel: the sum, in rank order, of the ranks' 4 partial values at
// `off` of this rank's receive buffer ([nparts][stride] tagged 64-bit words),
// once every word carries `tag`.  Ranks go in groups of 2: a group's words are
// requested at once and only those still without the tag are polled again, so
// the wait costs about one memory round trip per group, not one per rank.
// Gives up after peer_ns (zeros, DEV_ERR_PEER_TIMEOUT).
__device__ __forceinline__ void ar_gather4(const unsigned long long *part, size_t stride, int nparts, size_t off,
                                        uint32_t tag, uint64_t peer_ns, uint32_t *err, float (&s)[4])
{
    constexpr int ARG = 2; // ranks per group
    s[0] = s[1] = s[2] = s[3] = 0.0f;
    for (int q0 = 0; q0 < nparts; q0 += ARG) {
        ulonglong2 wa[ARG], wc[ARG];
#pragma unroll
        for (int g = 0; g < ARG; g++) {
            const unsigned long long *src = part + (size_t)min(q0 + g, nparts - 1) * stride + off;
            wa[g] = ld_volatile_u64x2(src);
            wc[g] = ld_volatile_u64x2(src + 2);
        }
        auto arrived = [&](int g) {
            return (uint32_t)(wa[g].x >> 32) == tag && (uint32_t)(wa[g].y >> 32) == tag &&
                   (uint32_t)(wc[g].x >> 32) == tag && (uint32_t)(wc[g].y >> 32) == tag;
        };
        uint64_t t0 = 0;
        for (uint32_t spin = 0;; spin++) {
            bool all = true;
#pragma unroll
            for (int g = 0; g < ARG; g++)
                all = all && arrived(g);
            if (all)
                break;
#pragma unroll
            for (int g = 0; g < ARG; g++)
                if (!arrived(g)) {
                    const unsigned long long *src = part + (size_t)min(q0 + g, nparts - 1) * stride + off;
                    wa[g] = ld_volatile_u64x2(src);
                    wc[g] = ld_volatile_u64x2(src + 2);
                }
            if ((spin & 63u) == 0u) {
                const uint64_t now = globaltimer_ns();
                if (spin == 0u)
                    t0 = now;
                else if (now - t0 > peer_ns || *reinterpret_cast<volatile uint32_t *>(err) == DEV_ERR_PEER_TIMEOUT) {
                    atomicCAS(err, 0u, (uint32_t)DEV_ERR_PEER_TIMEOUT);
#pragma unroll
                    for (int g = 0; g < ARG; g++)
                        wa[g] = wc[g] = make_ulonglong2(0ull, 0ull);
                    break;
                }
            }
        }
#pragma unroll
        for (int g = 0; g < ARG; g++) {
            if (q0 + g >= nparts)
                break;
            const float w[4] = {__uint_as_float((uint32_t)wa[g].x), __uint_as_float((uint32_t)wa[g].y),
                                __uint_as_float((uint32_t)wc[g].x), __uint_as_float((uint32_t)wc[g].y)};
#pragma unroll
            for (int i = 0; i < 4; i++)
                s[i] = (q0 + g == 0) ? w[i] : __fadd_rn(s[i], w[i]);
        }
    }
}

// dep_wait: this thread has not yet waited for the previous kernel; the loads
// that do not depend on it (RMSNorm weights) are issued first, then the wait.
// `pro` is a GemvPro: a run-time value in the decode kernel (one binary serves
// every prologue, so the step's kernels share their code in the instruction
// cache), a constant where a caller inlines it for one prologue.
template <int WF, bool TPK = false>
__device__ __forceinline__ void load_activation(const GemvParams &p, const int pro, uint32_t *act, float *act_s,
                                                int *act_c, float *red, int tid, int nthr, int bar, uint64_t *issued,
                                                bool dep_wait = false)
{
    const int K = p.K, nb = K >> 5;
    const bool has = tid < nb;
    // TPK: this instantiation serves tensor-parallel launches (the peer-polling
    // prologue is compiled only there, out of the single-GPU kernel)
    const bool NORM = pro == PRO_NORM || pro == PRO_EMBED_NORM || (TPK && pro == PRO_AR_NORM);
    const bool AR = TPK && pro == PRO_AR_NORM;
    const bool EARLY_W = pro == PRO_NORM || pro == PRO_EMBED_NORM; // norm weights loaded before the wait
    if (!EARLY_W && dep_wait) {
        griddep_wait();
        if (tid == 0)
            trace_go(p.trace, p.trace_slot);
    }
    if (pro == PRO_Q8) {
        uint4 c0 = make_uint4(0, 0, 0, 0), c1 = c0;
        float xs = 0.0f;
        if (has) {
            c0 = __ldcg(reinterpret_cast<const uint4 *>(p.xq + (size_t)tid * 32));
            c1 = __ldcg(reinterpret_cast<const uint4 *>(p.xq + (size_t)tid * 32) + 1);
            xs = __ldcg(p.xs + tid);
        }
        signal_issued(issued, tid);
        if (has) {
            pack_q8_block<WF>(c0, c1, act + (size_t)tid * 8, act_c + tid);
            act_s[tid] = xs;
        }
        for (int b = tid + nthr; b < nb; b += nthr) {
            const uint4 d0 = __ldcg(reinterpret_cast<const uint4 *>(p.xq + (size_t)b * 32));
            const uint4 d1 = __ldcg(reinterpret_cast<const uint4 *>(p.xq + (size_t)b * 32) + 1);
            pack_q8_block<WF>(d0, d1, act + (size_t)b * 8, act_c + b);
            act_s[b] = __ldcg(p.xs + b);
        }
        return;
    }
    // Register buffer of 8 rounds: x in rounds [0, XR); with a norm, its
    // weights for rounds 0..3 sit in buf[4..7].
    constexpr int NBUF = 8;
    const int XR = NORM ? 4 : 8;
    const int warp = tid >> 5, lane = tid & 31, sub = lane >> 3, j = lane & 7;
    const int nwarps = nthr >> 5;
    const int rounds = (nb + 4 * nwarps - 1) / (4 * nwarps);
    const float *x = p.x;
    if (pro == PRO_EMBED_NORM) {
        int tok = p.state->token;
        if (tok < 0 || tok >= p.vocab) {
            if (tid == 0)
                atomicCAS(p.err, 0u, (uint32_t)DEV_ERR_BAD_TOKEN);
            tok = 0;
        }
        x = p.embed + (size_t)tok * K;
    }
    const unsigned long long *part = nullptr; // AR: this rank's receive buffer [size][K]
    int nparts = 0;
    uint32_t tag = 0;
    if (AR) {
        // the weight stream need not wait for the other ranks
        signal_issued(issued, tid);
        const TpLink *tp = p.tp;
        part = tp->ar[p.ar_kind][tp->rank];
        nparts = tp->size;
        tag = ar_tag(p);
    }
    // AR: a rank's 8-byte words carry this exchange's tag (each word is
    // written whole, so a matching tag means its value is the one sent); the
    // wait gives up after p.peer_ns (default 5 s)
    const uint64_t peer_ns = p.peer_ns ? p.peer_ns : 5000000000ull;
    // the 4 values of block b this lane holds: x, or (AR) the ranks' partial
    // sums in rank order, then + x
    auto load4 = [&](int b, float (&u)[4]) {
        const size_t off = (size_t)b * 32 + 4 * j;
        const float4 t = __ldcg(reinterpret_cast<const float4 *>(x + off));
        u[0] = t.x;
        u[1] = t.y;
        u[2] = t.z;
        u[3] = t.w;
        if (AR) {
            float s[4];
            ar_gather4(part, (size_t)K, nparts, off, tag, peer_ns, p.err, s);
#pragma unroll
            for (int i = 0; i < 4; i++)
                u[i] = __fadd_rn(s[i], u[i]);
        }
    };
    auto load4w = [&](int b, float (&u)[4]) {
        const float4 t = __ldg(reinterpret_cast<const float4 *>(p.norm_w + (size_t)b * 32 + 4 * j));
        u[0] = t.x;
        u[1] = t.y;
        u[2] = t.z;
        u[3] = t.w;
    };
    const bool store_x = (pro == PRO_EMBED_NORM || AR) && blockIdx.x == 0; // the residual stream's new value
    float buf[NBUF][4];
    if (NORM) { // the RMSNorm weights do not depend on the previous kernel
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int b = (r * nwarps + warp) * 4 + sub;
            if (r < rounds && b < nb)
                load4w(b, buf[4 + r]);
        }
        if (EARLY_W && dep_wait) {
            griddep_wait();
            if (tid == 0)
                trace_go(p.trace, p.trace_slot);
        }
    }
    if (AR) { // spins on peers' words: one rolled copy of that code
#pragma unroll 1
        for (int r = 0; r < 4 && r < rounds; r++) {
            const int b = (r * nwarps + warp) * 4 + sub;
            if (b < nb) {
                float u[4];
                load4(b, u);
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        if (q == r)
                            buf[q][i] = u[i];
            }
        }
    } else {
#pragma unroll
        for (int r = 0; r < NBUF; r++) {
            const int b = (r * nwarps + warp) * 4 + sub;
            if (r < XR && r < rounds && b < nb)
                load4(b, buf[r]);
        }
        signal_issued(issued, tid);
    }
    float scale = 1.0f;
    if (NORM) {
        // sum of squares in a fixed order: per lane, per warp (tree), warps in order
        float ss = 0.0f;
        auto add_ss = [&](const float (&u)[4]) {
#pragma unroll
            for (int i = 0; i < 4; i++)
                ss = __fadd_rn(ss, __fmul_rn(u[i], u[i]));
        };
#pragma unroll
        for (int r = 0; r < 4; r++)
            if (r < rounds && (r * nwarps + warp) * 4 + sub < nb)
                add_ss(buf[r]);
#pragma unroll 1
        for (int r = XR; r < rounds; r++) {
            const int b = (r * nwarps + warp) * 4 + sub;
            if (b < nb) {
                float u[4];
                load4(b, u);
                add_ss(u);
            }
        }
        ss = warp_sum(ss);
        if (lane == 0)
            red[warp] = ss;
        named_bar_sync(bar, nthr);
        float tot = red[0];
        for (int w = 1; w < nwarps; w++)
            tot = __fadd_rn(tot, red[w]);
        const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), p.eps));
        scale = __fdiv_rn(1.0f, rms);
    }
    // normalise (where fused), quantise and store one round's block; every
    // lane of the warp joins the shuffles, dead 8-lane groups skip the stores
    auto finish = [&](int b, bool live, float (&u)[4], const float (&wn)[4]) {
        if (store_x && live)
            *reinterpret_cast<float4 *>(p.x_out + (size_t)b * 32 + 4 * j) = make_float4(u[0], u[1], u[2], u[3]);
        if (NORM)
#pragma unroll
            for (int i = 0; i < 4; i++)
                u[i] = __fmul_rn(__fmul_rn(u[i], scale), wn[i]);
        quantize_block8<WF>(u, j, live, act + (size_t)b * 8, act_s + b, act_c + b);
    };
    // one rolled copy of the quantiser: round r's registers are picked by value
#pragma unroll 1
    for (int r = 0; r < XR && r < rounds; r++) {
        const int b0 = (r * nwarps + warp) * 4;
        if (b0 >= nb)
            break; // warp-uniform
        const int b = b0 + sub;
        const bool live = b < nb;
        float u[4] = {0.0f, 0.0f, 0.0f, 0.0f}, wn[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int q = 0; q < NBUF; q++)
            if (q == r)
#pragma unroll
                for (int i = 0; i < 4; i++)
                    u[i] = live ? buf[q][i] : 0.0f;
        if (NORM)
#pragma unroll
            for (int q = 0; q < 4; q++)
                if (q == r)
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        wn[i] = live ? buf[4 + q][i] : 0.0f;
        finish(b, live, u, wn);
    }
#pragma unroll 1
    for (int r = XR; r < rounds; r++) {
        const int b0 = (r * nwarps + warp) * 4;
        if (b0 >= nb)
            break; // warp-uniform
        const int b = b0 + sub;
        const bool live = b < nb;
        float u[4] = {0.0f, 0.0f, 0.0f, 0.0f}, wn[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (live) {
            load4(b, u);
            if (NORM)
                load4w(b, wn);
        }
        finish(b, live, u, wn);
    }
}

// Tensor parallel: this row's partial sum goes to every rank's buffer as one
// 64-bit word carrying the exchange's tag, so a reader knows the value has
// arrived without a fence or a counter (a word is written whole).
__device__ __forceinline__ void partial_store(const GemvParams &p, int row, float acc)
{
    const unsigned long long w = ((unsigned long long)ar_tag(p) << 32) | __float_as_uint(acc);
    const size_t off = (size_t)p.tp->rank * p.N + row;
    for (int q = 0; q < p.tp->size; q++)
        st_volatile_u64(p.tp->ar[p.ar_kind][q] + off, w);
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
__device__ __forceinline__ void argmax_finalize(const GemvParams &p, unsigned long long key, int tid, int nthr, int bar)
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
                if (wait_counter(tp->cnt[tp->rank] + TP_CNT_KEY, (epoch + 1) * (unsigned long long)tp->size, p.err,
                                 p.peer_ns ? p.peer_ns : 5000000000ull))
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

// ------------------------------------------------------------ one GEMV op
// Shared-memory view of the GEMV machinery of one CTA.
struct GemvSmem {
    uint8_t *ring;           // S stages of stage_bytes
    size_t stage_bytes, scale_off;
    int S;                   // stages, a multiple of NG
    uint64_t *full, *empty;  // [S] each: filled by the producer / released by a warp group
    uint64_t *issued;        // activation requested (one-kernel path only; nullptr otherwise)
    uint64_t *pfull, *pempty; // [PSLOTS]: product slot written by a group / summed by a summer
    unsigned long long *sbest; // summers' best argmax key
    uint32_t *act;           // quantised activation, packed per block
    float *act_s;            // activation block scales
    int *act_c;              // per block: -8 * sum(q) (Q4 offset)
    float *tbuf, *red;
    float *prod;             // [PSLOTS][TR][TBS] block products (aliases tbuf: a CTA uses one)
};

// This CTA's share of a GEMV: rows [r0, r1) in tiles of B rows.  TPS tile sets
// are worked on at once (4 when the CTA has >= 4 tiles, else 2 or 1); the
// GT = NG / TPS groups of a set take its (tile, chunk) steps u = 0, 1, ... in
// turn, group q of the set taking u = q, q + GT, ...  With GT = 1 a row's
// running sum stays in registers; with GT > 1 it is handed from group to group
// through shared memory (one mbarrier per warp), which keeps the reference's
// block order while GT chunks are computed at once.  Group g owns ring stages
// g, g + NG, ...: a stage barrier is only awaited by the group that consumed
// its previous phase.
struct GemvWork {
    int r0, r1, B, ntiles, nb, nchunks, TPS, GT;
};

__device__ __forceinline__ GemvWork gemv_work(const GemvParams &p, int cta)
{
    GemvWork w;
    w.B = p.box_rows;
    w.r0 = cta * p.rows_per_cta;
    w.r1 = min(p.N, w.r0 + p.rows_per_cta);
    w.ntiles = w.r1 > w.r0 ? (w.r1 - w.r0 + w.B - 1) / w.B : 0;
    w.nb = p.K >> 5;
    w.nchunks = (w.nb + CB - 1) / CB;
    w.TPS = w.ntiles >= NG ? NG : (w.ntiles >= 2 ? 2 : 1);
    w.GT = NG / w.TPS;
    return w;
}

__device__ __forceinline__ int gemv_group_iters(const GemvWork &w, int g)
{
    const int set = g % w.TPS, q = g / w.TPS;
    const int nset = w.ntiles > set ? (w.ntiles - 1 - set) / w.TPS + 1 : 0;
    const int U = nset * w.nchunks;
    return U > q ? (U - 1 - q) / w.GT + 1 : 0;
}

// Parity of the number of times each ring stage is filled by one GEMV op of
// this CTA (bit s).
__device__ __forceinline__ uint32_t gemv_stage_use_parity(const GemvWork &w, int S)
{
    const int spg = S / NG;
    uint32_t m = 0;
    for (int g = 0; g < NG; g++) {
        const int it = gemv_group_iters(w, g);
        for (int j = 0; j < spg; j++) {
            const int uses = it > j ? (it - 1 - j) / spg + 1 : 0;
            m |= (uint32_t)(uses & 1) << (g + NG * j);
        }
    }
    return m;
}

// Bound on the stages a producer has requested that have not landed yet.  A
// deep queue of bulk copies makes every other memory access of the SM (the
// activation loads, epilogue stores, completion counters) wait behind it; a
// few stages in flight (about the bandwidth-delay product of one SM) keep the
// HBM busy without that.
struct InFlight {
    int cap = 0; // 0: unbounded
    int n = 0, head = 0;
    uint8_t st[8], seq[8]; // stage and fill number of each outstanding fill, oldest at head
    uint8_t fills[8] = {}; // fills of each stage so far (mod 256)
};

// Before a new request: while `cap` are outstanding, wait for the oldest to
// land.  An entry whose stage has been filled again since has landed (the
// refill needed its consumption), so it is dropped without waiting.
__device__ __forceinline__ bool inflight_admit(InFlight &q, uint64_t *full, uint32_t *err)
{
    while (q.cap > 0 && q.n >= q.cap) {
        const int s = q.st[q.head];
        if (q.fills[s] == (uint8_t)(q.seq[q.head] + 1) && !mbar_wait(&full[s], q.seq[q.head] & 1u, err))
            return false;
        q.head = (q.head + 1) & 7;
        q.n--;
    }
    return true;
}

// after requesting a fill of stage s (its full barrier completes phase fills[s])
__device__ __forceinline__ void inflight_push(InFlight &q, int s)
{
    if (q.cap > 0) {
        const int t = (q.head + q.n) & 7;
        q.st[t] = (uint8_t)s;
        q.seq[t] = q.fills[s];
        q.n++;
    }
    q.fills[s]++;
}

// Producer (one thread): stream this CTA's stages of one GEMV.  fill_par /
// filled: per stage, parity of its fills so far / filled at least once (kept
// across ops).  pre >= 0: after `pre` stages wait until the consumers have
// requested the activation.  Returns false if a wait timed out.
template <int WF, int ST>
__device__ __forceinline__ bool gemv_produce(const CUtensorMap *tw, const CUtensorMap *ts, const GemvParams &p, const GemvWork &w,
                             const GemvSmem &sm, uint32_t &fill_par, uint32_t &filled, uint64_t pol, int pre,
                             InFlight &q)
{
    constexpr int W_ROW = CB * wbytes_per_block(WF);
    constexpr int S_ROW = CB * sbytes(ST);
    const int SPG = sm.S / NG;
    const uint32_t stage_tx = (uint32_t)(w.B * (W_ROW + S_ROW)); // whole boxes (OOB is zero-filled)
    // One thread issues every stage, so its loop is kept free of divisions:
    // per group, the step's chunk and tile advance by GT.
    int gi[NG], gc[NG], gt[NG];
#pragma unroll
    for (int g = 0; g < NG; g++) {
        gi[g] = gemv_group_iters(w, g);
        gc[g] = g / w.TPS; // first step u = q: chunk u % nchunks of tile set g % TPS
        gt[g] = g % w.TPS;
        while (gc[g] >= w.nchunks) {
            gc[g] -= w.nchunks;
            gt[g] += w.TPS;
        }
    }
    int issued_n = 0;
    for (int k = 0; k < gi[0]; k++) { // group 0 has the most steps
        const int slot = k & (SPG - 1);
#pragma unroll
        for (int g = 0; g < NG; g++) {
            if (k >= gi[g])
                continue;
            if (pre >= 0 && issued_n++ == pre && !mbar_wait(sm.issued, 0, p.err))
                return false;
            const int s = g + NG * slot;
            const uint32_t bit = 1u << s;
            LLMRS_TRACE_BEGIN(0);
            if ((filled & bit) && !mbar_wait(&sm.empty[s], (fill_par & bit) ? 0u : 1u, p.err))
                return false;
            if (!inflight_admit(q, sm.full, p.err))
                return false;
            LLMRS_TRACE_END(0);
            const int y = w.r0 + gt[g] * w.B, c = gc[g];
            uint8_t *st = sm.ring + (size_t)s * sm.stage_bytes;
            mbar_arrive_expect_tx(&sm.full[s], stage_tx);
            tma_load_2d(st, tw, c * (W_ROW / 4), y, &sm.full[s], pol);
            tma_load_2d(st + sm.scale_off, ts, c * CB, y, &sm.full[s], pol);
            inflight_push(q, s);
            fill_par ^= bit;
            filled |= bit;
            gc[g] += w.GT;
            while (gc[g] >= w.nchunks) {
                gc[g] -= w.nchunks;
                gt[g] += w.TPS;
            }
        }
    }
    return true;
}

// Output of one finished row (valid: this lane holds a row of the tile).
// Every lane of the warp calls it (the SiLU pair crosses lanes).
__device__ __forceinline__ void gemv_epilogue(const GemvParams &p, const int epi, int row, bool valid, float acc,
                                              unsigned long long &best)
{
    if (epi == EPI_STORE) {
        if (valid)
            p.y[row] = acc;
    } else if (epi == EPI_RESIDUAL) {
        if (valid)
            p.y[row] = __fadd_rn(acc, __ldcg(p.residual + row));
    } else if (epi == EPI_SILU) {
        const float up = __shfl_down_sync(0xffffffffu, acc, 1);
        if (valid && (row & 1) == 0) {
            const float silu = __fdiv_rn(acc, __fadd_rn(1.0f, expf(-acc)));
            p.y[row >> 1] = __fmul_rn(silu, up);
        }
    } else if (epi == EPI_ARGMAX) {
        if (valid) {
            if (p.y)
                p.y[row] = acc;
            const unsigned long long key = argmax_key(acc, (uint32_t)(row + p.row_offset));
            best = key > best ? key : best;
        }
    } else if (epi == EPI_PARTIAL) {
        if (valid)
            partial_store(p, row, acc);
    }
}

// Consumers (the NW consumer warps, ctid = 0 .. NW*32-1): prologue, steps,
// epilogue of one GEMV.  cpar: per stage, parity of the full-barrier phase to
// wait for next (advanced to the op's end on return).  dep_wait: the prologue
// waits for the previous kernel itself (after the loads that do not depend on
// it); otherwise the caller has already waited for the op's input.
template <int WF, int ST, bool TPK = false>
__device__ __forceinline__ void gemv_consume(const GemvParams &p, const int pro, const int epi, const GemvWork &w,
                                             const GemvSmem &sm, uint32_t &cpar, int ctid,
                                             bool dep_wait = false)
{
    constexpr int W_ROW = CB * wbytes_per_block(WF);
    constexpr int S_ROW = CB * sbytes(ST);
    const int warp = ctid >> 5, lane = ctid & 31;
    const int SPG = sm.S / NG;
    LLMRS_TRACE_BEGIN(2);
    load_activation<WF, TPK>(p, pro, sm.act, sm.act_s, sm.act_c, sm.red, ctid, PRO_THREADS, 1, sm.issued, dep_wait);
    named_bar_sync(1, PRO_THREADS);
    if (ctid == 0) {
        trace_ready(p.trace, p.trace_slot);
    }
    LLMRS_TRACE_END(2);

    // warp (grp, wq): group grp = warp / WPG takes its steps of its tile set;
    // wq = warp % WPG takes tile rows wq*RPW .. +RPW-1.  Lane l = block l of the chunk.
    const int grp = warp / WPG, wq = warp % WPG;
    float *tb = sm.tbuf + (size_t)warp * RPW * TBS;
    // transposed roles: lane j sums row ri = j % RPW over blocks seg*8 .. seg*8+7
    const int ri = lane % RPW, seg = lane / RPW;
    unsigned long long best = 0ull;
    bool ok = true;
    uint32_t mypar = cpar; // this group's stages flip as it consumes them
    // the step loop (one copy for every number of groups per tile set)
    {
        const int GT = w.GT, TPS = w.TPS;
        float acc = 0.0f; // running sum of row ri (complete in the segment-3 lanes)
        const int tset = grp % TPS, q = grp / TPS;
        const int my_iters = gemv_group_iters(w, grp);
        int c = q, tile = tset; // this group's first step u = q
        while (c >= w.nchunks) {
            c -= w.nchunks;
            tile += TPS;
        }
        for (int k = 0; k < my_iters; k++) {
            if (k > 0) { // next step: u += GT
                c += GT;
                while (c >= w.nchunks) {
                    c -= w.nchunks;
                    tile += TPS;
                }
            }
            const int s = grp + NG * (k & (SPG - 1));
            const uint32_t bit = 1u << s;
            const int u = k * GT + q;
            const int trow0 = w.r0 + tile * w.B;
            const int rows = min(w.B, w.r1 - trow0);
            const int nbc = min(CB, w.nb - c * CB);
            LLMRS_TRACE_BEGIN(3);
            if (ok && !mbar_wait(&sm.full[s], (mypar & bit) ? 1u : 0u, p.err))
                ok = false;
            mypar ^= bit;
            LLMRS_TRACE_END(3);
            LLMRS_TRACE_BEGIN(4);
            const uint8_t *st = sm.ring + (size_t)s * sm.stage_bytes;
            float t[RPW];
            {
                const int b = c * CB + min(lane, nbc - 1);
                const uint4 a0 = reinterpret_cast<const uint4 *>(sm.act)[2 * b];
                const uint4 a1 = reinterpret_cast<const uint4 *>(sm.act)[2 * b + 1];
                const float sa = sm.act_s[b];
                const int cz = sm.act_c[b];
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
                    const float sw = load_scale<ST>(st + sm.scale_off + (size_t)lr * S_ROW, lane);
                    t[i] = __fmul_rn((float)isum, __fmul_rn(sw, sa));
                }
            }
            // products are in registers: hand the stage back to the producer
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&sm.empty[s]);
            if (GT > 1) {
                // groups share the tile: the products go to the set's slot for
                // step u, and the set's summer warp adds them in block order
                const int ps = PSLOTS / TPS;
                const int slot = tset * ps + u % ps, use = u / ps;
                if (use > 0 && ok && !mbar_wait(&sm.pempty[slot], (uint32_t)((use - 1) & 1), p.err))
                    ok = false;
                float *P = sm.prod + (size_t)slot * TR * TBS + (size_t)(wq * RPW) * TBS + lane;
#pragma unroll
                for (int i = 0; i < RPW; i++)
                    P[i * TBS] = t[i];
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&sm.pfull[slot]);
                LLMRS_TRACE_END(4);
                continue;
            }
            // transpose: lane j then holds row ri's products for blocks seg*8 .. +7
#pragma unroll
            for (int i = 0; i < RPW; i++)
                tb[i * TBS + lane] = t[i];
            __syncwarp();
            const float4 v0 = *reinterpret_cast<const float4 *>(tb + ri * TBS + seg * 8);
            const float4 v1 = *reinterpret_cast<const float4 *>(tb + ri * TBS + seg * 8 + 4);
            const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
            { // the running sum moves from the segment-3 lane to the segment-0 lane
                const float carry = __shfl_sync(0xffffffffu, acc, 3 * RPW + ri);
                acc = (c > 0 && seg == 0) ? carry : 0.0f;
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
                    for (int kk = 0; kk < 8; kk++)
                        if (sg * 8 + kk < nbc)
                            acc = __fadd_rn(acc, v[kk]);
                }
            }
            LLMRS_TRACE_END(4);
            if (c == w.nchunks - 1) // epilogue: lanes of segment 3 hold the complete rows
                gemv_epilogue(p, epi, trow0 + wq * RPW + ri, seg == 3 && live_row, acc, best);
        }
    }
    // every consumer thread advances the op-start parities identically
    cpar ^= gemv_stage_use_parity(w, sm.S);
    if (epi == EPI_ARGMAX) {
        // rows summed by the summer warps (groups sharing a tile) add their key
        named_bar_sync(2, PRO_THREADS + NSUM * 32);
        const unsigned long long sb = *reinterpret_cast<volatile unsigned long long *>(sm.sbest);
        best = sb > best ? sb : best;
        argmax_finalize(p, best, ctid, PRO_THREADS, 1);
    }
}

// Summer warp `tset` of a CTA whose groups share tiles (GT > 1): lane r adds
// row r's block products of every step of tile set tset in block order (the
// reference's sequential sum), releases each product slot as soon as its
// values are in registers, and runs the epilogue of the tile's rows.
__device__ __forceinline__ void gemv_sum(const GemvParams &p, const int epi, const GemvWork &w, const GemvSmem &sm,
                                         int tset)
{
    const int lane = threadIdx.x & 31;
    unsigned long long best = 0ull;
    if (w.GT > 1 && tset < w.TPS) {
        const int TPS = w.TPS, ps = PSLOTS / TPS;
        const int nset = w.ntiles > tset ? (w.ntiles - 1 - tset) / TPS + 1 : 0;
        const int U = nset * w.nchunks;
        float acc = 0.0f;
        int c = 0, tile = tset;
        bool ok = true;
        for (int u = 0; u < U; u++) {
            const int slot = tset * ps + u % ps;
            if (ok && !mbar_wait(&sm.pfull[slot], (uint32_t)((u / ps) & 1), p.err))
                ok = false;
            const float4 *P = reinterpret_cast<const float4 *>(sm.prod + (size_t)slot * TR * TBS + (size_t)lane * TBS);
            float v[CB];
#pragma unroll
            for (int j = 0; j < CB / 4; j++) {
                const float4 f = P[j];
                v[4 * j] = f.x;
                v[4 * j + 1] = f.y;
                v[4 * j + 2] = f.z;
                v[4 * j + 3] = f.w;
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&sm.pempty[slot]);
            const int nbc = min(CB, w.nb - c * CB);
            if (c == 0)
                acc = 0.0f;
#pragma unroll
            for (int kk = 0; kk < CB; kk++)
                if (kk < nbc)
                    acc = __fadd_rn(acc, v[kk]);
            if (c == w.nchunks - 1) {
                const int trow0 = w.r0 + tile * w.B;
                gemv_epilogue(p, epi, trow0 + lane, lane < min(w.B, w.r1 - trow0), acc, best);
            }
            if (++c == w.nchunks) {
                c = 0;
                tile += TPS;
            }
        }
    }
    if (epi == EPI_ARGMAX) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0 && best)
            atomicMax(sm.sbest, best);
        named_bar_sync(2, PRO_THREADS + NSUM * 32);
    }
}

} // namespace

} // namespace llmrs
