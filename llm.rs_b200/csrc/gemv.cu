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
// Data movement: each CTA owns a balanced, contiguous range of rows.  A
// producer warp streams 32-row x 32-block chunks of nibbles (or int8 codes)
// and their block scales from HBM into a ring of shared-memory stages with 1-D
// bulk TMA copies (cp.async.bulk, mbarrier complete_tx), so HBM reads are
// whole contiguous row segments.  Eight consumer warps compute with dp4a: lane
// l takes block l of the chunk for each of its rows, so a warp reads 512
// contiguous smem bytes per row (conflict-free).  The per-block products are
// transposed through a small smem buffer so one lane per row adds them in the
// reference's sequential block order.
//
// The producer does not depend on the previous kernel, so with programmatic
// dependent launch it starts streaming weights while the previous kernel is
// still running; consumers call griddepcontrol.wait before reading activations.
#include <cuda_fp16.h>

#include "common.cuh"
#include "gemv.cuh"

namespace llmrs {

namespace {

constexpr int CW = 8;   // consumer warps
constexpr int TR = 32;  // rows per tile (4 per consumer warp)
constexpr int CB = 32;  // blocks per chunk (1024 weights)
constexpr int NTHREADS = (CW + 1) * 32;
constexpr int TB_STRIDE = 36; // floats per row of the transpose buffer (16-byte aligned, conflict-free)
constexpr size_t SMEM_BUDGET = 112 * 1024; // two CTAs per SM (current + PDL-prefetching next kernel)

__host__ __device__ constexpr int wbytes_per_block(int wf) { return wf == 0 ? 16 : 32; }
__host__ __device__ constexpr int sbytes(int st) { return st == 0 ? 2 : 4; }
__host__ __device__ constexpr size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

struct SmemLayout {
    size_t stage_bytes, act_off, acts_off, actc_off, tbuf_off, bar_off, red_off, total;
};

__host__ __device__ inline SmemLayout smem_layout(int wf, int st, int K, int stages)
{
    SmemLayout L;
    int nb = K / 32;
    L.stage_bytes = (size_t)TR * CB * (wbytes_per_block(wf) + sbytes(st));
    L.act_off = L.stage_bytes * stages;
    L.acts_off = L.act_off + (size_t)nb * 32;
    L.actc_off = align16(L.acts_off + (size_t)nb * 4);
    L.tbuf_off = align16(L.actc_off + (size_t)nb * 4);
    L.bar_off = align16(L.tbuf_off + (size_t)CW * 4 * TB_STRIDE * 4);
    L.red_off = L.bar_off + (size_t)stages * 2 * 8;
    L.total = align16(L.red_off + 16 * 4);
    return L;
}

// byte k (0..3) of packed word j (0..7) comes from lane src_lane(j, k)
template <int WF>
__device__ __forceinline__ int src_lane(int j, int k)
{
    if (WF == 0) // Q4 order: words 0-3 = even elements of each 8, words 4-7 = odd
        return j < 4 ? 8 * j + 2 * k : 8 * (j - 4) + 2 * k + 1;
    return 4 * j + k; // natural order
}

// Quantise one 32-value block held one value per lane (bit-exact Q8_0) and store
// its packed codes (32 bytes), scale and correction term to shared memory.
template <int WF>
__device__ __forceinline__ void quantize_block(float v, int lane, uint32_t *dst_words, float *dst_s, int *dst_c)
{
    float amax = warp_max(fabsf(v));
    int q = 0;
    float scale = 0.0f;
    if (amax != 0.0f) {
        scale = __fdiv_rn(amax, 127.0f);
        float inv = __fdiv_rn(1.0f, scale);
        float r = roundf(__fmul_rn(v, inv));
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        q = (r != r) ? 0 : (int)r;
    }
    uint32_t word = 0;
    int j = lane & 7;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        uint32_t b = (uint32_t)__shfl_sync(0xffffffffu, q & 0xFF, src_lane<WF>(j, k));
        word |= b << (8 * k);
    }
    if (lane < 8)
        dst_words[lane] = word;
    int sum = warp_sum_int(q);
    if (lane == 0) {
        *dst_s = scale;
        *dst_c = WF == 0 ? -8 * sum : 0;
    }
}

// Fill the shared-memory activation (codes, scales, corrections) from the
// selected source.  Runs on the CW consumer warps (named barrier 1).
template <int WF, int PRO>
__device__ void load_activation(const GemvParams &p, uint32_t *act, float *act_s, int *act_c, float *red,
                                int ctid, int warp, int lane)
{
    const int K = p.K, nb = K >> 5;
    if (PRO == PRO_Q8) {
        for (int b = warp; b < nb; b += CW) {
            int q = p.xq[(size_t)b * 32 + lane];
            uint32_t word = 0;
            int j = lane & 7;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                uint32_t v = (uint32_t)__shfl_sync(0xffffffffu, q & 0xFF, src_lane<WF>(j, k));
                word |= v << (8 * k);
            }
            if (lane < 8)
                act[b * 8 + lane] = word;
            int sum = warp_sum_int(q);
            if (lane == 0) {
                act_s[b] = p.xs[b];
                act_c[b] = WF == 0 ? -8 * sum : 0;
            }
        }
        return;
    }
    const float *x = p.x;
    if (PRO == PRO_EMBED_NORM) {
        int tok = p.state->token;
        if (tok < 0 || tok >= p.vocab) {
            if (ctid == 0)
                atomicCAS(p.err, 0u, (uint32_t)DEV_ERR_BAD_TOKEN);
            tok = 0;
        }
        x = p.embed + (size_t)tok * K;
        if (blockIdx.x == 0)
            for (int i = ctid; i < K; i += CW * 32)
                p.x_out[i] = x[i];
    }
    float scale = 1.0f;
    if (PRO == PRO_NORM || PRO == PRO_EMBED_NORM) {
        float ss = 0.0f;
        for (int i = ctid; i < K; i += CW * 32)
            ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
        ss = warp_sum(ss);
        if (lane == 0)
            red[warp] = ss;
        named_bar_sync(1, CW * 32);
        float tot = red[0];
#pragma unroll
        for (int w = 1; w < CW; w++)
            tot = __fadd_rn(tot, red[w]);
        float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), p.eps));
        scale = __fdiv_rn(1.0f, rms);
    }
    for (int b = warp; b < nb; b += CW) {
        float v = x[(size_t)b * 32 + lane];
        if (PRO == PRO_NORM || PRO == PRO_EMBED_NORM)
            v = __fmul_rn(__fmul_rn(v, scale), p.norm_w[(size_t)b * 32 + lane]);
        quantize_block<WF>(v, lane, act + (size_t)b * 8, act_s + b, act_c + b);
    }
}

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

// local row (within a 32-row tile) of slot s (0..3) of consumer warp w:
// row pairs are dealt round-robin so partial tiles stay balanced and the two
// rows of a pair (gate/up) sit in adjacent lanes of one warp.
__device__ __forceinline__ int slot_row(int w, int s) { return 2 * (w + CW * (s >> 1)) + (s & 1); }

// Last CTA of an argmax GEMV publishes the step's greedy token and advances
// the decode position; the state is then ready for the next step.
__device__ void argmax_finalize(const GemvParams &p, unsigned long long key)
{
    __shared__ unsigned long long s_key[CW];
    __shared__ unsigned int s_ticket;
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
    }
    if (lane == 0)
        s_key[warp] = key;
    named_bar_sync(1, CW * 32);
    if (threadIdx.x == 0) {
        unsigned long long k = s_key[0];
        for (int w = 1; w < CW; w++)
            k = s_key[w] > k ? s_key[w] : k;
        atomicMax(&p.state->key, k);
        __threadfence();
        s_ticket = atomicAdd(&p.state->done, 1u);
        if (s_ticket == gridDim.x - 1) {
            __threadfence();
            unsigned long long best = atomicAdd(&p.state->key, 0ull);
            int tok = (int)argmax_key_index(best);
            StepState *st = p.state;
            int n = st->n_log;
            if (p.token_log && n < st->log_cap)
                p.token_log[n] = tok;
            st->n_log = n + 1;
            st->token = tok;
            st->pos = st->pos + 1;
            st->key = 0ull;
            st->done = 0u;
            __threadfence();
        }
    }
}

template <int WF, int ST, int PRO, int EPI>
__global__ void __launch_bounds__(NTHREADS, 1) gemv_tma_kernel(const GemvParams p)
{
    constexpr int WB = wbytes_per_block(WF);
    constexpr int W_ROW = CB * WB;
    constexpr int S_ROW = CB * sbytes(ST);
    extern __shared__ __align__(128) uint8_t smem[];

    griddep_launch_dependents();

    const int S = p.n_stages;
    const int K = p.K, nb = K >> 5;
    const int nchunks = (nb + CB - 1) / CB;
    const SmemLayout L = smem_layout(WF, ST, K, S);
    uint8_t *stages = smem;
    uint32_t *act = reinterpret_cast<uint32_t *>(smem + L.act_off);
    float *act_s = reinterpret_cast<float *>(smem + L.acts_off);
    int *act_c = reinterpret_cast<int *>(smem + L.actc_off);
    float *tbuf = reinterpret_cast<float *>(smem + L.tbuf_off);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar_off);
    uint64_t *empty = full + S;
    float *red = reinterpret_cast<float *>(smem + L.red_off);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // balanced contiguous row range in units of row pairs
    const int n_units = p.N >> 1;
    const int u0 = (int)(((long long)blockIdx.x * n_units) / gridDim.x);
    const int u1 = (int)(((long long)(blockIdx.x + 1) * n_units) / gridDim.x);
    const int r0 = 2 * u0, r1 = 2 * u1;
    const int ntiles = (r1 - r0 + TR - 1) / TR;
    const int iters = ntiles * nchunks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == CW) {
        // ------------------------------------------------------------ producer
        const uint64_t pol = policy_evict_first();
        const size_t w_row_bytes = (size_t)nb * WB;
        const size_t s_row_bytes = (size_t)nb * sbytes(ST);
        const uint8_t *wbase = p.w;
        const uint8_t *sbase = reinterpret_cast<const uint8_t *>(p.scales);
        for (int it = 0; it < iters; it++) {
            const int s = it % S;
            if (it >= S && !mbar_wait(&empty[s], ((it / S) - 1) & 1, p.err))
                return;
            const int tile = it / nchunks, c = it % nchunks;
            const int trow0 = r0 + tile * TR;
            const int rows = min(TR, r1 - trow0);
            const int nbc = min(CB, nb - c * CB);
            if (lane == 0)
                mbar_arrive_expect_tx(&full[s], (uint32_t)(rows * nbc * (WB + sbytes(ST))));
            __syncwarp();
            if (lane < rows) {
                const int row = trow0 + lane;
                uint8_t *st = stages + (size_t)s * L.stage_bytes;
                bulk_g2s(st + (size_t)lane * W_ROW, wbase + (size_t)row * w_row_bytes + (size_t)c * W_ROW,
                         (uint32_t)(nbc * WB), &full[s], pol);
                bulk_g2s(st + (size_t)TR * W_ROW + (size_t)lane * S_ROW,
                         sbase + (size_t)row * s_row_bytes + (size_t)c * S_ROW, (uint32_t)(nbc * sbytes(ST)),
                         &full[s], pol);
            }
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    griddep_wait();
    const int ctid = threadIdx.x;
    load_activation<WF, PRO>(p, act, act_s, act_c, red, ctid, warp, lane);
    named_bar_sync(1, CW * 32);

    float *tb = tbuf + (size_t)warp * 4 * TB_STRIDE;
    unsigned long long best = 0ull;
    bool ok = true;
    for (int tile = 0; tile < ntiles; tile++) {
        const int trow0 = r0 + tile * TR;
        const int rows = min(TR, r1 - trow0);
        float acc = 0.0f; // lane s < 4 owns the row of slot s
        for (int c = 0; c < nchunks; c++) {
            const int it = tile * nchunks + c;
            const int s = it % S;
            // after a timeout the warp keeps its control flow (results are
            // discarded by the host, which sees the error word) but stops waiting
            if (ok && !mbar_wait(&full[s], (it / S) & 1, p.err))
                ok = false;
            const uint8_t *st = stages + (size_t)s * L.stage_bytes;
            const uint8_t *ssc = st + (size_t)TR * W_ROW;
            const int nbc = min(CB, nb - c * CB);
            const int b = c * CB + lane;
            float t[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (lane < nbc) {
                const uint4 a0 = reinterpret_cast<const uint4 *>(act)[2 * b];
                const uint4 a1 = reinterpret_cast<const uint4 *>(act)[2 * b + 1];
                const float sa = act_s[b];
                const int cz = act_c[b];
#pragma unroll
                for (int sl = 0; sl < 4; sl++) {
                    const int lr = slot_row(warp, sl);
                    if (lr < rows) {
                        int isum;
                        if (WF == 0) {
                            const uint4 wv = *reinterpret_cast<const uint4 *>(st + (size_t)lr * W_ROW + lane * 16);
                            isum = dot_block_q4(wv, a0, a1, cz);
                        } else {
                            const uint4 *wp = reinterpret_cast<const uint4 *>(st + (size_t)lr * W_ROW + lane * 32);
                            isum = dot_block_q8(wp[0], wp[1], a0, a1, cz);
                        }
                        const float sw = load_scale<ST>(ssc + (size_t)lr * S_ROW, lane);
                        t[sl] = __fmul_rn((float)isum, __fmul_rn(sw, sa));
                    }
                }
            }
#pragma unroll
            for (int sl = 0; sl < 4; sl++)
                tb[sl * TB_STRIDE + lane] = t[sl];
            __syncwarp();
            if (lane < 4 && slot_row(warp, lane) < rows) {
                const float *src = tb + lane * TB_STRIDE;
                for (int j = 0; j < nbc; j += 4) {
                    const float4 v = *reinterpret_cast<const float4 *>(src + j);
                    acc = __fadd_rn(acc, v.x);
                    acc = __fadd_rn(acc, v.y);
                    acc = __fadd_rn(acc, v.z);
                    acc = __fadd_rn(acc, v.w);
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&empty[s]);
        }
        // ---- epilogue for this tile
        const int lr = slot_row(warp, lane & 3);
        const bool valid = lane < 4 && lr < rows;
        const int row = trow0 + lr;
        if (EPI == EPI_STORE) {
            if (valid)
                p.y[row] = acc;
        } else if (EPI == EPI_RESIDUAL) {
            if (valid)
                p.y[row] = __fadd_rn(acc, p.residual[row]);
        } else if (EPI == EPI_SILU) {
            const float up = __shfl_down_sync(0xffffffffu, acc, 1);
            if (valid && (lane & 1) == 0) {
                const float g = acc;
                const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
                p.y[row >> 1] = __fmul_rn(silu, up);
            }
        } else if (EPI == EPI_ARGMAX) {
            if (valid) {
                if (p.y)
                    p.y[row] = acc;
                const unsigned long long k = argmax_key(acc, (uint32_t)row);
                best = k > best ? k : best;
            }
        }
    }
    if (EPI == EPI_ARGMAX)
        argmax_finalize(p, best);
}

// ------------------------------------------------------------------ fallback
// One thread per output row, same arithmetic; activation quantised into smem.
template <int WF, int ST, int PRO, int EPI>
__global__ void __launch_bounds__(256) gemv_simple_kernel(const GemvParams p)
{
    extern __shared__ __align__(16) uint8_t smem[];
    griddep_launch_dependents();
    const int K = p.K, nb = K >> 5;
    uint32_t *act = reinterpret_cast<uint32_t *>(smem);
    float *act_s = reinterpret_cast<float *>(smem + (size_t)nb * 32);
    int *act_c = reinterpret_cast<int *>(act_s + nb);
    float *red = reinterpret_cast<float *>(act_c + nb);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    griddep_wait();
    // the prologue helper assumes CW warps; run it on warps 0..CW-1 (256 threads)
    load_activation<WF, PRO>(p, act, act_s, act_c, red, threadIdx.x, warp, lane);
    named_bar_sync(1, CW * 32);
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
            best = argmax_key(acc, (uint32_t)row);
        }
    }
    if (EPI == EPI_SILU) {
        // rows (2i, 2i+1) are threads (2i, 2i+1) of this block
        __shared__ float rows_acc[256];
        rows_acc[threadIdx.x] = row_acc;
        __syncthreads();
        if (row < p.N && (row & 1) == 0 && row + 1 < p.N) {
            const float g = row_acc, up = rows_acc[threadIdx.x + 1];
            const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
            p.y[row >> 1] = __fmul_rn(silu, up);
        }
    }
    if (EPI == EPI_ARGMAX)
        argmax_finalize(p, best);
}

constexpr int SIMPLE_SMEM_MAX = 200 * 1024;

template <int WF, int ST, int PRO, int EPI>
cudaError_t prepare_one()
{
    cudaError_t e = cudaFuncSetAttribute(gemv_tma_kernel<WF, ST, PRO, EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BUDGET + 4096);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemv_simple_kernel<WF, ST, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 SIMPLE_SMEM_MAX);
    return e;
}

template <int WF, int ST, int PRO, int EPI>
int launch_one(const GemvParams &p0, bool fast, cudaStream_t stream, bool pdl, int max_ctas)
{
    GemvParams p = p0;
    if (fast) {
        int stages = 0;
        size_t smem = gemv_smem_bytes(WF, ST, p.K, &stages);
        p.n_stages = stages;
        int grid = min(max_ctas, p.N / 2);
        LLMRS_CUDA_TRY(launch(gemv_tma_kernel<WF, ST, PRO, EPI>, dim3(grid), dim3(NTHREADS), smem, stream, pdl, p));
    } else {
        const int nb = p.K / 32;
        size_t smem = (size_t)nb * 40 + 64;
        LLMRS_CHECK_ARG(smem <= (size_t)SIMPLE_SMEM_MAX, "gemv: K=%d too large", p.K);
        int grid = (p.N + 255) / 256;
        LLMRS_CUDA_TRY(launch(gemv_simple_kernel<WF, ST, PRO, EPI>, dim3(grid), dim3(256), smem, stream, pdl, p));
    }
    return LLMRS_OK;
}

} // namespace

size_t gemv_smem_bytes(int wf, int st, int K, int *stages)
{
    int best = 0;
    for (int s = 6; s >= 2; s--) {
        if (smem_layout(wf, st, K, s).total <= SMEM_BUDGET) {
            best = s;
            break;
        }
    }
    if (stages)
        *stages = best;
    return best ? smem_layout(wf, st, K, best).total : 0;
}

bool gemv_fast_ok(const GemvParams &p, int wf, int st)
{
    if (p.K % 256 != 0 || p.N % 2 != 0 || p.N < 2)
        return false;
    if ((reinterpret_cast<uintptr_t>(p.w) & 15) || (reinterpret_cast<uintptr_t>(p.scales) & 15))
        return false;
    return gemv_smem_bytes(wf, st, p.K, nullptr) != 0;
}

// every (weight format, scale dtype, prologue, epilogue) the op-level API and the decode step use
#define LLMRS_GEMV_VARIANTS(X) \
    X(0, 0, PRO_F32, EPI_STORE) \
    X(0, 0, PRO_NORM, EPI_STORE) \
    X(0, 0, PRO_EMBED_NORM, EPI_STORE) \
    X(0, 0, PRO_F32, EPI_RESIDUAL) \
    X(0, 0, PRO_NORM, EPI_SILU) \
    X(0, 0, PRO_NORM, EPI_ARGMAX) \
    X(0, 1, PRO_F32, EPI_STORE) \
    X(0, 1, PRO_NORM, EPI_STORE) \
    X(0, 1, PRO_EMBED_NORM, EPI_STORE) \
    X(0, 1, PRO_F32, EPI_RESIDUAL) \
    X(0, 1, PRO_NORM, EPI_SILU) \
    X(0, 1, PRO_NORM, EPI_ARGMAX) \
    X(1, 0, PRO_F32, EPI_STORE) \
    X(1, 0, PRO_NORM, EPI_STORE) \
    X(1, 0, PRO_EMBED_NORM, EPI_STORE) \
    X(1, 0, PRO_F32, EPI_RESIDUAL) \
    X(1, 0, PRO_NORM, EPI_SILU) \
    X(1, 0, PRO_NORM, EPI_ARGMAX) \
    X(1, 1, PRO_F32, EPI_STORE) \
    X(1, 1, PRO_NORM, EPI_STORE) \
    X(1, 1, PRO_EMBED_NORM, EPI_STORE) \
    X(1, 1, PRO_F32, EPI_RESIDUAL) \
    X(1, 1, PRO_NORM, EPI_SILU) \
    X(1, 1, PRO_NORM, EPI_ARGMAX)

int gemv_launch(const GemvParams &p, int wf, int st, int pro, int epi, cudaStream_t stream, bool pdl, int max_ctas)
{
    LLMRS_CHECK_ARG(p.K > 0 && p.K % 32 == 0, "gemv: K=%d must be a positive multiple of 32", p.K);
    LLMRS_CHECK_ARG(p.N > 0, "gemv: N=%d must be positive", p.N);
    LLMRS_CHECK_ARG(epi != EPI_SILU || p.N % 2 == 0, "gemv: SiLU epilogue needs an even row count");
    const bool fast = gemv_fast_ok(p, wf, st);
#define LLMRS_GEMV_CASE(WF, ST, PRO, EPI)                                                                   \
    if (wf == WF && st == ST && pro == PRO && epi == EPI)                                                  \
        return launch_one<WF, ST, PRO, EPI>(p, fast, stream, pdl, max_ctas);
    LLMRS_GEMV_VARIANTS(LLMRS_GEMV_CASE)
#undef LLMRS_GEMV_CASE
    return fail(LLMRS_ENOTSUP, "gemv: unsupported variant wf=%d st=%d pro=%d epi=%d", wf, st, pro, epi);
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
