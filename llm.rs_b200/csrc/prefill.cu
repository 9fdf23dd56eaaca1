// prefill.cu - the M>1 path on the tcgen05 tensor cores.
//
// Reference (src/backend/cpu.rs:90-110 with the block kernel of
// src/backend/cpu.rs:888-941): every row m of A is quantised to Q8_0 on its
// own, and output (m, n) is
//     acc = 0; for b in blocks: acc += (float)isum_b * (s_w[n,b] * s_a[m,b])
// with isum_b the exact int32 dot of block b and every product rounded to f32
// (no FMA).  The 32-wide integer dots are one tcgen05.mma.kind::i8 each
// (M = 128 weight rows on the TMEM lanes, N = 128 token rows on the TMEM
// columns, K = 32 = one block), written to their own TMEM buffer; the epilogue
// warps read each block's int32 tile and apply the scales and the in-order f32
// sum in registers, so every output is bit-identical to the reference (and to
// the batch-1 GEMV).  The per-block epilogue, not the tensor core, bounds the
// kernel: 4 f32 operations per (m, n, block) against one 64-cycle MMA per
// 128x128x32 tile-block.
//
// Pipeline (one CTA per SM, persistent over 128x128 output tiles):
//   warp 0, lane 0: TMA loads of 256-wide K stages (weights and activations as
//     128-byte-swizzled K-major boxes, both scale tables as plain boxes);
//   warp 1, lane 0: one MMA per 32-block into TMEM buffer g % 4, committed to
//     that buffer's barrier; a stage is released after its 8 MMAs complete;
//   warps 2..17: TMEM -> registers (32 columns x 32 lanes each), scales, sums;
//     each warp hands the TMEM buffer back at once and the stage's scales when
//     it finishes the stage's last block.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <stdlib.h>

#include <mutex>

#include "attention_core.cuh"
#include "common.cuh"
#include "gemv_core.cuh"
#include "prefill.cuh"

namespace llmrs {

namespace {

// the row quantiser runs the batch-1 GEMV's prologue with its thread count, so
// both paths sum the RMSNorm squares in the same order
constexpr int PG_QUANT_THREADS = PRO_THREADS;
constexpr int PG_TBUF = 4;                           // TMEM accumulator buffers (128 columns each)
constexpr int PG_EPI_WARPS = 16;
constexpr int PG_THREADS = (2 + PG_EPI_WARPS) * 32;  // producer warp, MMA warp, epilogue warps
constexpr uint32_t PG_TMEM_COLS = PG_TBUF * PG_TILE; // 512: all of TMEM
// int32 i with |i| < 2^22, plus these bits, is the float 1.5*2^23 + i exactly
constexpr int PG_MAGIC = 0x4B400000;
constexpr float PG_MAGIC_F = 12582912.0f;

// per-stage shared memory (bytes; every piece 1024-aligned).  Q4_0 weights
// arrive as a plain box of nibbles (NIB) that the producer warp unpacks into
// the same swizzled int8 layout TMA writes for Q8_0.
constexpr int PG_BOX = PG_TILE * 128; // one 128-row x 128-byte box
template <int WF>
struct PgLay {
    static constexpr int STAGES = WF ? 3 : 2;
    static constexpr int OFF_W = 0;                     // int8 weights: 2 swizzled boxes (K 0..127, 128..255)
    static constexpr int OFF_A = OFF_W + 2 * PG_BOX;    // activations: 2 swizzled boxes
    static constexpr int OFF_WS = OFF_A + 2 * PG_BOX;   // weight scales [128 rows][8 blocks] (f16 or f32)
    static constexpr int OFF_AS = OFF_WS + 4096;        // activation scales [8 blocks][128 tokens] f32
    static constexpr int OFF_AC = OFF_AS + 4096;        // Q4: conversion bias [8 blocks][128 tokens] i32
    static constexpr int OFF_NIB = OFF_AC + (WF ? 0 : 4096); // Q4: nibbles [128 rows][128 bytes]
    static constexpr int STAGE = OFF_NIB + (WF ? 0 : PG_BOX);
    static constexpr int BAR_OFF = STAGES * STAGE;
    static constexpr int SMEM = BAR_OFF + 256 + 1024;   // barriers + alignment slack
    static_assert(SMEM <= 232448, "prefill GEMM shared memory over the per-block limit");
};

// ------------------------------------------------------------ tcgen05 helpers
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// whole warp: allocate ncols TMEM columns, base address written to *slot
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// shared-memory matrix descriptor: K-major operand in 128-byte-swizzled
// 8-row x 128-byte atoms stacked every 1024 bytes (what a TMA box of
// 128-byte rows with SWIZZLE_128B writes)
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);        // start address
    d |= (uint64_t)1u << 16;                        // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;              // stride byte offset: next 8-row atom
    d |= (uint64_t)1u << 46;                        // descriptor version (sm_100)
    d |= (uint64_t)2u << 61;                        // SWIZZLE_128B
    return d;
}

// instruction descriptor, kind::i8: s32 accumulator, A (weights) signed or
// unsigned, B (activations) signed, both K-major, M = 128, N = 128
template <bool A_SIGNED>
__host__ __device__ constexpr uint32_t i8_idesc()
{
    return (2u << 4) | ((A_SIGNED ? 1u : 0u) << 7) | (1u << 10) | ((uint32_t)(PG_TILE >> 3) << 17) |
           ((uint32_t)(PG_TILE >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc)
{
    // enable-input-d false: each block's dot lands in a cleared accumulator
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0)
        : "memory");
}

// arrive on bar once every tcgen05 operation this thread issued has completed
__device__ __forceinline__ void tc_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: lane l gets TMEM lane (base lane
// + l), columns col .. col+31.  The wait is tied to the registers so no use
// of them is scheduled before it.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                   "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                   "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]),
                   "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]),
                   "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns (no wait)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                 "%13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15])
                 : "r"(taddr)
                 : "memory");
}

// wait for this thread's TMEM loads; tied to r so no use of r moves above it
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[16])
{
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                   "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                   "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}

// packed f32 pairs, round-to-nearest (explicit .rn: never contracted to FMA)
__device__ __forceinline__ float2 add2(float2 a, float2 b)
{
    float2 c;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(reinterpret_cast<uint64_t &>(c))
        : "l"(reinterpret_cast<uint64_t &>(a)), "l"(reinterpret_cast<uint64_t &>(b)));
    return c;
}

__device__ __forceinline__ float2 mul2(float2 a, float2 b)
{
    float2 c;
    asm("mul.rn.f32x2 %0, %1, %2;"
        : "=l"(reinterpret_cast<uint64_t &>(c))
        : "l"(reinterpret_cast<uint64_t &>(a)), "l"(reinterpret_cast<uint64_t &>(b)));
    return c;
}

// acc[i] += (float)isum_i * (sw * sa[i]) for 16 token columns, each product
// rounded to f32.  isum arrives as raw int32 TMEM words and is converted
// exactly through the float bits of 1.5*2^23 + isum: Q8_0 adds the constant
// bias, Q4_0 the per-(token, block) bias 1.5*2^23 - 8*sum(codes) that also
// removes the nibble offset.  Products are packed f32 pairs; the running sums
// stay scalar, because ptxas contracts a packed multiply feeding a packed add
// into one FMA, which would skip the product's rounding.
template <int WF>
__device__ __forceinline__ void block_sum16(float *acc, const uint32_t (&r)[16], float sw, const float *sa,
                                            const int *ac)
{
    const float2 sw2 = make_float2(sw, sw);
    const float2 neg_magic = make_float2(-PG_MAGIC_F, -PG_MAGIC_F);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 a = reinterpret_cast<const float4 *>(sa)[i]; // the same address in every lane: broadcast
        int4 bias = make_int4(PG_MAGIC, PG_MAGIC, PG_MAGIC, PG_MAGIC);
        if (!WF)
            bias = reinterpret_cast<const int4 *>(ac)[i];
        float2 f0 = make_float2(__int_as_float((int)r[4 * i] + bias.x), __int_as_float((int)r[4 * i + 1] + bias.y));
        float2 f1 = make_float2(__int_as_float((int)r[4 * i + 2] + bias.z), __int_as_float((int)r[4 * i + 3] + bias.w));
        f0 = add2(f0, neg_magic); // exact: (float)isum
        f1 = add2(f1, neg_magic);
        const float2 t0 = mul2(f0, mul2(sw2, make_float2(a.x, a.y)));
        const float2 t1 = mul2(f1, mul2(sw2, make_float2(a.z, a.w)));
        acc[4 * i] = __fadd_rn(acc[4 * i], t0.x);
        acc[4 * i + 1] = __fadd_rn(acc[4 * i + 1], t0.y);
        acc[4 * i + 2] = __fadd_rn(acc[4 * i + 2], t1.x);
        acc[4 * i + 3] = __fadd_rn(acc[4 * i + 3], t1.y);
    }
}

struct PgParams {
    float *y;
    const float *residual;
    int N, K, M, ldy, ldr;
    int tiles_n, tiles_m;
    uint32_t *err;
};

__device__ __forceinline__ uint8_t *align1024(uint8_t *p)
{
    return reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// ------------------------------------------------------------------ the GEMM
// Q4_0: unpack one stage's nibble box into the swizzled int8 layout the MMA
// reads (whole producer warp).  Block b of a row becomes [lo nibbles of its 16
// bytes | hi nibbles] = [elements 0,2,..,30 | 1,3,..,31] as unsigned 0..15,
// the order the Q4 activation rows use; the -8 offset is folded into the
// per-block bias of the epilogue.
__device__ __forceinline__ void unpack_q4_stage(const uint8_t *nib, uint8_t *w, int lane)
{
    const uint32_t m = 0x0F0F0F0Fu;
    const int b = lane & 7, c0 = (b & 3) * 2;
    uint8_t *box = w + (b >> 2) * PG_BOX;
#pragma unroll 4
    for (int r0 = 0; r0 < PG_TILE; r0 += 4) {
        const int row = r0 + (lane >> 3);
        const uint4 v = *reinterpret_cast<const uint4 *>(nib + row * 128 + b * 16);
        const uint4 lo = make_uint4(v.x & m, v.y & m, v.z & m, v.w & m);
        const uint4 hi = make_uint4((v.x >> 4) & m, (v.y >> 4) & m, (v.z >> 4) & m, (v.w >> 4) & m);
        uint8_t *rp = box + row * 128;
        *reinterpret_cast<uint4 *>(rp + ((c0 ^ (row & 7)) << 4)) = lo;
        *reinterpret_cast<uint4 *>(rp + (((c0 + 1) ^ (row & 7)) << 4)) = hi;
    }
}

// WF: 1 = Q8_0 weights (int8 codes), 0 = Q4_0 (planar nibbles).
// ST: weight scale storage 0 = f16, 1 = f32.
template <int WF, int ST, int EPI>
__global__ void __launch_bounds__(PG_THREADS, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tws,
                        const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tas,
                        const __grid_constant__ CUtensorMap tac, const PgParams p)
{
    using Lay = PgLay<WF>;
    constexpr int S = Lay::STAGES;
    extern __shared__ uint8_t pg_smem_raw[];
    uint8_t *sm = align1024(pg_smem_raw);
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + Lay::BAR_OFF);
    uint64_t *empty = full + S;
    uint64_t *conv = empty + S; // Q4: the stage's weights are unpacked
    uint64_t *tfull = conv + S;
    uint64_t *tempty = tfull + PG_TBUF;
    uint64_t *drain = tempty + PG_TBUF;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + PG_EPI_WARPS); // MMA commit + every epilogue warp (the stage's scales)
            mbar_init(&conv[s], 1);
        }
        for (int b = 0; b < PG_TBUF; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], PG_EPI_WARPS);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    if (warp == 1)
        tmem_alloc(tmem_slot, PG_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int nks = p.K / PG_KSTAGE;
    const int ntiles = p.tiles_n * p.tiles_m;
    constexpr uint32_t STAGE_TX = (WF ? 2 * PG_BOX : PG_BOX) + 2 * PG_BOX + PG_TILE * 8 * (ST ? 4 : 2) +
                                  8 * PG_TILE * 4 * (WF ? 1 : 2);

    if (warp == 0) {
        // ---------------------------------------------------------- producer
        const uint64_t pol_w = policy_evict_first(); // weights: each row set is read by tiles_m CTAs at once
        const uint64_t pol_a = policy_evict_last();  // activations: read by every weight tile
        uint32_t it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
            const int tm = tile % p.tiles_m, tn = tile / p.tiles_m;
            for (int ks = 0; ks < nks; ks++, it++) {
                const int s = it % S;
                uint8_t *st = sm + s * Lay::STAGE;
                if (lane == 0) {
                    ok = mbar_wait(&empty[s], ((it / S) & 1) ^ 1, p.err);
                    if (ok) {
                        mbar_arrive_expect_tx(&full[s], STAGE_TX);
                        const int k0 = ks * PG_KSTAGE;
                        if (WF) {
                            tma_load_2d(st + Lay::OFF_W, &tw, k0, tn * PG_TILE, &full[s], pol_w);
                            tma_load_2d(st + Lay::OFF_W + PG_BOX, &tw, k0 + 128, tn * PG_TILE, &full[s], pol_w);
                        } else {
                            tma_load_2d(st + Lay::OFF_NIB, &tw, k0 / 2, tn * PG_TILE, &full[s], pol_w);
                            tma_load_2d(st + Lay::OFF_AC, &tac, tm * PG_TILE, ks * 8, &full[s], pol_a);
                        }
                        tma_load_2d(st + Lay::OFF_A, &ta, k0, tm * PG_TILE, &full[s], pol_a);
                        tma_load_2d(st + Lay::OFF_A + PG_BOX, &ta, k0 + 128, tm * PG_TILE, &full[s], pol_a);
                        tma_load_2d(st + Lay::OFF_WS, &tws, ks * 8, tn * PG_TILE, &full[s], pol_w);
                        tma_load_2d(st + Lay::OFF_AS, &tas, tm * PG_TILE, ks * 8, &full[s], pol_a);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok)
                    break;
                if (!WF) {
                    // the nibbles of this stage, then the whole warp unpacks them
                    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (it / S) & 1, p.err))) {
                        ok = false;
                        break;
                    }
                    unpack_q4_stage(st + Lay::OFF_NIB, st + Lay::OFF_W, lane);
                    fence_proxy_async_smem(); // generic-proxy writes before the tensor core reads them
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive(&conv[s]);
                }
            }
        }
    } else if (warp == 1) {
        // --------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t IDESC = i8_idesc<WF == 1>();
            uint32_t it = 0, g = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                for (int ks = 0; ks < nks; ks++, it++) {
                    const int s = it % S;
                    if (!mbar_wait(WF ? &full[s] : &conv[s], (it / S) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t wb = smem_addr(sm + s * Lay::STAGE + Lay::OFF_W);
                    const uint32_t ab = smem_addr(sm + s * Lay::STAGE + Lay::OFF_A);
#pragma unroll 1
                    for (int j = 0; j < 8; j++, g++) {
                        const int buf = g % PG_TBUF;
                        if (!mbar_wait(&tempty[buf], ((g / PG_TBUF) & 1) ^ 1, p.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t koff = (uint32_t)((j >> 2) * PG_BOX + (j & 3) * 32);
                        mma_i8(tmem + (uint32_t)(buf * PG_TILE), sw128_desc(wb + koff), sw128_desc(ab + koff), IDESC);
                        tc_commit(&tfull[buf]);
                    }
                    if (!ok)
                        break;
                    tc_commit(&empty[s]); // operands of this stage no longer read
                }
            }
            // every MMA this thread issued has completed before TMEM is freed
            tc_commit(drain);
            mbar_wait(drain, 0, p.err);
        }
    } else {
        // ----------------------------------------------------------- epilogue
        // Each warp owns 32 TMEM lanes (weight rows) x 32 columns (tokens) and
        // reads them in halves of 16 columns: the load of the next half is in
        // flight while the current half is summed.
        const int q = warp & 3;           // TMEM lane quarter this warp may access
        const int cg = (warp - 2) >> 2;   // token columns cg*32 .. +31
        const int row_l = q * 32 + lane;  // weight row within the tile
        const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cg * 32);
        const int my_tiles = (int)blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
        const uint32_t total = (uint32_t)my_tiles * (uint32_t)nks * 8u; // blocks this CTA sums
        uint32_t it = 0, g = 0;
        bool ok = true;
        uint32_t ra[16], rb[16];
        auto buf_of = [](uint32_t gg) { return (uint32_t)(gg % PG_TBUF) * PG_TILE; };
        if (total > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(&tfull[0], 0, p.err));
            tc_fence_after();
            if (ok)
                tmem_ld16(tl, ra);
        }
        for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
            const int tm = tile % p.tiles_m, tn = tile / p.tiles_m;
            float acc[32];
#pragma unroll
            for (int i = 0; i < 32; i++)
                acc[i] = 0.0f;
            for (int ks = 0; ok && ks < nks; ks++, it++) {
                const int s = it % S;
                // the stage's scale boxes are visible once its loads completed
                if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (it / S) & 1, p.err))) {
                    ok = false;
                    break;
                }
                const uint8_t *st = sm + s * Lay::STAGE;
                float sw[8];
                if (ST) {
                    const float4 a = *reinterpret_cast<const float4 *>(st + Lay::OFF_WS + row_l * 32);
                    const float4 b = *reinterpret_cast<const float4 *>(st + Lay::OFF_WS + row_l * 32 + 16);
                    sw[0] = a.x; sw[1] = a.y; sw[2] = a.z; sw[3] = a.w;
                    sw[4] = b.x; sw[5] = b.y; sw[6] = b.z; sw[7] = b.w;
                } else {
                    const uint4 h = *reinterpret_cast<const uint4 *>(st + Lay::OFF_WS + row_l * 16);
                    const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        sw[2 * i] = __half2float(__ushort_as_half((unsigned short)(hw[i] & 0xFFFFu)));
                        sw[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(hw[i] >> 16)));
                    }
                }
                const float *sas = reinterpret_cast<const float *>(st + Lay::OFF_AS) + cg * 32;
                const int *acs = reinterpret_cast<const int *>(st + Lay::OFF_AC) + cg * 32;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float *saj = sas + j * PG_TILE;
                    const int *acj = acs + j * PG_TILE;
                    const float swj = sw[j];
                    tmem_wait_ld(ra);
                    tmem_ld16(tl + buf_of(g) + 16, rb);
                    block_sum16<WF>(acc, ra, swj, saj, acj);
                    tmem_wait_ld(rb);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive(&tempty[g % PG_TBUF]); // both halves are in registers
                    g++;
                    if (g < total) {
                        if (!__all_sync(0xffffffffu, mbar_wait(&tfull[g % PG_TBUF], (g / PG_TBUF) & 1, p.err)))
                            ok = false;
                        tc_fence_after();
                        if (ok)
                            tmem_ld16(tl + buf_of(g), ra);
                    }
                    block_sum16<WF>(acc + 16, rb, swj, saj + 16, acj + 16);
                    if (!ok)
                        break;
                }
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&empty[s]); // this warp is done with the stage's scales
            }
            if (!ok)
                break;
            // ---- store: lanes write 32 consecutive weight rows of one token row
            const int n = tn * PG_TILE + row_l;
            const int m0 = tm * PG_TILE + cg * 32;
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const float v = acc[i];
                const int m = m0 + i;
                if (EPI == PEPI_SILU) {
                    const float up = __shfl_down_sync(0xffffffffu, v, 1);
                    if (m < p.M && n < p.N && (n & 1) == 0) {
                        const float silu = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
                        p.y[(size_t)m * p.ldy + (n >> 1)] = __fmul_rn(silu, up);
                    }
                } else if (m < p.M && n < p.N) {
                    if (EPI == PEPI_RESIDUAL)
                        p.y[(size_t)m * p.ldy + n] = __fadd_rn(v, p.residual[(size_t)m * p.ldr + n]);
                    else
                        p.y[(size_t)m * p.ldy + n] = v;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, PG_TMEM_COLS);
    }
}

// ------------------------------------------------- the GEMM, bf16 operands
// Codes are small integers, exact in bf16, and every partial sum of a block's
// 32 products is an integer below 2^20, exact in the f32 accumulator: two
// tcgen05.mma.kind::f16 (K = 16 each) per Q8_0 block leave the block's dot
// already as a float, so the epilogue is s_w*s_a, isum*(s_w*s_a) and the
// in-order sum (3 FP32-pipe operations per output and block instead of 4 plus
// an integer add).  Operands are twice the bytes: a stage is 4 blocks.
constexpr int PB_BLOCKS = 4;                          // Q8_0 blocks per stage
constexpr int PB_BOX = PG_TILE * 128;                 // 128 rows x 64 bf16 (one swizzle span)
struct PbLay {
    static constexpr int STAGES = 3;
    static constexpr int OFF_W = 0;                   // 2 swizzled boxes: K 0..63, 64..127 of the stage
    static constexpr int OFF_A = OFF_W + 2 * PB_BOX;  // 2 swizzled boxes
    static constexpr int OFF_WS = OFF_A + 2 * PB_BOX; // weight scales [4 blocks][128 rows] f32
    static constexpr int OFF_AS = OFF_WS + 2048;      // activation scales [4 blocks][128 tokens] f32
    static constexpr int STAGE = OFF_AS + 2048;       // 68 KB
    static constexpr int BAR_OFF = STAGES * STAGE;
    static constexpr int SMEM = BAR_OFF + 256 + 1024;
    static_assert(SMEM <= 232448, "prefill bf16 GEMM shared memory over the per-block limit");
};

// kind::f16 instruction descriptor: f32 accumulator, A and B bf16, K-major,
// M = 128, N = 128
__host__ __device__ constexpr uint32_t bf16_idesc()
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(PG_TILE >> 3) << 17) | ((uint32_t)(PG_TILE >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

// acc[i] += f_i * (sw * sa[i]) for 16 token columns (f_i: the block's dot as float)
__device__ __forceinline__ void block_sum16_f(float *acc, const uint32_t (&r)[16], float sw, const float *sa)
{
    const float2 sw2 = make_float2(sw, sw);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 a = reinterpret_cast<const float4 *>(sa)[i]; // broadcast
        const float2 f0 = make_float2(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]));
        const float2 f1 = make_float2(__uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
        const float2 t0 = mul2(f0, mul2(sw2, make_float2(a.x, a.y)));
        const float2 t1 = mul2(f1, mul2(sw2, make_float2(a.z, a.w)));
        acc[4 * i] = __fadd_rn(acc[4 * i], t0.x);
        acc[4 * i + 1] = __fadd_rn(acc[4 * i + 1], t0.y);
        acc[4 * i + 2] = __fadd_rn(acc[4 * i + 2], t1.x);
        acc[4 * i + 3] = __fadd_rn(acc[4 * i + 3], t1.y);
    }
}

template <int EPI>
__global__ void __launch_bounds__(PG_THREADS, 1)
    prefill_gemm_bf16_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tws,
                             const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tas,
                             const PgParams p)
{
    using Lay = PbLay;
    constexpr int S = Lay::STAGES;
    extern __shared__ uint8_t pg_smem_raw[];
    uint8_t *sm = align1024(pg_smem_raw);
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + Lay::BAR_OFF);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;
    uint64_t *tempty = tfull + PG_TBUF;
    uint64_t *drain = tempty + PG_TBUF;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + PG_EPI_WARPS);
        }
        for (int b = 0; b < PG_TBUF; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], PG_EPI_WARPS);
        }
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    if (warp == 1)
        tmem_alloc(tmem_slot, PG_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int nks = p.K / (PB_BLOCKS * 32);
    const int ntiles = p.tiles_n * p.tiles_m;
    constexpr uint32_t STAGE_TX = 4 * PB_BOX + 2 * PB_BLOCKS * PG_TILE * 4;

    if (warp == 0) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_a = policy_evict_last();
            uint32_t it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                const int tm = tile % p.tiles_m, tn = tile / p.tiles_m;
                for (int ks = 0; ks < nks; ks++, it++) {
                    const int s = it % S;
                    if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1, p.err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = sm + s * Lay::STAGE;
                    mbar_arrive_expect_tx(&full[s], STAGE_TX);
                    const int k0 = ks * PB_BLOCKS * 32; // element index
                    tma_load_2d(st + Lay::OFF_W, &tw, k0, tn * PG_TILE, &full[s], pol_w);
                    tma_load_2d(st + Lay::OFF_W + PB_BOX, &tw, k0 + 64, tn * PG_TILE, &full[s], pol_w);
                    tma_load_2d(st + Lay::OFF_A, &ta, k0, tm * PG_TILE, &full[s], pol_a);
                    tma_load_2d(st + Lay::OFF_A + PB_BOX, &ta, k0 + 64, tm * PG_TILE, &full[s], pol_a);
                    tma_load_2d(st + Lay::OFF_WS, &tws, tn * PG_TILE, ks * PB_BLOCKS, &full[s], pol_w);
                    tma_load_2d(st + Lay::OFF_AS, &tas, tm * PG_TILE, ks * PB_BLOCKS, &full[s], pol_a);
                }
            }
        }
    } else if (warp == 1) {
        // --------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t IDESC = bf16_idesc();
            uint32_t it = 0, g = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
                for (int ks = 0; ks < nks; ks++, it++) {
                    const int s = it % S;
                    if (!mbar_wait(&full[s], (it / S) & 1, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t wb = smem_addr(sm + s * Lay::STAGE + Lay::OFF_W);
                    const uint32_t ab = smem_addr(sm + s * Lay::STAGE + Lay::OFF_A);
#pragma unroll 1
                    for (int j = 0; j < PB_BLOCKS; j++, g++) {
                        const int buf = g % PG_TBUF;
                        if (!mbar_wait(&tempty[buf], ((g / PG_TBUF) & 1) ^ 1, p.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        // block j: 64 bytes at (j % 2) * 64 of box j / 2; two K = 16 halves
                        const uint32_t koff = (uint32_t)((j >> 1) * PB_BOX + (j & 1) * 64);
                        const uint32_t d = tmem + (uint32_t)(buf * PG_TILE);
                        mma_bf16(d, sw128_desc(wb + koff), sw128_desc(ab + koff), IDESC, 0);
                        mma_bf16(d, sw128_desc(wb + koff + 32), sw128_desc(ab + koff + 32), IDESC, 1);
                        tc_commit(&tfull[buf]);
                    }
                    if (!ok)
                        break;
                    tc_commit(&empty[s]);
                }
            }
            tc_commit(drain);
            mbar_wait(drain, 0, p.err);
        }
    } else {
        // ----------------------------------------------------------- epilogue
        const int q = warp & 3;
        const int cg = (warp - 2) >> 2;
        const int row_l = q * 32 + lane;
        const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cg * 32);
        const int my_tiles = (int)blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
        const uint32_t total = (uint32_t)my_tiles * (uint32_t)nks * PB_BLOCKS;
        uint32_t it = 0, g = 0;
        bool ok = true;
        uint32_t ra[16], rb[16];
        auto buf_of = [](uint32_t gg) { return (uint32_t)(gg % PG_TBUF) * PG_TILE; };
        if (total > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(&tfull[0], 0, p.err));
            tc_fence_after();
            if (ok)
                tmem_ld16(tl, ra);
        }
        for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
            const int tm = tile % p.tiles_m, tn = tile / p.tiles_m;
            float acc[32];
#pragma unroll
            for (int i = 0; i < 32; i++)
                acc[i] = 0.0f;
            for (int ks = 0; ok && ks < nks; ks++, it++) {
                const int s = it % S;
                if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (it / S) & 1, p.err))) {
                    ok = false;
                    break;
                }
                const uint8_t *st = sm + s * Lay::STAGE;
                const float *wss = reinterpret_cast<const float *>(st + Lay::OFF_WS) + row_l;
                const float *sas = reinterpret_cast<const float *>(st + Lay::OFF_AS) + cg * 32;
#pragma unroll
                for (int j = 0; j < PB_BLOCKS; j++) {
                    const float swj = wss[j * PG_TILE];
                    const float *saj = sas + j * PG_TILE;
                    tmem_wait_ld(ra);
                    tmem_ld16(tl + buf_of(g) + 16, rb);
                    block_sum16_f(acc, ra, swj, saj);
                    tmem_wait_ld(rb);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive(&tempty[g % PG_TBUF]);
                    g++;
                    if (g < total) {
                        if (!__all_sync(0xffffffffu, mbar_wait(&tfull[g % PG_TBUF], (g / PG_TBUF) & 1, p.err)))
                            ok = false;
                        tc_fence_after();
                        if (ok)
                            tmem_ld16(tl + buf_of(g), ra);
                    }
                    block_sum16_f(acc + 16, rb, swj, saj + 16);
                    if (!ok)
                        break;
                }
                __syncwarp();
                if (lane == 0)
                    mbar_arrive(&empty[s]);
            }
            if (!ok)
                break;
            const int n = tn * PG_TILE + row_l;
            const int m0 = tm * PG_TILE + cg * 32;
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const float v = acc[i];
                const int m = m0 + i;
                if (EPI == PEPI_SILU) {
                    const float up = __shfl_down_sync(0xffffffffu, v, 1);
                    if (m < p.M && n < p.N && (n & 1) == 0) {
                        const float silu = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
                        p.y[(size_t)m * p.ldy + (n >> 1)] = __fmul_rn(silu, up);
                    }
                } else if (m < p.M && n < p.N) {
                    if (EPI == PEPI_RESIDUAL)
                        p.y[(size_t)m * p.ldy + n] = __fadd_rn(v, p.residual[(size_t)m * p.ldr + n]);
                    else
                        p.y[(size_t)m * p.ldy + n] = v;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, PG_TMEM_COLS);
    }
}

// ------------------------------------------------- per-row activation quantise
struct PqParams {
    const float *x;
    const float *norm_w;
    int8_t *q;
    float *s;
    int *c;
    int ldx, K, Mpad;
    float eps;
    uint32_t *err;
};

// One CTA per row: the GEMV's activation prologue (same thread layout, so the
// RMSNorm sum of squares and every rounding match the batch-1 path bit for
// bit), then the row's codes and block-major scales go out to global memory.
template <int WF, int PRO, bool BF>
__global__ void __launch_bounds__(PG_QUANT_THREADS) prefill_quant_kernel(const PqParams a)
{
    extern __shared__ __align__(16) uint8_t qsm[];
    const int m = blockIdx.x, K = a.K, nb = K >> 5;
    uint32_t *act = reinterpret_cast<uint32_t *>(qsm); // K/4 words
    float *act_s = reinterpret_cast<float *>(act + K / 4);
    int *act_c = reinterpret_cast<int *>(act_s + nb);
    float *red = reinterpret_cast<float *>(act_c + nb);
    GemvParams p{};
    p.x = a.x + (size_t)m * a.ldx;
    p.norm_w = a.norm_w;
    p.eps = a.eps;
    p.K = K;
    p.err = a.err;
    load_activation<WF>(p, PRO, act, act_s, act_c, red, threadIdx.x, PG_QUANT_THREADS, 1, nullptr);
    __syncthreads();
    if (BF) { // codes as bf16 (exact: |code| <= 127), 8 per 16-byte store
        uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(a.q) + (size_t)m * K);
        for (int i = threadIdx.x; i < K / 8; i += PG_QUANT_THREADS) {
            const uint2 c = reinterpret_cast<const uint2 *>(act)[i];
            const uint32_t w[2] = {c.x, c.y};
            uint32_t o[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint32_t src = w[k >> 1] >> (16 * (k & 1));
                const __nv_bfloat16 lo = __float2bfloat16_rn((float)(int8_t)(src & 0xFF));
                const __nv_bfloat16 hi = __float2bfloat16_rn((float)(int8_t)((src >> 8) & 0xFF));
                o[k] = (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
            }
            dst[i] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    } else {
        uint4 *dst = reinterpret_cast<uint4 *>(a.q + (size_t)m * K);
        for (int i = threadIdx.x; i < K / 16; i += PG_QUANT_THREADS)
            dst[i] = reinterpret_cast<const uint4 *>(act)[i];
    }
    for (int b = threadIdx.x; b < nb; b += PG_QUANT_THREADS) {
        a.s[(size_t)b * a.Mpad + m] = act_s[b];
        if (WF == 0 && !BF)
            a.c[(size_t)b * a.Mpad + m] = PG_MAGIC + act_c[b];
    }
}

// bf16 copy of one linear: thread = (row n, block b); Q4 codes become
// nibble - 8 in natural element order; scales f32, block-major [K/32][N]
template <int WF, int ST>
__global__ void prefill_to_bf16_kernel(const uint8_t *codes, const void *scales, __nv_bfloat16 *wbf, float *sbf, int N,
                                       int K)
{
    const int nb = K / 32;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)N * nb)
        return;
    const int n = (int)(i / nb), b = (int)(i % nb);
    uint32_t o[16];
    if (WF) {
        const uint4 *src = reinterpret_cast<const uint4 *>(codes + (size_t)n * K + (size_t)b * 32);
        const uint4 v0 = src[0], v1 = src[1];
        const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const uint32_t x = w[k >> 1] >> (16 * (k & 1));
            o[k] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn((float)(int8_t)(x & 0xFF))) |
                   ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn((float)(int8_t)((x >> 8) & 0xFF))) << 16);
        }
    } else {
        const uint4 v = *reinterpret_cast<const uint4 *>(codes + (size_t)n * (K / 2) + (size_t)b * 16);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 16; k++) { // byte k: element 2k (low nibble), 2k+1 (high)
            const uint32_t byte = (w[k >> 2] >> (8 * (k & 3))) & 0xFF;
            o[k] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn((float)((int)(byte & 15) - 8))) |
                   ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn((float)((int)(byte >> 4) - 8))) << 16);
        }
    }
    uint4 *dst = reinterpret_cast<uint4 *>(wbf + (size_t)n * K + (size_t)b * 32);
#pragma unroll
    for (int k = 0; k < 4; k++)
        dst[k] = make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
    float sc;
    if (ST)
        sc = reinterpret_cast<const float *>(scales)[(size_t)n * nb + b];
    else
        sc = __half2float(reinterpret_cast<const __half *>(scales)[(size_t)n * nb + b]);
    sbf[(size_t)b * N + n] = sc;
}

size_t quant_smem(int K) { return (size_t)K + (size_t)(K / 32) * 8 + 32 * 4; }

// ------------------------------------------------------ RoPE + KV append
// one warp per (row m, head h), h over q heads, k heads, v heads
template <int D>
__global__ void prefill_rope_append_kernel(float *qkv, float *kc, float *vc, const float *rope_cos,
                                           const float *rope_sin, int M, int start, int Hq, int Hkv, int S)
{
    constexpr int DL = D / 32;
    const int gw = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    const int nh = Hq + 2 * Hkv;
    if (gw >= M * nh)
        return;
    const int m = gw / nh, h = gw % nh, pos = start + m;
    float *src = qkv + (size_t)m * nh * D + (size_t)h * D + lane * DL;
    float x[DL];
#pragma unroll
    for (int k = 0; k < DL; k++)
        x[k] = src[k];
    if (h < Hq + Hkv) {
        float c[DL], s[DL];
        rope_table_lane<D>(c, s, lane, rope_cos + (size_t)pos * (D / 2), rope_sin + (size_t)pos * (D / 2));
        rope_lane<D>(x, lane, c, s);
    }
    float *dst;
    if (h < Hq)
        dst = src;
    else if (h < Hq + Hkv)
        dst = kc + ((size_t)(h - Hq) * S + pos) * D + lane * DL;
    else
        dst = vc + ((size_t)(h - Hq - Hkv) * S + pos) * D + lane * DL;
#pragma unroll
    for (int k = 0; k < DL; k++)
        dst[k] = x[k];
}

// ------------------------------------------------------------- attention
// CTA = (RB query rows, KV head g), twice when few cached positions precede
// the rows: row blocks b and nblk-1-b, so every CTA sees about the same number
// of causal positions.  The RB * NREP = 64 query vectors of the NREP heads of
// g share every K/V chunk of 32 positions, staged in shared memory with
// cp.async (double-buffered).  Per chunk:
//   scores: thread = 2 query vectors x 4 positions; each score sums q[d]*k[d]
//     for d = 0..D-1 in order, unfused, then * 1/sqrt(D) -- bit-exact with
//     the reference's f32 dot (src/backend/cpu.rs:458-551, non-aarch64) --
//     and positions past the row's own are masked (src/core/layer.rs:260-269);
//   online softmax per query vector (8 lanes share one);
//   P.V: thread = 4 query vectors x D/16 dims, f32 FMA.
constexpr int PA_KC = 32;       // positions per chunk
constexpr int PA_QV = 64;       // query vectors per CTA
constexpr int PA_THREADS = 256;

template <int D>
struct PaLayout {
    static constexpr int QS = D + 4;                                     // padded rows: conflict-free 16-byte loads
    static constexpr int Q_OFF = 0;                                      // [PA_QV][QS]
    static constexpr int K_OFF = Q_OFF + PA_QV * QS * 4;                 // [2][PA_KC][QS]
    static constexpr int V_OFF = K_OFF + 2 * PA_KC * QS * 4;             // [2][PA_KC][D]
    static constexpr int PS = PA_QV + 4;                                 // padded probability rows
    static constexpr int P_OFF = V_OFF + 2 * PA_KC * D * 4;              // [PA_KC][PS] probabilities
    static constexpr int C_OFF = P_OFF + PA_KC * PS * 4;                 // [PA_QV] rescale of the running sums
    static constexpr int BYTES = C_OFF + PA_QV * 4;
};

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <int D, int NREP>
__global__ void __launch_bounds__(PA_THREADS, 2) prefill_attention_kernel(const float *qkv, const float *kc,
                                                                          const float *vc, float *ctx, int M,
                                                                          int start, int Hq, int Hkv, int S,
                                                                          float inv_sqrt_d, int pair)
{
    using Lay = PaLayout<D>;
    constexpr int RB = PA_QV / NREP; // query rows per CTA
    constexpr int QS = Lay::QS;
    constexpr int DPT = D / 16;      // P.V dims per thread
    extern __shared__ __align__(16) uint8_t pasm[];
    float *q_s = reinterpret_cast<float *>(pasm + Lay::Q_OFF);
    float *k_s = reinterpret_cast<float *>(pasm + Lay::K_OFF);
    float *v_s = reinterpret_cast<float *>(pasm + Lay::V_OFF);
    float *p_s = reinterpret_cast<float *>(pasm + Lay::P_OFF);
    float *c_s = reinterpret_cast<float *>(pasm + Lay::C_OFF);
    const int tid = threadIdx.x, lane = tid & 31;
    const int g = blockIdx.y;
    const int ld = (Hq + 2 * Hkv) * D;
    // pair: row blocks b and nblk-1-b, a short causal block and a long one
    const int nblk = (M + RB - 1) / RB;
    for (int pass = 0; pass < 2; pass++) {
        const int blk = pass == 0 ? (int)blockIdx.x : nblk - 1 - (int)blockIdx.x;
        if (pass == 1 && (!pair || blk <= (int)blockIdx.x))
            break;
        __syncthreads(); // the previous block's shared-memory reads are done
        const int m0 = blk * RB;
        const int rows = min(RB, M - m0);
        const int last = start + m0 + rows - 1; // highest position any row of the CTA sees
        const int nch = last / PA_KC + 1;
        const float *kg = kc + (size_t)g * S * D;
        const float *vg = vc + (size_t)g * S * D;

        // chunk loader: K rows into padded rows, V rows plain; positions past
        // `last` are zero-filled (and masked)
        auto load_chunk = [&](int c, int buf) {
            const int t0 = c * PA_KC;
            for (int e = tid; e < PA_KC * D / 4; e += PA_THREADS) {
                const int r = e / (D / 4), d4 = e % (D / 4);
                const int t = t0 + r;
                const bool ok = t <= last;
                const size_t off = (size_t)(ok ? t : 0) * D + d4 * 4;
                cp_async16(k_s + (size_t)(buf * PA_KC + r) * QS + d4 * 4, kg + off, ok);
                cp_async16(v_s + (size_t)(buf * PA_KC + r) * D + d4 * 4, vg + off, ok);
            }
            cp_async_commit();
        };
        load_chunk(0, 0);
        // query vectors qv = r * NREP + h (row m0 + r, head g*NREP + h)
        for (int e = tid; e < PA_QV * D / 4; e += PA_THREADS) {
            const int qv = e / (D / 4), d4 = e % (D / 4);
            const int r = qv / NREP, h = qv % NREP;
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (r < rows)
                v = *reinterpret_cast<const float4 *>(qkv + (size_t)(m0 + r) * ld + (size_t)(g * NREP + h) * D + d4 * 4);
            *reinterpret_cast<float4 *>(q_s + qv * QS + d4 * 4) = v;
        }

        // score-phase roles: query vectors sq, sq+1; positions kq, kq+8, kq+16,
        // kq+24 of the chunk (8 lanes read 8 consecutive K rows: distinct banks)
        constexpr int PS = Lay::PS;
        const int sq = (tid >> 3) * 2, kq = tid & 7;
        int pos_s[2];
#pragma unroll
        for (int i = 0; i < 2; i++)
            pos_s[i] = start + m0 + (sq + i) / NREP;
        float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
        // P.V roles: query vectors oq .. oq+3, dims od .. od+DPT-1
        const int oq = (tid >> 4) * 4, od = (tid & 15) * DPT;
        float o[4][DPT];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < DPT; j++)
                o[i][j] = 0.0f;

        for (int c = 0; c < nch; c++) {
            const int buf = c & 1;
            if (c + 1 < nch) {
                load_chunk(c + 1, buf ^ 1);
                cp_async_wait_1();
            } else {
                cp_async_wait_0();
            }
            __syncthreads(); // chunk c (and q_s) visible
            const float *kb = k_s + (size_t)buf * PA_KC * QS;
            const float *vb = v_s + (size_t)buf * PA_KC * D;
            // ---- scores, d in order, unfused
            float sc[2][4];
#pragma unroll
            for (int i = 0; i < 2; i++)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    sc[i][j] = 0.0f;
#pragma unroll 4
            for (int d4 = 0; d4 < D / 4; d4++) {
                float4 qv[2], kv[4];
#pragma unroll
                for (int i = 0; i < 2; i++)
                    qv[i] = *reinterpret_cast<const float4 *>(q_s + (sq + i) * QS + d4 * 4);
#pragma unroll
                for (int j = 0; j < 4; j++)
                    kv[j] = *reinterpret_cast<const float4 *>(kb + (kq + 8 * j) * QS + d4 * 4);
#pragma unroll
                for (int i = 0; i < 2; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        float t = sc[i][j];
                        t = __fadd_rn(t, __fmul_rn(qv[i].x, kv[j].x));
                        t = __fadd_rn(t, __fmul_rn(qv[i].y, kv[j].y));
                        t = __fadd_rn(t, __fmul_rn(qv[i].z, kv[j].z));
                        t = __fadd_rn(t, __fmul_rn(qv[i].w, kv[j].w));
                        sc[i][j] = t;
                    }
            }
            // ---- online softmax (the 8 lanes of a query-vector pair share it)
            const int t0 = c * PA_KC;
#pragma unroll
            for (int i = 0; i < 2; i++) {
                float mx = -INFINITY;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    sc[i][j] = (t0 + kq + 8 * j <= pos_s[i]) ? __fmul_rn(sc[i][j], inv_sqrt_d) : -INFINITY;
                    mx = fmaxf(mx, sc[i][j]);
                }
#pragma unroll
                for (int off = 1; off < 8; off <<= 1)
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
                const float m_new = fmaxf(m_run[i], mx);
                const float corr = (m_run[i] == -INFINITY) ? 0.0f : expf(m_run[i] - m_new);
                float ps = 0.0f;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float pr = (sc[i][j] == -INFINITY) ? 0.0f : expf(sc[i][j] - m_new);
                    p_s[(kq + 8 * j) * PS + sq + i] = pr;
                    ps += pr;
                }
#pragma unroll
                for (int off = 1; off < 8; off <<= 1)
                    ps += __shfl_xor_sync(0xffffffffu, ps, off);
                l_run[i] = l_run[i] * corr + ps;
                m_run[i] = m_new;
                if ((lane & 7) == 0)
                    c_s[sq + i] = corr;
            }
            __syncthreads(); // probabilities and rescales visible
            // ---- P.V
            float cr[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                cr[i] = c_s[oq + i];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < DPT; j++)
                    o[i][j] *= cr[i];
#pragma unroll 4
            for (int k = 0; k < PA_KC; k++) {
                const float4 pv = *reinterpret_cast<const float4 *>(p_s + k * PS + oq);
                const float pk[4] = {pv.x, pv.y, pv.z, pv.w};
                float vv[DPT];
#pragma unroll
                for (int j = 0; j < DPT; j += 4) {
                    const float4 t = *reinterpret_cast<const float4 *>(vb + k * D + od + j);
                    vv[j] = t.x;
                    vv[j + 1] = t.y;
                    vv[j + 2] = t.z;
                    vv[j + 3] = t.w;
                }
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < DPT; j++)
                        o[i][j] = fmaf(pk[i], vv[j], o[i][j]);
            }
            __syncthreads(); // buffers free for the next loads
        }
        // ---- normalise and store: l of query vector qv lives with the score lanes
        // (sq, sq+1): hand it over through shared memory
        if ((lane & 7) == 0) {
            c_s[sq] = l_run[0];
            c_s[sq + 1] = l_run[1];
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int qv = oq + i, r = qv / NREP, h = qv % NREP;
            if (r >= rows)
                continue;
            const float l = c_s[qv];
            float *dst = ctx + (size_t)(m0 + r) * Hq * D + (size_t)(g * NREP + h) * D + od;
#pragma unroll
            for (int j = 0; j < DPT; j += 4)
                *reinterpret_cast<float4 *>(dst + j) =
                    make_float4(o[i][j] / l, o[i][j + 1] / l, o[i][j + 2] / l, o[i][j + 3] / l);
        }
    } // row blocks
}

// ------------------------------------------------------------- embedding
__global__ void prefill_embed_kernel(const float *embed, const int *ids, float *x, int M, int H, int V, uint32_t *err)
{
    const int m = blockIdx.x;
    int id = ids[m];
    if (id < 0 || id >= V) {
        if (threadIdx.x == 0)
            atomicCAS(err, 0u, (uint32_t)DEV_ERR_BAD_TOKEN);
        id = 0;
    }
    const float4 *src = reinterpret_cast<const float4 *>(embed + (size_t)id * H);
    float4 *dst = reinterpret_cast<float4 *>(x + (size_t)m * H);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x)
        dst[i] = src[i];
}

// 2-D tensor map: `rows` rows of `inner` elements of `elem` bytes, row pitch
// `pitch` bytes
int encode_map(CUtensorMap *map, const void *base, CUtensorMapDataType dt, int elem, size_t inner, size_t rows,
               size_t pitch, int box_x, int box_y, CUtensorMapSwizzle swz)
{
    auto fn = tensor_map_encoder();
    if (!fn)
        return fail(LLMRS_ECUDA, "cuTensorMapEncodeTiled unavailable");
    (void)elem;
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)pitch};
    cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_y};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(LLMRS_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return LLMRS_OK;
}

} // namespace

// ================================================================ host side
size_t prefill_acts_bytes(int M, int K)
{
    const size_t Mpad = (size_t)((M + PG_TILE - 1) / PG_TILE) * PG_TILE;
    const size_t nb = (size_t)K / 32;
    auto up = [](size_t b) { return (b + 1023) & ~size_t(1023); };
    return up(Mpad * K * 2) + up(nb * Mpad * 4) + up(nb * Mpad * 4) + 1024;
}

int prefill_acts_init(PrefillActs *a, void *buf, int M, int K, int wf, int bf16)
{
    LLMRS_CHECK_ARG(a && buf && M > 0 && K > 0 && K % PG_KSTAGE == 0, "prefill acts: bad arguments");
    const int Mpad = (M + PG_TILE - 1) / PG_TILE * PG_TILE;
    const size_t nb = (size_t)K / 32;
    auto up = [](size_t b) { return (b + 1023) & ~size_t(1023); };
    uint8_t *p = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(buf) + 1023) & ~uintptr_t(1023));
    a->q = reinterpret_cast<int8_t *>(p);
    p += up((size_t)Mpad * K * 2);
    a->s = reinterpret_cast<float *>(p);
    p += up(nb * Mpad * 4);
    a->c = reinterpret_cast<int *>(p);
    a->M = M;
    a->Mpad = Mpad;
    a->K = K;
    a->wf = wf;
    a->bf16 = bf16;
    // rows past M read as zero (TMA fill), so padded columns stay finite
    if (bf16)
        LLMRS_TRY(encode_map(&a->tq, a->q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (size_t)K, (size_t)M, (size_t)K * 2,
                             64, PG_TILE, CU_TENSOR_MAP_SWIZZLE_128B));
    else
        LLMRS_TRY(encode_map(&a->tq, a->q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (size_t)K, (size_t)M, (size_t)K, 128,
                             PG_TILE, CU_TENSOR_MAP_SWIZZLE_128B));
    LLMRS_TRY(encode_map(&a->ts, a->s, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (size_t)M, nb, (size_t)Mpad * 4, PG_TILE,
                         bf16 ? PB_BLOCKS : 8, CU_TENSOR_MAP_SWIZZLE_NONE));
    LLMRS_TRY(encode_map(&a->tc, a->c, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, (size_t)M, nb, (size_t)Mpad * 4, PG_TILE, 8,
                         CU_TENSOR_MAP_SWIZZLE_NONE));
    return LLMRS_OK;
}

int prefill_weights_init(PrefillWeights *w, const void *codes, const void *scales, int N, int K, int wf, int st)
{
    LLMRS_CHECK_ARG(w && codes && scales && N > 0 && K > 0, "prefill weights: bad arguments");
    *w = PrefillWeights();
    w->wf = wf;
    w->st = st;
    w->N = N;
    w->K = K;
    const bool aligned = !((uintptr_t)codes & 15) && !((uintptr_t)scales & 15);
    if ((wf != 0 && wf != 1) || K % PG_KSTAGE != 0 || !aligned)
        return LLMRS_OK; // not on the tensor-core path: callers fall back to batch-1 rows
    if (wf == 1) // int8 codes straight into the MMA layout
        LLMRS_TRY(encode_map(&w->tw, codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (size_t)K, (size_t)N, (size_t)K, 128,
                             PG_TILE, CU_TENSOR_MAP_SWIZZLE_128B));
    else // nibble rows, unpacked in shared memory
        LLMRS_TRY(encode_map(&w->tw, codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (size_t)K / 2, (size_t)N, (size_t)K / 2,
                             128, PG_TILE, CU_TENSOR_MAP_SWIZZLE_NONE));
    const size_t sb = st == LLMRS_F32 ? 4 : 2;
    LLMRS_TRY(encode_map(&w->ts, scales, st == LLMRS_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                         (int)sb, (size_t)K / 32, (size_t)N, (size_t)K / 32 * sb, 8, PG_TILE,
                         CU_TENSOR_MAP_SWIZZLE_NONE));
    w->ok = 1;
    return LLMRS_OK;
}

size_t prefill_bf16_bytes(int N, int K)
{
    auto up = [](size_t b) { return (b + 1023) & ~size_t(1023); };
    return up((size_t)N * K * 2) + up((size_t)N * (K / 32) * 4) + 1024;
}

int prefill_weights_to_bf16(PrefillWeights *w, const void *codes, const void *scales, void *buf, cudaStream_t stream)
{
    LLMRS_CHECK_ARG(w && w->ok && codes && scales && buf, "prefill bf16 weights: bad arguments");
    LLMRS_CHECK_ARG(w->N % 4 == 0, "prefill bf16 weights: N=%d not a multiple of 4", w->N);
    const int N = w->N, K = w->K, nb = K / 32;
    auto up = [](size_t b) { return (b + 1023) & ~size_t(1023); };
    uint8_t *p = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(buf) + 1023) & ~uintptr_t(1023));
    w->wbf = p;
    w->sbf = reinterpret_cast<float *>(p + up((size_t)N * K * 2));
    const size_t items = (size_t)N * nb;
    const unsigned grid = (unsigned)((items + 255) / 256);
    __nv_bfloat16 *wb = reinterpret_cast<__nv_bfloat16 *>(w->wbf);
    const uint8_t *c = reinterpret_cast<const uint8_t *>(codes);
    if (w->wf == 1 && w->st == LLMRS_F32)
        prefill_to_bf16_kernel<1, 1><<<grid, 256, 0, stream>>>(c, scales, wb, w->sbf, N, K);
    else if (w->wf == 1)
        prefill_to_bf16_kernel<1, 0><<<grid, 256, 0, stream>>>(c, scales, wb, w->sbf, N, K);
    else if (w->st == LLMRS_F32)
        prefill_to_bf16_kernel<0, 1><<<grid, 256, 0, stream>>>(c, scales, wb, w->sbf, N, K);
    else
        prefill_to_bf16_kernel<0, 0><<<grid, 256, 0, stream>>>(c, scales, wb, w->sbf, N, K);
    LLMRS_CUDA_TRY(cudaGetLastError());
    LLMRS_TRY(encode_map(&w->tw16, w->wbf, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (size_t)K, (size_t)N, (size_t)K * 2,
                         64, PG_TILE, CU_TENSOR_MAP_SWIZZLE_128B));
    LLMRS_TRY(encode_map(&w->ts16, w->sbf, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (size_t)N, (size_t)nb, (size_t)N * 4,
                         PG_TILE, PB_BLOCKS, CU_TENSOR_MAP_SWIZZLE_NONE));
    w->bf16 = 1;
    return LLMRS_OK;
}

int prefill_use_bf16(void)
{
    static const int v = [] {
        const char *e = getenv("LLMRS_PREFILL_BF16");
        return e ? (e[0] == '1' ? 1 : 0) : 1;
    }();
    return v;
}

int prefill_quantize(const float *x, int ldx, const float *norm_w, float eps, PrefillActs &a, uint32_t *err,
                     cudaStream_t stream)
{
    LLMRS_CHECK_ARG(x && a.q && ldx >= a.K && !((uintptr_t)x & 15) && ldx % 4 == 0,
                    "prefill quantize: bad arguments");
    PqParams p{};
    p.x = x;
    p.norm_w = norm_w;
    p.q = a.q;
    p.s = a.s;
    p.c = a.c;
    p.ldx = ldx;
    p.K = a.K;
    p.Mpad = a.Mpad;
    p.eps = eps;
    p.err = err;
    const size_t smem = quant_smem(a.K);
    const dim3 grid(a.M), block(PG_QUANT_THREADS);
    if (a.bf16) { // natural element order for both weight formats
        if (norm_w)
            prefill_quant_kernel<1, PRO_NORM, true><<<grid, block, smem, stream>>>(p);
        else
            prefill_quant_kernel<1, PRO_F32, true><<<grid, block, smem, stream>>>(p);
    } else if (a.wf == 1) {
        if (norm_w)
            prefill_quant_kernel<1, PRO_NORM, false><<<grid, block, smem, stream>>>(p);
        else
            prefill_quant_kernel<1, PRO_F32, false><<<grid, block, smem, stream>>>(p);
    } else {
        if (norm_w)
            prefill_quant_kernel<0, PRO_NORM, false><<<grid, block, smem, stream>>>(p);
        else
            prefill_quant_kernel<0, PRO_F32, false><<<grid, block, smem, stream>>>(p);
    }
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

#define LLMRS_PG_VARIANTS(X)                                                                                \
    X(1, 0, PEPI_STORE) X(1, 0, PEPI_RESIDUAL) X(1, 0, PEPI_SILU) X(1, 1, PEPI_STORE) X(1, 1, PEPI_RESIDUAL) \
    X(1, 1, PEPI_SILU) X(0, 0, PEPI_STORE) X(0, 0, PEPI_RESIDUAL) X(0, 0, PEPI_SILU) X(0, 1, PEPI_STORE)     \
    X(0, 1, PEPI_RESIDUAL) X(0, 1, PEPI_SILU)

int prefill_gemm(const PrefillWeights &w, const PrefillActs &a, int epi, float *y, int ldy, const float *residual,
                 int ldr, uint32_t *err, int sms, cudaStream_t stream)
{
    LLMRS_CHECK_ARG(w.ok, "prefill GEMM: weights not on the tensor-core path");
    LLMRS_CHECK_ARG(a.K == w.K && (a.bf16 ? w.bf16 == 1 : a.wf == w.wf),
                    "prefill GEMM: activation rows do not match the weights");
    LLMRS_CHECK_ARG(y && (epi != PEPI_RESIDUAL || residual) && (epi != PEPI_SILU || w.N % 2 == 0),
                    "prefill GEMM: bad output arguments");
    PgParams p{};
    p.y = y;
    p.residual = residual;
    p.N = w.N;
    p.K = w.K;
    p.M = a.M;
    p.ldy = ldy;
    p.ldr = ldr;
    p.tiles_n = (w.N + PG_TILE - 1) / PG_TILE;
    p.tiles_m = (a.M + PG_TILE - 1) / PG_TILE;
    p.err = err;
    const int tiles = p.tiles_n * p.tiles_m;
    const int grid = tiles < sms ? tiles : sms;
    if (a.bf16) {
#define LLMRS_PB_CASE(EPI)                                                                                    \
    if (epi == EPI) {                                                                                         \
        prefill_gemm_bf16_kernel<EPI><<<grid, PG_THREADS, PbLay::SMEM, stream>>>(w.tw16, w.ts16, a.tq, a.ts, p); \
        LLMRS_CUDA_TRY(cudaGetLastError());                                                                   \
        return LLMRS_OK;                                                                                      \
    }
        LLMRS_PB_CASE(PEPI_STORE) LLMRS_PB_CASE(PEPI_RESIDUAL) LLMRS_PB_CASE(PEPI_SILU)
#undef LLMRS_PB_CASE
        return fail(LLMRS_ENOTSUP, "prefill GEMM: no bf16 kernel for epi=%d", epi);
    }
#define LLMRS_PG_CASE(WF, ST, EPI)                                                                        \
    if (w.wf == WF && (w.st == LLMRS_F32 ? 1 : 0) == ST && epi == EPI) {                                 \
        prefill_gemm_kernel<WF, ST, EPI><<<grid, PG_THREADS, PgLay<WF>::SMEM, stream>>>(w.tw, w.ts, a.tq, a.ts, a.tc, p); \
        LLMRS_CUDA_TRY(cudaGetLastError());                                                               \
        return LLMRS_OK;                                                                                  \
    }
    LLMRS_PG_VARIANTS(LLMRS_PG_CASE)
#undef LLMRS_PG_CASE
    return fail(LLMRS_ENOTSUP, "prefill GEMM: no kernel for wf=%d st=%d epi=%d", w.wf, w.st, epi);
}

int prefill_prepare(void)
{
#define LLMRS_PG_ATTR(WF, ST, EPI)                                                                          \
    LLMRS_CUDA_TRY(cudaFuncSetAttribute(prefill_gemm_kernel<WF, ST, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                        PgLay<WF>::SMEM));
    LLMRS_PG_VARIANTS(LLMRS_PG_ATTR)
#undef LLMRS_PG_ATTR
    LLMRS_CUDA_TRY(cudaFuncSetAttribute(prefill_gemm_bf16_kernel<PEPI_STORE>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, PbLay::SMEM));
    LLMRS_CUDA_TRY(cudaFuncSetAttribute(prefill_gemm_bf16_kernel<PEPI_RESIDUAL>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, PbLay::SMEM));
    LLMRS_CUDA_TRY(cudaFuncSetAttribute(prefill_gemm_bf16_kernel<PEPI_SILU>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, PbLay::SMEM));
    LLMRS_CUDA_TRY(cudaFuncSetAttribute(prefill_attention_kernel<128, 4>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, PaLayout<128>::BYTES));
    LLMRS_CUDA_TRY(cudaFuncSetAttribute(prefill_attention_kernel<128, 8>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, PaLayout<128>::BYTES));
    LLMRS_CUDA_TRY(cudaFuncSetAttribute(prefill_attention_kernel<64, 4>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, PaLayout<64>::BYTES));
    LLMRS_CUDA_TRY(cudaFuncSetAttribute(prefill_attention_kernel<64, 8>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, PaLayout<64>::BYTES));
    return LLMRS_OK;
}

int prefill_rope_append(float *qkv, float *kc, float *vc, const float *rope_cos, const float *rope_sin, int M,
                        int start, int Hq, int Hkv, int D, int S, cudaStream_t stream)
{
    LLMRS_CHECK_ARG(M > 0 && start >= 0 && start + M <= S, "prefill rope: positions out of range");
    const long long warps = (long long)M * (Hq + 2 * Hkv);
    const int block = 256;
    const unsigned grid = (unsigned)((warps * 32 + block - 1) / block);
    if (D == 128)
        prefill_rope_append_kernel<128><<<grid, block, 0, stream>>>(qkv, kc, vc, rope_cos, rope_sin, M, start, Hq, Hkv, S);
    else if (D == 64)
        prefill_rope_append_kernel<64><<<grid, block, 0, stream>>>(qkv, kc, vc, rope_cos, rope_sin, M, start, Hq, Hkv, S);
    else
        return fail(LLMRS_ENOTSUP, "prefill rope: head_dim %d", D);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

int prefill_attention(const float *qkv, const float *kc, const float *vc, float *ctx, int M, int start, int Hq,
                      int Hkv, int D, int S, float inv_sqrt_d, cudaStream_t stream)
{
    LLMRS_CHECK_ARG(M > 0 && start >= 0 && start + M <= S, "prefill attention: positions out of range");
    const int nrep = Hq / Hkv;
    // pair a short and a long row block per CTA when the causal triangle
    // dominates (few cached positions before the rows); else one block each
    const int pair = start < M ? 1 : 0;
#define LLMRS_PA_CASE(DD, NR)                                                                              \
    if (D == DD && nrep == NR) {                                                                           \
        const int nblk = (M + PA_QV / NR - 1) / (PA_QV / NR);                                              \
        const dim3 grid(pair ? (nblk + 1) / 2 : nblk, Hkv);                                                \
        prefill_attention_kernel<DD, NR><<<grid, PA_THREADS, PaLayout<DD>::BYTES, stream>>>(               \
            qkv, kc, vc, ctx, M, start, Hq, Hkv, S, inv_sqrt_d, pair);                                     \
        LLMRS_CUDA_TRY(cudaGetLastError());                                                                \
        return LLMRS_OK;                                                                                   \
    }
    LLMRS_PA_CASE(128, 4) LLMRS_PA_CASE(128, 8) LLMRS_PA_CASE(64, 4) LLMRS_PA_CASE(64, 8)
#undef LLMRS_PA_CASE
    return fail(LLMRS_ENOTSUP, "prefill attention: head_dim %d with %d query heads per KV head", D, nrep);
}

int prefill_embed(const float *embed, const int *ids, float *x, int M, int H, int V, uint32_t *err,
                  cudaStream_t stream)
{
    LLMRS_CHECK_ARG(H % 4 == 0, "prefill embed: hidden %d not a multiple of 4", H);
    prefill_embed_kernel<<<M, 256, 0, stream>>>(embed, ids, x, M, H, V, err);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
}

} // namespace llmrs
