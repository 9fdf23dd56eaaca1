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

#include "gemv_core.cuh"

namespace llmrs {

namespace {

// One binary per (weight format, scale format): the prologue and epilogue are
// run-time choices (p.pro, p.epi), so the five GEMVs of a decode layer run the
// same code and keep it in the SM's instruction cache from launch to launch
// (one instantiation per variant made every launch refetch its code).
template <int WF, int ST, bool TPK>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap ts, const GemvParams p)
{
    extern __shared__ __align__(128) uint8_t smem_raw[];

    griddep_launch_dependents();
    LLMRS_TRACE_PROLOG

    uint8_t *smem = smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u);
    const int S = p.n_stages;
    const SmemLayout L = smem_layout(WF, ST, p.K, S);
    GemvSmem sm;
    sm.ring = smem;
    sm.stage_bytes = L.stage_bytes;
    sm.scale_off = L.scale_off;
    sm.S = S;
    sm.act = reinterpret_cast<uint32_t *>(smem + L.act_off);
    sm.act_s = reinterpret_cast<float *>(smem + L.acts_off);
    sm.act_c = reinterpret_cast<int *>(smem + L.actc_off);
    sm.tbuf = reinterpret_cast<float *>(smem + L.tb_off);
    sm.prod = sm.tbuf; // a CTA uses the transpose buffers or the product slots, never both
    sm.full = reinterpret_cast<uint64_t *>(smem + L.bar_off);
    sm.empty = sm.full + S;
    sm.issued = sm.empty + S;
    sm.pfull = sm.issued + 1;
    sm.pempty = sm.pfull + PSLOTS;
    sm.sbest = reinterpret_cast<unsigned long long *>(sm.pempty + PSLOTS);
    sm.red = reinterpret_cast<float *>(smem + L.red_off);
    const GemvWork w = gemv_work(p, blockIdx.x);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], WPG); // released by the group's warps
        }
        mbar_init(sm.issued, NW);
        for (int i = 0; i < PSLOTS; i++) {
            mbar_init(&sm.pfull[i], WPG); // written by the 4 warps of a group
            mbar_init(&sm.pempty[i], 1);  // released by a summer warp
        }
        *sm.sbest = 0ull;
        fence_mbar_init();
        trace_start(p.trace, p.trace_slot);
    }
    __syncthreads();

    if (warp >= NW && warp < NW + NSUM) { // summer warps (used when groups share a tile)
        gemv_sum(p, p.epi, w, sm, warp - NW);
        return;
    }
    if (warp == NW + NSUM) {
        // Weights do not depend on the previous kernel: the first n_pre stages
        // stream right away, the rest once the consumers have requested the
        // activation (queued behind the weight stream it would arrive last).
        if (lane == 0) {
            uint32_t fill_par = 0, filled = 0;
            InFlight q; // unbounded: one op per kernel, nothing else to wait behind it
            gemv_produce<WF, ST>(&tw, &ts, p, w, sm, fill_par, filled, policy_evict_first(), min(p.n_pre, S), q);
            LLMRS_TRACE_FLUSH(1);
        }
        return;
    }
    const int ctid = threadIdx.x;
    uint32_t cpar = 0;
    gemv_consume<WF, ST, TPK>(p, p.pro, p.epi, w, sm, cpar, ctid, true); // waits for the previous kernel itself
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
    load_activation<WF, PRO == PRO_AR_NORM>(p, PRO, act, act_s, act_c, red, threadIdx.x, SIMPLE_THREADS, 1, nullptr);
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

// RMSNorm + Q8_0 of one row exactly as the decode GEMVs' prologue computes it
// (the same PRO_THREADS threads, block mapping and reduction tree), codes in
// natural order; for parity checks of that prologue.
__global__ void __launch_bounds__(PRO_THREADS) norm_quant_kernel(const GemvParams p, int8_t *q, float *s)
{
    extern __shared__ __align__(16) uint8_t smem[];
    const int nb = p.K >> 5;
    uint32_t *act = reinterpret_cast<uint32_t *>(smem);
    float *act_s = reinterpret_cast<float *>(smem + (size_t)nb * 32);
    int *act_c = reinterpret_cast<int *>(act_s + nb);
    float *red = reinterpret_cast<float *>(act_c + nb);
    load_activation<1>(p, PRO_NORM, act, act_s, act_c, red, threadIdx.x, PRO_THREADS, 1, nullptr);
    named_bar_sync(1, PRO_THREADS);
    for (int i = threadIdx.x; i < nb * 8; i += PRO_THREADS)
        reinterpret_cast<uint32_t *>(q)[i] = act[i];
    for (int b = threadIdx.x; b < nb; b += PRO_THREADS)
        s[b] = act_s[b];
}

constexpr int SIMPLE_SMEM_MAX = 200 * 1024;

template <int WF, int ST>
cudaError_t prepare_fast()
{
    cudaError_t e = cudaFuncSetAttribute(gemv_tma_kernel<WF, ST, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)SMEM_BUDGET + 2048);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemv_tma_kernel<WF, ST, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)SMEM_BUDGET + 2048);
    return e;
}

template <int WF, int ST, int PRO, int EPI>
cudaError_t prepare_one()
{
    return cudaFuncSetAttribute(gemv_simple_kernel<WF, ST, PRO, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                SIMPLE_SMEM_MAX);
}

template <int WF, int ST>
int launch_fast(const GemvPlan &plan, const GemvParams &p0, int pro, int epi, cudaStream_t stream, bool pdl)
{
    GemvParams p = p0;
    p.pro = pro;
    p.epi = epi;
    p.n_stages = plan.stages;
    p.n_pre = gemv_prefetch_stages();
    p.box_rows = plan.box_rows;
    p.rows_per_cta = plan.rows_per_cta;
    // tensor-parallel launches (every GEMV of a tensor-parallel step) share the
    // instantiation that holds the peer-polling prologue
    if (p.tp)
        LLMRS_CUDA_TRY(launch(gemv_tma_kernel<WF, ST, true>, dim3(plan.grid), dim3(NTHREADS), plan.smem, stream, pdl,
                              plan.tw, plan.ts, p));
    else
        LLMRS_CUDA_TRY(launch(gemv_tma_kernel<WF, ST, false>, dim3(plan.grid), dim3(NTHREADS), plan.smem, stream, pdl,
                              plan.tw, plan.ts, p));
    return LLMRS_OK;
}

template <int WF, int ST, int PRO, int EPI>
int launch_one(const GemvPlan &plan, const GemvParams &p0, cudaStream_t stream, bool pdl)
{
    GemvParams p = p0;
    p.pro = PRO;
    p.epi = EPI;
    {
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
    bool known = false; // a variant the library instantiates (the fast kernel takes any of them at run time)
#define LLMRS_GEMV_KNOWN(WF, ST, PRO, EPI)                                                                  \
    if (pro == PRO && epi == EPI)                                                                          \
        known = true;
    LLMRS_GEMV_VARIANTS(LLMRS_GEMV_KNOWN)
#undef LLMRS_GEMV_KNOWN
    if (plan.fast && known) {
        if (wf == 0 && st == 0)
            return launch_fast<0, 0>(plan, p, pro, epi, stream, pdl);
        if (wf == 0 && st == 1)
            return launch_fast<0, 1>(plan, p, pro, epi, stream, pdl);
        if (wf == 1 && st == 0)
            return launch_fast<1, 0>(plan, p, pro, epi, stream, pdl);
        if (wf == 1 && st == 1)
            return launch_fast<1, 1>(plan, p, pro, epi, stream, pdl);
    }
#define LLMRS_GEMV_CASE(WF, ST, PRO, EPI)                                                                   \
    if (wf == WF && st == ST && pro == PRO && epi == EPI)                                                  \
        return launch_one<WF, ST, PRO, EPI>(plan, p, stream, pdl);
    LLMRS_GEMV_VARIANTS(LLMRS_GEMV_CASE)
#undef LLMRS_GEMV_CASE
    return fail(LLMRS_ENOTSUP, "gemv: unsupported variant wf=%d st=%d pro=%d epi=%d", wf, st, pro, epi);
}

int gemv_norm_quantize(const float *x, const float *w, int K, float eps, int8_t *q, float *s, uint32_t *err,
                       cudaStream_t stream)
{
    LLMRS_CHECK_ARG(x && w && q && s, "NULL argument");
    LLMRS_CHECK_ARG(K > 0 && K % 32 == 0, "rms_norm_quantize: k=%d must be a positive multiple of 32", K);
    LLMRS_CHECK_ARG(!((uintptr_t)x & 15) && !((uintptr_t)w & 15) && !((uintptr_t)q & 15),
                    "rms_norm_quantize: x, w and q must be 16-byte aligned");
    const size_t smem = (size_t)(K / 32) * 40 + 64;
    LLMRS_CHECK_ARG(smem <= 48 * 1024, "rms_norm_quantize: k=%d too large", K);
    GemvParams p{};
    p.K = K;
    p.x = x;
    p.norm_w = w;
    p.eps = eps;
    p.err = err;
    norm_quant_kernel<<<1, PRO_THREADS, smem, stream>>>(p, q, s);
    LLMRS_CUDA_TRY(cudaGetLastError());
    return LLMRS_OK;
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
    cudaError_t e = prepare_fast<0, 0>();
    if (e == cudaSuccess)
        e = prepare_fast<0, 1>();
    if (e == cudaSuccess)
        e = prepare_fast<1, 0>();
    if (e == cudaSuccess)
        e = prepare_fast<1, 1>();
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
