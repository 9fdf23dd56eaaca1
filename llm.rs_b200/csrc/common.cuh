// common.cuh - shared device/host helpers for the llm.rs B200 backend.
//
// PTX wrappers for the Blackwell data-movement path (mbarrier, bulk TMA copies,
// programmatic dependent launch), bounded spin-waits that report a timeout
// through a device error word instead of hanging, and host-side status
// handling for the C ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <string>

#include "../../include/llmrs_cuda.h"

namespace llmrs {

// ---------------------------------------------------------------- host status
void set_error(const char *fmt, ...);
int fail(int code, const char *fmt, ...);

#define LLMRS_CUDA_TRY(expr)                                                                   \
    do {                                                                                       \
        cudaError_t _e = (expr);                                                               \
        if (_e != cudaSuccess)                                                                 \
            return ::llmrs::fail(LLMRS_ECUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), \
                                 __FILE__, __LINE__);                                          \
    } while (0)

#define LLMRS_CHECK_ARG(cond, ...)                                                             \
    do {                                                                                       \
        if (!(cond))                                                                           \
            return ::llmrs::fail(LLMRS_EINVAL, __VA_ARGS__);                                   \
    } while (0)

#define LLMRS_TRY(expr)                                                                        \
    do {                                                                                       \
        int _rc = (expr);                                                                      \
        if (_rc != LLMRS_OK)                                                                   \
            return _rc;                                                                        \
    } while (0)

int num_sms(int device);

// error word written by kernels whose bounded waits ran out (0 = none)
enum : uint32_t {
    DEV_ERR_NONE = 0,
    DEV_ERR_MBAR_TIMEOUT = 1,
    DEV_ERR_PEER_TIMEOUT = 2,
    DEV_ERR_BAD_TOKEN = 3,
    DEV_ERR_BAD_POS = 4,
};

// launch a kernel; with pdl=true it may begin before the previous kernel in the
// stream finishes (it must call griddep_wait() before reading that kernel's output)
template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          bool pdl, Args &&...args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ------------------------------------------------------------- device helpers
__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void griddep_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void griddep_launch_dependents()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// 3-D tensor-map TMA load of a box at (x, y, z) into shared memory
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar,
                                            uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// order this thread's earlier generic-proxy shared-memory accesses before its
// later async-proxy (bulk copy) accesses of the same bytes
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_n(uint64_t *bar, uint32_t n)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(n) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Wait until *c >= target (a counter other GPUs raise over NVLink); gives up
// after limit_ns, records DEV_ERR_PEER_TIMEOUT and returns false.
__device__ __forceinline__ bool wait_counter(const unsigned long long *c, unsigned long long target, uint32_t *err,
                                             uint64_t limit_ns = 5000000000ull)
{
    if (ld_acquire_sys(c) >= target)
        return true;
    if (err && *reinterpret_cast<volatile uint32_t *>(err) != 0)
        return false; // an earlier wait of this step already gave up: do not wait again
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        __nanosleep(64);
        if (ld_acquire_sys(c) >= target)
            return true;
        if (globaltimer_ns() - t0 > limit_ns) {
            if (err)
                atomicCAS(err, 0u, (uint32_t)DEV_ERR_PEER_TIMEOUT);
            return false;
        }
    }
}


// Wait for the given phase parity; gives up after ~limit_ns and records the
// timeout in *err.  Returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t *err,
                                          uint64_t limit_ns = 500000000ull)
{
    if (mbar_try_wait(bar, parity))
        return true;
    if (err) { // after one timeout in this launch, later waits give up at once
        const uint32_t e = *reinterpret_cast<volatile uint32_t *>(err);
        if (e == DEV_ERR_MBAR_TIMEOUT || e == DEV_ERR_PEER_TIMEOUT)
            return false;
    }
    uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity))
            return true;
        if ((it & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) {
            if (err)
                atomicCAS(err, 0u, (uint32_t)DEV_ERR_MBAR_TIMEOUT);
            return false;
        }
    }
}

// 1-D bulk copy global -> shared (TMA engine); completes on `bar` with complete_tx.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t policy_evict_last()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Timeline marks of a traced decode step (globaltimer ns), four per kernel:
// [4*slot] first CTA start, [4*slot+1] first CTA past griddepcontrol.wait,
// [4*slot+2] last CTA ready to consume its stream (activation prologue done),
// [4*slot+3] last CTA end.
constexpr int TRACE_MARKS = 4;

__device__ __forceinline__ void trace_start(unsigned long long *trace, int slot)
{
    if (trace)
        atomicMin(&trace[TRACE_MARKS * slot], (unsigned long long)globaltimer_ns());
}

__device__ __forceinline__ void trace_go(unsigned long long *trace, int slot)
{
    if (trace)
        atomicMin(&trace[TRACE_MARKS * slot + 1], (unsigned long long)globaltimer_ns());
}

__device__ __forceinline__ void trace_ready(unsigned long long *trace, int slot)
{
    if (trace)
        atomicMax(&trace[TRACE_MARKS * slot + 2], (unsigned long long)globaltimer_ns());
}

__device__ __forceinline__ void trace_end(unsigned long long *trace, int slot)
{
    if (trace)
        atomicMax(&trace[TRACE_MARKS * slot + 3], (unsigned long long)globaltimer_ns());
}

// order-preserving key for a float + lowest-index tie break (max of keys = argmax)
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx)
{
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}

__host__ __device__ __forceinline__ uint32_t argmax_key_index(unsigned long long key)
{
    return 0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull);
}

__host__ __device__ __forceinline__ float argmax_key_value(unsigned long long key)
{
    uint32_t b = (uint32_t)(key >> 32);
    b = (b & 0x80000000u) ? (b & 0x7FFFFFFFu) : ~b;
#ifdef __CUDA_ARCH__
    return __uint_as_float(b);
#else
    float f;
    memcpy(&f, &b, 4);
    return f;
#endif
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ int warp_sum_int(int v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// deterministic (fixed-tree) f32 warp sum
__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

} // namespace llmrs
