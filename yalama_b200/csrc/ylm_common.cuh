// Shared device helpers for the yalama B200 engine (sm_100a only).
//
// PTX wrappers for mbarriers, TMA (tiled and bulk, never with cluster
// multicast), programmatic dependent launch, and the rounding helpers that
// reproduce LibTorch's FP16 storage semantics: every elementwise op computes in
// FP32 and rounds to FP16 (the reference chains such ops, e.g.
// src/models/ModelBase.cpp:731-735, 797-815).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include "ylm_kernels.h"

// A bounded wait gives up after this many nanoseconds of %globaltimer.
#define YLM_WAIT_LIMIT_NS 2000000000ull

namespace ylm {

__device__ __forceinline__ float h2f(__half h) { return __half2float(h); }
__device__ __forceinline__ __half f2h(float f) { return __float2half_rn(f); }
// round an FP32 value to the nearest FP16 value, kept as FP32
__device__ __forceinline__ float rh(float f) { return __half2float(__float2half_rn(f)); }

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(smem_u32(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete, for at most YLM_WAIT_LIMIT_NS.
// On expiry record `code` in *err and return false; the caller unwinds.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *err, int code)
{
    if (mbar_try_wait(bar, parity))
        return true;
    uint64_t t0 = globaltimer_ns();
    for (;;)
    {
        for (int i = 0; i < 64; i++)
            if (mbar_try_wait(bar, parity))
                return true;
        if (globaltimer_ns() - t0 > YLM_WAIT_LIMIT_NS)
        {
            if (err)
                atomicExch(err, code);
            return false;
        }
    }
}

// ---------------------------------------------------------------- TMA
// 2D tiled load of box {x (inner), y} into shared memory, completing on `bar`.
// x * sizeof(elem) must be a multiple of 16 bytes (callers pass multiples of 256 halves).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int32_t x, int32_t y, uint64_t *bar)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
                     smem_u32(dst)),
                 "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
                 : "memory");
}

// Same, with an L2 eviction-priority hint (weights streamed once per token).
__device__ __forceinline__ void tma_load_2d_hint(void *dst, const CUtensorMap *map, int32_t x, int32_t y, uint64_t *bar,
                                                 uint64_t policy)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(
                     smem_u32(dst)),
                 "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
                 : "memory");
}

// 1D bulk copy global -> shared (both 16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---------------------------------------------------------------- PDL
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// named barrier over `n` threads (a multiple of 32)
__device__ __forceinline__ void named_bar_sync(int id, int n)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sampling keys: an FP16 value as a 16-bit unsigned integer with the same
// order (ord16), and a 64-bit key (ordered value, then the complement of the
// index) whose maximum is the largest value at its lowest index: argmax's
// choice among ties.
__device__ __forceinline__ uint32_t ord16(uint32_t h)
{
    return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
}
__device__ __forceinline__ uint32_t unord16(uint32_t o) { return (o & 0x8000u) ? (o & 0x7FFFu) : (~o & 0xFFFFu); }

__device__ __forceinline__ uint64_t make_key(uint32_t ord, uint32_t idx)
{
    return ((uint64_t)ord << 32) | (uint64_t)(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint32_t key_idx(uint64_t k) { return 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFu); }

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    return v;
}

// dot of 8 FP16 weights (one 16-byte vector) with 8 FP32 inputs
__device__ __forceinline__ float dot8(uint4 w, const float *x, float acc)
{
    const __half2 *h = reinterpret_cast<const __half2 *>(&w);
#pragma unroll
    for (int i = 0; i < 4; i++)
    {
        float2 f = __half22float2(h[i]);
        acc = fmaf(f.x, x[2 * i], acc);
        acc = fmaf(f.y, x[2 * i + 1], acc);
    }
    return acc;
}

__device__ __forceinline__ void unpack8(uint4 v, float *x)
{
    const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; i++)
    {
        float2 f = __half22float2(h[i]);
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}

} // namespace ylm
