// Prefill GEMM on the 5th-generation tensor cores: C[T, N] = A[T, K] W[N, K]^T,
// FP16 operands, FP32 accumulation in tensor memory, FP16 output with the
// reference's epilogue roundings (bias, residual add, SwiGLU), replacing the
// prompt-wide torch::matmul calls of the reference's prefill
// (src/models/ModelBase.cpp:763, 772, 781, 838, 744-750).
//
// One CTA computes a 128 x 256 output tile:
//   warp 0      TMA producer: A box [128 x 64] and W box [256 x 64] per stage
//               (128-byte swizzle, no multicast), 4 stages, mbarrier ring
//   warp 1      allocates 256 TMEM columns; one thread issues tcgen05.mma
//               (M=128, N=256, K=16, kind::f16, both operands K-major) and
//               tcgen05.commit frees each stage and finally signals the epilogue
//   warps 2-9   epilogue: tcgen05.ld of their 32-lane quadrant (two warps per
//               quadrant, each half of the 256 columns), 32 columns at a
//               time, epilogue op, FP16 stores
// Every wait is bounded; on expiry the kernel records an error, drains its own
// copies and MMAs, releases TMEM and returns.
#include "ylm_common.cuh"
#include "ylm_kernels.h"
#include <cudaTypedefs.h>

namespace ylm {

constexpr int TC_BM = 128, TC_BN = 256, TC_BK = 64, TC_ST = 4;
constexpr int TC_THREADS = 320; // producer, MMA issuer, 8 epilogue warps
constexpr int TC_EPI_COLS = TC_BN / 2; // columns per epilogue warp
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2; // 16 KB
constexpr int TC_B_BYTES = TC_BN * TC_BK * 2; // 32 KB
constexpr int TC_TMEM_COLS = 512; // two accumulators of TC_BN columns
constexpr size_t TC_SMEM = 1024 + (size_t)TC_ST * (TC_A_BYTES + TC_B_BYTES) + 256;

struct TcArgs
{
    int T, N, K, epi;
    const __half *bias;
    __half *C;
    int ldc;
    int *err;
};

// K-major operand tile in shared memory with the 128-byte swizzle: rows of 64
// FP16 (128 B), 8-row atoms of 1024 B (stride byte offset), SM100 descriptor
// version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc_k128(uint32_t saddr)
{
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: D FP32, A/B FP16, both K-major, N>>3, M>>4.
__host__ __device__ constexpr uint32_t tc_idesc(int m, int n)
{
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
                 "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
                 : "memory");
}

// The same with A read from tensor memory (lane = row of A, its K elements
// packed two FP16 per 32-bit column).
__device__ __forceinline__ void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
                 "r"(tmem_a), "l"(b), "r"(idesc), "r"(accumulate)
                 : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v)
{
    uint32_t r[32];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                   "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                   "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++)
        v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v)
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
                 "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
                 "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
                 "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
                 "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
                 "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
                 "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
                 "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
                 "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
                 "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
                 "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
                 "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
                 "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
                 : "memory");
}

// One output tile's epilogue for this thread: TMEM lane quadrant q, columns
// [cbeg, cbeg + TC_EPI_COLS) of the accumulator at TMEM address tacc.
__device__ __forceinline__ void tc_epilogue_tile(const TcArgs &p, uint32_t tacc, int m0, int n0, int q, int cbeg,
                                                 int lane)
{
    const int row = m0 + q * 32 + lane;
    for (int c0 = cbeg; c0 < cbeg + TC_EPI_COLS; c0 += 32)
    {
        float v[32];
        tmem_ld32(tacc + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
        const int col0 = n0 + c0;
        if (row >= p.T || col0 >= p.N)
            continue;
        __half *crow = p.C + (int64_t)row * p.ldc;
        // this thread's 32 columns are 64 contiguous bytes of its row:
        // 16-byte accesses where the row start keeps them aligned
        // (a warp's lanes are 32 different rows, so 2-byte accesses
        // would cost one memory transaction per element)
        const bool vec = col0 + 32 <= p.N && (p.ldc % 8) == 0;
        if (p.epi == GEMM_SWIGLU)
        {
            __half *dst = crow + (col0 >> 1);
            if (vec && (reinterpret_cast<uintptr_t>(dst) & 15) == 0)
            {
                uint4 pk[2];
                __half *hh = reinterpret_cast<__half *>(pk);
#pragma unroll
                for (int j = 0; j < 16; j++)
                {
                    const float g = rh(v[2 * j]), u = rh(v[2 * j + 1]);
                    const float sg = rh(g / (1.0f + expf(-g)));
                    hh[j] = f2h(sg * u);
                }
                reinterpret_cast<uint4 *>(dst)[0] = pk[0];
                reinterpret_cast<uint4 *>(dst)[1] = pk[1];
            }
            else
            {
#pragma unroll
                for (int j = 0; j < 32; j += 2)
                {
                    const int col = col0 + j;
                    if (col < p.N)
                    {
                        const float g = rh(v[j]), u = rh(v[j + 1]);
                        const float sg = rh(g / (1.0f + expf(-g)));
                        crow[col >> 1] = f2h(sg * u);
                    }
                }
            }
        }
        else if (p.epi == GEMM_RESID)
        {
            if (vec && (reinterpret_cast<uintptr_t>(crow + col0) & 15) == 0)
            {
                uint4 *rp = reinterpret_cast<uint4 *>(crow + col0);
                uint4 r[4];
#pragma unroll
                for (int j = 0; j < 4; j++)
                    r[j] = rp[j];
                __half *rr = reinterpret_cast<__half *>(r);
#pragma unroll
                for (int j = 0; j < 32; j++)
                    rr[j] = f2h(h2f(rr[j]) + rh(v[j]));
#pragma unroll
                for (int j = 0; j < 4; j++)
                    rp[j] = r[j];
            }
            else
            {
#pragma unroll
                for (int j = 0; j < 32; j++)
                    if (col0 + j < p.N)
                        crow[col0 + j] = f2h(h2f(crow[col0 + j]) + rh(v[j]));
            }
        }
        else
        {
            if (vec && (reinterpret_cast<uintptr_t>(crow + col0) & 15) == 0 &&
                (!p.bias || (reinterpret_cast<uintptr_t>(p.bias + col0) & 15) == 0))
            {
                uint4 pk[4];
                __half *hh = reinterpret_cast<__half *>(pk);
                if (p.bias)
                {
                    uint4 bq[4];
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        bq[j] = reinterpret_cast<const uint4 *>(p.bias + col0)[j];
                    const __half *bb = reinterpret_cast<const __half *>(bq);
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        hh[j] = f2h(rh(v[j]) + h2f(bb[j]));
                }
                else
                {
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        hh[j] = f2h(v[j]);
                }
                uint4 *dst = reinterpret_cast<uint4 *>(crow + col0);
#pragma unroll
                for (int j = 0; j < 4; j++)
                    dst[j] = pk[j];
            }
            else
            {
#pragma unroll
                for (int j = 0; j < 32; j++)
                    if (col0 + j < p.N)
                    {
                        float y = v[j];
                        if (p.bias)
                            y = rh(y) + h2f(p.bias[col0 + j]);
                        crow[col0 + j] = f2h(y);
                    }
            }
        }
    }
}

// Persistent: one CTA per SM walks the output tiles blockIdx.x, + gridDim.x,
// ... (M-fastest order: the CTAs of a wave that share a W tile run together,
// so each W tile comes from HBM once and A stays in L2). The producer's ring
// of operand stages runs on across tiles; the accumulator is double-buffered in
// TMEM (2 x 256 columns), so the epilogue warps drain tile i while the MMA
// warp accumulates tile i + 1.
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap wmap, const TcArgs p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sa = smem;
    uint8_t *sb = smem + (size_t)TC_ST * TC_A_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(sb + (size_t)TC_ST * TC_B_BYTES);
    uint64_t *empty = full + TC_ST;
    uint64_t *acc_full = empty + TC_ST; // [2] MMA -> epilogue
    uint64_t *acc_empty = acc_full + 2; // [2] epilogue (8 warps) -> MMA
    uint64_t *done = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = (p.T + TC_BM - 1) / TC_BM;
    const int tiles = mt * ((p.N + TC_BN - 1) / TC_BN);
    const int KT = (p.K + TC_BK - 1) / TC_BK;

    if (threadIdx.x == 0)
    {
        for (int s = 0; s < TC_ST; s++)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++)
        {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], TC_THREADS / 32 - 2);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0)
    {
        if (lane == 0)
        {
            prefetch_tensormap(&amap);
            prefetch_tensormap(&wmap);
            int g = 0; // k-stages issued by this CTA, over all its tiles
            for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x)
            {
                const int n0 = (t / mt) * TC_BN, m0 = (t % mt) * TC_BM;
                for (int kt = 0; kt < KT; kt++, g++)
                {
                    const int s = g % TC_ST;
                    if (g >= TC_ST &&
                        !mbar_wait_bounded(&empty[s], ((g / TC_ST) - 1) & 1, p.err, YLM_DEV_ERR_TIMEOUT_EMPTY))
                    {
                        *abort_flag = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], TC_A_BYTES + TC_B_BYTES);
                    tma_load_2d(sa + (size_t)s * TC_A_BYTES, &amap, kt * TC_BK, m0, &full[s]);
                    tma_load_2d(sb + (size_t)s * TC_B_BYTES, &wmap, kt * TC_BK, n0, &full[s]);
                }
            }
            // every issued copy has landed before the CTA can exit
            for (int h = g > TC_ST ? g - TC_ST : 0; h < g; h++)
                mbar_wait_bounded(&full[h % TC_ST], (h / TC_ST) & 1, p.err, YLM_DEV_ERR_TIMEOUT_DRAIN);
        }
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            const uint32_t idesc = tc_idesc(TC_BM, TC_BN);
            int g = 0;
            bool ok = true;
            int i = 0; // this CTA's tile count
            for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, i++)
            {
                const int b = i & 1;
                const uint32_t tacc = tmem + (uint32_t)(b * TC_BN);
                // the epilogue has drained this accumulator's previous tile
                if (i >= 2 && !mbar_wait_bounded(&acc_empty[b], ((i >> 1) - 1) & 1, p.err, YLM_DEV_ERR_TIMEOUT_EMPTY))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kt = 0; kt < KT; kt++, g++)
                {
                    const int s = g % TC_ST;
                    if (!mbar_wait_bounded(&full[s], (g / TC_ST) & 1, p.err, YLM_DEV_ERR_TIMEOUT_FULL))
                    {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sa + (size_t)s * TC_A_BYTES);
                    const uint32_t b0 = smem_u32(sb + (size_t)s * TC_B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 16; kk++)
                        tc_mma(tacc, smem_desc_k128(a0 + kk * 32), smem_desc_k128(b0 + kk * 32), idesc,
                               (kt | kk) != 0 ? 1u : 0u);
                    tc_commit(&empty[s]); // stage free once these MMAs have read it
                }
                if (ok)
                    tc_commit(&acc_full[b]); // this tile's MMAs complete -> epilogue
            }
            if (!ok)
                *abort_flag = 1;
            // all issued MMAs complete before TMEM is released
            tc_commit(done);
            mbar_wait_bounded(done, 0, p.err, YLM_DEV_ERR_TIMEOUT_DRAIN);
        }
        __syncwarp();
    }
    else
    {
        // epilogue warps 2..9 -> TMEM lane quadrant (warp % 4); warps 2-5 take
        // columns [0, 128), warps 6-9 columns [128, 256) of each tile
        const int q = warp & 3;
        const int cbeg = ((warp - 2) >> 2) * TC_EPI_COLS;
        int i = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, i++)
        {
            const int b = i & 1;
            // (a warp-wide vote: the TMEM loads below are warp-collective)
            const bool ok = mbar_wait_bounded(&acc_full[b], (i >> 1) & 1, p.err, YLM_DEV_ERR_TIMEOUT_FULL) &&
                            !*abort_flag;
            if (!__all_sync(0xffffffffu, ok))
            {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            tc_epilogue_tile(p, tmem + (uint32_t)(b * TC_BN), (t % mt) * TC_BM, (t / mt) * TC_BN, q, cbeg, lane);
            // this warp's reads of the accumulator are done: it may be reused
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&acc_empty[b]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1)
    {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS) : "memory");
    }
}

// ------------------------------------------------------------------ prefill attention (tcgen05)
// Causal flash attention of a prompt on the 5th-generation tensor cores: the
// prefill SDPA of ModelBase.cpp:671-693 with the causal mask of :620-636
// (implicit) and no ExpandKV (:695-707): query head h reads KV head h / G from
// the cache. One CTA per 128 query rows of one head, 10 warps:
//   warp 0      TMA: the Q tile once, then K tiles of 128 keys (three
//               stages, two tiles ahead) and V tiles (two stages) from 3-D
//               tensor maps whose key extent is the prompt length, so keys
//               past it arrive as zeros
//   warp 1      one thread issues S = Q K^T (M=128, N=128, K=128, both K-major)
//               into TMEM columns [0, 128), then O += P V into [128, 256)
//               (P from TMEM, V MN-major: the tile as stored)
//   warps 2-9   one query row per two threads (their TMEM lane; 64 of the
//               row's columns each, maxima and sums exchanged through shared
//               memory): scale, causal mask,
//               running max, P = exp2(s - m) rounded to FP16 and packed into
//               the tile's TMEM score buffer; O accumulates in TMEM across
//               tiles and is rescaled in place (tcgen05.ld / st) before the
//               next P V when a row's maximum rose by more than 2^8
// All waits are bounded; a timeout records YLM_DEV_ERR_TIMEOUT_* and unwinds.
constexpr int FT_BM = 128, FT_BN = 128, FT_THREADS = 320; // TMA, MMA, 8 softmax warps
constexpr int FT_TILE = 128 * 128 * 2; // one 128 x 128 FP16 tile: two 64-column atoms of 16 KB
constexpr int FT_TMEM_COLS = 512; // S for two key tiles (double-buffered), then O
constexpr int FT_KST = 3, FT_VST = 2;  // K and V stages
constexpr size_t FT_SMEM = 1024 + (size_t)FT_TILE * (1 + FT_KST + FT_VST) + 256 + 2 * 2 * 128 * 4; // Q, K, V, barriers, row exchange

// MN-major operand tile with the 128-byte swizzle: 64-element rows along MN,
// `lbo` bytes between 64-element MN blocks, `sbo` bytes between 8-row K groups.
__device__ __forceinline__ uint64_t smem_desc_mn128(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int32_t x, int32_t y, int32_t z,
                                            uint64_t *bar)
{
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
                     smem_u32(dst)),
                 "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
                 : "memory");
}

struct FtArgs
{
    int T, hq, hkv;
    __half *out; // [T][hq * 128]
    int *err;
};

// 2^x with the PTX ex2.approx instruction, subnormal results flushed to zero:
// the softmax's arguments are <= 0, and values below 2^-126 vanish in FP16 P.
__device__ __forceinline__ float ex2_ftz(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__global__ void __launch_bounds__(FT_THREADS, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap, const FtArgs p)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sq = smem;
    uint8_t *sk = sq + FT_TILE;           // FT_KST stages
    uint8_t *sv = sk + FT_KST * FT_TILE;  // FT_VST stages
    uint64_t *bars = reinterpret_cast<uint64_t *>(sv + FT_VST * FT_TILE);
    // K and V have rings of their own: a K stage is free once its S = Q K^T
    // completes, a V stage once its P V does, so the next tiles' keys load
    // while the current P V waits for its softmax
    uint64_t *q_full = bars, *k_full = bars + 1, *k_empty = k_full + FT_KST, *v_full = k_empty + FT_KST,
             *v_empty = v_full + FT_VST, *s_full = v_empty + FT_VST, *p_full = s_full + 2, *o_full = p_full + 1,
             *done = o_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(done + 2);
    uint64_t *xbar = done + 3; // row exchange between the two softmax halves (256 arrivals)
    float *xrow = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(bars) + 256); // maxima [2 halves][128 rows]
    float *xsum = xrow + 256;                                                          // sums [2][128]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // heaviest query tiles first: linear block i (the order blocks start in)
    // takes tile nq - 1 - i / hq of head i % hq, so the causal tiles with the
    // most key tiles fill the first waves and the short ones the last
    const int lin = blockIdx.y * gridDim.x + blockIdx.x;
    const int qb = (int)gridDim.x - 1 - lin / p.hq, h = lin % p.hq, g = h / (p.hq / p.hkv);
    const int r0 = qb * FT_BM;
    const int nt = qb + 1; // key tiles 0 .. the diagonal one

    if (threadIdx.x == 0)
    {
        mbar_init(q_full, 1);
        for (int s = 0; s < FT_KST; s++)
        {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < FT_VST; s++)
        {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        mbar_init(p_full, 256);
        mbar_init(xbar, 256);
        mbar_init(o_full, 1);
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(FT_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0)
    {
        if (lane == 0)
        {
            prefetch_tensormap(&qmap);
            prefetch_tensormap(&kmap);
            prefetch_tensormap(&vmap);
            mbar_arrive_expect_tx(q_full, FT_TILE);
            tma_load_2d(sq, &qmap, h * 128, r0, q_full);
            tma_load_2d(sq + FT_TILE / 2, &qmap, h * 128 + 64, r0, q_full);
            // K tile j into stage j % FT_KST once S of tile j - FT_KST is done;
            // V tile j into stage j % FT_VST once P V of tile j - FT_VST is
            // done; the keys run FT_KST - 1 tiles ahead of the values
            int kissued = 0, vissued = 0;
            auto load_k = [&](int j) {
                const int s = j % FT_KST;
                if (j >= FT_KST &&
                    !mbar_wait_bounded(&k_empty[s], (j / FT_KST - 1) & 1, p.err, YLM_DEV_ERR_TIMEOUT_EMPTY))
                    return false;
                mbar_arrive_expect_tx(&k_full[s], FT_TILE);
                tma_load_3d(sk + s * FT_TILE, &kmap, 0, j * FT_BN, g, &k_full[s]);
                tma_load_3d(sk + s * FT_TILE + FT_TILE / 2, &kmap, 64, j * FT_BN, g, &k_full[s]);
                kissued++;
                return true;
            };
            auto load_v = [&](int j) {
                const int s = j % FT_VST;
                if (j >= FT_VST &&
                    !mbar_wait_bounded(&v_empty[s], (j / FT_VST - 1) & 1, p.err, YLM_DEV_ERR_TIMEOUT_EMPTY))
                    return false;
                mbar_arrive_expect_tx(&v_full[s], FT_TILE);
                tma_load_3d(sv + s * FT_TILE, &vmap, 0, j * FT_BN, g, &v_full[s]);
                tma_load_3d(sv + s * FT_TILE + FT_TILE / 2, &vmap, 64, j * FT_BN, g, &v_full[s]);
                vissued++;
                return true;
            };
            constexpr int AHEAD = FT_KST - 1;
            for (int j = 0; j < nt + AHEAD; j++)
            {
                if (*abort_flag)
                    break;
                if ((j < nt && !load_k(j)) || (j >= AHEAD && !load_v(j - AHEAD)))
                {
                    *abort_flag = 1;
                    break;
                }
            }
            // every issued copy has landed before the CTA can exit
            mbar_wait_bounded(q_full, 0, p.err, YLM_DEV_ERR_TIMEOUT_DRAIN);
            for (int j = kissued > FT_KST ? kissued - FT_KST : 0; j < kissued; j++)
                mbar_wait_bounded(&k_full[j % FT_KST], (j / FT_KST) & 1, p.err, YLM_DEV_ERR_TIMEOUT_DRAIN);
            for (int j = vissued > FT_VST ? vissued - FT_VST : 0; j < vissued; j++)
                mbar_wait_bounded(&v_full[j % FT_VST], (j / FT_VST) & 1, p.err, YLM_DEV_ERR_TIMEOUT_DRAIN);
        }
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            const uint32_t idesc_s = tc_idesc(FT_BM, FT_BN);
            const uint32_t idesc_o = tc_idesc(FT_BM, 128) | (1u << 16); // B (V) MN-major
            bool ok = mbar_wait_bounded(q_full, 0, p.err, YLM_DEV_ERR_TIMEOUT_FULL);
            const uint32_t q0 = smem_u32(sq);
            // S_j = Q K_j^T into TMEM columns [128 (j & 1), +128)
            auto issue_s = [&](int j) {
                const int s = j & 1, ks = j % FT_KST;
                if (!mbar_wait_bounded(&k_full[ks], (j / FT_KST) & 1, p.err, YLM_DEV_ERR_TIMEOUT_FULL))
                    return false;
                tc_fence_after();
                const uint32_t k0 = smem_u32(sk + ks * FT_TILE);
#pragma unroll
                for (int kk = 0; kk < 8; kk++)
                {
                    const uint32_t off = (uint32_t)((kk >> 2) * (FT_TILE / 2) + (kk & 3) * 32);
                    tc_mma(tmem + 128u * s, smem_desc_k128(q0 + off), smem_desc_k128(k0 + off), idesc_s, kk ? 1u : 0u);
                }
                tc_commit(&s_full[s]);
                tc_commit(&k_empty[ks]);
                return true;
            };
            ok = ok && issue_s(0);
            for (int j = 0; ok && j < nt; j++)
            {
                const int s = j & 1;
                // the next tile's scores run on the tensor cores while the
                // softmax warps work on this one (its S buffer was freed when
                // tile j - 1's P arrived)
                if (j + 1 < nt && !issue_s(j + 1))
                {
                    ok = false;
                    break;
                }
                const int vs = j % FT_VST;
                if (!mbar_wait_bounded(p_full, j & 1, p.err, YLM_DEV_ERR_TIMEOUT_FULL) ||
                    !mbar_wait_bounded(&v_full[vs], (j / FT_VST) & 1, p.err, YLM_DEV_ERR_TIMEOUT_FULL))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t v0 = smem_u32(sv + vs * FT_TILE);
                // O += P V with P (FP16, packed by the softmax warps over the
                // first 64 columns of this tile's S buffer) as A from TMEM:
                // keys 16 kk .. 16 kk + 15 are columns 8 kk .. 8 kk + 7
#pragma unroll
                for (int kk = 0; kk < 8; kk++)
                    tc_mma_ts(tmem + 256, tmem + 128u * (uint32_t)s + 8u * (uint32_t)kk,
                              smem_desc_mn128(v0 + kk * 2048, FT_TILE / 2, 1024), idesc_o, (j | kk) ? 1u : 0u);
                tc_commit(o_full);
                tc_commit(&v_empty[vs]);
            }
            if (!ok)
                *abort_flag = 1;
            // all issued MMAs complete before TMEM is released
            tc_commit(done);
            mbar_wait_bounded(done, 0, p.err, YLM_DEV_ERR_TIMEOUT_DRAIN);
        }
        __syncwarp();
    }
    else
    {
        const int q = warp & 3;           // TMEM lane quadrant of this warp
        const int hf = (warp - 2) >> 2;   // which 64 of the row's 128 keys / dims (warps 2-5: 0, 6-9: 1)
        const int row = q * 32 + lane;    // query row in the tile
        const int grow = r0 + row;
        const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
        const int cb = hf * 64;           // this thread's columns [cb, cb + 64)
        const float sl2 = 0.08838834764831845f * 1.4426950408889634f; // 1/sqrt(128) * log2(e)
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nt; j++)
        {
            // (every wait ends in a warp-wide vote: the TMEM accesses below are
            // warp-collective, so the lanes leave together or not at all)
            const bool sw = mbar_wait_bounded(&s_full[j & 1], (j >> 1) & 1, p.err, YLM_DEV_ERR_TIMEOUT_FULL) &&
                            !*abort_flag;
            const uint32_t tS = trow + 128u * (uint32_t)(j & 1); // this tile's scores
            if (!__all_sync(0xffffffffu, sw))
            {
                ok = false;
                break;
            }
            tc_fence_after();
            const int key0 = j * FT_BN;
            // only the diagonal tile holds keys past some of its rows
            const bool diag = j == nt - 1;
            // this thread's 64 scores, read from TMEM once, scaled to base 2;
            // pass 1: the row maximum of this tile (masked keys excluded)
            float v[64];
            tmem_ld32(tS + (uint32_t)cb, v);
            tmem_ld32(tS + (uint32_t)cb + 32u, v + 32);
            float mx = -INFINITY;
            if (diag)
            {
#pragma unroll
                for (int i = 0; i < 64; i++)
                {
                    v[i] = key0 + cb + i <= grow ? v[i] * sl2 : -INFINITY;
                    mx = fmaxf(mx, v[i]);
                }
            }
            else
            {
#pragma unroll
                for (int i = 0; i < 64; i++)
                {
                    v[i] *= sl2;
                    mx = fmaxf(mx, v[i]);
                }
            }
            // the row's other half, through shared memory (a thread writes the
            // next tile's value only after both halves arrived on p_full for
            // this one, so the partner has read it); phase j of xbar
            xrow[hf * 128 + row] = mx;
            mbar_arrive(xbar);
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(xbar, j & 1, p.err, YLM_DEV_ERR_TIMEOUT_FULL)))
            {
                ok = false;
                break;
            }
            mx = fmaxf(mx, xrow[(hf ^ 1) * 128 + row]);
            // each tile holds key j*128 <= every row of this block: mx is finite.
            // The exponent base m moves only when the row maximum rises by more
            // than 8 (base 2): P = exp2(s - m) <= 2^8 stays exact in FP16 range,
            // O and l carry the same factor, and O is rescaled (waiting for the
            // previous P V) only on such a rise, not on every new maximum.
            float corr = 1.f;
            if (j == 0)
                m = mx;
            else if (__any_sync(0xffffffffu, mx > m + 8.f))
            {
                if (!__all_sync(0xffffffffu, mbar_wait_bounded(o_full, (j - 1) & 1, p.err, YLM_DEV_ERR_TIMEOUT_FULL)))
                {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (mx > m + 8.f)
                {
                    corr = exp2f(m - mx);
                    m = mx;
                }
#pragma unroll
                for (int c0 = cb; c0 < cb + 64; c0 += 32)
                {
                    float v[32];
                    tmem_ld32(trow + 256u + (uint32_t)c0, v);
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        v[i] *= corr;
                    tmem_st32(trow + 256u + (uint32_t)c0, v);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            }
            const float mn = m;
            // pass 2: P = exp2(s - m) in FP16, packed two per column into this
            // tile's S buffer, columns [32 hf, 32 hf + 32) (this thread's keys;
            // both halves have read their scores by now: xbar)
            // (masked keys hold -inf: exp2 gives 0)
            float sum = 0.f;
            uint32_t pk[32];
#pragma unroll
            for (int i = 0; i < 64; i += 2)
            {
                const float p0 = ex2_ftz(v[i] - mn);
                const float p1 = ex2_ftz(v[i + 1] - mn);
                sum += p0 + p1;
                const __half2 hp = __floats2half2_rn(p0, p1);
                pk[i >> 1] = *reinterpret_cast<const uint32_t *>(&hp);
            }
            tmem_st32(tS + 32u * (uint32_t)hf, reinterpret_cast<const float *>(pk));
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            l = l * corr + sum;
            // P visible to the tensor cores
            tc_fence_before();
            mbar_arrive(p_full);
        }
        // the row sum over both halves: phase nt of xbar
        bool fw = ok;
        if (fw)
        {
            xsum[hf * 128 + row] = l;
            mbar_arrive(xbar);
            fw = mbar_wait_bounded(xbar, nt & 1, p.err, YLM_DEV_ERR_TIMEOUT_FULL);
            l += xsum[(hf ^ 1) * 128 + row];
        }
        // every MMA of the CTA has completed (`done`, committed once after the
        // last P V: its single phase cannot alias, while o_full may be one or
        // two phases behind this warp's last wait on it)
        fw = fw && mbar_wait_bounded(done, 0, p.err, YLM_DEV_ERR_TIMEOUT_FULL) && !*abort_flag;
        if (__all_sync(0xffffffffu, fw))
        {
            tc_fence_after();
            const float inv = 1.f / l;
            __half *dst = p.out + (int64_t)grow * p.hq * 128 + h * 128;
#pragma unroll
            for (int c0 = cb; c0 < cb + 64; c0 += 32)
            {
                float v[32];
                tmem_ld32(trow + 256u + (uint32_t)c0, v);
                if (grow < p.T)
                {
#pragma unroll
                    for (int c8 = 0; c8 < 32; c8 += 8)
                    {
                        uint4 pk;
                        __half2 *hh = reinterpret_cast<__half2 *>(&pk);
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            hh[i] = __floats2half2_rn(v[c8 + 2 * i] * inv, v[c8 + 2 * i + 1] * inv);
                        *reinterpret_cast<uint4 *>(dst + c0 + c8) = pk;
                    }
                }
            }
        }
        else
            *abort_flag = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1)
    {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(FT_TMEM_COLS) : "memory");
    }
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 encoder()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn)
    {
        cudaDriverEntryPointQueryResult q;
        void *f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    return fn;
}

// K-major FP16 operand [rows, K] with row stride ld (elements), box [box_rows x 64], 128-byte swizzle.
bool tc_make_operand_map(CUtensorMap *map, const __half *p, int rows, int K, int ld, int box_rows)
{
    auto enc = encoder();
    if (!enc || (ld % 8) || (reinterpret_cast<uintptr_t>(p) % 16) || rows <= 0 || K <= 0)
        return false;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(p), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tc_make_a_map(CUtensorMap *map, const __half *A, int T, int K, int lda)
{
    return tc_make_operand_map(map, A, T, K, lda, TC_BM);
}

bool tc_make_w_map(CUtensorMap *map, const __half *W, int N, int K)
{
    return tc_make_operand_map(map, W, N, K, K, TC_BN);
}

cudaError_t gemm_tc_prepare()
{
    return cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM);
}

cudaError_t gemm_tc_launch(const CUtensorMap &amap, const CUtensorMap &wmap, int T, int N, int K, int epi,
                           const __half *bias, __half *C, int ldc, int *err, cudaStream_t s)
{
    if (T <= 0)
        return cudaSuccess;
    TcArgs a;
    a.T = T;
    a.N = N;
    a.K = K;
    a.epi = epi;
    a.bias = bias;
    a.C = C;
    a.ldc = ldc;
    a.err = err;
    // persistent: at most one CTA per SM, each walking its share of the tiles
    static int sms = 0;
    if (!sms)
    {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0)
            sms = 148;
    }
    const int tiles = ((N + TC_BN - 1) / TC_BN) * ((T + TC_BM - 1) / TC_BM);
    dim3 grid((unsigned)std::min(tiles, sms));
    gemm_tc_kernel<<<grid, TC_THREADS, TC_SMEM, s>>>(amap, wmap, a);
    return cudaGetLastError();
}


// Tensor maps of the prefill attention: Q [T][hq*128] in 64 x 128 boxes; K and
// V of one layer as [hkv][T of cap][128] in 64 x 128 x 1 boxes (the key extent
// is T, so rows past the prompt are filled with zeros).
static bool ft_make_maps(CUtensorMap *qm, CUtensorMap *km, CUtensorMap *vm, const __half *q, const __half *k,
                         const __half *v, int cap, int hq, int hkv, int T)
{
    auto enc = encoder();
    if (!enc || (reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) % 16)
        return false;
    {
        cuuint64_t dims[2] = {(cuuint64_t)hq * 128, (cuuint64_t)T};
        cuuint64_t strides[1] = {(cuuint64_t)hq * 128 * 2};
        cuuint32_t box[2] = {64, 128};
        cuuint32_t estr[2] = {1, 1};
        if (enc(qm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(q), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    cuuint64_t dims[3] = {128, (cuuint64_t)T, (cuuint64_t)hkv};
    cuuint64_t strides[2] = {256, (cuuint64_t)cap * 256};
    cuuint32_t box[3] = {64, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    for (int i = 0; i < 2; i++)
        if (enc(i ? vm : km, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half *>(i ? v : k), dims, strides, box,
                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    return true;
}

cudaError_t attn_prefill_tc_prepare()
{
    return cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FT_SMEM);
}

cudaError_t attn_prefill_tc_launch(const __half *q, const __half *k_cache, const __half *v_cache, int cap, int hq,
                                   int hkv, int T, __half *out, int *err, cudaStream_t s)
{
    if (T <= 0)
        return cudaSuccess;
    if (T > cap || hkv <= 0 || hq % hkv)
        return cudaErrorInvalidValue;
    CUtensorMap qm, km, vm;
    if (!ft_make_maps(&qm, &km, &vm, q, k_cache, v_cache, cap, hq, hkv, T))
        return cudaErrorNotSupported;
    FtArgs a;
    a.T = T;
    a.hq = hq;
    a.hkv = hkv;
    a.out = out;
    a.err = err;
    attn_prefill_tc_kernel<<<dim3((T + FT_BM - 1) / FT_BM, hq), FT_THREADS, FT_SMEM, s>>>(qm, km, vm, a);
    return cudaGetLastError();
}

} // namespace ylm
