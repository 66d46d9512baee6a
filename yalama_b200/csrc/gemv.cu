// Batch-1 FP16 GEMV for the decode projections (QKV, O, gate-up, down, lm_head).
//
// y = W x with W [N, K] row-major FP16, FP32 accumulation. Replaces the
// per-token torch::matmul calls of the reference (src/models/ModelBase.cpp:763,
// 772, 781 (QKV), 838 (o_proj), 744-750 (FFN), 451 (lm_head)) and fuses the
// elementwise work around them:
//   prologue  RMSNorm of the residual stream (ModelBase.cpp:724-736), or the
//             embedding gather + RMSNorm for layer 0 (ModelBase.cpp:841-851)
//   epilogue  bias (Qwen2_5Model.cpp:25-47), residual add (ModelBase.cpp:426,
//             437), SwiGLU (ModelBase.cpp:744-749)
// with the reference's FP16 rounding after every op.
//
// Decode is HBM-bound (about one FMA per weight byte), so this kernel keeps
// tensor cores idle and streams weights with TMA: one producer warp issues 2D
// tiled loads (box = rb rows x 256 columns, no multicast) into a ring of
// shared-memory stages guarded by mbarriers, eight consumer warps read 16 bytes
// per lane per row and reduce with warp shuffles. Each CTA owns whole row
// blocks, so every weight byte is read exactly once. The producer never waits
// on the previous kernel (weights are constant): under programmatic dependent
// launch the next projection's weights stream in while the current one
// finishes; only the consumers execute griddepcontrol.wait before reading x.
#include "ylm_common.cuh"
#include "ylm_kernels.h"
#include <cudaTypedefs.h>
#include <algorithm>

namespace ylm {

constexpr int GEMV_CWARPS = 8;
constexpr int GEMV_THREADS = (GEMV_CWARPS + 1) * 32;
constexpr int GEMV_KC = 256;
constexpr int GEMV_MAX_RB = 64;
constexpr int GEMV_MAXJ = GEMV_MAX_RB / GEMV_CWARPS;
constexpr size_t GEMV_SMEM_BUDGET = 112 * 1024;

struct GemvDev
{
    int N, K, rb, n_blocks, nst, k_pad, n_chunks;
    GemvArgs a;
};

template <int PAIR>
__device__ __forceinline__ int gemv_row_of(int j, int warp)
{
    return PAIR ? 2 * (warp + GEMV_CWARPS * (j >> 1)) + (j & 1) : warp + GEMV_CWARPS * j;
}

template <int PRO>
__device__ __forceinline__ void gemv_prologue(const GemvDev &p, __half *xs, float *red, int tid)
{
    const int K = p.K, kp = p.k_pad;
    const int warp = tid >> 5, lane = tid & 31;
    if (PRO == PRO_VEC)
    {
        for (int i = tid * 8; i < kp; i += 256 * 8)
        {
            uint4 v = make_uint4(0, 0, 0, 0);
            if (i < K)
                v = *reinterpret_cast<const uint4 *>(p.a.x + i);
            *reinterpret_cast<uint4 *>(xs + i) = v;
        }
        return;
    }
    const __half *src = p.a.x;
    if (PRO == PRO_EMBED_RMSNORM)
    {
        int64_t tok = p.a.state->token;
        if (tok < 0 || tok >= p.a.vocab)
        {
            if (tid == 0 && p.a.err)
                atomicExch(p.a.err, YLM_DEV_ERR_BAD_TOKEN);
            tok = 0;
        }
        src = p.a.emb + tok * (int64_t)K;
        if (blockIdx.x == 0)
            for (int i = tid * 8; i < K; i += 256 * 8)
                *reinterpret_cast<uint4 *>(p.a.resid_out + i) = *reinterpret_cast<const uint4 *>(src + i);
    }
    // mean(x*x): squares rounded to FP16, FP32 sum, times 1/K, rounded (ModelBase.cpp:731)
    float ss = 0.f;
    for (int i = tid * 8; i < K; i += 256 * 8)
    {
        float f[8];
        unpack8(*reinterpret_cast<const uint4 *>(src + i), f);
#pragma unroll
        for (int e = 0; e < 8; e++)
            ss += rh(f[e] * f[e]);
    }
    ss = warp_sum(ss);
    if (lane == 0)
        red[warp] = ss;
    named_bar_sync(1, 256);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < GEMV_CWARPS; w++)
        tot += red[w];
    const float mean = rh(tot * (1.0f / (float)K));
    const float d = rh(rsqrtf(mean + p.a.eps)); // ModelBase.cpp:732
    for (int i = tid * 8; i < kp; i += 256 * 8)
    {
        uint4 o = make_uint4(0, 0, 0, 0);
        if (i < K)
        {
            float f[8], w[8];
            unpack8(*reinterpret_cast<const uint4 *>(src + i), f);
            unpack8(*reinterpret_cast<const uint4 *>(p.a.norm_w + i), w);
            __half2 *oh = reinterpret_cast<__half2 *>(&o);
#pragma unroll
            for (int e = 0; e < 4; e++)
                oh[e] = __halves2half2(f2h(rh(f[2 * e] * d) * w[2 * e]), f2h(rh(f[2 * e + 1] * d) * w[2 * e + 1]));
        }
        *reinterpret_cast<uint4 *>(xs + i) = o;
    }
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(GEMV_THREADS, 1) gemv_kernel(const __grid_constant__ CUtensorMap wmap, const GemvDev p)
{
    constexpr int PAIR = (EPI == EPI_SWIGLU) ? 1 : 0;
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int stage_bytes = p.rb * (GEMV_KC * 2);
    __half *xs = reinterpret_cast<__half *>(smem + (size_t)p.nst * stage_bytes);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)p.nst * stage_bytes + (size_t)p.k_pad * 2);
    uint64_t *empty = full + p.nst;
    float *red = reinterpret_cast<float *>(empty + p.nst);

    pdl_launch_dependents();
    if (tid == 0)
    {
        for (int s = 0; s < p.nst; s++)
        {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], GEMV_CWARPS);
        }
        fence_mbar_init();
    }
    __syncthreads();

    const int my_blocks = (p.n_blocks - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    const int total = my_blocks * p.n_chunks;

    if (warp == GEMV_CWARPS)
    {
        // ---------------- producer: stream this CTA's row blocks, chunk by chunk
        if (lane == 0)
        {
            prefetch_tensormap(&wmap);
            const uint64_t pol = l2_policy_evict_first();
            int issued = 0;
            for (int it = 0; it < total; it++)
            {
                const int s = it % p.nst;
                if (it >= p.nst &&
                    !mbar_wait_bounded(&empty[s], ((it / p.nst) - 1) & 1, p.a.err, YLM_DEV_ERR_TIMEOUT_EMPTY))
                    break;
                const int bi = it / p.n_chunks, kc = it % p.n_chunks;
                const int b = (int)blockIdx.x + bi * (int)gridDim.x;
                mbar_arrive_expect_tx(&full[s], stage_bytes);
                tma_load_2d_hint(smem + (size_t)s * stage_bytes, &wmap, kc * GEMV_KC, b * p.rb, &full[s], pol);
                issued++;
            }
            // every issued copy has landed before the CTA may exit
            for (int it = issued > p.nst ? issued - p.nst : 0; it < issued; it++)
                mbar_wait_bounded(&full[it % p.nst], (it / p.nst) & 1, p.a.err, YLM_DEV_ERR_TIMEOUT_DRAIN);
        }
        return;
    }

    // ---------------- consumers
    pdl_wait();
    gemv_prologue<PRO>(p, xs, red, tid);
    named_bar_sync(1, 256);

    int it = 0;
    bool ok = true;
    for (int bi = 0; bi < my_blocks && ok; bi++)
    {
        const int b = (int)blockIdx.x + bi * (int)gridDim.x;
        float acc[GEMV_MAXJ];
#pragma unroll
        for (int j = 0; j < GEMV_MAXJ; j++)
            acc[j] = 0.f;
        for (int kc = 0; kc < p.n_chunks; kc++, it++)
        {
            const int s = it % p.nst;
            if (!mbar_wait_bounded(&full[s], (it / p.nst) & 1, p.a.err, YLM_DEV_ERR_TIMEOUT_FULL))
            {
                ok = false;
                break;
            }
            float xv[8];
            unpack8(*reinterpret_cast<const uint4 *>(xs + kc * GEMV_KC + lane * 8), xv);
            const uint8_t *st = smem + (size_t)s * stage_bytes + lane * 16;
#pragma unroll
            for (int j = 0; j < GEMV_MAXJ; j++)
            {
                const int r = gemv_row_of<PAIR>(j, warp);
                if (r < p.rb)
                    acc[j] = dot8(*reinterpret_cast<const uint4 *>(st + r * (GEMV_KC * 2)), xv, acc[j]);
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&empty[s]);
        }
        if (!ok)
            break;
#pragma unroll
        for (int j = 0; j < GEMV_MAXJ; j++)
            acc[j] = warp_sum(acc[j]);
        if (lane != 0)
            continue;
        if (EPI == EPI_SWIGLU)
        {
#pragma unroll
            for (int j = 0; j < GEMV_MAXJ; j += 2)
            {
                const int r = gemv_row_of<1>(j, warp);
                const int row = b * p.rb + r;
                if (r < p.rb && row < p.N)
                {
                    const float g = rh(acc[j]);
                    const float u = rh(acc[j + 1]);
                    const float sg = rh(g / (1.0f + expf(-g)));
                    p.a.out[row >> 1] = f2h(sg * u);
                }
            }
        }
        else
        {
#pragma unroll
            for (int j = 0; j < GEMV_MAXJ; j++)
            {
                const int r = gemv_row_of<0>(j, warp);
                const int row = b * p.rb + r;
                if (r < p.rb && row < p.N)
                {
                    if (EPI == EPI_STORE)
                    {
                        float y = acc[j];
                        if (p.a.bias)
                            y = rh(y) + h2f(p.a.bias[row]);
                        p.a.out[row] = f2h(y);
                    }
                    else
                    {
                        p.a.resid[row] = f2h(h2f(p.a.resid[row]) + rh(acc[j]));
                    }
                }
            }
        }
    }
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder()
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

bool gemv_make_plan(GemvPlan *pl, const __half *w, int N, int K, int pair, int num_sms)
{
    if (N <= 0 || K <= 0 || (K % 8) != 0 || (reinterpret_cast<uintptr_t>(w) % 16) != 0 || (pair && (N % 2)))
        return false;
    pl->w = w;
    pl->N = N;
    pl->K = K;
    pl->pair = pair;
    const int per = num_sms * GEMV_MAX_RB;
    const int m = (N + per - 1) / per;
    int rb = (N + num_sms * m - 1) / (num_sms * m);
    rb = std::max(rb, std::min(N, 8));
    if (pair)
        rb = (rb + 1) & ~1;
    rb = std::min(rb, GEMV_MAX_RB);
    pl->rb = rb;
    pl->n_blocks = (N + rb - 1) / rb;
    pl->grid = std::min(pl->n_blocks, num_sms);
    pl->k_pad = (K + GEMV_KC - 1) / GEMV_KC * GEMV_KC;
    const size_t stage = (size_t)rb * GEMV_KC * 2;
    const size_t xb = (size_t)pl->k_pad * 2;
    const size_t fixed = xb + 16 * 8 + 64;
    int nst = 2;
    if (GEMV_SMEM_BUDGET > fixed)
        nst = (int)std::max<size_t>(2, std::min<size_t>(8, (GEMV_SMEM_BUDGET - fixed) / stage));
    pl->nst = nst;
    pl->smem = nst * stage + fixed;
    if (pl->smem > 220 * 1024)
        return false;

    auto enc = tensor_map_encoder();
    if (!enc)
        return false;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {(cuuint32_t)GEMV_KC, (cuuint32_t)rb};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&pl->map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(w), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int PRO, int EPI>
static cudaError_t gemv_launch_t(const GemvPlan &pl, const GemvArgs &a, cudaStream_t s, bool pdl)
{
    GemvDev d;
    d.N = pl.N;
    d.K = pl.K;
    d.rb = pl.rb;
    d.n_blocks = pl.n_blocks;
    d.nst = pl.nst;
    d.k_pad = pl.k_pad;
    d.n_chunks = pl.k_pad / GEMV_KC;
    d.a = a;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(GEMV_THREADS);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_kernel<PRO, EPI>, pl.map, d);
}

// Opt every instantiation in to large dynamic shared memory, once per device,
// before any launch (and so never inside a stream capture).
cudaError_t gemv_prepare()
{
    const void *fns[] = {(const void *)gemv_kernel<PRO_VEC, EPI_STORE>,          (const void *)gemv_kernel<PRO_VEC, EPI_RESID>,
                         (const void *)gemv_kernel<PRO_VEC, EPI_SWIGLU>,         (const void *)gemv_kernel<PRO_RMSNORM, EPI_STORE>,
                         (const void *)gemv_kernel<PRO_RMSNORM, EPI_RESID>,      (const void *)gemv_kernel<PRO_RMSNORM, EPI_SWIGLU>,
                         (const void *)gemv_kernel<PRO_EMBED_RMSNORM, EPI_STORE>};
    for (const void *f : fns)
    {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
        if (e != cudaSuccess)
            return e;
    }
    return cudaSuccess;
}

cudaError_t gemv_launch(const GemvPlan &pl, int pro, int epi, const GemvArgs &a, cudaStream_t s, bool pdl)
{
    if ((epi == EPI_SWIGLU) != (pl.pair != 0))
        return cudaErrorInvalidValue;
#define YLM_GEMV_CASE(P, E) \
    if (pro == P && epi == E) \
        return gemv_launch_t<P, E>(pl, a, s, pdl);
    YLM_GEMV_CASE(PRO_VEC, EPI_STORE)
    YLM_GEMV_CASE(PRO_VEC, EPI_RESID)
    YLM_GEMV_CASE(PRO_VEC, EPI_SWIGLU)
    YLM_GEMV_CASE(PRO_RMSNORM, EPI_STORE)
    YLM_GEMV_CASE(PRO_RMSNORM, EPI_RESID)
    YLM_GEMV_CASE(PRO_RMSNORM, EPI_SWIGLU)
    YLM_GEMV_CASE(PRO_EMBED_RMSNORM, EPI_STORE)
#undef YLM_GEMV_CASE
    return cudaErrorInvalidValue;
}

} // namespace ylm
