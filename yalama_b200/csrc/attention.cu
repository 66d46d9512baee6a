// Split-K GQA decode attention over the fixed KV cache, with the per-token work
// of the reference fused in front of it:
//   q/k per-head RMSNorm        src/models/Qwen3Model.cpp:26-33
//   RoPE (rotate-half)          src/models/ModelBase.cpp:784-820, decode call :577-578
//   KV append at slot last+1    src/models/ModelBase.cpp:580-581
//   SDPA over slots [0, last+2) src/models/ModelBase.cpp:583-584, 638, 671-693
// The reference materialises the GQA head repeat (ExpandKV, ModelBase.cpp:695-707);
// here the query heads of one KV group share a single read of that group's K/V.
//
// Grid: (KV head, split). Each CTA owns a contiguous token range of one KV head
// and all G = hq/hkv query heads of the group. K/V rows of earlier steps are
// constant during the step, so thread 0 bulk-copies them (cp.async.bulk, 256 B
// per token, no multicast) into a ring of shared-memory tiles before
// griddepcontrol.wait; the new token's k/v are computed from the QKV output and
// used from shared memory. Half-warps take one token each (16 lanes x 8
// elements of D), online softmax in FP32 (base 2), partials per split go to a
// scratch buffer and the last CTA of each KV head combines them and writes the
// FP16 attention output [hq * 128].
#include "ylm_common.cuh"
#include "ylm_kernels.h"
#include <algorithm>

namespace ylm {

constexpr int ATT_THREADS = 128;
constexpr int ATT_TT = 32;  // tokens per tile
constexpr int ATT_NST = 4;  // tiles in flight
constexpr int ATT_ROW = 2 + YLM_HEAD_DIM;
constexpr float ATT_SCALE_LOG2 = 0.08838834764831845f * 1.4426950408889634f;

// One warp prepares one head: optional per-head RMSNorm, then RoPE at `pos`.
// Lane l holds elements [4l, 4l+4); its rotate-half partner is lane l ^ 16.
__device__ __forceinline__ void prep_head(const __half *src, const __half *norm_w, float eps, const __half *cosr,
                                          const __half *sinr, bool rope, float *dst, int lane)
{
    float x[4];
    {
        const __half2 *s2 = reinterpret_cast<const __half2 *>(src + lane * 4);
        float2 a = __half22float2(s2[0]), b = __half22float2(s2[1]);
        x[0] = a.x;
        x[1] = a.y;
        x[2] = b.x;
        x[3] = b.y;
    }
    if (norm_w)
    {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 4; e++)
            ss += rh(x[e] * x[e]);
        ss = warp_sum(ss);
        const float mean = rh(ss * (1.0f / YLM_HEAD_DIM));
        const float d = rh(rsqrtf(mean + eps));
#pragma unroll
        for (int e = 0; e < 4; e++)
            x[e] = rh(rh(x[e] * d) * h2f(norm_w[lane * 4 + e]));
    }
    if (rope)
    {
        float px[4];
#pragma unroll
        for (int e = 0; e < 4; e++)
            px[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
#pragma unroll
        for (int e = 0; e < 4; e++)
        {
            const int d = lane * 4 + e;
            const float c = h2f(cosr[d & 63]), s = h2f(sinr[d & 63]);
            const float rot = d < 64 ? -px[e] : px[e];
            x[e] = rh(rh(x[e] * c) + rh(rot * s));
        }
    }
#pragma unroll
    for (int e = 0; e < 4; e++)
        dst[lane * 4 + e] = x[e];
}

__device__ __forceinline__ void att_update(float &m, float &l, float *o, float sc, const float *v)
{
    const float mn = fmaxf(m, sc);
    const float c = exp2f(m - mn);
    const float p = exp2f(sc - mn);
    l = l * c + p;
#pragma unroll
    for (int e = 0; e < 8; e++)
        o[e] = o[e] * c + p * v[e];
    m = mn;
}

template <int G>
__global__ void __launch_bounds__(ATT_THREADS) attn_decode_kernel(const AttnArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int TILE_BYTES = ATT_TT * YLM_HEAD_DIM * 2;
    uint8_t *tiles = smem; // ATT_NST x (K tile, V tile)
    float *q_s = reinterpret_cast<float *>(smem + ATT_NST * 2 * TILE_BYTES);
    float *kn_s = q_s + G * YLM_HEAD_DIM;
    float *vn_s = kn_s + YLM_HEAD_DIM;
    uint64_t *bars = reinterpret_cast<uint64_t *>(vn_s + YLM_HEAD_DIM);
    int *flags = reinterpret_cast<int *>(bars + ATT_NST); // [0] abort, [1] ticket, [2] tiles issued
    float *merge = reinterpret_cast<float *>(tiles); // aliases the tiles after the token loop

    const int g = blockIdx.x, sp = blockIdx.y, S = gridDim.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    pdl_launch_dependents();
    const int slot = a.state->slot;
    const int pos = a.state->rope_pos;
    if (slot < 0 || slot >= a.cap || pos < 0 || pos >= a.max_pos)
    {
        if (tid == 0 && a.err)
            atomicExch(a.err, YLM_DEV_ERR_BAD_STATE);
        return;
    }
    const int n = slot + 1;
    const int chunk = (n + S - 1) / S;
    const int t0 = min(n, sp * chunk), t1 = min(n, t0 + chunk);
    const bool owns_new = slot >= t0 && slot < t1;
    const int te = owns_new ? slot : t1;
    const int n_tiles = (te - t0 + ATT_TT - 1) / ATT_TT;
    const __half *kc = a.k_cache + (size_t)g * a.cap * YLM_HEAD_DIM;
    const __half *vc = a.v_cache + (size_t)g * a.cap * YLM_HEAD_DIM;

    auto issue = [&](int i) {
        const int s = i % ATT_NST;
        const int ta = t0 + i * ATT_TT;
        const int nt = min(ATT_TT, te - ta);
        const uint32_t bytes = nt * YLM_HEAD_DIM * 2;
        mbar_arrive_expect_tx(&bars[s], 2 * bytes);
        bulk_load(tiles + (size_t)s * 2 * TILE_BYTES, kc + (size_t)ta * YLM_HEAD_DIM, bytes, &bars[s]);
        bulk_load(tiles + (size_t)s * 2 * TILE_BYTES + TILE_BYTES, vc + (size_t)ta * YLM_HEAD_DIM, bytes, &bars[s]);
        flags[2] = i + 1; // tiles issued so far (thread 0 only)
    };

    if (tid == 0)
    {
        for (int s = 0; s < ATT_NST; s++)
            mbar_init(&bars[s], 1);
        flags[0] = 0;
        flags[2] = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0)
        for (int i = 0; i < min(ATT_NST, n_tiles); i++)
            issue(i);

    // ---- wait for the QKV projection, then prepare q (and the new k, v)
    pdl_wait();
    const __half *cosr = a.rope_cos + (size_t)pos * 64;
    const __half *sinr = a.rope_sin + (size_t)pos * 64;
    for (int h = warp; h < G; h += ATT_THREADS / 32)
        prep_head(a.qkv + (size_t)(g * G + h) * YLM_HEAD_DIM, a.q_norm, a.eps, cosr, sinr, true,
                  q_s + h * YLM_HEAD_DIM, lane);
    if (owns_new)
    {
        if (warp == 0)
        {
            prep_head(a.qkv + (size_t)(a.hq + g) * YLM_HEAD_DIM, a.k_norm, a.eps, cosr, sinr, true, kn_s, lane);
            __syncwarp();
            for (int d = lane; d < YLM_HEAD_DIM; d += 32)
                a.k_cache[((size_t)g * a.cap + slot) * YLM_HEAD_DIM + d] = f2h(kn_s[d]);
        }
        else if (warp == 1)
        {
            for (int d = lane; d < YLM_HEAD_DIM; d += 32)
            {
                const __half v = a.qkv[(size_t)(a.hq + a.hkv + g) * YLM_HEAD_DIM + d];
                vn_s[d] = h2f(v);
                a.v_cache[((size_t)g * a.cap + slot) * YLM_HEAD_DIM + d] = v;
            }
        }
    }
    __syncthreads();

    // ---- token loop: half-warp hw takes tokens hw, hw+8, ... of each tile
    const int hw = tid >> 4, l16 = tid & 15;
    float q[G][8], o[G][8], m[G], l[G];
#pragma unroll
    for (int h = 0; h < G; h++)
    {
#pragma unroll
        for (int e = 0; e < 8; e++)
        {
            q[h][e] = q_s[h * YLM_HEAD_DIM + l16 * 8 + e] * ATT_SCALE_LOG2;
            o[h][e] = 0.f;
        }
        m[h] = -INFINITY;
        l[h] = 0.f;
    }
    bool ok = true;
    for (int i = 0; i < n_tiles; i++)
    {
        const int s = i % ATT_NST;
        if (!mbar_wait_bounded(&bars[s], (i / ATT_NST) & 1, a.err, YLM_DEV_ERR_TIMEOUT_FULL))
            ok = false;
        if (ok)
        {
            const int nt = min(ATT_TT, te - (t0 + i * ATT_TT));
            const __half *kt = reinterpret_cast<const __half *>(tiles + (size_t)s * 2 * TILE_BYTES);
            const __half *vt = kt + ATT_TT * YLM_HEAD_DIM;
            // both half-warps of a warp run the same trip count (warp-uniform
            // bound) so the full-mask shuffles below never diverge
            for (int kb = 2 * warp; kb < nt; kb += 8)
            {
                const int k = kb + (hw & 1);
                const bool valid = k < nt;
                float kf[8], vf[8];
                const int kr = valid ? k : kb;
                unpack8(*reinterpret_cast<const uint4 *>(kt + kr * YLM_HEAD_DIM + l16 * 8), kf);
                unpack8(*reinterpret_cast<const uint4 *>(vt + kr * YLM_HEAD_DIM + l16 * 8), vf);
#pragma unroll
                for (int h = 0; h < G; h++)
                {
                    float sc = 0.f;
#pragma unroll
                    for (int e = 0; e < 8; e++)
                        sc = fmaf(q[h][e], kf[e], sc);
                    sc += __shfl_xor_sync(0xffffffffu, sc, 8, 16);
                    sc += __shfl_xor_sync(0xffffffffu, sc, 4, 16);
                    sc += __shfl_xor_sync(0xffffffffu, sc, 2, 16);
                    sc += __shfl_xor_sync(0xffffffffu, sc, 1, 16);
                    if (valid)
                        att_update(m[h], l[h], o[h], sc, vf);
                }
            }
        }
        __syncthreads();
        if (!ok)
            flags[0] = 1;
        if (tid == 0 && ok && i + ATT_NST < n_tiles)
            issue(i + ATT_NST);
        __syncthreads();
        if (flags[0])
            break;
    }
    if (flags[0])
    {
        // drain copies still in flight, then leave without touching the counters
        if (tid == 0)
            for (int i = max(0, flags[2] - ATT_NST); i < flags[2]; i++)
                mbar_wait_bounded(&bars[i % ATT_NST], (i / ATT_NST) & 1, a.err, YLM_DEV_ERR_TIMEOUT_DRAIN);
        return;
    }
    if (owns_new && hw == 0)
    {
        float kf[8], vf[8];
#pragma unroll
        for (int e = 0; e < 8; e++)
        {
            kf[e] = kn_s[l16 * 8 + e];
            vf[e] = vn_s[l16 * 8 + e];
        }
#pragma unroll
        for (int h = 0; h < G; h++)
        {
            float sc = 0.f;
#pragma unroll
            for (int e = 0; e < 8; e++)
                sc = fmaf(q[h][e], kf[e], sc);
            sc += __shfl_xor_sync(0x0000ffffu, sc, 8, 16);
            sc += __shfl_xor_sync(0x0000ffffu, sc, 4, 16);
            sc += __shfl_xor_sync(0x0000ffffu, sc, 2, 16);
            sc += __shfl_xor_sync(0x0000ffffu, sc, 1, 16);
            att_update(m[h], l[h], o[h], sc, vf);
        }
    }

    // ---- merge the 8 half-warps, then write this split's partial
#pragma unroll
    for (int h = 0; h < G; h++)
    {
        float *row = merge + (hw * G + h) * ATT_ROW;
        if (l16 == 0)
        {
            row[0] = m[h];
            row[1] = l[h];
        }
#pragma unroll
        for (int e = 0; e < 8; e++)
            row[2 + l16 * 8 + e] = o[h][e];
    }
    __syncthreads();
    const int d = tid;
#pragma unroll 1
    for (int h = 0; h < G; h++)
    {
        float M = -INFINITY;
        for (int w = 0; w < 8; w++)
            M = fmaxf(M, merge[(w * G + h) * ATT_ROW]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY)
            for (int w = 0; w < 8; w++)
            {
                const float *row = merge + (w * G + h) * ATT_ROW;
                const float c = exp2f(row[0] - M);
                L += row[1] * c;
                O += row[2 + d] * c;
            }
        float *pr = a.partial + ((size_t)(g * G + h) * S + sp) * ATT_ROW;
        pr[2 + d] = O;
        if (d == 0)
        {
            pr[0] = M;
            pr[1] = L;
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0)
        flags[1] = atomicAdd(&a.counters[g], 1);
    __syncthreads();
    if (flags[1] != S - 1)
        return;

    // ---- last CTA of this KV head: combine the splits
    __threadfence();
#pragma unroll 1
    for (int h = 0; h < G; h++)
    {
        const float *base = a.partial + (size_t)(g * G + h) * S * ATT_ROW;
        float M = -INFINITY;
        for (int s = 0; s < S; s++)
            M = fmaxf(M, __ldcg(base + s * ATT_ROW));
        float L = 0.f, O = 0.f;
        for (int s = 0; s < S; s++)
        {
            const float ms = __ldcg(base + s * ATT_ROW);
            if (ms == -INFINITY)
                continue;
            const float c = exp2f(ms - M);
            L += __ldcg(base + s * ATT_ROW + 1) * c;
            O += __ldcg(base + s * ATT_ROW + 2 + d) * c;
        }
        a.out[(size_t)(g * G + h) * YLM_HEAD_DIM + d] = f2h(O / L);
    }
    if (tid == 0)
        a.counters[g] = 0;
}

size_t attn_partial_floats(int hq, int splits) { return (size_t)hq * splits * ATT_ROW; }

int attn_default_splits(int hkv, int num_sms) { return std::max(1, num_sms / std::max(1, hkv)); }

static size_t attn_smem_bytes(int G)
{
    size_t tiles = (size_t)ATT_NST * 2 * ATT_TT * YLM_HEAD_DIM * 2;
    size_t merge = (size_t)8 * G * ATT_ROW * 4;
    return std::max(tiles, merge) + (size_t)(G + 2) * YLM_HEAD_DIM * 4 + ATT_NST * 8 + 16;
}

template <int G>
static cudaError_t attn_launch_t(const AttnArgs &a, cudaStream_t s, bool pdl)
{
    const size_t smem = attn_smem_bytes(G);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.hkv, a.splits);
    cfg.blockDim = dim3(ATT_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, attn_decode_kernel<G>, a);
}

template <int G> static cudaError_t attn_prepare_t()
{
    return cudaFuncSetAttribute(attn_decode_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)attn_smem_bytes(G));
}

cudaError_t attn_prepare()
{
    cudaError_t e = cudaSuccess;
    if (e == cudaSuccess) e = attn_prepare_t<1>();
    if (e == cudaSuccess) e = attn_prepare_t<2>();
    if (e == cudaSuccess) e = attn_prepare_t<3>();
    if (e == cudaSuccess) e = attn_prepare_t<4>();
    if (e == cudaSuccess) e = attn_prepare_t<5>();
    if (e == cudaSuccess) e = attn_prepare_t<6>();
    if (e == cudaSuccess) e = attn_prepare_t<7>();
    if (e == cudaSuccess) e = attn_prepare_t<8>();
    return e;
}

cudaError_t attn_decode_launch(const AttnArgs &a, cudaStream_t s, bool pdl)
{
    if (a.hkv <= 0 || a.hq % a.hkv != 0 || a.splits <= 0)
        return cudaErrorInvalidValue;
    switch (a.hq / a.hkv)
    {
    case 1: return attn_launch_t<1>(a, s, pdl);
    case 2: return attn_launch_t<2>(a, s, pdl);
    case 3: return attn_launch_t<3>(a, s, pdl);
    case 4: return attn_launch_t<4>(a, s, pdl);
    case 5: return attn_launch_t<5>(a, s, pdl);
    case 6: return attn_launch_t<6>(a, s, pdl);
    case 7: return attn_launch_t<7>(a, s, pdl);
    case 8: return attn_launch_t<8>(a, s, pdl);
    default: return cudaErrorInvalidValue;
    }
}

} // namespace ylm
