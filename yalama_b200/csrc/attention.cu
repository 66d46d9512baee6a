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
// and all G = hq/hkv query heads of the group. Half-warps take one token at a
// time (16 lanes x 8 elements of D, one 16-byte streaming load of K and one of
// V per lane), ATT_UT tokens per half-warp in flight, online softmax in FP32
// (base 2). K/V rows of earlier steps are constant during the step, so the
// first group of loads is issued before griddepcontrol.wait; the new token's
// k/v are computed from the QKV output and used from shared memory. Partials
// per split go to a scratch buffer and the last CTA of each KV head (atomic
// ticket) combines them and writes the FP16 attention output [hq * 128].
#include "ylm_common.cuh"
#include "ylm_kernels.h"
#include <algorithm>
#include <cooperative_groups.h>

namespace ylm {

constexpr int ATT_THREADS = 128;
constexpr int ATT_HW = ATT_THREADS / 16; // half-warps
constexpr int ATT_UT = 4;                // tokens in flight per half-warp
constexpr int ATT_ROW = 2 + YLM_HEAD_DIM;
constexpr int ATT_MIN_SPLIT = 64;        // tokens per split, at least
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

__device__ __forceinline__ uint4 ldg_nc(const void *p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

template <int G>
__global__ void __launch_bounds__(ATT_THREADS) attn_decode_kernel(const AttnArgs a)
{
    __shared__ float q_s[G * YLM_HEAD_DIM];
    __shared__ float kn_s[YLM_HEAD_DIM], vn_s[YLM_HEAD_DIM];
    __shared__ float merge[ATT_HW * G * ATT_ROW];
    __shared__ int ticket;

    const int g = blockIdx.x, sp = blockIdx.y, S = gridDim.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hw = tid >> 4, l16 = tid & 15;

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
    // at least ATT_MIN_SPLIT tokens per split: short contexts use fewer splits
    // (the rest of the grid exits at once) and a cheaper combine
    const int chunk = max(ATT_MIN_SPLIT, (n + S - 1) / S);
    const int S_eff = (n + chunk - 1) / chunk;
    if (sp >= S_eff)
        return;
    const int t0 = sp * chunk, t1 = min(n, t0 + chunk);
    const bool owns_new = slot >= t0 && slot < t1;
    const int te = owns_new ? slot : t1; // cached tokens [t0, te); the new one comes from qkv
    const __half *kc = a.k_cache + (size_t)g * a.cap * YLM_HEAD_DIM + l16 * 8;
    const __half *vc = a.v_cache + (size_t)g * a.cap * YLM_HEAD_DIM + l16 * 8;

    // token i of this half-warp's sequence: t0 + hw + ATT_HW * i
    uint4 kr[ATT_UT], vr[ATT_UT];
    auto load_group = [&](int i0) {
#pragma unroll
        for (int u = 0; u < ATT_UT; u++)
        {
            const int t = t0 + hw + ATT_HW * (i0 + u);
            if (t < te)
            {
                kr[u] = ldg_nc(kc + (size_t)t * YLM_HEAD_DIM);
                vr[u] = ldg_nc(vc + (size_t)t * YLM_HEAD_DIM);
            }
        }
    };
    // earlier slots are constant during this step: start their loads before the wait
    load_group(0);

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
    // both half-warps of a warp run the same number of groups (warp-uniform
    // bound), so the full-mask shuffles below never diverge
    const int ntok = max(0, te - t0);
    const int per_hw = (ntok + ATT_HW - 1) / ATT_HW; // tokens of half-warp 0, the largest share
    for (int i0 = 0; i0 < per_hw; i0 += ATT_UT)
    {
        uint4 kc_u[ATT_UT], vc_u[ATT_UT];
#pragma unroll
        for (int u = 0; u < ATT_UT; u++)
        {
            kc_u[u] = kr[u];
            vc_u[u] = vr[u];
        }
        if (i0 + ATT_UT < per_hw)
            load_group(i0 + ATT_UT);
#pragma unroll
        for (int u = 0; u < ATT_UT; u++)
        {
            const int t = t0 + hw + ATT_HW * (i0 + u);
            const bool valid = t < te;
            float kf[8], vf[8];
            unpack8(kc_u[u], kf);
            unpack8(vc_u[u], vf);
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

    // ---- merge the half-warps, then write this split's partial
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
        for (int w = 0; w < ATT_HW; w++)
            M = fmaxf(M, merge[(w * G + h) * ATT_ROW]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY)
            for (int w = 0; w < ATT_HW; w++)
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
        ticket = atomicAdd(&a.counters[g], 1);
    __syncthreads();
    if (ticket != S_eff - 1)
        return;

    // ---- last CTA of this KV head: combine the splits. The (M, L) pairs are
    // fetched in parallel into shared memory (the merge buffer is free now),
    // then each thread sums its output dimension over the splits with the
    // loads unrolled.
    __threadfence();
    float *Ms = merge;                 // [G][S_eff]
    float *Ls = merge + G * S_eff;     // [G][S_eff]
    for (int i = tid; i < G * S_eff; i += ATT_THREADS)
    {
        const int h = i / S_eff, s = i % S_eff;
        const float *pr = a.partial + ((size_t)(g * G + h) * S + s) * ATT_ROW;
        Ms[i] = __ldcg(pr);
        Ls[i] = __ldcg(pr + 1);
    }
    __syncthreads();
#pragma unroll 1
    for (int h = 0; h < G; h++)
    {
        float M = -INFINITY;
        for (int s = 0; s < S_eff; s++)
            M = fmaxf(M, Ms[h * S_eff + s]);
        const float *base = a.partial + (size_t)(g * G + h) * S * ATT_ROW + 2 + d;
        float L = 0.f, O = 0.f;
#pragma unroll 8
        for (int s = 0; s < S_eff; s++)
        {
            const float ms = Ms[h * S_eff + s];
            const float c = ms == -INFINITY ? 0.f : exp2f(ms - M);
            L += Ls[h * S_eff + s] * c;
            O += __ldcg(base + (size_t)s * ATT_ROW) * c;
        }
        a.out[(size_t)(g * G + h) * YLM_HEAD_DIM + d] = f2h(O / L);
    }
    if (tid == 0)
        a.counters[g] = 0;
}

// ---------------------------------------------------------------- cluster variant
// One thread-block cluster per KV head, one CTA per split of the cached
// tokens (S = cluster size: 8, or 16 for launches over 4 KV heads or fewer,
// where the device schedules them; see attn_cluster_size). Inside a CTA each warp takes whole tokens (lane l holds dimensions
// 4l..4l+3), ATC_UT tokens per batch: all their scores first, then one
// rescale of the running softmax state. The 8 warp states are merged in
// shared memory; each CTA then stores its partial (M, L and one slice of O per
// head) into the shared memory of the rank that owns that slice (distributed
// shared memory), and after one cluster barrier every rank combines its slice
// of the S partials and writes it. No global scratch, fence or atomic ticket.
// D (rows 0..7 of a 16 x 8 FP32 tile, d0 d1) += A B with A rows 8..15 zero:
// mma.sync m16n8k16, FP16 operands (a0 = A[r][2q..], a2 = A[r][2q+8..]),
// z0 z1 the unused rows 8..15 of D (they stay zero).
__device__ __forceinline__ void atm_mma(float &d0, float &d1, float &z0, float &z1, uint32_t a0, uint32_t a2,
                                        uint32_t b0, uint32_t b1)
{
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d0), "+f"(d1), "+f"(z0), "+f"(z1)
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

constexpr int ATC_THREADS = 256;
constexpr int ATC_QF = 20; // words per packed Q-fragment row (16 used)
constexpr int ATC_WARPS = ATC_THREADS / 32;
constexpr int ATC_MAX_SPLITS = 16; // largest cluster the kernel supports
constexpr int ATC_MIN_SPLITS = 8;  // smallest cluster (the portable size)

static int g_cluster_splits = 0; // largest schedulable cluster: 16, 8, or 0 (no cluster launch: split-K kernel)
static int g_force_split = 0;    // 1: the split-K kernel even where clusters launch (tests, diagnostics)

template <int G>
__global__ void __launch_bounds__(ATC_THREADS) attn_cluster_kernel(const AttnArgs a)
{
    __shared__ __align__(16) float q_s[G * YLM_HEAD_DIM];
    __shared__ float kn_s[YLM_HEAD_DIM], vn_s[YLM_HEAD_DIM];
    __shared__ __align__(16) float mrg[ATC_WARPS * G * ATT_ROW];
    // Q's A fragments, packed by the warps that prepare the heads: head h,
    // quarter kq at words [(4 h + kq) * ATC_QF, + 16) (k-step j: words 2 j,
    // 2 j + 1); the padded stride makes the lanes' 16-byte reads conflict-free.
    // It lives in mrg until the warp states are written there.
    uint32_t *qfrag = reinterpret_cast<uint32_t *>(mrg);
    __shared__ float recv[ATC_MAX_SPLITS * G * (2 + YLM_HEAD_DIM / ATC_MIN_SPLITS)]; // [rank][head][M, L, slice]
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    const int S = (int)cl.num_blocks();
    const int sp = (int)cl.block_rank();
    const int g = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // every CTA of the cluster must have started before another one writes
    // into its shared memory: arrive now, wait before the first remote store
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    pdl_launch_dependents();
    const int slot = a.state->slot;
    const int pos = a.state->rope_pos;
    const bool ok = slot >= 0 && slot < a.cap && pos >= 0 && pos < a.max_pos;
    if (!ok && sp == 0 && g == 0 && tid == 0 && a.err)
        atomicExch(a.err, YLM_DEV_ERR_BAD_STATE);
    const int n = ok ? slot + 1 : 0;
    const int chunk = (n + S - 1) / S;
    const int t0 = min(n, sp * chunk), t1 = min(n, t0 + chunk);
    const bool owns_new = ok && slot >= t0 && slot < t1;
    const int te = owns_new ? slot : t1; // cached tokens [t0, te); the new one comes from qkv

    // Cached tokens [t0, te) in chunks of 16, chunk c = tokens t0 + 16 c ...,
    // warp w taking chunks w, w + 8, ...; both products of a chunk on the
    // tensor cores (mma.sync m16n8k16, FP16 inputs, FP32 accumulation), the G
    // query heads of the group as rows 0..G-1 of M (rows G..15 zero).
    // Lane l works on head row m = l / 4 and quarter kq = l % 4.
    //  S = Q K^T: the head dimension is summed in a permuted order so that
    //    every B fragment comes from 16-byte loads of K rows: in k-step
    //    j = 2 s + t, k positions 2 kq + {0, 1} and 2 kq + 8 + {0, 1} are
    //    dimensions 32 kq + 8 s + 4 t + {0, 1} and + {2, 3}; n position p of
    //    n-tile b is token 8 b + p of the chunk. Lane l loads dimensions
    //    [32 kq, 32 kq + 32) of tokens l / 4 and 8 + l / 4.
    //  O += P V: k = the chunk's 16 tokens (P straight from the S
    //    accumulators), n-tile i position p = dimension 16 p + i, so lane l
    //    loads dimensions [16 (l / 4), + 16) of tokens 2 kq + {0, 1, 8, 9},
    //    and its O accumulators are head m, dimensions 32 kq + 16 c + i.
    // Earlier slots are constant during the step: each warp's first chunk is
    // loaded before griddepcontrol.wait.
    const int nchunks = (te - t0 + 15) >> 4;
    const int hm = lane >> 2, kq = lane & 3;
    const __half *kc = a.k_cache + (size_t)g * a.cap * YLM_HEAD_DIM;
    const __half *vc = a.v_cache + (size_t)g * a.cap * YLM_HEAD_DIM;
    struct Chunk
    {
        uint4 k[2][4]; // [n-tile][16-byte piece]: token 8 b + hm, dims 32 kq + 8 s ..
        uint4 v[4][2]; // [token 2 kq + {0, 1, 8, 9}][half]: dims 16 hm ..
    };
    auto load_chunk = [&](Chunk &ch, int c) {
        const int c0 = t0 + 16 * c;
#pragma unroll
        for (int b = 0; b < 2; b++)
        {
            const int t = c0 + 8 * b + hm;
            const uint4 *src = reinterpret_cast<const uint4 *>(kc + (size_t)t * YLM_HEAD_DIM + 32 * kq);
#pragma unroll
            for (int s = 0; s < 4; s++)
                ch.k[b][s] = t < te ? __ldg(src + s) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int r = 0; r < 4; r++)
        {
            const int t = c0 + 2 * kq + (r & 1) + 8 * (r >> 1);
            const uint4 *src = reinterpret_cast<const uint4 *>(vc + (size_t)t * YLM_HEAD_DIM + 16 * hm);
#pragma unroll
            for (int hh = 0; hh < 2; hh++)
                ch.v[r][hh] = t < te ? __ldg(src + hh) : make_uint4(0, 0, 0, 0);
        }
    };
    Chunk bufA, bufB;
    if (warp < nchunks)
        load_chunk(bufA, warp);
    pdl_wait();

    if (ok)
    {
        const __half *cosr = a.rope_cos + (size_t)pos * 64;
        const __half *sinr = a.rope_sin + (size_t)pos * 64;
        for (int h = warp; h < G + 2; h += ATC_WARPS)
        {
            if (h < G)
            {
                prep_head(a.qkv + (size_t)(g * G + h) * YLM_HEAD_DIM, a.q_norm, a.eps, cosr, sinr, true,
                          q_s + h * YLM_HEAD_DIM, lane);
                __syncwarp();
                // lane l holds dimensions 4 l .. 4 l + 3 = quarter l / 8, k-step
                // l % 8 (32 kq + 8 s + 4 t = 4 l); FP16 values (prep_head rounds)
                const float4 v = *reinterpret_cast<const float4 *>(q_s + h * YLM_HEAD_DIM + 4 * lane);
                const __half2 lo = __floats2half2_rn(v.x, v.y), hi = __floats2half2_rn(v.z, v.w);
                *reinterpret_cast<uint2 *>(qfrag + (4 * h + (lane >> 3)) * ATC_QF + 2 * (lane & 7)) =
                    make_uint2(*reinterpret_cast<const uint32_t *>(&lo), *reinterpret_cast<const uint32_t *>(&hi));
            }
            else if (h == G && owns_new)
            {
                prep_head(a.qkv + (size_t)(a.hq + g) * YLM_HEAD_DIM, a.k_norm, a.eps, cosr, sinr, true, kn_s, lane);
                __syncwarp();
                for (int d = lane; d < YLM_HEAD_DIM; d += 32)
                    a.k_cache[((size_t)g * a.cap + slot) * YLM_HEAD_DIM + d] = f2h(kn_s[d]);
            }
            else if (h == G + 1 && owns_new)
                for (int d = lane; d < YLM_HEAD_DIM; d += 32)
                {
                    const __half v = a.qkv[(size_t)(a.hq + a.hkv + g) * YLM_HEAD_DIM + d];
                    vn_s[d] = h2f(v);
                    a.v_cache[((size_t)g * a.cap + slot) * YLM_HEAD_DIM + d] = v;
                }
        }
    }
    __syncthreads();

    // A fragments of Q, rows >= G zero (only warps with chunks use them)
    const bool real = hm < G;
    uint32_t qa[8][2];
    if (real && warp < nchunks)
    {
        const uint4 *f = reinterpret_cast<const uint4 *>(qfrag + (4 * hm + kq) * ATC_QF);
#pragma unroll
        for (int r = 0; r < 4; r++)
        {
            const uint4 w = f[r];
            qa[2 * r][0] = w.x;
            qa[2 * r][1] = w.y;
            qa[2 * r + 1][0] = w.z;
            qa[2 * r + 1][1] = w.w;
        }
    }
    else
#pragma unroll
        for (int j = 0; j < 8; j++)
            qa[j][0] = qa[j][1] = 0u;
    __syncthreads(); // qfrag is read before any warp writes its state into mrg
    float o[16][2];
#pragma unroll
    for (int i = 0; i < 16; i++)
        o[i][0] = o[i][1] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    auto process = [&](const Chunk &ch, int c) {
        const int c0 = t0 + 16 * c;
        float sc[2][2];
        float z0 = 0.f, z1 = 0.f; // rows 8..15 (A rows zero: stay zero)
#pragma unroll
        for (int b = 0; b < 2; b++)
        {
            sc[b][0] = sc[b][1] = 0.f;
#pragma unroll
            for (int j = 0; j < 8; j++)
            {
                const uint4 &w = ch.k[b][j >> 1];
                const uint32_t b0 = (j & 1) ? w.z : w.x, b1 = (j & 1) ? w.w : w.y;
                atm_mma(sc[b][0], sc[b][1], z0, z1, qa[j][0], qa[j][1], b0, b1);
            }
        }
        // online softmax of this lane's head over the chunk (base 2); the 4
        // lanes of a head row hold its 16 scores
        float s4[4];
#pragma unroll
        for (int e = 0; e < 4; e++)
        {
            const int t = c0 + 8 * (e >> 1) + 2 * kq + (e & 1);
            s4[e] = t < te ? sc[e >> 1][e & 1] * ATT_SCALE_LOG2 : -INFINITY;
        }
        float mx = fmaxf(fmaxf(s4[0], s4[1]), fmaxf(s4[2], s4[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m_run, mx);
        const bool none = mn == -INFINITY || !real;
        const float cs = none ? 1.f : exp2f(m_run - mn);
        float p[4];
#pragma unroll
        for (int e = 0; e < 4; e++)
            p[e] = none ? 0.f : exp2f(s4[e] - mn);
        l_run = l_run * cs + ((p[0] + p[1]) + (p[2] + p[3]));
        m_run = none ? m_run : mn;
        const __half2 p01 = __floats2half2_rn(p[0], p[1]), p23 = __floats2half2_rn(p[2], p[3]);
        const uint32_t pa0 = *reinterpret_cast<const uint32_t *>(&p01);
        const uint32_t pa2 = *reinterpret_cast<const uint32_t *>(&p23);
#pragma unroll
        for (int i = 0; i < 16; i++)
        {
            // V of tokens 2 kq + {0, 1} / + {8, 9} at dimension 16 hm + i
            const uint32_t w0 = reinterpret_cast<const uint32_t *>(&ch.v[0][i >> 3])[(i >> 1) & 3];
            const uint32_t w1 = reinterpret_cast<const uint32_t *>(&ch.v[1][i >> 3])[(i >> 1) & 3];
            const uint32_t w2 = reinterpret_cast<const uint32_t *>(&ch.v[2][i >> 3])[(i >> 1) & 3];
            const uint32_t w3 = reinterpret_cast<const uint32_t *>(&ch.v[3][i >> 3])[(i >> 1) & 3];
            const uint32_t sel = (i & 1) ? 0x7632u : 0x5410u;
            o[i][0] *= cs;
            o[i][1] *= cs;
            atm_mma(o[i][0], o[i][1], z0, z1, pa0, pa2, __byte_perm(w0, w1, sel), __byte_perm(w2, w3, sel));
        }
    };
    for (int c = warp; c < nchunks; c += 2 * ATC_WARPS)
    {
        if (c + ATC_WARPS < nchunks)
            load_chunk(bufB, c + ATC_WARPS);
        process(bufA, c);
        if (c + ATC_WARPS >= nchunks)
            break;
        if (c + 2 * ATC_WARPS < nchunks)
            load_chunk(bufA, c + 2 * ATC_WARPS);
        process(bufB, c + ATC_WARPS);
    }
    if (owns_new && warp == 0)
    {
        // the new token, from shared memory, in FP32: this lane's quarter of
        // the score, summed over the head row's 4 lanes
        float sn = 0.f;
        if (real)
#pragma unroll 8
            for (int d = 0; d < 32; d++)
                sn = fmaf(q_s[hm * YLM_HEAD_DIM + 32 * kq + d], kn_s[32 * kq + d], sn);
        sn += __shfl_xor_sync(0xffffffffu, sn, 1);
        sn += __shfl_xor_sync(0xffffffffu, sn, 2);
        sn *= ATT_SCALE_LOG2;
        if (real)
        {
            const float mn = fmaxf(m_run, sn);
            const float cs = exp2f(m_run - mn);
            const float ps = exp2f(sn - mn);
            l_run = l_run * cs + (kq == 0 ? ps : 0.f);
#pragma unroll
            for (int i = 0; i < 16; i++)
#pragma unroll
                for (int c = 0; c < 2; c++)
                    o[i][c] = o[i][c] * cs + ps * vn_s[32 * kq + 16 * c + i];
            m_run = mn;
        }
    }
    // warp states -> this CTA's partial (M, L, O per head)
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if (real)
    {
        float *row = mrg + (warp * G + hm) * ATT_ROW;
        if (kq == 0)
        {
            row[0] = m_run;
            row[1] = l_run;
        }
#pragma unroll
        for (int i = 0; i < 16; i++)
#pragma unroll
            for (int c = 0; c < 2; c++)
                row[2 + 32 * kq + 16 * c + i] = o[i][c];
    }
    __syncthreads();
    // this CTA's partial, pushed straight into the cluster: rank q combines
    // dimensions [q * slice, (q + 1) * slice) of every head, so it receives
    // every rank's (M, L) and that slice of every rank's O (remote stores,
    // no round trips); one cluster barrier then publishes them
    const int slice = YLM_HEAD_DIM / S;
    const int RW = 2 + slice;
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
    for (int k = tid; k < G * YLM_HEAD_DIM; k += ATC_THREADS)
    {
        const int h = k >> 7, d = k & 127;
        float M = -INFINITY;
        for (int w = 0; w < ATC_WARPS; w++)
            M = fmaxf(M, mrg[(w * G + h) * ATT_ROW]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY)
            for (int w = 0; w < ATC_WARPS; w++)
            {
                const float *row = mrg + (w * G + h) * ATT_ROW;
                const float c = exp2f(row[0] - M);
                L += row[1] * c;
                O += row[2 + d] * c;
            }
        const int qd = d / slice;
        float *dst = cl.map_shared_rank(recv, qd) + (sp * G + h) * RW;
        dst[2 + d - qd * slice] = O;
        if (d - qd * slice == 0)
        {
            dst[0] = M;
            dst[1] = L;
        }
    }
    cl.sync(); // every rank's slices have landed
    if (ok)
        for (int k = tid; k < G * slice; k += ATC_THREADS)
        {
            const int h = k / slice, dl = k - h * slice;
            float M = -INFINITY;
            for (int r = 0; r < S; r++)
                M = fmaxf(M, recv[(r * G + h) * RW]);
            float L = 0.f, O = 0.f;
            for (int r = 0; r < S; r++)
            {
                const float *row = recv + (r * G + h) * RW;
                const float c = row[0] == -INFINITY ? 0.f : exp2f(row[0] - M);
                L += row[1] * c;
                O += row[2 + dl] * c;
            }
            a.out[(size_t)(g * G + h) * YLM_HEAD_DIM + sp * slice + dl] = f2h(O / L);
        }
}

template <int G>
static cudaError_t attn_cluster_launch_t(const AttnArgs &a, int S, cudaStream_t s, bool pdl)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, a.hkv);
    cfg.blockDim = dim3(ATC_THREADS);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = S;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    na++;
    if (pdl)
    {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, attn_cluster_kernel<G>, a);
}

// Largest cluster size (16, else 8) that the device can schedule for G, or 0.
template <int G> static int attn_cluster_prepare_t()
{
    if (cudaFuncSetAttribute(attn_cluster_kernel<G>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
        cudaSuccess)
        cudaGetLastError();
    for (int S : {16, 8})
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(S, 1);
        cfg.blockDim = dim3(ATC_THREADS);
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = S;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int nc = 0;
        if (cudaOccupancyMaxActiveClusters(&nc, attn_cluster_kernel<G>, &cfg) == cudaSuccess && nc >= 1)
            return S;
        cudaGetLastError();
    }
    return 0;
}

size_t attn_partial_floats(int hq, int splits) { return (size_t)hq * splits * ATT_ROW; }

// about two CTAs per SM over all KV heads
int attn_default_splits(int hkv, int num_sms) { return std::max(1, 2 * num_sms / std::max(1, hkv)); }

template <int G>
static cudaError_t attn_launch_t(const AttnArgs &a, cudaStream_t s, bool pdl)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.hkv, a.splits);
    cfg.blockDim = dim3(ATT_THREADS);
    cfg.dynamicSmemBytes = 0;
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
    return cudaFuncSetAttribute(attn_decode_kernel<G>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                (int)cudaSharedmemCarveoutMaxShared);
}

cudaError_t attn_prepare()
{
    int S = 16;
    S = std::min(S, attn_cluster_prepare_t<1>());
    S = std::min(S, attn_cluster_prepare_t<2>());
    S = std::min(S, attn_cluster_prepare_t<3>());
    S = std::min(S, attn_cluster_prepare_t<4>());
    S = std::min(S, attn_cluster_prepare_t<5>());
    S = std::min(S, attn_cluster_prepare_t<6>());
    S = std::min(S, attn_cluster_prepare_t<7>());
    S = std::min(S, attn_cluster_prepare_t<8>());
    g_cluster_splits = S;
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

void attn_force_split_kernel(bool on) { g_force_split = on ? 1 : 0; }

bool attn_uses_split_kernel() { return g_force_split || g_cluster_splits == 0; }

// Cluster size for a launch over `hkv` KV heads: 8 CTAs per head with 8 or
// more heads (the Llama-3.1-8B shape on one GPU, 2048-token prompt, measured
// 3.03 ms per decode step with 8-CTA clusters against 3.19 with 16 and 3.12
// with 4; Qwen3-0.6B, 32-token prompt, 0.83 ms against 0.94 and 0.82: fewer
// CTAs only pay at short contexts), 16 with fewer heads (a tensor-parallel
// rank's share), so the launch still spreads over more SMs.
static int attn_cluster_size(int hkv)
{
    if (g_force_split || g_cluster_splits == 0)
        return 0;
    return hkv <= 4 ? g_cluster_splits : std::min(8, g_cluster_splits);
}

cudaError_t attn_decode_launch(const AttnArgs &a, cudaStream_t s, bool pdl)
{
    if (a.hkv <= 0 || a.hq % a.hkv != 0 || a.splits <= 0)
        return cudaErrorInvalidValue;
    const int S = attn_cluster_size(a.hkv);
    if (S > 0)
        switch (a.hq / a.hkv)
        {
        case 1: return attn_cluster_launch_t<1>(a, S, s, pdl);
        case 2: return attn_cluster_launch_t<2>(a, S, s, pdl);
        case 3: return attn_cluster_launch_t<3>(a, S, s, pdl);
        case 4: return attn_cluster_launch_t<4>(a, S, s, pdl);
        case 5: return attn_cluster_launch_t<5>(a, S, s, pdl);
        case 6: return attn_cluster_launch_t<6>(a, S, s, pdl);
        case 7: return attn_cluster_launch_t<7>(a, S, s, pdl);
        case 8: return attn_cluster_launch_t<8>(a, S, s, pdl);
        default: return cudaErrorInvalidValue;
        }
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
