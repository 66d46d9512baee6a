// The whole decode-step forward in one cooperative kernel: for every layer the
// QKV projection (RMSNorm prologue, embedding gather on layer 0), attention
// with q/k-norm, RoPE and the KV append, the O projection with its residual
// add, gate-up with SwiGLU, down with its residual add, and finally the
// lm_head. It replaces the per-op chain of src/models/ModelBase.cpp:566-586
// (decode branch of ModelBase::Infer) -> ModelBase::Forward (:403-466) ->
// per-layer attention / FFN (:724-838) with one launch per token.
//
// Why one kernel: at batch 1 each projection is a GEMV that streams its
// weights once. Run as separate launches, every one of the ~5 x layers
// kernels starts cold (launch, first-load latency, tail), which costs several
// microseconds per weight matrix. Here one CTA per SM stays resident for the
// whole step; consecutive projections are separated by a grid-wide barrier
// (one arrival counter per phase), and each warp keeps the next DS_D - 1
// tasks' weights in flight in registers, including the first tasks of the
// next projection while the barrier is pending: weights do not depend on the
// activations, so their HBM reads never wait for the barrier.
//
// The projections reproduce the per-op kernels bit for bit: the GEMV tasks
// (one row x 2048 columns, FP32 fused multiply-adds in column order, warp
// butterfly, per-row chunk sums in order), the RMSNorm sum order and the
// epilogue roundings are the same. Attention computes the same softmax with
// another summation order (whole tokens per warp, grouped rescaling), so its
// FP16 output can differ from attn_decode_kernel's in the last bit.
//
// Data produced inside the launch (qkv, the attention output, the residual
// stream, the SwiGLU activations, attention partials) is read through L2 only
// (ld.global.cg), since an SM's L1 may still hold the previous layer's values
// at the same addresses. Weights, norms, the embedding and cached K/V of
// earlier steps are constant during the launch and use the streaming path.
//
// The barrier counters are never reset: launch n (n = *gen at entry) waits
// until a phase's counter reaches C * (n + 1); CTA 0 increments *gen at exit.
// Every wait is bounded (YLM_WAIT_LIMIT_NS) and records
// YLM_DEV_ERR_TIMEOUT_PEER in the step state's error word; the host then
// resets the counters.
#include "ylm_common.cuh"
#include "ylm_kernels.h"
#include <algorithm>

namespace ylm {

constexpr int DS_THREADS = 384; // 12 warps: 168 registers per thread, no spills
constexpr int DS_WARPS = DS_THREADS / 32;
constexpr int DS_U = 8;              // 16-byte vectors per lane per task
constexpr int DS_KC = 32 * 8 * DS_U; // columns per task (2048)
constexpr int DS_D = 3;              // register ring: DS_D - 1 tasks in flight per warp
constexpr int DS_ATT_UT = 4;         // attention tokens in flight per warp
constexpr int DS_ATT_ROW = 2 + YLM_HEAD_DIM;
constexpr int DS_ATT_MIN_SPLIT = 32; // tokens per split, at least
constexpr float DS_ATT_SCALE_LOG2 = 0.08838834764831845f * 1.4426950408889634f;

struct DsTab
{
    int r0, rows, nkc, ntask; // this CTA's rows of one GEMV phase
};

__device__ __forceinline__ uint4 ds_ldg_stream(const void *p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 ds_ldcg16(const void *p)
{
    uint4 v;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// fp16 x fp16 + fp32 with one rounding: the same value as
// fmaf(float(w), float(x), acc), without the two conversions
__device__ __forceinline__ float ds_dot8(uint4 w, uint4 x, float acc)
{
    const uint32_t *pw = reinterpret_cast<const uint32_t *>(&w);
    const uint32_t *px = reinterpret_cast<const uint32_t *>(&x);
#pragma unroll
    for (int i = 0; i < 4; i++)
        asm("{\n\t.reg .f16 wl, wh, xl, xh;\n\tmov.b32 {wl, wh}, %1;\n\tmov.b32 {xl, xh}, %2;\n\t"
            "fma.rn.f32.f16 %0, wl, xl, %0;\n\tfma.rn.f32.f16 %0, wh, xh, %0;\n\t}"
            : "+f"(acc)
            : "r"(pw[i]), "r"(px[i]));
    return acc;
}

// ------------------------------------------------------------ grid barrier
__device__ __forceinline__ void ds_arrive(const DsArgs &a, int i, int tid)
{
    named_bar_sync(1, DS_THREADS); // every thread's writes of phase i are done
    if (tid == 0)
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar + i) : "memory");
}

__device__ __forceinline__ void ds_poll(const DsArgs &a, int i, unsigned target)
{
    uint64_t t0 = 0;
    for (int n = 0;; n++)
    {
        unsigned v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.bar + i) : "memory");
        if ((int)(v - target) >= 0)
            break;
        if (n == 0)
            t0 = globaltimer_ns();
        else if ((n & 63) == 0)
        {
            // after any error (an earlier expired wait included) give up at
            // once, so a failed step ends in one wait limit, not one per phase
            if (*reinterpret_cast<volatile int *>(a.err) != 0)
                break;
            if (globaltimer_ns() - t0 > YLM_WAIT_LIMIT_NS)
            {
                atomicExch(a.err, YLM_DEV_ERR_TIMEOUT_PEER);
                break;
            }
        }
    }
}

__device__ __forceinline__ void ds_wait(const DsArgs &a, int i, unsigned target, int tid)
{
    if (tid == 0)
        ds_poll(a, i, target);
    named_bar_sync(1, DS_THREADS);
}

// The same wait for a thread that also has cp.async copies in flight (`drain`):
// they complete while thread 0 polls, before the closing barrier publishes them.
__device__ __forceinline__ void ds_wait_drain(const DsArgs &a, int i, unsigned target, int tid, bool drain)
{
    if (tid == 0)
        ds_poll(a, i, target);
    if (drain)
        asm volatile("cp.async.wait_all;" ::: "memory");
    named_bar_sync(1, DS_THREADS);
}

// ------------------------------------------------------------ GEMV phases
// Input vector of phase p into shared memory (all threads). The RMSNorm sum
// runs on threads 0-255 with the per-op kernel's order. `xr`: this CTA's rows
// of the residual stream (see ds_epilogue).
__device__ __forceinline__ void ds_prologue(const DsArgs &a, const DsPhase &p, int kpad, __half *xs, float *red,
                                            __half *xr, int tid)
{
    const int K = p.K;
    const int warp = tid >> 5, lane = tid & 31;
    if (p.pro == PRO_VEC)
    {
        for (int i = tid * 8; i < kpad; i += DS_THREADS * 8)
            *reinterpret_cast<uint4 *>(xs + i) = i < K ? ds_ldcg16(p.x + i) : make_uint4(0, 0, 0, 0);
        named_bar_sync(1, DS_THREADS);
        return;
    }
    // raw input into shared memory (one global round trip), then the norm in place
    const __half *src = p.x;
    const bool from_emb = p.pro == PRO_EMBED_RMSNORM;
    if (from_emb)
    {
        int64_t tok = a.state->token;
        if (tok < 0 || tok >= a.vocab)
        {
            if (tid == 0)
                atomicExch(a.err, YLM_DEV_ERR_BAD_TOKEN);
            tok = 0;
        }
        src = a.emb + tok * (int64_t)K;
    }
    for (int i = tid * 8; i < kpad; i += DS_THREADS * 8)
    {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (i < K)
            v = from_emb ? *reinterpret_cast<const uint4 *>(src + i) : ds_ldcg16(src + i);
        *reinterpret_cast<uint4 *>(xs + i) = v;
    }
    named_bar_sync(1, DS_THREADS);
    if (from_emb)
    {
        // this CTA's rows of the residual stream start as the embedding row:
        // the global copy (read by every CTA's RMSNorm) and the CTA's own copy
        const int xr0 = (int)((long long)a.hidden * blockIdx.x / gridDim.x);
        const int xrn = (int)((long long)a.hidden * (blockIdx.x + 1) / gridDim.x) - xr0;
        for (int r = tid; r < xrn; r += DS_THREADS)
        {
            const __half v = xs[xr0 + r];
            xr[r] = v;
            p.resid[xr0 + r] = v;
        }
    }
    // sum of squares on threads 0-255 in the per-op kernel's order
    if (tid < 256)
    {
        float ss = 0.f;
        for (int i = tid * 8; i < K; i += 256 * 8)
        {
            const uint4 v = *reinterpret_cast<const uint4 *>(xs + i);
            const uint32_t *vw = reinterpret_cast<const uint32_t *>(&v);
#pragma unroll
            for (int e = 0; e < 4; e++)
            {
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(vw + e));
                ss += rh(f.x * f.x);
                ss += rh(f.y * f.y);
            }
        }
        ss = warp_sum(ss);
        if (lane == 0)
            red[warp] = ss;
    }
    named_bar_sync(1, DS_THREADS);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; w++)
        tot += red[w];
    const float mean = rh(tot * (1.0f / (float)K));
    const float d = rh(rsqrtf(mean + a.eps));
    for (int i = tid * 8; i < K; i += DS_THREADS * 8)
    {
        const uint4 v = *reinterpret_cast<const uint4 *>(xs + i);
        const uint4 wv = *reinterpret_cast<const uint4 *>(p.norm_w + i);
        const uint32_t *vw = reinterpret_cast<const uint32_t *>(&v);
        const uint32_t *ww = reinterpret_cast<const uint32_t *>(&wv);
        uint4 o;
        uint32_t *ow = reinterpret_cast<uint32_t *>(&o);
#pragma unroll
        for (int e = 0; e < 4; e++)
        {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(vw + e));
            const float2 w = __half22float2(*reinterpret_cast<const __half2 *>(ww + e));
            const __half2 r = __halves2half2(f2h(rh(f.x * d) * w.x), f2h(rh(f.y * d) * w.y));
            ow[e] = *reinterpret_cast<const uint32_t *>(&r);
        }
        *reinterpret_cast<uint4 *>(xs + i) = o;
    }
    named_bar_sync(1, DS_THREADS);
}

// Row sums of the chunk partials in order, then the epilogue of the per-op kernel.
__device__ __forceinline__ void ds_epilogue(const DsPhase &p, const DsTab &t, const float *part, __half *xr,
                                            int hidden, int tid)
{
    named_bar_sync(1, DS_THREADS); // all partials of the phase are in shared memory
    if (p.epi == EPI_SWIGLU)
    {
        for (int q = tid; q < t.rows / 2; q += DS_THREADS)
        {
            float gs = 0.f, us = 0.f;
            for (int c = 0; c < t.nkc; c++)
            {
                gs += part[(2 * q) * t.nkc + c];
                us += part[(2 * q + 1) * t.nkc + c];
            }
            const float g = rh(gs), u = rh(us);
            const float sg = rh(g / (1.0f + expf(-g)));
            p.out[(t.r0 + 2 * q) >> 1] = f2h(sg * u);
        }
        return;
    }
    for (int r = tid; r < t.rows; r += DS_THREADS)
    {
        float y = 0.f;
        for (int c = 0; c < t.nkc; c++)
            y += part[r * t.nkc + c];
        const int row = t.r0 + r;
        if (p.epi == EPI_STORE)
        {
            if (p.bias)
                y = rh(y) + h2f(p.bias[row]);
            p.out[row] = f2h(y);
        }
        else if (p.N == hidden)
        {
            // residual stream: every residual phase has N = H and the same row
            // split, so this CTA alone updates these rows and keeps them in
            // shared memory (its layer-0 prologue seeded them)
            const __half v = f2h(h2f(xr[r]) + rh(y));
            xr[r] = v;
            p.resid[row] = v;
        }
        else
            p.resid[row] = f2h(h2f(__ldcg(p.resid + row)) + rh(y));
    }
}

// A run of consecutive GEMV phases [i0, i1). Each warp walks its task stream
// (phase, task = warp, warp + 16, ...) with a ring of DS_D register buffers
// whose roles are fixed by unrolling, so a buffer is never copied while its
// loads are in flight. `pending`: the barrier of phase i0 - 1 has been arrived
// at but not waited for; the first loads are issued before that wait. The
// barrier of the last phase is left pending for the caller.
__device__ __forceinline__ void ds_segment(const DsArgs &a, int i0, int i1, bool pending, const DsTab *tab,
                                           __half *xs, float *part, float *red, __half *xr, unsigned target, int tid)
{
    const int warp = tid >> 5, lane = tid & 31;
    int pp = i0, pt = warp; // prefetch cursor
    while (pp < i1 && pt >= tab[pp].ntask)
    {
        pp++;
        pt = warp;
    }
    int cp = pp, ct = pt; // compute cursor
    uint4 buf[DS_D][DS_U];
    auto load = [&](uint4 *w) {
        if (pp >= i1)
            return;
        const DsTab &t = tab[pp];
        const DsPhase &p = a.ph[pp];
        const int row = t.r0 + pt / t.nkc, kc = pt % t.nkc;
        const __half *base = p.w + (size_t)row * p.K + kc * DS_KC + lane * 8;
        const int lim = p.K - kc * DS_KC - lane * 8;
#pragma unroll
        for (int u = 0; u < DS_U; u++)
            w[u] = u * 256 < lim ? ds_ldg_stream(base + u * 256) : make_uint4(0, 0, 0, 0);
        pt += DS_WARPS;
        while (pp < i1 && pt >= tab[pp].ntask)
        {
            pp++;
            pt = warp;
        }
    };
#pragma unroll
    for (int d = 0; d < DS_D - 1; d++)
        load(buf[d]);
    if (pending)
        ds_wait(a, i0 - 1, target, tid);
    int cur = i0;
    ds_prologue(a, a.ph[cur], tab[cur].nkc * DS_KC, xs, red, xr, tid);
    // finish phase `cur` (every warp is past its tasks) and open the next one
    auto advance = [&]() {
        ds_epilogue(a.ph[cur], tab[cur], part, xr, a.hidden, tid);
        ds_arrive(a, cur, tid);
        if (cur + 1 < i1)
            ds_wait(a, cur, target, tid);
        cur++;
        if (cur < i1)
            ds_prologue(a, a.ph[cur], tab[cur].nkc * DS_KC, xs, red, xr, tid);
    };
    for (;;)
    {
#pragma unroll
        for (int d = 0; d < DS_D; d++)
        {
            while (cur < cp && cur < i1)
                advance();
            if (cp >= i1)
                goto done;
            load(buf[(d + DS_D - 1) % DS_D]);
            {
                const DsTab &t = tab[cp];
                const int kc = ct % t.nkc;
                const __half *xk = xs + kc * DS_KC + lane * 8;
                float acc = 0.f;
#pragma unroll
                for (int u = 0; u < DS_U; u++)
                    acc = ds_dot8(buf[d][u], *reinterpret_cast<const uint4 *>(xk + u * 256), acc);
                acc = warp_sum(acc);
                if (lane == 0)
                    part[ct] = acc; // slot (row ct / nkc, chunk ct % nkc)
                ct += DS_WARPS;
                while (cp < i1 && ct >= tab[cp].ntask)
                {
                    cp++;
                    ct = warp;
                }
            }
        }
    }
done:
    while (cur < i1)
        advance();
}

// ------------------------------------------------------------ attention
// One warp prepares one head: optional per-head RMSNorm, then RoPE at the
// step's position (the math of attention.cu's prep_head, reading qkv via L2).
// Lane l holds elements 4l..4l+3; rope = [cos(64), sin(64)] of the step's
// position and nw the norm weights, staged in shared memory.
__device__ __forceinline__ void ds_prep_head(const __half *src, bool norm, const __half *nw, float eps,
                                             const __half *rope, float *dst, int lane)
{
    float x[4];
    {
        const uint2 raw = __ldcg(reinterpret_cast<const uint2 *>(src + lane * 4));
        const __half2 *s2 = reinterpret_cast<const __half2 *>(&raw);
        const float2 a = __half22float2(s2[0]), b = __half22float2(s2[1]);
        x[0] = a.x;
        x[1] = a.y;
        x[2] = b.x;
        x[3] = b.y;
    }
    if (norm)
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
            x[e] = rh(rh(x[e] * d) * h2f(nw[lane * 4 + e]));
    }
    float px[4];
#pragma unroll
    for (int e = 0; e < 4; e++)
        px[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
#pragma unroll
    for (int e = 0; e < 4; e++)
    {
        const int d = lane * 4 + e;
        const float rot = d < 64 ? -px[e] : px[e];
        dst[d] = rh(rh(x[e] * h2f(rope[d & 63])) + rh(rot * h2f(rope[64 + (d & 63)])));
    }
}

// Attention phase i: unit (KV head g, split sp) = CTA g * S + sp; split-K
// over the cached tokens with the split sizes of attn_decode_kernel. Inside a
// CTA every warp takes whole tokens (lane l holds dimensions 4l..4l+3), so a
// thread keeps 4 values of q and of the output per head; the 16 per-warp
// softmax states are merged through shared memory, and the last split of a
// head (atomic ticket) combines the splits and writes the group's output.
// The first K/V loads (earlier steps' slots, constant) go out before the wait
// for the QKV phase.
// (not inlined: its registers are allocated apart from the GEMV segments',
// which keep the projection loop free of spills)
template <int G>
__device__ __noinline__ void ds_attention(const DsArgs &a, int i, bool pending, uint8_t *work, unsigned target,
                                             int tid)
{
    float *q_s = reinterpret_cast<float *>(work);   // [4][128]
    float *kn_s = q_s + 4 * YLM_HEAD_DIM;           // [128]
    float *vn_s = kn_s + YLM_HEAD_DIM;              // [128]
    float *mrg = vn_s + YLM_HEAD_DIM;               // [16 warps][4][130]
    __half *rope_h = reinterpret_cast<__half *>(mrg + DS_WARPS * 4 * DS_ATT_ROW); // [cos 64 | sin 64]
    __half *nq_h = rope_h + YLM_HEAD_DIM;                                         // [128]
    __half *nk_h = nq_h + YLM_HEAD_DIM;                                           // [128]
    int *ticket = reinterpret_cast<int *>(nk_h + YLM_HEAD_DIM);
    const int warp = tid >> 5, lane = tid & 31;
    const DsLayerAttn la = a.la[a.ph[i].layer];
    const int C = gridDim.x;
    const int S = max(1, min(a.splits, C / a.hkv));
    const int g = blockIdx.x / S, sp = blockIdx.x % S;
    // volatile: read here, not hoisted out of the phase loop (those registers
    // would stay live through the GEMV segments)
    const int slot = *reinterpret_cast<volatile const int *>(&a.state->slot);
    const int pos = *reinterpret_cast<volatile const int *>(&a.state->rope_pos);
    const bool ok_state = slot >= 0 && slot < a.cap && pos >= 0 && pos < a.max_pos;
    if (!ok_state && blockIdx.x == 0 && tid == 0)
        atomicExch(a.err, YLM_DEV_ERR_BAD_STATE);
    const int n = slot + 1;
    const int chunk = max(DS_ATT_MIN_SPLIT, (n + S - 1) / S);
    const int S_eff = (n + chunk - 1) / chunk;
    const bool active = ok_state && blockIdx.x < a.hkv * S && sp < S_eff; // uniform over the CTA
    const int t0 = sp * chunk, t1 = min(n, t0 + chunk);
    const bool owns_new = slot >= t0 && slot < t1;
    const int te = owns_new ? slot : t1; // cached tokens [t0, te); the new one comes from qkv
    const __half *kc = la.kc + (size_t)g * a.cap * YLM_HEAD_DIM + lane * 4;
    const __half *vc = la.vc + (size_t)g * a.cap * YLM_HEAD_DIM + lane * 4;

    // token j of this warp: t0 + warp + 16 * j
    uint2 kr[DS_ATT_UT], vr[DS_ATT_UT];
    auto load_group = [&](int j0) {
#pragma unroll
        for (int u = 0; u < DS_ATT_UT; u++)
        {
            const int t = t0 + warp + DS_WARPS * (j0 + u);
            if (t < te)
            {
                kr[u] = __ldg(reinterpret_cast<const uint2 *>(kc + (size_t)t * YLM_HEAD_DIM));
                vr[u] = __ldg(reinterpret_cast<const uint2 *>(vc + (size_t)t * YLM_HEAD_DIM));
            }
        }
    };
    // RoPE row of this step's position and the per-head norm weights: constant
    // during the step, copied to shared memory asynchronously (cp.async, 16 B
    // per thread of warps 1-2) before the wait, whose closing barrier
    // publishes them
    bool copying = false;
    if (active)
    {
        load_group(0);
        const int k = tid - 32;
        const __half *src = nullptr;
        __half *dst = nullptr;
        if (k >= 0 && k < 8)
        {
            src = a.rope_cos + (size_t)pos * 64 + k * 8;
            dst = rope_h + k * 8;
        }
        else if (k >= 8 && k < 16)
        {
            src = a.rope_sin + (size_t)pos * 64 + (k - 8) * 8;
            dst = rope_h + 64 + (k - 8) * 8;
        }
        else if (k >= 16 && k < 32 && la.qn)
        {
            src = la.qn + (k - 16) * 8;
            dst = nq_h + (k - 16) * 8;
        }
        else if (k >= 32 && k < 48 && la.kn)
        {
            src = la.kn + (k - 32) * 8;
            dst = nk_h + (k - 32) * 8;
        }
        if (src)
        {
            asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
            copying = true;
        }
    }
    if (pending)
        ds_wait_drain(a, i - 1, target, tid, copying);
    else
    {
        if (copying)
            asm volatile("cp.async.wait_all;" ::: "memory");
        named_bar_sync(1, DS_THREADS);
    }

    if (active)
    {
        if (warp < G)
            ds_prep_head(la.qkv + (size_t)(g * G + warp) * YLM_HEAD_DIM, la.qn != nullptr, nq_h, a.eps, rope_h,
                         q_s + warp * YLM_HEAD_DIM, lane);
        else if (owns_new && warp == G)
        {
            ds_prep_head(la.qkv + (size_t)(a.hq + g) * YLM_HEAD_DIM, la.kn != nullptr, nk_h, a.eps, rope_h, kn_s,
                         lane);
            __syncwarp();
            for (int d = lane; d < YLM_HEAD_DIM; d += 32)
                la.kc[((size_t)g * a.cap + slot) * YLM_HEAD_DIM + d] = f2h(kn_s[d]);
        }
        else if (owns_new && warp == G + 1)
        {
            for (int d = lane; d < YLM_HEAD_DIM; d += 32)
            {
                const __half v = __ldcg(la.qkv + (size_t)(a.hq + a.hkv + g) * YLM_HEAD_DIM + d);
                vn_s[d] = h2f(v);
                la.vc[((size_t)g * a.cap + slot) * YLM_HEAD_DIM + d] = v;
            }
        }
        named_bar_sync(1, DS_THREADS);

        float q[G][4], o[G][4], m[G], l[G];
#pragma unroll
        for (int h = 0; h < G; h++)
        {
#pragma unroll
            for (int e = 0; e < 4; e++)
            {
                q[h][e] = q_s[h * YLM_HEAD_DIM + lane * 4 + e] * DS_ATT_SCALE_LOG2;
                o[h][e] = 0.f;
            }
            m[h] = -INFINITY;
            l[h] = 0.f;
        }
        // one token: sequential online-softmax update (used for the new token)
        auto token = [&](const float *kf, const float *vf) {
#pragma unroll
            for (int h = 0; h < G; h++)
            {
                float sc = 0.f;
#pragma unroll
                for (int e = 0; e < 4; e++)
                    sc = fmaf(q[h][e], kf[e], sc);
                sc = warp_sum(sc);
                const float mn = fmaxf(m[h], sc);
                const float cs = exp2f(m[h] - mn);
                const float ps = exp2f(sc - mn);
                l[h] = l[h] * cs + ps;
#pragma unroll
                for (int e = 0; e < 4; e++)
                    o[h][e] = o[h][e] * cs + ps * vf[e];
                m[h] = mn;
            }
        };
        // a group of DS_ATT_UT cached tokens: all scores first (independent dot
        // products and reductions), then one rescale of the running state
        const int ntok = max(0, te - t0 - warp);
        const int per_w = (ntok + DS_WARPS - 1) / DS_WARPS; // this warp's tokens
        for (int j0 = 0; j0 < per_w; j0 += DS_ATT_UT)
        {
            uint2 kcur[DS_ATT_UT], vcur[DS_ATT_UT];
#pragma unroll
            for (int u = 0; u < DS_ATT_UT; u++)
            {
                kcur[u] = kr[u];
                vcur[u] = vr[u];
            }
            if (j0 + DS_ATT_UT < per_w)
                load_group(j0 + DS_ATT_UT);
            float sc[DS_ATT_UT][G];
#pragma unroll
            for (int u = 0; u < DS_ATT_UT; u++)
            {
                float kf[4];
                const __half2 *k2 = reinterpret_cast<const __half2 *>(&kcur[u]);
                const float2 ka = __half22float2(k2[0]), kb = __half22float2(k2[1]);
                kf[0] = ka.x;
                kf[1] = ka.y;
                kf[2] = kb.x;
                kf[3] = kb.y;
#pragma unroll
                for (int h = 0; h < G; h++)
                {
                    float t = 0.f;
#pragma unroll
                    for (int e = 0; e < 4; e++)
                        t = fmaf(q[h][e], kf[e], t);
                    sc[u][h] = t;
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int u = 0; u < DS_ATT_UT; u++)
#pragma unroll
                    for (int h = 0; h < G; h++)
                        sc[u][h] += __shfl_xor_sync(0xffffffffu, sc[u][h], off);
#pragma unroll
            for (int h = 0; h < G; h++)
            {
                float mx = m[h];
#pragma unroll
                for (int u = 0; u < DS_ATT_UT; u++)
                    if (j0 + u < per_w)
                        mx = fmaxf(mx, sc[u][h]);
                const float cs = exp2f(m[h] - mx);
                l[h] *= cs;
#pragma unroll
                for (int e = 0; e < 4; e++)
                    o[h][e] *= cs;
#pragma unroll
                for (int u = 0; u < DS_ATT_UT; u++)
                    if (j0 + u < per_w)
                    {
                        const float ps = exp2f(sc[u][h] - mx);
                        const __half2 *v2 = reinterpret_cast<const __half2 *>(&vcur[u]);
                        const float2 va = __half22float2(v2[0]), vb = __half22float2(v2[1]);
                        l[h] += ps;
                        o[h][0] += ps * va.x;
                        o[h][1] += ps * va.y;
                        o[h][2] += ps * vb.x;
                        o[h][3] += ps * vb.y;
                    }
                m[h] = mx;
            }
        }
        if (owns_new && warp == 0)
        {
            float kf[4], vf[4];
#pragma unroll
            for (int e = 0; e < 4; e++)
            {
                kf[e] = kn_s[lane * 4 + e];
                vf[e] = vn_s[lane * 4 + e];
            }
            token(kf, vf);
        }
        // per-warp states -> shared memory, merged per (head, dimension)
#pragma unroll
        for (int h = 0; h < G; h++)
        {
            float *row = mrg + (warp * 4 + h) * DS_ATT_ROW;
            if (lane == 0)
            {
                row[0] = m[h];
                row[1] = l[h];
            }
#pragma unroll
            for (int e = 0; e < 4; e++)
                row[2 + lane * 4 + e] = o[h][e];
        }
        named_bar_sync(1, DS_THREADS);
        for (int k = tid; k < G * YLM_HEAD_DIM; k += DS_THREADS)
        {
            const int hh = k >> 7, d = k & 127; // (head, dimension)
            float M = -INFINITY;
            for (int w = 0; w < DS_WARPS; w++)
                M = fmaxf(M, mrg[(w * 4 + hh) * DS_ATT_ROW]);
            float L = 0.f, O = 0.f;
            if (M != -INFINITY)
                for (int w = 0; w < DS_WARPS; w++)
                {
                    const float *row = mrg + (w * 4 + hh) * DS_ATT_ROW;
                    const float cw = exp2f(row[0] - M);
                    L += row[1] * cw;
                    O += row[2 + d] * cw;
                }
            float *pr = a.partial + ((size_t)(g * G + hh) * S + sp) * DS_ATT_ROW;
            pr[2 + d] = O;
            if (d == 0)
            {
                pr[0] = M;
                pr[1] = L;
            }
        }
        // ticket with release/acquire semantics: the barrier orders this CTA's
        // partial writes before thread 0's release, and the last split's
        // acquire (then the barrier) orders every split's partials before its reads
        named_bar_sync(1, DS_THREADS);
        if (tid == 0)
        {
            int t;
            asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(t) : "l"(a.counters + g) : "memory");
            *ticket = t;
        }
        named_bar_sync(1, DS_THREADS);
        if (*ticket == S_eff - 1)
        {
            // last split of this KV head: fetch every split's partial of the
            // group with one parallel load (the merge buffer is free now), then
            // combine per (head, dimension)
            const int rowsn = G * S_eff;
            const bool staged = rowsn * DS_ATT_ROW <= DS_WARPS * 4 * DS_ATT_ROW;
            if (staged)
            {
                for (int k = tid; k < rowsn * DS_ATT_ROW; k += DS_THREADS)
                {
                    const int r = k / DS_ATT_ROW, e = k - r * DS_ATT_ROW;
                    const int hh = r / S_eff, sv = r - hh * S_eff;
                    mrg[k] = __ldcg(a.partial + ((size_t)(g * G + hh) * S + sv) * DS_ATT_ROW + e);
                }
                named_bar_sync(1, DS_THREADS);
            }
            for (int k = tid; k < G * YLM_HEAD_DIM; k += DS_THREADS)
            {
                const int hh = k >> 7, d = k & 127;
                const float *base = staged ? mrg + (size_t)hh * S_eff * DS_ATT_ROW
                                           : a.partial + (size_t)(g * G + hh) * S * DS_ATT_ROW;
                float M = -INFINITY;
                for (int sv = 0; sv < S_eff; sv++)
                    M = fmaxf(M, staged ? base[sv * DS_ATT_ROW] : __ldcg(base + (size_t)sv * DS_ATT_ROW));
                float L = 0.f, O = 0.f;
                for (int sv = 0; sv < S_eff; sv++)
                {
                    const float *pr = base + (size_t)sv * DS_ATT_ROW;
                    const float ms = staged ? pr[0] : __ldcg(pr);
                    const float cs = ms == -INFINITY ? 0.f : exp2f(ms - M);
                    L += (staged ? pr[1] : __ldcg(pr + 1)) * cs;
                    O += (staged ? pr[2 + d] : __ldcg(pr + 2 + d)) * cs;
                }
                la.out[(size_t)(g * G + hh) * YLM_HEAD_DIM + d] = f2h(O / L);
            }
            if (tid == 0)
                a.counters[g] = 0;
        }
    }
    ds_arrive(a, i, tid);
}

// ------------------------------------------------------------ the kernel
template <int G>
__global__ void __launch_bounds__(DS_THREADS, 1) decode_step_kernel(const DsArgs a)
{
    extern __shared__ __align__(16) uint8_t smem[];
    DsTab *tab = reinterpret_cast<DsTab *>(smem);
    uint8_t *work = smem + a.tab_bytes;
    __half *xs = reinterpret_cast<__half *>(work);
    float *part = reinterpret_cast<float *>(work + (size_t)a.kpad_max * 2);
    float *red = part + a.part_max;
    __half *xr = reinterpret_cast<__half *>(smem + a.tab_bytes + a.work_bytes); // this CTA's residual rows
    const int tid = threadIdx.x, C = gridDim.x, c = blockIdx.x;
    const unsigned gen = *reinterpret_cast<volatile const unsigned *>(a.gen);
    const unsigned target = (unsigned)C * (gen + 1u);

    for (int i = tid; i < a.nph; i += DS_THREADS)
    {
        const DsPhase &p = a.ph[i];
        DsTab t = {0, 0, 1, 0};
        if (p.kind == DS_GEMV)
        {
            if (p.epi == EPI_SWIGLU)
            {
                const long long np = p.N / 2;
                const int q0 = (int)(np * c / C), q1 = (int)(np * (c + 1) / C);
                t.r0 = 2 * q0;
                t.rows = 2 * (q1 - q0);
            }
            else
            {
                t.r0 = (int)((long long)p.N * c / C);
                t.rows = (int)((long long)p.N * (c + 1) / C) - t.r0;
            }
            t.nkc = (p.K + DS_KC - 1) / DS_KC;
            t.ntask = t.rows * t.nkc;
        }
        tab[i] = t;
    }
    __syncthreads();

    int i = 0;
    bool pending = false;
    while (i < a.nph)
    {
        if (a.ph[i].kind == DS_ATTN)
        {
            ds_attention<G>(a, i, pending, work, target, tid);
            pending = true;
            i++;
            continue;
        }
        int j = i;
        while (j < a.nph && a.ph[j].kind == DS_GEMV)
            j++;
        ds_segment(a, i, j, pending, tab, xs, part, red, xr, target, tid);
        pending = true;
        i = j;
    }
    // every CTA has arrived at the second-to-last phase, so all have read *gen
    if (c == 0 && tid == 0)
        *a.gen = gen + 1u;
}

// ------------------------------------------------------------ host side
size_t ds_attn_smem_bytes()
{
    return (size_t)(4 * YLM_HEAD_DIM + 2 * YLM_HEAD_DIM + DS_WARPS * 4 * DS_ATT_ROW + 3 * YLM_HEAD_DIM) *
               sizeof(float) +
           16;
}

int ds_max_heads_per_group() { return 4; }

int ds_threads() { return DS_THREADS; }

int ds_task_cols() { return DS_KC; }

template <int G> static cudaError_t ds_prepare_t(size_t smem)
{
    return cudaFuncSetAttribute(decode_step_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

template <int G> static void *ds_fn() { return reinterpret_cast<void *>(decode_step_kernel<G>); }

static void *ds_kernel_for(int G)
{
    switch (G)
    {
    case 1: return ds_fn<1>();
    case 2: return ds_fn<2>();
    case 3: return ds_fn<3>();
    case 4: return ds_fn<4>();
    default: return nullptr;
    }
}

cudaError_t ds_prepare(int G, size_t smem, int *blocks_per_sm)
{
    cudaError_t e = cudaErrorInvalidValue;
    switch (G)
    {
    case 1: e = ds_prepare_t<1>(smem); break;
    case 2: e = ds_prepare_t<2>(smem); break;
    case 3: e = ds_prepare_t<3>(smem); break;
    case 4: e = ds_prepare_t<4>(smem); break;
    default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess)
        return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, ds_kernel_for(G), DS_THREADS, smem);
}

cudaError_t ds_launch(const DsArgs &a, int G, size_t smem, int grid, cudaStream_t s)
{
    void *fn = ds_kernel_for(G);
    if (!fn)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(DS_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {const_cast<DsArgs *>(&a)};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

} // namespace ylm
