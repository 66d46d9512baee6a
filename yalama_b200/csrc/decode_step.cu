// The projections of a decode step as persistent GEMV segments. Between two
// attention launches a decode step is a chain of matrix-vector products that
// each need the whole output of the previous one: O projection (+ residual),
// gate-up (RMSNorm prologue, SwiGLU epilogue), down (+ residual), and the
// next layer's QKV (RMSNorm prologue; on layer 0 the embedding gather); the
// last segment ends with the lm_head. They replace the per-op chain of
// src/models/ModelBase.cpp:566-586 (decode branch of ModelBase::Infer) ->
// ModelBase::Forward (:403-466) -> per-layer attention / FFN (:724-838); the
// attention between segments is attn_cluster_kernel (attention.cu).
//
// Why persistent: at batch 1 each projection is a GEMV that streams its
// weights once. Run as separate launches, every kernel starts cold (launch,
// first-load latency, tail), several microseconds per weight matrix. Here one
// CTA per SM stays resident for a whole segment, and each warp keeps the next
// DS_D - 1 tasks' weights in flight in registers, including the first tasks
// of the next projection while that projection's input is not ready yet:
// weights do not depend on the activations, so their HBM reads never wait.
// (Attention stays a separate kernel: folded into this one, its registers
// pushed the GEMV loop into spills and slowed every phase.)
//
// Activations inside a segment carry their own readiness. The residual stream
// and the SwiGLU activations are 32-bit words, FP16 value in the low half and
// a tag in the high half naming the step and the phase that wrote it; a
// prologue polls exactly the words it needs until their tags match (one L2
// round trip after the producer's store), with no grid barrier between
// phases. Every phase consumes the whole output of the previous one, so by the
// time a CTA writes a buffer again, every CTA has finished reading it (each
// reader wrote an output of a later phase that the writer consumed).
//
// The projections reproduce the per-op kernels bit for bit: the GEMV tasks
// (one row x 2048 columns, FP32 fused multiply-adds in column order, warp
// butterfly, per-row chunk sums in order), the RMSNorm sum order and the
// epilogue roundings are the same.
//
// Weights, norms and the embedding are constant and use the streaming path;
// activations are read through L2 only (ld.global.cg). Every wait is bounded
// (DsArgs::wait_ns, 2 s unless the engine sets it) and records YLM_DEV_ERR_TIMEOUT_PEER in the step
// state's error word; after any recorded error the remaining waits give up at
// once, and the host clears the tagged buffers.
//
// With tensor parallelism the O and down projections end in an all-reduce
// fused into their epilogue: each CTA stores its partial rows, tagged, into
// every rank's mailbox over NVLink (plain peer stores), then sums its rows of
// all ranks' partials from its own mailbox and adds the residual. O and down
// use separate mailbox sets: a rank can only reach the next layer's O after
// receiving every peer's down partials, which each peer sends after reading
// its O mailbox, so no slot is overwritten before it is read.
#include "ylm_common.cuh"
#include "ylm_kernels.h"
#include <algorithm>

namespace ylm {

#ifndef DS_U_OPT
#define DS_U_OPT 8
#endif
#ifndef DS_D_OPT
#define DS_D_OPT 3
#endif
#ifndef DS_THREADS_OPT
#define DS_THREADS_OPT 384
#endif
constexpr int DS_THREADS = DS_THREADS_OPT; // 12 warps, one CTA per SM (168 registers per thread)
constexpr int DS_WARPS = DS_THREADS / 32;
constexpr int DS_U = DS_U_OPT;       // 16-byte vectors per lane per task
constexpr int DS_KC = 32 * 8 * DS_U; // columns per task
constexpr int DS_D = DS_D_OPT;       // register ring: DS_D - 1 tasks in flight per warp
static_assert(DS_U % 4 == 0, "four accumulators per lane");

// This CTA's share of one GEMV phase, and the steps of a warp's task cursor
// (tasks t = warp, warp + DS_WARPS, ...; task t is row r0 + t / nkc, chunk
// t % nkc), so the task loop needs no division.
struct DsTab
{
    const __half *w; // the phase's weights [N, K]
    int K, nkc;      // columns, DS_KC-column chunks per row
    int r0, rows;    // this CTA's rows
    int drow, dkc;   // DS_WARPS tasks = drow rows + dkc chunks
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

// ------------------------------------------------------------ shared memory
// [this CTA's table of the launch's phases | work area (GEMV input, partials,
// RMSNorm scratch) | this CTA's residual rows].
extern __shared__ __align__(16) uint8_t ds_smem[];

struct DsSmem
{
    DsTab *tab;
    __half *xs;
    float *part, *red;
    __half *xr;
};

__device__ __forceinline__ DsSmem ds_smem_map(const DsArgs &a)
{
    DsSmem m;
    m.tab = reinterpret_cast<DsTab *>(ds_smem);
    uint8_t *work = ds_smem + a.tab_bytes;
    m.xs = reinterpret_cast<__half *>(work);
    m.part = reinterpret_cast<float *>(work + (size_t)a.kpad_max * 2);
    m.red = m.part + a.part_max;
    m.xr = reinterpret_cast<__half *>(ds_smem + a.tab_bytes + a.work_bytes);
    return m;
}

// ------------------------------------------------------------ tagged activations
// The tag of phase q in step `gen`: distinct for every phase of a step and
// between consecutive steps (a word is rewritten at least once per step).
__device__ __forceinline__ uint32_t ds_tag(unsigned gen, int nph, int q)
{
    return ((gen * (unsigned)nph + (unsigned)q + 1u) & 0xffffu) << 16;
}

__device__ __forceinline__ uint32_t ds_tagged(uint32_t tag, __half v)
{
    return tag | (uint32_t)__half_as_ushort(v);
}

// 8 tagged words at w (16-byte aligned) -> 8 halves, once every tag is `want`.
// Bounded: after a.wait_ns, or at once after any recorded error, the
// current words are used.
__device__ __forceinline__ uint4 ds_read_tagged8(const DsArgs &a, const uint32_t *w, uint32_t want)
{
    uint4 lo = ds_ldcg16(w), hi = ds_ldcg16(w + 4);
    auto ready = [&]() {
        return ((lo.x & 0xffff0000u) == want) & ((lo.y & 0xffff0000u) == want) & ((lo.z & 0xffff0000u) == want) &
               ((lo.w & 0xffff0000u) == want) & ((hi.x & 0xffff0000u) == want) & ((hi.y & 0xffff0000u) == want) &
               ((hi.z & 0xffff0000u) == want) & ((hi.w & 0xffff0000u) == want);
    };
    if (!ready())
    {
        const uint64_t t0 = globaltimer_ns();
        for (int n = 1;; n++)
        {
            // back off: every waiting thread of every CTA polls, and those L2
            // reads compete with the weight stream
            __nanosleep(256);
            lo = ds_ldcg16(w);
            hi = ds_ldcg16(w + 4);
            if (ready())
                break;
            if ((n & 31) == 0)
            {
                if (*reinterpret_cast<volatile int *>(a.err) != 0)
                    break;
                if (globaltimer_ns() - t0 > a.wait_ns)
                {
                    atomicExch(a.err, YLM_DEV_ERR_TIMEOUT_PEER);
                    break;
                }
            }
        }
    }
    uint4 o;
    o.x = (lo.x & 0xffffu) | (lo.y << 16);
    o.y = (lo.z & 0xffffu) | (lo.w << 16);
    o.z = (hi.x & 0xffffu) | (hi.y << 16);
    o.w = (hi.z & 0xffffu) | (hi.w << 16);
    return o;
}

// One tagged word (a peer's partial in this rank's mailbox) -> its half.
__device__ __forceinline__ __half ds_read_tagged1(const DsArgs &a, const uint32_t *w, uint32_t want)
{
    uint32_t v = __ldcg(w);
    if ((v & 0xffff0000u) != want)
    {
        const uint64_t t0 = globaltimer_ns();
        for (int n = 1;; n++)
        {
            __nanosleep(256);
            v = __ldcg(w);
            if ((v & 0xffff0000u) == want)
                break;
            if ((n & 31) == 0)
            {
                if (*reinterpret_cast<volatile int *>(a.err) != 0)
                    break;
                if (globaltimer_ns() - t0 > a.wait_ns)
                {
                    atomicExch(a.err, YLM_DEV_ERR_TIMEOUT_PEER);
                    break;
                }
            }
        }
    }
    return __ushort_as_half((unsigned short)(v & 0xffffu));
}

// ------------------------------------------------------------ GEMV phases
// Input vector of phase p into shared memory (all threads): polled from the
// tagged words a previous phase of this launch wrote, or loaded from an
// untagged buffer a previous launch wrote, or gathered from the embedding.
// The RMSNorm sum runs on threads 0-255 with the per-op kernel's order. `xr`:
// this CTA's rows of the residual stream (see ds_epilogue).
__device__ __forceinline__ void ds_prologue(const DsArgs &a, const DsPhase &p, int q, int kpad, unsigned gen,
                                            __half *xs, float *red, __half *xr, int tid)
{
    const int K = p.K;
    const int warp = tid >> 5, lane = tid & 31;
    const bool from_emb = p.pro == PRO_EMBED_RMSNORM;
    const __half *src = p.x;
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
    const uint32_t want = p.xt ? ds_tag(gen, a.nph, p.src) : 0u;
    for (int i = tid * 8; i < kpad; i += DS_THREADS * 8)
    {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (i < K)
        {
            if (p.xt)
                v = ds_read_tagged8(a, p.xt + i, want);
            else if (from_emb)
                v = *reinterpret_cast<const uint4 *>(src + i);
            else
                v = ds_ldcg16(src + i);
        }
        *reinterpret_cast<uint4 *>(xs + i) = v;
    }
    named_bar_sync(1, DS_THREADS);
    if (from_emb)
    {
        // this CTA's rows of the residual stream start as the embedding row:
        // its own copy, and the tagged words the next segment seeds from
        const uint32_t tag = ds_tag(gen, a.nph, q);
        const int xr0 = (int)((long long)a.hidden * blockIdx.x / gridDim.x);
        const int xrn = (int)((long long)a.hidden * (blockIdx.x + 1) / gridDim.x) - xr0;
        for (int r = tid; r < xrn; r += DS_THREADS)
        {
            const __half v = xs[xr0 + r];
            xr[r] = v;
            p.resid_t[xr0 + r] = ds_tagged(tag, v);
        }
    }
    if (p.pro == PRO_VEC)
        return;
    // (the prefetched weights of the coming tasks are live in registers here:
    // keep this code's own working set small, one half2 at a time)
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

// Greedy sampling fused into the lm_head epilogue (ChatSession::Sample's
// argmax, src/ChatSession.cpp:564-567; the sampler kernel's greedy path):
// the CTA's best key to pick_cand, then the last CTA to arrive takes the
// maximum over all CTAs and updates the step state as the sampler does.
__shared__ uint64_t ds_pick[DS_WARPS];
__shared__ int ds_pick_last;

// One 16-bit payload from a tagged word of this rank's pick mailbox, once the
// word carries `tag`; bounded as the other waits (after wait_ns, or at once
// after a recorded error, the current word is used).
__device__ __forceinline__ uint32_t ds_pick_poll(const uint32_t *w, uint32_t tag, unsigned long long wait_ns, int *err)
{
    uint32_t v = __ldcg(w);
    if ((v & 0xffff0000u) != tag)
    {
        const uint64_t t0 = globaltimer_ns();
        for (int n = 1;; n++)
        {
            __nanosleep(64);
            v = __ldcg(w);
            if ((v & 0xffff0000u) == tag)
                break;
            if ((n & 31) == 0)
            {
                if (*reinterpret_cast<volatile int *>(err) != 0)
                    break;
                if (globaltimer_ns() - t0 > wait_ns)
                {
                    atomicExch(err, YLM_DEV_ERR_TIMEOUT_PEER);
                    break;
                }
            }
        }
    }
    return v & 0xffffu;
}

// Tensor parallelism: this rank's best key (over its vocabulary rows, global
// index) to slot `rank` of every rank's pick mailbox as three tagged words
// (ordered value, index high and low 16 bits; plain stores, over NVLink to the
// peers), then the maximum over every rank's slot of this rank's own mailbox.
// Every rank computes the same maximum: the argmax over the whole vocabulary,
// lowest index among equal values, as the gathered logits' argmax.
__device__ __forceinline__ uint64_t ds_pick_exchange(uint64_t b, uint32_t *const *pick_mb, int tp, int rank,
                                                     uint32_t tag, unsigned long long wait_ns, int *err)
{
    const uint32_t ord = (uint32_t)(b >> 32) & 0xffffu, idx = key_idx(b);
    const uint32_t w0 = tag | ord, w1 = tag | (idx >> 16), w2 = tag | (idx & 0xffffu);
    for (int q = 0; q < tp; q++)
    {
        uint32_t *d = pick_mb[q] + 4 * rank;
        d[0] = w0;
        d[1] = w1;
        d[2] = w2;
    }
    const uint32_t *mine = pick_mb[rank];
    uint64_t best = 0;
    for (int q = 0; q < tp; q++)
    {
        const uint32_t o = ds_pick_poll(mine + 4 * q, tag, wait_ns, err);
        const uint32_t hi = ds_pick_poll(mine + 4 * q + 1, tag, wait_ns, err);
        const uint32_t lo = ds_pick_poll(mine + 4 * q + 2, tag, wait_ns, err);
        const uint64_t k = make_key(o, (hi << 16) | lo);
        best = k > best ? k : best;
    }
    return best;
}

// (out of line with its arguments by value: a reference to the kernel
// parameters would copy them all to the stack)
__device__ __noinline__ void ds_greedy_pick(StepState *state, unsigned long long *cand, int *counter, uint64_t best,
                                            int tid, uint32_t *const *pick_mb, int tp, int rank, uint32_t tag,
                                            unsigned long long wait_ns, int *err)
{
    const int warp = tid >> 5, lane = tid & 31;
    best = warp_max_u64(best);
    if (lane == 0)
        ds_pick[warp] = best;
    named_bar_sync(1, DS_THREADS);
    if (tid == 0)
    {
        uint64_t b = 0;
        for (int w = 0; w < DS_WARPS; w++)
            b = ds_pick[w] > b ? ds_pick[w] : b;
        cand[blockIdx.x] = b;
        __threadfence();
        ds_pick_last = atomicAdd(counter, 1) == (int)gridDim.x - 1;
    }
    named_bar_sync(1, DS_THREADS);
    if (!ds_pick_last)
        return;
    __threadfence();
    uint64_t k = 0;
    for (int c = tid; c < (int)gridDim.x; c += DS_THREADS)
    {
        const uint64_t v = __ldcg(cand + c);
        k = v > k ? v : k;
    }
    k = warp_max_u64(k);
    if (lane == 0)
        ds_pick[warp] = k;
    named_bar_sync(1, DS_THREADS);
    if (tid == 0)
    {
        uint64_t b = 0;
        for (int w = 0; w < DS_WARPS; w++)
            b = ds_pick[w] > b ? ds_pick[w] : b;
        if (tp > 1)
            b = ds_pick_exchange(b, pick_mb, tp, rank, tag, wait_ns, err);
        StepState *s = state;
        const int64_t id = (int64_t)key_idx(b);
        s->next_token = id;
        s->sample_calls = s->sample_calls + 1;
        if (s->advance)
        {
            s->token = id;
            s->slot = s->slot + 1;
            s->rope_pos = s->rope_pos + 1;
        }
        *counter = 0;
    }
}

// Row sums of the chunk partials in order, then the epilogue of the per-op
// kernel; activations consumed inside the launch are written tagged.
__device__ __forceinline__ void ds_epilogue(const DsArgs &a, const DsPhase &p, const DsTab &t, const float *part,
                                            __half *xr, uint32_t tag, int tid)
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
            p.out_t[(t.r0 + 2 * q) >> 1] = ds_tagged(tag, f2h(sg * u));
        }
        return;
    }
    if (p.epi == EPI_RESID && p.mbox)
    {
        // tensor parallel: this rank's partial of the rows (FP16, as the per-op
        // path's all-reduce input) goes to slot `rank` of every rank's mailbox;
        // then this CTA sums its rows over all ranks' slots of its own mailbox,
        // in rank order, and adds the residual, identically on every rank
        uint32_t *const *mb = a.mb[p.mbox - 1];
        const bool stamp = a.xstat && blockIdx.x == 0 && tid == 0;
        const uint64_t ts0 = stamp ? globaltimer_ns() : 0;
        for (int r = tid; r < t.rows; r += DS_THREADS)
        {
            float y = 0.f;
            for (int c = 0; c < t.nkc; c++)
                y += part[r * t.nkc + c];
            const uint32_t w = ds_tagged(tag, f2h(y));
            const size_t off = (size_t)a.rank * a.hidden + t.r0 + r;
            for (int q = 0; q < a.tp; q++)
                mb[q][off] = w;
        }
        for (int r = tid; r < t.rows; r += DS_THREADS)
        {
            float sum = 0.f;
            for (int q = 0; q < a.tp; q++)
                sum += h2f(ds_read_tagged1(a, mb[a.rank] + (size_t)q * a.hidden + t.r0 + r, tag));
            const __half v = f2h(h2f(xr[r]) + rh(sum));
            xr[r] = v;
            p.resid_t[t.r0 + r] = ds_tagged(tag, v);
        }
        if (stamp)
        {
            a.xstat[0] += globaltimer_ns() - ts0;
            a.xstat[1] += 1ull;
        }
        return;
    }
    uint64_t best = 0; // greedy_pick: this thread's best (value, index) key
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
            const __half h = f2h(y);
            p.out[row] = h;
            if (p.greedy_pick)
            {
                // the vocabulary index: this rank's rows follow rank * N
                const uint64_t k = make_key(ord16(__half_as_ushort(h)), (uint32_t)(a.rank * p.N + row));
                best = k > best ? k : best;
            }
        }
        else
        {
            // residual stream: every residual phase has N = H and the same row
            // split, so this CTA alone updates these rows and keeps them in
            // shared memory (seeded at launch entry)
            const __half v = f2h(h2f(xr[r]) + rh(y));
            xr[r] = v;
            p.resid_t[row] = ds_tagged(tag, v);
        }
    }
    if (p.greedy_pick)
        ds_greedy_pick(a.pick_state, a.pick_cand, a.pick_counter, best, tid, a.pick_mb, a.tp, a.rank, tag, a.wait_ns,
                       a.err);
}

// Task cursor of one warp through the phases of a launch: phase, row, chunk,
// task index (the partial's slot) and tasks left in the phase.
struct DsCursor
{
    int ph, row, kc, t, left;
};

// Move `c` to the first task of this warp in phase c.ph or a later one.
__device__ __forceinline__ void ds_cursor_enter(const DsTab *tab, int p0, int i1, int warp, DsCursor &c)
{
    for (; c.ph < i1; c.ph++)
    {
        const DsTab &tb = tab[c.ph - p0];
        const int ntask = tb.rows * tb.nkc;
        if (warp < ntask)
        {
            c.row = tb.r0 + warp / tb.nkc;
            c.kc = warp % tb.nkc;
            c.t = warp;
            c.left = (ntask - warp + DS_WARPS - 1) / DS_WARPS;
            return;
        }
    }
}

__device__ __forceinline__ void ds_cursor_step(const DsTab *tab, int p0, int i1, int warp, DsCursor &c)
{
    if (--c.left == 0)
    {
        c.ph++;
        ds_cursor_enter(tab, p0, i1, warp, c);
        return;
    }
    const DsTab &tb = tab[c.ph - p0];
    c.t += DS_WARPS;
    c.row += tb.drow;
    c.kc += tb.dkc;
    if (c.kc >= tb.nkc)
    {
        c.kc -= tb.nkc;
        c.row++;
    }
}

// A run of consecutive GEMV phases [i0, i1). Each warp walks its task stream
// (phase, task = warp, warp + DS_WARPS, ...) with a ring of DS_D register
// buffers whose roles are fixed by unrolling, so a buffer is never copied
// while its loads are in flight; the first tasks of a phase are loaded while
// the previous phase is still finishing.
__device__ __forceinline__ void ds_segment(const DsArgs &a, int i0, int i1, unsigned &gen, int tid)
{
    const DsSmem sm = ds_smem_map(a);
    const DsTab *tab = sm.tab;
    __half *xs = sm.xs;
    float *part = sm.part, *red = sm.red;
    __half *xr = sm.xr;
    const int warp = tid >> 5, lane = tid & 31;
    DsCursor pc{i0, 0, 0, 0, 0}; // loads
    ds_cursor_enter(tab, a.p0, i1, warp, pc);
    DsCursor cc = pc; // arithmetic
    uint4 buf[DS_D][DS_U];
    auto load = [&](uint4 *w) {
        if (pc.ph >= i1)
            return;
        const DsTab &tb = tab[pc.ph - a.p0];
        const __half *base = tb.w + (size_t)pc.row * tb.K + pc.kc * DS_KC + lane * 8;
        const int lim = tb.K - pc.kc * DS_KC - lane * 8;
#pragma unroll
        for (int u = 0; u < DS_U; u++)
            w[u] = u * 256 < lim ? ds_ldg_stream(base + u * 256) : make_uint4(0, 0, 0, 0);
        ds_cursor_step(tab, a.p0, i1, warp, pc);
    };
#pragma unroll
    for (int d = 0; d < DS_D - 1; d++)
        load(buf[d]);
    // everything below reads what earlier kernels wrote (the step generation,
    // the residual stream, attention output, the step state): wait for the
    // preceding kernel, once the first weight loads are out
    pdl_wait();
    gen = *reinterpret_cast<volatile const unsigned *>(a.gen);
    // this CTA's rows of the residual stream, as the previous launch left them
    // (at most one per thread): loaded now, stored after the first prologue so
    // the two L2 round trips overlap (a layer-0 embedding prologue replaces them)
    const int xr0 = (int)((long long)a.hidden * blockIdx.x / gridDim.x);
    const int xrn = (int)((long long)a.hidden * (blockIdx.x + 1) / gridDim.x) - xr0;
    uint32_t xrv = tid < xrn ? __ldcg(a.xt + xr0 + tid) : 0u;
    int cur = i0;
    if (a.ph[cur - a.p0].pro == PRO_EMBED_RMSNORM)
        xrv = 0u; // (not needed: the prologue writes the rows)
    ds_prologue(a, a.ph[cur - a.p0], cur, tab[cur - a.p0].nkc * DS_KC, gen, xs, red, xr, tid);
    if (tid < xrn && a.ph[i0 - a.p0].pro != PRO_EMBED_RMSNORM)
        xr[tid] = __ushort_as_half((unsigned short)(xrv & 0xffffu));
    // (the first epilogue starts with a barrier, which publishes xr)
    // finish phase `cur` (every warp is past its tasks) and open the next one
    auto advance = [&]() {
        ds_epilogue(a, a.ph[cur - a.p0], tab[cur - a.p0], part, xr, ds_tag(gen, a.nph, cur), tid);
        cur++;
        if (cur < i1)
            ds_prologue(a, a.ph[cur - a.p0], cur, tab[cur - a.p0].nkc * DS_KC, gen, xs, red, xr, tid);
    };
    for (;;)
    {
#pragma unroll
        for (int d = 0; d < DS_D; d++)
        {
            while (cur < cc.ph && cur < i1)
                advance();
            if (cc.ph >= i1)
                goto done;
            load(buf[(d + DS_D - 1) % DS_D]);
            {
                // four interleaved accumulators (vectors u = j mod 4), as gemv_kernel
                const __half *xk = xs + cc.kc * DS_KC + lane * 8;
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int u = 0; u < DS_U; u++)
                    acc[u & 3] = ds_dot8(buf[d][u], *reinterpret_cast<const uint4 *>(xk + u * 256), acc[u & 3]);
                const float y = warp_sum((acc[0] + acc[1]) + (acc[2] + acc[3]));
                if (lane == 0)
                    part[cc.t] = y; // slot (row t / nkc, chunk t % nkc)
                ds_cursor_step(tab, a.p0, i1, warp, cc);
            }
        }
    }
done:
    while (cur < i1)
        advance();
}

// ------------------------------------------------------------ the kernel
// Phases [a.p0, a.p1) of the step's table, all GEMV.
__global__ void __launch_bounds__(DS_THREADS, 1) decode_segment_kernel(const DsArgs a)
{
    DsTab *tab = reinterpret_cast<DsTab *>(ds_smem);
    const int tid = threadIdx.x, C = gridDim.x, c = blockIdx.x;

    for (int i = a.p0 + tid; i < a.p1; i += DS_THREADS)
    {
        const DsPhase &p = a.ph[i - a.p0];
        DsTab t;
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
        t.w = p.w;
        t.K = p.K;
        t.nkc = (p.K + DS_KC - 1) / DS_KC;
        t.drow = DS_WARPS / t.nkc;
        t.dkc = DS_WARPS % t.nkc;
        tab[i - a.p0] = t;
    }
    __syncthreads();

    unsigned gen = 0;
    ds_segment(a, a.p0, a.p1, gen, tid);
    // the step's last segment ends with a phase whose input is every CTA's
    // output of an earlier phase of this launch, so all CTAs have read *gen
    if (a.last && c == 0 && tid == 0)
        *a.gen = gen + 1u;
}

// ------------------------------------------------------------ host side
int ds_threads() { return DS_THREADS; }

int ds_task_cols() { return DS_KC; }

int ds_tab_bytes() { return (int)((DS_MAX_SEG_PHASES * sizeof(DsTab) + 15) & ~(size_t)15); }

cudaError_t ds_prepare(size_t smem, int *blocks_per_sm)
{
    cudaError_t e = cudaFuncSetAttribute(decode_segment_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess)
        return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, decode_segment_kernel, DS_THREADS, smem);
}

cudaError_t ds_launch(const DsArgs &a, size_t smem, int grid, cudaStream_t s)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(DS_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    // Programmatic dependent launch: the CTAs start as the preceding kernel's
    // CTAs exit and issue their first weight loads before griddepcontrol.wait.
    // Not a cooperative launch (measured 2.3 % slower per decode step): the
    // CTAs wait on one another, so they must all be resident, which holds
    // because the grid is one CTA per SM and only one fits per SM; the only
    // grid that can share the device with it is its predecessor (attention or
    // the sampler), whose CTAs are all resident before these start and finish
    // without waiting on them. Two segment launches never overlap: attention
    // between them is launched without this attribute. Every wait is bounded
    // (a missing CTA ends as YLM_DEV_ERR_TIMEOUT_PEER, not a hang).
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_segment_kernel, a);
}

} // namespace ylm
