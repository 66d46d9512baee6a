// On-device sampling of the next token from the last-row logits, replacing
// ChatSession::Sample (src/ChatSession.cpp:560-593) and its blocking
// .to(kCPU) per token:
//   greedy  argmax over the raw logits, lowest index among ties (torch argmax)
//   top-k   logits * (1/temp) rounded to FP16, masked special ids -> -inf
//           (the reference writes -1e9, which is -inf in FP16), the K largest
//           values sorted descending with ties to the lower index (torch::topk),
//           softmax over them rounded to FP16, then one categorical draw.
// The reference draws with torch::multinomial; this kernel draws by inverse CDF
// from one uniform per call, taken from Philox4x32-10 (Salmon et al., SC'11)
// keyed by the engine seed with the call index as counter, so the engine is
// reproducible and a CPU restatement can check it bit for bit. The softmax exp
// is computed with explicit round-to-nearest FP32 operations (Cody-Waite range
// reduction with ln 2 split as in Cephes, degree-7 Taylor polynomial).
//
// One kernel, two phases: every CTA selects the top candidates of its slice of
// the vocabulary (radix select on the 16-bit ordered FP16 value, ties resolved
// in index order with block scans); the last CTA to finish (atomic ticket)
// merges the candidate lists the same way, sorts the final K and draws.
#include "ylm_common.cuh"
#include "ylm_kernels.h"
#include <algorithm>

namespace ylm {

constexpr int SMP_THREADS = 256;
constexpr int SMP_KMAX = 64;
constexpr int SMP_E = 8; // elements per thread in phase 1

// exclusive scan over the block of one int per thread; returns the total in *total
__device__ __forceinline__ int block_excl_scan(int v, int *wsum, int *total)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1)
    {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o)
            x += y;
    }
    if (lane == 31)
        wsum[warp] = x;
    __syncthreads();
    int base = 0, tot = 0;
    for (int w = 0; w < SMP_THREADS / 32; w++)
    {
        if (w < warp)
            base += wsum[w];
        tot += wsum[w];
    }
    __syncthreads();
    *total = tot;
    return base + x - v;
}

// Philox4x32-10, word 0 of the output block for counter (ctr, 0, 0) and key seed.
__device__ __forceinline__ uint32_t philox_x0(uint64_t seed, uint64_t ctr)
{
    uint32_t c0 = (uint32_t)ctr, c1 = (uint32_t)(ctr >> 32), c2 = 0, c3 = 0;
    uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
    for (int r = 0; r < 10; r++)
    {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
        const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0;
        c1 = lo1;
        c2 = n2;
        c3 = lo0;
        if (r < 9)
        {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
    }
    return c0;
}

// e^x for x <= 0 with explicitly rounded FP32 steps (no contraction).
__device__ __forceinline__ float exp_rn(float x)
{
    if (!(x >= -87.0f))
        return 0.0f;
    const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
    float r = __fsub_rn(x, __fmul_rn(n, 0.693359375f));
    r = __fsub_rn(r, __fmul_rn(n, -2.12194440e-4f));
    float p = (float)(1.0 / 5040.0);
    p = __fadd_rn(__fmul_rn(p, r), (float)(1.0 / 720.0));
    p = __fadd_rn(__fmul_rn(p, r), (float)(1.0 / 120.0));
    p = __fadd_rn(__fmul_rn(p, r), (float)(1.0 / 24.0));
    p = __fadd_rn(__fmul_rn(p, r), (float)(1.0 / 6.0));
    p = __fadd_rn(__fmul_rn(p, r), 0.5f);
    p = __fadd_rn(__fmul_rn(p, r), 1.0f);
    p = __fadd_rn(__fmul_rn(p, r), 1.0f);
    int ni = (int)n;
    ni = ni < -126 ? -126 : (ni > 0 ? 0 : ni);
    return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

struct SelectShared
{
    int hist[256];
    int wsum[SMP_THREADS / 32];
    int sel[4]; // B1, gt1, B0, gt
};

// Threshold T (16-bit ordered value) such that fewer than k values exceed T and
// at least k are >= T; also returns how many exceed it. `val(i)` gives the
// ordered value of element i of this thread (valid(i) false -> ignored).
// Add one to hist[bin] for every lane with valid == true; lanes that share a
// bin are combined first (__match_any_sync), so clustered values (the top
// logits often share a few FP16 bins) cost one shared atomic per distinct bin.
__device__ __forceinline__ void hist_add(int *hist, uint32_t bin, bool valid)
{
    const int lane = threadIdx.x & 31;
    const uint32_t key = valid ? bin : 0x10000u + (uint32_t)lane;
    const uint32_t peers = __match_any_sync(0xffffffffu, key);
    if (valid && lane == __ffs(peers) - 1)
        atomicAdd(&hist[bin], __popc(peers));
}

// The bin of the k-th largest value in sh.hist, counting `above` values
// already known to lie above every bin: the highest bin b with
// above + count(bins > b) < k <= above + count(bins >= b), or bin 0 when the
// bins hold fewer than k (then count(bins > 0)). Thread t looks at bin 255 - t
// so one block-wide exclusive scan gives every bin's count above it.
// Writes sh.sel[out] = b, sh.sel[out + 1] = above + count(bins > b).
__device__ __forceinline__ void threshold_bin(int k, int above, SelectShared &sh, int out)
{
    static_assert(SMP_THREADS == 256, "one thread per bin");
    const int b = 255 - (int)threadIdx.x;
    const int hv = sh.hist[b];
    int tot;
    const int excl = above + block_excl_scan(hv, sh.wsum, &tot);
    if (excl < k && (excl + hv >= k || b == 0))
    {
        sh.sel[out] = b;
        sh.sel[out + 1] = excl;
    }
    __syncthreads();
}

// Threshold T (16-bit ordered value) such that fewer than k values exceed T and
// at least k are >= T; also returns how many exceed it. `val(e)` gives the
// ordered value of element e of this thread, e < n_mine; every thread loops to
// n_max (block-uniform) so the warp-level aggregation stays convergent.
template <typename ValF>
__device__ __forceinline__ void radix_threshold(int k, int n_mine, int n_max, ValF val, SelectShared &sh,
                                                uint32_t *T_out, int *gt_out)
{
    const int tid = threadIdx.x;
    for (int b = tid; b < 256; b += SMP_THREADS)
        sh.hist[b] = 0;
    __syncthreads();
    for (int e = 0; e < n_max; e++)
    {
        const bool ok = e < n_mine;
        hist_add(sh.hist, ok ? (val(e) >> 8) : 0u, ok);
    }
    __syncthreads();
    threshold_bin(k, 0, sh, 0);
    const uint32_t B1 = (uint32_t)sh.sel[0];
    const int gt1 = sh.sel[1];
    for (int b = tid; b < 256; b += SMP_THREADS)
        sh.hist[b] = 0;
    __syncthreads();
    for (int e = 0; e < n_max; e++)
    {
        const bool ok = e < n_mine;
        const uint32_t v = ok ? val(e) : 0u;
        hist_add(sh.hist, v & 255, ok && (v >> 8) == B1);
    }
    __syncthreads();
    threshold_bin(k, gt1, sh, 2);
    *T_out = (B1 << 8) | (uint32_t)sh.sel[2];
    *gt_out = sh.sel[3];
    __syncthreads();
}

__global__ void __launch_bounds__(SMP_THREADS) sample_kernel(const SampleArgs a)
{
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ SelectShared sh;
    __shared__ uint64_t fin[SMP_KMAX];
    __shared__ uint64_t sorted[SMP_KMAX];
    __shared__ int ticket;
    __shared__ uint64_t wbest[SMP_THREADS / 32];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int c = blockIdx.x, P = a.parts;
    pdl_launch_dependents();
    pdl_wait(); // logits from the lm_head projection

    const StepState *st = a.state;
    const int greedy = st->greedy;
    const int K = greedy ? 1 : max(1, min(st->top_k, SMP_KMAX));
    const float inv_t = st->inv_temp;
    const int64_t V = a.vocab;
    const int64_t chunk = (V + P - 1) / P;
    const int64_t base = (int64_t)c * chunk;
    const int cnt = (int)max((int64_t)0, min(chunk, V - base));
    const int E = (int)((chunk + SMP_THREADS - 1) / SMP_THREADS);

    // ---------------- phase 1: this CTA's slice, elements [tid*E, tid*E+E)
    uint32_t ov[SMP_E];
    int n_mine = 0;
#pragma unroll
    for (int e = 0; e < SMP_E; e++)
    {
        ov[e] = 0;
        const int i = tid * E + e;
        if (e < E && i < cnt)
        {
            const int64_t gi = base + i;
            uint32_t h = __half_as_ushort(a.logits[gi]);
            if (!greedy)
            {
                h = __half_as_ushort(__float2half_rn(__fmul_rn(__half2float(__ushort_as_half((unsigned short)h)), inv_t)));
                if (a.mask_bits && ((a.mask_bits[gi >> 5] >> (gi & 31)) & 1u))
                    h = 0xFC00u; // -inf
            }
            ov[e] = ord16(h);
            n_mine = e + 1;
        }
    }
    uint64_t *cand = a.cand + (size_t)c * SMP_KMAX;
    if (greedy)
    {
        uint64_t best = 0;
        for (int e = 0; e < n_mine; e++)
        {
            const uint64_t k = make_key(ov[e], (uint32_t)(base + tid * E + e));
            best = k > best ? k : best;
        }
        best = warp_max_u64(best);
        if (lane == 0)
            wbest[warp] = best;
        __syncthreads();
        if (tid == 0)
        {
            uint64_t b = 0;
            for (int w = 0; w < SMP_THREADS / 32; w++)
                b = wbest[w] > b ? wbest[w] : b;
            cand[0] = b;
            a.cand_count[c] = cnt > 0 ? 1 : 0;
        }
    }
    else
    {
        const int keff = min(K, cnt);
        if (keff > 0)
        {
            uint32_t T;
            int gt;
            radix_threshold(keff, n_mine, E, [&](int e) { return ov[e]; }, sh, &T, &gt);
            const int need = keff - gt;
            int n_eq = 0;
            for (int e = 0; e < n_mine; e++)
                n_eq += ov[e] == T;
            int tot;
            const int eq_base = block_excl_scan(n_eq, sh.wsum, &tot);
            int n_sel = 0, r = eq_base;
            for (int e = 0; e < n_mine; e++)
                if (ov[e] > T || (ov[e] == T && r++ < need))
                    n_sel++;
            const int pos0 = block_excl_scan(n_sel, sh.wsum, &tot);
            int pos = pos0;
            r = eq_base;
            for (int e = 0; e < n_mine; e++)
                if (ov[e] > T || (ov[e] == T && r++ < need))
                    cand[pos++] = make_key(ov[e], (uint32_t)(base + tid * E + e));
        }
        if (tid == 0)
            a.cand_count[c] = max(keff, 0);
    }

    // ---------------- ticket: the last CTA merges
    __threadfence();
    __syncthreads();
    if (tid == 0)
        ticket = atomicAdd(a.counter, 1);
    __syncthreads();
    if (ticket != P - 1)
        return;
    __threadfence();

    uint64_t pick_key = 0;
    StepState *stw = a.state;
    if (greedy)
    {
        uint64_t best = 0;
        for (int p = tid; p < P; p += SMP_THREADS)
            if (__ldcg(a.cand_count + p) > 0)
            {
                const uint64_t k = __ldcg(reinterpret_cast<const unsigned long long *>(a.cand) + (size_t)p * SMP_KMAX);
                best = k > best ? k : best;
            }
        best = warp_max_u64(best);
        if (lane == 0)
            wbest[warp] = best;
        __syncthreads();
        if (tid == 0)
        {
            uint64_t b = 0;
            for (int w = 0; w < SMP_THREADS / 32; w++)
                b = wbest[w] > b ? wbest[w] : b;
            pick_key = b;
        }
    }
    else
    {
        // gather all candidate lists in part order (= vocabulary order): counts
        // and offsets first, then every slot copied by its own thread
        uint64_t *all = reinterpret_cast<uint64_t *>(smem);
        __shared__ int offs[SMP_THREADS + 1];
        int tot = 0;
        {
            const int ppt = (P + SMP_THREADS - 1) / SMP_THREADS; // parts per thread, contiguous runs
            int mycnt = 0;
            for (int q = 0; q < ppt; q++)
            {
                const int p = tid * ppt + q;
                if (p < P)
                    mycnt += __ldcg(a.cand_count + p);
            }
            const int off = block_excl_scan(mycnt, sh.wsum, &tot);
            int o = off;
            for (int q = 0; q < ppt; q++)
            {
                const int p = tid * ppt + q;
                if (p < P)
                {
                    offs[p] = o;
                    o += __ldcg(a.cand_count + p);
                }
            }
            __syncthreads();
            // eight independent loads in flight per thread, then the stores
            for (int i0 = tid; i0 < P * SMP_KMAX; i0 += SMP_THREADS * 8)
            {
                unsigned long long v[8];
                int dst[8];
#pragma unroll
                for (int u = 0; u < 8; u++)
                {
                    const int i = i0 + u * SMP_THREADS;
                    const int p = i / SMP_KMAX, j = i % SMP_KMAX;
                    dst[u] = -1;
                    if (i < P * SMP_KMAX)
                    {
                        const int cnt = (p + 1 < P ? offs[p + 1] : tot) - offs[p];
                        if (j < cnt)
                        {
                            dst[u] = offs[p] + j;
                            v[u] = __ldcg(reinterpret_cast<const unsigned long long *>(a.cand) + (size_t)p * SMP_KMAX + j);
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < 8; u++)
                    if (dst[u] >= 0)
                        all[dst[u]] = v[u];
            }
        }
        __syncthreads();
        const int M = tot;
        const int keff = min(K, M);
        const int E2 = (M + SMP_THREADS - 1) / SMP_THREADS;
        const int lo = min(M, tid * E2), hi = min(M, lo + E2);
        uint32_t T;
        int gt;
        radix_threshold(keff, hi - lo, E2, [&](int e) { return (uint32_t)(all[lo + e] >> 32); }, sh, &T, &gt);
        const int need = keff - gt;
        int n_eq = 0;
        for (int i = lo; i < hi; i++)
            n_eq += (uint32_t)(all[i] >> 32) == T;
        int t2;
        const int eq_base = block_excl_scan(n_eq, sh.wsum, &t2);
        int n_sel = 0, r = eq_base;
        for (int i = lo; i < hi; i++)
        {
            const uint32_t v = (uint32_t)(all[i] >> 32);
            if (v > T || (v == T && r++ < need))
                n_sel++;
        }
        int pos = block_excl_scan(n_sel, sh.wsum, &t2);
        r = eq_base;
        for (int i = lo; i < hi; i++)
        {
            const uint32_t v = (uint32_t)(all[i] >> 32);
            if (v > T || (v == T && r++ < need))
                fin[pos++] = all[i];
        }
        __syncthreads();
        // rank sort, descending key = value descending, then index ascending
        if (tid < keff)
        {
            const uint64_t k = fin[tid];
            int rank = 0;
            for (int j = 0; j < keff; j++)
                rank += fin[j] > k;
            sorted[rank] = k;
        }
        __syncthreads();
        // softmax over the sorted K values: exps in parallel (one lane per
        // candidate), the sums sequentially in candidate order on lane 0 (the
        // order the CPU restatement uses), then the inverse-CDF walk
        __shared__ float ev[SMP_KMAX];
        __shared__ float ssum;
        if (warp == 0)
        {
            for (int i = lane; i < keff; i += 32)
            {
                const float v0 = __half2float(__ushort_as_half((unsigned short)unord16((uint32_t)(sorted[0] >> 32))));
                const float vi = __half2float(__ushort_as_half((unsigned short)unord16((uint32_t)(sorted[i] >> 32))));
                ev[i] = v0 == -INFINITY ? 0.f : exp_rn(__fsub_rn(vi, v0));
            }
            __syncwarp();
            if (lane == 0)
            {
                float sacc = 0.f;
                for (int i = 0; i < keff; i++)
                    sacc = __fadd_rn(sacc, ev[i]);
                ssum = sacc;
            }
            __syncwarp();
            for (int i = lane; i < keff; i += 32)
                ev[i] = ssum > 0.f ? __half2float(__float2half_rn(__fdiv_rn(ev[i], ssum))) : 0.f;
            __syncwarp();
            if (lane == 0)
            {
                float u;
                if (st->u_override >= 0.f)
                    u = st->u_override;
                else
                {
                    const uint32_t x0 = philox_x0(st->seed, (uint64_t)st->sample_calls);
                    u = (float)(2u * (x0 >> 9) + 1u) * 5.9604644775390625e-08f;
                }
                int pick = 0;
                if (keff > 0 && ssum > 0.f)
                {
                    float total = 0.f;
                    for (int i = 0; i < keff; i++)
                        total = __fadd_rn(total, ev[i]);
                    const float target = __fmul_rn(u, total);
                    float cum = 0.f;
                    int last_pos = 0;
                    pick = -1;
                    for (int i = 0; i < keff; i++)
                    {
                        if (ev[i] > 0.f)
                            last_pos = i;
                        cum = __fadd_rn(cum, ev[i]);
                        if (cum > target)
                        {
                            pick = i;
                            break;
                        }
                    }
                    if (pick < 0)
                        pick = last_pos;
                }
                stw->u_used = u;
                pick_key = keff > 0 ? sorted[pick] : 0;
            }
            if (a.dbg_ids)
                for (int i = lane; i < keff; i += 32)
                {
                    a.dbg_ids[i] = key_idx(sorted[i]);
                    a.dbg_probs[i] = ev[i];
                }
        }
    }
    if (tid == 0)
    {
        const int64_t id = (int64_t)key_idx(pick_key);
        stw->next_token = id;
        stw->sample_calls = st->sample_calls + 1;
        if (stw->advance)
        {
            stw->token = id;
            stw->slot = st->slot + 1;
            stw->rope_pos = st->rope_pos + 1;
        }
        *a.counter = 0;
    }
}

// As few parts as the per-thread register budget allows (SMP_E elements a
// thread): the last CTA merges parts x K candidates, so fewer, fuller parts
// shorten the serial end of the kernel (63 parts at a 128k vocabulary: top-k
// step overhead 30.8 -> 24.8 us at the Llama-3.2-3B shape against 126).
int sample_parts(int64_t vocab, int num_sms)
{
    (void)num_sms;
    const int64_t p = (vocab + SMP_THREADS * SMP_E - 1) / (SMP_THREADS * SMP_E);
    return (int)std::max<int64_t>(1, p);
}

cudaError_t sample_prepare()
{
    cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared);
    return e;
}

cudaError_t sample_launch(const SampleArgs &a, cudaStream_t s, bool pdl)
{
    const int64_t chunk = (a.vocab + a.parts - 1) / a.parts;
    if (chunk > SMP_THREADS * SMP_E || a.parts > SMP_THREADS)
        return cudaErrorInvalidValue;
    const size_t smem = (size_t)a.parts * SMP_KMAX * sizeof(uint64_t);
    if (smem > 160 * 1024)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.parts);
    cfg.blockDim = dim3(SMP_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, sample_kernel, a);
}

} // namespace ylm
