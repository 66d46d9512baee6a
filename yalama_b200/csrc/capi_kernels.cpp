// Kernel-level C ABI entry points (include/yalama_b200.h, "kernel-level entry
// points"): the decode GEMV, the prefill GEMM, one decode-attention step and the
// sampler, on caller-owned device buffers and the caller's stream. Scratch that
// a kernel needs (split partials, tickets, step state) is allocated
// stream-ordered (cudaMallocAsync / cudaFreeAsync) on that stream, so calls on
// different streams never share it.
#include "../../include/yalama_b200.h"
#include "ylm_kernels.h"

#include <cuda_runtime.h>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

using namespace ylm;

namespace {

int sm_count()
{
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? YLM_OK : YLM_CUDA_ERROR; }

} // namespace

namespace ylm {
// shared-memory opt-in of the kernels, once per device
cudaError_t prepare_device()
{
    static std::mutex mu;
    static bool done[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64)
        return e != cudaSuccess ? e : cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(mu);
    if (!done[dev])
    {
        e = kernels_prepare();
        if (e != cudaSuccess)
            return e;
        done[dev] = true;
    }
    return cudaSuccess;
}
} // namespace ylm

extern "C" {

int ylm_set_attention_path(int32_t split_kernel)
{
    if (split_kernel != 0 && split_kernel != 1)
        return YLM_INVALID_ARG;
    attn_force_split_kernel(split_kernel != 0);
    return YLM_OK;
}

int ylm_k_gemv(const void *w, int32_t n, int32_t k, const void *x, void *y, void *stream)
{
    if (!w || !x || !y || n <= 0 || k <= 0)
        return YLM_INVALID_ARG;
    if (prepare_device() != cudaSuccess)
        return YLM_CUDA_ERROR;
    // plans (tensor map + tiling) are cached per (device, weight, shape)
    static std::mutex mu;
    static std::map<std::tuple<int, const void *, int, int>, GemvPlan> plans;
    int dev = 0;
    cudaGetDevice(&dev);
    GemvPlan plan;
    {
        std::lock_guard<std::mutex> g(mu);
        auto key = std::make_tuple(dev, w, n, k);
        auto it = plans.find(key);
        if (it == plans.end())
        {
            if (!gemv_make_plan(&plan, static_cast<const __half *>(w), n, k, 0, sm_count()))
                return YLM_UNSUPPORTED;
            if (plans.size() > 4096)
                plans.clear();
            plans[key] = plan;
        }
        else
            plan = it->second;
    }
    GemvArgs a;
    a.x = static_cast<const __half *>(x);
    a.out = static_cast<__half *>(y);
    return cuda_status(gemv_launch(plan, PRO_VEC, EPI_STORE, a, static_cast<cudaStream_t>(stream), false));
}

int ylm_k_gemm(const void *a, const void *w, int32_t t, int32_t n, int32_t k, void *c, int32_t tensor_cores,
               void *stream)
{
    if (!a || !w || !c || t <= 0 || n <= 0 || k <= 0)
        return YLM_INVALID_ARG;
    if (prepare_device() != cudaSuccess)
        return YLM_CUDA_ERROR;
    if (tensor_cores)
    {
        CUtensorMap am, wm;
        if (!tc_make_a_map(&am, static_cast<const __half *>(a), t, k, k) ||
            !tc_make_w_map(&wm, static_cast<const __half *>(w), n, k))
            return YLM_UNSUPPORTED;
        return cuda_status(gemm_tc_launch(am, wm, t, n, k, GEMM_STORE, nullptr, static_cast<__half *>(c), n, nullptr,
                                          static_cast<cudaStream_t>(stream)));
    }
    return cuda_status(gemm_launch(static_cast<const __half *>(a), k, static_cast<const __half *>(w), t, n, k,
                                   GEMM_STORE, nullptr, static_cast<__half *>(c), n,
                                   static_cast<cudaStream_t>(stream)));
}

int ylm_k_prefill_attention(const void *q, const void *k_cache, const void *v_cache, int32_t cap, int32_t hq,
                            int32_t hkv, int32_t t, void *out, int32_t tensor_cores, void *stream)
{
    if (!q || !k_cache || !v_cache || !out || t <= 0 || t > cap || hkv <= 0 || hq <= 0 || hq % hkv)
        return YLM_INVALID_ARG;
    if (prepare_device() != cudaSuccess)
        return YLM_CUDA_ERROR;
    const __half *qh = static_cast<const __half *>(q), *kh = static_cast<const __half *>(k_cache),
                 *vh = static_cast<const __half *>(v_cache);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (tensor_cores)
        return cuda_status(attn_prefill_tc_launch(qh, kh, vh, cap, hq, hkv, t, static_cast<__half *>(out), nullptr, s));
    return cuda_status(attn_prefill_launch(qh, kh, vh, cap, hq, hkv, t, static_cast<__half *>(out), s));
}

int ylm_k_decode_attention(const void *qkv, const void *q_norm, const void *k_norm, float eps, const void *rope_cos,
                           const void *rope_sin, int32_t max_pos, void *k_cache, void *v_cache, int32_t cap,
                           int32_t hq, int32_t hkv, int32_t slot, int32_t rope_pos, void *out, void *stream)
{
    if (!qkv || !rope_cos || !rope_sin || !k_cache || !v_cache || !out || hkv <= 0 || hq <= 0 || hq % hkv ||
        hq / hkv > 8 || slot < 0 || slot >= cap || rope_pos < 0 || rope_pos >= max_pos)
        return YLM_INVALID_ARG;
    if (prepare_device() != cudaSuccess)
        return YLM_CUDA_ERROR;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int splits = attn_default_splits(hkv, sm_count());
    const size_t part_bytes = attn_partial_floats(hq, splits) * sizeof(float);
    const size_t bytes = sizeof(StepState) + part_bytes + sizeof(int) * hkv;
    void *scratch = nullptr;
    cudaError_t e = cudaMallocAsync(&scratch, bytes, s);
    if (e != cudaSuccess)
        return YLM_CUDA_ERROR;
    StepState st;
    memset(&st, 0, sizeof(st));
    st.slot = slot;
    st.rope_pos = rope_pos;
    StepState *dstate = static_cast<StepState *>(scratch);
    float *partial = reinterpret_cast<float *>(static_cast<char *>(scratch) + sizeof(StepState));
    int *counters = reinterpret_cast<int *>(static_cast<char *>(scratch) + sizeof(StepState) + part_bytes);
    e = cudaMemcpyAsync(dstate, &st, sizeof(st), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemsetAsync(counters, 0, sizeof(int) * hkv, s);
    if (e == cudaSuccess)
    {
        AttnArgs a;
        a.qkv = static_cast<const __half *>(qkv);
        a.q_norm = static_cast<const __half *>(q_norm);
        a.k_norm = static_cast<const __half *>(k_norm);
        a.eps = eps;
        a.rope_cos = static_cast<const __half *>(rope_cos);
        a.rope_sin = static_cast<const __half *>(rope_sin);
        a.max_pos = max_pos;
        a.k_cache = static_cast<__half *>(k_cache);
        a.v_cache = static_cast<__half *>(v_cache);
        a.cap = cap;
        a.hq = hq;
        a.hkv = hkv;
        a.splits = splits;
        a.partial = partial;
        a.counters = counters;
        a.out = static_cast<__half *>(out);
        a.state = dstate;
        a.err = &dstate->err;
        e = attn_decode_launch(a, s, false);
    }
    cudaError_t f = cudaFreeAsync(scratch, s);
    return cuda_status(e != cudaSuccess ? e : f);
}

int ylm_k_sample(const void *logits, int64_t vocab, int32_t greedy, int32_t top_k, float temperature,
                 const uint32_t *mask_bits_dev, float u, int64_t *out_id, int64_t *topk_ids, float *topk_probs,
                 void *stream)
{
    if (!logits || vocab <= 0 || !out_id || (!greedy && (top_k < 1 || top_k > 64 || !(temperature > 0.f))))
        return YLM_INVALID_ARG;
    if (prepare_device() != cudaSuccess)
        return YLM_CUDA_ERROR;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int parts = sample_parts(vocab, sm_count());
    const size_t bytes = sizeof(StepState) + (size_t)parts * 64 * 8 + sizeof(int) * (parts + 1) + 64 * 8 + 64 * 4;
    void *scratch = nullptr;
    if (cudaMallocAsync(&scratch, bytes, s) != cudaSuccess)
        return YLM_CUDA_ERROR;
    char *p = static_cast<char *>(scratch);
    StepState *dstate = reinterpret_cast<StepState *>(p);
    uint64_t *cand = reinterpret_cast<uint64_t *>(p + sizeof(StepState));
    int64_t *dbg_ids = reinterpret_cast<int64_t *>(p + sizeof(StepState) + (size_t)parts * 64 * 8);
    float *dbg_probs = reinterpret_cast<float *>(reinterpret_cast<char *>(dbg_ids) + 64 * 8);
    int *cand_count = reinterpret_cast<int *>(reinterpret_cast<char *>(dbg_probs) + 64 * 4);
    int *counter = cand_count + parts;
    StepState st;
    memset(&st, 0, sizeof(st));
    st.greedy = greedy ? 1 : 0;
    st.top_k = top_k;
    st.inv_temp = 1.0f / (temperature > 0.f ? temperature : 1.f);
    st.u_override = u;
    StepState back;
    cudaError_t e = cudaMemcpyAsync(dstate, &st, sizeof(st), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemsetAsync(counter, 0, sizeof(int), s);
    if (e == cudaSuccess)
    {
        SampleArgs a;
        a.logits = static_cast<const __half *>(logits);
        a.vocab = vocab;
        a.mask_bits = mask_bits_dev;
        a.state = dstate;
        a.cand = cand;
        a.cand_count = cand_count;
        a.counter = counter;
        a.parts = parts;
        a.dbg_ids = dbg_ids;
        a.dbg_probs = dbg_probs;
        a.err = &dstate->err;
        e = sample_launch(a, s, false);
    }
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(&back, dstate, sizeof(back), cudaMemcpyDeviceToHost, s);
    const int k = greedy ? 0 : top_k;
    if (e == cudaSuccess && k > 0 && topk_ids)
        e = cudaMemcpyAsync(topk_ids, dbg_ids, sizeof(int64_t) * k, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && k > 0 && topk_probs)
        e = cudaMemcpyAsync(topk_probs, dbg_probs, sizeof(float) * k, cudaMemcpyDeviceToHost, s);
    cudaError_t f = cudaFreeAsync(scratch, s);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(s);
    if (e != cudaSuccess || f != cudaSuccess)
        return YLM_CUDA_ERROR;
    *out_id = back.next_token;
    return YLM_OK;
}

} // extern "C"
