// Decode attention without any device allocation.
//
// ylm_k_decode_attention takes its scratch (split partials, per-KV-head
// tickets, step state) from cudaMallocAsync on the caller's stream. Some
// callers cannot allocate device memory at all: a host whose device memory is
// owned entirely by its own pool allocator, code that must not trigger the
// device-wide synchronisation or latency an allocation can cause, or a plugin
// that is only handed input and output buffers. For them this file provides
// ylm_k_decode_attention_noalloc: the same kernel, with its scratch in one
// file-scope __device__ array that this library reserves on every GPU that loads
// it, for the life of the process.
//
// Limits and rules (also stated in include/yalama_b200.h):
//   - scratch is YLM_NOALLOC_SCRATCH_BYTES (2 MiB). The cluster kernel (the
//     path on B200) needs only the 256-byte step state; the split-K kernel
//     (where cluster launches are unavailable, or forced with
//     ylm_set_attention_path) also needs hq x splits x 130 floats of partials
//     and one ticket per KV head, and shapes whose partials do not fit return
//     YLM_UNSUPPORTED. With at most 8 query heads per KV head and about two
//     CTAs per SM over the KV heads, that limit is reached only past ~4000
//     query heads;
//   - every call shares the array, so calls that overlap on the GPU (different
//     streams, or other threads) race; serialise them;
//   - the array keeps the previous call's contents: the tickets are cleared and
//     the step state is written by a one-thread kernel on the caller's stream
//     before each launch;
//   - the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current); make that first call
//     before any stream capture.
#include "ylm_common.cuh"
#include "ylm_kernels.h"
#include "../../include/yalama_b200.h"

#include <cstdio>
#include <mutex>

namespace ylm {

constexpr size_t YLM_NOALLOC_SCRATCH_BYTES = 2u << 20;

static __device__ __align__(256) unsigned char g_attn_scratch[YLM_NOALLOC_SCRATCH_BYTES];

// Writes the slot and RoPE position and clears the tickets: the array holds
// whatever the previous call left there.
__global__ void noalloc_reset_kernel(StepState *st, int *tickets, int hkv, int slot, int rope_pos)
{
    StepState s = {};
    s.slot = slot;
    s.rope_pos = rope_pos;
    *st = s;
    for (int i = 0; i < hkv; i++)
        tickets[i] = 0;
}

namespace {
std::mutex g_mu;
void *g_ptr[64] = {};

// device address of g_attn_scratch on the current device (looked up once per device)
cudaError_t scratch_address(void **out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return e;
    if (dev < 0 || dev >= 64)
        return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(g_mu);
    if (!g_ptr[dev])
    {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess)
            return e;
        g_ptr[dev] = p;
    }
    *out = g_ptr[dev];
    return cudaSuccess;
}
} // namespace

} // namespace ylm

using namespace ylm;

extern "C" int ylm_k_decode_attention_noalloc(const void *qkv, const void *q_norm, const void *k_norm, float eps,
                                              const void *rope_cos, const void *rope_sin, int32_t max_pos,
                                              void *k_cache, void *v_cache, int32_t cap, int32_t hq, int32_t hkv,
                                              int32_t slot, int32_t rope_pos, void *out, void *stream)
{
    if (!qkv || !rope_cos || !rope_sin || !k_cache || !v_cache || !out || hkv <= 0 || hq <= 0 || hq % hkv ||
        hq / hkv > 8 || slot < 0 || slot >= cap || rope_pos < 0 || rope_pos >= max_pos)
        return YLM_INVALID_ARG;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return YLM_CUDA_ERROR;
    const int splits = attn_default_splits(hkv, sms);
    static_assert(sizeof(StepState) <= 256, "step state must fit its 256-byte slot");
    const size_t state_bytes = 256; // StepState, padded to the array's alignment
    // the kernels' shared-memory settings and the attention path, once per
    // device (no allocation)
    if (prepare_device() != cudaSuccess)
        return YLM_CUDA_ERROR;
    const bool split_kernel = attn_uses_split_kernel();
    const size_t part_bytes = split_kernel ? attn_partial_floats(hq, splits) * sizeof(float) : 0;
    const size_t need = state_bytes + part_bytes + (split_kernel ? sizeof(int) * (size_t)hkv : 0);
    if (need > YLM_NOALLOC_SCRATCH_BYTES)
    {
        set_last_error("split-K partials exceed the fixed 2 MiB scratch");
        return YLM_UNSUPPORTED; // hq x splits too large for the fixed scratch
    }
    void *base = nullptr;
    if (scratch_address(&base) != cudaSuccess)
        return YLM_CUDA_ERROR;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // an error left pending by an unrelated earlier runtime call is only named
    // in this call's message (peeked, so the caller still sees it)
    const cudaError_t stale = cudaPeekAtLastError();
    StepState *state = static_cast<StepState *>(base);
    float *partial = reinterpret_cast<float *>(static_cast<char *>(base) + state_bytes);
    int *tickets = reinterpret_cast<int *>(static_cast<char *>(base) + state_bytes + part_bytes);
    // launched through the runtime call that returns this launch's own status
    int n_tickets = split_kernel ? hkv : 0;
    void *rargs[] = {&state, &tickets, &n_tickets, &slot, &rope_pos};
    cudaError_t le = cudaLaunchKernel((const void *)noalloc_reset_kernel, dim3(1), dim3(1), rargs, 0, s);
    if (le != cudaSuccess)
    {
        char msg[160];
        snprintf(msg, sizeof(msg), "reset launch: %s (earlier pending error: %s)", cudaGetErrorName(le),
                 cudaGetErrorName(stale));
        set_last_error(msg);
        return YLM_CUDA_ERROR;
    }
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
    a.counters = tickets;
    a.out = static_cast<__half *>(out);
    a.state = state;
    a.err = &state->err;
    le = attn_decode_launch(a, s, false);
    if (le != cudaSuccess)
    {
        char msg[160];
        snprintf(msg, sizeof(msg), "attention launch: %s (earlier pending error: %s)", cudaGetErrorName(le),
                 cudaGetErrorName(stale));
        set_last_error(msg);
        return YLM_CUDA_ERROR;
    }
    set_last_error("");
    return YLM_OK;
}
