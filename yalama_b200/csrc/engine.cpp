// yalama_b200 engine: the host side of the batch-1 decode path, behind the C
// ABI of include/yalama_b200.h.
//
// It owns what ModelBase owns in the reference (src/models/ModelBase.cpp): the
// weights, the fixed-size KV cache, the RoPE tables and the
// _LastKVCacheTokenIndex state machine, and it drives the sm_100a kernels of
// this directory instead of LibTorch ops. Decode steps are captured once as a
// CUDA graph (kernels chained with programmatic dependent launch); per-step
// values (token, KV slot, RoPE position, sampling state) live in a small
// device-resident StepState so the same graph serves every step. Tensor
// parallelism (Megatron-style: column-split QKV / gate-up, row-split O / down,
// KV heads and vocabulary sharded) adds NCCL all-reduces after O and down and an
// all-gather of the logits.
#include "../../include/yalama_b200.h"
#include "json_lite.h"
#include "ylm_kernels.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <dirent.h>
#include <fcntl.h>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <thread>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <vector>

using namespace ylm;

// ------------------------------------------------------------------ errors
namespace {
thread_local std::string g_last_error;

struct YlmError : std::runtime_error
{
    int status;
    YlmError(int s, const std::string &m) : std::runtime_error(m), status(s) {}
};

[[noreturn]] void fail(int status, const char *fmt, ...)
{
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    throw YlmError(status, buf);
}

#define CK(call)                                                                                                      \
    do                                                                                                                \
    {                                                                                                                 \
        cudaError_t e_ = (call);                                                                                      \
        if (e_ != cudaSuccess)                                                                                        \
            fail(YLM_CUDA_ERROR, "%s:%d %s: %s", __FILE__, __LINE__, #call, cudaGetErrorString(e_));                  \
    } while (0)

#define NK(call)                                                                                                      \
    do                                                                                                                \
    {                                                                                                                 \
        ncclResult_t r_ = (call);                                                                                     \
        if (r_ != ncclSuccess)                                                                                        \
            fail(YLM_COMM_ERROR, "%s:%d %s: %s", __FILE__, __LINE__, #call, ncclGetErrorString(r_));                  \
    } while (0)

} // namespace

// for the kernel-level entry points outside this file
void ylm::set_last_error(const char *msg) { g_last_error = msg ? msg : ""; }

namespace {
template <typename F> int guarded(F &&f)
{
    try
    {
        g_last_error.clear();
        return f();
    }
    catch (const YlmError &e)
    {
        g_last_error = e.what();
        return e.status;
    }
    catch (const std::exception &e)
    {
        g_last_error = e.what();
        return YLM_LOAD_ERROR;
    }
}

std::string read_file(const std::string &p)
{
    std::ifstream f(p, std::ios::binary);
    if (!f)
        fail(YLM_LOAD_ERROR, "cannot open %s", p.c_str());
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

// FNV-1a 64 of a tensor name and the SplitMix64 finaliser: the stream key of
// the counter-based initialiser (yalama_b200/synth.py, init.cu).
uint64_t fnv1a64(const std::string &s)
{
    uint64_t h = 0xCBF29CE484222325ull;
    for (unsigned char c : s)
    {
        h ^= c;
        h *= 0x100000001B3ull;
    }
    return h;
}
uint64_t mix64(uint64_t z)
{
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// ------------------------------------------------------------------ safetensors
struct StTensor
{
    std::string dtype; // F16 / BF16 / F32
    std::vector<int64_t> shape;
    const uint8_t *data = nullptr;
    size_t bytes = 0;
};

struct StFile
{
    int fd = -1;
    void *map = nullptr;
    size_t size = 0;
    ~StFile()
    {
        if (map && map != MAP_FAILED)
            munmap(map, size);
        if (fd >= 0)
            close(fd);
    }
};

// mmap every *.safetensors shard of a snapshot folder and index its tensors
// (ModelBase.cpp:42-85 and include/safetensors.h:37-111).
struct Snapshot
{
    std::vector<std::unique_ptr<StFile>> files;
    std::map<std::string, StTensor> tensors;

    void open_dir(const std::string &dir)
    {
        DIR *d = opendir(dir.c_str());
        if (!d)
            fail(YLM_LOAD_ERROR, "Invalid model folder: %s", dir.c_str());
        std::vector<std::string> names;
        while (dirent *e = readdir(d))
        {
            std::string n = e->d_name;
            if (n.size() > 12 && n.substr(n.size() - 12) == ".safetensors")
                names.push_back(dir + "/" + n);
        }
        closedir(d);
        std::sort(names.begin(), names.end());
        if (names.empty())
            fail(YLM_LOAD_ERROR, "Folder (%s) has no model weight files", dir.c_str());
        for (auto &p : names)
            add_file(p);
    }

    void add_file(const std::string &path)
    {
        auto f = std::make_unique<StFile>();
        f->fd = ::open(path.c_str(), O_RDONLY);
        if (f->fd < 0)
            fail(YLM_LOAD_ERROR, "open failed: %s", path.c_str());
        struct stat sb;
        fstat(f->fd, &sb);
        f->size = (size_t)sb.st_size;
        if (f->size < 8)
            fail(YLM_LOAD_ERROR, "bad safetensors file: %s", path.c_str());
        f->map = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
        if (f->map == MAP_FAILED)
            fail(YLM_LOAD_ERROR, "mmap failed: %s", path.c_str());
        const uint8_t *base = static_cast<const uint8_t *>(f->map);
        uint64_t hlen;
        memcpy(&hlen, base, 8);
        if (hlen == 0 || hlen > (1ull << 30) || 8 + hlen > f->size)
            fail(YLM_LOAD_ERROR, "bad header size in %s", path.c_str());
        JVal h = json_parse(std::string(reinterpret_cast<const char *>(base + 8), hlen));
        const uint8_t *data = base + 8 + hlen;
        const size_t dsize = f->size - 8 - hlen;
        for (auto &kv : h.obj)
        {
            const JVal &v = kv.second;
            if (v.kind != JVal::Obj || !v.has("dtype") || !v.has("shape") || !v.has("data_offsets"))
                continue;
            StTensor t;
            t.dtype = v.get("dtype")->str;
            for (auto &s : v.get("shape")->arr)
                t.shape.push_back((int64_t)s.as_num());
            const auto &off = v.get("data_offsets")->arr;
            const size_t o0 = (size_t)off.at(0).as_num(), o1 = (size_t)off.at(1).as_num();
            if (o1 < o0 || o1 > dsize)
                fail(YLM_LOAD_ERROR, "tensor %s out of file bounds", kv.first.c_str());
            t.data = data + o0;
            t.bytes = o1 - o0;
            if (!tensors.count(kv.first))
                tensors[kv.first] = t;
        }
        files.push_back(std::move(f));
    }

    const StTensor *find(const std::string &n) const
    {
        auto it = tensors.find(n);
        return it == tensors.end() ? nullptr : &it->second;
    }
};

int dtype_code(const std::string &d)
{
    if (d == "F16")
        return 0;
    if (d == "BF16")
        return 1;
    if (d == "F32")
        return 2;
    fail(YLM_LOAD_ERROR, "unsupported dtype %s", d.c_str());
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

} // namespace

// ------------------------------------------------------------------ engine
struct ylm_engine
{
    ylm_model_config cfg{};
    ylm_engine_options opt{};
    int dev = 0, sms = 148;
    cudaStream_t st = nullptr;

    int H = 0, L = 0, D = YLM_HEAD_DIM, Hq = 0, Hkv = 0, hq = 0, hkv = 0, I = 0, inter = 0, qkv_rows = 0;
    int64_t V = 0, v_local = 0;
    int tp = 1, rank = 0;

    uint8_t *wblob = nullptr;
    size_t wbytes = 0;
    __half *emb = nullptr, *lm = nullptr, *fnorm = nullptr;
    struct Layer
    {
        __half *wqkv = nullptr, *bqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wd = nullptr;
        __half *ln1 = nullptr, *ln2 = nullptr, *qn = nullptr, *kn = nullptr;
        GemvPlan pq, po, pgu, pd;
        CUtensorMap tq, to, tgu, td; // tcgen05 operand maps of the four weights
    };
    std::vector<Layer> layers;
    GemvPlan plm;

    __half *kc = nullptr, *vc = nullptr;
    int cap = 0;
    size_t kv_layer = 0; // elements per layer (one of K or V)
    __half *rcos = nullptr, *rsin = nullptr;
    int max_pos = 0;

    // decode workspace
    __half *x = nullptr, *x2 = nullptr, *qkv = nullptr, *att = nullptr, *act = nullptr, *logits = nullptr,
           *logits_local = nullptr, *ar = nullptr;
    float *partial = nullptr;
    int *counters = nullptr;
    int splits = 1;
    StepState *dstate = nullptr, *hin = nullptr, *hout = nullptr;
    uint64_t *cand = nullptr;
    int *cand_count = nullptr, *smp_counter = nullptr;
    int parts = 1;
    int64_t *dbg_ids = nullptr;
    float *dbg_probs = nullptr;
    uint32_t *mask_bits = nullptr;

    // prefill workspace
    int pf_cap = 0;
    __half *pX = nullptr, *pXn = nullptr, *pQKV = nullptr, *pQ = nullptr, *pO = nullptr, *pA = nullptr;
    int64_t *pIds = nullptr;

    cudaGraphExec_t g_fwd = nullptr, g_fwd_sample = nullptr;
    cudaGraphExec_t g_fwd_greedy = nullptr; // persistent path, greedy pick fused into the lm_head
    unsigned long long *pick_cand = nullptr; // its per-CTA keys [sms]
    int *pick_counter = nullptr;

    // persistent GEMV segments (decode_step.cu): phase table, barrier counters,
    // one argument block per segment (layer 0's QKV; O, gate-up, down and the
    // next QKV per layer; the last ends with the lm_head)
    bool ds_on = false;
    bool ds_graph_ok = true; // cleared if the segment launches cannot be captured
    size_t ds_smem = 0;
    int ds_nph = 0;
    std::vector<DsPhase> ds_phases; // the step's GEMV phases (host copy)
    uint32_t *ds_mb_local[2] = {nullptr, nullptr};  // this rank's two mailbox sets [tp][H] (set 0: + [tp][4] pick slots)
    size_t ds_mb_words[2] = {0, 0};
    uint32_t **ds_pick_mb = nullptr;                 // device [tp]: every rank's pick slots, mapped here
    bool logits_partial = false;                     // tensor parallel: only this rank's logits rows are current
    std::vector<void *> ds_mb_peer;                  // peers' mailboxes mapped through CUDA IPC
    uint32_t *ds_xt = nullptr, *ds_actt = nullptr; // tagged residual stream and SwiGLU activations
    unsigned *ds_gen = nullptr;
    unsigned long long *ds_xstat = nullptr; // exchange timing (tensor parallel): ns, exchanges
    int64_t xstat_steps = 0;                // decode steps since the last reset of ds_xstat
    std::vector<DsArgs> ds_seg;
    std::vector<DsArgs> ds_seg_saved; // ylm_debug_drop_output: the segments as set up
    uint32_t *ds_sink = nullptr;      // where a dropped output goes

    bool ready = false;
    int last = 0;
    int max_seq = 0;
    bool has_logits = false;

    int greedy = 1, top_k = 40;
    float temp = 0.6f;
    uint64_t seed = 0;
    float u_next = -1.f;
    int64_t calls = 0;
    int last_k = 0;

    ncclComm_t comm = nullptr;
    cudaEvent_t ev_a = nullptr, ev_b = nullptr;
    StepState *hring[2] = {nullptr, nullptr}; // ylm_generate: step states read one step behind
    cudaEvent_t ev_ring[2] = {nullptr, nullptr};
    double prefill_ms = 0.0;

    ~ylm_engine() { release(); }

    void release()
    {
        if (dev >= 0)
            cudaSetDevice(dev);
        if (g_fwd)
            cudaGraphExecDestroy(g_fwd);
        if (g_fwd_sample)
            cudaGraphExecDestroy(g_fwd_sample);
        if (g_fwd_greedy)
            cudaGraphExecDestroy(g_fwd_greedy);
        g_fwd = g_fwd_sample = g_fwd_greedy = nullptr;
        for (void *pm : ds_mb_peer)
            cudaIpcCloseMemHandle(pm);
        ds_mb_peer.clear();
        for (uint32_t *&m : ds_mb_local)
        {
            if (m)
                cudaFree(m);
            m = nullptr;
        }
        if (comm)
            ncclCommDestroy(comm);
        comm = nullptr;
        if (ev_a)
            cudaEventDestroy(ev_a);
        if (ev_b)
            cudaEventDestroy(ev_b);
        ev_a = ev_b = nullptr;
        for (int k = 0; k < 2; k++)
        {
            if (ev_ring[k])
                cudaEventDestroy(ev_ring[k]);
            if (hring[k])
                cudaFreeHost(hring[k]);
            ev_ring[k] = nullptr;
            hring[k] = nullptr;
        }
        for (void *p : {(void *)wblob, (void *)kc, (void *)vc, (void *)rcos, (void *)rsin, (void *)x, (void *)x2,
                        (void *)qkv, (void *)att, (void *)act, (void *)logits, (void *)logits_local, (void *)ar,
                        (void *)partial, (void *)counters, (void *)dstate, (void *)cand, (void *)cand_count,
                        (void *)smp_counter, (void *)dbg_ids, (void *)dbg_probs, (void *)mask_bits, (void *)pX,
                        (void *)pXn, (void *)pQKV, (void *)pQ, (void *)pO, (void *)pA, (void *)pIds, (void *)ds_xt, (void *)ds_actt, (void *)ds_gen, (void *)ds_xstat,
                        (void *)ds_sink, (void *)pick_cand, (void *)pick_counter, (void *)ds_pick_mb})
            // logits_local is logits itself without tensor parallelism: free once
            if (p && !(p == (void *)logits_local && logits_local == logits))
                cudaFree(p);
        wblob = nullptr;
        kc = vc = nullptr;
        if (hin)
            cudaFreeHost(hin);
        if (hout)
            cudaFreeHost(hout);
        hin = hout = nullptr;
        if (st)
            cudaStreamDestroy(st);
        st = nullptr;
    }

    // Every engine buffer is used on the engine stream `st`, a non-blocking
    // stream: work on the legacy default stream (plain cudaMemset, cudaMemcpy)
    // is not ordered before it. So buffers are zeroed, and host data is copied
    // in, on `st` itself. (A zeroing on the default stream once raced the first
    // prefill of a new size, whose workspace it had just allocated.)
    template <typename T> T *dalloc(size_t n)
    {
        void *p = nullptr;
        CK(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
        CK(cudaMemsetAsync(p, 0, std::max<size_t>(n, 1) * sizeof(T), st));
        return static_cast<T *>(p);
    }

    // host -> device on the engine stream, complete on return (the source may be
    // pageable or reused right after)
    void h2d(void *dst, const void *src, size_t bytes)
    {
        CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, st));
        CK(cudaStreamSynchronize(st));
    }

    // device -> host on the engine stream, after the work already queued on it
    void d2h(void *dst, const void *src, size_t bytes)
    {
        CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
    }


    // -------------------------------------------------------------- set-up
    void init(const char *snapshot_dir, const ylm_model_config &c, const ylm_engine_options &o)
    {
        cfg = c;
        opt = o;
        dev = o.device;
        tp = std::max(1, o.tp_size);
        rank = o.tp_rank;
        H = c.hidden_size;
        L = c.num_layers;
        Hq = c.num_heads;
        Hkv = c.num_kv_heads;
        I = c.intermediate_size;
        V = c.vocab_size;
        if (c.head_dim != YLM_HEAD_DIM)
            fail(YLM_UNSUPPORTED, "head_dim %d: kernels are built for 128", c.head_dim);
        if (H <= 0 || L <= 0 || Hq <= 0 || Hkv <= 0 || I <= 0 || V <= 0 || Hq % Hkv)
            fail(YLM_INVALID_ARG, "invalid model shape");
        if (Hq / Hkv > 8)
            fail(YLM_UNSUPPORTED, "more than 8 query heads per KV head");
        if (H % 8 || I % 8)
            fail(YLM_UNSUPPORTED, "hidden and intermediate sizes must be multiples of 8");
        if (rank < 0 || rank >= tp || Hkv % tp || I % tp || V % tp)
            fail(YLM_INVALID_ARG, "tensor parallel %d does not divide KV heads, intermediate or vocab", tp);
        hq = Hq / tp;
        hkv = Hkv / tp;
        inter = I / tp;
        v_local = V / tp;
        qkv_rows = (hq + 2 * hkv) * D;

        CK(cudaSetDevice(dev));
        CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        CK(kernels_prepare());
        CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));

        if (tp > 1)
        {
            if (!o.nccl_id)
                fail(YLM_INVALID_ARG, "tp_size > 1 needs an NCCL unique id");
            ncclUniqueId id;
            memcpy(&id, o.nccl_id, sizeof(id));
            NK(ncclCommInitRank(&comm, tp, id, rank));
        }

        alloc_weights();
        if (snapshot_dir)
            load_weights(snapshot_dir);
        else
            random_weights();
        build_plans();
        alloc_kv();
        build_rope();
        alloc_workspace();
        setup_persistent();
        CK(cudaStreamSynchronize(st));
        compute_max_seq();
        CK(cudaStreamSynchronize(st));
    }

    void alloc_weights()
    {
        const bool bias = cfg.model_type == YLM_MODEL_QWEN2_5;
        const bool qkn = cfg.model_type == YLM_MODEL_QWEN3;
        size_t off = 0;
        auto take = [&](size_t elems) {
            size_t o = off;
            off = align_up(off + elems * 2, 256);
            return o;
        };
        struct Off
        {
            size_t wqkv, bqkv, wo, wgu, wd, ln1, ln2, qn, kn;
        };
        std::vector<Off> lo(L);
        const size_t o_emb = take((size_t)V * H);
        const size_t o_fn = take(H);
        const bool own_lm = !cfg.tie_word_embeddings || tp > 1;
        const size_t o_lm = own_lm ? take((size_t)v_local * H) : 0;
        for (int l = 0; l < L; l++)
        {
            lo[l].wqkv = take((size_t)qkv_rows * H);
            lo[l].bqkv = bias ? take(qkv_rows) : SIZE_MAX;
            lo[l].wo = take((size_t)H * hq * D);
            lo[l].wgu = take((size_t)2 * inter * H);
            lo[l].wd = take((size_t)H * inter);
            lo[l].ln1 = take(H);
            lo[l].ln2 = take(H);
            lo[l].qn = qkn ? take(D) : SIZE_MAX;
            lo[l].kn = qkn ? take(D) : SIZE_MAX;
        }
        wbytes = off;
        CK(cudaMalloc(&wblob, wbytes));
        auto P = [&](size_t o) { return o == SIZE_MAX ? nullptr : reinterpret_cast<__half *>(wblob + o); };
        emb = P(o_emb);
        fnorm = P(o_fn);
        lm = own_lm ? P(o_lm) : emb;
        layers.resize(L);
        for (int l = 0; l < L; l++)
        {
            Layer &y = layers[l];
            y.wqkv = P(lo[l].wqkv);
            y.bqkv = P(lo[l].bqkv);
            y.wo = P(lo[l].wo);
            y.wgu = P(lo[l].wgu);
            y.wd = P(lo[l].wd);
            y.ln1 = P(lo[l].ln1);
            y.ln2 = P(lo[l].ln2);
            y.qn = P(lo[l].qn);
            y.kn = P(lo[l].kn);
        }
    }

    // Each destination block of a weight: rows [r0, r0+nr) and columns [c0, c0+nc)
    // of the HF tensor `name`, written with row pitch `ld` (elements).
    struct Piece
    {
        std::string name;
        __half *dst;
        int64_t r0, nr, c0, nc, ld;
        bool ones; // norm weight
    };

    std::vector<Piece> pieces()
    {
        std::vector<Piece> ps;
        const bool bias = cfg.model_type == YLM_MODEL_QWEN2_5;
        const bool qkn = cfg.model_type == YLM_MODEL_QWEN3;
        ps.push_back({"model.embed_tokens.weight", emb, 0, V, 0, H, H, false});
        ps.push_back({"model.norm.weight", fnorm, 0, 1, 0, H, H, true});
        if (lm != emb)
        {
            const char *nm = cfg.tie_word_embeddings ? "model.embed_tokens.weight" : "lm_head.weight";
            ps.push_back({nm, lm, rank * v_local, v_local, 0, H, H, false});
        }
        for (int l = 0; l < L; l++)
        {
            const std::string p = "model.layers." + std::to_string(l) + ".";
            Layer &y = layers[l];
            const int64_t q0 = (int64_t)rank * hq * D, k0 = (int64_t)rank * hkv * D;
            ps.push_back({p + "self_attn.q_proj.weight", y.wqkv, q0, hq * D, 0, H, H, false});
            ps.push_back({p + "self_attn.k_proj.weight", y.wqkv + (size_t)hq * D * H, k0, hkv * D, 0, H, H, false});
            ps.push_back({p + "self_attn.v_proj.weight", y.wqkv + (size_t)(hq + hkv) * D * H, k0, hkv * D, 0, H, H,
                          false});
            if (bias)
            {
                ps.push_back({p + "self_attn.q_proj.bias", y.bqkv, 0, 1, q0, hq * D, hq * D, false});
                ps.push_back({p + "self_attn.k_proj.bias", y.bqkv + hq * D, 0, 1, k0, hkv * D, hkv * D, false});
                ps.push_back({p + "self_attn.v_proj.bias", y.bqkv + (hq + hkv) * D, 0, 1, k0, hkv * D, hkv * D, false});
            }
            if (qkn)
            {
                ps.push_back({p + "self_attn.q_norm.weight", y.qn, 0, 1, 0, D, D, true});
                ps.push_back({p + "self_attn.k_norm.weight", y.kn, 0, 1, 0, D, D, true});
            }
            ps.push_back({p + "self_attn.o_proj.weight", y.wo, 0, H, q0, hq * D, hq * D, false});
            ps.push_back({p + "input_layernorm.weight", y.ln1, 0, 1, 0, H, H, true});
            ps.push_back({p + "post_attention_layernorm.weight", y.ln2, 0, 1, 0, H, H, true});
            // gate and up interleaved by row: row 2j = gate_j, row 2j+1 = up_j
            const int64_t i0 = (int64_t)rank * inter;
            ps.push_back({p + "mlp.gate_proj.weight", y.wgu, i0, inter, 0, H, 2 * (int64_t)H, false});
            ps.push_back({p + "mlp.up_proj.weight", y.wgu + H, i0, inter, 0, H, 2 * (int64_t)H, false});
            ps.push_back({p + "mlp.down_proj.weight", y.wd, 0, H, i0, inter, inter, false});
        }
        return ps;
    }

    void random_weights()
    {
        const double stdv = opt.init_std > 0 ? opt.init_std : 0.02;
        for (auto &p : pieces())
        {
            if (p.ones)
            {
                CK(fill_const_launch(p.dst, p.nc, 1.0f, st));
                continue;
            }
            // full column count of the HF tensor: 1-D tensors (biases) are one row
            int64_t full_cols;
            if (p.name.find("o_proj") != std::string::npos)
                full_cols = (int64_t)Hq * D;
            else if (p.name.find("down_proj") != std::string::npos)
                full_cols = I;
            else if (p.name.find(".bias") != std::string::npos)
                full_cols = p.name.find("q_proj") != std::string::npos ? (int64_t)Hq * D : (int64_t)Hkv * D;
            else
                full_cols = H;
            const uint64_t key = mix64(opt.init_seed) ^ fnv1a64(p.name);
            CK(fill_normal_launch(p.dst, p.nr, p.nc, p.ld, key, p.r0, p.c0, full_cols, stdv, st));
        }
    }

    // Row bands of every piece move through a ring of pinned host buffers:
    // host threads copy band k out of the mapped shard (the page faults of a
    // cold file are spread over them) while the engine stream copies earlier
    // bands to the device; BF16 / F32 bands land in a device staging buffer
    // and are converted to FP16 there (round to nearest even, as on the host).
    // Each piece's slice is read straight from the mapping: a rank's rows or
    // columns only (tensor parallelism).
    void load_weights(const char *dir)
    {
        Snapshot snap;
        snap.open_dir(dir);
        constexpr int NB = 3;
        constexpr size_t CH = (size_t)64 << 20;
        struct Ring
        {
            void *host[NB] = {}, *dev[NB] = {};
            cudaEvent_t ev[NB] = {};
            bool used[NB] = {};
            ~Ring()
            {
                for (int k = 0; k < NB; k++)
                {
                    if (ev[k])
                    {
                        cudaEventSynchronize(ev[k]);
                        cudaEventDestroy(ev[k]);
                    }
                    if (host[k])
                        cudaFreeHost(host[k]);
                    if (dev[k])
                        cudaFree(dev[k]);
                }
            }
        } ring;
        for (int k = 0; k < NB; k++)
        {
            CK(cudaHostAlloc(&ring.host[k], CH, cudaHostAllocDefault));
            CK(cudaMalloc(&ring.dev[k], CH));
            CK(cudaEventCreateWithFlags(&ring.ev[k], cudaEventDisableTiming));
        }
        const unsigned hc = std::thread::hardware_concurrency();
        const int nthreads = (int)std::max(1u, std::min(8u, hc ? hc : 1u));
        int k = 0;
        for (auto &p : pieces())
        {
            const StTensor *t = snap.find(p.name);
            if (!t)
                fail(YLM_LOAD_ERROR, "missing tensor %s", p.name.c_str());
            const int dc = dtype_code(t->dtype);
            const size_t es = dc == 2 ? 4 : 2;
            int64_t rows = 1, cols = 1;
            if (t->shape.size() == 2)
            {
                rows = t->shape[0];
                cols = t->shape[1];
            }
            else if (t->shape.size() == 1)
                cols = t->shape[0];
            else
                fail(YLM_LOAD_ERROR, "tensor %s: rank %zu", p.name.c_str(), t->shape.size());
            if (p.r0 + p.nr > rows || p.c0 + p.nc > cols || (size_t)(rows * cols) * es != t->bytes)
                fail(YLM_LOAD_ERROR, "tensor %s: shape does not match the model config", p.name.c_str());
            const size_t row_bytes = (size_t)p.nc * es, src_stride = (size_t)cols * es;
            if (row_bytes > CH)
                fail(YLM_LOAD_ERROR, "tensor %s: rows wider than the staging buffer", p.name.c_str());
            const uint8_t *src = t->data + ((size_t)p.r0 * cols + p.c0) * es;
            const int64_t band = std::min<int64_t>(65535, std::max<int64_t>(1, (int64_t)(CH / row_bytes)));
            for (int64_t r = 0; r < p.nr; r += band)
            {
                const int64_t nr = std::min(band, p.nr - r);
                if (ring.used[k])
                    CK(cudaEventSynchronize(ring.ev[k]));
                uint8_t *hb = static_cast<uint8_t *>(ring.host[k]);
                const uint8_t *s0 = src + (size_t)r * src_stride;
                auto copy_rows = [&](int64_t a, int64_t b) {
                    if (row_bytes == src_stride)
                        memcpy(hb + (size_t)a * row_bytes, s0 + (size_t)a * src_stride, (size_t)(b - a) * row_bytes);
                    else
                        for (int64_t i = a; i < b; i++)
                            memcpy(hb + (size_t)i * row_bytes, s0 + (size_t)i * src_stride, row_bytes);
                };
                const int nt = (int)std::min<int64_t>(nthreads, std::max<int64_t>(1, (int64_t)(nr * row_bytes >> 22)));
                if (nt <= 1)
                    copy_rows(0, nr);
                else
                {
                    std::vector<std::thread> th;
                    for (int q = 0; q < nt; q++)
                        th.emplace_back(copy_rows, nr * q / nt, nr * (q + 1) / nt);
                    for (auto &x : th)
                        x.join();
                }
                if (dc == 0)
                    CK(cudaMemcpy2DAsync(p.dst + (size_t)r * p.ld, p.ld * 2, hb, row_bytes, row_bytes, nr,
                                         cudaMemcpyHostToDevice, st));
                else
                {
                    CK(cudaMemcpyAsync(ring.dev[k], hb, (size_t)nr * row_bytes, cudaMemcpyHostToDevice, st));
                    CK(convert_rows_launch(ring.dev[k], dc, nr, p.nc, p.dst + (size_t)r * p.ld, p.ld, st));
                }
                CK(cudaEventRecord(ring.ev[k], st));
                ring.used[k] = true;
                k = (k + 1) % NB;
            }
        }
        CK(cudaStreamSynchronize(st));
    }

    void build_plans()
    {
        for (auto &y : layers)
        {
            if (!gemv_make_plan(&y.pq, y.wqkv, qkv_rows, H, 0, sms) || !gemv_make_plan(&y.po, y.wo, H, hq * D, 0, sms) ||
                !gemv_make_plan(&y.pgu, y.wgu, 2 * inter, H, 1, sms) || !gemv_make_plan(&y.pd, y.wd, H, inter, 0, sms))
                fail(YLM_UNSUPPORTED, "GEMV plan failed (tensor map encode)");
        }
        if (!gemv_make_plan(&plm, lm, (int)v_local, H, 0, sms))
            fail(YLM_UNSUPPORTED, "GEMV plan failed for lm_head");
        for (auto &y : layers)
            if (!tc_make_w_map(&y.tq, y.wqkv, qkv_rows, H) || !tc_make_w_map(&y.to, y.wo, H, hq * D) ||
                !tc_make_w_map(&y.tgu, y.wgu, 2 * inter, H) || !tc_make_w_map(&y.td, y.wd, H, inter))
                fail(YLM_UNSUPPORTED, "tensor map encode failed for a prefill weight");
    }

    // ModelBase::InitKVCache (ModelBase.cpp:340-370): capacity from the GB
    // budget with BF16-sized slots; this rank holds its KV heads for every slot.
    void alloc_kv()
    {
        const size_t total = (size_t)((double)std::max(1, opt.kv_cache_gb) * 1024.0 * 1024.0 * 1024.0);
        const size_t per_token = (size_t)Hkv * D * 2;
        cap = (int)((total / per_token) / (size_t)L / 2);
        kv_layer = (size_t)hkv * cap * D;
        kc = dalloc<__half>(kv_layer * L);
        vc = dalloc<__half>(kv_layer * L);
    }

    // ModelBase::BuildRopeCache (ModelBase.cpp:372-394), half-width tables
    // [max_pos][64] (the two halves of cat(freqs, freqs) are equal).
    void build_rope()
    {
        max_pos = cfg.max_position_embeddings;
        const int half = D / 2;
        std::vector<float> inv(half);
        for (int i = 0; i < half; i++)
        {
            const float e = (float)i / (float)half;
            inv[i] = (float)(1.0 / std::pow((double)cfg.rope_theta, (double)e));
        }
        if (opt.rope_scaling && cfg.rope_factor > 0 && cfg.rope_orig_max_pos > 0)
        {
            // Llama 3.1 frequency scaling (published with the Llama 3.1 release)
            const double f = cfg.rope_factor, lo = cfg.rope_low_freq, hi = cfg.rope_high_freq;
            const double orig = cfg.rope_orig_max_pos;
            const double lo_wl = orig / lo, hi_wl = orig / hi;
            for (int i = 0; i < half; i++)
            {
                const double v = inv[i];
                const double wl = 2.0 * M_PI / v;
                double out = wl > lo_wl ? v / f : v;
                if (wl <= lo_wl && wl >= hi_wl)
                {
                    const double sm = (orig / wl - lo) / (hi - lo);
                    out = (1.0 - sm) * v / f + sm * v;
                }
                inv[i] = (float)out;
            }
        }
        std::vector<__half> hc((size_t)max_pos * half), hs((size_t)max_pos * half);
        for (int p = 0; p < max_pos; p++)
            for (int i = 0; i < half; i++)
            {
                const float a = (float)p * inv[i];
                hc[(size_t)p * half + i] = __float2half_rn((float)std::cos((double)a));
                hs[(size_t)p * half + i] = __float2half_rn((float)std::sin((double)a));
            }
        rcos = dalloc<__half>(hc.size());
        rsin = dalloc<__half>(hs.size());
        h2d(rcos, hc.data(), hc.size() * 2);
        h2d(rsin, hs.data(), hs.size() * 2);
    }

    void alloc_workspace()
    {
        x = dalloc<__half>(H);
        x2 = dalloc<__half>(H);
        qkv = dalloc<__half>(qkv_rows);
        att = dalloc<__half>((size_t)hq * D);
        act = dalloc<__half>(inter);
        logits = dalloc<__half>(V);
        logits_local = tp > 1 ? dalloc<__half>(v_local) : logits;
        ar = dalloc<__half>(H);
        splits = attn_default_splits(hkv, sms);
        partial = dalloc<float>(attn_partial_floats(hq, splits));
        counters = dalloc<int>(hkv);
        dstate = dalloc<StepState>(1);
        CK(cudaMallocHost(&hin, sizeof(StepState)));
        CK(cudaMallocHost(&hout, sizeof(StepState)));
        memset(hin, 0, sizeof(StepState));
        memset(hout, 0, sizeof(StepState));
        parts = sample_parts(V, sms);
        cand = dalloc<uint64_t>((size_t)parts * 64);
        cand_count = dalloc<int>(parts);
        smp_counter = dalloc<int>(1);
        dbg_ids = dalloc<int64_t>(64);
        dbg_probs = dalloc<float>(64);
    }

    // Persistent GEMV segments: one launch of one CTA per SM per run of
    // projections between two attention launches, where the device can keep
    // one CTA per SM resident; otherwise the per-op graph. With tensor
    // parallelism the O and down epilogues all-reduce through peer mailboxes.
    void setup_persistent()
    {
        ds_on = false;
        if (!opt.decode_persistent || tp > 8)
            return;
        ds_xt = dalloc<uint32_t>(H);
        ds_actt = dalloc<uint32_t>(inter);
        std::vector<DsPhase> ph;
        // in: plain input from an earlier launch; it/src: tagged input written by phase src
        auto gemv = [&](int pro, int epi, const __half *w, int N, int K, const __half *in, const uint32_t *it,
                        int src, const __half *nw, __half *out, uint32_t *out_t, const __half *bias) {
            DsPhase p{};
            p.pro = pro;
            p.epi = epi;
            p.w = w;
            p.N = N;
            p.K = K;
            p.x = in;
            p.xt = it;
            p.src = src;
            p.norm_w = nw;
            p.out = out;
            p.out_t = out_t;
            p.bias = bias;
            p.resid_t = ds_xt;
            ph.push_back(p);
            return (int)ph.size() - 1;
        };
        // phase order: QKV0 | O0 GU0 D0 QKV1 | ... | O(L-1) GU D lm_head
        std::vector<int> cut; // segment boundaries
        cut.push_back(0);
        int down = -1; // the phase that last wrote the residual stream
        for (int l = 0; l < L; l++)
        {
            Layer &y = layers[l];
            if (l == 0)
                gemv(PRO_EMBED_RMSNORM, EPI_STORE, y.wqkv, qkv_rows, H, nullptr, nullptr, 0, y.ln1, qkv, nullptr,
                     y.bqkv);
            else
                gemv(PRO_RMSNORM, EPI_STORE, y.wqkv, qkv_rows, H, nullptr, ds_xt, down, y.ln1, qkv, nullptr, y.bqkv);
            cut.push_back((int)ph.size()); // attention of layer l runs here
            const int o = gemv(PRO_VEC, EPI_RESID, y.wo, H, hq * D, att, nullptr, 0, nullptr, nullptr, nullptr, nullptr);
            ph[o].mbox = tp > 1 ? 1 : 0; // all-reduce of the O partials (tensor parallel)
            const int gu = gemv(PRO_RMSNORM, EPI_SWIGLU, y.wgu, 2 * inter, H, nullptr, ds_xt, o, y.ln2, nullptr, ds_actt,
                                nullptr);
            down = gemv(PRO_VEC, EPI_RESID, y.wd, H, inter, nullptr, ds_actt, gu, nullptr, nullptr, nullptr, nullptr);
            ph[down].mbox = tp > 1 ? 2 : 0;
        }
        gemv(PRO_RMSNORM, EPI_STORE, lm, (int)v_local, H, nullptr, ds_xt, down, fnorm, logits_local, nullptr, nullptr);
        cut.push_back((int)ph.size());
        const int C = sms;
        if ((H + C - 1) / C > ds_threads())
            return; // each thread seeds at most one residual row
        const int kc_cols = ds_task_cols();
        int kpad_max = 0, part_max = 0;
        for (const DsPhase &p : ph)
        {
            const int nkc = (p.K + kc_cols - 1) / kc_cols;
            kpad_max = std::max(kpad_max, nkc * kc_cols);
            const int rows = p.epi == EPI_SWIGLU ? 2 * ((p.N / 2 + C - 1) / C) : (p.N + C - 1) / C;
            part_max = std::max(part_max, rows * nkc);
        }
        const int nph = (int)ph.size();
        for (size_t k = 0; k + 1 < cut.size(); k++)
            if (cut[k + 1] - cut[k] > DS_MAX_SEG_PHASES)
                return;
        const size_t tab_bytes = (size_t)ds_tab_bytes();
        const size_t work_bytes = ((size_t)kpad_max * 2 + (size_t)part_max * 4 + 32 * 4 + 15) & ~(size_t)15;
        const size_t xr_bytes = ((size_t)(H + C - 1) / C * 2 + 15) & ~(size_t)15;
        const size_t smem = tab_bytes + work_bytes + xr_bytes;
        if (smem > 220 * 1024)
            return;
        int bps = 0;
        if (ds_prepare(smem, &bps) != cudaSuccess || bps < 1)
        {
            cudaGetLastError();
            return;
        }
        ds_gen = dalloc<unsigned>(1);
        pick_cand = dalloc<unsigned long long>(C);
        pick_counter = dalloc<int>(1);
        DsArgs d{};
        d.nph = nph;
        d.tp = tp;
        d.rank = rank;
        if (tp > 1)
        {
            setup_mailboxes(d);
            ds_xstat = dalloc<unsigned long long>(2);
            d.xstat = ds_xstat;
        }
        d.eps = cfg.rms_eps;
        d.emb = emb;
        d.vocab = V;
        d.state = dstate;
        d.xt = ds_xt;
        d.hidden = H;
        d.gen = ds_gen;
        d.err = &dstate->err;
        d.wait_ns = opt.wait_limit_us > 0 ? (unsigned long long)opt.wait_limit_us * 1000ull : 2000000000ull;
        d.tab_bytes = (int)tab_bytes;
        d.work_bytes = (int)work_bytes;
        d.kpad_max = kpad_max;
        d.part_max = part_max;
        ds_seg.clear();
        ds_phases = ph;
        for (size_t k = 0; k + 1 < cut.size(); k++)
        {
            d.p0 = cut[k];
            d.p1 = cut[k + 1];
            d.last = k + 2 == cut.size() ? 1 : 0;
            for (int i = d.p0; i < d.p1; i++)
                d.ph[i - d.p0] = ph[i];
            ds_seg.push_back(d);
        }
        ds_nph = nph;
        ds_smem = smem;
        ds_on = true;
    }

    // Tensor parallel all-reduce mailboxes: two sets of [tp][H] tagged words
    // per rank; every rank maps every peer's through CUDA IPC (handles
    // exchanged with one NCCL all-gather), and writes its partials into slot
    // `rank` of each with plain peer stores over NVLink.
    void setup_mailboxes(DsArgs &d)
    {
        cudaIpcMemHandle_t mine[2];
        for (int s = 0; s < 2; s++)
        {
            ds_mb_words[s] = (size_t)tp * H + (s == 0 ? 4 * (size_t)tp : 0);
            ds_mb_local[s] = dalloc<uint32_t>(ds_mb_words[s]);
            CK(cudaIpcGetMemHandle(&mine[s], ds_mb_local[s]));
        }
        char *dsend = dalloc<char>(sizeof(mine));
        char *drecv = dalloc<char>(sizeof(mine) * tp);
        h2d(dsend, mine, sizeof(mine));
        NK(ncclAllGather(dsend, drecv, sizeof(mine), ncclChar, comm, st));
        CK(cudaStreamSynchronize(st));
        std::vector<cudaIpcMemHandle_t> all(2 * (size_t)tp);
        d2h(all.data(), drecv, sizeof(mine) * tp);
        cudaFree(dsend);
        cudaFree(drecv);
        for (int s = 0; s < 2; s++)
            for (int q = 0; q < tp; q++)
            {
                if (q == rank)
                {
                    d.mb[s][q] = ds_mb_local[s];
                    continue;
                }
                void *pm = nullptr;
                CK(cudaIpcOpenMemHandle(&pm, all[2 * (size_t)q + s], cudaIpcMemLazyEnablePeerAccess));
                ds_mb_peer.push_back(pm);
                d.mb[s][q] = static_cast<uint32_t *>(pm);
            }
        // greedy pick slots: after the [tp][H] partials of set 0
        std::vector<uint32_t *> pm(tp);
        for (int q = 0; q < tp; q++)
            pm[q] = d.mb[0][q] + (size_t)tp * H;
        ds_pick_mb = dalloc<uint32_t *>(tp);
        h2d(ds_pick_mb, pm.data(), sizeof(uint32_t *) * tp);
    }

    // Clear the persistent path's step generation and tagged activations, so no
    // word left by a failed or timing launch can match a coming tag.
    void ds_reset()
    {
        cudaMemsetAsync(ds_gen, 0, sizeof(unsigned), st);
        cudaMemsetAsync(ds_xt, 0, sizeof(uint32_t) * H, st);
        cudaMemsetAsync(ds_actt, 0, sizeof(uint32_t) * inter, st);
        if (pick_counter)
            cudaMemsetAsync(pick_counter, 0, sizeof(int), st);
        for (int s = 0; s < 2; s++)
            if (ds_mb_local[s])
                cudaMemsetAsync(ds_mb_local[s], 0, sizeof(uint32_t) * ds_mb_words[s], st);
    }

    // ModelBase::CalculateMaxSequenceLength (ModelBase.cpp:312-338)
    void compute_max_seq()
    {
        size_t fr = 0, to = 0;
        CK(cudaMemGetInfo(&fr, &to));
        const size_t per_tok = (size_t)Hq * D * 2 * 3 * L;
        const long long by_mem = (long long)((double)fr * 0.8 / (double)per_tok);
        max_seq = (int)std::min<long long>(cfg.max_position_embeddings, by_mem);
        if (max_seq < 512)
            fail(YLM_LOAD_ERROR, "GPU memory too low: runtime cannot support the minimum context of 512 tokens");
    }

    void ensure_prefill(int T)
    {
        if (T <= pf_cap)
            return;
        int n = std::max(T, 64);
        for (void *p : {(void *)pX, (void *)pXn, (void *)pQKV, (void *)pQ, (void *)pO, (void *)pA, (void *)pIds})
            if (p)
                cudaFree(p);
        pX = dalloc<__half>((size_t)n * H);
        pXn = dalloc<__half>((size_t)n * H);
        pQKV = dalloc<__half>((size_t)n * qkv_rows);
        pQ = dalloc<__half>((size_t)n * hq * D);
        pO = dalloc<__half>((size_t)n * std::max(hq * D, H));
        pA = dalloc<__half>((size_t)n * inter);
        pIds = dalloc<int64_t>(n);
        pf_cap = n;
    }

    // -------------------------------------------------------------- decode step
    AttnArgs attn_args(int l)
    {
        AttnArgs a;
        a.qkv = qkv;
        a.q_norm = layers[l].qn;
        a.k_norm = layers[l].kn;
        a.eps = cfg.rms_eps;
        a.rope_cos = rcos;
        a.rope_sin = rsin;
        a.max_pos = max_pos;
        a.k_cache = kc + (size_t)l * kv_layer;
        a.v_cache = vc + (size_t)l * kv_layer;
        a.cap = cap;
        a.hq = hq;
        a.hkv = hkv;
        a.splits = splits;
        a.partial = partial;
        a.counters = counters;
        a.out = att;
        a.state = dstate;
        a.err = &dstate->err;
        return a;
    }

    // what a decode step ends with: nothing, the sampler kernel, or (persistent
    // path on one GPU, greedy) the argmax fused into the lm_head epilogue
    enum { STEP_NO_SAMPLE = 0, STEP_SAMPLER = 1, STEP_GREEDY_FUSED = 2 };

    int step_mode(bool sample, bool greedy) const
    {
        if (!sample)
            return STEP_NO_SAMPLE;
        return greedy && ds_on && pick_counter ? STEP_GREEDY_FUSED : STEP_SAMPLER;
    }

    void enqueue_forward(int mode)
    {
        const bool sample = mode != STEP_NO_SAMPLE;
        if (ds_on)
        {
            // segment 0 (layer 0's QKV), then attention l and segment l + 1
            for (int l = 0; l <= L; l++)
            {
                if (l == L && mode == STEP_GREEDY_FUSED)
                {
                    DsArgs d = ds_seg[l];
                    d.ph[d.p1 - 1 - d.p0].greedy_pick = 1; // the lm_head phase
                    d.pick_state = dstate;
                    d.pick_cand = pick_cand;
                    d.pick_counter = pick_counter;
                    d.pick_mb = tp > 1 ? ds_pick_mb : nullptr;
                    CK(ds_launch(d, ds_smem, sms, st));
                    return;
                }
                CK(ds_launch(ds_seg[l], ds_smem, sms, st));
                if (l < L)
                    CK(attn_decode_launch(attn_args(l), st, false));
            }
            if (tp > 1)
                NK(ncclAllGather(logits_local, logits, v_local, ncclHalf, comm, st));
            if (sample)
                CK(sample_launch(sample_args(), st, false));
            return;
        }
        // use_pdl: 1 every kernel may start early; 2 only the projections (the
        // attention and the sampler wait for their producer to finish); 0 none
        const bool pdl = opt.use_pdl != 0;
        const bool pdl_other = opt.use_pdl == 1;
        int *err = &dstate->err;
        for (int l = 0; l < L; l++)
        {
            Layer &y = layers[l];
            GemvArgs a;
            a.x = x;
            a.norm_w = y.ln1;
            a.eps = cfg.rms_eps;
            a.emb = emb;
            a.vocab = V;
            a.state = dstate;
            a.resid_out = x;
            a.out = qkv;
            a.bias = y.bqkv;
            a.err = err;
            CK(gemv_launch(y.pq, l == 0 ? PRO_EMBED_RMSNORM : PRO_RMSNORM, EPI_STORE, a, st, pdl));
            CK(attn_decode_launch(attn_args(l), st, pdl_other));
            GemvArgs o;
            o.x = att;
            o.err = err;
            if (tp == 1)
            {
                o.resid = x;
                CK(gemv_launch(y.po, PRO_VEC, EPI_RESID, o, st, pdl));
            }
            else
            {
                o.out = ar;
                CK(gemv_launch(y.po, PRO_VEC, EPI_STORE, o, st, pdl));
                NK(ncclAllReduce(ar, ar, H, ncclHalf, ncclSum, comm, st));
                CK(resid_add_launch(x, ar, H));
            }
            GemvArgs g;
            g.x = x;
            g.norm_w = y.ln2;
            g.eps = cfg.rms_eps;
            g.out = act;
            g.err = err;
            CK(gemv_launch(y.pgu, PRO_RMSNORM, EPI_SWIGLU, g, st, pdl));
            GemvArgs d;
            d.x = act;
            d.err = err;
            if (tp == 1)
            {
                d.resid = x;
                CK(gemv_launch(y.pd, PRO_VEC, EPI_RESID, d, st, pdl));
            }
            else
            {
                d.out = ar;
                CK(gemv_launch(y.pd, PRO_VEC, EPI_STORE, d, st, pdl));
                NK(ncclAllReduce(ar, ar, H, ncclHalf, ncclSum, comm, st));
                CK(resid_add_launch(x, ar, H));
            }
        }
        GemvArgs f;
        f.x = x;
        f.norm_w = fnorm;
        f.eps = cfg.rms_eps;
        f.out = logits_local;
        f.err = err;
        CK(gemv_launch(plm, PRO_RMSNORM, EPI_STORE, f, st, pdl));
        if (tp > 1)
            NK(ncclAllGather(logits_local, logits, v_local, ncclHalf, comm, st));
        if (sample)
            CK(sample_launch(sample_args(), st, pdl_other));
    }

    cudaError_t resid_add_launch(__half *xx, const __half *y, int64_t n)
    {
        return resid_add_rows_launch(xx, y, n, st);
    }

    SampleArgs sample_args()
    {
        SampleArgs s;
        s.logits = logits;
        s.vocab = V;
        s.mask_bits = mask_bits;
        s.state = dstate;
        s.cand = cand;
        s.cand_count = cand_count;
        s.counter = smp_counter;
        s.parts = parts;
        s.dbg_ids = dbg_ids;
        s.dbg_probs = dbg_probs;
        s.err = &dstate->err;
        return s;
    }

    cudaGraphExec_t capture(int mode)
    {
        cudaGraph_t g = nullptr;
        CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        try
        {
            enqueue_forward(mode);
        }
        catch (...)
        {
            cudaStreamEndCapture(st, &g);
            if (g)
                cudaGraphDestroy(g);
            throw;
        }
        CK(cudaStreamEndCapture(st, &g));
        cudaGraphExec_t ex = nullptr;
        cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        CK(e);
        return ex;
    }

    cudaGraphExec_t &graph_for(int mode)
    {
        return mode == STEP_GREEDY_FUSED ? g_fwd_greedy : (mode == STEP_SAMPLER ? g_fwd_sample : g_fwd);
    }

    // one decode step; `greedy`: the sample (if any) is an argmax
    void launch_forward(bool sample, bool greedy = false)
    {
        xstat_steps++;
        const int mode = step_mode(sample, greedy);
        // the fused greedy pick exchanges each rank's best candidate instead of
        // gathering the logits rows: until gather_logits(), each rank holds its own
        logits_partial = tp > 1 && mode == STEP_GREEDY_FUSED;
        if (ds_on && opt.use_cuda_graph && ds_graph_ok)
        {
            cudaGraphExec_t &ex = graph_for(mode);
            if (!ex)
            {
                try
                {
                    ex = capture(mode);
                }
                catch (...)
                {
                    // segment launches that do not capture: launch them directly
                    ds_graph_ok = false;
                    ex = nullptr;
                    cudaGetLastError();
                }
            }
            if (ex)
            {
                CK(cudaGraphLaunch(ex, st));
                return;
            }
        }
        if (ds_on)
        {
            enqueue_forward(mode);
            return;
        }
        if (opt.use_cuda_graph)
        {
            cudaGraphExec_t &ex = graph_for(mode);
            if (!ex)
                ex = capture(mode);
            CK(cudaGraphLaunch(ex, st));
        }
        else
            enqueue_forward(mode);
    }

    void fill_state(int64_t token, int slot, int pos, bool do_greedy, int advance)
    {
        hin->token = token;
        hin->next_token = -1;
        hin->sample_calls = calls;
        hin->slot = slot;
        hin->rope_pos = pos;
        hin->err = 0;
        hin->greedy = do_greedy ? 1 : 0;
        hin->top_k = std::max(1, std::min(top_k, 64));
        hin->inv_temp = 1.0f / temp;
        hin->u_override = u_next;
        hin->advance = advance;
        hin->seed = seed;
        hin->u_used = -1.f;
    }

    void push_state() { CK(cudaMemcpyAsync(dstate, hin, sizeof(StepState), cudaMemcpyHostToDevice, st)); }

    void ensure_ring()
    {
        for (int k = 0; k < 2; k++)
        {
            if (!hring[k])
                CK(cudaMallocHost(&hring[k], sizeof(StepState)));
            if (!ev_ring[k])
                CK(cudaEventCreateWithFlags(&ev_ring[k], cudaEventDisableTiming));
        }
    }


    void pull_state_sync()
    {
        CK(cudaMemcpyAsync(hout, dstate, sizeof(StepState), cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        check_dev_err();
    }

    void check_dev_err()
    {
        if (hout->err != 0)
        {
            const int e = hout->err;
            // counters may be left mid-step: reset them so the next step starts clean
            cudaMemsetAsync(counters, 0, sizeof(int) * hkv, st);
            cudaMemsetAsync(smp_counter, 0, sizeof(int), st);
            if (ds_gen)
                ds_reset(); // (clears the fused pick's counter too)
            cudaStreamSynchronize(st);
            if (e == YLM_DEV_ERR_BAD_TOKEN)
                fail(YLM_INVALID_ARG, "token id out of range");
            if (e == YLM_DEV_ERR_BAD_STATE)
                fail(YLM_INVALID_ARG, "slot or RoPE position out of range");
            fail(YLM_DEVICE_TIMEOUT, "device wait expired (code %d)", e);
        }
    }

    // -------------------------------------------------------------- prefill
    // one prefill GEMM: tcgen05 (default) or CUDA cores
    void pgemm(const __half *A, const CUtensorMap &am, int lda, const __half *W, const CUtensorMap &wm, int T, int N,
               int K, int epi, const __half *bias, __half *C, int ldc)
    {
        if (opt.prefill_tensor_cores)
            CK(gemm_tc_launch(am, wm, T, N, K, epi, bias, C, ldc, &dstate->err, st));
        else
            CK(gemm_launch(A, lda, W, T, N, K, epi, bias, C, ldc, st));
    }

    void run_prefill(int T)
    {
        const float eps = cfg.rms_eps;
        int *err = &dstate->err;
        CUtensorMap m_xn, m_o, m_a;
        if (!tc_make_a_map(&m_xn, pXn, T, H, H) || !tc_make_a_map(&m_o, pO, T, hq * D, hq * D) ||
            !tc_make_a_map(&m_a, pA, T, inter, inter))
            fail(YLM_UNSUPPORTED, "tensor map encode failed for a prefill activation");
        CK(embed_rows_launch(pIds, T, emb, V, H, pX, err, st));
        for (int l = 0; l < L; l++)
        {
            Layer &y = layers[l];
            __half *kl = kc + (size_t)l * kv_layer, *vl = vc + (size_t)l * kv_layer;
            CK(rmsnorm_rows_launch(pX, y.ln1, eps, T, H, pXn, st));
            pgemm(pXn, m_xn, H, y.wqkv, y.tq, T, qkv_rows, H, GEMM_STORE, y.bqkv, pQKV, qkv_rows);
            QkvPostArgs q;
            q.qkv = pQKV;
            q.q_norm = y.qn;
            q.k_norm = y.kn;
            q.eps = eps;
            q.rope_cos = rcos;
            q.rope_sin = rsin;
            q.q_out = pQ;
            q.k_cache = kl;
            q.v_cache = vl;
            q.cap = cap;
            q.hq = hq;
            q.hkv = hkv;
            q.T = T;
            q.pos0 = 0;
            CK(qkv_post_prefill_launch(q, st));
            // tcgen05 (measured 327 / 229 TF/s at 8192 / 2048 tokens against
            // 252 / 195 for the mma.sync kernel, which prefill_tensor_cores = 0 selects)
            if (opt.prefill_tensor_cores)
                CK(attn_prefill_tc_launch(pQ, kl, vl, cap, hq, hkv, T, pO, &dstate->err, st));
            else
                CK(attn_prefill_launch(pQ, kl, vl, cap, hq, hkv, T, pO, st));
            if (tp == 1)
                pgemm(pO, m_o, hq * D, y.wo, y.to, T, H, hq * D, GEMM_RESID, nullptr, pX, H);
            else
            {
                pgemm(pO, m_o, hq * D, y.wo, y.to, T, H, hq * D, GEMM_STORE, nullptr, pXn, H);
                NK(ncclAllReduce(pXn, pXn, (size_t)T * H, ncclHalf, ncclSum, comm, st));
                CK(resid_add_launch(pX, pXn, T * H));
            }
            CK(rmsnorm_rows_launch(pX, y.ln2, eps, T, H, pXn, st));
            pgemm(pXn, m_xn, H, y.wgu, y.tgu, T, 2 * inter, H, GEMM_SWIGLU, nullptr, pA, inter);
            if (tp == 1)
                pgemm(pA, m_a, inter, y.wd, y.td, T, H, inter, GEMM_RESID, nullptr, pX, H);
            else
            {
                pgemm(pA, m_a, inter, y.wd, y.td, T, H, inter, GEMM_STORE, nullptr, pXn, H);
                NK(ncclAllReduce(pXn, pXn, (size_t)T * H, ncclHalf, ncclSum, comm, st));
                CK(resid_add_launch(pX, pXn, T * H));
            }
        }
        GemvArgs f;
        f.x = pX + (size_t)(T - 1) * H;
        f.norm_w = fnorm;
        f.eps = eps;
        f.out = logits_local;
        f.err = err;
        CK(gemv_launch(plm, PRO_RMSNORM, EPI_STORE, f, st, false));
        if (tp > 1)
            NK(ncclAllGather(logits_local, logits, v_local, ncclHalf, comm, st));
        logits_partial = false;
    }

    // -------------------------------------------------------------- Model::Infer
    // ModelBase::Infer (ModelBase.cpp:396-471) without its per-op launches.
    int infer(int64_t *ids, int32_t *n_ids, int32_t *eos, int32_t *n_eos)
    {
        if (!ready)
            fail(YLM_NOT_READY, "Call BeginInfer() first");
        if (!ids || !n_ids || *n_ids <= 0)
            fail(YLM_INVALID_ARG, "empty input");
        // EnsureSequenceLength (ModelBase.cpp:473-505)
        int n = *n_ids;
        int ne = (eos && n_eos) ? *n_eos : 0;
        while (n > max_seq)
        {
            int drop = 1;
            if (ne > 0)
            {
                drop = eos[0] + 1;
                for (int i = 1; i < ne; i++)
                    eos[i - 1] = eos[i] - drop;
                ne--;
            }
            drop = std::min(drop, n);
            memmove(ids, ids + drop, sizeof(int64_t) * (n - drop));
            n -= drop;
        }
        *n_ids = n;
        if (n_eos)
            *n_eos = ne;
        if (n <= 0)
            fail(YLM_INVALID_ARG, "empty input after trimming");

        const bool kv = opt.kv_cache_enabled != 0;
        if (last == 0)
        {
            // prefill, or every call with the KV cache off (ModelBase.cpp:539-565);
            // with the cache off it still serves as the K/V workspace
            if (n > cap - last)
                return YLM_KV_CACHE_EXCEEDED;
            if (n > max_pos)
                fail(YLM_SEQUENCE_LENGTH_EXCEEDED, "prompt longer than the RoPE table");
            ensure_prefill(n);
            hin->err = 0;
            fill_state(0, 0, 0, true, 0);
            push_state();
            CK(cudaMemcpyAsync(pIds, ids, sizeof(int64_t) * n, cudaMemcpyHostToDevice, st));
            if (!ev_a)
            {
                CK(cudaEventCreate(&ev_a));
                CK(cudaEventCreate(&ev_b));
            }
            CK(cudaEventRecord(ev_a, st));
            run_prefill(n);
            CK(cudaEventRecord(ev_b, st));
            pull_state_sync();
            float pf = 0.f;
            CK(cudaEventElapsedTime(&pf, ev_a, ev_b));
            prefill_ms = pf;
            if (kv)
                last = n - 1;
        }
        else
        {
            // decode (ModelBase.cpp:566-586)
            if (n != 1)
                fail(YLM_INVALID_ARG, "decode takes one token per call");
            if (last + 1 > cap - last)
                return YLM_KV_CACHE_EXCEEDED;
            const int slot = last + 1;
            const int pos = opt.rope_compat ? last : last + 1;
            if (pos >= max_pos)
                fail(YLM_SEQUENCE_LENGTH_EXCEEDED, "position beyond the RoPE table");
            fill_state(ids[0], slot, pos, true, 0);
            push_state();
            launch_forward(false);
            pull_state_sync();
            last++;
        }
        has_logits = true;
        return YLM_OK;
    }

    // Tensor parallel, after a fused greedy step: the logits rows of every rank
    // into `logits` (one NCCL all-gather, so every rank makes this call in the
    // same order, as every other engine call).
    void gather_logits()
    {
        if (!logits_partial)
            return;
        NK(ncclAllGather(logits_local, logits, v_local, ncclHalf, comm, st));
        logits_partial = false;
    }

    int64_t sample(bool do_greedy)
    {
        if (!has_logits)
            fail(YLM_NOT_READY, "no logits to sample");
        gather_logits();
        fill_state(0, 0, 0, do_greedy, 0);
        push_state();
        CK(sample_launch(sample_args(), st, false));
        pull_state_sync();
        note_sample(do_greedy);
        return hout->next_token;
    }

    void note_sample(bool do_greedy)
    {
        calls++;
        u_next = -1.f;
        last_k = do_greedy ? 0 : std::max(1, std::min(top_k, 64));
    }

    // one decode step + sample (one graph launch)
    int decode(int64_t id, bool do_greedy, int64_t *next)
    {
        if (!ready)
            fail(YLM_NOT_READY, "Call BeginInfer() first");
        if (last == 0)
        {
            // the reference treats this call as a prefill (P6: one-token prompt)
            int64_t ids1[1] = {id};
            int32_t n1 = 1;
            int r = infer(ids1, &n1, nullptr, nullptr);
            if (r != YLM_OK)
                return r;
            *next = sample(do_greedy);
            return YLM_OK;
        }
        if (last + 1 > cap - last)
            return YLM_KV_CACHE_EXCEEDED;
        const int slot = last + 1;
        const int pos = opt.rope_compat ? last : last + 1;
        if (pos >= max_pos)
            fail(YLM_SEQUENCE_LENGTH_EXCEEDED, "position beyond the RoPE table");
        fill_state(id, slot, pos, do_greedy, 0);
        push_state();
        launch_forward(true, do_greedy);
        pull_state_sync();
        last++;
        has_logits = true;
        note_sample(do_greedy);
        *next = hout->next_token;
        return YLM_OK;
    }

    void begin()
    {
        ready = true;
        last = 0;
        has_logits = false;
        if (opt.zero_kv_on_begin && opt.kv_cache_enabled)
        {
            CK(cudaMemsetAsync(kc, 0, kv_layer * L * 2, st));
            CK(cudaMemsetAsync(vc, 0, kv_layer * L * 2, st));
            CK(cudaStreamSynchronize(st));
        }
    }
};

// ------------------------------------------------------------------ C ABI
extern "C" {

const char *ylm_status_string(int s)
{
    switch (s)
    {
    case YLM_OK: return "ok";
    case YLM_SEQUENCE_LENGTH_EXCEEDED: return "sequence length exceeded";
    case YLM_KV_CACHE_EXCEEDED: return "KV cache capacity exceeded";
    case YLM_INVALID_PROMPT: return "invalid prompt";
    case YLM_CANCELED: return "canceled";
    case YLM_GPU_QUEUE_TIMED_OUT: return "GPU queue timed out";
    case YLM_INVALID_ARG: return "invalid argument";
    case YLM_NOT_READY: return "not ready (call ylm_begin_infer first)";
    case YLM_LOAD_ERROR: return "load error";
    case YLM_CUDA_ERROR: return "CUDA error";
    case YLM_DEVICE_TIMEOUT: return "device wait timed out";
    case YLM_COMM_ERROR: return "communication error";
    case YLM_UNSUPPORTED: return "unsupported";
    default: return "unknown status";
    }
}

const char *ylm_last_error(void) { return g_last_error.c_str(); }

int ylm_options_default(ylm_engine_options *o)
{
    if (!o)
        return YLM_INVALID_ARG;
    memset(o, 0, sizeof(*o));
    o->kv_cache_gb = 2;
    o->kv_cache_enabled = 1;
    o->rope_compat = 1;
    o->rope_scaling = 0;
    o->use_cuda_graph = 1;
    o->use_pdl = 0; // measured slower than plain graph launches on B200
    o->tp_size = 1;
    o->init_std = 0.02;
    o->zero_kv_on_begin = 1;
    o->prefill_tensor_cores = 1;
    o->decode_persistent = 1;
    return YLM_OK;
}

int ylm_config_from_json(const char *path, ylm_model_config *c)
{
    return guarded([&]() -> int {
        if (!path || !c)
            fail(YLM_INVALID_ARG, "null argument");
        JVal j = json_parse(read_file(path));
        memset(c, 0, sizeof(*c));
        auto num = [&](const char *k) -> double {
            const JVal *v = j.get(k);
            if (!v)
                fail(YLM_LOAD_ERROR, "config.json: missing %s", k);
            return v->as_num();
        };
        const JVal *mt = j.get("model_type");
        if (!mt)
            fail(YLM_LOAD_ERROR, "config.json: missing model_type");
        std::string t = mt->str;
        for (auto &ch : t)
            ch = (char)tolower(ch);
        if (t == "llama")
            c->model_type = YLM_MODEL_LLAMA;
        else if (t == "mistral")
            c->model_type = YLM_MODEL_MISTRAL;
        else if (t == "qwen2")
            c->model_type = YLM_MODEL_QWEN2_5;
        else if (t == "qwen3")
            c->model_type = YLM_MODEL_QWEN3;
        else
            fail(YLM_LOAD_ERROR, "Unsupported model type: %s", t.c_str());
        c->num_layers = (int)num("num_hidden_layers");
        c->hidden_size = (int)num("hidden_size");
        c->num_heads = (int)num("num_attention_heads");
        c->num_kv_heads = (int)num("num_key_value_heads");
        c->vocab_size = (int64_t)num("vocab_size");
        c->rms_eps = (float)num("rms_norm_eps");
        c->rope_theta = (float)num("rope_theta");
        c->max_position_embeddings = (int)num("max_position_embeddings");
        c->intermediate_size = (int)num("intermediate_size");
        c->head_dim = j.has("head_dim") ? (int)num("head_dim") : c->hidden_size / std::max(1, c->num_heads);
        const JVal *tie = j.get("tie_word_embeddings");
        c->tie_word_embeddings = tie ? (tie->kind == JVal::Bool ? tie->b : tie->as_num() != 0) : 0;
        c->rope_factor = 1.f;
        c->rope_low_freq = 1.f;
        c->rope_high_freq = 1.f;
        c->rope_orig_max_pos = c->max_position_embeddings;
        if (const JVal *rs = j.get("rope_scaling"))
            if (rs->kind == JVal::Obj)
            {
                if (rs->has("factor"))
                    c->rope_factor = (float)rs->get("factor")->as_num();
                if (rs->has("low_freq_factor"))
                    c->rope_low_freq = (float)rs->get("low_freq_factor")->as_num();
                if (rs->has("high_freq_factor"))
                    c->rope_high_freq = (float)rs->get("high_freq_factor")->as_num();
                if (rs->has("original_max_position_embeddings"))
                    c->rope_orig_max_pos = (int)rs->get("original_max_position_embeddings")->as_num();
            }
        if (const JVal *e = j.get("eos_token_id"))
        {
            if (e->kind == JVal::Arr)
                for (auto &v : e->arr)
                {
                    if (c->n_eos < 8)
                        c->eos_ids[c->n_eos++] = (int)v.as_num();
                }
            else if (e->kind == JVal::Num)
                c->eos_ids[c->n_eos++] = (int)e->num;
        }
        if (c->hidden_size % std::max(1, c->num_heads))
            fail(YLM_LOAD_ERROR, "HiddenSize must be divisible by NumHeads");
        return YLM_OK;
    });
}

int ylm_resolve_snapshot(const char *root, char *out, int32_t out_len)
{
    return guarded([&]() -> int {
        if (!root || !out || out_len <= 0)
            fail(YLM_INVALID_ARG, "null argument");
        std::string ref = std::string(root) + "/refs/main";
        std::ifstream f(ref);
        if (!f)
            fail(YLM_LOAD_ERROR, "Invalid HuggingFace repo: refs/main not found in %s", root);
        std::string h;
        std::getline(f, h);
        std::string snap = std::string(root) + "/snapshots/" + h;
        struct stat sb;
        if (stat(snap.c_str(), &sb) != 0)
            fail(YLM_LOAD_ERROR, "Snapshot folder does not exist: %s", snap.c_str());
        if ((int)snap.size() + 1 > out_len)
            fail(YLM_INVALID_ARG, "output buffer too small");
        memcpy(out, snap.c_str(), snap.size() + 1);
        return YLM_OK;
    });
}

int ylm_nccl_unique_id(void *out128)
{
    return guarded([&]() -> int {
        if (!out128)
            fail(YLM_INVALID_ARG, "null argument");
        ncclUniqueId id;
        NK(ncclGetUniqueId(&id));
        memcpy(out128, &id, sizeof(id));
        return YLM_OK;
    });
}

int ylm_create(const char *snapshot_dir, const ylm_model_config *cfg, const ylm_engine_options *opt, ylm_engine **out)
{
    return guarded([&]() -> int {
        if (!cfg || !out)
            fail(YLM_INVALID_ARG, "null argument");
        ylm_engine_options o;
        if (opt)
            o = *opt;
        else
            ylm_options_default(&o);
        auto e = std::make_unique<ylm_engine>();
        e->init(snapshot_dir, *cfg, o);
        *out = e.release();
        return YLM_OK;
    });
}

int ylm_destroy(ylm_engine *e)
{
    delete e;
    return YLM_OK;
}

int ylm_begin_infer(ylm_engine *e)
{
    return guarded([&]() -> int {
        if (!e)
            fail(YLM_INVALID_ARG, "null engine");
        CK(cudaSetDevice(e->dev));
        e->begin();
        return YLM_OK;
    });
}

int ylm_infer(ylm_engine *e, int64_t *ids, int32_t *n_ids, int32_t *eos, int32_t *n_eos)
{
    return guarded([&]() -> int {
        if (!e)
            fail(YLM_INVALID_ARG, "null engine");
        CK(cudaSetDevice(e->dev));
        return e->infer(ids, n_ids, eos, n_eos);
    });
}

int ylm_logits(ylm_engine *e, void *host_out, int32_t as_float32)
{
    return guarded([&]() -> int {
        if (!e || !host_out)
            fail(YLM_INVALID_ARG, "null argument");
        if (!e->has_logits)
            fail(YLM_NOT_READY, "no logits yet");
        CK(cudaSetDevice(e->dev));
        e->gather_logits();
        if (!as_float32)
        {
            CK(cudaMemcpyAsync(host_out, e->logits, e->V * 2, cudaMemcpyDeviceToHost, e->st));
            CK(cudaStreamSynchronize(e->st));
            return YLM_OK;
        }
        std::vector<__half> tmp(e->V);
        CK(cudaMemcpyAsync(tmp.data(), e->logits, e->V * 2, cudaMemcpyDeviceToHost, e->st));
        CK(cudaStreamSynchronize(e->st));
        float *o = static_cast<float *>(host_out);
        for (int64_t i = 0; i < e->V; i++)
            o[i] = __half2float(tmp[i]);
        return YLM_OK;
    });
}

int ylm_logits_device(ylm_engine *e, const void **dev_ptr, int64_t *vocab)
{
    return guarded([&]() -> int {
        if (!e || !dev_ptr)
            fail(YLM_INVALID_ARG, "null argument");
        if (e->logits_partial)
        {
            CK(cudaSetDevice(e->dev));
            e->gather_logits();
            CK(cudaStreamSynchronize(e->st));
        }
        *dev_ptr = e->logits;
        if (vocab)
            *vocab = e->V;
        return YLM_OK;
    });
}

int ylm_set_sampling(ylm_engine *e, const ylm_sampling *s)
{
    return guarded([&]() -> int {
        if (!e || !s)
            fail(YLM_INVALID_ARG, "null argument");
        if (!s->greedy && (s->top_k < 1 || s->top_k > 64 || !(s->temperature > 0.f)))
            fail(YLM_INVALID_ARG, "top_k must be in 1..64 and temperature > 0");
        CK(cudaSetDevice(e->dev));
        e->greedy = s->greedy;
        e->top_k = s->top_k;
        e->temp = s->temperature > 0.f ? s->temperature : 1.f;
        e->seed = s->seed;
        // special-token mask bitmap (ChatSession.cpp:41-61)
        if (e->mask_bits)
        {
            cudaFree(e->mask_bits);
            e->mask_bits = nullptr;
        }
        if (s->n_masked > 0 && s->masked_ids)
        {
            std::vector<uint32_t> bits((e->V + 31) / 32, 0u);
            for (int i = 0; i < s->n_masked; i++)
            {
                const int64_t id = s->masked_ids[i];
                if (id >= 0 && id < e->V)
                    bits[id >> 5] |= 1u << (id & 31);
            }
            e->mask_bits = e->dalloc<uint32_t>(bits.size());
            e->h2d(e->mask_bits, bits.data(), bits.size() * 4);
        }
        // the graph with the sampler bakes in the mask pointer: rebuild it
        if (e->g_fwd_sample)
        {
            cudaGraphExecDestroy(e->g_fwd_sample);
            e->g_fwd_sample = nullptr;
        }
        return YLM_OK;
    });
}

int ylm_sample(ylm_engine *e, int32_t greedy, int64_t *next_id)
{
    return guarded([&]() -> int {
        if (!e || !next_id)
            fail(YLM_INVALID_ARG, "null argument");
        CK(cudaSetDevice(e->dev));
        *next_id = e->sample(greedy != 0);
        return YLM_OK;
    });
}

int ylm_decode(ylm_engine *e, int64_t id, int32_t greedy, int64_t *next_id)
{
    return guarded([&]() -> int {
        if (!e || !next_id)
            fail(YLM_INVALID_ARG, "null argument");
        CK(cudaSetDevice(e->dev));
        return e->decode(id, greedy != 0, next_id);
    });
}

int ylm_generate(ylm_engine *e, const int64_t *prompt, int32_t n_prompt, int32_t max_new, const int64_t *eos_ids,
                 int32_t n_eos, int64_t *out_ids, int32_t *n_out, double *first_ms, double *decode_ms)
{
    return guarded([&]() -> int {
        if (!e || !prompt || n_prompt <= 0 || !out_ids || !n_out || max_new < 0)
            fail(YLM_INVALID_ARG, "bad argument");
        CK(cudaSetDevice(e->dev));
        using clk = std::chrono::steady_clock;
        auto ms_since = [](clk::time_point a) { return std::chrono::duration<double, std::milli>(clk::now() - a).count(); };
        *n_out = 0;
        double t_first = 0, t_dec = 0;
        e->begin();
        std::vector<int64_t> ids(prompt, prompt + n_prompt);
        int generated = 0;
        int64_t next = -1;
        int status = YLM_OK;
        const bool kv = e->opt.kv_cache_enabled != 0;
        auto finish = [&]() {
            if (first_ms)
                *first_ms = t_first;
            if (decode_ms)
                *decode_ms = t_dec;
            return status;
        };
        // stop rules of ChatSession.cpp:151-161: an EOS id, or prompt + generated
        // reaching MaxSequenceLength; the token that ends the loop is not emitted
        auto ends = [&](int64_t tok) {
            return std::find(eos_ids, eos_ids + n_eos, tok) != eos_ids + n_eos || n_prompt + generated >= e->max_seq;
        };
        if (max_new == 0)
            return finish();

        // the first token: prefill + greedy sample (ChatSession.cpp:140)
        auto t0 = clk::now();
        {
            int32_t n = (int32_t)ids.size();
            status = e->infer(ids.data(), &n, nullptr, nullptr);
            ids.resize(n);
            if (status != YLM_OK)
                return finish();
            next = e->sample(true);
        }
        t_first = ms_since(t0);
        generated = 1;
        if (ends(next))
            return finish();
        out_ids[(*n_out)++] = next;
        if (!kv)
            ids.push_back(next);

        if (!kv || e->last == 0 || e->u_next >= 0.f || !e->opt.use_cuda_graph)
        {
            // one synchronous call per token: the KV cache disabled (every call
            // a prefill), a one-token prompt (ModelBase.cpp:539-547), or a test's
            // fixed uniform for the next draw
            while (generated < max_new)
            {
                t0 = clk::now();
                int r;
                if (!kv || e->last == 0)
                {
                    int32_t n = (int32_t)ids.size();
                    r = e->infer(ids.data(), &n, nullptr, nullptr);
                    ids.resize(n);
                    if (r == YLM_OK)
                        next = e->sample(e->greedy != 0);
                }
                else
                    r = e->decode(next, e->greedy != 0, &next);
                if (r != YLM_OK)
                {
                    status = r;
                    break;
                }
                t_dec += ms_since(t0);
                generated++;
                if (ends(next))
                    break;
                out_ids[(*n_out)++] = next;
                if (!kv)
                    ids.push_back(next);
            }
            return finish();
        }

        // Later tokens, one step in flight ahead of the host: each decode step
        // runs in the device's advance mode (its sampler writes the next input
        // token and moves the slot and RoPE position on), so step s + 1 is
        // launched before the host reads step s's token; the host-side checks of
        // a token overlap the next step. A step launched past the end (an EOS)
        // is rolled back: its KV slot is beyond `last` and is written again by
        // the next call that reaches it.
        e->ensure_ring();
        const bool greedy = e->greedy != 0;
        // the capacity rule (ModelBase.cpp:853-866) and the RoPE table, checked
        // for the step that would follow `last`
        auto step_fits = [&](int *why) {
            if (e->last + 1 > e->cap - e->last)
            {
                *why = YLM_KV_CACHE_EXCEEDED;
                return false;
            }
            const int pos = e->opt.rope_compat ? e->last : e->last + 1;
            if (pos >= e->max_pos)
            {
                *why = YLM_SEQUENCE_LENGTH_EXCEEDED;
                return false;
            }
            return true;
        };
        auto launch = [&](int k) {
            e->launch_forward(true, greedy);
            CK(cudaMemcpyAsync(e->hring[k & 1], e->dstate, sizeof(StepState), cudaMemcpyDeviceToHost, e->st));
            CK(cudaEventRecord(e->ev_ring[k & 1], e->st));
            e->last++;
            e->note_sample(greedy);
        };
        int why = YLM_OK;
        if (!step_fits(&why))
        {
            status = why;
            if (why == YLM_SEQUENCE_LENGTH_EXCEEDED)
                fail(why, "position beyond the RoPE table");
            return finish();
        }
        e->fill_state(next, e->last + 1, e->opt.rope_compat ? e->last : e->last + 1, greedy, 1);
        e->push_state();
        auto t_prev = clk::now();
        launch(0);
        for (int k = 0;; k++)
        {
            // step k + 1 goes out before step k's token is read, if it may follow
            why = YLM_OK;
            const bool more = generated + 1 < max_new && n_prompt + generated + 1 < e->max_seq && step_fits(&why);
            if (more)
                launch(k + 1);
            CK(cudaEventSynchronize(e->ev_ring[k & 1]));
            *e->hout = *e->hring[k & 1];
            if (e->hout->err != 0)
            {
                cudaStreamSynchronize(e->st);
                e->check_dev_err(); // throws
            }
            next = e->hout->next_token;
            t_dec += ms_since(t_prev);
            t_prev = clk::now();
            generated++;
            if (ends(next))
            {
                if (more)
                {
                    // discard the step launched past the end
                    CK(cudaStreamSynchronize(e->st));
                    e->last--;
                    e->calls--;
                }
                break;
            }
            out_ids[(*n_out)++] = next;
            if (!more)
            {
                if (why != YLM_OK && generated < max_new)
                {
                    status = why;
                    if (why == YLM_SEQUENCE_LENGTH_EXCEEDED)
                        fail(why, "position beyond the RoPE table");
                }
                break;
            }
        }
        e->has_logits = true;
        return finish();
    });
}

int ylm_set_draw(ylm_engine *e, float u)
{
    if (!e)
        return YLM_INVALID_ARG;
    e->u_next = u;
    return YLM_OK;
}

int ylm_last_topk(ylm_engine *e, int64_t *ids, float *probs, int32_t *k, float *u)
{
    return guarded([&]() -> int {
        if (!e)
            fail(YLM_INVALID_ARG, "null engine");
        CK(cudaSetDevice(e->dev));
        if (k)
            *k = e->last_k;
        if (u)
            *u = e->hout->u_used;
        if (e->last_k > 0)
        {
            if (ids)
                e->d2h(ids, e->dbg_ids, sizeof(int64_t) * e->last_k);
            if (probs)
                e->d2h(probs, e->dbg_probs, sizeof(float) * e->last_k);
        }
        return YLM_OK;
    });
}

int ylm_info(ylm_engine *e, int32_t *kv_capacity, int32_t *last_kv_index, int32_t *max_seq_len)
{
    if (!e)
        return YLM_INVALID_ARG;
    if (kv_capacity)
        *kv_capacity = e->cap;
    if (last_kv_index)
        *last_kv_index = e->last;
    if (max_seq_len)
        *max_seq_len = e->max_seq;
    return YLM_OK;
}

int ylm_last_prefill_ms(ylm_engine *e, double *ms)
{
    if (!e || !ms)
        return YLM_INVALID_ARG;
    *ms = e->prefill_ms;
    return YLM_OK;
}

int ylm_decode_path(ylm_engine *e, int32_t *persistent)
{
    if (!e || !persistent)
        return YLM_INVALID_ARG;
    *persistent = e->ds_on ? 1 : 0;
    return YLM_OK;
}

int ylm_time_segment(ylm_engine *e, int32_t layer, int32_t iters, double *ms_per_launch, double *weight_bytes)
{
    return guarded([&]() -> int {
        if (!e || iters <= 0 || !ms_per_launch || !weight_bytes)
            fail(YLM_INVALID_ARG, "bad argument");
        if (!e->ds_on)
            return (int)YLM_UNSUPPORTED;
        // with tensor parallelism a segment waits on its peers' partials
        if (e->tp > 1)
            return (int)YLM_UNSUPPORTED;
        if (layer < 0 || layer >= e->L)
            fail(YLM_INVALID_ARG, "layer out of range");
        CK(cudaSetDevice(e->dev));
        // segment layer + 1 runs layer's O, gate-up, down and the next QKV (or the lm_head)
        // each timed launch must tag its activations apart from the previous
        // one's: this copy of the segment advances *gen at exit; afterwards the
        // generation and the tagged buffers are cleared, which keeps the next
        // decode step consistent
        DsArgs d = e->ds_seg[layer + 1];
        d.last = 1;
        double bytes = 0;
        for (int i = d.p0; i < d.p1; i++)
            bytes += 2.0 * e->ds_phases[i].N * e->ds_phases[i].K;
        cudaEvent_t a, b;
        CK(cudaEventCreate(&a));
        CK(cudaEventCreate(&b));
        auto launch_one = [&]() { CK(ds_launch(d, e->ds_smem, e->sms, e->st)); };
        launch_one(); // warm
        CK(cudaEventRecord(a, e->st));
        for (int i = 0; i < iters; i++)
            launch_one();
        CK(cudaEventRecord(b, e->st));
        CK(cudaEventSynchronize(b));
        float ms = 0;
        CK(cudaEventElapsedTime(&ms, a, b));
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        e->ds_reset();
        e->pull_state_sync();
        *ms_per_launch = ms / iters;
        *weight_bytes = bytes;
        return YLM_OK;
    });
}

int ylm_debug_drop_output(ylm_engine *e, int32_t layer)
{
    return guarded([&]() -> int {
        if (!e)
            fail(YLM_INVALID_ARG, "null engine");
        if (!e->ds_on)
            return (int)YLM_UNSUPPORTED;
        if (layer >= e->L)
            fail(YLM_INVALID_ARG, "layer out of range");
        CK(cudaSetDevice(e->dev));
        CK(cudaStreamSynchronize(e->st));
        if (e->ds_seg_saved.empty())
            e->ds_seg_saved = e->ds_seg;
        e->ds_seg = e->ds_seg_saved;
        if (layer >= 0)
        {
            // the SwiGLU activation of `layer`, which the down projection polls
            if (!e->ds_sink)
                e->ds_sink = e->dalloc<uint32_t>(e->inter);
            bool done = false;
            for (DsArgs &d : e->ds_seg)
                for (int i = d.p0; i < d.p1 && !done; i++)
                    if (d.ph[i - d.p0].epi == EPI_SWIGLU && d.ph[i - d.p0].w == e->layers[layer].wgu)
                    {
                        d.ph[i - d.p0].out_t = e->ds_sink;
                        done = true;
                    }
            if (!done)
                fail(YLM_INVALID_ARG, "no gate-up phase for layer %d", layer);
        }
        // the captured graphs hold the segments' arguments: capture again
        for (cudaGraphExec_t *g : {&e->g_fwd, &e->g_fwd_sample, &e->g_fwd_greedy})
            if (*g)
            {
                cudaGraphExecDestroy(*g);
                *g = nullptr;
            }
        return YLM_OK;
    });
}

int ylm_exchange_stats(ylm_engine *e, int32_t reset, double *wait_ms, double *exchanges, double *steps)
{
    return guarded([&]() -> int {
        if (!e)
            fail(YLM_INVALID_ARG, "null engine");
        CK(cudaSetDevice(e->dev));
        unsigned long long v[2] = {0, 0};
        if (e->ds_xstat)
        {
            CK(cudaStreamSynchronize(e->st));
            e->d2h(v, e->ds_xstat, sizeof(v));
        }
        if (wait_ms)
            *wait_ms = (double)v[0] * 1e-6;
        if (exchanges)
            *exchanges = (double)v[1];
        if (steps)
            *steps = (double)e->xstat_steps;
        if (reset)
        {
            if (e->ds_xstat)
                CK(cudaMemsetAsync(e->ds_xstat, 0, sizeof(v), e->st));
            e->xstat_steps = 0;
        }
        return YLM_OK;
    });
}

int ylm_time_allreduce(ylm_engine *e, int32_t iters, double *ms_per_step)
{
    return guarded([&]() -> int {
        if (!e || iters <= 0 || !ms_per_step)
            fail(YLM_INVALID_ARG, "bad argument");
        if (e->tp <= 1)
            return (int)YLM_UNSUPPORTED;
        CK(cudaSetDevice(e->dev));
        // the decode step's collectives: 2L all-reduces of [hidden] FP16, back
        // to back in one graph (the per-op path's exchange, without the GEMVs)
        cudaGraph_t g = nullptr;
        cudaGraphExec_t ex = nullptr;
        CK(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
        ncclResult_t nr = ncclSuccess;
        for (int i = 0; i < 2 * e->L && nr == ncclSuccess; i++)
            nr = ncclAllReduce(e->ar, e->ar, e->H, ncclHalf, ncclSum, e->comm, e->st);
        cudaError_t ce = cudaStreamEndCapture(e->st, &g);
        if (nr != ncclSuccess || ce != cudaSuccess)
        {
            if (g)
                cudaGraphDestroy(g);
            NK(nr);
            CK(ce);
        }
        ce = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        CK(ce);
        cudaEvent_t a = nullptr, b = nullptr;
        float ms = 0;
        auto run = [&]() {
            CK(cudaGraphLaunch(ex, e->st)); // warm
            NK(ncclAllReduce(e->ar, e->ar, 1, ncclHalf, ncclSum, e->comm, e->st));
            CK(cudaEventCreate(&a));
            CK(cudaEventCreate(&b));
            CK(cudaEventRecord(a, e->st));
            for (int i = 0; i < iters; i++)
                CK(cudaGraphLaunch(ex, e->st));
            CK(cudaEventRecord(b, e->st));
            CK(cudaEventSynchronize(b));
            CK(cudaEventElapsedTime(&ms, a, b));
        };
        try
        {
            run();
        }
        catch (...)
        {
            cudaStreamSynchronize(e->st);
            cudaGraphExecDestroy(ex);
            if (a)
                cudaEventDestroy(a);
            if (b)
                cudaEventDestroy(b);
            throw;
        }
        cudaGraphExecDestroy(ex); // a graph holding NCCL calls must not outlive the communicator
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        CK(cudaMemsetAsync(e->ar, 0, sizeof(__half) * e->H, e->st));
        CK(cudaStreamSynchronize(e->st));
        *ms_per_step = ms / iters;
        return YLM_OK;
    });
}

int ylm_time_decode(ylm_engine *e, int32_t iters, double *ms_per_step)
{
    return guarded([&]() -> int {
        if (!e || iters <= 0 || !ms_per_step)
            fail(YLM_INVALID_ARG, "bad argument");
        if (!e->ready || e->last == 0)
            fail(YLM_NOT_READY, "run a prefill first");
        // every step must pass the decode capacity rule last + 1 <= cap - last
        if (2 * (e->last + iters) - 1 > e->cap || e->last + iters >= e->max_pos)
            return (int)YLM_KV_CACHE_EXCEEDED;
        CK(cudaSetDevice(e->dev));
        // device-side chaining: the sampler writes the next token and advances slot/pos
        e->fill_state(0, e->last + 1, e->opt.rope_compat ? e->last : e->last + 1, e->greedy != 0, 1);
        e->hin->token = e->hout->next_token >= 0 ? e->hout->next_token : 0;
        e->push_state();
        // the first launch captures the graph (outside the timed region)
        const bool greedy = e->greedy != 0;
        if (!e->graph_for(e->step_mode(true, greedy)) && e->opt.use_cuda_graph && (!e->ds_on || e->ds_graph_ok))
        {
            e->launch_forward(true, greedy);
            CK(cudaStreamSynchronize(e->st));
            e->pull_state_sync();
            e->last += 1;
            e->calls += 1;
            iters -= 1;
            if (iters <= 0)
            {
                *ms_per_step = 0.0;
                return YLM_OK;
            }
        }
        cudaEvent_t a, b;
        CK(cudaEventCreate(&a));
        CK(cudaEventCreate(&b));
        // with tensor parallelism the ranks' host threads reach this point at
        // different times; a one-element all-reduce lines their streams up, so
        // the timed steps start together instead of the earliest rank's first
        // step absorbing the others' host lag (its segments wait for their
        // partials)
        if (e->tp > 1)
            NK(ncclAllReduce(e->ar, e->ar, 1, ncclHalf, ncclSum, e->comm, e->st));
        CK(cudaEventRecord(a, e->st));
        for (int i = 0; i < iters; i++)
            e->launch_forward(true, greedy);
        CK(cudaEventRecord(b, e->st));
        CK(cudaEventSynchronize(b));
        float ms = 0;
        CK(cudaEventElapsedTime(&ms, a, b));
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        e->pull_state_sync();
        e->last += iters;
        e->calls += iters;
        *ms_per_step = ms / iters;
        return YLM_OK;
    });
}

} // extern "C"
