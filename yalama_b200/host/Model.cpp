// Drop-in replacement for the reference's src/models/Model.cpp: the same static
// `Model` facade (include/models/Model.h:7-17, Init / BeginInfer / Infer), backed
// by the B200 engine through its C ABI (include/yalama_b200.h) instead of the
// LibTorch ModelBase forward. ChatSession, the OpenAI service, the REPL, the
// tokenizer and ConfigManager compile unchanged against it; only this file and
// the engine library change in the link.
//
//   Model::Init        src/models/Model.cpp:10-34   -> ylm_config_from_json + ylm_create
//   Model::BeginInfer  src/models/Model.cpp:36-41   -> ylm_begin_infer
//   Model::Infer       src/models/Model.cpp:43-48   -> ylm_infer (+ in/out trimming)
//
// Logits come back as a [1, T, V] FP16 CUDA tensor whose row stride is 0: the
// engine computes the last row only, and ChatSession selects row T-1
// (src/ChatSession.cpp:138). Recoverable failures map to GenerationError, the
// rest throw std::runtime_error as the reference does (ModelBase.cpp:401-402,
// Model.cpp:29-30).
//
// Also provided: Model_SampleOnDevice(), the engine's on-device sampler for the
// current logits (the replacement for ChatSession::Sample's LibTorch ops), and
// Model_RecordInputs() / Model_RecordedInputs(), which keep the token ids of
// every Infer call (off by default; tests compare them with the engine's own
// token loop).
#include "Model.h"
#include "ConfigManager.h"
#include "TraceLogger.h"
#include "yalama_b200.h"

#include <stdexcept>
#include <string>
#include <vector>

// Model.h's private `_model` (a ModelBase) is not defined: nothing here uses it,
// and defining it would pull ModelBase's vtable (src/models/ModelBase.cpp) into
// the link. The step counter ChatSession advances (src/ChatSession.cpp:226) is
// defined in ModelBase.cpp:17, which this file replaces, so it lives here.
int TraceLogger::_TraceStep = 0;

namespace
{
ylm_engine *g_engine = nullptr;
bool g_record = false;
std::vector<std::vector<int64_t>> g_inputs;

[[noreturn]] void throw_status(int status, const char *where)
{
    throw std::runtime_error(std::string(where) + ": " + ylm_status_string(status) + ": " + ylm_last_error());
}
} // namespace

void Model::Init()
{
    ylm_model_config cfg;
    const std::string cfg_path = ConfigManager::ModelPath + "/config.json";
    int st = ylm_config_from_json(cfg_path.c_str(), &cfg);
    if (st == YLM_UNSUPPORTED)
        throw_status(st, "Unrecognized/unsupported model type. Supported: Llama 3+, Mistral");
    if (st != YLM_OK)
        throw_status(st, ("Model::Init: cannot read " + cfg_path).c_str());
    // ConfigManager has already resolved these (src/ConfigManager.cpp:410-471)
    cfg.model_type = static_cast<int32_t>(ConfigManager::ModelLoadedType);
    cfg.num_layers = ConfigManager::NumLayers;
    cfg.hidden_size = ConfigManager::HiddenSize;
    cfg.num_heads = ConfigManager::NumHeads;
    cfg.num_kv_heads = ConfigManager::NumKVHeads;
    cfg.head_dim = ConfigManager::HeadDim;
    cfg.vocab_size = ConfigManager::VocabSize;
    cfg.rms_eps = ConfigManager::Eps;
    cfg.rope_theta = ConfigManager::RopeTheta;
    cfg.max_position_embeddings = ConfigManager::MaxSequenceLength;

    ylm_engine_options opt;
    ylm_options_default(&opt);
    opt.kv_cache_gb = ConfigManager::KVCacheSizeInGB;
    opt.kv_cache_enabled = ConfigManager::IsKVCacheEnabled.value_or(true) ? 1 : 0;

    if (g_engine)
        ylm_destroy(g_engine);
    g_engine = nullptr;
    st = ylm_create(ConfigManager::ModelPath.c_str(), &cfg, &opt, &g_engine);
    if (st != YLM_OK)
        throw_status(st, "Model::Init");

    // MaxSequenceLength is capped by free device memory, as ModelBase.cpp:312-338 does
    int32_t cap = 0, last = 0, max_seq = 0;
    ylm_info(g_engine, &cap, &last, &max_seq);
    ConfigManager::MaxSequenceLength = max_seq;
}

void Model::BeginInfer()
{
    EnsureModelIsInitialized();
    TraceLogger::_TraceStep = 0; // ModelBase::BeginInfer, ModelBase.cpp:298
    const int st = ylm_begin_infer(g_engine);
    if (st != YLM_OK)
        throw_status(st, "Model::BeginInfer");
}

GenerationResult Model::Infer(torch::Tensor &tokenVectors, std::vector<int> &eosPerPrompt)
{
    EnsureModelIsInitialized();
    GenerationResult result;

    torch::Tensor host = tokenVectors.to(torch::kCPU, torch::kInt64).contiguous().view({-1});
    std::vector<int64_t> ids(host.data_ptr<int64_t>(), host.data_ptr<int64_t>() + host.numel());
    if (g_record)
        g_inputs.push_back(ids);
    int32_t n = static_cast<int32_t>(ids.size());
    int32_t n_eos = static_cast<int32_t>(eosPerPrompt.size());
    std::vector<int32_t> eos(eosPerPrompt.begin(), eosPerPrompt.end());

    const int st = ylm_infer(g_engine, ids.data(), &n, eos.empty() ? nullptr : eos.data(), &n_eos);
    if (st != YLM_OK && st > YLM_GPU_QUEUE_TIMED_OUT)
        throw_status(st, "Model::Infer");

    // in/out trimming (ModelBase.cpp:473-505)
    if (n != static_cast<int32_t>(host.numel()))
    {
        ids.resize(n);
        tokenVectors = torch::tensor(ids, torch::kInt64).unsqueeze(0).to(tokenVectors.device());
        eosPerPrompt.assign(eos.begin(), eos.begin() + n_eos);
    }

    if (st != YLM_OK)
    {
        result.IsSuccess = false;
        result.Error = static_cast<GenerationError>(st);
        return result;
    }
    const void *dev = nullptr;
    int64_t vocab = 0;
    ylm_logits_device(g_engine, &dev, &vocab);
    auto opts = torch::TensorOptions().dtype(torch::kHalf).device(torch::kCUDA);
    torch::Tensor last_row = torch::from_blob(const_cast<void *>(dev), {1, 1, vocab}, opts);
    result.Logits = last_row.expand({1, tokenVectors.size(1), vocab});
    return result;
}

void Model::EnsureModelIsInitialized()
{
    if (g_engine == nullptr)
        throw std::runtime_error(
            "You must explicitly call Init() function at program startup once before calling any other functions");
}

// The engine's sampler on the current logits: greedy, or top-k + temperature
// over the same masked special ids ChatSession uses (ChatSession.cpp:41-61).
int64_t Model_SampleOnDevice(bool greedy, const std::vector<int64_t> &masked_ids, uint64_t seed)
{
    if (g_engine == nullptr)
        throw std::runtime_error("Model::Init() has not been called");
    // the sampling set-up (mask bitmap upload) is redone only when it changes
    static std::vector<int64_t> last_mask;
    static int last_k = -1;
    static float last_temp = -1.f;
    static uint64_t last_seed = 0;
    int st = YLM_OK;
    if (masked_ids != last_mask || last_k != ConfigManager::TopK || last_temp != ConfigManager::Temp ||
        last_seed != seed)
    {
        ylm_sampling s;
        s.greedy = 0;
        s.top_k = ConfigManager::TopK;
        s.temperature = ConfigManager::Temp;
        s.seed = seed;
        s.masked_ids = masked_ids.empty() ? nullptr : masked_ids.data();
        s.n_masked = static_cast<int32_t>(masked_ids.size());
        st = ylm_set_sampling(g_engine, &s);
        if (st != YLM_OK)
            throw_status(st, "ylm_set_sampling");
        last_mask = masked_ids;
        last_k = ConfigManager::TopK;
        last_temp = ConfigManager::Temp;
        last_seed = seed;
    }
    int64_t id = -1;
    st = ylm_sample(g_engine, greedy ? 1 : 0, &id);
    if (st != YLM_OK)
        throw_status(st, "ylm_sample");
    return id;
}

void Model_RecordInputs(bool on)
{
    g_record = on;
    g_inputs.clear();
}

const std::vector<std::vector<int64_t>> &Model_RecordedInputs() { return g_inputs; }
