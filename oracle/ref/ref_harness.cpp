// Test infrastructure only (oracle side): a driver for the reference's own
// model code. It links the reference's unmodified Model / ModelBase / family
// sources and ConfigManager (compiled where they lie, see oracle/ref/Makefile)
// and runs the token loop that ChatSession::Generate runs
// (src/ChatSession.cpp:113-230), without the tokenizer and chat templates:
//
//   ConfigManager::Load            src/ConfigManager.cpp:11-504 (HF layout, config.json)
//   Model::Init / BeginInfer       src/models/Model.cpp:10-41
//   Model::Infer                   src/models/Model.cpp:43-48 -> ModelBase::Infer
//   last-row select + Sample       src/ChatSession.cpp:136-140, 560-593
//
// It writes the last-row logits of every step (float32) and the chosen ids to
// a binary file, and prints one JSON line with the per-token wall time measured
// the way ChatSession does (src/ChatSession.cpp:129-147, 242: the first token is
// excluded).
//
// Usage:
//   ref_harness --model <hf_repo_root> --prompt <ids.bin int64> --decode <n>
//               [--out <file>] [--kvgb <n>] [--nokv] [--topk K --temp T --seed S]
//               [--mask <ids.bin int64>] [--threads N] [--warmup W]
//   ref_harness --sample-fixture <in.bin> <out.bin> --topk K --temp T [--mask <ids.bin int64>]
// --warmup W leaves the first W decode tokens out of the timed sum.
// --sample-fixture runs only ChatSession::Sample's LibTorch ops (without the
// draw) on given FP16 logit rows on the CUDA device: in.bin = int64 rows,
// int64 V, rows x V FP16 bit patterns; out.bin per row = int64 argmax id,
// K x int64 top-k ids, K x FP16 top-k values, K x FP16 softmax probabilities.
#include "Model.h"
#include "ConfigManager.h"
#include <torch/torch.h>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <limits>
#include <iostream>
#include <string>
#include <vector>

namespace
{
std::vector<int64_t> read_ids(const std::string &path)
{
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f)
        throw std::runtime_error("cannot open " + path);
    auto n = static_cast<size_t>(f.tellg()) / sizeof(int64_t);
    std::vector<int64_t> v(n);
    f.seekg(0);
    f.read(reinterpret_cast<char *>(v.data()), n * sizeof(int64_t));
    return v;
}

// Restatement of ChatSession::Sample (src/ChatSession.cpp:560-593) with the
// same LibTorch ops in the same order: greedy argmax, or divide by the
// temperature in the working dtype, set every masked special id to -1e9,
// topk(K), softmax over the K values, multinomial(p, 1), gather.
int64_t sample_like_reference(torch::Tensor &last, bool greedy, int topk, float temp,
                              const std::vector<int64_t> &masked)
{
    torch::Tensor next;
    if (greedy)
    {
        next = last.argmax(-1);
    }
    else
    {
        torch::Tensor scaled = last / temp;
        for (auto id : masked)
            scaled[0][id] = -1e9f;
        auto tk = torch::topk(scaled, topk, -1);
        torch::Tensor probs = torch::softmax(std::get<0>(tk), -1);
        torch::Tensor pick = torch::multinomial(probs, 1);
        next = std::get<1>(tk).gather(-1, pick);
    }
    return next.to(torch::kCPU, false, true).item<int64_t>();
}
// The greedy pick and the top-k candidates of ChatSession::Sample
// (src/ChatSession.cpp:560-593) on FP16 rows, with the same ops in the same
// order, everything before torch::multinomial.
int sample_fixture(const std::string &in_path, const std::string &out_path, int topk, float temp,
                   const std::vector<int64_t> &masked)
{
    std::ifstream f(in_path, std::ios::binary);
    if (!f)
        throw std::runtime_error("cannot open " + in_path);
    int64_t rows = 0, V = 0;
    f.read(reinterpret_cast<char *>(&rows), 8);
    f.read(reinterpret_cast<char *>(&V), 8);
    std::vector<uint16_t> buf((size_t)V);
    FILE *out = std::fopen(out_path.c_str(), "wb");
    if (!out)
        throw std::runtime_error("cannot write " + out_path);
    for (int64_t r = 0; r < rows; r++)
    {
        f.read(reinterpret_cast<char *>(buf.data()), V * 2);
        torch::Tensor last = torch::from_blob(buf.data(), {1, V}, torch::kInt16)
                                 .clone()
                                 .view(torch::kHalf)
                                 .to(torch::Device(torch::kCUDA));
        int64_t greedy = last.argmax(-1).to(torch::kCPU).item<int64_t>();
        torch::Tensor scaled = last / temp;
        // ChatSession writes -1e9f (ChatSession.cpp:573-576), which BF16 holds;
        // LibTorch refuses to convert it to FP16 ("cannot be converted to type
        // c10::Half without overflow"), so on FP16 logits the masked ids get
        // -inf, the value -1e9 takes in any FP16 rounding
        for (auto id : masked)
            scaled[0][id] = -std::numeric_limits<float>::infinity();
        auto tk = torch::topk(scaled, topk, -1);
        torch::Tensor probs = torch::softmax(std::get<0>(tk), -1);
        torch::Tensor ids = std::get<1>(tk).to(torch::kCPU).contiguous();
        torch::Tensor vals = std::get<0>(tk).to(torch::kCPU).contiguous().view(torch::kInt16);
        torch::Tensor pr = probs.to(torch::kCPU).contiguous().view(torch::kInt16);
        std::fwrite(&greedy, 8, 1, out);
        std::fwrite(ids.data_ptr<int64_t>(), 8, topk, out);
        std::fwrite(vals.data_ptr<int16_t>(), 2, topk, out);
        std::fwrite(pr.data_ptr<int16_t>(), 2, topk, out);
    }
    std::fclose(out);
    std::printf("{\"rows\": %lld, \"vocab\": %lld, \"topk\": %d}\n", (long long)rows, (long long)V, topk);
    return 0;
}
} // namespace

int main(int argc, char **argv)
{
    std::string model, prompt_path, out_path, mask_path;
    int n_decode = 8, kvgb = 2, topk = 0, threads = 0, warmup = 0;
    float temp = 0.6f;
    int64_t seed = 0;
    bool kv = true;
    std::string fixture_in, fixture_out;

    for (int i = 1; i < argc; i++)
    {
        std::string a = argv[i];
        auto next = [&](void) -> std::string {
            if (i + 1 >= argc)
                throw std::runtime_error("missing value for " + a);
            return argv[++i];
        };
        if (a == "--model") model = next();
        else if (a == "--prompt") prompt_path = next();
        else if (a == "--decode") n_decode = std::stoi(next());
        else if (a == "--out") out_path = next();
        else if (a == "--kvgb") kvgb = std::stoi(next());
        else if (a == "--nokv") kv = false;
        else if (a == "--topk") topk = std::stoi(next());
        else if (a == "--temp") temp = std::stof(next());
        else if (a == "--seed") seed = std::stoll(next());
        else if (a == "--mask") mask_path = next();
        else if (a == "--threads") threads = std::stoi(next());
        else if (a == "--warmup") warmup = std::stoi(next());
        else if (a == "--sample-fixture")
        {
            fixture_in = next();
            fixture_out = next();
        }
        else throw std::runtime_error("unknown argument " + a);
    }
    if (threads > 0)
        torch::set_num_threads(threads);
    torch::manual_seed(seed);
    if (!fixture_in.empty())
        return sample_fixture(fixture_in, fixture_out, topk, temp,
                              mask_path.empty() ? std::vector<int64_t>() : read_ids(mask_path));

    // CLI-level settings, as src/main.cpp:20-402 would set them; ConfigManager::Load
    // then fills the rest from the HF snapshot (refs/main -> snapshots/<hash>).
    ConfigManager::ModelPath = model;
    ConfigManager::KVCacheSizeInGB = kvgb;
    ConfigManager::IsKVCacheEnabled = kv;
    ConfigManager::IsGreedy = (topk == 0);
    ConfigManager::TopK = topk > 0 ? topk : 40;
    ConfigManager::Temp = temp;
    ConfigManager::IsShowLoadedWeights = true;
    ConfigManager::IsDebuggingEnabled = false;
    ConfigManager::IsTorchChecksEnabled = false;
    ConfigManager::IsServicesRunMode = false;
    ConfigManager::IsServiceLoggingEnabled = false;
    std::string no_cfg_dir = "/nonexistent-yalama-config-dir";
    ConfigManager::Load(no_cfg_dir);

    std::vector<int64_t> prompt = read_ids(prompt_path);
    std::vector<int64_t> masked;
    if (!mask_path.empty())
        masked = read_ids(mask_path);

    auto t_load0 = std::chrono::steady_clock::now();
    Model::Init();
    auto t_load1 = std::chrono::steady_clock::now();

    FILE *out = nullptr;
    if (!out_path.empty())
    {
        out = std::fopen(out_path.c_str(), "wb");
        if (!out)
            throw std::runtime_error("cannot write " + out_path);
    }

    std::vector<int> eos_per_prompt;
    torch::Tensor input = torch::tensor(prompt, torch::kInt64).unsqueeze(0).to(torch::kCUDA);
    Model::BeginInfer();

    double token_times = 0.0, first_time = 0.0;
    int generated = 0;
    int error = 0;
    std::vector<int64_t> ids;
    for (int step = 0; step <= n_decode; step++)
    {
        auto t0 = std::chrono::steady_clock::now();
        GenerationResult r = Model::Infer(input, eos_per_prompt);
        if (!r.IsSuccess)
        {
            error = static_cast<int>(r.Error);
            break;
        }
        torch::Tensor last = r.Logits.select(1, input.size(1) - 1);
        bool greedy = ConfigManager::IsGreedy.value() || generated == 0;
        int64_t id = sample_like_reference(last, greedy, ConfigManager::TopK, ConfigManager::Temp, masked);
        auto t1 = std::chrono::steady_clock::now();
        double dt = std::chrono::duration<double>(t1 - t0).count();
        if (generated > warmup)
            token_times += dt;
        else if (generated == 0)
            first_time = dt;
        generated++;
        ids.push_back(id);
        if (out)
        {
            torch::Tensor row = last.to(torch::kCPU).to(torch::kFloat32).contiguous().view({-1});
            int64_t v = row.numel();
            std::fwrite(&v, sizeof(v), 1, out);
            std::fwrite(row.data_ptr<float>(), sizeof(float), v, out);
            std::fwrite(&id, sizeof(id), 1, out);
        }
        // next input: the sampled id alone with the KV cache, or the whole
        // sequence without it (src/ChatSession.cpp:216-224)
        torch::Tensor nxt = torch::tensor({id}, torch::TensorOptions().dtype(torch::kInt64).device(torch::kCUDA)).unsqueeze(0);
        input = kv ? nxt : torch::cat({input, nxt}, 1);
    }
    if (out)
        std::fclose(out);

    const int timed = generated - 1 - warmup;
    double tps = (timed <= 0 ? 0.0 : timed / (token_times == 0.0 ? 1.0 : token_times));
    std::printf("{\"generated\": %d, \"error\": %d, \"first_token_s\": %.6f, \"decode_s\": %.6f, "
                "\"tokens_per_second\": %.6f, \"load_s\": %.3f, \"threads\": %d, \"prompt_len\": %zu, \"timed_tokens\": %d}\n",
                generated, error, first_time, token_times, tps,
                std::chrono::duration<double>(t_load1 - t_load0).count(),
                (int)torch::get_num_threads(), prompt.size(), timed > 0 ? timed : 0);
    return 0;
}
