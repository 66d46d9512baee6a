// A chat driver over the drop-in Model facade: the reference's own
// ChatSession, tokenizer, chat templates and ConfigManager (compiled
// unmodified where they lie, see yalama_b200/host/Makefile) on top of
// yalama_b200/host/Model.cpp and the engine library, instead of the LibTorch
// ModelBase forward. It sets ConfigManager up the way src/main.cpp:20-458 does
// for the REPL, runs ChatSession::Generate (src/ChatSession.cpp:64-277) on one
// OpenAI-style request, and prints one JSON line with the emitted text and the
// token ids every Model::Infer call received (the prompt, then each generated
// id that ChatSession fed back).
//
//   facade_chat --model <hf_root> --message <text> [--kvgb N] [--topk K --temp T]
#include "ChatSession.h"
#include "ConfigManager.h"
#include "Model.h"

#include <cstdio>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

void Model_RecordInputs(bool on);
const std::vector<std::vector<int64_t>> &Model_RecordedInputs();

namespace
{
std::string json_escape(const std::string &s)
{
    std::ostringstream o;
    for (unsigned char c : s)
    {
        if (c == '"' || c == '\\')
            o << '\\' << c;
        else if (c < 0x20)
        {
            char b[8];
            std::snprintf(b, sizeof(b), "\\u%04x", c);
            o << b;
        }
        else
            o << c;
    }
    return o.str();
}

std::string ids_json(const std::vector<int64_t> &v)
{
    std::ostringstream o;
    o << '[';
    for (size_t i = 0; i < v.size(); i++)
        o << (i ? "," : "") << v[i];
    o << ']';
    return o.str();
}
} // namespace

int main(int argc, char **argv)
{
    std::string model, message = "Hello there";
    int kvgb = 2, topk = 0;
    float temp = 0.6f;
    for (int i = 1; i < argc; i++)
    {
        std::string a = argv[i];
        auto next = [&]() -> std::string {
            if (i + 1 >= argc)
                throw std::runtime_error("missing value for " + a);
            return argv[++i];
        };
        if (a == "--model") model = next();
        else if (a == "--message") message = next();
        else if (a == "--kvgb") kvgb = std::stoi(next());
        else if (a == "--topk") topk = std::stoi(next());
        else if (a == "--temp") temp = std::stof(next());
        else
        {
            std::cerr << "usage: facade_chat --model <hf_root> --message <text> [--kvgb N] [--topk K --temp T]\n";
            return 2;
        }
    }
    if (model.empty())
    {
        std::cerr << "usage: facade_chat --model <hf_root> --message <text> [--kvgb N] [--topk K --temp T]\n";
        return 2;
    }

    // the REPL's settings (src/main.cpp), then the HF snapshot's config
    ConfigManager::ModelPath = model;
    ConfigManager::KVCacheSizeInGB = kvgb;
    ConfigManager::IsKVCacheEnabled = true;
    ConfigManager::IsGreedy = (topk == 0);
    ConfigManager::TopK = topk > 0 ? topk : 40;
    ConfigManager::Temp = temp;
    ConfigManager::IsServicesRunMode = false;
    ConfigManager::IsServiceLoggingEnabled = false;
    ConfigManager::IsShowLoadedWeights = false;
    ConfigManager::IsDebuggingEnabled = false;
    ConfigManager::IsTorchChecksEnabled = false;
    ConfigManager::IsThinkingEnabled = false;
    ConfigManager::isPrintChatTemplateOutput = false;
    std::string no_cfg_dir = "/nonexistent-yalama-config-dir";
    ConfigManager::Load(no_cfg_dir);

    Model::Init();
    Model_RecordInputs(true);
    ChatSession session;
    std::ostringstream req;
    req << "{\"messages\":[{\"role\":\"user\",\"content\":\"" << json_escape(message) << "\"}]}";
    std::string request = req.str();
    std::string text;
    bool cancel = false;
    GenerationResult r = session.Generate(request, [&](const std::string &piece) { text += piece; }, cancel);

    const auto &inputs = Model_RecordedInputs();
    std::vector<int64_t> prompt, fed;
    if (!inputs.empty())
        prompt = inputs[0];
    for (size_t i = 1; i < inputs.size(); i++)
        fed.insert(fed.end(), inputs[i].begin(), inputs[i].end());
    std::cout << "\n{\"ok\": " << (r.IsSuccess ? "true" : "false") << ", \"error\": " << static_cast<int>(r.Error)
              << ", \"max_seq\": " << ConfigManager::MaxSequenceLength << ", \"prompt\": " << ids_json(prompt)
              << ", \"fed\": " << ids_json(fed) << ", \"text\": \"" << json_escape(text) << "\"}" << std::endl;
    return r.IsSuccess ? 0 : 1;
}
