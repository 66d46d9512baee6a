// Encode one text with the reference's tokenizer class and with its FastBpe
// wrapper (FastTokenizer.h), check that the ids are equal and time both.
//
//   tokenizer_bench --model <dir with tokenizer.json> --family llama|qwen|mistral
//                   --text <file> [--reps N] [--ref-reps M] [--ids-out <file>]
//
// Prints one JSON line: token count, equality, the first differing position
// (-1 if none), and the median wall time of each encoder in milliseconds
// (EncodeWithoutChatTemplate: byte encoding, special-token segmentation, BPE
// and the vocabulary lookup, as TokenizerBase::Encode runs them). The BPE cache
// is cleared before every timed encode, so each one does the full work.
#include "ConfigManager.h"
#include "FastTokenizer.h"

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <fstream>
#include <iostream>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace
{
// Exposes the protected members the bench needs (cache reset) without
// changing the tokenizer's behaviour.
template <class T> struct Probe : T
{
    void clear_cache() { this->_bpeCache.clear(); }
};

template <class T> double time_encode(Probe<T> &tok, const std::string &text, int reps, std::vector<int64_t> &ids)
{
    std::vector<double> ms;
    for (int r = 0; r < reps; r++)
    {
        tok.clear_cache();
        std::string t = text;
        const auto t0 = std::chrono::steady_clock::now();
        ids = tok.EncodeWithoutChatTemplate(t);
        const auto t1 = std::chrono::steady_clock::now();
        ms.push_back(std::chrono::duration<double, std::milli>(t1 - t0).count());
    }
    std::sort(ms.begin(), ms.end());
    return ms[ms.size() / 2];
}

template <class Ref, class Fast>
int run(const std::string &text, int reps, int ref_reps, const std::string &ids_out)
{
    Probe<Ref> ref;
    Probe<Fast> fast;
    ref.Init();
    fast.Init();
    std::vector<int64_t> a, b;
    const double ms_fast = time_encode(fast, text, reps, b);
    const double ms_ref = ref_reps > 0 ? time_encode(ref, text, ref_reps, a) : -1.0;
    long first_diff = -1;
    if (ref_reps > 0)
    {
        const size_t n = std::min(a.size(), b.size());
        for (size_t i = 0; i < n && first_diff < 0; i++)
            if (a[i] != b[i])
                first_diff = (long)i;
        if (first_diff < 0 && a.size() != b.size())
            first_diff = (long)n;
    }
    if (!ids_out.empty())
    {
        std::ofstream f(ids_out, std::ios::binary);
        f.write(reinterpret_cast<const char *>(b.data()), (std::streamsize)(b.size() * sizeof(int64_t)));
    }
    std::printf("{\"bytes\": %zu, \"tokens\": %zu, \"ref_tokens\": %zu, \"equal\": %s, \"first_diff\": %ld, "
                "\"fast_ms\": %.4f, \"ref_ms\": %.4f, \"reps\": %d, \"ref_reps\": %d}\n",
                text.size(), b.size(), a.size(), (ref_reps > 0 && first_diff < 0) ? "true" : "false", first_diff,
                ms_fast, ms_ref, reps, ref_reps);
    return 0;
}
} // namespace

int main(int argc, char **argv)
{
    std::string model, family, text_path, ids_out;
    int reps = 5, ref_reps = 1;
    for (int i = 1; i < argc; i++)
    {
        const std::string a = argv[i];
        auto next = [&]() -> std::string {
            if (i + 1 >= argc)
                throw std::runtime_error("missing value for " + a);
            return argv[++i];
        };
        if (a == "--model") model = next();
        else if (a == "--family") family = next();
        else if (a == "--text") text_path = next();
        else if (a == "--reps") reps = std::stoi(next());
        else if (a == "--ref-reps") ref_reps = std::stoi(next());
        else if (a == "--ids-out") ids_out = next();
        else
        {
            std::cerr << "usage: tokenizer_bench --model <dir> --family llama|qwen|mistral --text <file> "
                         "[--reps N] [--ref-reps M] [--ids-out <file>]\n";
            return 2;
        }
    }
    if (model.empty() || text_path.empty() || reps < 1)
    {
        std::cerr << "tokenizer_bench: --model and --text are required\n";
        return 2;
    }
    std::ifstream f(text_path, std::ios::binary);
    if (!f)
    {
        std::cerr << "tokenizer_bench: cannot read " << text_path << "\n";
        return 2;
    }
    std::stringstream ss;
    ss << f.rdbuf();
    const std::string text = ss.str();
    ConfigManager::ModelPath = model;
    ConfigManager::IsDebuggingEnabled = false;
    // LoadFromJson prints one line to stdout: keep stdout for the JSON result
    std::streambuf *saved = std::cout.rdbuf(std::cerr.rdbuf());
    int rc = 2;
    try
    {
        if (family == "llama")
            rc = run<LlamaTokenizer, ylm_host::FastLlamaTokenizer>(text, reps, ref_reps, ids_out);
        else if (family == "qwen")
            rc = run<QwenTokenizer, ylm_host::FastQwenTokenizer>(text, reps, ref_reps, ids_out);
        else if (family == "mistral")
            rc = run<MistralTokenizer, ylm_host::FastMistralTokenizer>(text, reps, ref_reps, ids_out);
        else
            std::cerr << "tokenizer_bench: unknown family " << family << "\n";
    }
    catch (const std::exception &e)
    {
        std::cout.rdbuf(saved);
        std::cerr << "tokenizer_bench: " << e.what() << "\n";
        return 1;
    }
    std::cout.rdbuf(saved);
    return rc;
}
