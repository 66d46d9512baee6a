// Byte-level BPE encoding in O(n log n) behind the reference's tokenizer
// classes.
//
// TokenizerBase::ApplyBPE (src/tokenizer/TokenizerBase.cpp:270-424) finds
// each merge by rescanning the rank of every adjacent pair and erasing from the
// middle of a vector, so one piece of n symbols costs O(n^2). The Qwen and
// Mistral tokenizers hand it the whole text between special tokens as one
// piece (src/tokenizer/QwenTokenizer.cpp:8-15, MistralTokenizer.cpp:9-16), so
// the cost grows with the square of the prompt. SegmentInput
// (TokenizerBase.cpp:622-684) searches the whole rest of the text for every
// special token once per special token found.
//
// FastBpe<Base> overrides those two members of any of the reference's
// tokenizer classes and returns the same pieces in the same order:
//  - ApplyBPE: the symbols in a doubly linked list, candidate pairs in a
//    min-heap keyed by (merge rank, position of the left symbol). Popping the
//    smallest key is the reference's choice (lowest rank, leftmost among equal
//    ranks: positions keep list order because a merged symbol keeps its left
//    part's position). Entries made stale by a merge are skipped by checking
//    that both symbols are unchanged since the entry was pushed.
//  - SegmentInput: one cached next occurrence per special token, searched
//    again only once the cursor has passed it; the earliest occurrence wins and
//    equal positions go to the token met first in the same iteration order of
//    _specialTokens, as in the reference.
// Everything else (vocabulary, merges, byte encoders, Encode, Decode, the BPE
// cache and its 50000-entry limit) is the base class's.
#pragma once

#include "LlamaTokenizer.h"
#include "MistralTokenizer.h"
#include "QwenTokenizer.h"

#include <string>
#include <unordered_map>
#include <vector>

namespace ylm_host
{
// Merge `symbols` by the ranks in `merge_ranks` ("left right" -> rank).
std::vector<std::string> bpe_merge(const std::vector<std::string> &symbols,
                                   const std::unordered_map<std::string, int> &merge_ranks);

// Split `text` at the special tokens: the text between them goes through
// `split` (the tokenizer's SplitText), each special token is one piece.
template <class SplitFn>
std::vector<std::string> segment_specials(const std::string &text, const std::unordered_map<int, std::string> &specials,
                                          SplitFn split)
{
    struct Cand
    {
        const std::string *tok;
        size_t next;
    };
    std::vector<Cand> cands;
    cands.reserve(specials.size());
    for (const auto &kv : specials)
        if (!kv.second.empty()) // an empty token would match everywhere (the reference would not terminate)
            cands.push_back({&kv.second, text.find(kv.second)});
    std::vector<std::string> out;
    size_t off = 0;
    const size_t n = text.size();
    while (off < n)
    {
        size_t best = std::string::npos;
        const std::string *tok = nullptr;
        for (auto &c : cands)
        {
            if (c.next != std::string::npos && c.next < off)
                c.next = text.find(*c.tok, off);
            if (c.next != std::string::npos && (best == std::string::npos || c.next < best))
            {
                best = c.next;
                tok = c.tok;
            }
        }
        if (tok == nullptr)
        {
            std::vector<std::string> s = split(text.substr(off));
            out.insert(out.end(), std::make_move_iterator(s.begin()), std::make_move_iterator(s.end()));
            break;
        }
        if (best > off)
        {
            std::vector<std::string> s = split(text.substr(off, best - off));
            out.insert(out.end(), std::make_move_iterator(s.begin()), std::make_move_iterator(s.end()));
        }
        out.push_back(*tok);
        off = best + tok->size();
    }
    return out;
}

template <class Base> class FastBpe : public Base
{
  public:
    FastBpe() = default;

  protected:
    std::vector<std::string> ApplyBPE(const std::vector<std::string> &inputChars) override
    {
        // the reference's cache policy (TokenizerBase.cpp:272-280, 414-419)
        auto it = this->_bpeCache.find(inputChars);
        if (it != this->_bpeCache.end())
            return it->second;
        std::vector<std::string> result = bpe_merge(inputChars, this->_mergeRanks);
        if (this->_bpeCache.size() > 50000)
            this->_bpeCache.clear();
        this->_bpeCache[inputChars] = result;
        return result;
    }

    std::vector<std::string> SegmentInput(std::string &encodedInput) override
    {
        std::vector<std::string> out = segment_specials(encodedInput, this->_specialTokens,
                                                        [this](const std::string &s) { return this->SplitText(s); });
        encodedInput.clear(); // the reference consumes its argument
        return out;
    }
};

using FastLlamaTokenizer = FastBpe<LlamaTokenizer>;
using FastQwenTokenizer = FastBpe<QwenTokenizer>;
using FastMistralTokenizer = FastBpe<MistralTokenizer>;
} // namespace ylm_host
