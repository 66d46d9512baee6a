// The O(n log n) merge loop behind FastBpe::ApplyBPE (see FastTokenizer.h).
#include "FastTokenizer.h"

#include <climits>
#include <cstdint>
#include <queue>

namespace ylm_host
{
namespace
{
struct Cand
{
    int rank;
    int left;            // position of the left symbol (list order = position order)
    int right;           // position of the right symbol when pushed
    uint32_t vl, vr;     // both symbols' versions when pushed
    bool operator>(const Cand &o) const { return rank != o.rank ? rank > o.rank : left > o.left; }
};
} // namespace

std::vector<std::string> bpe_merge(const std::vector<std::string> &symbols,
                                   const std::unordered_map<std::string, int> &merge_ranks)
{
    const int n = (int)symbols.size();
    if (n < 2)
        return symbols;
    std::vector<std::string> sym(symbols);
    std::vector<int> next(n), prev(n);
    std::vector<uint32_t> ver(n, 0);
    for (int i = 0; i < n; i++)
    {
        next[i] = i + 1 < n ? i + 1 : -1;
        prev[i] = i - 1;
    }
    std::string key;
    key.reserve(64);
    // the rank of the pair (a, b): "a b" in the merge table (TokenizerBase.cpp:294-313)
    auto rank_of = [&](int a, int b) {
        key.assign(sym[a]);
        key.push_back(' ');
        key.append(sym[b]);
        auto it = merge_ranks.find(key);
        return it == merge_ranks.end() ? INT_MAX : it->second;
    };
    std::vector<Cand> store;
    store.reserve((size_t)n * 2);
    std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> heap(std::greater<Cand>(), std::move(store));
    auto push = [&](int a) {
        const int b = next[a];
        if (b < 0)
            return;
        const int r = rank_of(a, b);
        if (r != INT_MAX)
            heap.push({r, a, b, ver[a], ver[b]});
    };
    for (int i = 0; i + 1 < n; i++)
        push(i);
    while (!heap.empty())
    {
        const Cand c = heap.top();
        heap.pop();
        // stale: either symbol merged (or died) since the pair was pushed
        if (ver[c.left] != c.vl || ver[c.right] != c.vr || next[c.left] != c.right)
            continue;
        const int a = c.left, b = c.right;
        sym[a] += sym[b];
        sym[b].clear();
        ver[a]++;
        ver[b]++; // b is gone: every pair that names it is stale
        next[a] = next[b];
        if (next[b] >= 0)
            prev[next[b]] = a;
        next[b] = -1;
        if (prev[a] >= 0)
            push(prev[a]);
        push(a);
    }
    std::vector<std::string> out;
    out.reserve(n);
    for (int i = 0; i >= 0; i = next[i])
        out.push_back(std::move(sym[i]));
    return out;
}
} // namespace ylm_host
