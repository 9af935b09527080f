// prompt_fit.h — the prompt decisions fish_generate makes before the first
// forward: fitting an over-long prompt into the context, and how much of it
// the one-slot KV prefix cache already holds. Host code only; the generation
// loop in c_api.cpp and the host-only fbx_prompt_* entry points both call it.
#pragma once

#include <algorithm>
#include <cstdint>
#include <vector>

namespace fb {

// The last cut of an over-long prompt: kept = ids[0, head) + ids[drop_end, n).
// It is applied again while it still fits and the head tokens are the same,
// so the kept prompt of the next turn extends the cached one.
struct PromptCut {
    int head = 0, drop_end = 0;
    std::vector<int32_t> head_ids;
};

// Head + tail fit of generate_ids_locked (model/fish/src/c_api.cpp:516-552):
// reserve max(64, min(max_tokens, n_ctx/4)) positions for the answer, keep the
// prompt when it fits the remaining budget (at least 32), otherwise reuse the
// previous cut if it still fits, else cut anew with a head of budget/4 and a
// tail of budget - budget/4 - budget/4 (at least 1), dropping a quarter of the
// budget more than needed so the following turns fit under the same cut.
// `max_tokens` is the caller's value after <= 0 was replaced by n_ctx.
// Returns true when `ids` was cut.
inline bool fit_prompt(std::vector<int32_t>& ids, int n_ctx, int max_tokens, PromptCut& cut) {
    const int reserve = std::max(64, std::min(max_tokens, n_ctx / 4));
    const int budget = std::max(32, n_ctx - reserve);
    const int n = (int)ids.size();
    if (n <= budget) {
        cut = PromptCut{};
        return false;
    }
    int head = cut.head, drop_end = cut.drop_end;
    const bool reuse = head > 0 && drop_end > head && drop_end < n && n - (drop_end - head) <= budget &&
                       (int)cut.head_ids.size() == head && std::equal(cut.head_ids.begin(), cut.head_ids.end(), ids.begin());
    if (!reuse) {
        head = budget / 4;
        const int tail = std::max(1, budget - head - budget / 4);
        drop_end = n - tail;
        cut.head = head;
        cut.drop_end = drop_end;
        cut.head_ids.assign(ids.begin(), ids.begin() + head);
    }
    std::vector<int32_t> kept(ids.begin(), ids.begin() + head);
    kept.insert(kept.end(), ids.begin() + drop_end, ids.end());
    ids.swap(kept);
    return true;
}

// Tokens of `ids` whose KV the cache already holds (c_api.cpp:555-567): the
// longest common prefix with the cached ids, one less for an identical prompt
// (its last token must run to give logits), and 0 below 8 tokens.
inline int cached_prefix(const std::vector<int32_t>& ids, const std::vector<int32_t>& cache_ids) {
    const int lim = (int)std::min(ids.size(), cache_ids.size());
    int prefix = 0;
    while (prefix < lim && ids[prefix] == cache_ids[prefix]) ++prefix;
    if (prefix >= (int)ids.size()) prefix = (int)ids.size() - 1;
    if (prefix < 8) prefix = 0;
    return prefix;
}

}  // namespace fb
