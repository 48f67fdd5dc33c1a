// sampler.cpp — the reference's host-side nucleus sampler (src/model/qwen3.cu:351-460), restated
// step for step so that, given the same logits and the same mt19937 state, it returns the same id:
//   1. repetition penalty applied once per occurrence in the history (duplicates compound):
//      logit > 0 ? logit / rp : logit * rp
//   2. min-p: logits below max + log(min_p) are dropped (set to -1e30)
//   3. entropy-scaled temperature: T *= clamp(H / 2, 0.5, 2), H over the surviving softmax
//   4. softmax at temperature T over survivors, full descending sort (std::sort, as the reference)
//   5. top-k limit, then the shortest prefix whose cumulative mass reaches top_p
//   6. std::discrete_distribution over the kept (un-renormalised) probabilities
// The only deliberate difference: the engine seeds its mt19937 explicitly where the reference
// draws the seed from std::random_device.
#include <algorithm>
#include <cmath>
#include <random>
#include <utility>
#include <vector>

namespace fence {

int host_sample_nucleus(const float* logits_in, int vocab, const int* history, int n_history, float temperature,
                        float top_p, int top_k, float rep_penalty, float min_p, bool dynamic_temp,
                        std::mt19937& rng) {
    std::vector<float> l(logits_in, logits_in + vocab);
    if (rep_penalty > 1.0f && n_history > 0) {
        for (int h = 0; h < n_history; ++h) {
            const int tok = history[h];
            if (tok >= 0 && tok < vocab) {
                if (l[tok] > 0) l[tok] /= rep_penalty;
                else l[tok] *= rep_penalty;
            }
        }
    }
    float max_l = -1e30f;
    for (int i = 0; i < vocab; ++i) max_l = std::max(max_l, l[i]);
    if (min_p > 0.0f) {
        const float thr = max_l + logf(min_p);
        for (int i = 0; i < vocab; ++i)
            if (l[i] < thr) l[i] = -1e30f;
    }
    float temp = temperature;
    if (dynamic_temp) {
        float dyn_sum = 0.0f;
        for (int i = 0; i < vocab; ++i)
            if (l[i] > -1e20f) dyn_sum += expf(l[i] - max_l);
        float entropy = 0.0f;
        for (int i = 0; i < vocab; ++i)
            if (l[i] > -1e20f) {
                const float p = expf(l[i] - max_l) / dyn_sum;
                if (p > 1e-6f) entropy -= p * logf(p);
            }
        const float scale = std::clamp(entropy / 2.0f, 0.5f, 2.0f);
        temp *= scale;
    }
    float sum = 0.0f;
    for (int i = 0; i < vocab; ++i) {
        if (l[i] < -1e20f) {
            l[i] = 0.0f;
            continue;
        }
        const float p = expf((l[i] - max_l) / temp);
        l[i] = p;
        sum += p;
    }
    for (int i = 0; i < vocab; ++i) l[i] /= sum;
    std::vector<std::pair<float, int>> probs;
    probs.reserve(vocab);
    for (int i = 0; i < vocab; ++i) probs.push_back({l[i], i});
    std::sort(probs.begin(), probs.end(), [](const auto& a, const auto& b) { return a.first > b.first; });
    const int limit = std::min(vocab, top_k);
    float cumul = 0.0f;
    int actual_k = limit;
    for (int i = 0; i < limit; ++i) {
        cumul += probs[i].first;
        if (cumul >= top_p) {
            actual_k = i + 1;
            break;
        }
    }
    std::vector<float> final_probs(actual_k);
    for (int i = 0; i < actual_k; ++i) final_probs[i] = probs[i].first;
    std::discrete_distribution<int> dist(final_probs.begin(), final_probs.end());
    return probs[dist(rng)].second;
}

}  // namespace fence
