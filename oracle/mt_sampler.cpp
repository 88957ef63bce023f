// TEST INFRASTRUCTURE ONLY (oracle): the reference's host sampler restated with the same C++
// standard-library engine and distribution (sharjeel103/bz-ggml src/sampling.cpp:9-60):
// suppression, per-occurrence repetition penalty, top-k by partial sort, softmax at
// temperature, optional top-p, then std::discrete_distribution over std::mt19937. Used by the
// tests to check the engine's Philox sampler distributionally against this one.
#include <algorithm>
#include <cmath>
#include <random>
#include <vector>

namespace {
int sample_once(std::vector<float> logits, float temp_in, int top_k, float top_p, float rep, const int * hist,
                int n_hist, int sup_lo, int sup_hi, std::mt19937 & rng) {
    const int n = (int) logits.size();
    for (int t = sup_lo; t < sup_hi; t++)
        if (t >= 0 && t < n) logits[t] = -std::numeric_limits<float>::infinity();
    if (hist && rep != 1.0f) {
        for (int i = 0; i < n_hist; i++) {
            const int t = hist[i];
            if (t < 0 || t >= n) continue;
            logits[t] = logits[t] > 0 ? logits[t] / rep : logits[t] * rep;
        }
    }
    const float temp = temp_in > 0 ? temp_in : 1.0f;
    std::vector<int> idx(n);
    for (int i = 0; i < n; i++) idx[i] = i;
    const int keep = (top_k > 0 && top_k < n) ? top_k : n;
    std::partial_sort(idx.begin(), idx.begin() + keep, idx.end(), [&](int a, int b) { return logits[a] > logits[b]; });
    idx.resize(keep);
    const float maxl = logits[idx[0]];
    std::vector<float> probs(keep);
    float sum = 0.0f;
    for (int i = 0; i < keep; i++) {
        probs[i] = std::exp((logits[idx[i]] - maxl) / temp);
        sum += probs[i];
    }
    for (float & v : probs) v /= sum;
    if (top_p < 1.0f) {
        float cum = 0.0f;
        int cut = keep;
        for (int i = 0; i < keep; i++) {
            cum += probs[i];
            if (cum >= top_p) { cut = i + 1; break; }
        }
        probs.resize(cut);
        idx.resize(cut);
        float s = 0.0f;
        for (float v : probs) s += v;
        for (float & v : probs) v /= s;
    }
    std::discrete_distribution<int> dist(probs.begin(), probs.end());
    return idx[dist(rng)];
}
}  // namespace

extern "C" int oracle_sample_mt(const float * logits, int n, float temp, int top_k, float top_p, float rep,
                                const int * hist, int n_hist, int sup_lo, int sup_hi, unsigned seed, int n_draws,
                                int * out) {
    std::mt19937 rng(seed);
    std::vector<float> l(logits, logits + n);
    for (int d = 0; d < n_draws; d++) out[d] = sample_once(l, temp, top_k, top_p, rep, hist, n_hist, sup_lo, sup_hi, rng);
    return 0;
}
