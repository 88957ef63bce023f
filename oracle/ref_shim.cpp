// TEST INFRASTRUCTURE ONLY (oracle). C entry points over the reference's own host code, which
// is compiled unmodified from its sources by `make -C oracle ref`:
//   breeze::sample_token      sharjeel103/bz-ggml src/sampling.cpp:9-60
//   breeze::save_voice/load   sharjeel103/bz-ggml src/voice.cpp:16-67
//   breeze::split_text        sharjeel103/bz-ggml src/text_split.cpp:89-111
//   breeze::write_wav         sharjeel103/bz-ggml src/audio.cpp:80-107
// The tests use them to pin the engine's sampler semantics (suppression, repetition penalty,
// top-k, temperature), the BRZV voice-file format, the long-text splitter and the WAV layout
// against the reference itself.
#include "breeze/audio.h"
#include "breeze/generation.h"
#include "breeze/sampling.h"
#include "breeze/voice.h"

#include <cstring>
#include <random>
#include <string>
#include <vector>

extern "C" int ref_sample_tokens(const float * logits, int n, float temp, int top_k, float top_p, float rep,
                                 const int * hist, int n_hist, int sup_lo, int sup_hi, unsigned seed, int n_draws,
                                 int * out) {
    // one std::mt19937 per call, seeded like the reference's per-session engine; every draw
    // starts from the unmodified logits (sample_token edits its argument in place)
    std::mt19937 rng(seed);
    breeze::SampleParams p;
    p.temperature = temp;
    p.top_k = top_k;
    p.top_p = top_p;
    p.repetition_penalty = rep;
    std::vector<int> h(hist, hist + (hist ? n_hist : 0));
    std::vector<int> sup;
    for (int t = sup_lo; t < sup_hi; t++) sup.push_back(t);
    for (int d = 0; d < n_draws; d++) {
        std::vector<float> l(logits, logits + n);
        out[d] = breeze::sample_token(l, p, rng, h.empty() ? nullptr : &h, sup.empty() ? nullptr : &sup);
    }
    return 0;
}

extern "C" int ref_voice_save(const char * path, const char * text, const int * codes, int frames, int n_codebooks,
                              int sample_rate) {
    breeze::Voice v;
    v.text = text ? text : "";
    v.frames = frames;
    v.n_codebooks = n_codebooks;
    v.sample_rate = sample_rate;
    v.codes.assign(codes, codes + (size_t) frames * n_codebooks);
    return breeze::save_voice(path, v) ? 0 : -1;
}

// returns frames*n_codebooks codes written to out (up to max_codes), or -1
extern "C" int ref_voice_load(const char * path, char * name, int name_cap, char * text, int text_cap, int * out,
                              int max_codes, int * frames, int * n_codebooks, int * sample_rate) {
    breeze::Voice v;
    if (!breeze::load_voice(path, v)) return -1;
    if ((int) v.codes.size() > max_codes) return -1;
    std::memcpy(out, v.codes.data(), v.codes.size() * sizeof(int));
    if (name && name_cap > 0) {
        std::strncpy(name, v.name.c_str(), name_cap - 1);
        name[name_cap - 1] = 0;
    }
    if (text && text_cap > 0) {
        std::strncpy(text, v.text.c_str(), text_cap - 1);
        text[text_cap - 1] = 0;
    }
    *frames = v.frames;
    *n_codebooks = v.n_codebooks;
    *sample_rate = v.sample_rate;
    return (int) v.codes.size();
}

// pieces NUL-terminated one after another; returns the count, or -(bytes needed)
extern "C" int ref_split_text(const char * text, int budget, int first_budget, char * out, int cap) {
    const std::vector<std::string> parts = breeze::split_text(text, budget, first_budget);
    size_t need = 0;
    for (const std::string & p : parts) need += p.size() + 1;
    if ((size_t) cap < need) return -(int) need;
    for (const std::string & p : parts) {
        std::memcpy(out, p.data(), p.size());
        out += p.size();
        *out++ = 0;
    }
    return (int) parts.size();
}

extern "C" int ref_write_wav(const char * path, const float * samples, int n, int sample_rate) {
    return breeze::write_wav(path, std::vector<float>(samples, samples + n), sample_rate) ? 0 : -1;
}
