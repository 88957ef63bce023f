// Single-request streaming generation over the GPU engine and vocoder (reference:
// src/generation.cpp:83-273, src/text_split.cpp:1-118, src/audio.cpp:80-107).
#include "generate.h"

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <stdexcept>

namespace bzb {

namespace {

using Clock = std::chrono::steady_clock;
double ms_since(Clock::time_point t) { return std::chrono::duration<double, std::milli>(Clock::now() - t).count(); }

// ---------------------------------------------------------------------------------- text split
// bytes of the UTF-8 sequence that starts with byte c (a stray continuation byte counts as one)
size_t utf8_bytes(unsigned char c) {
    if (c < 0x80) return 1;
    if ((c & 0xE0) == 0xC0) return 2;
    if ((c & 0xF0) == 0xE0) return 3;
    if ((c & 0xF8) == 0xF0) return 4;
    return 1;
}

// spoken weight: one per ASCII character, three per multi-byte (CJK) character
int text_weight(const std::string & s) {
    int w = 0;
    for (size_t i = 0; i < s.size(); i += utf8_bytes((unsigned char) s[i]))
        w += utf8_bytes((unsigned char) s[i]) == 1 ? 1 : 3;
    return w;
}

// full-width sentence stops: 。 ！ ？ ； … ．
bool cjk_sentence_stop(const std::string & ch) {
    static const char * const kStops[] = { "\xe3\x80\x82", "\xef\xbc\x81", "\xef\xbc\x9f", "\xef\xbc\x9b",
                                           "\xe2\x80\xa6", "\xef\xbc\x8e" };
    for (const char * s : kStops)
        if (ch == s) return true;
    return false;
}

// sentences end at a newline, at . ! ? ; followed (after closing quotes or brackets) by a space,
// a newline or the end, or at a full-width stop
std::vector<std::string> sentences_of(const std::string & t) {
    std::vector<std::string> out;
    std::string cur;
    size_t i = 0;
    while (i < t.size()) {
        const size_t n = utf8_bytes((unsigned char) t[i]);
        const std::string ch = t.substr(i, n);
        cur += ch;
        i += n;
        bool end = false;
        if (n > 1) {
            end = cjk_sentence_stop(ch);
        } else if (ch[0] == '\n') {
            end = true;
        } else if (std::strchr(".!?;", ch[0])) {
            size_t j = i;
            while (j < t.size() && std::strchr("\"')]", t[j])) j++;
            end = j == t.size() || t[j] == ' ' || t[j] == '\n';
            if (end) {
                cur.append(t, i, j - i);
                i = j;
            }
        }
        if (end) {
            out.push_back(cur);
            cur.clear();
        }
    }
    if (!cur.empty()) out.push_back(cur);
    return out;
}

// a sentence heavier than the budget is cut after a comma-like mark (, ， 、 :) or, once a quarter
// budget has passed since the last mark, after a space
std::vector<std::string> clauses_of(const std::string & s, int budget) {
    if (text_weight(s) <= budget) return { s };
    std::vector<std::string> out;
    std::string cur;
    int weight = 0, since_mark = 0;
    size_t i = 0;
    while (i < s.size()) {
        const size_t n = utf8_bytes((unsigned char) s[i]);
        const std::string ch = s.substr(i, n);
        i += n;
        cur += ch;
        const int w = n == 1 ? 1 : 3;
        weight += w;
        since_mark += w;
        const bool comma = ch == "," || ch == ":" || ch == "\xef\xbc\x8c" || ch == "\xe3\x80\x81";
        const bool space = ch == " ";
        if (weight >= budget && (comma || (space && since_mark > budget / 4))) {
            out.push_back(cur);
            cur.clear();
            weight = 0;
            since_mark = 0;
        } else if (comma || space) {
            since_mark = 0;
        }
    }
    if (!cur.empty()) out.push_back(cur);
    return out;
}

// ---------------------------------------------------------------------------------- one piece
constexpr int kGenSession = 0x47454E31;  // the engine session of the piece being generated

struct Anchor {  // the reference a piece conditions on (src/generation.cpp:78-83)
    std::vector<int> codes;
    int n_frames = 0;
    std::string text;
};

// src/generation.cpp:85-207 for one piece of text; false when the callback asked to stop
bool generate_piece(Engine & eng, Vocoder & voc, const GenRequest & req, const std::string & text,
                    const Anchor & ref, uint32_t seed, const AudioCallback & cb, GenTimings & tm,
                    Clock::time_point t_start, Anchor & made, std::vector<int> * codes_out) {
    const ModelConfig & c = eng.cfg;
    const int nc = c.nc, spf = Vocoder::kSamplesPerFrame;
    const bool has_ref = !ref.codes.empty() && !ref.text.empty();
    const bool use_cfg = req.cfg_scale != 1.0f;
    const Tokenizer & tok = eng.tokenizer();
    const std::string spk = "[S0]";
    // prompts (src/generation.cpp:26-44): the unconditional branch drops the instruction
    std::vector<std::vector<int>> segs, segs_u;
    if (has_ref) segs.push_back(tok.encode(spk + ref.text, true));
    segs.push_back(tok.encode(spk + "<ins_bos>" + req.instruction + "<ins_eos>" + text, true));
    if (use_cfg) {
        if (has_ref) segs_u.push_back(segs[0]);
        segs_u.push_back(tok.encode(spk + text, true));
    }
    const int max_new = req.max_new_tokens > 0 ? req.max_new_tokens : c.max_new_tokens;
    made = Anchor();
    made.text = text;
    if (max_new <= 0) return true;
    // sampler: the request's values, zero meaning the GGUF's (src/generation.cpp:122-126); the
    // depth codes use the GGUF's depth sampler (src/depth_decoder.cpp:134-137)
    SessionParams sp;
    sp.cfg = req.cfg_scale;
    sp.temp = req.temperature > 0.0f ? req.temperature : c.temperature;
    sp.top_k = req.top_k > 0 ? req.top_k : c.top_k;
    sp.top_p = req.top_p > 0.0f ? req.top_p : c.top_p;
    sp.rep = req.repetition_penalty > 0.0f ? req.repetition_penalty : c.rep;
    sp.dtemp = c.depth_temperature;
    sp.dtop_k = c.depth_top_k;
    sp.dtop_p = c.depth_top_p;

    auto t0 = Clock::now();
    int cb0 = -1;
    eng.session_create_tokens(kGenSession, segs, use_cfg ? &segs_u : nullptr, has_ref ? ref.codes.data() : nullptr,
                              has_ref ? ref.n_frames : 0, seed, max_new, sp, false, &cb0, nullptr);
    tm.prefill += ms_since(t0);

    std::vector<int> frames;
    std::vector<float> audio;
    int emitted = 0;
    const int chunk_max = std::max(1, req.chunk_max);
    int chunk = std::min(std::max(1, req.chunk_first), chunk_max);
    // left context of each vocoder window: the transformer window plus the convolutions' reach
    const int ctx = c.voc.window + 16;
    // src/generation.cpp:143-168
    auto flush = [&](bool final_flush) {
        const int have = (int) frames.size() / nc;
        while (have - emitted >= chunk || (final_flush && have > emitted)) {
            const int start = emitted;
            const int count = final_flush ? have - emitted : chunk;
            const int ctx_start = start > ctx ? start - ctx : 0;
            const int sub_T = start + count - ctx_start;
            audio.resize((size_t) sub_T * spf);
            const auto tv = Clock::now();
            voc.decode(frames.data() + (size_t) ctx_start * nc, sub_T, audio.data());
            tm.vocoder += ms_since(tv);
            tm.flushes++;
            if (tm.first_audio == 0) tm.first_audio = ms_since(t_start);
            if (!cb(audio.data() + (size_t) (start - ctx_start) * spf, count * spf)) return false;
            emitted += count;
            chunk = std::min(chunk + chunk / 3 + 1, chunk_max);
            if (!final_flush && have - emitted < chunk) break;
        }
        return true;
    };

    bool stopped = false;
    try {
        // an EOS first cb0 ends the piece before any frame (src/generation.cpp:171)
        bool alive = cb0 != c.bb_eos;
        int produced = 0;
        std::vector<int> burst;
        while (alive && produced < max_new && !stopped) {
            // step exactly the frames the next flush needs, so audio starts as early as frame by frame
            const int have = (int) frames.size() / nc;
            const int K = std::min({ std::max(1, chunk - (have - emitted)), max_new - produced, 64 });
            burst.assign((size_t) K * nc, -1);
            int next = -1;
            const auto ts = Clock::now();
            const StepResult r = eng.step(&kGenSession, 1, K, nullptr, true, burst.data(), nc, &next, true, true);
            tm.steps += ms_since(ts);
            for (int k = 0; k < r.steps_executed && !stopped; k++) {
                const int * f = burst.data() + (size_t) k * nc;
                produced++;
                // an all-pad frame is fed back but not voiced (src/generation.cpp:181-188)
                bool pad = true;
                for (int j = 0; j < nc; j++) pad = pad && f[j] == c.cb_pad;
                if (pad) continue;
                frames.insert(frames.end(), f, f + nc);
                tm.frames++;
                if (!flush(false)) stopped = true;
            }
            if (r.steps_executed < K || next < 0) alive = false;
        }
        if (!stopped) stopped = !flush(true);
    } catch (...) {
        eng.session_free(kGenSession);
        throw;
    }
    eng.session_free(kGenSession);
    if (codes_out) codes_out->insert(codes_out->end(), frames.begin(), frames.end());
    made.n_frames = (int) frames.size() / nc;
    made.codes = std::move(frames);
    return !stopped;
}

}  // namespace

std::vector<std::string> split_text(const std::string & text, int budget, int first_budget) {
    if (budget <= 0 || text_weight(text) <= budget) return { text };
    std::vector<std::string> out;
    std::string cur;
    int weight = 0;
    int limit = first_budget > 0 ? first_budget : budget;
    for (const std::string & sentence : sentences_of(text)) {
        for (const std::string & part : clauses_of(sentence, budget)) {
            const int w = text_weight(part);
            if (weight > 0 && weight + w > limit) {
                out.push_back(cur);
                cur.clear();
                weight = 0;
                limit = budget;
            }
            cur += part;
            weight += w;
        }
    }
    if (!cur.empty()) out.push_back(cur);
    if (out.empty()) out.push_back(text);
    return out;
}

bool generate(Engine & eng, Vocoder & voc, const GenRequest & req, const AudioCallback & cb, GenTimings * timings,
              std::vector<int> * codes_out) {
    GenTimings sink;
    GenTimings & tm = timings ? *timings : sink;
    const auto t_start = Clock::now();
    // the voice to keep (src/generation.cpp:209-229): given codes, else the first piece
    Anchor anchor;
    if (!req.ref_codes.empty() && req.ref_frames > 0 && !req.ref_text.empty()) {
        if ((int) req.ref_codes.size() < req.ref_frames * eng.cfg.nc) throw std::runtime_error("reference codes shorter than ref_frames");
        anchor.codes.assign(req.ref_codes.begin(), req.ref_codes.begin() + (size_t) req.ref_frames * eng.cfg.nc);
        anchor.n_frames = req.ref_frames;
        anchor.text = req.ref_text;
    } else if (!req.ref_audio.empty() && !req.ref_text.empty()) {
        throw std::runtime_error("a reference clip must be encoded to codes first (the codec encoder is not part of this library)");
    }
    // with no reference the opening piece becomes the voice, so it stays near a clip's length
    // (src/generation.cpp:255-262)
    const int anchor_chars = 200;
    const std::vector<std::string> pieces = split_text(req.text, req.split_chars, anchor.codes.empty() ? anchor_chars : 0);
    uint32_t piece = 0;
    for (const std::string & text : pieces) {
        Anchor made;
        const bool ok = generate_piece(eng, voc, req, text, anchor, (uint32_t) req.seed + piece, cb, tm, t_start, made,
                                       codes_out);
        piece++;
        tm.pieces++;
        if (ok && anchor.codes.empty() && made.n_frames > 0) anchor = std::move(made);
        if (!ok) return false;
    }
    return true;
}

std::string filler_text(double seconds) {
    static const char * const kLines[] = {
        "A calm voice reads a short passage at an even pace. ",
        "Each sentence here is plain and carries no special meaning. ",
        "The reading goes on for a while in the same steady tone. ",
        "There is nothing to remember from these words at all. ",
    };
    const size_t want = (size_t) (seconds * 17.0) + 16;
    std::string s;
    for (int i = 0; s.size() < want; i++) s += kLines[i % 4];
    return s;
}

bool write_wav(const std::string & path, const std::vector<float> & samples, int sample_rate) {
    FILE * f = std::fopen(path.c_str(), "wb");
    if (!f) return false;
    std::vector<uint8_t> bytes(44 + samples.size() * 2);
    uint8_t * p = bytes.data();
    auto put = [&](uint32_t v, int n) {
        for (int i = 0; i < n; i++) *p++ = (uint8_t) (v >> (8 * i));
    };
    auto tag = [&](const char * s) {
        std::memcpy(p, s, 4);
        p += 4;
    };
    const uint32_t data_len = (uint32_t) samples.size() * 2;
    tag("RIFF"); put(36 + data_len, 4); tag("WAVE");
    tag("fmt "); put(16, 4); put(1, 2); put(1, 2); put((uint32_t) sample_rate, 4); put((uint32_t) sample_rate * 2, 4);
    put(2, 2); put(16, 2);
    tag("data"); put(data_len, 4);
    for (float v : samples) {
        v = std::min(1.0f, std::max(-1.0f, v));
        put((uint32_t) (uint16_t) (int16_t) (v * 32767.0f), 2);
    }
    const bool ok = std::fwrite(bytes.data(), 1, bytes.size(), f) == bytes.size();
    return std::fclose(f) == 0 && ok;
}

}  // namespace bzb
