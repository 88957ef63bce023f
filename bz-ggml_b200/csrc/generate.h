// Single-request streaming generation (breeze_generate / breeze_generate_wav): the reference's
// generate / GenSession / generate_chunk (src/generation.cpp:83-273) over the GPU engine and the
// GPU vocoder, and its text splitter (src/text_split.cpp:1-118) and WAV writer (src/audio.cpp:80-107).
#pragma once

#include "engine.h"
#include "vocoder.h"

#include <functional>
#include <string>
#include <vector>

namespace bzb {

// src/generation.h GenRequest (defaults kept)
struct GenRequest {
    std::string text;
    std::string instruction = "Speak clearly and naturally.";
    std::string ref_text;
    std::vector<float> ref_audio;       // needs the codec encoder, which this library does not provide
    std::vector<int> ref_codes;         // frame-major [ref_frames][nc]
    int ref_frames = 0;
    float cfg_scale = 1.0f;
    int seed = 42;
    float temperature = 0.0f;           // zero keeps the GGUF's value
    int top_k = 0;
    float top_p = 0.0f;
    float repetition_penalty = 0.0f;
    int max_new_tokens = 0;             // 0: the GGUF's max_new_tokens
    int chunk_first = 4;                // frames per streamed chunk, ramping up to chunk_max
    int chunk_max = 25;
    int split_chars = 600;              // 0 keeps long text in one pass
};

// wall-clock milliseconds of the stages (src/generation.h GenTimings, the fields this path fills)
struct GenTimings {
    double prefill = 0, steps = 0, vocoder = 0, first_audio = 0;
    int frames = 0, flushes = 0, pieces = 0;
};

using AudioCallback = std::function<bool(const float * samples, int n)>;

// src/text_split.cpp:89-111: pieces of about `budget` weighted characters (CJK counts 3) split at
// sentence ends, then clause boundaries; the first piece sized by first_budget when > 0
std::vector<std::string> split_text(const std::string & text, int budget, int first_budget = 0);

// generates every piece of req.text, streaming PCM through cb (false stops); returns false when
// the callback stopped it. `codes_out` (optional) receives every generated frame [F][nc].
bool generate(Engine & eng, Vocoder & voc, const GenRequest & req, const AudioCallback & cb,
              GenTimings * timings = nullptr, std::vector<int> * codes_out = nullptr);

// a transcript stand-in for voice conversion without one: neutral sentences repeated to about
// 17 characters per second of source audio plus 16 (the length rule of src/generation.cpp:287-299;
// the reference states the wording does not matter, and these sentences are this library's own)
std::string filler_text(double seconds);

// 16-bit mono PCM WAV (src/audio.cpp:80-107: clamp, scale by 32767, truncate)
bool write_wav(const std::string & path, const std::vector<float> & samples, int sample_rate);

}  // namespace bzb
