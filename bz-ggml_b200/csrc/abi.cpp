// extern "C" surface of libbreeze.so: the reference's breeze.h entry points (same names,
// arguments, buffer conventions and return codes; see include/breeze.h for the line each
// one replaces) plus the bzb_* extensions of include/bzb_ext.h. Exceptions never cross the
// boundary; they become the reference's error returns plus breeze_last_error().
#include "../../include/bzb_ext.h"
#include "engine.h"
#include "generate.h"
#include "vocoder.h"

#include <cerrno>
#include <climits>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <memory>
#include <mutex>
#include <string>
#include <functional>
#include <vector>

struct breeze_generator {
    std::unique_ptr<bzb::Engine> eng;
    int device = 0;
    std::unique_ptr<bzb::CodecEncoder> enc;  // built on first use (encode_audio, convert_voice)
    std::unique_ptr<bzb::Vocoder> voc;       // built on first use (convert_voice PCM)
    bzb::CodecEncoder & encoder() {
        if (!enc) enc = std::make_unique<bzb::CodecEncoder>(eng->gguf(), eng->cfg, device);
        return *enc;
    }
    bzb::Vocoder & vocoder() {
        if (!voc) voc = std::make_unique<bzb::Vocoder>(eng->gguf(), eng->cfg, device);
        return *voc;
    }
};

// a vocoder either owns its model file (breeze_vocoder_init) or decodes with the weights of a
// generator's model (breeze_vocoder_create_from_generator; the generator must outlive it, as in
// the reference, src/c_api.cpp:971-991)
struct breeze_vocoder {
    int device = 0;
    std::unique_ptr<bzb::GgufFile> own_file;
    std::unique_ptr<bzb::Vocoder> voc;
};

// breeze_init's context: a generator and a vocoder sharing its model (src/c_api.cpp:22-25)
struct breeze_context {
    breeze_generator * gen = nullptr;
    std::unique_ptr<bzb::Vocoder> voc;
};

namespace {
// Every call that reaches a handle's GPU runs with the handle's device current and gives the
// calling thread its previous device back: one process may serve islands on several GPUs from
// several threads, each thread with whatever device it last used.
class OnDevice {
public:
    explicit OnDevice(int device) {
        if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
        // never throws (some callers are outside a try block): a device that cannot be selected
        // makes the call's first CUDA operation fail, and that failure is reported
        if (prev_ != device) cudaSetDevice(device);
        restore_ = prev_ >= 0 && prev_ != device;
    }
    ~OnDevice() {
        if (restore_) cudaSetDevice(prev_);
    }
    OnDevice(const OnDevice &) = delete;
    OnDevice & operator=(const OnDevice &) = delete;

private:
    int prev_ = -1;
    bool restore_ = false;
};

// per-thread last error: the reference keeps one unsynchronised global (src/c_api.cpp:28);
// each calling thread reads the message of its own last failing call here
thread_local std::string g_error;

void set_error(const std::string & e) { g_error = e; }

constexpr int kLegacySession = INT_MIN;
constexpr int kConvertSession = INT_MIN + 1;  // the engine session of a voice conversion
constexpr int kAbiFrameWidth = 16;

// breeze_request -> GenRequest (src/c_api.cpp:30-48)
bzb::GenRequest to_gen_request(const breeze_request * r) {
    bzb::GenRequest g;
    g.text = r->text ? r->text : "";
    g.instruction = r->instruction ? r->instruction : "Speak clearly and naturally.";
    g.ref_text = r->ref_text ? r->ref_text : "";
    if (r->ref_audio && r->ref_audio_len > 0) g.ref_audio.assign(r->ref_audio, r->ref_audio + r->ref_audio_len);
    g.cfg_scale = r->cfg_scale > 0 ? r->cfg_scale : 1.0f;
    g.seed = r->seed;
    g.max_new_tokens = r->max_new_tokens;
    if (r->split_chars != 0) g.split_chars = r->split_chars < 0 ? 0 : r->split_chars;
    g.temperature = r->temperature;
    g.top_k = r->top_k;
    g.top_p = r->top_p;
    g.repetition_penalty = r->repetition_penalty;
    return g;
}

// a reference clip with its transcript becomes encoded reference codes (src/generation.cpp:219-228)
void encode_ref_audio(breeze_context * ctx, bzb::GenRequest & g) {
    if (!g.ref_codes.empty() || g.ref_audio.empty() || g.ref_text.empty()) return;
    std::vector<int> codes;
    g.ref_frames = ctx->gen->encoder().encode(g.ref_audio.data(), (int) g.ref_audio.size(), codes);
    g.ref_codes = std::move(codes);
    g.ref_audio.clear();
}

// breeze_generate with optional encoded reference codes, the generated frames and stage timings
int generate_impl(breeze_context * ctx, const breeze_request * req, const int * ref_codes, int ref_frames,
                  breeze_audio_cb cb, void * user, int * out_codes, int max_frames, int * out_n_frames,
                  double * out_timings) {
    if (!ctx || !req) { set_error("null context or request"); return 1; }
    try {
        OnDevice on_device_(ctx->gen->device);
        bzb::GenRequest g = to_gen_request(req);
        const int nc = ctx->gen->eng->cfg.nc;
        if (ref_codes && ref_frames > 0) g.ref_codes.assign(ref_codes, ref_codes + (size_t) ref_frames * nc), g.ref_frames = ref_frames;
        encode_ref_audio(ctx, g);
        std::vector<int> codes;
        bzb::GenTimings tm;
        bzb::generate(*ctx->gen->eng, *ctx->voc, g, [&](const float * s, int n) { return cb ? cb(s, n, user) == 0 : true; },
                      &tm, out_codes || out_n_frames ? &codes : nullptr);
        const int F = (int) codes.size() / nc;
        if (out_n_frames) *out_n_frames = F;
        if (out_codes) std::memcpy(out_codes, codes.data(), (size_t) std::min(F, max_frames) * nc * sizeof(int));
        if (out_timings) {
            const double t[7] = { tm.prefill, tm.steps, tm.vocoder, tm.first_audio, (double) tm.frames,
                                  (double) tm.flushes, (double) tm.pieces };
            std::memcpy(out_timings, t, sizeof(t));
        }
    } catch (const std::exception & e) {
        set_error(e.what());
        return 1;
    }
    return 0;
}

int burst_impl(breeze_generator * gen, const int * ids, int n, int K, const unsigned int * seeds, int * out,
               int width, int * next) {
    // the engine runs up to 64 steps per graph batch; longer bursts continue with seeds + step
    std::fill_n(out, (size_t) K * n * width, -1);
    for (int i = 0; i < n; i++) next[i] = -1;
    int done = 0;
    std::vector<int> nx(n);
    std::vector<unsigned int> sd(n);
    while (done < K) {
        const int k = std::min(64, K - done);
        if (seeds)
            for (int i = 0; i < n; i++) sd[i] = seeds[i] + (unsigned) done;
        const bzb::StepResult r = gen->eng->step(ids, n, k, seeds ? sd.data() : nullptr, true,
                                                 out + (size_t) done * n * width, width, nx.data(), true);
        // a session stepped in this chunk reports its last cb0 or -1 when it finished; one not
        // stepped had finished earlier (or never ran) and reports -1 as well
        if (r.steps_executed > 0)
            for (int i = 0; i < n; i++) next[i] = nx[i];
        done += r.steps_executed;
        if (r.steps_executed < k) break;
    }
    return done;
}
}  // namespace

extern "C" {

// ------------------------------------------------------------------------------------ one-shot
breeze_context * breeze_init(const char * gguf_path, int use_gpu) {
    if (!gguf_path) { set_error("null model path"); return nullptr; }
    if (!use_gpu) { set_error("this library runs on CUDA devices only; use_gpu=0 has no CPU backend here"); return nullptr; }
    breeze_generator * gen = breeze_generator_init(gguf_path, 0);
    if (!gen) return nullptr;
    try {
        auto ctx = std::make_unique<breeze_context>();
        ctx->gen = gen;
        ctx->voc = std::make_unique<bzb::Vocoder>(gen->eng->gguf(), gen->eng->cfg, gen->device);
        return ctx.release();
    } catch (const std::exception & e) {
        set_error(e.what());
        breeze_generator_free(gen);
        return nullptr;
    }
}

void breeze_free(breeze_context * ctx) {
    if (!ctx) return;
    OnDevice on_device_(ctx->gen ? ctx->gen->device : 0);
    ctx->voc.reset();
    breeze_generator_free(ctx->gen);
    delete ctx;
}

int breeze_sample_rate(breeze_context * ctx) {
    return (ctx && ctx->gen && ctx->gen->eng) ? ctx->gen->eng->cfg.sample_rate : 0;
}

int breeze_generate(breeze_context * ctx, const breeze_request * req, breeze_audio_cb cb, void * user) {
    return generate_impl(ctx, req, nullptr, 0, cb, user, nullptr, 0, nullptr, nullptr);
}

int breeze_generate_wav(breeze_context * ctx, const breeze_request * req, const char * out_path) {
    if (!ctx || !req || !out_path) { set_error("null argument"); return 1; }
    try {
        OnDevice on_device_(ctx->gen->device);
        std::vector<float> audio;
        bzb::GenRequest g = to_gen_request(req);
        encode_ref_audio(ctx, g);
        bzb::generate(*ctx->gen->eng, *ctx->voc, g, [&](const float * s, int n) {
            audio.insert(audio.end(), s, s + n);
            return true;
        });
        if (!bzb::write_wav(out_path, audio, ctx->gen->eng->cfg.sample_rate)) {
            set_error("failed to write wav");
            return 1;
        }
    } catch (const std::exception & e) {
        set_error(e.what());
        return 1;
    }
    return 0;
}

const char * breeze_last_error(void) { return g_error.c_str(); }

// ------------------------------------------------------------------------------------ generator
breeze_generator * breeze_generator_init(const char * gguf_path, int cuda_device) {
    if (!gguf_path) { set_error("null model path"); return nullptr; }
    breeze_generator * gen = new breeze_generator();
    gen->device = cuda_device;
    try {
        gen->eng.reset(new bzb::Engine(gguf_path, cuda_device));
        return gen;
    } catch (const std::exception & e) {
        set_error(e.what());
        delete gen;
        return nullptr;
    }
}

void breeze_generator_free(breeze_generator * gen) {
    if (!gen) return;
    OnDevice on_device_(gen->device);
    delete gen;
}

int breeze_generator_prefill(breeze_generator * gen, const char * text, const char * instruction, unsigned int seed,
                             int * out_cb0) {
    if (!gen || !text || !out_cb0) return -1;
    try {
        OnDevice on_device_(gen->device);
        int alloc = 0;
        gen->eng->session_create(kLegacySession, text, instruction, nullptr, nullptr, 0, 1.0f, seed,
                                 gen->eng->cfg.max_new_tokens > 0 ? gen->eng->cfg.max_new_tokens : 2048, out_cb0, &alloc);
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int breeze_generator_step_frame(breeze_generator * gen, int cb0, unsigned int seed, int * out_frame_16) {
    (void) cb0;  // the session's own last cb0 is the one the reference's caller passes back
    if (!gen || !out_frame_16 || !gen->eng->session_active(kLegacySession)) return -1;
    try {
        OnDevice on_device_(gen->device);
        const int sid = kLegacySession;
        int next = -1;
        // depth codes from the GGUF's depth sampler with the call's seed (src/c_api.cpp:297-299)
        gen->eng->step(&sid, 1, 1, nullptr, false, out_frame_16, kAbiFrameWidth, &next, false, true, &seed);
        return next;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int breeze_generator_session_create_ext(breeze_generator * gen, int session_id, const char * text,
                                        const char * instruction, const char * ref_text, const int * ref_codes,
                                        int ref_frames, float cfg_scale, unsigned int seed, int max_new_tokens,
                                        int * out_cb0, int * out_allocated_tokens) {
    if (!gen || !text || !out_cb0) return -1;
    try {
        OnDevice on_device_(gen->device);
        gen->eng->session_create(session_id, text, instruction, ref_text, ref_codes, ref_frames, cfg_scale, seed,
                                 max_new_tokens, out_cb0, out_allocated_tokens);
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int breeze_generator_session_create(breeze_generator * gen, int session_id, const char * text,
                                    const char * instruction, float cfg_scale, unsigned int seed, int * out_cb0) {
    return breeze_generator_session_create_ext(gen, session_id, text, instruction, nullptr, nullptr, 0, cfg_scale,
                                               seed, 0, out_cb0, nullptr);
}

int breeze_generator_session_step(breeze_generator * gen, int session_id, unsigned int seed, int * out_frame_16) {
    if (!gen || !out_frame_16) return -1;
    if (!gen->eng->session_active(session_id)) return -1;
    try {
        OnDevice on_device_(gen->device);
        int next = -1;
        // depth codes from the GGUF's depth sampler with the call's seed (src/c_api.cpp:468-479)
        gen->eng->step(&session_id, 1, 1, nullptr, false, out_frame_16, kAbiFrameWidth, &next, false, true, &seed);
        return next;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int breeze_generator_session_free(breeze_generator * gen, int session_id) {
    if (!gen) return -1;
    try {
        OnDevice on_device_(gen->device);
        return gen->eng->session_free(session_id) ? 0 : -1;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int breeze_generator_load_q4_depth(breeze_generator * gen, const char * q4_gguf_path) {
    if (!gen || !q4_gguf_path) return -1;
    try {
        OnDevice on_device_(gen->device);
        gen->eng->load_q4_depth(q4_gguf_path);
        return 0;
    } catch (const std::exception & e) {
        set_error(std::string("failed to load the Q4 depth decoder: ") + e.what());
        return -1;
    }
}

int breeze_generator_session_set_q4(breeze_generator * gen, int session_id, int use_q4) {
    if (!gen) return -1;
    OnDevice on_device_(gen->device);
    // without a loaded Q4 depth piece the flag resolves to off (src/c_api.cpp:576)
    return gen->eng->session_set_q4(session_id, use_q4 != 0) ? 0 : -1;
}

int breeze_generator_session_count(breeze_generator * gen) { return gen ? gen->eng->session_count() : 0; }

int breeze_generator_sessions_step_round(breeze_generator * gen, const int * session_ids, int num_sessions,
                                         unsigned int seed, int * out_frames_16, int * out_next_cb0) {
    if (!gen || !session_ids || num_sessions <= 0 || !out_frames_16 || !out_next_cb0) return 0;
    int completed = 0;
    for (int i = 0; i < num_sessions; i++) {
        const int nb = breeze_generator_session_step(gen, session_ids[i], seed + (unsigned) i, out_frames_16 + (size_t) i * 16);
        out_next_cb0[i] = nb;
        if (nb >= 0) completed++;
    }
    return completed;
}

int breeze_generator_sessions_step_batched(breeze_generator * gen, const int * session_ids, int num_sessions,
                                           const unsigned int * seeds, int * out_frames_16, int * out_next_cb0) {
    if (!gen || !session_ids || num_sessions <= 0 || !out_frames_16 || !out_next_cb0) return 0;
    try {
        OnDevice on_device_(gen->device);
        const bzb::StepResult r = gen->eng->step(session_ids, num_sessions, 1, seeds, false, out_frames_16,
                                                 kAbiFrameWidth, out_next_cb0, false);
        return r.steps_executed == 0 ? 0 : r.still_active;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int breeze_generator_sessions_step_burst(breeze_generator * gen, const int * session_ids, int num_sessions,
                                         int burst_steps, const unsigned int * seeds, int * out_frames_burst,
                                         int * out_next_cb0) {
    if (!gen || !session_ids || num_sessions <= 0 || burst_steps <= 0 || !out_frames_burst || !out_next_cb0) return 0;
    try {
        OnDevice on_device_(gen->device);
        return burst_impl(gen, session_ids, num_sessions, burst_steps, seeds, out_frames_burst, kAbiFrameWidth, out_next_cb0);
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int breeze_generator_convert_voice(breeze_generator * gen, const int * src_codes, int src_T, const float * ref_audio,
                                   int ref_audio_len, const int * ref_codes, int ref_frames, const char * ref_text,
                                   const char * src_text, float cfg_scale, int keep_acoustic, int feed_source,
                                   unsigned int seed, int * out_codes, float * out_pcm, int max_out_pcm) {
    if (!gen || !src_codes || src_T <= 0) return -1;
    try {
        OnDevice on_device_(gen->device);
        bzb::Engine & eng = *gen->eng;
        const int nc = eng.cfg.nc, spf = bzb::Vocoder::kSamplesPerFrame;
        // frames are num_codebooks codes apart (the reference indexes them so, src/generation.cpp:346-364);
        // the ABI copies 16 codes per frame (src/c_api.cpp:1262, 1271), which bounds num_codebooks
        if (nc > kAbiFrameWidth) throw std::runtime_error("voice conversion through the generator ABI needs num_codebooks <= 16");
        // the reference voice: given codes, else the clip encoded (src/generation.cpp:319-325)
        std::vector<int> ref;
        int ref_T = 0;
        if (ref_codes && ref_frames > 0) {
            ref.assign(ref_codes, ref_codes + (size_t) ref_frames * nc);
            ref_T = ref_frames;
        } else if (ref_audio && ref_audio_len > 0) {
            ref_T = gen->encoder().encode(ref_audio, ref_audio_len, ref);
        }
        const std::string text = (src_text && std::strlen(src_text) > 0)
                                     ? std::string(src_text)
                                     : bzb::filler_text((double) src_T * spf / eng.cfg.sample_rate);
        // prompts (src/generation.cpp:332-337): the conditional one always carries the reference
        // (its text, frames and EOS frame) and no instruction; the unconditional one drops it
        const bzb::Tokenizer & tok = eng.tokenizer();
        std::vector<std::vector<int>> segs = { tok.encode("[S0]" + std::string(ref_text ? ref_text : ""), true),
                                               tok.encode("[S0]" + text, true) };
        std::vector<std::vector<int>> segs_u = { tok.encode("[S0]" + text, true) };
        const bool use_cfg = cfg_scale != 1.0f;
        // ConvertOptions (src/generation.h:48-63): the depth codes take the top-1 of temperature 0.3
        bzb::SessionParams sp;
        sp.cfg = cfg_scale;
        sp.dtemp = 0.3f; sp.dtop_k = 1; sp.dtop_p = 1.0f;
        const int sid = kConvertSession;
        int cb0 = 0;
        const int dummy = 0;
        eng.session_create_tokens(sid, segs, use_cfg ? &segs_u : nullptr, ref.empty() ? &dummy : ref.data(), ref_T, seed,
                                  src_T, sp, false, &cb0, nullptr, false);
        std::vector<int> out((size_t) src_T * nc);
        try {
            const int keep = std::max(0, std::min(keep_acoustic, nc - 1));
            std::vector<int> force, feed;
            for (int t0 = 0; t0 < src_T; t0 += 64) {
                const int K = std::min(64, src_T - t0);
                force.assign((size_t) K * nc, -1);
                feed.assign(src_codes + (size_t) t0 * nc, src_codes + (size_t) (t0 + K) * nc);
                for (int k = 0; k < K; k++)
                    for (int c = 0; c <= keep; c++) force[(size_t) k * nc + c] = src_codes[(size_t) (t0 + k) * nc + c];
                bzb::StepForce fs;
                fs.codes = force.data();
                fs.feed = feed_source ? feed.data() : nullptr;
                int next = 0;
                const bzb::StepResult r = eng.step(&sid, 1, K, nullptr, true, out.data() + (size_t) t0 * nc, nc, &next, true,
                                                   true, nullptr, &fs);
                if (r.steps_executed != K) throw std::runtime_error("voice conversion stopped early");
            }
        } catch (...) {
            eng.session_free(sid);
            throw;
        }
        eng.session_free(sid);
        if (out_codes) std::memcpy(out_codes, out.data(), out.size() * sizeof(int));
        if (!out_pcm || max_out_pcm <= 0) return src_T;  // tokens only
        // PCM in windows of 40 frames with sliding_window + 16 frames of left context
        // (src/generation.cpp:374-387)
        bzb::Vocoder & voc = gen->vocoder();
        const int ctx = eng.cfg.voc.window + 16, step = 40;
        std::vector<float> audio, part;
        audio.reserve((size_t) src_T * spf);
        for (int start = 0; start < src_T; start += step) {
            const int count = std::min(step, src_T - start), cs = start > ctx ? start - ctx : 0;
            part.resize((size_t) (start + count - cs) * spf);
            voc.decode(out.data() + (size_t) cs * nc, start + count - cs, part.data());
            audio.insert(audio.end(), part.begin() + (size_t) (start - cs) * spf, part.begin() + (size_t) (start - cs + count) * spf);
        }
        const int written = (int) std::min<size_t>(audio.size(), (size_t) max_out_pcm);
        std::memcpy(out_pcm, audio.data(), (size_t) written * sizeof(float));
        return written;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int breeze_generator_encode_audio(breeze_generator * gen, const float * pcm, int n_samples, int * out_codes,
                                  int * out_n_frames) {
    if (!gen || !pcm || n_samples <= 0 || !out_codes || !out_n_frames) return -1;
    try {
        OnDevice on_device_(gen->device);
        // frames of min(num_codebooks, 16) codes: the ABI's frame width (the bindings size the
        // buffer at 16 codes per frame, python/bz_ggml/bindings.py:444-446)
        std::vector<int> codes;
        const int T = gen->encoder().encode(pcm, n_samples, codes);
        const int nc = gen->eng->cfg.nc, w = std::min(nc, kAbiFrameWidth);
        for (int f = 0; f < T; f++) std::memcpy(out_codes + (size_t) f * w, codes.data() + (size_t) f * nc, (size_t) w * sizeof(int));
        *out_n_frames = T;
        return T * w;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

// ------------------------------------------------------------------------------------ vocoder
breeze_vocoder * breeze_vocoder_init(const char * gguf_path, int cuda_device) {
    if (!gguf_path) {
        set_error("null model path");
        return nullptr;
    }
    try {
        auto v = std::make_unique<breeze_vocoder>();
        v->device = cuda_device;
        v->own_file = std::make_unique<bzb::GgufFile>();
        std::string err;
        if (!v->own_file->open(gguf_path, err)) throw std::runtime_error(err);
        const bzb::ModelConfig cfg = bzb::parse_config(*v->own_file);
        v->voc = std::make_unique<bzb::Vocoder>(*v->own_file, cfg, cuda_device);
        return v.release();
    } catch (const std::exception & e) {
        set_error(e.what());
        return nullptr;
    }
}

void breeze_vocoder_free(breeze_vocoder * voc) {
    if (!voc) return;
    OnDevice on_device_(voc->device);
    delete voc;
}

breeze_vocoder * breeze_vocoder_create_from_generator(breeze_generator * gen) {
    if (!gen) return nullptr;
    try {
        OnDevice on_device_(gen->device);
        auto v = std::make_unique<breeze_vocoder>();
        v->device = gen->device;
        // the generator's stream: decodes are ordered after its frame steps and may read their
        // frames on the device (bzb_generator_step_pcm_device)
        v->voc = std::make_unique<bzb::Vocoder>(gen->eng->gguf(), gen->eng->cfg, gen->device, gen->eng->stream());
        return v.release();
    } catch (const std::exception & e) {
        set_error(e.what());
        return nullptr;
    }
}

int breeze_vocoder_session_create(breeze_vocoder * voc, int session_id) {
    if (!voc || !voc->voc) return -1;
    OnDevice on_device_(voc->device);
    voc->voc->session_create(session_id);
    return 0;
}

int breeze_vocoder_session_decode(breeze_vocoder * voc, int session_id, const int * frames, int n_frames,
                                  float * out_pcm) {
    if (!voc || !voc->voc || !frames || n_frames <= 0 || !out_pcm) return 0;
    try {
        OnDevice on_device_(voc->device);
        return voc->voc->session_decode(session_id, frames, n_frames, out_pcm);
    } catch (const std::exception & e) {
        set_error(e.what());
        return 0;
    }
}

int breeze_vocoder_session_decode_batch(breeze_vocoder * voc, int batch_size, const int * session_ids,
                                        const int * flat_tokens, const int * token_offsets,
                                        const int * n_frames_per_stream, float * flat_pcm, const int * pcm_offsets,
                                        int * out_n_samples) {
    if (!voc || !voc->voc || batch_size <= 0 || !session_ids || !flat_tokens || !n_frames_per_stream || !flat_pcm) return 0;
    try {
        OnDevice on_device_(voc->device);
        return voc->voc->session_decode_batch(batch_size, session_ids, flat_tokens, token_offsets, n_frames_per_stream,
                                              flat_pcm, pcm_offsets, out_n_samples);
    } catch (const std::exception & e) {
        set_error(e.what());
        return 0;
    }
}

int breeze_vocoder_session_free(breeze_vocoder * voc, int session_id) {
    if (!voc || !voc->voc) return -1;
    OnDevice on_device_(voc->device);
    return voc->voc->session_free(session_id) ? 0 : -1;
}

int breeze_vocoder_stream_decode(breeze_vocoder * voc, const int * frames, int n_frames, float * out_pcm) {
    if (!voc || !voc->voc || !frames || n_frames <= 0 || !out_pcm) return 0;
    try {
        OnDevice on_device_(voc->device);
        return voc->voc->stream_decode(frames, n_frames, out_pcm);
    } catch (const std::exception & e) {
        set_error(e.what());
        return 0;
    }
}

int breeze_vocoder_stream_decode_batch(breeze_vocoder * voc, int batch_size, const int * flat_tokens,
                                       const int * token_offsets, const int * n_frames_per_stream, float * flat_pcm,
                                       const int * pcm_offsets, int * out_n_samples) {
    if (!voc || !voc->voc || batch_size <= 0 || !flat_tokens || !n_frames_per_stream || !flat_pcm) return 0;
    try {
        OnDevice on_device_(voc->device);
        return voc->voc->stream_decode_batch(batch_size, flat_tokens, token_offsets, n_frames_per_stream, flat_pcm,
                                             pcm_offsets, out_n_samples);
    } catch (const std::exception & e) {
        set_error(e.what());
        return 0;
    }
}

// ------------------------------------------------------------------------------------ voice files
// BRZV v1: "BRZV", u32 version, sample_rate, n_codebooks, frames, text_len, text bytes, then
// frames*n_codebooks little-endian i32 codes (layout of src/voice.cpp:16-69)
int breeze_voice_save_file(const char * path, const char * name, const char * text, const int * codes, int n_frames,
                           int n_codebooks, int sample_rate) {
    if (!path || !name || !text || !codes || n_frames <= 0 || n_codebooks <= 0) return -1;
    try {
        std::error_code ec;
        const std::filesystem::path p(path);
        if (p.has_parent_path()) std::filesystem::create_directories(p.parent_path(), ec);
        FILE * f = std::fopen(path, "wb");
        if (!f) return -1;
        const uint32_t hdr[5] = { 1u, (uint32_t) (sample_rate > 0 ? sample_rate : 24000), (uint32_t) n_codebooks,
                                  (uint32_t) n_frames, (uint32_t) std::strlen(text) };
        bool ok = std::fwrite("BRZV", 1, 4, f) == 4 && std::fwrite(hdr, 4, 5, f) == 5;
        if (ok && hdr[4]) ok = std::fwrite(text, 1, hdr[4], f) == hdr[4];
        const size_t n = (size_t) n_frames * n_codebooks;
        if (ok) ok = std::fwrite(codes, 4, n, f) == n;
        std::fclose(f);
        if (!ok) std::filesystem::remove(path, ec);
        return ok ? 0 : -1;
    } catch (...) {
        return -1;
    }
}

int breeze_voice_load_file(const char * path, char * out_name, int name_max, char * out_text, int text_max,
                           int * out_codes, int * out_n_frames, int * out_n_codebooks, int * out_sample_rate) {
    if (!path || !out_codes || !out_n_frames || !out_n_codebooks) return -1;
    try {
        FILE * f = std::fopen(path, "rb");
        if (!f) return -1;
        char magic[4];
        uint32_t hdr[5] = {};
        bool ok = std::fread(magic, 1, 4, f) == 4 && std::memcmp(magic, "BRZV", 4) == 0 &&
                  std::fread(hdr, 4, 5, f) == 5 && hdr[0] == 1u;
        // a corrupt header must not become a giant allocation
        if (ok) ok = hdr[2] > 0 && hdr[2] <= 64 && hdr[3] > 0 && hdr[3] <= 100000 && hdr[4] <= (1u << 20);
        std::string text;
        std::vector<int32_t> codes;
        if (ok) {
            text.resize(hdr[4]);
            if (hdr[4]) ok = std::fread(&text[0], 1, hdr[4], f) == hdr[4];
        }
        if (ok) {
            codes.resize((size_t) hdr[3] * hdr[2]);
            ok = std::fread(codes.data(), 4, codes.size(), f) == codes.size();
        }
        std::fclose(f);
        if (!ok) return -1;
        const std::string name = std::filesystem::path(path).stem().string();
        if (out_name && name_max > 0) {
            std::strncpy(out_name, name.c_str(), name_max - 1);
            out_name[name_max - 1] = '\0';
        }
        if (out_text && text_max > 0) {
            std::strncpy(out_text, text.c_str(), text_max - 1);
            out_text[text_max - 1] = '\0';
        }
        *out_n_frames = (int) hdr[3];
        *out_n_codebooks = (int) hdr[2];
        if (out_sample_rate) *out_sample_rate = (int) hdr[1];
        std::memcpy(out_codes, codes.data(), codes.size() * sizeof(int));
        return (int) codes.size();
    } catch (...) {
        return -1;
    }
}

// ------------------------------------------------------------------------------------ extensions
int bzb_generator_num_codebooks(breeze_generator * gen) { return gen ? gen->eng->nc() : 0; }

int bzb_generator_sessions_step_frames(breeze_generator * gen, const int * session_ids, int num_sessions,
                                       int burst_steps, const unsigned int * seeds, int * out_frames,
                                       int * out_next_cb0) {
    if (!gen || !session_ids || num_sessions <= 0 || burst_steps <= 0 || !out_frames || !out_next_cb0) return 0;
    try {
        OnDevice on_device_(gen->device);
        return burst_impl(gen, session_ids, num_sessions, burst_steps, seeds, out_frames, gen->eng->nc(), out_next_cb0);
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_generator_step_device(breeze_generator * gen, int burst_steps) {
    if (!gen || burst_steps <= 0) return -1;
    try {
        OnDevice on_device_(gen->device);
        gen->eng->step_device_only(burst_steps);
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_generator_sync(breeze_generator * gen) {
    if (!gen) return -1;
    try {
        OnDevice on_device_(gen->device);
        gen->eng->sync();
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

void * bzb_generator_stream(breeze_generator * gen) { return gen ? (void *) gen->eng->stream() : nullptr; }

long long bzb_generator_weight_bytes_per_step(breeze_generator * gen) {
    return gen ? (long long) gen->eng->weight_bytes_per_step() : -1;
}

long long bzb_generator_kv_bytes_per_position(breeze_generator * gen) {
    return gen ? (long long) gen->eng->kv_bytes_per_position() : -1;
}

int bzb_generator_launches_per_step(breeze_generator * gen) { return gen ? gen->eng->launches_per_step() : -1; }

int bzb_generator_profile_step(breeze_generator * gen, double * out7) {
    if (!gen || !out7) return -1;
    try {
        OnDevice on_device_(gen->device);
        gen->eng->profile_step(out7);
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_generator_debug_hidden(breeze_generator * gen, int session_id, float * out) {
    if (!gen || !out) return -1;
    try {
        OnDevice on_device_(gen->device);
        gen->eng->debug_hidden(session_id, out);
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_generator_debug_depth(breeze_generator * gen, int n, const float * hidden, const int * cb0, const int * forced,
                              int * out_codes, float * out_logits) {
    if (!gen || !hidden || !cb0 || !out_codes || !out_logits) return -1;
    try {
        OnDevice on_device_(gen->device);
        gen->eng->debug_depth(n, hidden, cb0, forced, out_codes, out_logits);
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_generator_debug_gemv(breeze_generator * gen, const char * tensor, int sub, int rows, const float * x, float * y) {
    if (!gen || !tensor || rows <= 0 || !x || !y) return -1;
    try {
        OnDevice on_device_(gen->device);
        gen->eng->debug_gemv(tensor, sub, rows, x, y);
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

// ------------------------------------------------------------------------------------ streams
int bzb_vocoder_stream_open(breeze_vocoder * voc, int stream_id) {
    if (!voc) return -1;
    try {
        OnDevice on_device_(voc->device);
        voc->voc->stream_open(stream_id);
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_vocoder_stream_close(breeze_vocoder * voc, int stream_id) {
    if (!voc) return -1;
    OnDevice on_device_(voc->device);
    return voc->voc->stream_close(stream_id) ? 0 : -1;
}

int bzb_vocoder_streams_decode(breeze_vocoder * voc, int n, const int * stream_ids, const int * codes, int n_frames,
                               float * out_pcm) {
    if (!voc || n <= 0 || !stream_ids || !codes || n_frames <= 0 || !out_pcm) {
        set_error("streams_decode: bad arguments");
        return -1;
    }
    try {
        OnDevice on_device_(voc->device);
        voc->voc->streams_decode(n, stream_ids, nullptr, codes, n_frames, out_pcm);
        return n;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_vocoder_kernels_per_decode(breeze_vocoder * voc, int n_streams, int n_frames) {
    if (!voc || n_streams <= 0 || n_frames <= 0) return -1;
    try {
        OnDevice on_device_(voc->device);
        return voc->voc->kernels_per_decode(n_streams, n_frames);
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_vocoder_last_pcm(breeze_vocoder * voc, float * out, int n_samples) {
    if (!voc || !out || n_samples < 0) return -1;
    try {
        OnDevice on_device_(voc->device);
        voc->voc->check_device_error();
        if (cudaMemcpy(out, voc->voc->last_pcm(), (size_t) n_samples * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess)
            throw std::runtime_error("last_pcm: copy failed");
        return n_samples;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

static bool same_device_stream(breeze_generator * gen, breeze_vocoder * voc) {
    if (voc->voc->stream() != gen->eng->stream()) {
        set_error("the vocoder must come from breeze_vocoder_create_from_generator of this generator");
        return false;
    }
    return true;
}

int bzb_generator_sessions_step_pcm(breeze_generator * gen, breeze_vocoder * voc, const int * session_ids, int n,
                                    const unsigned int * seeds, int * out_frames, int * out_next_cb0, float * out_pcm) {
    if (!gen || !voc || !session_ids || n <= 0 || !out_next_cb0) {
        set_error("sessions_step_pcm: bad arguments");
        return -1;
    }
    try {
        OnDevice on_device_(gen->device);
        if (!same_device_stream(gen, voc)) return -1;
        bzb::Engine & eng = *gen->eng;
        const int nc = eng.nc();
        constexpr int spf = bzb::Vocoder::kSamplesPerFrame;
        // every session the host knows as live decodes its new frame on its stream (keyed by
        // session id, restarted when the id's session was created again), enqueued right after
        // the frame step on the device frames: no host round trip between the two. A session
        // that finished on the device in the previous step has no frame now; it is decoded once
        // more from its -1 codes (its stream, which no later frame continues, moves on by that
        // frame) and its PCM is returned as zeros, like that of every row without a frame.
        std::vector<int> ids, rows;
        std::vector<unsigned long long> epochs;
        for (int i = 0; i < n; i++)
            if (eng.session_active(session_ids[i])) {
                ids.push_back(session_ids[i]);
                rows.push_back(i);
                epochs.push_back(eng.session_epoch(session_ids[i]));
            }
        const int m = (int) ids.size();
        const bool identity = m == n;
        const std::function<void(int)> decode = [&](int k) {
            if (m > 0)
                voc->voc->streams_decode_rows_async(m, ids.data(), epochs.data(), eng.device_frames(k), nc,
                                                    identity ? nullptr : rows.data());
        };
        std::vector<int> frames((size_t) n * nc);
        const bzb::StepResult r = eng.step(session_ids, n, 1, seeds, true, frames.data(), nc, out_next_cb0, true,
                                           false, nullptr, nullptr, &decode);
        voc->voc->check_device_error();
        if (out_frames) std::memcpy(out_frames, frames.data(), frames.size() * sizeof(int));
        if (out_pcm) {
            std::fill_n(out_pcm, (size_t) n * spf, 0.0f);
            const float * ph = voc->voc->pinned_pcm();
            for (int j = 0; j < m; j++)
                if (frames[(size_t) rows[j] * nc] >= 0) std::memcpy(out_pcm + (size_t) rows[j] * spf, ph + (size_t) j * spf, spf * sizeof(float));
        }
        return r.steps_executed == 0 ? 0 : r.still_active;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_generator_step_pcm_device(breeze_generator * gen, breeze_vocoder * voc, const int * session_ids, int n,
                                  const unsigned int * seeds, int burst_steps) {
    if (!gen || !voc || !session_ids || n <= 0 || burst_steps <= 0) {
        set_error("step_pcm_device: bad arguments");
        return -1;
    }
    try {
        OnDevice on_device_(gen->device);
        if (!same_device_stream(gen, voc)) return -1;
        bzb::Engine & eng = *gen->eng;
        std::vector<unsigned long long> epochs(n);
        for (int i = 0; i < n; i++) epochs[i] = eng.session_epoch(session_ids[i]);
        eng.step_launch_device(session_ids, n, seeds, burst_steps, [&](int k) {
            voc->voc->streams_decode_device(n, session_ids, epochs.data(), eng.device_frames(k), eng.nc(), 1, nullptr);
        });
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_generator_debug_sample(breeze_generator * gen, const float * logits, int V, int rows, int top_k, float temp,
                               float top_p, unsigned int seed, int draws, int force_sort, int * out_picks) {
    if (!gen || !logits || !out_picks) {
        set_error("debug_sample: null argument");
        return -1;
    }
    try {
        OnDevice on_device_(gen->device);
        gen->eng->debug_sample(logits, V, rows, top_k, temp, top_p, seed, draws, force_sort, out_picks);
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_generator_debug_grid_spin(breeze_generator * gen, long long polls) {
    if (!gen) return -1;
    gen->eng->set_debug_grid_spin(polls);
    return 0;
}

int bzb_debug_mbar_timeout(int device, long long polls) {
    if (polls <= 0) {
        set_error("mbar_timeout: the poll limit must be positive");
        return -1;
    }
    try {
        if (cudaSetDevice(device) != cudaSuccess) throw std::runtime_error("no such CUDA device");
        return bzb::probe_mbar_timeout(polls);
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

long long bzb_generator_debug_gemm(breeze_generator * gen, const char * name, int rows, const float * x, float * y,
                                   int repeats, int flags, int * out_where, int where_cap) {
    if (!gen || !name || rows <= 0 || !x || !y || repeats < 0 || where_cap < 0) {
        set_error("debug_gemm: bad arguments");
        return -1;
    }
    try {
        return gen->eng->debug_gemm(name, rows, x, y, repeats, flags, out_where, where_cap);
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_generator_gemm_noalloc(breeze_generator * gen, const char * tensor, int rows, const void * x16, int ldx,
                               float * y, int ldy, void * stream) {
    if (!gen || !tensor) {
        set_error("gemm_noalloc: null generator or tensor name");
        return -1;
    }
    try {
        OnDevice on_device_(gen->device);
        gen->eng->gemm_noalloc(tensor, rows, static_cast<const half *>(x16), ldx, y, ldy,
                               static_cast<cudaStream_t>(stream));
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_generator_depth_trace(breeze_generator * gen, double * out, int capacity) {
    if (!gen) return -1;
    try {
        OnDevice on_device_(gen->device);
        return gen->eng->depth_trace(out, capacity);
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

double bzb_generator_bench_gemv(breeze_generator * gen, const char * tensor, int sub, int rows, int iters, int epilogue) {
    if (!gen || !tensor || rows <= 0 || iters <= 0) return -1.0;
    try {
        return gen->eng->bench_gemv(tensor, sub, rows, iters, epilogue);
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1.0;
    }
}

int bzb_gguf_inspect(const char * gguf_path, int * out_hidden, int * out_num_codebooks, int * out_n_tensors) {
    if (!gguf_path) return -1;
    try {
        bzb::GgufFile g;
        std::string err;
        if (!g.open(gguf_path, err)) { set_error(err); return -1; }
        const bzb::ModelConfig c = bzb::parse_config(g);
        if (out_hidden) *out_hidden = c.hidden;
        if (out_num_codebooks) *out_num_codebooks = c.nc;
        if (out_n_tensors) *out_n_tensors = (int) g.tensors.size();
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_tokenize(const char * gguf_path, const char * text, int add_bos, int * out_ids, int max_ids) {
    if (!gguf_path || !text || !out_ids || max_ids < 0) return -1;
    try {
        bzb::GgufFile g;
        std::string err;
        if (!g.open(gguf_path, err)) { set_error(err); return -1; }
        bzb::Tokenizer t;
        if (!t.load(g)) { set_error("GGUF has no tokenizer.ggml.tokens"); return -1; }
        const std::vector<int> ids = t.encode(text, add_bos != 0);
        const int n = (int) std::min<size_t>(ids.size(), (size_t) max_ids);
        std::memcpy(out_ids, ids.data(), (size_t) n * sizeof(int));
        return (int) ids.size();
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_generate_codes(breeze_context * ctx, const breeze_request * req, const int * ref_codes, int ref_frames,
                       breeze_audio_cb cb, void * user, int * out_codes, int max_frames, int * out_n_frames,
                       double * out_timings7) {
    if (out_codes && max_frames < 0) { set_error("negative max_frames"); return 1; }
    return generate_impl(ctx, req, ref_codes, ref_frames, cb, user, out_codes, max_frames, out_n_frames, out_timings7);
}

int bzb_generator_sessions_create_batch(breeze_generator * gen, int n, const int * session_ids,
                                        const char * const * texts, const char * const * instructions,
                                        const char * const * ref_texts, const int * const * ref_codes,
                                        const int * ref_frames, const float * cfg_scales, const unsigned int * seeds,
                                        const int * max_new_tokens, int * out_cb0, int * out_allocated_tokens) {
    if (!gen || n < 0 || (n > 0 && (!session_ids || !texts || !out_cb0))) return -1;
    try {
        OnDevice on_device_(gen->device);
        std::vector<bzb::CreateSpec> specs(n);
        for (int i = 0; i < n; i++) {
            if (!texts[i]) throw std::runtime_error("null text");
            bzb::CreateSpec & c = specs[i];
            c.sid = session_ids[i];
            c.text = texts[i];
            c.instruction = instructions ? instructions[i] : nullptr;
            c.ref_text = ref_texts ? ref_texts[i] : nullptr;
            c.ref_codes = ref_codes ? ref_codes[i] : nullptr;
            c.ref_frames = ref_frames ? ref_frames[i] : 0;
            c.cfg_scale = cfg_scales ? cfg_scales[i] : 1.0f;
            c.seed = seeds ? seeds[i] : 42u;
            c.max_new_tokens = max_new_tokens ? max_new_tokens[i] : 0;
        }
        gen->eng->sessions_create_batch(specs, out_cb0, out_allocated_tokens);
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_generator_encode_audio_full(breeze_generator * gen, const float * pcm, int n_samples, int * out_codes,
                                    int max_frames, int * out_n_frames) {
    if (!gen || !pcm || n_samples <= 0 || !out_codes || max_frames < 0 || !out_n_frames) return -1;
    try {
        OnDevice on_device_(gen->device);
        std::vector<int> codes;
        const int T = gen->encoder().encode(pcm, n_samples, codes);
        const int nc = gen->eng->cfg.nc;
        std::memcpy(out_codes, codes.data(), (size_t) std::min(T, max_frames) * nc * sizeof(int));
        *out_n_frames = T;
        return T * nc;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_write_wav(const char * path, const float * samples, int n, int sample_rate) {
    if (!path || n < 0 || (n > 0 && !samples)) { set_error("bad arguments"); return -1; }
    try {
        if (!bzb::write_wav(path, std::vector<float>(samples, samples + n), sample_rate)) {
            set_error("failed to write wav");
            return -1;
        }
        return 0;
    } catch (const std::exception & e) {
        set_error(e.what());
        return -1;
    }
}

int bzb_split_text(const char * text, int budget, int first_budget, char * out, int capacity) {
    if (!text || (capacity > 0 && !out)) return -1;
    try {
        const std::vector<std::string> parts = bzb::split_text(text, budget, first_budget);
        size_t need = 0;
        for (const std::string & p : parts) need += p.size() + 1;
        if (out && (size_t) capacity >= need) {
            char * w = out;
            for (const std::string & p : parts) {
                std::memcpy(w, p.data(), p.size());
                w += p.size();
                *w++ = '\0';
            }
        }
        return (size_t) capacity >= need ? (int) parts.size() : -(int) need;
    } catch (const std::exception & e) {
        set_error(e.what());
        return 0;
    }
}

}  // extern "C"
