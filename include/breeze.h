/*
 * breeze.h -- C ABI of libbreeze.so, the B200-native Breeze-TTS-2 generation library.
 *
 * Every entry point keeps the name, signature, buffer conventions and return codes of the
 * reference interface it replaces (sharjeel103/bz-ggml include/breeze/breeze.h and
 * src/c_api.cpp), so python/bz_ggml/bindings.py binds this library unchanged. The
 * reference line each declaration replaces is cited beside it. Plain pointers and sizes
 * only; handles are opaque and owned by the library; output buffers are caller-owned and
 * sized by the reference's conventions (16 codes per frame per session, n_frames*1920
 * samples per vocoder stream).
 */
#ifndef BREEZE_H
#define BREEZE_H

#include <stddef.h>

#if defined(_WIN32)
#define BREEZE_API
#else
#define BREEZE_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct breeze_context breeze_context;
typedef int (*breeze_audio_cb)(const float * samples, int n_samples, void * user);

/* request of the one-shot API (reference include/breeze/breeze.h:25-40) */
typedef struct {
    const char * text;
    const char * instruction;
    const char * ref_text;
    const float * ref_audio;
    int ref_audio_len;
    float cfg_scale;
    int seed;
    int max_new_tokens;
    int split_chars;
    float temperature;
    int top_k;
    float top_p;
    float repetition_penalty;
} breeze_request;

/* one-shot API (reference breeze.h:42-54, src/c_api.cpp:23-112) */
BREEZE_API breeze_context * breeze_init(const char * gguf_path, int use_gpu);          /* c_api.cpp:33-64 */
BREEZE_API void breeze_free(breeze_context * ctx);                                       /* c_api.cpp:66-72 */
BREEZE_API int breeze_sample_rate(breeze_context * ctx);                                 /* c_api.cpp:74-76 */
BREEZE_API int breeze_generate(breeze_context * ctx, const breeze_request * req,
                               breeze_audio_cb cb, void * user);                        /* c_api.cpp:78-89 */
BREEZE_API int breeze_generate_wav(breeze_context * ctx, const breeze_request * req,
                                   const char * out_path);                               /* c_api.cpp:91-108 */
BREEZE_API const char * breeze_last_error(void);                                         /* c_api.cpp:110-112 */

typedef struct breeze_generator breeze_generator;
typedef struct breeze_vocoder breeze_vocoder;

/* generator (reference breeze.h:60-73, c_api.cpp:211-322) */
BREEZE_API breeze_generator * breeze_generator_init(const char * gguf_path, int cuda_device);   /* c_api.cpp:211-232 */
BREEZE_API void breeze_generator_free(breeze_generator * gen);                                  /* c_api.cpp:234-250 */
BREEZE_API int breeze_generator_prefill(breeze_generator * gen, const char * text,
                                        const char * instruction, unsigned int seed,
                                        int * out_cb0);                                          /* c_api.cpp:253-290 */
BREEZE_API int breeze_generator_step_frame(breeze_generator * gen, int cb0,
                                           unsigned int seed, int * out_frame_16);              /* c_api.cpp:292-322 */

/* vocoder (reference breeze.h:74-103, c_api.cpp:952-1229) */
BREEZE_API breeze_vocoder * breeze_vocoder_init(const char * gguf_path, int cuda_device);       /* c_api.cpp:952-969 */
BREEZE_API void breeze_vocoder_free(breeze_vocoder * voc);                                      /* c_api.cpp:982-991 */
BREEZE_API breeze_vocoder * breeze_vocoder_create_from_generator(breeze_generator * gen);      /* c_api.cpp:971-980 */
BREEZE_API int breeze_vocoder_session_create(breeze_vocoder * voc, int session_id);            /* c_api.cpp:993-1002 */
BREEZE_API int breeze_vocoder_session_decode(breeze_vocoder * voc, int session_id,
                                             const int * frames, int n_frames,
                                             float * out_pcm);                                   /* c_api.cpp:1004-1064 */
BREEZE_API int breeze_vocoder_session_decode_batch(breeze_vocoder * voc, int batch_size,
                                                   const int * session_ids,
                                                   const int * flat_tokens, const int * token_offsets,
                                                   const int * n_frames_per_stream,
                                                   float * flat_pcm, const int * pcm_offsets,
                                                   int * out_n_samples);                         /* c_api.cpp:1066-1162 */
BREEZE_API int breeze_vocoder_session_free(breeze_vocoder * voc, int session_id);              /* c_api.cpp:1164-1173 */
BREEZE_API int breeze_vocoder_stream_decode(breeze_vocoder * voc, const int * frames,
                                            int n_frames, float * out_pcm);                     /* c_api.cpp:1175-1194 */
BREEZE_API int breeze_vocoder_stream_decode_batch(breeze_vocoder * voc, int batch_size,
                                                  const int * flat_tokens, const int * token_offsets,
                                                  const int * n_frames_per_stream,
                                                  float * flat_pcm, const int * pcm_offsets,
                                                  int * out_n_samples);                          /* c_api.cpp:1196-1229 */

/* multi-session continuous batching (reference breeze.h:105-155, c_api.cpp:325-949) */
BREEZE_API int breeze_generator_session_create(breeze_generator * gen, int session_id,
                                               const char * text, const char * instruction,
                                               float cfg_scale, unsigned int seed, int * out_cb0);    /* c_api.cpp:453-457 */
BREEZE_API int breeze_generator_session_create_ext(breeze_generator * gen, int session_id,
                                                   const char * text, const char * instruction,
                                                   const char * ref_text, const int * ref_codes, int ref_frames,
                                                   float cfg_scale, unsigned int seed, int max_new_tokens,
                                                   int * out_cb0, int * out_allocated_tokens);        /* c_api.cpp:325-451 */
BREEZE_API int breeze_generator_session_step(breeze_generator * gen, int session_id,
                                             unsigned int seed, int * out_frame_16);                  /* c_api.cpp:459-519 */
BREEZE_API int breeze_generator_session_free(breeze_generator * gen, int session_id);               /* c_api.cpp:521-530 */
BREEZE_API int breeze_generator_load_q4_depth(breeze_generator * gen, const char * q4_gguf_path);    /* c_api.cpp:532-570 */
BREEZE_API int breeze_generator_session_set_q4(breeze_generator * gen, int session_id, int use_q4);  /* c_api.cpp:572-578 */
BREEZE_API int breeze_generator_session_count(breeze_generator * gen);                              /* c_api.cpp:580-582 */
BREEZE_API int breeze_generator_sessions_step_round(breeze_generator * gen,
                                                    const int * session_ids, int num_sessions,
                                                    unsigned int seed,
                                                    int * out_frames_16, int * out_next_cb0);        /* c_api.cpp:584-599 */
BREEZE_API int breeze_generator_sessions_step_batched(breeze_generator * gen,
                                                      const int * session_ids, int num_sessions,
                                                      const unsigned int * seeds,
                                                      int * out_frames_16, int * out_next_cb0);      /* c_api.cpp:601-762 */
BREEZE_API int breeze_generator_sessions_step_burst(breeze_generator * gen,
                                                    const int * session_ids, int num_sessions,
                                                    int burst_steps,
                                                    const unsigned int * seeds,
                                                    int * out_frames_burst, int * out_next_cb0);     /* c_api.cpp:764-949 */
BREEZE_API int breeze_generator_convert_voice(breeze_generator * gen,
                                              const int * src_codes, int src_T,
                                              const float * ref_audio, int ref_audio_len,
                                              const int * ref_codes, int ref_frames,
                                              const char * ref_text, const char * src_text,
                                              float cfg_scale, int keep_acoustic, int feed_source,
                                              unsigned int seed, int * out_codes,
                                              float * out_pcm, int max_out_pcm);                      /* c_api.cpp:1231-1306 */
BREEZE_API int breeze_generator_encode_audio(breeze_generator * gen, const float * pcm, int n_samples,
                                             int * out_codes, int * out_n_frames);                    /* c_api.cpp:1308-1336 */

/* voice package files (reference breeze.h:177-184, c_api.cpp:1338-1375, src/voice.cpp:10-69) */
BREEZE_API int breeze_voice_save_file(const char * path, const char * name, const char * text,
                                      const int * codes, int n_frames, int n_codebooks, int sample_rate);
BREEZE_API int breeze_voice_load_file(const char * path, char * out_name, int name_max,
                                      char * out_text, int text_max, int * out_codes,
                                      int * out_n_frames, int * out_n_codebooks, int * out_sample_rate);

#ifdef __cplusplus
}
#endif

#endif
