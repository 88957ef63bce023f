/*
 * bzb_ext.h -- entry points of libbreeze.so beyond the reference ABI.
 *
 * The reference generator ABI writes 16 codes per frame (src/c_api.cpp:672, 857); models
 * with more codebooks need the full-width frame, and the measurement and parity harnesses
 * need device-resident timing and intermediate values. These functions have no counterpart
 * in the reference; the breeze.h entry points remain the drop-in interface.
 */
#ifndef BZB_EXT_H
#define BZB_EXT_H

#include "breeze.h"

#ifdef __cplusplus
extern "C" {
#endif

/* number of codebooks per frame of the loaded model (breeze.num_codebooks) */
BREEZE_API int bzb_generator_num_codebooks(breeze_generator * gen);

/* sessions_step_burst with full-width frames: out_frames is [burst_steps][num_sessions][nc].
   Same return codes and -1 conventions as breeze_generator_sessions_step_burst. */
BREEZE_API int bzb_generator_sessions_step_frames(breeze_generator * gen, const int * session_ids,
                                                  int num_sessions, int burst_steps,
                                                  const unsigned int * seeds, int * out_frames,
                                                  int * out_next_cb0);

/* re-runs the last stepped batch K more frames on the device with no host copies (timing);
   returns 0, or -1 with breeze_last_error() set */
BREEZE_API int bzb_generator_step_device(breeze_generator * gen, int burst_steps);
BREEZE_API int bzb_generator_sync(breeze_generator * gen);
/* the CUDA stream (cudaStream_t) every generator kernel is launched on */
BREEZE_API void * bzb_generator_stream(breeze_generator * gen);

/* algorithmic bytes of one frame step: Q8_0 weight bytes, and KV bytes per cached position */
BREEZE_API long long bzb_generator_weight_bytes_per_step(breeze_generator * gen);
BREEZE_API long long bzb_generator_kv_bytes_per_position(breeze_generator * gen);

/* kernels in one captured frame step (graph nodes of the last captured bucket) */
BREEZE_API int bzb_generator_launches_per_step(breeze_generator * gen);
/* one eager frame step of the last batch with CUDA events around every dequant-GEMM launch and
   the persistent depth decoder: out7 = {step_ms, gemm_ms, gemm_launches, gemm_algorithmic_bytes,
   launches_counted, depth_ms, depth_algorithmic_bytes} (depth values 0 when the batch uses the
   per-operation depth path) */
BREEZE_API int bzb_generator_profile_step(breeze_generator * gen, double * out7);

/* parity probes: the session's last normed backbone hidden [hidden]; one depth decode of n
   rows (hidden [n][hidden] f32, cb0 [n]; forced [n][nc-1] replaces each argmax as the next
   input when non-null) returning codes [n][nc-1] and logits [n][nc-1][audio_vocab]; one
   dequant-GEMM of a named Q8_0 tensor (slice `sub` of a 3-D tensor, or -1) on x [rows][K] */
BREEZE_API int bzb_generator_debug_hidden(breeze_generator * gen, int session_id, float * out);
BREEZE_API int bzb_generator_debug_depth(breeze_generator * gen, int n, const float * hidden, const int * cb0,
                                         const int * forced, int * out_codes, float * out_logits);
BREEZE_API int bzb_generator_debug_gemv(breeze_generator * gen, const char * tensor, int sub, int rows,
                                        const float * x, float * y);

/* parity probe of a matrix exactly as the frame step holds it: `name` is a resident matrix --
   {bb,dd,te}.blk.N.{attn_qkv, attn_output, ffn_gate_up, ffn_down} (attn_qkv: q, k and v rows
   fused; ffn_gate_up: gate and up interleaved, run with the step's SwiGLU or GeGLU epilogue),
   bb.lm_head.weight, dd.in_proj.weight, te.proj.weight or dd.head.J (depth head J) -- on x
   [rows][K] (f32, rounded to f16 as the step's activations are). y receives [rows][M], or
   [rows][M/2] of gated outputs (f16 values widened to f32). With repeats > 0 the launch is
   captured `repeats` more times in one CUDA graph under programmatic dependent launch, and each
   result is compared bit for bit on the device with the first (flags bit 0: capture without
   programmatic dependent launch). Returns the number of 32-bit words that differed (0 for a
   deterministic kernel), or -1 with breeze_last_error(); out_where, when non-null, receives the
   first where_cap differences as (word index into y's rows, repeat index) int pairs. */
BREEZE_API long long bzb_generator_debug_gemm(breeze_generator * gen, const char * name, int rows, const float * x,
                                              float * y, int repeats, int flags, int * out_where, int where_cap);

/* Streaming PCM (no counterpart in the reference, whose vocoder sessions re-decode up to 32
   frames of history with every call, src/c_api.cpp:1004-1162). A stream carries the codec
   decoder's causal state from call to call -- the last inputs of every causal convolution and
   the transformer's keys and values over its attention window -- so each call decodes only its
   new frames, and the PCM of a stream equals that of one decode of all its frames at once. Calls
   for many streams run as one batch: every linear is one GEMM and every convolution one launch
   over all of them. A vocoder holds up to BZB_VOC_STREAMS streams (default 256; about 5 MB of
   device memory each, allocated with the first stream) of at most 8192 frames, and takes at
   most 56 new frames per stream and call.
   bzb_vocoder_stream_open starts (or restarts) a stream; bzb_vocoder_stream_close releases it
   (-1 when unknown). bzb_vocoder_streams_decode decodes n_frames new frames of each of n
   distinct streams: codes [n][n_frames][num_codebooks], out_pcm [n][n_frames * 1920] (host
   buffers); unknown ids are opened. Returns n, or -1 with breeze_last_error(). */
BREEZE_API int bzb_vocoder_stream_open(breeze_vocoder * voc, int stream_id);
BREEZE_API int bzb_vocoder_stream_close(breeze_vocoder * voc, int stream_id);
BREEZE_API int bzb_vocoder_streams_decode(breeze_vocoder * voc, int n, const int * stream_ids, const int * codes,
                                          int n_frames, float * out_pcm);

/* One serving step: breeze_generator_sessions_step_burst for one frame (full-width frames) and
   the PCM of every new frame, decoded on the stream of its session id (restarted whenever a
   session with that id is created). voc must come from breeze_vocoder_create_from_generator of
   this generator. out_frames [n][num_codebooks] (optional; -1 rows for sessions that did not
   step), out_next_cb0 [n], out_pcm [n][1920] (optional; zero rows for sessions that did not
   step). Returns the number of sessions still active, or -1 with breeze_last_error(). */
BREEZE_API int bzb_generator_sessions_step_pcm(breeze_generator * gen, breeze_vocoder * voc, const int * session_ids,
                                               int n, const unsigned int * seeds, int * out_frames, int * out_next_cb0,
                                               float * out_pcm);
/* The same steps resident on the device (timing and serving loops that keep PCM on the GPU):
   burst_steps frame steps of the listed sessions, each followed by the streaming decode of the
   new frames, with no host copies and no synchronisation. Every listed session must be active.
   The last step's PCM stays in the vocoder ([n][1920]; bzb_vocoder_last_pcm copies it out after
   synchronising). Returns 0, or -1 with breeze_last_error(). */
BREEZE_API int bzb_generator_step_pcm_device(breeze_generator * gen, breeze_vocoder * voc, const int * session_ids,
                                             int n, const unsigned int * seeds, int burst_steps);
BREEZE_API int bzb_vocoder_last_pcm(breeze_vocoder * voc, float * out, int n_samples);
/* kernels one batched decode of n_streams streams x n_frames frames launches, or -1 */
BREEZE_API int bzb_vocoder_kernels_per_decode(breeze_vocoder * voc, int n_streams, int n_frames);

/* Tests of the bounded device waits (no reference counterpart). Every spin-wait in the kernels
   gives up after a poll limit, records an error code, lets the copies and MMAs it issued land,
   frees its tensor memory and returns; the host then reports the code and clears it.
   bzb_generator_debug_grid_spin sets the poll limit of the persistent depth decoder's grid
   barriers for the launches bzb_generator_debug_depth makes (0 restores the default; frame-step
   graphs never use it): a limit of a few polls makes a barrier run out, and that call then returns
   -1 with breeze_last_error() naming the timeout while the generator stays usable.
   bzb_debug_mbar_timeout runs the tcgen05 pipelines' mbarrier wait with `polls` polls on a
   barrier that nothing arrives on, on `device`, and returns the error code it recorded (1 for a
   wait that gave up), or -1 with breeze_last_error(). */
BREEZE_API int bzb_generator_debug_grid_spin(breeze_generator * gen, long long polls);
/* Test of the cb0 sampler's two top-k paths (no reference counterpart): draws `draws` picks per
   row from logits [rows][V] (V <= 4096) with the given top-k, temperature and top-p (no
   suppression or penalty; Philox key seed + row), into out_picks [draws][rows]; force_sort != 0
   takes the full sort where top-k <= 64 would select. 0, or -1 with breeze_last_error(). */
BREEZE_API int bzb_generator_debug_sample(breeze_generator * gen, const float * logits, int V, int rows, int top_k,
                                          float temp, float top_p, unsigned int seed, int draws, int force_sort,
                                          int * out_picks);
BREEZE_API int bzb_debug_mbar_timeout(int device, long long polls);

/* average microseconds of back-to-back launches of one dequant-GEMM of a named Q8_0 tensor on
   `rows` activation rows (epilogue 0 store, 1 residual add, 2 SwiGLU, 3 GeGLU), or -1 */
BREEZE_API double bzb_generator_bench_gemv(breeze_generator * gen, const char * tensor, int sub, int rows, int iters,
                                           int epilogue);

/* timeline of one persistent depth-decoder launch for the last stepped batch (profiling):
   out = {n_phases, grid, slots, phase type[n_phases] (0 GEMM, 1 reduce, 2 attention, 3 arg-max),
   timeline[n_phases][grid][slots]} with the slots of DpParams::trace in microseconds from the
   first CTA's start (-1 where not reached). Returns the doubles written -- the size needed when
   out is NULL -- 0 when the batch does not use the persistent decoder, or -1 with
   breeze_last_error() */
BREEZE_API int bzb_generator_depth_trace(breeze_generator * gen, double * out, int capacity);

/* Allocation-free dequant-GEMM (no counterpart in the reference): y[rows][ldy] = x16[rows][ldx]
   . W^T for a weight matrix already resident in the generator -- bb.lm_head.weight,
   dd.in_proj.weight, or {bb,dd}.blk.N.{attn_output,ffn_down}.weight -- on caller-owned device
   buffers (x16: f16 bits, 4-byte aligned, even ldx >= K; y: f32, ldy >= the matrix rows).
   It performs no device or host allocation: its split-K scratch is a fixed static device
   array (10 MiB of partials, 4096 counters), so a caller that has handed every free byte of
   HBM to its own pools, or that runs inside a real-time loop where cudaMalloc/cudaFree may
   synchronise the device and stall the other streams, can still run it. Limits: 1 <= rows <= 256; larger inputs are rejected with
   -1 and breeze_last_error(). Asynchronous on `stream` (a cudaStream_t; NULL = the
   generator's stream); it returns after enqueueing. The first call on a device sets up the
   scratch address (once per device) and should come before any stream capture. Calls that
   overlap on one device (other streams, other generators) share the scratch and race.
   Returns 0, or -1 with breeze_last_error(). */
BREEZE_API int bzb_generator_gemm_noalloc(breeze_generator * gen, const char * tensor, int rows, const void * x16,
                                          int ldx, float * y, int ldy, void * stream);

/* GGUF inspection without a GPU: 0 and the config values, or -1 with breeze_last_error() */
BREEZE_API int bzb_gguf_inspect(const char * gguf_path, int * out_hidden, int * out_num_codebooks,
                                int * out_n_tensors);
/* tokenizer without a GPU: writes up to max_ids ids, returns the count or -1 */
/* breeze_generate (include/breeze.h; reference src/c_api.cpp:78-89) with encoded reference codes
 * (ref_frames x num_codebooks, frame-major; the reference's GenRequest::ref_codes,
 * src/generation.h:19-22, which breeze_request cannot carry), and with the generated frames
 * (frame-major, at most max_frames written, the total in *out_n_frames) and the stage timings
 * out_timings7 = {prefill ms, frame steps ms, vocoder ms, first audio ms, frames, flushes,
 * pieces}. Every output pointer may be null. Returns 0, or 1 with breeze_last_error(). */
BREEZE_API int bzb_generate_codes(breeze_context * ctx, const breeze_request * req, const int * ref_codes,
                                  int ref_frames, breeze_audio_cb cb, void * user, int * out_codes, int max_frames,
                                  int * out_n_frames, double * out_timings7);
/* The long-text splitter of breeze_generate (reference src/text_split.cpp:89-111): writes the
 * pieces NUL-terminated one after another into out and returns their count, or -(bytes needed)
 * when capacity is too small. */
/* breeze_generator_encode_audio (reference src/c_api.cpp:1302-1331) at the model's full width:
 * num_codebooks codes per frame, frame-major, at most max_frames frames written; returns the
 * codes produced (frames * num_codebooks) or -1. */
BREEZE_API int bzb_generator_encode_audio_full(breeze_generator * gen, const float * pcm, int n_samples, int * out_codes,
                                               int max_frames, int * out_n_frames);
/* The WAV writer of breeze_generate_wav (reference src/audio.cpp:80-107): 16-bit mono PCM at
 * sample_rate. Returns 0, or -1 with breeze_last_error(). */
/* breeze_generator_session_create_ext (reference src/c_api.cpp:326-445) for n sessions at once:
 * session i takes session_ids[i], texts[i], instructions[i], ref_texts[i], ref_codes[i] (frame-major
 * [ref_frames[i]][num_codebooks]), ref_frames[i], cfg_scales[i], seeds[i] and max_new_tokens[i],
 * and gets the same prompt, budget, slot pages and first cb0 as that call. A NULL list means NULL
 * entries (instructions: the default instruction; ref_*: no reference), cfg 1, seed 42 or the
 * length estimate. The prompts of all sessions and both guidance branches are prefilled together as
 * packed rows (one text-encoder and one backbone pass per group of up to 16384 rows and 256
 * branches). Returns 0 with out_cb0[i] and out_allocated_tokens[i] (optional) filled, or -1 with
 * breeze_last_error(); on an error the sessions of earlier groups stay created, those of the failing
 * group do not. A session id that appears twice is an error. */
BREEZE_API int bzb_generator_sessions_create_batch(breeze_generator * gen, int n, const int * session_ids,
                                                   const char * const * texts, const char * const * instructions,
                                                   const char * const * ref_texts, const int * const * ref_codes,
                                                   const int * ref_frames, const float * cfg_scales,
                                                   const unsigned int * seeds, const int * max_new_tokens,
                                                   int * out_cb0, int * out_allocated_tokens);
BREEZE_API int bzb_write_wav(const char * path, const float * samples, int n, int sample_rate);
BREEZE_API int bzb_split_text(const char * text, int budget, int first_budget, char * out, int capacity);
BREEZE_API int bzb_tokenize(const char * gguf_path, const char * text, int add_bos, int * out_ids, int max_ids);

#ifdef __cplusplus
}
#endif

#endif
