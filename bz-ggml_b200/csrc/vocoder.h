// The codec decoder ("vocoder"): codebook frames -> 24 kHz PCM on the GPU, with the reference's
// session semantics (src/c_api.cpp:952-1229) and decode graph (src/codec_decoder.cpp:65-98).
#pragma once

#include "host.h"
#include "kernels.cuh"

#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace bzb {

class Vocoder {
public:
    // loads the `codec.*` tensors of an open GGUF onto `device`; with `stream` every kernel runs on
    // that stream (a generator's, so that decodes are ordered after its frame steps), otherwise on
    // a stream of its own
    Vocoder(const GgufFile & gg, const ModelConfig & cfg, int device, cudaStream_t stream = nullptr);
    ~Vocoder();

    static constexpr int kSamplesPerFrame = 1920;  // a constant of the reference C API
    static constexpr int kMaxHistory = 32;          // frames kept per session for the causal lookback
    static constexpr int kMaxStreamFrames = 8192;   // positions a stream can reach (its RoPE table)

    // codes frame-major [T][nc] (host) -> PCM [T * 1920] (host), clamped to [-1, 1]
    void decode(const int * codes, int T, float * pcm);

    // One segment of a batched decode: the stream slot whose carried state continues, the copy of
    // its state to read (-1: a new stream, zero state) and its first frame's position.
    struct Segment { int slot = 0, par = -1, pos = 0; };
    // S segments of T frames each decoded as one batch on the device (every linear one GEMM over
    // all S T frames, every convolution one launch), asynchronously on the vocoder's stream:
    // codes_dev rows [S T][ld_codes] ints, segment-major; pcm_dev [S][T 1920]. segs null: each
    // segment is a whole decode (zero left context, positions 0..T-1); otherwise segs[b] continues
    // that stream, whose state for the next call is then written to copy voc-state-next(par).
    void decode_segments(const int * codes_dev, int ld_codes, int S, int T, const Segment * segs, float * pcm_dev);

    // Streams (no counterpart in the reference): per-stream carried state -- every causal
    // convolution's last inputs and the transformer's keys and values of the last `window`
    // positions -- so that each call decodes only its new frames and the PCM equals that of one
    // decode of the stream's whole history. Opening an id resets its stream.
    void stream_open(int id);
    bool stream_close(int id);
    int stream_count() const { return (int) streams_.size(); }
    // T new frames for each of n distinct streams: codes [n][T][nc] (host) -> pcm [n][T 1920]
    // (host); unknown ids are opened; epochs (optional) as for streams_decode_device
    void streams_decode(int n, const int * ids, const unsigned long long * epochs, const int * codes, int T, float * pcm);
    // the same on device buffers without a host synchronisation: stream i's frames are rows
    // i T .. i T + T - 1 of codes_dev (row stride ld_codes ints); pcm_dev null: the vocoder's own
    // buffer (last_pcm()); when epochs is given, a stream whose stored epoch differs from
    // epochs[i] starts over (its session was created again)
    void streams_decode_device(int n, const int * ids, const unsigned long long * epochs, const int * codes_dev,
                              int ld_codes, int T, float * pcm_dev);
    const float * last_pcm() const { return pcm_; }
    // the serving step's decode: one new frame for each of m streams, stream j's frame being row
    // rows[j] of the device frames (row stride ld ints; rows null: row j), enqueued without a host
    // synchronisation; the PCM goes on into the vocoder's pinned host buffer ([m][1920],
    // pinned_pcm()) asynchronously and is valid once the stream has been synchronised
    void streams_decode_rows_async(int m, const int * ids, const unsigned long long * epochs, const int * frames_dev,
                                   int ld, const int * rows);
    const float * pinned_pcm() const { return pcm_host_; }
    // kernels one batched decode of S segments of T frames launches (counted from a captured,
    // never launched graph of a whole-decode call; a streaming call launches the same ones)
    int kernels_per_decode(int S, int T);
    // reads the device error word after the calls so far (a bounded wait timed out when it is
    // nonzero: it is cleared and the failure thrown)
    void check_device_error();
    cudaStream_t stream() const { return stream_; }

    // reference session API (breeze_vocoder_session_*); every call serialised on one mutex
    void session_create(int sid);
    int session_decode(int sid, const int * frames, int n_frames, float * out_pcm);
    int session_decode_batch(int batch, const int * sids, const int * flat_tokens, const int * token_offsets,
                             const int * n_frames, float * flat_pcm, const int * pcm_offsets, int * out_n_samples);
    bool session_free(int sid);
    int stream_decode(const int * frames, int n_frames, float * out_pcm);
    int stream_decode_batch(int batch, const int * flat_tokens, const int * token_offsets, const int * n_frames,
                            float * flat_pcm, const int * pcm_offsets, int * out_n_samples);

    int nc() const { return cfg_.nc; }
    int device() const { return device_; }

private:
    struct StreamInfo {
        int slot = 0, par = -1, pos = 0;
        unsigned long long epoch = 0;
    };
    void ensure_streams();
    void ensure_segments(int S);
    // the segments of n stream ids for T new frames (opening unknown ids; with epochs, restarting
    // streams whose epoch changed); advance() moves them past the decoded frames
    std::vector<Segment> stream_segments(int n, const int * ids, const unsigned long long * epochs, int T);
    void advance(int n, const int * ids, int T);
    struct Conv {
        // [phases][Cout][taps][Cin] (tap-major): a conv has one phase of K taps; a stride-s
        // transposed conv has s phases of ceil(K / s) taps (depthwise: [K][C])
        float * w = nullptr;
        float * b = nullptr;
        int cin = 0, cout = 0, K = 0;
        int taps = 0, phases = 1, stride = 0;
        // the tcgen05 convolution's weights: f16 tiles [otiles][kchunks][taps] of nt output
        // columns x 64 input channels, each the 128-byte-swizzled K-major image one bulk copy
        // brings into shared memory. Column g is output channel g / phases of phase g % phases:
        // every phase of a transposed conv reads the same input window, so the phases are more
        // output columns of one GEMM (rows past cout x phases and channels past cin are zero)
        half * w16 = nullptr;
        int nt = 0, otiles = 0, kchunks = 0;
    };
    struct Layer {
        // qkv: the q, k and v rows stacked (one GEMM); gate_up: gate and up rows interleaved in
        // 16-row groups for the GEMM's SwiGLU epilogue (tcgen05 layout only)
        QMat qkv, o, gate_up, down;
        float * attn_norm = nullptr, * ffn_norm = nullptr, * attn_scale = nullptr, * ffn_scale = nullptr;
    };
    struct Up {  // ConvNeXt upsampling stage
        Conv up, dw;
        float * norm_w = nullptr, * norm_b = nullptr, * pw1_b = nullptr, * pw2_b = nullptr, * gamma = nullptr;
        QMat pw1, pw2;
        int ratio = 0;
    };
    struct Res {
        float * a1 = nullptr, * b1 = nullptr, * a2 = nullptr, * b2 = nullptr;  // exp(log alpha), exp(log beta)
        Conv c1, c2;
    };
    struct Blk {
        float * alpha = nullptr, * beta = nullptr;
        Conv up;
        Res res[3];
        int rate = 0;
    };

    const GgufTensor & need(const std::string & name) const;
    float * load_f32(const std::string & name, int64_t expect, bool exp_of = false, bool recip = false);
    QMat load_q8_fused(const std::vector<std::string> & names, bool interleave_pairs);
    QMat load_q8(const std::string & name);  // Q8_0 (mma.sync layout) or Q4_K (tcgen05 layout)
    void linear(const QMat & w, const half * x16, int ldx, int rows, const GemvOut & out, cudaStream_t s);
    // stride 0: a causal conv; stride s > 0: a transposed conv, split into s phase convs
    Conv load_conv(const std::string & name, int K, int cin, int cout, int stride);
    // the f16 tiles of a conv from its tap-major f32 weights [phases][cout][taps][cin]
    void tile_conv_f16(Conv & c, const std::vector<float> & tapmajor);
    void ensure(int T);
    template <class T> T * dalloc(size_t n);

    const GgufFile & gg_;
    ModelConfig cfg_;
    VocConfig vc_;
    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    bool own_stream_ = true;
    std::vector<void *> allocs_;
    std::vector<void *> scratch_allocs_;

    // weights
    float * emb_first_ = nullptr;
    std::vector<float *> emb_rest_;
    int dq_ = 0, cbdim_ = 0, latent_ = 0, dec_ = 0;
    QMat dq_first_out_, dq_rest_out_, in_proj_, out_proj_;
    float * in_proj_b_ = nullptr, * out_proj_b_ = nullptr, * out_norm_ = nullptr;
    Conv dpre_, dhead_, dfin_;
    float * fin_alpha_ = nullptr, * fin_beta_ = nullptr;
    std::vector<Layer> layers_;
    std::vector<Up> ups_;
    std::vector<Blk> blks_;
    float2 * rope_ = nullptr;
    int rope_max_ = 0;
    GemvScratch scr_;
    int * err_ = nullptr;  // bounded-wait error flag of the tcgen05 GEMM

    // activations, grown on demand (T frames at a time)
    int tcap_ = 0;
    size_t act_elems_ = 0;
    float * a_ = nullptr, * b_ = nullptr, * c_ = nullptr;   // conv-stack ping-pong [C][L]
    float * t32_ = nullptr, * q_ = nullptr, * o_ = nullptr;  // q_: rows of q | k | v
    float * pcm_ = nullptr;
    float * part_ = nullptr;  // channel-split partial sums of the convolutions
    half * t16_ = nullptr, * att16_ = nullptr, * f16_ = nullptr;
    int * codes_ = nullptr;
    float * fring_ = nullptr;  // keys and values of whole-decode segments [S][T][2][kv dim]
    float * pcm_host_ = nullptr;  // pinned PCM of the serving step's decode
    size_t pcm_host_cap_ = 0;     // floats
    int * rows_dev_ = nullptr;    // frame rows of the serving step's streams
    int rows_cap_ = 0;

    // streams: carried convolution states [slot][st_floats_] (every state layer's [2][cin][P] at
    // st_off_[layer], in decode order), key/value rings [slot][layer][ring_R_][2][kv dim]
    std::map<int, StreamInfo> streams_;
    std::vector<int> free_slots_;
    int stream_cap_ = 0;
    std::vector<size_t> st_off_;
    size_t st_floats_ = 0;
    float * st_pool_ = nullptr, * ring_ = nullptr;
    int ring_R_ = 0;
    float2 * srope_ = nullptr;  // RoPE table for kMaxStreamFrames positions
    int * seg_dev_ = nullptr;   // [3][seg_cap_]: slot, copy, first position of each segment
    int * seg_ident_ = nullptr; // [2][seg_cap_]: 0, 1, 2, ... and zeros (whole-decode segments)
    int seg_cap_ = 0;
    std::vector<void *> stream_allocs_;

    std::mutex mu_;
    std::map<int, std::vector<int>> history_;
};

// The codec encoder: 24 kHz PCM -> codebook frames (MimiCodec::encode, src/codec.cpp:80-123) on
// the GPU: the SEANet encoder's convolutions on the vocoder's TF32 conv kernel (strided convs as
// polyphase causal convs), the Mimi encoder transformer, the stride-2 downsample, the quantiser
// projections and the semantic + residual acoustic nearest-codebook search.
class CodecEncoder {
public:
    CodecEncoder(const GgufFile & gg, const ModelConfig & cfg, int device);
    ~CodecEncoder();
    static constexpr int kSamplesPerFrame = 1920;
    // PCM [n] -> codes frame-major [T][nc] with T = n / 1920 (a trailing partial frame does not
    // change the frames before it: every stage is causal); returns T
    int encode(const float * pcm, int n, std::vector<int> & codes);
    int nc() const { return cfg_.nc; }

private:
    struct Conv {
        float * w = nullptr, * b = nullptr;  // tap-major [cout][taps][cin * stride]
        int cin = 0, cout = 0, taps = 0, stride = 1;
    };
    struct Layer {
        QMat q, k, v, o, up, down;
        float * an_w = nullptr, * an_b = nullptr, * fn_w = nullptr, * fn_b = nullptr;
        float * attn_scale = nullptr, * ffn_scale = nullptr;
    };
    const GgufTensor & need(const std::string & name) const;
    float * upload(const std::vector<float> & h);
    float * load_f32(const std::string & name, int64_t expect);
    QMat load_lin(const std::string & name);
    Conv load_conv(const std::string & name, int cin, int cout, int stride, bool bias);
    void ensure(int L);
    void conv(const Conv & c, const float * x, int Lin, float * y, bool elu_out, const float * res, float * y2, bool elu2,
              cudaStream_t s);

    const GgufFile & gg_;
    ModelConfig cfg_;
    EncConfig ec_;
    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    std::vector<void *> allocs_, scratch_;
    Conv c0_, c14_, down_;
    Conv res1_[4], res3_[4], strided_[4];
    std::vector<Layer> layers_;
    QMat sq_in_, aq_in_;
    float * books_ = nullptr;  // [nc][dim][codebook size]: the semantic book, then the acoustic ones, transposed
    int book_n_ = 0;
    float2 * rope_ = nullptr;
    int rope_max_ = 0;
    GemvScratch scr_;
    int * err_ = nullptr;
    // activations (grown on demand)
    int lcap_ = 0;
    size_t act_ = 0;
    float * X_ = nullptr, * E_ = nullptr, * H_ = nullptr, * part_ = nullptr;
    float * t32_ = nullptr, * q_ = nullptr, * k_ = nullptr, * v_ = nullptr, * o_ = nullptr, * res_ = nullptr;
    half * t16_ = nullptr, * att16_ = nullptr, * f16_ = nullptr;
    float * dpart_ = nullptr;
    int * ipart_ = nullptr, * codes_ = nullptr;
    std::mutex mu_;
};

}  // namespace bzb
