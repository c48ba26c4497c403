// Host-side model: configuration, device weights, workspace and the batched
// chunk-loop runner behind the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <functional>
#include <string>
#include <vector>

#include "n3d_cache.h"
#include "n3d_internal.h"

namespace n3d {

// ----------------------------------------------------------------- config

// config.json + processor_config.json, the fields src/config.rs:43-131 reads.
struct Config {
    int hidden = 0, layers = 0, heads = 0, kv_heads = 0, inter = 0, n_mels = 0, sub = 0;
    double rope_theta = 10000.0;
    int head_hidden = 0, num_speakers = 0;
    // streaming_config
    int s_fifo = 0, cache_len = 0, n_sil = 0, s_period = 0, s_sub = 0, s_ns = 0;
    float thr = 0, min_pos_rate = 0, strong_rate = 0, weak_rate = 0, latest_boost = 0;
    // offline chunking
    int chunk_length = 0, chunk_rc = 0, o_fifo = 0, o_period = 0;
    // feature extractor
    int feature_size = 0, n_fft = 0, hop = 0, win = 0, sr = 0;
    float preemph = 0;
    int proc_sub = 0;
    int modes[3][2] = {{0, 0}, {0, 0}, {0, 0}};
    // CacheConfig::from_model derived counts (src/streaming.rs:54-72)
    int min_pos = 0, k_strong = 0, k_weak = 0;
};

Config load_config(const std::string& dir);

// ----------------------------------------------------------------- weights

// A linear layer's weight [out, in] in the fp16 split (scale s: h + l = w s) plus an
// optional bias.
struct DevLinear {
    void* h = nullptr;
    void* l = nullptr;
    float* bias = nullptr;
    int out = 0, in = 0;
    float scale = 1.0f;
    SplitOperand op() const { return SplitOperand{h, l, out, in, in, scale}; }
};

// Workspace for an activation in the fp16 split (base_h / base_l), rows_cap = rows the
// buffers hold.  The scale belongs to the producer and consumer of each use.
struct SplitBuf {
    void* h = nullptr;
    void* l = nullptr;
    long long rows_cap = 0, cols = 0;
    SplitOperand op(float scale) const { return SplitOperand{h, l, rows_cap, cols, cols, scale}; }
    SplitOut out(float scale) const { return SplitOut{h, l, scale, nullptr}; }
};

// Per layer: LayerNorm parameters, weights, and the fp16-split scales of the layer's
// GEMM inputs, each from a bound on the tensor's magnitude known at load: the two
// LayerNorm outputs (sqrt(cols - 1) max|w| + max|b|), the attention context (a convex
// combination of V rows: max row L1 norm of W_v times the LayerNorm bound; also V's
// own scale), GELU(fc1) (|gelu(x)| <= |x|: max over rows of L1(W_fc1) times the bound
// plus |b|), and the attention operands Q and K (rotate-half RoPE at most doubles the
// bound of W_q n or W_k n).
struct DevLayer {
    float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
    DevLinear qkv, o, fc1, fc2;
    float s_ln1 = 1.0f, s_ln2 = 1.0f, s_ctx = 1.0f, s_ffn = 1.0f, s_q = 1.0f, s_k = 1.0f;
};

// ----------------------------------------------------------------- schedule

struct MelSeg {           // one log_mel call of the reference
    long long audio_off;  // within the clip
    long long len;
    int centered;
    int frames;           // frame_count(len)
    int groups;           // ceil(mel rows / sub); mel rows are padded with zeros to groups * sub
    long long group_base; // global row in the [groups, sub * n_mels] view (set at batch assembly)
    int frame_lo = 0;     // first frame computed (group g of this launch starts at frame_lo + g * sub)
};

// Frames of `m` computed in one mel launch: [frame_lo, frame_lo + mel_frames).
inline int mel_frames(const MelSeg& m, int sub) {
    const int end = m.frames < m.frame_lo + m.groups * sub ? m.frames : m.frame_lo + m.groups * sub;
    return end > m.frame_lo ? end - m.frame_lo : 0;
}

struct StepPlan {
    int S, valid, ncache, nfifo, nchunk, popped, compress, was_compressed, keep_rows;
    int seg;              // mel segment holding this step's new frames
    int group_lo;         // first group of that segment the step embeds
    int n_new;            // groups of that segment it embeds
    // Embedding rows taken from the previous step instead (streaming middle chunks): the
    // window's new rows are the previous step's last `reuse` rows, then the n_new rows
    // from group_lo on.  0 = none.
    int reuse;
};

struct ClipPlan {
    std::vector<MelSeg> segs;
    std::vector<StepPlan> steps;
    long long emitted_rows = 0;  // 10 ms rows written by the steps
    long long out_rows = 0;      // rows returned (offline truncates to valid + 1)
    int num_chunks = 0, cache_compressed = 0, cache_frames = 0, fifo_frames = 0;
};

ClipPlan plan_offline(const Config& c, long long n);
ClipPlan plan_streaming(const Config& c, long long n, int mode);

// One chunk of Model::streaming_chunks (src/model.rs:343-365): samples [start,
// start + len) of the recording, centred or not, the mel frames its log_mel keeps, and
// the encoder frames held back as look-ahead.
struct StreamChunk {
    long long start, len, mel_frames;
    int centered, lookahead;
};
std::vector<StreamChunk> streaming_chunks(const Config& c, long long n, int mode);

// ----------------------------------------------------------------- sessions

class Model;

// Incremental streaming (one recording arriving in pieces).  The chunk schedule is
// run_streaming's (src/model.rs:343-365): chunk 0 runs once its (c+r)·8 mel frames of
// audio have arrived, every later full chunk once its samples are complete, and the
// final centred chunk at close; the speaker cache stays on the device between calls.
struct Session {
    Model* model = nullptr;
    int mode = 0;
    long long received = 0;   // samples pushed so far
    long long base = 0;       // absolute index of audio[0]; earlier samples are no longer needed
    std::vector<float> audio;
    int next_chunk = 0;
    bool done = false;        // the final chunk has run
    bool closed = false;
    bool failed = false;      // a call failed part-way; the session can only be freed
    int ncache = 0, nfifo = 0, compressed = 0, num_chunks = 0;
    long long steps = 0;      // steps run (ping-pong parity of the state buffers)
    float* pre = nullptr;     // [2, s_cap, hidden]: cache ++ FIFO embeddings
    float* cprob = nullptr;   // [2, s_cap, num_speakers]: their stored probabilities
};

// ----------------------------------------------------------------- model

struct Buf {
    void* p = nullptr;
    size_t bytes = 0;
};

// Per-kernel-class device time, measured with CUDA events on the model's stream.
enum KernelClass : int {
    K_GEMM = 0, K_ATTN, K_LN, K_MEL, K_CACHE, K_ASSEMBLE, K_OTHER,
    K_GEMM_QKV, K_GEMM_O, K_GEMM_FC1, K_GEMM_FC2, K_GEMM_PROJ, K_GEMM_CONV, K_GEMM_DENSE, K_GEMM_EMBED, K_NCLASS
};
struct ProfTotals {
    long long launches = 0;
    double ms = 0.0, flops = 0.0, bytes = 0.0;
};

class Model {
  public:
    Model(const std::string& dir, int device);
    ~Model();

    const Config& cfg() const { return cfg_; }
    int device() const { return device_; }

    // Batched chunk loop over independent clips (offline mode = 3).  Host or
    // device audio; results either copied to host vectors or left in d_logits.
    // Host destination of one clip's logits: given the clip index and the float count,
    // returns where to write them (called once per clip, from the calling thread).
    using HostSink = std::function<float*(int clip, size_t n)>;
    void run_batch(int mode, const std::vector<const float*>& host_audio, const float* d_audio,
                   const std::vector<long long>& offsets, const std::vector<long long>& lens,
                   const HostSink* host_out, float* d_logits, const std::vector<long long>* out_offsets,
                   std::vector<ClipPlan>* plans_out);

    // Sessions of this model (freed before the model).  sessions_push appends
    // samples[i] to ss[i] and runs every chunk that is complete, the steps of all
    // sessions batched round by round; with `close` it also runs the final chunks.
    // rows[i] receives session i's new logits rows ([rows, num_speakers]).
    struct SessionChunk;  // one ready chunk of one session (model.cpp)
    Session* session_open(int mode);
    void session_free(Session* s);
    void sessions_push(const std::vector<Session*>& ss, const std::vector<const float*>& samples,
                       const std::vector<long long>& lens, bool close, std::vector<std::vector<float>>& rows);

    // Stage entry points (single sequence, host buffers).
    int log_mel(const float* samples, long long n, bool centered, std::vector<float>& out);
    void embed_range(const float* mel, long long num_frames, long long lo, long long hi, float* out);
    void forward_window(const float* embeds, int frames, int valid, float* enc_out, float* logits);
    void head_forward(const float* enc, int frames, float* logits);

    // Work runs on `s` (caller-owned) or, for nullptr, on the model's own stream.
    void set_stream(cudaStream_t s);

    // Profiling of the launches of run_batch (off by default).
    void profile_enable(bool on);
    const ProfTotals* profile_totals() const { return totals_; }
    // Device time of every chunk-loop step (all sequences of the batch), two
    // events per step; enabling clears the list.
    void step_timing_enable(bool on);
    const std::vector<float>& step_times() const { return step_ms_; }

  private:
    void prof_begin();
    void prof_end(int cls, double flops, double bytes);
    void prof_collect();
    void upload_weights(const std::string& dir);
    void tower(int B, int S, const int* d_seq_len, const int* d_valid, float* enc_plain);
    // The tower of one chunk-loop step.  Small batches (at most kGraphMaxSeqs
    // sequences: the windows of a single long clip, a few sessions) are latency-bound
    // chains of ~220 short kernels, so the tower runs as a CUDA graph, one per (B, S),
    // captured on the second step of that shape (the first sizes the workspace) and
    // captured again after any workspace buffer is reallocated.  The step's key counts
    // go through fixed slot buffers so that one graph serves every step.
    void tower_step(int B, int S, const int* d_len, const int* d_valid);
    // `widen` (a power of two >= 1) lowers the scales of the head's GEMM inputs below
    // the final LayerNorm's for inputs that exceed its bound (head_forward's caller data).
    void head(int B, int S, const int* d_seq_len, float widen = 1.0f);
    // Log-mel + embedder of `segs` (segment i's samples start at d_audio[base[i]]).
    // mel_prepare uploads the segment table (from host memory, so call it before the
    // stream is busy); mel_launch runs the mel and the embedder GEMM.  `parts`
    // (optional): frame ranges [previous end, end) whose audio arrives on the copy
    // stream; the mel of each range waits for its event.  `tag` names the workspace
    // buffers, so that two prepared launches can be in flight.
    struct MelJob {
        long long groups = 0, frames = 0;
        const MelSegDev* segs = nullptr;
        int nsegs = 0;
        std::string tag;
    };
    MelJob mel_prepare(const std::vector<long long>& base, const std::vector<MelSeg>& segs, long long total_groups,
                       long long total_frames, const char* tag = "");
    const float* mel_launch(const float* d_audio, const MelJob& job,
                            const std::vector<std::pair<long long, cudaEvent_t>>* parts = nullptr);
    const float* mel_embed(const float* d_audio, const std::vector<long long>& base, const std::vector<MelSeg>& segs,
                           long long total_groups, long long total_frames) {
        return mel_launch(d_audio, mel_prepare(base, segs, total_groups, total_frames));
    }
    // One chunk-loop step of B sequences (rows of stride S): window assembly, tower,
    // head, cache update.
    void run_step(const SeqStep* d_steps, int B, int S, const int* d_len, const int* d_valid, const float* embeds);
    void session_round(std::vector<SessionChunk>& items, std::vector<std::vector<float>>& rows);
    void* ws(const char* name, size_t bytes);
    SplitBuf ws2(const std::string& base, long long rows, long long cols);
    // The fp16-split scale of n floats on the device from their max |x| (one readback).
    float dyn_scale(const float* d, long long n);
    void check_dev_error();

    Config cfg_;
    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    cudaStream_t own_stream_ = nullptr;
    // Host audio of a batch is uploaded on copy_stream_ in parts of kUploadClips
    // clips, so the mel of part k overlaps the upload of part k + 1.
    static constexpr int kUploadClips = 16;
    cudaStream_t copy_stream_ = nullptr;
    static constexpr int kGraphMaxSeqs = 16;
    static constexpr int kGraphCacheMax = 64;
    struct TowerGraph {
        cudaGraphExec_t exec = nullptr;
        uint64_t gen = 0;  // ws_gen_ at capture
    };
    std::map<std::pair<int, int>, TowerGraph> tower_graphs_;
    uint64_t ws_gen_ = 0;  // bumped whenever a workspace buffer is (re)allocated
    cudaStream_t capture_stream_ = nullptr;
    // Pinned staging of a batch's logits on their way to the host (grown on demand).
    float* host_stage_ = nullptr;
    size_t host_stage_bytes_ = 0;
    float* host_stage(size_t bytes);
    cudaEvent_t upload_start_ = nullptr;
    std::vector<cudaEvent_t> upload_ev_;
    int* dev_err_ = nullptr;

    DevLinear embed_, proj_, conv_, dense_;
    // fp16-split scales of the other GEMM inputs: the log-mel (|ln x| <= 89 for any
    // finite positive x >= 2^-24), the final LayerNorm output, proj's output and the
    // conv's ReLU output (row L1 bounds as for the layers).
    float s_mel_ = 1.0f, s_fin_ = 1.0f, s_proj_ = 1.0f, s_conv_ = 1.0f;
    std::vector<DevLayer> layers_;
    float *in_ln_w_, *in_ln_b_, *fin_ln_w_, *fin_ln_b_;
    float *out_w_, *out_b_, *silence_;
    MelTables mel_tab_;  // log-mel window, twiddles and transposed filterbank
    float *rope_cos_, *rope_sin_;
    int s_cap_ = 1024;  // MAX_SEQ, src/gpu_engine.rs:12
    std::vector<void*> owned_;
    bool prof_ = false;
    bool step_timing_ = false;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> step_ev_;
    std::vector<float> step_ms_;
    cudaEvent_t pool_event();
    struct ProfRec {
        int cls;
        cudaEvent_t a, b;
        double flops, bytes;
    };
    std::vector<ProfRec> pending_;
    std::vector<cudaEvent_t> event_pool_;
    cudaEvent_t cur_begin_ = nullptr;
    ProfTotals totals_[K_NCLASS];
    std::map<std::string, Buf> ws_;
};

}  // namespace n3d
