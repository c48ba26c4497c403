/*
 * n3d.h -- C ABI of the B200 (sm_100a) backend for the Nemotron-3 diarization
 * forward pass.
 *
 * This is the `extern "C"` layer a Rust `Model` would bind with `extern "C"`
 * declarations.  It replaces the reference crate's public
 * API (src/lib.rs:45-64) and its accelerator plug point
 * `Model.accel: Option<RefCell<GpuEngine>>` (src/model.rs:137-139):
 *
 *   Model::load_gpu              -> n3d_model_load_gpu
 *   Model::run_offline           -> n3d_run_offline
 *   Model::run_streaming         -> n3d_run_streaming
 *   Model::num_speakers          -> n3d_num_speakers
 *   extract_speaker_dict         -> n3d_extract_speaker_dict
 *   GpuEngine::{embed_mel_range, forward_embeds, head_forward, forward_window}
 *                                -> n3d_embed_range, n3d_forward_embeds,
 *                                   n3d_head_forward, n3d_forward_window
 *
 * Conventions: all pointers are plain host pointers unless a parameter name
 * starts with `d_` (device memory on the model's GPU).  Every call returns an
 * n3d_status; on failure n3d_last_error() holds a thread-local message.
 * Calls on one model are serialised by the caller (the reference `Model` is
 * not Sync either); different models may be used from different threads.
 * Outputs allocated by the library are released with the matching *_free.
 */
#ifndef N3D_H
#define N3D_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Mirrors DiarizationError (src/error.rs:7-45) plus the CUDA-specific cases. */
typedef enum n3d_status {
    N3D_OK = 0,
    N3D_ERR_IO = 1,
    N3D_ERR_JSON = 2,
    N3D_ERR_SAFETENSORS = 3,
    N3D_ERR_TENSOR_DTYPE = 4,
    N3D_ERR_MISSING_TENSOR = 5,
    N3D_ERR_TENSOR_SHAPE = 6,
    N3D_ERR_UNSUPPORTED_AUDIO = 7,
    N3D_ERR_NPY = 8,
    N3D_ERR_GPU = 9,
    N3D_ERR_CUDA = 10,
    N3D_ERR_TIMEOUT = 11, /* a bounded device-side wait gave up; the context is still usable */
    N3D_ERR_NO_DEVICE = 12,
    N3D_ERR_INVALID_ARGUMENT = 13
} n3d_status;

/* StreamingMode, src/config.rs:21-27. */
typedef enum n3d_mode {
    N3D_MODE_LOW_LATENCY = 0,
    N3D_MODE_VERY_LOW_LATENCY = 1,
    N3D_MODE_ULTRA_LOW_LATENCY = 2,
    N3D_MODE_OFFLINE = 3
} n3d_mode;

typedef struct n3d_model n3d_model;

/* RunOutput, src/model.rs:43-53.  `logits` is [num_frames, num_speakers], pre-sigmoid. */
typedef struct n3d_run_output {
    float *logits;
    size_t num_frames;
    size_t num_speakers;
    size_t num_chunks;
    int cache_compressed;
    size_t cache_frames;
    size_t fifo_frames;
} n3d_run_output;

/* Segment, src/segments.rs:9-14. */
typedef struct n3d_segment {
    float start;
    float end;
    size_t speaker;
} n3d_segment;

/* ------------------------------------------------------------- model + runs */

/* Model::load_gpu (src/model.rs:160-166): reads config.json, processor_config.json
 * and model.safetensors from `dir` and uploads the weights to CUDA device `device`. */
n3d_status n3d_model_load_gpu(const char *dir, int device, n3d_model **out);
void n3d_model_free(n3d_model *model);

/* Run the model's work on the caller's CUDA stream (a cudaStream_t passed as
 * void*), or on the model's own stream again when `stream` is NULL.  No
 * reference counterpart (wgpu owns its single queue, src/gpu.rs:55-64). */
n3d_status n3d_model_set_stream(n3d_model *model, void *stream);

/* Model::num_speakers (src/model.rs:211-213) and Model::hidden_size (src/model.rs:215-217). */
size_t n3d_num_speakers(const n3d_model *model);
size_t n3d_hidden_size(const n3d_model *model);

/* Model::gpu_describe (src/model.rs:207-209; GpuEngine::describe, src/gpu_engine.rs:534):
 * the device the model runs on and this library's build, e.g. "NVIDIA B200 (device 0,
 * sm_100, 148 SMs, 179 GiB) | n3d-b200 ...".  The string belongs to the model and stays
 * valid until the next call on it or n3d_model_free; NULL for a NULL model. */
const char *n3d_model_describe(n3d_model *model);

/* Model::run_offline (src/model.rs:232-234). */
n3d_status n3d_run_offline(n3d_model *model, const float *samples, size_t n, n3d_run_output *out);

/* Model::run_streaming (src/model.rs:313-336). `mode` must not be N3D_MODE_OFFLINE. */
n3d_status n3d_run_streaming(n3d_model *model, const float *samples, size_t n, n3d_mode mode,
                             n3d_run_output *out);

void n3d_run_output_free(n3d_run_output *out);

/* Many independent clips in one call (no reference counterpart: the reference
 * runs one clip per call).  outs[i] is clip i's RunOutput, exactly what
 * n3d_run_offline / n3d_run_streaming returns for it alone. */
n3d_status n3d_run_batch(n3d_model *model, n3d_mode mode, const float *const *samples, const size_t *lens,
                         size_t n_clips, n3d_run_output *outs);

/* Device-resident batch (inputs already in HBM): clip i is d_audio[offsets[i] ..
 * offsets[i] + lens[i]); its logits land at d_logits[out_offsets[i] * num_speakers]
 * with n3d_batch_out_frames() rows.  Runs on the model's stream and returns
 * after the device work completes. */
n3d_status n3d_batch_out_frames(const n3d_model *model, n3d_mode mode, const size_t *lens, size_t n_clips,
                                size_t *frames_out);
n3d_status n3d_run_batch_device(n3d_model *model, n3d_mode mode, const float *d_audio, const size_t *offsets,
                                const size_t *lens, size_t n_clips, float *d_logits, const size_t *out_offsets);

/* ---------------------------------------------------------- streaming sessions */

/* Incremental streaming: one recording that arrives in pieces (a live call, a
 * microphone).  No reference counterpart: Model::run_streaming (src/model.rs:313-336)
 * takes the whole recording; a session produces the same logits as that call on the
 * concatenated audio, but emits each chunk's rows as soon as the chunk's samples are
 * complete.  The chunk schedule is the reference's (Model::streaming_chunks,
 * src/model.rs:343-365): chunk 0 runs once its (c+r)*8 mel frames of audio have
 * arrived, each later full chunk once all of its samples have, and the final, centred
 * chunk at n3d_session_close.  The speaker cache and FIFO stay in device memory between
 * calls (about 4 MiB per session).
 *
 * Each call fills `out` with the NEW logits rows only (out->num_frames of them, freed
 * with n3d_run_output_free, also when there are none) and the running totals:
 * num_chunks so far, cache_compressed, cache_frames, fifo_frames.  After close these
 * totals equal run_streaming's RunOutput fields.  A session belongs to one model and
 * must be freed before it; calls on one model (sessions included) are serialised by
 * the caller.  After a call fails the session can only be freed. */
typedef struct n3d_session n3d_session;
n3d_status n3d_session_open(n3d_model *model, n3d_mode mode, n3d_session **out);
n3d_status n3d_session_push(n3d_session *session, const float *samples, size_t n, n3d_run_output *out);
n3d_status n3d_session_close(n3d_session *session, n3d_run_output *out);
void n3d_session_free(n3d_session *session);

/* Many sessions of one model at once (a server's concurrent streams): appends
 * samples[i] (lens[i] of them) to sessions[i], then runs every ready chunk of every
 * session, the steps of different sessions batched into the same kernels; with
 * `close` != 0 it also runs each session's final chunk.  outs[i] as for
 * n3d_session_push.  Results equal pushing to each session alone. */
n3d_status n3d_sessions_push(n3d_session *const *sessions, const float *const *samples, const size_t *lens,
                             size_t count, int close, n3d_run_output *outs);

/* ------------------------------------------------------------------ stages */

/* mel::log_mel (src/mel.rs:160-225) on the device.  `out` holds
 * frame_count(n) * 128 floats; *frames receives that count. */
n3d_status n3d_log_mel(n3d_model *model, const float *samples, size_t n, int centered, float *out,
                       size_t out_cap, size_t *frames);

/* GpuEngine::embed_mel_range (src/gpu_engine.rs:1335-1379) / Tower::embed_range
 * (src/encoder.rs:126-146): groups lo..hi of 8 stacked mel frames -> [hi-lo, hidden],
 * frames past num_frames read as zeros.  At most 1024 groups per call, as the
 * reference's MAX_SEQ. */
n3d_status n3d_embed_range(n3d_model *model, const float *mel, size_t num_frames, size_t lo, size_t hi,
                           float *out);

/* GpuEngine::forward_embeds (src/gpu_engine.rs:1506-1514): the 31-layer tower on one
 * window [frames, hidden] (1..1024 frames) with `valid` unmasked keys (clamped to
 * frames) -> final LayerNorm output. */
n3d_status n3d_forward_embeds(n3d_model *model, const float *embeds, size_t frames, size_t valid, float *out);

/* GpuEngine::head_forward (src/gpu_engine.rs:1695-1699): [frames, hidden] -> [frames*8, ns] logits. */
n3d_status n3d_head_forward(n3d_model *model, const float *encoder_out, size_t frames, float *logits);

/* GpuEngine::forward_window (src/gpu_engine.rs:1516-1520): tower + head on one window. */
n3d_status n3d_forward_window(n3d_model *model, const float *embeds, size_t frames, size_t valid, float *logits);

/* CacheConfig (src/streaming.rs:39-52): the speaker-cache policy, as
 * CacheConfig::from_model resolves it (src/streaming.rs:54-76). */
typedef struct n3d_cache_config {
    size_t fifo_length;
    size_t speaker_cache_length;
    size_t update_period;
    size_t num_silence_frames;
    float score_threshold;
    float latest_frames_score_boost;
    size_t num_speakers;
    size_t subsampling_factor;
    size_t min_positive_scores;
    size_t num_strong_boosted_frames;
    size_t num_weak_boosted_frames;
} n3d_cache_config;

/* SpeakerCache::trace_compress / compress (src/streaming.rs:353-482) on device
 * `device`, through the same selection and gather code the chunk loop's cache kernel
 * runs.  `probs` [frames, num_speakers] are the candidate frames' probabilities.
 * picked (room for speaker_cache_length entries) receives trace_compress's `picked`:
 * the first L = min(speaker_cache_length, num_speakers * (frames + num_silence_frames))
 * flat speaker-major indices in (score desc, index asc) order, -inf picks replaced by
 * *sentinel = num_speakers * (frames + num_silence_frames), sorted ascending; *count = L.
 * When `embeds` [frames, hidden] is not NULL, out_embeds [L, hidden] and out_probs
 * [L, num_speakers] receive compress()'s result: each pick's row and probabilities,
 * `silence` [hidden] and a zero row for silence slots and sentinels.  Host pointers.
 * 1 <= frames, num_speakers <= 16, hidden % 4 == 0, and the working set must fit one
 * CTA's shared memory (8 speakers: about 1500 frames). */
n3d_status n3d_cache_compress(int device, const n3d_cache_config *cfg, const float *probs, size_t frames,
                              const float *embeds, size_t hidden, const float *silence, size_t *picked,
                              size_t *sentinel, size_t *count, float *out_embeds, float *out_probs);

/* ------------------------------------------------------------ segments */

/* extract_speaker_dict (src/segments.rs:70-109).  `mask` may be NULL. */
n3d_status n3d_extract_speaker_dict(const float *logits, size_t num_frames, size_t num_speakers, float duration,
                                    const uint8_t *mask, float threshold, n3d_segment **out, size_t *count);
void n3d_segments_free(n3d_segment *segments);

/* activity_stats (src/segments.rs:113-141): returns the speech percentage and, when
 * per_speaker is not NULL, each speaker's active-frame count (num_speakers entries). */
float n3d_activity_stats(const float *logits, size_t num_frames, size_t num_speakers, const uint8_t *mask,
                         float threshold, size_t *per_speaker);

/* frame_duration (src/segments.rs:36-38). */
float n3d_frame_duration(size_t hop_length, uint32_t sampling_rate);

/* ------------------------------------------------------- chunk schedule (host) */
/* These need no GPU: they read the checkpoint's two JSON files and do the integer
 * chunk arithmetic the runs above follow. */

typedef struct n3d_config n3d_config;

/* load_configs (src/config.rs:221-225): config.json and processor_config.json of a
 * checkpoint directory.  Free with n3d_config_free. */
n3d_status n3d_config_load(const char *dir, n3d_config **out);
void n3d_config_free(n3d_config *cfg);

/* ModeParams (src/config.rs:127-147) as ModeParams::resolve / Model::params build it
 * (src/config.rs:152-195, src/model.rs:219-221).  Offline has zero chunk geometry and
 * the latency of the offline window. */
typedef struct n3d_mode_params {
    size_t hop_length;
    size_t n_fft;
    size_t subsampling;
    size_t mel_frames_per_chunk;
    size_t mel_frames_per_step;
    size_t lookahead_encoder_frames;
    size_t first_chunk_samples;
    size_t samples_per_chunk;
    size_t latency_ms;
} n3d_mode_params;
n3d_status n3d_mode_params_resolve(const n3d_config *cfg, n3d_mode mode, n3d_mode_params *out);

/* One chunk of Model::streaming_chunks (src/model.rs:343-365) without its mel
 * features: samples [start, start + len), centred or not, the mel frames log_mel
 * keeps (Chunk::num_mel_frames) and the look-ahead in encoder frames. */
typedef struct n3d_chunk {
    size_t start;
    size_t len;
    int centered;
    size_t num_mel_frames;
    size_t lookahead;
} n3d_chunk;
/* Writes min(count, cap) chunks; *count is the full number (call with cap 0 to size
 * the array).  Streaming modes only. */
n3d_status n3d_streaming_chunks(const n3d_config *cfg, size_t n_samples, n3d_mode mode, n3d_chunk *out,
                                size_t cap, size_t *count);

/* One chunk-loop step, the counts of ChunkTrace (src/model.rs:57-75): frames carried
 * in from the cache and FIFO, the window the tower sees, the frames the mask lets
 * through, the frames scored, and the cache and FIFO after the step's update. */
typedef struct n3d_step_plan {
    size_t cached_frames;
    size_t window_frames;
    size_t valid_frames;
    size_t scored_frames;
    size_t cache_frames;
    size_t fifo_frames;
    int cache_compressed;
} n3d_step_plan;
/* The steps a run of n_samples in `mode` takes (run_offline_capturing / run_streaming
 * with chunk_loop, src/model.rs:242-336, 478-538).  Writes min(count, cap) steps and
 * sets *count; `totals` (nullable) receives the RunOutput fields the run will return,
 * with logits NULL.  Streaming audio too short for the look-ahead fails with
 * N3D_ERR_UNSUPPORTED_AUDIO, as the runs do. */
n3d_status n3d_schedule(const n3d_config *cfg, n3d_mode mode, size_t n_samples, n3d_step_plan *steps,
                        size_t cap, size_t *count, n3d_run_output *totals);

/* -------------------------------------------------- single kernels (device) */
/* n3d_linear, n3d_layer_norm and n3d_attention run on a stream of the library's own
 * per device and return after it has finished; concurrent calls on one device take
 * turns. */

/* tensor::linear (src/tensor.rs:22-57) on device buffers: d_y[rows, out] =
 * d_x[rows, cols] * d_w[out, cols]^T + d_bias (nullable).  cols % 32 == 0.
 * Uses temporary device memory for the fp16 operand split (h, l, each operand
 * scaled by a power of two from its max |x|). */
n3d_status n3d_linear(int device, const float *d_x, size_t rows, size_t cols, const float *d_w, size_t out,
                      const float *d_bias, float *d_y);

/* n3d_linear for callers that cannot allocate device memory when they call
 * (a real-time audio thread that must not block in the driver's allocator, a
 * host framework that owns all GPU memory through its own pool, a process with
 * an allocation budget fixed at start-up).  No counterpart in the reference.
 * The operand split uses a fixed 16 MiB array inside the library's GPU image
 * instead of temporary memory, so the call allocates nothing.  Limits:
 * rows*cols + out*cols at most 4194240 (larger requests fail with
 * N3D_ERR_INVALID_ARGUMENT); every GPU that loads the library keeps the 16 MiB
 * until exit; all calls on a device share the array, so calls whose GPU work
 * overlaps race and must be serialised by the caller.  The first call on each
 * device does a one-time set-up; make it before any stream capture.  Runs on
 * `stream` (a cudaStream_t, NULL for the default stream) and returns after it
 * has finished. */
n3d_status n3d_linear_noalloc(int device, const float *d_x, size_t rows, size_t cols, const float *d_w,
                              size_t out, const float *d_bias, float *d_y, void *stream);

/* tensor::layer_norm (src/tensor.rs:97-110), cols 512 or 1024. */
n3d_status n3d_layer_norm(int device, const float *d_x, size_t rows, size_t cols, const float *d_w,
                          const float *d_b, float *d_y);

/* RoPE (src/encoder.rs:163-185, 281-296, positions 0..seq-1, when `rope` != 0) followed
 * by attention over the first `valid` keys (src/encoder.rs:302-329) on device buffers
 * q, k, v, out of shape [seq, heads * head_dim]; head_dim 64 or 128. */
n3d_status n3d_attention(int device, const float *d_q, const float *d_k, const float *d_v, size_t seq,
                         size_t heads, size_t head_dim, size_t valid, int rope, double rope_theta, float *d_out);

/* Probe benchmarks: GpuEngine::bench_gemm (src/gpu_engine.rs:562-596) and the
 * GEMM_BENCH / ATTN_BENCH / STAGE_BENCH probes (src/bin/gpu_check.rs:132-289), for
 * the kernels above.  Each sets up synthetic operands in the kernel's own device
 * layout (n3d_linear's split operands, the attention's packed operands), launches the
 * kernel 3 times untimed, then `iters` times between two CUDA events on the library's
 * stream of `device`, and returns the mean device time of one launch in *ms.  The
 * operands stay resident, so shapes smaller than the 126 MB L2 run L2-warm.
 * n3d_bench_linear times n3d_linear's GEMM (output [rows, out] fp32 with a bias);
 * n3d_bench_attention the attention over all `seq` keys (no RoPE); n3d_bench_layer_norm
 * n3d_layer_norm. */
n3d_status n3d_bench_linear(int device, size_t rows, size_t cols, size_t out, int iters, double *ms);
n3d_status n3d_bench_attention(int device, size_t seq, size_t heads, size_t head_dim, int iters, double *ms);
n3d_status n3d_bench_layer_norm(int device, size_t rows, size_t cols, int iters, double *ms);

/* Self-test of failure detection on the device, for a health check or a test: the
 * reference has no device-side wait to bound (its error path only reports wgpu
 * failures, src/gpu_engine.rs:1345-1349), while every wait of this library's kernels
 * gives up after a limit, records where, and lets the kernel return.  This runs one
 * such wait on `device` with a limit of `limit_ms` (0.001..2000) on a flag that
 * nothing sets, exactly as an expired wait in a real kernel would: the call returns
 * N3D_ERR_TIMEOUT, n3d_last_error() names the site, *waited_ms (nullable) receives the
 * device time the wait took, and the device stays usable for the next call. */
n3d_status n3d_selftest_wait_timeout(int device, double limit_ms, double *waited_ms);

/* ------------------------------------------------------------- profiling */

/* Device time per kernel class of the launches n3d_run_* make while profiling
 * is on, from CUDA events on the model's own stream.  No reference
 * counterpart: replaces the env-gated wall-clock timers GPU_PROFILE /
 * STEP_PROFILE / STAGE_BENCH (src/gpu_engine.rs:1682-1690, src/model.rs:417-473,
 * src/bin/gpu_check.rs:132-289).  Enabling resets the counters. */
typedef struct n3d_kernel_stats {
    const char *name;     /* "attention", "layer_norm", "mel", "cache_update", "assemble", and one
                             "gemm_*" class per GEMM site (qkv, o, fc1, fc2, head_proj, head_conv,
                             head_dense, embed) */
    size_t launches;
    double ms;            /* summed device time */
    double flops;         /* algorithmic FLOPs of those launches (2*M*N*K for GEMMs) */
    double bytes;         /* algorithmic DRAM bytes (memory-bound classes) */
} n3d_kernel_stats;
n3d_status n3d_profile_enable(n3d_model *model, int on);
size_t n3d_profile_read(const n3d_model *model, n3d_kernel_stats *out, size_t cap);

/* Device time of each chunk-loop step (one step of every clip in the batch:
 * window assembly, tower, head, cache update), from two CUDA events per step.
 * Replaces STEP_PROFILE (src/model.rs:314, 417-473).  Enabling clears the list;
 * n3d_step_times copies up to `cap` values (ms) and returns how many exist. */
n3d_status n3d_step_timing_enable(n3d_model *model, int on);
size_t n3d_step_times(const n3d_model *model, double *ms, size_t cap);

/* ------------------------------------------------------------------ misc */

/* The message of this thread's last failed call (empty after a success): the text the
 * reference's DiarizationError carries (src/error.rs:7-45).  Valid until this thread's
 * next call into the library. */
const char *n3d_last_error(void);
/* This build: library version, target architecture and precision scheme.  No reference
 * counterpart (a static string). */
const char *n3d_version(void);

#ifdef __cplusplus
}
#endif
#endif
