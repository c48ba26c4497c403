/*
 * CPU restatement of the reference's pure-Rust CPU path for the Nemotron-3
 * diarization forward pass.  TEST INFRASTRUCTURE ONLY: the parity checker for
 * the CUDA product path and the timed CPU baseline.  Nothing in the product
 * library links or calls this code.
 *
 * Every function follows the reference file:line cited beside it, with the
 * same reduction order (sequential sums, separate multiply and add, no FMA:
 * build with -ffp-contract=off) and row-parallelism over OpenMP where the
 * reference uses rayon.  The FFT is this file's own radix-2 transform: the
 * reference uses rustfft 6.4.1, whose summation order is not reproducible
 * here, so FFT-level bit parity is unpinned (mel values agree to float
 * rounding).
 */
#ifndef N3D_ORACLE_H
#define N3D_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Feature-extractor settings, src/config.rs:101-109. */
typedef struct {
    size_t feature_size, n_fft, hop_length, win_length, sampling_rate;
    float preemphasis;
} orc_fe;

/* Speaker-cache policy, src/streaming.rs:39-51. */
typedef struct {
    size_t fifo_length, speaker_cache_length, update_period, num_silence_frames;
    float score_threshold, latest_frames_score_boost;
    size_t num_speakers, subsampling_factor;
    size_t min_positive_scores, num_strong_boosted_frames, num_weak_boosted_frames;
} orc_cache_cfg;

/* Everything the model needs from config.json / processor_config.json. */
typedef struct {
    size_t hidden, layers, heads, inter, n_mels, sub;
    double rope_theta;
    size_t head_hidden, num_speakers;
    size_t chunk_length, chunk_right_context;
    orc_cache_cfg cache_stream;  /* CacheConfig::from_model */
    orc_cache_cfg cache_offline; /* CacheConfig::offline */
    orc_fe fe;
    size_t modes[3][2]; /* low, very_low, ultra_low: [chunk, right] */
} orc_cfg;

/* Borrowed weight pointers (row-major, checkpoint layout). Per-layer arrays hold `layers` pointers. */
typedef struct {
    const float *embed_proj, *in_ln_w, *in_ln_b, *fin_ln_w, *fin_ln_b;
    const float *const *ln1_w, *const *ln1_b, *const *q, *const *k, *const *v, *const *o, *const *o_b;
    const float *const *ln2_w, *const *ln2_b, *const *fc1, *const *fc1_b, *const *fc2, *const *fc2_b;
    const float *proj_w, *proj_b, *conv_w, *conv_b, *dense_w, *dense_b, *out_w, *out_b, *silence;
    const float *mel_filters; /* [n_mels, n_fft/2+1] */
} orc_weights;

typedef struct {
    float *logits; /* [num_frames, num_speakers], malloc'd; free with orc_run_output_free */
    size_t num_frames, num_chunks;
    int cache_compressed;
    size_t cache_frames, fifo_frames;
} orc_run_output;

/* One chunk-loop step as seen by src/model.rs:371-475 (ChunkTrace, src/model.rs:57-75). */
typedef struct {
    size_t step, cached_frames, window_frames, valid_frames, scored_frames;
    const float *window;      /* [window_frames, hidden] encoder input */
    const float *encoder_out; /* [window_frames, hidden] */
    const float *step_logits; /* [window_frames*sub, ns] */
    const float *cache_embeds, *cache_probs, *fifo;
    size_t cache_frames, fifo_frames;
    int cache_compressed;
} orc_step_trace;
typedef void (*orc_step_cb)(void *user, const orc_step_trace *t);

typedef struct {
    float start, end;
    size_t speaker;
} orc_segment;

/* ---- src/tensor.rs ---- */
void orc_linear(const float *x, size_t rows, size_t cols, const float *w, size_t out, const float *bias, float *y);
void orc_matmul(const float *a, size_t m, size_t k, const float *b, size_t n, float *c);
void orc_layer_norm(const float *x, size_t rows, size_t cols, const float *w, const float *b, float *y);
void orc_gelu(const float *x, size_t n, float *y);
void orc_relu(const float *x, size_t n, float *y);
void orc_softmax_last(float *x, size_t rows, size_t cols);

/* ---- src/mel.rs ---- */
void orc_hann_periodic_false(size_t n, float *out);
void orc_slaney_mel_filterbank(size_t n_mels, size_t n_fft, size_t sample_rate, double fmin, double fmax, float *out);
void orc_mel_filters(const orc_fe *fe, float *out);
size_t orc_frame_count(size_t n_samples, const orc_fe *fe, int centered);
size_t orc_log_mel(const float *samples, size_t n, const orc_fe *fe, int centered, const float *filters, float *out);
void orc_fft(float *re, float *im, size_t n);

/* ---- src/encoder.rs ---- */
void orc_rope_tables(size_t seq, size_t hd, double theta, size_t offset, float *cos_out, float *sin_out);
void orc_apply_rope(float *x, size_t seq, size_t nh, size_t hd, const float *cos_t, const float *sin_t);
void orc_attention(const float *q, const float *k, const float *v, size_t seq, size_t nh, size_t hd, size_t valid,
                   float *out);
void orc_embed_range(const orc_cfg *c, const orc_weights *w, const float *mel, size_t num_frames, size_t lo,
                     size_t hi, float *out);
void orc_forward_embeds(const orc_cfg *c, const orc_weights *w, const float *embeds, size_t groups, size_t valid,
                        float *out);

/* ---- src/head.rs ---- */
void orc_head_forward(const orc_cfg *c, const orc_weights *w, const float *enc, size_t frames, float *logits);

/* ---- src/streaming.rs ---- */
void orc_pool_probs(const orc_cache_cfg *cc, const float *logits, size_t num_mel_frames, const uint8_t *mask,
                    size_t mask_len, float *out);
size_t orc_num_popped(const orc_cache_cfg *cc, size_t num_fifo_frames);
void orc_frame_scores(const orc_cache_cfg *cc, const float *probs, size_t num_frames, float *scores);
void orc_boost_top(const orc_cache_cfg *cc, float *scores, size_t num_frames, size_t k, float boost);
/* picked: cache_len indices (sentinel = ns*(num_frames+n_sil)); returns the sentinel */
size_t orc_compress_picked(const orc_cache_cfg *cc, const float *probs, size_t num_frames, size_t *picked);
void orc_compress(const orc_cache_cfg *cc, size_t hidden, const float *embeds, const float *probs,
                  size_t num_frames, const float *silence, float *out_embeds, float *out_probs);

/* ---- src/model.rs ---- */
int orc_run_offline(const orc_cfg *c, const orc_weights *w, const float *samples, size_t n, orc_run_output *out,
                    orc_step_cb cb, void *user);
/* mode: 0 low, 1 very low, 2 ultra low (src/config.rs:21-27) */
int orc_run_streaming(const orc_cfg *c, const orc_weights *w, const float *samples, size_t n, int mode,
                      orc_run_output *out, orc_step_cb cb, void *user);
void orc_run_output_free(orc_run_output *o);

/* ---- src/segments.rs ---- */
float orc_round2(float v);
void orc_sigmoid_above_half(const float *logits, size_t n, uint8_t *out);
size_t orc_extract_speaker_dict(const float *logits, size_t num_frames, size_t ns, float duration,
                                const uint8_t *mask, float threshold, orc_segment *out, size_t cap);
float orc_activity_stats(const float *logits, size_t num_frames, size_t ns, const uint8_t *mask, float threshold,
                         size_t *per_speaker);

void orc_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
