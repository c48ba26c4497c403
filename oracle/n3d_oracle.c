/*
 * CPU restatement of the reference's Rust CPU path -- TEST INFRASTRUCTURE ONLY
 * (parity checker and timed CPU baseline; never linked into the product).
 *
 * Build with -O3 -ffp-contract=off (no fast-math) so every `a += x * y`
 * stays a separate multiply and add, as Rust emits it.  OpenMP replaces
 * rayon's row-parallel loops; each output's reduction order is the
 * reference's sequential order, so results do not depend on thread count.
 */
#include "n3d_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

#define LN_EPS 1e-5f
#define LOG_ZERO_GUARD 5.9604645e-8f /* 2^-24, src/mel.rs:236-238 */
#define INV_SQRT2_F 0.70710678118654752f
#define LN2_F 0.69314718055994531f

void orc_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}

/* ------------------------------------------------------------ src/tensor.rs */

/* src/tensor.rs:22-57: y = x W^T + b, four outputs at a time, sequential i. */
void orc_linear(const float *x, size_t rows, size_t cols, const float *w, size_t out, const float *bias, float *y) {
#pragma omp parallel for schedule(static)
    for (long r = 0; r < (long)rows; r++) {
        const float *xr = x + (size_t)r * cols;
        float *yr = y + (size_t)r * out;
        size_t o = 0;
        while (o + 4 <= out) {
            const float *w0 = w + o * cols, *w1 = w0 + cols, *w2 = w1 + cols, *w3 = w2 + cols;
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
            for (size_t i = 0; i < cols; i++) {
                float v = xr[i];
                a0 += v * w0[i];
                a1 += v * w1[i];
                a2 += v * w2[i];
                a3 += v * w3[i];
            }
            yr[o] = a0 + (bias ? bias[o] : 0.0f);
            yr[o + 1] = a1 + (bias ? bias[o + 1] : 0.0f);
            yr[o + 2] = a2 + (bias ? bias[o + 2] : 0.0f);
            yr[o + 3] = a3 + (bias ? bias[o + 3] : 0.0f);
            o += 4;
        }
        while (o < out) {
            const float *wr = w + o * cols;
            float acc = 0.0f;
            for (size_t i = 0; i < cols; i++) acc += xr[i] * wr[i];
            yr[o] = acc + (bias ? bias[o] : 0.0f);
            o++;
        }
    }
}

/* src/tensor.rs:60-94 */
void orc_matmul(const float *a, size_t m, size_t k, const float *b, size_t n, float *c) {
#pragma omp parallel for schedule(static)
    for (long r = 0; r < (long)m; r++) {
        const float *ar = a + (size_t)r * k;
        float *cr = c + (size_t)r * n;
        size_t j = 0;
        while (j + 4 <= n) {
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
            for (size_t i = 0; i < k; i++) {
                float v = ar[i];
                a0 += v * b[i * n + j];
                a1 += v * b[i * n + j + 1];
                a2 += v * b[i * n + j + 2];
                a3 += v * b[i * n + j + 3];
            }
            cr[j] = a0;
            cr[j + 1] = a1;
            cr[j + 2] = a2;
            cr[j + 3] = a3;
            j += 4;
        }
        while (j < n) {
            float acc = 0.0f;
            for (size_t i = 0; i < k; i++) acc += ar[i] * b[i * n + j];
            cr[j] = acc;
            j++;
        }
    }
}

/* src/tensor.rs:97-110: two-pass population variance, eps 1e-5. */
void orc_layer_norm(const float *x, size_t rows, size_t cols, const float *w, const float *b, float *y) {
#pragma omp parallel for schedule(static)
    for (long r = 0; r < (long)rows; r++) {
        const float *src = x + (size_t)r * cols;
        float *row = y + (size_t)r * cols;
        float s = 0.0f;
        for (size_t i = 0; i < cols; i++) s += src[i];
        float mean = s / (float)cols;
        float v = 0.0f;
        for (size_t i = 0; i < cols; i++) v += (src[i] - mean) * (src[i] - mean);
        float var = v / (float)cols;
        float inv = 1.0f / sqrtf(var + LN_EPS);
        for (size_t i = 0; i < cols; i++) row[i] = (src[i] - mean) * inv * w[i] + b[i];
    }
}

/* src/tensor.rs:113-120: exact-erf GELU (libm erff). */
void orc_gelu(const float *x, size_t n, float *y) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < (long)n; i++) {
        float v = x[i];
        y[i] = 0.5f * v * (1.0f + erff(v * INV_SQRT2_F));
    }
}

/* src/tensor.rs:123-125 */
void orc_relu(const float *x, size_t n, float *y) {
    for (size_t i = 0; i < n; i++) y[i] = fmaxf(x[i], 0.0f);
}

static void softmax_row(float *row, size_t cols) {
    float mx = -INFINITY;
    for (size_t i = 0; i < cols; i++) mx = fmaxf(mx, row[i]);
    if (!isfinite(mx)) return;
    float sum = 0.0f;
    for (size_t i = 0; i < cols; i++) {
        row[i] = expf(row[i] - mx);
        sum += row[i];
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < cols; i++) row[i] *= inv;
}

/* src/tensor.rs:129-145 */
void orc_softmax_last(float *x, size_t rows, size_t cols) {
#pragma omp parallel for schedule(static)
    for (long r = 0; r < (long)rows; r++) softmax_row(x + (size_t)r * cols, cols);
}

/* --------------------------------------------------------------- src/mel.rs */

/* src/mel.rs:43-48: torch.hann_window(n, periodic=False) in f32. */
void orc_hann_periodic_false(size_t n, float *out) {
    float denom = (float)(n - 1);
    for (size_t i = 0; i < n; i++) {
        float a = 2.0f * 3.14159265358979323846f * (float)i / denom;
        out[i] = 0.5f * (1.0f - cosf(a));
    }
}

static double logstep(void) { return log(6.4) / 27.0; }
static double hz_to_mel(double f) {
    const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
    return f < min_log_hz ? f / f_sp : min_log_mel + log(f / min_log_hz) / logstep();
}
static double mel_to_hz(double m) {
    const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
    return m < min_log_mel ? f_sp * m : min_log_hz * exp(logstep() * (m - min_log_mel));
}

/* src/mel.rs:81-123: librosa slaney filterbank, computed in f64, stored f32. */
void orc_slaney_mel_filterbank(size_t n_mels, size_t n_fft, size_t sample_rate, double f_lo, double f_hi,
                               float *out) {
    size_t nf = n_fft / 2 + 1;
    double *fft_freqs = malloc(nf * sizeof(double));
    double *mel_f = malloc((n_mels + 2) * sizeof(double));
    for (size_t k = 0; k < nf; k++) fft_freqs[k] = (double)k * (double)sample_rate / (double)n_fft;
    double min_mel = hz_to_mel(f_lo), max_mel = hz_to_mel(f_hi);
    for (size_t i = 0; i < n_mels + 2; i++) {
        double t = (double)i / (double)(n_mels + 1);
        mel_f[i] = mel_to_hz(min_mel + t * (max_mel - min_mel));
    }
    for (size_t i = 0; i < n_mels; i++) {
        double enorm = 2.0 / (mel_f[i + 2] - mel_f[i]);
        double lower_den = mel_f[i + 1] - mel_f[i];
        double upper_den = mel_f[i + 2] - mel_f[i + 1];
        for (size_t k = 0; k < nf; k++) {
            double lower = -(mel_f[i] - fft_freqs[k]) / lower_den;
            double upper = (mel_f[i + 2] - fft_freqs[k]) / upper_den;
            double v = fmax(fmin(lower, upper), 0.0);
            out[i * nf + k] = (float)(v * enorm);
        }
    }
    free(fft_freqs);
    free(mel_f);
}

/* src/mel.rs:236-238 */
void orc_mel_filters(const orc_fe *fe, float *out) {
    orc_slaney_mel_filterbank(fe->feature_size, fe->n_fft, fe->sampling_rate, 0.0, (double)fe->sampling_rate / 2.0,
                              out);
}

/* src/mel.rs:143-154 */
size_t orc_frame_count(size_t n_samples, const orc_fe *fe, int centered) {
    if (centered) return n_samples / fe->hop_length;
    if (n_samples < fe->n_fft) return 0;
    return (n_samples - fe->n_fft) / fe->hop_length + 1;
}

/* Twiddle table for an n-point forward FFT: w_k = e^{-2 pi i k / n}, k < n/2,
 * evaluated in double and rounded to float. */
static void fft_twiddles(size_t n, float *twr, float *twi) {
    for (size_t k = 0; k < n / 2; k++) {
        double ang = -2.0 * 3.14159265358979323846 * (double)k / (double)n;
        twr[k] = (float)cos(ang);
        twi[k] = (float)sin(ang);
    }
}

/* In-place iterative radix-2 decimation-in-time FFT (forward).  The butterfly
 * is (a + w b, a - w b) with w b formed as two products and one add/sub per
 * component; the CUDA mel kernel runs this exact sequence. */
static void fft_table(float *re, float *im, size_t n, const float *twr, const float *twi) {
    size_t bits = 0;
    while (((size_t)1 << bits) < n) bits++;
    for (size_t i = 0; i < n; i++) {
        size_t r = 0;
        for (size_t b = 0; b < bits; b++)
            if (i & ((size_t)1 << b)) r |= (size_t)1 << (bits - 1 - b);
        if (r > i) {
            float t = re[i];
            re[i] = re[r];
            re[r] = t;
            t = im[i];
            im[i] = im[r];
            im[r] = t;
        }
    }
    for (size_t len = 2; len <= n; len <<= 1) {
        size_t half = len / 2, step = n / len;
        for (size_t i = 0; i < n; i += len) {
            for (size_t j = 0; j < half; j++) {
                float wr = twr[j * step], wi = twi[j * step];
                float xr = re[i + j + half], xi = im[i + j + half];
                float vr = xr * wr - xi * wi;
                float vi = xr * wi + xi * wr;
                float ur = re[i + j], ui = im[i + j];
                re[i + j] = ur + vr;
                im[i + j] = ui + vi;
                re[i + j + half] = ur - vr;
                im[i + j + half] = ui - vi;
            }
        }
    }
}

void orc_fft(float *re, float *im, size_t n) {
    float *twr = malloc(n / 2 * sizeof(float) + 4), *twi = malloc(n / 2 * sizeof(float) + 4);
    fft_twiddles(n, twr, twi);
    fft_table(re, im, n, twr, twi);
    free(twr);
    free(twi);
}

/* src/mel.rs:160-225: preemphasis -> padding -> window -> FFT -> power -> mel -> ln(x + 2^-24).
 * Returns the frame count; `out` must hold frame_count * feature_size floats. */
size_t orc_log_mel(const float *samples, size_t n, const orc_fe *fe, int centered, const float *filters, float *out) {
    size_t n_fft = fe->n_fft, hop = fe->hop_length, n_mels = fe->feature_size, nf = n_fft / 2 + 1;
    size_t n_frames = orc_frame_count(n, fe, centered);
    if (n_frames == 0) return 0;
    float *emph = malloc((n + n_fft) * sizeof(float));
    size_t off = centered ? n_fft / 2 : 0;
    memset(emph, 0, (n + n_fft) * sizeof(float));
    for (size_t i = 0; i < n; i++) emph[off + i] = samples[i];
    if (fe->preemphasis != 0.0f)
        for (size_t i = n; i-- > 1;) emph[off + i] -= fe->preemphasis * emph[off + i - 1];
    float *win = malloc(fe->win_length * sizeof(float));
    orc_hann_periodic_false(fe->win_length, win);
    float *fw = calloc(n_fft, sizeof(float));
    size_t left = n_fft > fe->win_length ? (n_fft - fe->win_length) / 2 : 0;
    memcpy(fw + left, win, fe->win_length * sizeof(float));
    float *twr = malloc(n_fft / 2 * sizeof(float) + 4), *twi = malloc(n_fft / 2 * sizeof(float) + 4);
    fft_twiddles(n_fft, twr, twi);
#pragma omp parallel
    {
        float *re = malloc(n_fft * sizeof(float)), *im = malloc(n_fft * sizeof(float));
        float *power = malloc(nf * sizeof(float));
#pragma omp for schedule(static)
        for (long t = 0; t < (long)n_frames; t++) {
            size_t start = (size_t)t * hop;
            for (size_t j = 0; j < n_fft; j++) {
                re[j] = emph[start + j] * fw[j];
                im[j] = 0.0f;
            }
            fft_table(re, im, n_fft, twr, twi);
            for (size_t k = 0; k < nf; k++) power[k] = re[k] * re[k] + im[k] * im[k];
            float *row = out + (size_t)t * n_mels;
            for (size_t m = 0; m < n_mels; m++) {
                float acc = 0.0f;
                for (size_t k = 0; k < nf; k++) acc += filters[m * nf + k] * power[k];
                row[m] = acc;
            }
        }
        free(re);
        free(im);
        free(power);
    }
    for (size_t i = 0; i < n_frames * n_mels; i++) out[i] = logf(out[i] + LOG_ZERO_GUARD);
    free(emph);
    free(win);
    free(fw);
    free(twr);
    free(twi);
    return n_frames;
}

/* ----------------------------------------------------------- src/encoder.rs */

/* src/encoder.rs:163-185: inv_freq in f64 -> f32, angle pos*inv in f32. */
void orc_rope_tables(size_t seq, size_t hd, double theta, size_t offset, float *cos_out, float *sin_out) {
    size_t half = hd / 2;
    float *inv = malloc(half * sizeof(float));
    for (size_t i = 0; i < half; i++) inv[i] = (float)(1.0 / pow(theta, 2.0 * (double)i / (double)hd));
    for (size_t p = 0; p < seq; p++) {
        float pos = (float)(offset + p);
        for (size_t i = 0; i < half; i++) {
            float a = pos * inv[i];
            cos_out[p * hd + i] = cosf(a);
            sin_out[p * hd + i] = sinf(a);
            cos_out[p * hd + half + i] = cos_out[p * hd + i];
            sin_out[p * hd + half + i] = sin_out[p * hd + i];
        }
    }
    free(inv);
}

/* src/encoder.rs:281-296: rotate-half RoPE on every head, in place. */
void orc_apply_rope(float *x, size_t seq, size_t nh, size_t hd, const float *cos_t, const float *sin_t) {
    size_t half = hd / 2;
#pragma omp parallel for schedule(static)
    for (long row = 0; row < (long)(seq * nh); row++) {
        float *head = x + (size_t)row * hd;
        size_t p = (size_t)row / nh;
        const float *c = cos_t + p * hd, *s = sin_t + p * hd;
        for (size_t i = 0; i < half; i++) {
            float x1 = head[i], x2 = head[half + i];
            head[i] = x1 * c[i] - x2 * s[i];
            head[half + i] = x2 * c[half + i] + x1 * s[half + i];
        }
    }
}

/* src/encoder.rs:302-329: softmax attention over the first `valid` keys. */
void orc_attention(const float *q, const float *k, const float *v, size_t seq, size_t nh, size_t hd, size_t valid,
                   float *out) {
    float scaling = 1.0f / sqrtf((float)hd);
#pragma omp parallel
    {
        float *scores = malloc((valid ? valid : 1) * sizeof(float));
#pragma omp for schedule(static)
        for (long qi = 0; qi < (long)seq; qi++) {
            float *orow = out + (size_t)qi * nh * hd;
            for (size_t head = 0; head < nh; head++) {
                size_t qb = ((size_t)qi * nh + head) * hd;
                for (size_t j = 0; j < valid; j++) {
                    size_t kb = (j * nh + head) * hd;
                    float acc = 0.0f;
                    for (size_t d = 0; d < hd; d++) acc += q[qb + d] * k[kb + d];
                    scores[j] = acc * scaling;
                }
                softmax_row(scores, valid);
                size_t ob = head * hd;
                for (size_t d = 0; d < hd; d++) {
                    float acc = 0.0f;
                    for (size_t j = 0; j < valid; j++) acc += scores[j] * v[(j * nh + head) * hd + d];
                    orow[ob + d] = acc;
                }
            }
        }
        free(scores);
    }
}

/* src/encoder.rs:126-146: groups lo..hi of 8 stacked mel frames, zero past num_frames. */
void orc_embed_range(const orc_cfg *c, const orc_weights *w, const float *mel, size_t num_frames, size_t lo,
                     size_t hi, float *out) {
    size_t sub = c->sub, mels = c->n_mels, h = c->hidden, groups = hi - lo;
    size_t end_mel = hi * sub < num_frames ? hi * sub : num_frames;
    float *buf = calloc(groups * sub * mels + 1, sizeof(float));
    if (lo * sub < end_mel) memcpy(buf, mel + lo * sub * mels, (end_mel - lo * sub) * mels * sizeof(float));
    orc_linear(buf, groups, sub * mels, w->embed_proj, h, NULL, out);
    free(buf);
}

/* src/encoder.rs:236-278: one pre-LN block, x updated in place. */
static void block(const orc_cfg *c, const orc_weights *w, size_t li, float *x, size_t seq, size_t valid,
                  const float *cos_t, const float *sin_t) {
    size_t h = c->hidden, nh = c->heads, hd = h / nh, inter = c->inter;
    float *n1 = malloc(seq * h * sizeof(float) + 4);
    float *q = malloc(seq * h * sizeof(float) + 4);
    float *k = malloc(seq * h * sizeof(float) + 4);
    float *v = malloc(seq * h * sizeof(float) + 4);
    float *ctx = malloc(seq * h * sizeof(float) + 4);
    float *attn_out = malloc(seq * h * sizeof(float) + 4);
    orc_layer_norm(x, seq, h, w->ln1_w[li], w->ln1_b[li], n1);
    orc_linear(n1, seq, h, w->q[li], h, NULL, q);
    orc_linear(n1, seq, h, w->k[li], h, NULL, k);
    orc_linear(n1, seq, h, w->v[li], h, NULL, v);
    orc_apply_rope(q, seq, nh, hd, cos_t, sin_t);
    orc_apply_rope(k, seq, nh, hd, cos_t, sin_t);
    orc_attention(q, k, v, seq, nh, hd, valid, ctx);
    orc_linear(ctx, seq, h, w->o[li], h, w->o_b[li], attn_out);
    for (size_t i = 0; i < seq * h; i++) x[i] += attn_out[i];
    float *ff = malloc(seq * inter * sizeof(float) + 4);
    orc_layer_norm(x, seq, h, w->ln2_w[li], w->ln2_b[li], n1);
    orc_linear(n1, seq, h, w->fc1[li], inter, w->fc1_b[li], ff);
    orc_gelu(ff, seq * inter, ff);
    orc_linear(ff, seq, inter, w->fc2[li], h, w->fc2_b[li], attn_out);
    for (size_t i = 0; i < seq * h; i++) x[i] += attn_out[i];
    free(n1);
    free(q);
    free(k);
    free(v);
    free(ctx);
    free(attn_out);
    free(ff);
}

/* src/encoder.rs:209-235: input LN, 31 blocks, final LN; positions 0..groups-1. */
void orc_forward_embeds(const orc_cfg *c, const orc_weights *w, const float *embeds, size_t groups, size_t valid,
                        float *out) {
    size_t h = c->hidden, hd = h / c->heads;
    if (valid > groups) valid = groups;
    float *x = malloc(groups * h * sizeof(float) + 4);
    float *cs = malloc(groups * hd * sizeof(float) + 4), *sn = malloc(groups * hd * sizeof(float) + 4);
    orc_layer_norm(embeds, groups, h, w->in_ln_w, w->in_ln_b, x);
    orc_rope_tables(groups, hd, c->rope_theta, 0, cs, sn);
    for (size_t li = 0; li < c->layers; li++) block(c, w, li, x, groups, valid, cs, sn);
    orc_layer_norm(x, groups, h, w->fin_ln_w, w->fin_ln_b, out);
    free(x);
    free(cs);
    free(sn);
}

/* -------------------------------------------------------------- src/head.rs */

/* src/head.rs:92-127: Conv1d(k=3, pad=1) then the sub-pixel reshape (a no-op on row-major memory). */
static void upsample(const orc_cfg *c, const orc_weights *w, const float *input, size_t frames, float *out) {
    size_t hh = c->head_hidden, up = c->sub, out_c = hh * up;
    float *pad = calloc((frames + 2) * hh, sizeof(float));
    memcpy(pad + hh, input, frames * hh * sizeof(float));
#pragma omp parallel for schedule(static)
    for (long t = 0; t < (long)frames; t++) {
        size_t p0 = (size_t)t * hh, p1 = ((size_t)t + 1) * hh, p2 = ((size_t)t + 2) * hh;
        float *orow = out + (size_t)t * out_c;
        for (size_t oc = 0; oc < out_c; oc++) {
            const float *wr = w->conv_w + oc * hh * 3;
            float acc = w->conv_b[oc];
            for (size_t ic = 0; ic < hh; ic++)
                acc += wr[ic * 3] * pad[p0 + ic] + wr[ic * 3 + 1] * pad[p1 + ic] + wr[ic * 3 + 2] * pad[p2 + ic];
            orow[oc] = acc;
        }
    }
    free(pad);
}

/* src/head.rs:147-157: proj -> upsample -> relu -> dense -> relu -> out_proj. */
void orc_head_forward(const orc_cfg *c, const orc_weights *w, const float *enc, size_t frames, float *logits) {
    size_t hh = c->head_hidden, up = c->sub, ns = c->num_speakers, upf = frames * up;
    float *proj = malloc(frames * hh * sizeof(float) + 4);
    float *u = malloc(upf * hh * sizeof(float) + 4);
    float *d = malloc(upf * hh * sizeof(float) + 4);
    orc_linear(enc, frames, c->hidden, w->proj_w, hh, w->proj_b, proj);
    upsample(c, w, proj, frames, u);
    orc_relu(u, upf * hh, u);
    orc_linear(u, upf, hh, w->dense_w, hh, w->dense_b, d);
    orc_relu(d, upf * hh, d);
    orc_linear(d, upf, hh, w->out_w, ns, w->out_b, logits);
    free(proj);
    free(u);
    free(d);
}

/* --------------------------------------------------------- src/streaming.rs */

/* src/streaming.rs:202-217 */
void orc_pool_probs(const orc_cache_cfg *cc, const float *logits, size_t num_mel_frames, const uint8_t *mask,
                    size_t mask_len, float *out) {
    size_t sub = cc->subsampling_factor, ns = cc->num_speakers, groups = num_mel_frames / sub;
    for (size_t g = 0; g < groups; g++) {
        int keep = g < mask_len ? mask[g] != 0 : 0;
        for (size_t c = 0; c < ns; c++) {
            float acc = 0.0f;
            for (size_t k = 0; k < sub; k++) acc += 1.0f / (1.0f + expf(-logits[(g * sub + k) * ns + c]));
            out[g * ns + c] = keep ? acc / (float)sub : 0.0f;
        }
    }
}

/* src/streaming.rs:220-228 */
size_t orc_num_popped(const orc_cache_cfg *cc, size_t n) {
    if (n <= cc->fifo_length) return 0;
    size_t over = n - cc->fifo_length;
    size_t p = cc->update_period > over ? cc->update_period : over;
    return p < n ? p : n;
}

/* src/streaming.rs:294-330 */
void orc_frame_scores(const orc_cache_cfg *cc, const float *probs, size_t nfr, float *scores) {
    size_t ns = cc->num_speakers;
    float thr = cc->score_threshold;
    float lp[64], lc[64];
    for (size_t f = 0; f < nfr; f++) {
        const float *row = probs + f * ns;
        float sum_lc = 0.0f;
        for (size_t s = 0; s < ns; s++) {
            lp[s] = logf(fmaxf(row[s], thr));
            lc[s] = logf(fmaxf(1.0f - row[s], thr));
        }
        for (size_t s = 0; s < ns; s++) sum_lc += lc[s];
        for (size_t s = 0; s < ns; s++) {
            float v = lp[s] - lc[s] + sum_lc + LN2_F;
            scores[f * ns + s] = row[s] > 0.5f ? v : -INFINITY;
        }
    }
    for (size_t s = 0; s < ns; s++) {
        size_t pos = 0;
        for (size_t f = 0; f < nfr; f++)
            if (scores[f * ns + s] > 0.0f) pos++;
        if (pos >= cc->min_positive_scores)
            for (size_t f = 0; f < nfr; f++) {
                size_t i = f * ns + s;
                if (scores[i] <= 0.0f && probs[i] > 0.5f) scores[i] = -INFINITY;
            }
    }
}

/* Rust's `partial_cmp(..).unwrap_or(Equal)`, descending: a goes first iff key[a] > key[b]. */
static int desc_before(float a, float b) { return a > b; }

/* Stable merge sort of idx[0..n) by descending key (the `sort_by` of src/streaming.rs:337-341, 452-453). */
static void stable_sort_desc(size_t *idx, size_t n, const float *key, size_t key_stride, size_t *tmp) {
    for (size_t width = 1; width < n; width *= 2) {
        for (size_t lo = 0; lo < n; lo += 2 * width) {
            size_t mid = lo + width < n ? lo + width : n, hi = lo + 2 * width < n ? lo + 2 * width : n;
            size_t i = lo, j = mid, o = lo;
            while (i < mid && j < hi) {
                if (desc_before(key[idx[j] * key_stride], key[idx[i] * key_stride]))
                    tmp[o++] = idx[j++];
                else
                    tmp[o++] = idx[i++];
            }
            while (i < mid) tmp[o++] = idx[i++];
            while (j < hi) tmp[o++] = idx[j++];
        }
        memcpy(idx, tmp, n * sizeof(size_t));
    }
}

/* src/streaming.rs:333-346: per-speaker boost of the k best frames. */
void orc_boost_top(const orc_cache_cfg *cc, float *scores, size_t nfr, size_t k, float boost) {
    size_t ns = cc->num_speakers;
    size_t *idx = malloc((nfr + 1) * sizeof(size_t)), *tmp = malloc((nfr + 1) * sizeof(size_t));
    for (size_t s = 0; s < ns; s++) {
        for (size_t f = 0; f < nfr; f++) idx[f] = f;
        stable_sort_desc(idx, nfr, scores + s, ns, tmp);
        size_t kk = k < nfr ? k : nfr;
        for (size_t i = 0; i < kk; i++) scores[idx[i] * ns + s] += boost;
    }
    free(idx);
    free(tmp);
}

static int cmp_size(const void *a, const void *b) {
    size_t x = *(const size_t *)a, y = *(const size_t *)b;
    return x < y ? -1 : x > y;
}

/* src/streaming.rs:410-462: scores, boosts, flat speaker-major ranking, sentinel remap, sorted picks. */
size_t orc_compress_picked(const orc_cache_cfg *cc, const float *probs, size_t nfr, size_t *picked) {
    size_t ns = cc->num_speakers, cache_len = cc->speaker_cache_length, n_sil = cc->num_silence_frames;
    float *scores = malloc((nfr * ns + 1) * sizeof(float));
    orc_frame_scores(cc, probs, nfr, scores);
    for (size_t f = cache_len; f < nfr; f++)
        for (size_t s = 0; s < ns; s++) scores[f * ns + s] += cc->latest_frames_score_boost;
    orc_boost_top(cc, scores, nfr, cc->num_strong_boosted_frames, 2.0f * LN2_F);
    orc_boost_top(cc, scores, nfr, cc->num_weak_boosted_frames, LN2_F);
    size_t num_scored = nfr + n_sil, total = ns * num_scored;
    float *flat = malloc(total * sizeof(float));
    for (size_t s = 0; s < ns; s++) {
        for (size_t f = 0; f < nfr; f++) flat[s * num_scored + f] = scores[f * ns + s];
        for (size_t k = 0; k < n_sil; k++) flat[s * num_scored + nfr + k] = INFINITY;
    }
    size_t sentinel = total;
    size_t *idx = malloc(total * sizeof(size_t)), *tmp = malloc(total * sizeof(size_t));
    for (size_t i = 0; i < total; i++) idx[i] = i;
    stable_sort_desc(idx, total, flat, 1, tmp);
    size_t kept = cache_len < total ? cache_len : total;
    for (size_t i = 0; i < kept; i++) picked[i] = flat[idx[i]] == -INFINITY ? sentinel : idx[i];
    qsort(picked, kept, sizeof(size_t), cmp_size);
    free(scores);
    free(flat);
    free(idx);
    free(tmp);
    return sentinel;
}

/* src/streaming.rs:464-481: gather the picks; silence slots get silence_embeds and zero probs. */
void orc_compress(const orc_cache_cfg *cc, size_t hidden, const float *embeds, const float *probs, size_t nfr,
                  const float *silence, float *oe, float *op) {
    size_t ns = cc->num_speakers, cache_len = cc->speaker_cache_length, num_scored = nfr + cc->num_silence_frames;
    size_t *picked = malloc(cache_len * sizeof(size_t));
    size_t sentinel = orc_compress_picked(cc, probs, nfr, picked);
    for (size_t i = 0; i < cache_len; i++) {
        size_t idx = picked[i];
        size_t frame = idx == sentinel ? nfr : (idx % num_scored < nfr ? idx % num_scored : nfr);
        if (frame == nfr) {
            memcpy(oe + i * hidden, silence, hidden * sizeof(float));
            memset(op + i * ns, 0, ns * sizeof(float));
        } else {
            memcpy(oe + i * hidden, embeds + frame * hidden, hidden * sizeof(float));
            memcpy(op + i * ns, probs + frame * ns, ns * sizeof(float));
        }
    }
    free(picked);
}

/* SpeakerCache state, src/streaming.rs:130-143. */
typedef struct {
    orc_cache_cfg cfg;
    size_t hidden, cache_frames, fifo_frames;
    float *embeds, *probs, *fifo;
    int is_compressed;
} cache_t;

static void cache_init(cache_t *c, const orc_cache_cfg *cfg, size_t hidden) {
    memset(c, 0, sizeof(*c));
    c->cfg = *cfg;
    c->hidden = hidden;
}
static void cache_free(cache_t *c) {
    free(c->embeds);
    free(c->probs);
    free(c->fifo);
}

/* src/streaming.rs:236-284 */
static void cache_update(cache_t *c, const float *window, size_t frames, const float *logits, const float *silence,
                         size_t n_chunk, const uint8_t *mask) {
    size_t ns = c->cfg.num_speakers, hidden = c->hidden;
    float *probs = malloc((frames * ns + 1) * sizeof(float));
    orc_pool_probs(&c->cfg, logits, frames * c->cfg.subsampling_factor, mask, frames, probs);
    size_t ncache = c->cache_frames, chunk_start = c->cache_frames + c->fifo_frames;
    size_t nfifo = c->fifo_frames + n_chunk;
    float *fifo = malloc((nfifo * hidden + 1) * sizeof(float));
    if (c->fifo_frames) memcpy(fifo, c->fifo, c->fifo_frames * hidden * sizeof(float));
    memcpy(fifo + c->fifo_frames * hidden, window + chunk_start * hidden, n_chunk * hidden * sizeof(float));
    size_t popped = orc_num_popped(&c->cfg, nfifo);
    if (popped > 0) {
        const float *fifo_probs = probs + ncache * ns;
        size_t ne = ncache + popped;
        float *ce = malloc((ne * hidden + 1) * sizeof(float)), *cp = malloc((ne * ns + 1) * sizeof(float));
        if (ncache) memcpy(ce, c->embeds, ncache * hidden * sizeof(float));
        memcpy(ce + ncache * hidden, fifo, popped * hidden * sizeof(float));
        if (ncache) memcpy(cp, c->is_compressed ? c->probs : probs, ncache * ns * sizeof(float));
        memcpy(cp + ncache * ns, fifo_probs, popped * ns * sizeof(float));
        memmove(fifo, fifo + popped * hidden, (nfifo - popped) * hidden * sizeof(float));
        nfifo -= popped;
        if (ne > c->cfg.speaker_cache_length) {
            size_t L = c->cfg.speaker_cache_length;
            float *oe = malloc(L * hidden * sizeof(float)), *op = malloc(L * ns * sizeof(float));
            orc_compress(&c->cfg, hidden, ce, cp, ne, silence, oe, op);
            free(ce);
            free(cp);
            ce = oe;
            cp = op;
            ne = L;
            c->is_compressed = 1;
        }
        free(c->embeds);
        free(c->probs);
        c->embeds = ce;
        c->probs = cp;
        c->cache_frames = ne;
    }
    free(c->fifo);
    c->fifo = fifo;
    c->fifo_frames = nfifo;
    free(probs);
}

/* -------------------------------------------------------------- src/model.rs */

typedef struct {
    float *data;
    size_t len, cap;
} fvec;
static void fvec_push(fvec *v, const float *src, size_t n) {
    if (v->len + n > v->cap) {
        size_t nc = v->cap ? v->cap * 2 : 4096;
        while (nc < v->len + n) nc *= 2;
        v->data = realloc(v->data, nc * sizeof(float));
        v->cap = nc;
    }
    memcpy(v->data + v->len, src, n * sizeof(float));
    v->len += n;
}

/* src/model.rs:371-475: window = prefix ++ embeds, forward, cache update, scored slice. */
static void step(const orc_cfg *c, const orc_weights *w, cache_t *cache, const float *embeds, size_t groups,
                 const uint8_t *mask, size_t n_chunk, size_t cap, fvec *logits, size_t step_idx, orc_step_cb cb,
                 void *user) {
    size_t sub = c->sub, ns = c->num_speakers, h = c->hidden;
    size_t cached = cache->cache_frames + cache->fifo_frames, frames = cached + groups;
    float *window = malloc((frames * h + 1) * sizeof(float));
    if (cache->cache_frames) memcpy(window, cache->embeds, cache->cache_frames * h * sizeof(float));
    if (cache->fifo_frames)
        memcpy(window + cache->cache_frames * h, cache->fifo, cache->fifo_frames * h * sizeof(float));
    memcpy(window + cached * h, embeds, groups * h * sizeof(float));
    uint8_t *step_mask = malloc(frames + 1);
    memset(step_mask, 1, cached);
    memcpy(step_mask + cached, mask, groups);
    size_t valid = 0;
    for (size_t i = 0; i < frames; i++) valid += step_mask[i] != 0;
    float *enc = malloc((frames * h + 1) * sizeof(float));
    float *sl = malloc((frames * sub * ns + 1) * sizeof(float));
    orc_forward_embeds(c, w, window, frames, valid, enc);
    orc_head_forward(c, w, enc, frames, sl);
    cache_update(cache, window, frames, sl, w->silence, n_chunk, step_mask);
    if (cb) {
        orc_step_trace t = {step_idx, cached, frames, valid, n_chunk, window, enc, sl, cache->embeds, cache->probs,
                            cache->fifo, cache->cache_frames, cache->fifo_frames, cache->is_compressed};
        cb(user, &t);
    }
    size_t s = cached * sub, e = (cached + n_chunk) * sub;
    size_t keep = (e - s) < cap ? (e - s) : cap;
    fvec_push(logits, sl + s * ns, keep * ns);
    free(window);
    free(step_mask);
    free(enc);
    free(sl);
}

static void finish(const orc_cfg *c, cache_t *cache, fvec *logits, size_t num_chunks, orc_run_output *out) {
    out->logits = logits->data;
    out->num_frames = logits->len / c->num_speakers;
    out->num_chunks = num_chunks;
    out->cache_compressed = cache->is_compressed;
    out->cache_frames = cache->cache_frames;
    out->fifo_frames = cache->fifo_frames;
}

/* src/model.rs:242-310 with the Offline arm of chunk_loop, src/model.rs:485-503. */
int orc_run_offline(const orc_cfg *c, const orc_weights *w, const float *samples, size_t n, orc_run_output *out,
                    orc_step_cb cb, void *user) {
    size_t sub = c->sub, mels = c->n_mels, h = c->hidden, ns = c->num_speakers;
    size_t valid = orc_frame_count(n, &c->fe, 1);
    float *mel = calloc((valid + 1) * mels + 1, sizeof(float));
    if (valid) orc_log_mel(samples, n, &c->fe, 1, w->mel_filters, mel);
    size_t groups = (valid + 1 + sub - 1) / sub;
    cache_t cache;
    cache_init(&cache, &c->cache_offline, h);
    fvec logits = {0};
    size_t num_chunks = 0;
    for (size_t start = 0; start < groups; start += c->chunk_length) {
        size_t end = start + c->chunk_length < groups ? start + c->chunk_length : groups;
        size_t hi = end + c->chunk_right_context < groups ? end + c->chunk_right_context : groups;
        size_t g = hi - start;
        float *emb = malloc((g * h + 1) * sizeof(float));
        orc_embed_range(c, w, mel, valid + 1, start, hi, emb);
        uint8_t *mask = malloc(g + 1);
        for (size_t i = 0; i < g; i++) mask[i] = (start + i) * sub < valid;
        step(c, w, &cache, emb, g, mask, end - start, (size_t)-1, &logits, num_chunks, cb, user);
        num_chunks++;
        free(emb);
        free(mask);
    }
    size_t total = (valid + 1) * ns;
    if (logits.len > total) logits.len = total;
    finish(c, &cache, &logits, num_chunks, out);
    cache_free(&cache);
    free(mel);
    return 0;
}

/* ModeParams::resolve, src/config.rs:152-193 (streaming modes only). */
typedef struct {
    size_t mel_per_chunk, mel_per_step, lookahead, first_chunk_samples, samples_per_chunk;
} mode_params;
static mode_params resolve(const orc_cfg *c, int mode) {
    mode_params p;
    size_t cl = c->modes[mode][0], rc = c->modes[mode][1];
    p.mel_per_chunk = (cl + rc) * c->sub;
    p.mel_per_step = cl * c->sub;
    p.lookahead = rc;
    p.first_chunk_samples = (p.mel_per_chunk - 1) * c->fe.hop_length + c->fe.win_length / 2;
    p.samples_per_chunk = p.mel_per_chunk * c->fe.hop_length + c->fe.win_length;
    return p;
}

/* src/model.rs:313-365 with the Streaming arm of chunk_loop, src/model.rs:504-510.
 * Returns -1 (the reference would panic) when a chunk holds fewer encoder frames than its look-ahead. */
int orc_run_streaming(const orc_cfg *c, const orc_weights *w, const float *samples, size_t n, int mode,
                      orc_run_output *out, orc_step_cb cb, void *user) {
    size_t sub = c->sub, mels = c->n_mels, h = c->hidden;
    mode_params mp = resolve(c, mode);
    /* chunk list: (offset, len, centered, lookahead) */
    size_t cap_chunks = 16 + n / (mp.mel_per_step * c->fe.hop_length + 1) + 2;
    size_t *c_off = malloc(cap_chunks * sizeof(size_t)), *c_len = malloc(cap_chunks * sizeof(size_t));
    int *c_cent = malloc(cap_chunks * sizeof(int));
    size_t *c_la = malloc(cap_chunks * sizeof(size_t));
    size_t nc = 0;
    c_off[nc] = 0;
    c_len[nc] = mp.first_chunk_samples < n ? mp.first_chunk_samples : n;
    c_cent[nc] = 1;
    c_la[nc++] = mp.lookahead;
    size_t mel_idx = mp.mel_per_step;
    size_t start = mel_idx * c->fe.hop_length - c->fe.n_fft / 2;
    while (start + mp.samples_per_chunk <= n) {
        c_off[nc] = start;
        c_len[nc] = mp.samples_per_chunk;
        c_cent[nc] = 0;
        c_la[nc++] = mp.lookahead;
        mel_idx += mp.mel_per_step;
        start = mel_idx * c->fe.hop_length - c->fe.n_fft / 2;
    }
    size_t ls = start < n ? start : n;
    c_off[nc] = ls;
    c_len[nc] = n - ls;
    c_cent[nc] = 1;
    c_la[nc++] = 0;

    cache_t cache;
    cache_init(&cache, &c->cache_stream, h);
    fvec logits = {0};
    int rc = 0;
    size_t steps = 0;
    for (size_t i = 0; i < nc; i++) {
        size_t nm = orc_frame_count(c_len[i], &c->fe, c_cent[i]);
        float *mel = calloc(nm * mels + 1, sizeof(float));
        if (nm) orc_log_mel(samples + c_off[i], c_len[i], &c->fe, c_cent[i], w->mel_filters, mel);
        size_t groups = (nm + sub - 1) / sub;
        if (groups < c_la[i]) {
            free(mel);
            rc = -1;
            break;
        }
        float *emb = malloc((groups * h + 1) * sizeof(float));
        orc_embed_range(c, w, mel, nm, 0, groups, emb);
        uint8_t *mask = malloc(groups + 1);
        memset(mask, 1, groups);
        step(c, w, &cache, emb, groups, mask, groups - c_la[i], nm, &logits, steps, cb, user);
        steps++;
        free(emb);
        free(mask);
        free(mel);
    }
    finish(c, &cache, &logits, steps, out);
    cache_free(&cache);
    free(c_off);
    free(c_len);
    free(c_cent);
    free(c_la);
    return rc;
}

void orc_run_output_free(orc_run_output *o) {
    free(o->logits);
    o->logits = NULL;
}

/* ----------------------------------------------------------- src/segments.rs */

/* src/segments.rs:51-62: Python round(x, 2), half to even on the f64 scale. */
float orc_round2(float v) {
    double scaled = (double)v * 100.0;
    double r = round(scaled);
    if (fabs(scaled - trunc(scaled)) == 0.5) {
        double t = trunc(scaled);
        r = ((long long)t % 2 == 0) ? t : t + 1.0;
    }
    return (float)(r / 100.0);
}

static float sigmoidf(float x) { return 1.0f / (1.0f + expf(-x)); }

/* frame_check's decision per logit (src/bin/frame_check.rs:188-190): the f32 sigmoid
 * above 0.5, with the same f32 exp the segments use, so that a counted flip and a
 * changed segment come from the same arithmetic. */
void orc_sigmoid_above_half(const float *logits, size_t n, uint8_t *out) {
    for (size_t i = 0; i < n; i++) out[i] = sigmoidf(logits[i]) > 0.5f;
}

static int seg_cmp(const void *a, const void *b) {
    const orc_segment *x = a, *y = b;
    if (x->start < y->start) return -1;
    if (x->start > y->start) return 1;
    return x->speaker < y->speaker ? -1 : x->speaker > y->speaker;
}

/* src/segments.rs:70-109.  Writes at most `cap` segments; returns the total count. */
size_t orc_extract_speaker_dict(const float *logits, size_t nfr, size_t ns, float duration, const uint8_t *mask,
                                float threshold, orc_segment *out, size_t cap) {
    size_t cnt = 0, alloc = 64;
    orc_segment *segs = malloc(alloc * sizeof(orc_segment));
    for (size_t s = 0; s < ns; s++) {
        long start = -1;
        for (size_t t = 0; t <= nfr; t++) {
            int active = t < nfr && sigmoidf(logits[t * ns + s]) > threshold && (!mask || mask[t]);
            if (active && start < 0)
                start = (long)t;
            else if (!active && start >= 0) {
                if (cnt == alloc) {
                    alloc *= 2;
                    segs = realloc(segs, alloc * sizeof(orc_segment));
                }
                segs[cnt].start = orc_round2((float)start * duration);
                segs[cnt].end = orc_round2((float)t * duration);
                segs[cnt].speaker = s;
                cnt++;
                start = -1;
            }
        }
    }
    qsort(segs, cnt, sizeof(orc_segment), seg_cmp);
    for (size_t i = 0; i < cnt && i < cap; i++) out[i] = segs[i];
    free(segs);
    return cnt;
}

/* src/segments.rs:113-141 */
float orc_activity_stats(const float *logits, size_t nfr, size_t ns, const uint8_t *mask, float threshold,
                         size_t *per_speaker) {
    size_t any = 0, total = 0;
    for (size_t s = 0; s < ns; s++) per_speaker[s] = 0;
    for (size_t t = 0; t < nfr; t++) {
        if (mask && !mask[t]) continue;
        total++;
        int hot = 0;
        for (size_t s = 0; s < ns; s++)
            if (sigmoidf(logits[t * ns + s]) > threshold) {
                per_speaker[s]++;
                hot = 1;
            }
        any += hot;
    }
    return total == 0 ? 0.0f : (float)any * 100.0f / (float)total;
}
