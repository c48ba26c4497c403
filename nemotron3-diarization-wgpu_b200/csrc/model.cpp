// Host runtime of the diarization path: config and checkpoint loading, weight
// upload, the data-independent chunk schedule, and the batched chunk loop.
//
// Mirrors the reference's `Model` (src/model.rs) and `GpuEngine`
// (src/gpu_engine.rs:238-532) but keeps the whole step on the device: mel,
// embedder, window assembly, tower, head and speaker cache run as kernels on
// one stream, and the host only ships audio in and logits out.

#include "model.h"

#include <memory>
#include <algorithm>
#include <array>
#include <climits>
#include <thread>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>

#include "json.h"
#include "safetensors.h"

namespace n3d {

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw Error(10 /*N3D_ERR_CUDA*/, std::string(what) + ": " + cudaGetErrorString(e));
}

namespace {

// n3d_status codes (include/n3d.h); the checkpoint reader's own are in safetensors.h
constexpr int kStatusIo = 1, kStatusJson = 2, kStatusShape = 6, kStatusAudio = 7, kStatusGpu = 9, kStatusTimeout = 11,
              kStatusNoDevice = 12, kStatusArg = 13, kStatusCuda = 10;

std::string read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw Error(kStatusIo, "io error at " + path + ": cannot open");
    std::ostringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

const json::Value& need(const json::Value& v, const char* key, const std::string& file) {
    const json::Value* p = v.get(key);
    if (!p) throw Error(kStatusJson, "failed to parse " + file + ": missing field `" + key + "`");
    return *p;
}
// A count: an integer of at least `lo` (the reference reads these fields as usize, so
// negative, fractional and non-numeric values are errors there too).  Fields that the
// schedule divides by or steps with pass lo = 1.
int count_value(const json::Value& x, const char* key, const std::string& f, int lo) {
    if (x.kind != json::Value::Num || x.num != std::floor(x.num) || x.num < lo || x.num > (double)(1 << 24))
        throw Error(kStatusJson, "failed to parse " + f + ": `" + key + "` must be an integer of at least " +
                                     std::to_string(lo));
    return (int)x.num;
}
int need_int(const json::Value& v, const char* key, const std::string& f, int lo = 1) {
    return count_value(need(v, key, f), key, f, lo);
}
double need_num(const json::Value& v, const char* key, const std::string& f) {
    const json::Value& x = need(v, key, f);
    if (x.kind != json::Value::Num) throw Error(kStatusJson, "failed to parse " + f + ": `" + key + "` must be a number");
    return x.num;
}

// Magnitude bounds for the fp16-split scales (see DevLayer).
double absmax_host(const float* p, size_t n) {
    double m = 0.0;
    for (size_t i = 0; i < n; i++) m = std::max(m, (double)std::fabs(p[i]));
    return m;
}
// Largest row L1 norm of w [out, in].
double row_l1_max(const float* w, long long out, long long in) {
    double m = 0.0;
    for (long long o = 0; o < out; o++) {
        double a = 0.0;
        for (long long i = 0; i < in; i++) a += std::fabs(w[o * in + i]);
        m = std::max(m, a);
    }
    return m;
}
// |LayerNorm(x)| <= sqrt(cols - 1) max|w| + max|b|: a normalised element is at most
// sqrt(cols - 1) standard deviations from the mean (population variance).
double ln_bound(const float* w, const float* b, long long cols) {
    return std::sqrt((double)(cols - 1)) * absmax_host(w, cols) + absmax_host(b, cols);
}
// |y| <= max over rows of (L1(w_row) * bound + |b|) for y = x w^T + b, |x| <= bound.
double linear_bound(const float* w, const float* b, long long out, long long in, double bound) {
    double m = 0.0;
    for (long long o = 0; o < out; o++) {
        double a = 0.0;
        for (long long i = 0; i < in; i++) a += std::fabs(w[o * in + i]);
        m = std::max(m, a * bound + (b ? std::fabs(b[o]) : 0.0));
    }
    return m;
}

// ------------------------------------------------------------- mel constants
// librosa slaney filterbank (src/mel.rs:81-123), f64 math stored as f32.
double logstep() { return std::log(6.4) / 27.0; }
double hz_to_mel(double f) {
    const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
    return f < min_log_hz ? f / f_sp : min_log_mel + std::log(f / min_log_hz) / logstep();
}
double mel_to_hz(double m) {
    const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp;
    return m < min_log_mel ? f_sp * m : min_log_hz * std::exp(logstep() * (m - min_log_mel));
}
std::vector<float> slaney(int n_mels, int n_fft, int sr, double fmin, double fmax) {
    const int nf = n_fft / 2 + 1;
    std::vector<double> freqs(nf), mel_f(n_mels + 2);
    for (int k = 0; k < nf; k++) freqs[k] = (double)k * (double)sr / (double)n_fft;
    const double lo = hz_to_mel(fmin), hi = hz_to_mel(fmax);
    for (int i = 0; i < n_mels + 2; i++) mel_f[i] = mel_to_hz(lo + ((double)i / (double)(n_mels + 1)) * (hi - lo));
    std::vector<float> w((size_t)n_mels * nf);
    for (int i = 0; i < n_mels; i++) {
        const double enorm = 2.0 / (mel_f[i + 2] - mel_f[i]);
        for (int k = 0; k < nf; k++) {
            const double lower = -(mel_f[i] - freqs[k]) / (mel_f[i + 1] - mel_f[i]);
            const double upper = (mel_f[i + 2] - freqs[k]) / (mel_f[i + 2] - mel_f[i + 1]);
            w[(size_t)i * nf + k] = (float)(std::max(std::min(lower, upper), 0.0) * enorm);
        }
    }
    return w;
}

long long frame_count(const Config& c, long long n, bool centered) {  // src/mel.rs:143-154
    if (centered) return n / c.hop;
    return n < c.n_fft ? 0 : (n - c.n_fft) / c.hop + 1;
}

long long ceil_div(long long a, long long b) { return (a + b - 1) / b; }

}  // namespace

// ------------------------------------------------------------------ config
Config load_config(const std::string& dir) {
    const std::string fc = dir + "/config.json", fp = dir + "/processor_config.json";
    json::Value m, p;
    try {
        m = json::parse(read_file(fc));
    } catch (const Error&) {
        throw;
    } catch (const std::exception& e) {
        throw Error(kStatusJson, "failed to parse " + fc + ": " + e.what());
    }
    try {
        p = json::parse(read_file(fp));
    } catch (const Error&) {
        throw;
    } catch (const std::exception& e) {
        throw Error(kStatusJson, "failed to parse " + fp + ": " + e.what());
    }
    Config c;
    const json::Value& a = need(m, "audio_config", fc);
    c.hidden = need_int(a, "hidden_size", fc);
    c.layers = need_int(a, "num_hidden_layers", fc);
    c.heads = need_int(a, "num_attention_heads", fc);
    c.kv_heads = need_int(a, "num_key_value_heads", fc);
    c.inter = need_int(a, "intermediate_size", fc);
    c.n_mels = need_int(a, "num_mel_bins", fc);
    c.sub = need_int(a, "subsampling_factor", fc);
    c.rope_theta = need_num(need(a, "rope_parameters", fc), "rope_theta", fc);
    const json::Value& h = need(m, "head_config", fc);
    c.head_hidden = need_int(h, "hidden_size", fc);
    c.num_speakers = need_int(h, "num_speakers", fc);
    const json::Value& s = need(m, "streaming_config", fc);
    c.s_fifo = need_int(s, "fifo_length", fc, 0);
    c.cache_len = need_int(s, "speaker_cache_length", fc);
    c.n_sil = need_int(s, "speaker_cache_silence_frames_per_speaker", fc, 0);
    c.s_period = need_int(s, "speaker_cache_update_period", fc, 0);
    c.thr = (float)need_num(s, "prediction_score_threshold", fc);
    c.min_pos_rate = (float)need_num(s, "min_positive_scores_rate", fc);
    c.strong_rate = (float)need_num(s, "strong_boost_rate", fc);
    c.weak_rate = (float)need_num(s, "weak_boost_rate", fc);
    c.latest_boost = (float)need_num(s, "latest_frames_score_boost", fc);
    c.s_sub = need_int(s, "subsampling_factor", fc);
    c.s_ns = need_int(s, "num_speakers", fc);
    c.chunk_length = need_int(m, "chunk_length", fc);
    c.chunk_rc = need_int(m, "chunk_right_context", fc, 0);
    c.o_fifo = need_int(m, "fifo_length", fc, 0);
    c.o_period = need_int(m, "speaker_cache_update_period", fc, 0);
    const json::Value& fe = need(p, "feature_extractor", fp);
    c.feature_size = need_int(fe, "feature_size", fp);
    c.n_fft = need_int(fe, "n_fft", fp);
    c.hop = need_int(fe, "hop_length", fp);
    c.win = need_int(fe, "win_length", fp);
    c.sr = need_int(fe, "sampling_rate", fp);
    c.preemph = (float)need_num(fe, "preemphasis", fp);
    c.proc_sub = need_int(p, "subsampling_factor", fp);
    const json::Value& sm = need(p, "streaming_modes", fp);
    const char* names[3] = {"low_latency", "very_low_latency", "ultra_low_latency"};
    for (int i = 0; i < 3; i++) {
        const json::Value& v = need(sm, names[i], fp);
        if (v.arr.size() != 2) throw Error(kStatusJson, "failed to parse " + fp + ": bad streaming mode");
        c.modes[i][0] = count_value(v.arr[0], names[i], fp, 1);  // chunk length, encoder frames
        c.modes[i][1] = count_value(v.arr[1], names[i], fp, 0);  // right context
    }
    // CacheConfig::from_model (src/streaming.rs:54-72); its usize arithmetic needs a
    // non-negative per-speaker budget
    const int budget = c.cache_len / c.s_ns - c.n_sil;
    if (budget < 0)
        throw Error(kStatusJson, "failed to parse " + fc + ": unsupported speaker cache geometry (" +
                                     std::to_string(c.cache_len) + " frames for " + std::to_string(c.s_ns) +
                                     " speakers with " + std::to_string(c.n_sil) + " silence frames each)");
    c.min_pos = (int)std::floor((float)budget * c.min_pos_rate);
    c.k_strong = (int)std::floor((float)budget * c.strong_rate);
    c.k_weak = (int)std::floor((float)budget * c.weak_rate);
    // Shapes the kernels are built for.
    auto unsupported = [&](const std::string& what) {
        throw Error(kStatusJson, "failed to parse " + fc + ": unsupported " + what);
    };
    if (c.hidden != 512 || c.heads * 64 != c.hidden || c.kv_heads != c.heads) unsupported("attention geometry");
    if (c.inter % 128 || c.n_mels != 128 || c.feature_size != 128 || c.n_fft != 512 || c.win > c.n_fft)
        unsupported("front-end geometry");
    if (c.head_hidden != 192 || c.num_speakers > 8 || c.num_speakers != c.s_ns || c.sub != c.proc_sub ||
        c.sub != c.s_sub || (c.sub * c.n_mels) % 32)
        unsupported("head geometry");
    return c;
}

// ---------------------------------------------------------------- schedule
namespace {

// SpeakerCache counts only (src/streaming.rs:220-284): data-independent.
struct CacheSim {
    int fifo_len, period, cache_len;
    int ncache = 0, nfifo = 0, compressed = 0;
    int num_popped(int n) const {  // src/streaming.rs:220-228
        if (n <= fifo_len) return 0;
        return std::min(std::max(period, n - fifo_len), n);
    }
    void step(StepPlan& sp) {
        sp.ncache = ncache;
        sp.nfifo = nfifo;
        sp.was_compressed = compressed;
        const int nf = nfifo + sp.nchunk;
        sp.popped = num_popped(nf);
        const int ne = ncache + sp.popped;
        sp.compress = sp.popped > 0 && ne > cache_len;
        if (sp.popped > 0) {
            ncache = sp.compress ? cache_len : ne;
            compressed |= sp.compress;
        }
        nfifo = nf - sp.popped;
    }
};

}  // namespace

// Model::run_offline_capturing + chunk_loop's Offline arm (src/model.rs:242-310, 485-503).
ClipPlan plan_offline(const Config& c, long long n) {
    ClipPlan p;
    const long long valid = frame_count(c, n, true);
    const long long groups = ceil_div(valid + 1, c.sub);
    MelSeg seg{0, n, 1, (int)valid, (int)groups, 0};
    p.segs.push_back(seg);
    CacheSim cs{c.o_fifo, c.o_period, c.cache_len};
    const long long valid_groups = ceil_div(valid, c.sub);  // g * sub < valid
    for (long long start = 0; start < groups; start += c.chunk_length) {
        const long long end = std::min(start + (long long)c.chunk_length, groups);
        const long long hi = std::min(end + (long long)c.chunk_rc, groups);
        StepPlan sp{};
        sp.seg = 0;
        sp.group_lo = (int)start;
        sp.n_new = (int)(hi - start);
        sp.nchunk = (int)(end - start);
        const int prefix = cs.ncache + cs.nfifo;
        sp.S = prefix + sp.n_new;
        sp.valid = prefix + (int)std::min(std::max(valid_groups - start, 0LL), hi - start);
        sp.keep_rows = sp.nchunk * c.sub;
        cs.step(sp);
        p.steps.push_back(sp);
        p.emitted_rows += sp.keep_rows;
    }
    p.out_rows = std::min(p.emitted_rows, valid + 1);
    p.num_chunks = (int)p.steps.size();
    p.cache_compressed = cs.compressed;
    p.cache_frames = cs.ncache;
    p.fifo_frames = cs.nfifo;
    return p;
}

// Model::streaming_chunks (src/model.rs:343-365), geometry from ModeParams::resolve
// (src/config.rs:152-202): the first chunk centred, later full chunks uncentred one
// step of mel frames apart, and what is left as a final centred chunk.
std::vector<StreamChunk> streaming_chunks(const Config& c, long long n, int mode) {
    if (mode < 0 || mode > 2) throw Error(kStatusArg, "streaming mode must be low, very low or ultra low latency");
    const int cl = c.modes[mode][0], rc = c.modes[mode][1];
    const long long mel_chunk = (long long)(cl + rc) * c.sub, mel_step = (long long)cl * c.sub;
    const long long first = (mel_chunk - 1) * c.hop + c.win / 2;
    const long long per_chunk = mel_chunk * c.hop + c.win;
    std::vector<StreamChunk> chunks;
    const long long f0 = std::min(first, n);
    chunks.push_back({0, f0, frame_count(c, f0, true), 1, rc});
    long long mel_idx = mel_step;
    long long start = mel_idx * c.hop - c.n_fft / 2;
    while (start + per_chunk <= n) {
        chunks.push_back({start, per_chunk, frame_count(c, per_chunk, false), 0, rc});
        mel_idx += mel_step;
        start = mel_idx * c.hop - c.n_fft / 2;
    }
    const long long ls = std::min(start, n);
    chunks.push_back({ls, n - ls, frame_count(c, n - ls, true), 1, 0});
    return chunks;
}

// run_streaming + chunk_loop's Streaming arm (src/model.rs:313-336, 504-510).
ClipPlan plan_streaming(const Config& c, long long n, int mode) {
    const std::vector<StreamChunk> chunks = streaming_chunks(c, n, mode);
    ClipPlan p;
    CacheSim cs{c.s_fifo, c.s_period, c.cache_len};
    for (size_t i = 0; i < chunks.size(); i++) {
        const StreamChunk& ch = chunks[i];
        const long long nm = ch.mel_frames;
        const long long groups = ceil_div(nm, c.sub);
        if (groups < ch.lookahead)
            throw Error(kStatusAudio, "unsupported audio: a streaming chunk holds " + std::to_string(groups) +
                                          " encoder frames, fewer than the look-ahead of " +
                                          std::to_string(ch.lookahead));
        p.segs.push_back(MelSeg{ch.start, ch.len, ch.centered, (int)nm, (int)groups, 0});
        StepPlan sp{};
        sp.seg = (int)i;
        sp.group_lo = 0;
        sp.n_new = (int)groups;
        // An uncentred chunk after the first or another uncentred chunk starts exactly
        // c * 8 mel frames later on the same frame grid (Model::streaming_chunks,
        // src/model.rs:343-365), so its first r = look-ahead groups are the previous
        // chunk's last r: the same samples, and the same pre-emphasised values wherever
        // the Hann window is non-zero (the chunk's own first sample, which has no
        // predecessor in its slice, falls under the window's zero taps).  Those
        // embeddings are taken from the previous step; only the c new groups are
        // computed.  The final chunk is centred on a shifted grid and computed whole.
        if (i > 0 && !ch.centered && (i == 1 || !chunks[i - 1].centered)) {
            const int r = chunks[i - 1].lookahead;
            const long long prev_groups = ceil_div(chunks[i - 1].mel_frames, c.sub);
            if (r > 0 && groups > r && prev_groups >= r) {
                sp.reuse = r;
                sp.group_lo = r;
                sp.n_new = (int)(groups - r);
            }
        }
        sp.nchunk = (int)(groups - ch.lookahead);
        const int prefix = cs.ncache + cs.nfifo;
        sp.S = prefix + sp.reuse + sp.n_new;
        sp.valid = sp.S;
        sp.keep_rows = (int)std::min((long long)sp.nchunk * c.sub, nm);
        cs.step(sp);
        p.steps.push_back(sp);
        p.emitted_rows += sp.keep_rows;
    }
    p.out_rows = p.emitted_rows;
    p.num_chunks = (int)p.steps.size();
    p.cache_compressed = cs.compressed;
    p.cache_frames = cs.ncache;
    p.fifo_frames = cs.nfifo;
    return p;
}

// ------------------------------------------------------------------ model

Model::Model(const std::string& dir, int device) : device_(device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) throw Error(kStatusNoDevice, "no CUDA device is visible");
    if (device < 0 || device >= n) throw Error(kStatusNoDevice, "CUDA device " + std::to_string(device) + " does not exist");
    N3D_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop{};
    N3D_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        throw Error(kStatusGpu, std::string("this build targets sm_100a (B200); device is ") + prop.name);
    cfg_ = load_config(dir);
    N3D_CUDA(cudaStreamCreateWithFlags(&own_stream_, cudaStreamNonBlocking));
    stream_ = own_stream_;
    N3D_CUDA(cudaStreamCreateWithFlags(&copy_stream_, cudaStreamNonBlocking));
    N3D_CUDA(cudaStreamCreateWithFlags(&capture_stream_, cudaStreamNonBlocking));
    N3D_CUDA(cudaEventCreateWithFlags(&upload_start_, cudaEventDisableTiming));
    N3D_CUDA(cudaMalloc(&dev_err_, sizeof(int)));
    N3D_CUDA(cudaMemset(dev_err_, 0, sizeof(int)));
    upload_weights(dir);
}

Model::~Model() {
    cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    for (const ProfRec& r : pending_) {
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    for (cudaEvent_t e : event_pool_) cudaEventDestroy(e);
    if (copy_stream_) cudaStreamSynchronize(copy_stream_);
    for (cudaEvent_t e : upload_ev_) cudaEventDestroy(e);
    if (host_stage_) cudaFreeHost(host_stage_);
    for (auto& kv : tower_graphs_)
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    if (capture_stream_) cudaStreamDestroy(capture_stream_);
    if (upload_start_) cudaEventDestroy(upload_start_);
    if (copy_stream_) cudaStreamDestroy(copy_stream_);
    for (void* p : owned_) cudaFree(p);
    for (auto& kv : ws_) cudaFree(kv.second.p);
    if (dev_err_) cudaFree(dev_err_);
    if (own_stream_) cudaStreamDestroy(own_stream_);
}

void Model::set_stream(cudaStream_t s) {
    N3D_CUDA(cudaSetDevice(device_));
    N3D_CUDA(cudaStreamSynchronize(stream_));
    prof_collect();
    stream_ = s ? s : own_stream_;
}

void Model::upload_weights(const std::string& dir) {
    SafeTensors st(dir + "/model.safetensors");
    const Config& c = cfg_;
    const long long h = c.hidden, hh = c.head_hidden;
    auto dev = [&](const std::vector<float>& v) {
        float* p = nullptr;
        N3D_CUDA(cudaMalloc(&p, v.size() * 4 + 16));
        N3D_CUDA(cudaMemcpy(p, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
        owned_.push_back(p);
        return p;
    };
    auto plain = [&](const std::string& name, std::vector<long long> shape) {
        const float* d = st.get(name, shape);
        long long n = 1;
        for (long long x : shape) n *= x;
        return dev(std::vector<float>(d, d + n));
    };
    // weights in the fp16 split with a per-matrix scale: h + l = w s, s from max |w|;
    // split on the device by the same kernel that splits activations
    auto split = [&](const std::vector<float>& w, int out, int in, const float* bias) {
        DevLinear L;
        L.scale = split_scale(absmax_host(w.data(), w.size()));
        float* tmp = nullptr;
        N3D_CUDA(cudaMalloc(&tmp, w.size() * 4 + 16));
        N3D_CUDA(cudaMemcpy(tmp, w.data(), w.size() * 4, cudaMemcpyHostToDevice));
        for (void** p : {&L.h, &L.l}) {
            N3D_CUDA(cudaMalloc(p, w.size() * 2 + 16));
            owned_.push_back(*p);
        }
        launch_split(nullptr, tmp, (long long)w.size(), SplitOut{L.h, L.l, L.scale, nullptr});
        N3D_CUDA(cudaDeviceSynchronize());
        N3D_CUDA(cudaFree(tmp));
        L.out = out;
        L.in = in;
        if (bias) L.bias = dev(std::vector<float>(bias, bias + out));
        return L;
    };
    auto linear = [&](const std::string& name, int out, int in, const char* bias_name) {
        const float* w = st.get(name, {out, in});
        const float* b = bias_name ? st.get(bias_name, {out}) : nullptr;
        return split(std::vector<float>(w, w + (size_t)out * in), out, in, b);
    };
    const std::string P = "model.audio_tower";
    if (h % 4 || hh % 64 || (c.sub * c.n_mels) % 32 || c.inter % 32)
        throw Error(kStatusShape, "the GEMMs need hidden % 4, head hidden % 64, sub * n_mels % 32 and "
                                  "intermediate % 32 to be 0");
    embed_ = linear(P + ".embedder.projection.weight", (int)h, c.sub * c.n_mels, nullptr);
    s_mel_ = split_scale(89.0);  // ln of any finite float >= 2^-24 lies in [-16.7, 88.8]
    in_ln_w_ = plain(P + ".input_layer_norm.weight", {h});
    in_ln_b_ = plain(P + ".input_layer_norm.bias", {h});
    fin_ln_w_ = plain(P + ".layer_norm.weight", {h});
    fin_ln_b_ = plain(P + ".layer_norm.bias", {h});
    for (int i = 0; i < c.layers; i++) {
        const std::string b = P + ".layers." + std::to_string(i);
        DevLayer L;
        L.ln1_w = plain(b + ".layer_norm1.weight", {h});
        L.ln1_b = plain(b + ".layer_norm1.bias", {h});
        L.ln2_w = plain(b + ".layer_norm2.weight", {h});
        L.ln2_b = plain(b + ".layer_norm2.bias", {h});
        // q, k, v stacked row-wise into one [3h, h] weight (src/gpu_engine.rs:263-276)
        std::vector<float> qkv;
        qkv.reserve((size_t)3 * h * h);
        for (const char* nm : {".self_attn.q_proj.weight", ".self_attn.k_proj.weight", ".self_attn.v_proj.weight"}) {
            const float* w = st.get(b + nm, {h, h});
            qkv.insert(qkv.end(), w, w + h * h);
        }
        L.qkv = split(qkv, (int)(3 * h), (int)h, nullptr);
        L.o = linear(b + ".self_attn.o_proj.weight", (int)h, (int)h, (b + ".self_attn.o_proj.bias").c_str());
        L.fc1 = linear(b + ".mlp.fc1.weight", c.inter, (int)h, (b + ".mlp.fc1.bias").c_str());
        L.fc2 = linear(b + ".mlp.fc2.weight", (int)h, c.inter, (b + ".mlp.fc2.bias").c_str());
        const double b1 = ln_bound(st.get(b + ".layer_norm1.weight", {h}), st.get(b + ".layer_norm1.bias", {h}), h);
        const double b2 = ln_bound(st.get(b + ".layer_norm2.weight", {h}), st.get(b + ".layer_norm2.bias", {h}), h);
        L.s_ln1 = split_scale(b1);
        L.s_ln2 = split_scale(b2);
        L.s_ctx = split_scale(row_l1_max(st.get(b + ".self_attn.v_proj.weight", {h, h}), h, h) * b1);
        L.s_q = split_scale(2.0 * row_l1_max(st.get(b + ".self_attn.q_proj.weight", {h, h}), h, h) * b1);
        L.s_k = split_scale(2.0 * row_l1_max(st.get(b + ".self_attn.k_proj.weight", {h, h}), h, h) * b1);
        L.s_ffn = split_scale(linear_bound(st.get(b + ".mlp.fc1.weight", {c.inter, h}),
                                           st.get(b + ".mlp.fc1.bias", {c.inter}), c.inter, h, b2));
        layers_.push_back(L);
    }
    proj_ = linear("model.proj.weight", (int)hh, (int)h, "model.proj.bias");
    {
        // Conv1d weight [out, in, 3] -> tap-major [out, 3 * in] so the k=3 conv is
        // a GEMM over three row-shifted copies of the padded input.
        const int oc = (int)hh * c.sub;
        const float* w = st.get("model.upsampler.conv.weight", {oc, hh, 3});
        const float* b = st.get("model.upsampler.conv.bias", {oc});
        std::vector<float> r((size_t)oc * 3 * hh);
        for (int o = 0; o < oc; o++)
            for (int ic = 0; ic < hh; ic++)
                for (int j = 0; j < 3; j++) r[(size_t)o * 3 * hh + j * hh + ic] = w[((size_t)o * hh + ic) * 3 + j];
        conv_ = split(r, oc, (int)(3 * hh), b);
    }
    dense_ = linear("classifier.dense.weight", (int)hh, (int)hh, "classifier.dense.bias");
    {
        const double bf = ln_bound(st.get(P + ".layer_norm.weight", {h}), st.get(P + ".layer_norm.bias", {h}), h);
        const double bp = linear_bound(st.get("model.proj.weight", {hh, h}), st.get("model.proj.bias", {hh}), hh, h, bf);
        const long long oc = hh * c.sub;
        const double bc = linear_bound(st.get("model.upsampler.conv.weight", {oc, hh, 3}),
                                       st.get("model.upsampler.conv.bias", {oc}), oc, 3 * hh, bp);
        s_fin_ = split_scale(bf);
        s_proj_ = split_scale(bp);
        s_conv_ = split_scale(bc);  // |relu(y)| <= |y|
    }
    out_w_ = plain("classifier.out_proj.weight", {c.num_speakers, hh});
    out_b_ = plain("classifier.out_proj.bias", {c.num_speakers});
    silence_ = plain("silence_embeds", {h});

    // front-end constants
    const int nf = c.n_fft / 2 + 1;
    std::vector<float> filt = slaney(c.n_mels, c.n_fft, c.sr, 0.0, (double)c.sr / 2.0);
    // each filter's support [lo, lo + w) (w = 0: an empty filter), and the weights
    // transposed: row i holds every filter's weight for its bin lo + i
    if (c.n_mels != 128 || c.n_fft != 512) throw Error(13, "the log-mel kernel is built for 128 mels of a 512 FFT");
    std::vector<int> flo(c.n_mels), fw(c.n_mels);
    int fb_w = 0;
    for (int m = 0; m < c.n_mels; m++) {
        int lo = nf, hi = -1;
        for (int k = 0; k < nf; k++)
            if (filt[(size_t)m * nf + k] != 0.0f) {
                lo = std::min(lo, k);
                hi = std::max(hi, k);
            }
        flo[m] = lo;
        fw[m] = hi >= lo ? hi - lo + 1 : 0;
        fb_w = std::max(fb_w, fw[m]);
        mel_tab_.group_w[m / 32] = std::max(mel_tab_.group_w[m / 32], fw[m]);
    }
    if (fb_w > MEL_FB_MAX_W) throw Error(13, "slaney filterbank: a filter wider than the log-mel kernel's table");
    std::vector<float> fbt((size_t)std::max(fb_w, 1) * c.n_mels, 0.0f);
    for (int m = 0; m < c.n_mels; m++)
        for (int i = 0; i < fw[m]; i++) fbt[(size_t)i * c.n_mels + m] = filt[(size_t)m * nf + flo[m] + i];
    auto devi = [&](const std::vector<int>& v) {
        int* p = nullptr;
        N3D_CUDA(cudaMalloc(&p, v.size() * 4));
        N3D_CUDA(cudaMemcpy(p, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
        owned_.push_back(p);
        return p;
    };
    mel_tab_.fbank_t = dev(fbt);
    mel_tab_.filt_lo = devi(flo);
    mel_tab_.filt_w = devi(fw);
    mel_tab_.fb_w = fb_w;
    // torch.hann_window(win, periodic=False) centred in the n_fft frame (src/mel.rs:43-48, 197-200)
    std::vector<float> window(c.n_fft, 0.0f);
    const int left = (c.n_fft - c.win) / 2;
    const float denom = (float)(c.win - 1);
    for (int i = 0; i < c.win; i++)
        window[left + i] = 0.5f * (1.0f - std::cos(2.0f * 3.14159265358979323846f * (float)i / denom));
    mel_tab_.window = dev(window);
    std::vector<float> tw(c.n_fft);
    for (int k = 0; k < c.n_fft / 2; k++) {
        const double ang = -2.0 * 3.14159265358979323846 * (double)k / (double)c.n_fft;
        tw[2 * k] = (float)std::cos(ang);
        tw[2 * k + 1] = (float)std::sin(ang);
    }
    mel_tab_.twiddle = dev(tw);
    // RoPE tables for positions 0..s_cap-1 (src/encoder.rs:163-185)
    const int hd = c.hidden / c.heads, half = hd / 2;
    std::vector<float> inv(half), cs((size_t)s_cap_ * hd), sn((size_t)s_cap_ * hd);
    for (int i = 0; i < half; i++) inv[i] = (float)(1.0 / std::pow(c.rope_theta, 2.0 * (double)i / (double)hd));
    for (int p = 0; p < s_cap_; p++)
        for (int i = 0; i < half; i++) {
            const float a = (float)p * inv[i];
            cs[(size_t)p * hd + i] = cs[(size_t)p * hd + half + i] = std::cos(a);
            sn[(size_t)p * hd + i] = sn[(size_t)p * hd + half + i] = std::sin(a);
        }
    rope_cos_ = dev(cs);
    rope_sin_ = dev(sn);
}

void* Model::ws(const char* name, size_t bytes) {
    bytes = (bytes + 255) & ~size_t(255);
    if (bytes == 0) bytes = 256;
    Buf& b = ws_[name];
    if (b.bytes < bytes) {
        if (b.p) {
            N3D_CUDA(cudaStreamSynchronize(stream_));
            N3D_CUDA(cudaFree(b.p));
        }
        b.p = nullptr;
        N3D_CUDA(cudaMalloc(&b.p, bytes));
        b.bytes = bytes;
        ws_gen_++;  // captured tower graphs may hold the old address
    }
    return b.p;
}

SplitBuf Model::ws2(const std::string& base, long long rows, long long cols) {
    SplitBuf b;
    b.h = ws((base + "_h").c_str(), (size_t)rows * cols * 2);
    b.l = ws((base + "_l").c_str(), (size_t)rows * cols * 2);
    b.cols = cols;
    b.rows_cap = std::min((long long)(ws_[base + "_h"].bytes / (cols * 2)),
                          (long long)(ws_[base + "_l"].bytes / (cols * 2)));
    return b;
}

float Model::dyn_scale(const float* d, long long n) {
    float* m = (float*)ws("absmax", 4);
    N3D_CUDA(cudaMemsetAsync(m, 0, 4, stream_));
    launch_absmax(stream_, d, n, m);
    float hm = 0.0f;
    N3D_CUDA(cudaMemcpyAsync(&hm, m, 4, cudaMemcpyDeviceToHost, stream_));
    N3D_CUDA(cudaStreamSynchronize(stream_));
    return split_scale(hm);
}

void Model::check_dev_error() {
    int e = 0;
    N3D_CUDA(cudaMemcpy(&e, dev_err_, sizeof(int), cudaMemcpyDeviceToHost));
    if (e != 0) {
        N3D_CUDA(cudaMemset(dev_err_, 0, sizeof(int)));
        throw Error(kStatusTimeout, "a device-side wait timed out (site " + std::to_string(e) + ")");
    }
}

void Model::profile_enable(bool on) {
    N3D_CUDA(cudaSetDevice(device_));
    N3D_CUDA(cudaStreamSynchronize(stream_));
    prof_collect();
    prof_ = on;
    for (auto& t : totals_) t = ProfTotals{};
}

void Model::step_timing_enable(bool on) {
    N3D_CUDA(cudaSetDevice(device_));
    N3D_CUDA(cudaStreamSynchronize(stream_));
    prof_collect();
    step_timing_ = on;
    step_ms_.clear();
}

cudaEvent_t Model::pool_event() {
    if (event_pool_.empty()) {
        for (int i = 0; i < 64; i++) {
            cudaEvent_t e;
            N3D_CUDA(cudaEventCreate(&e));
            event_pool_.push_back(e);
        }
    }
    cudaEvent_t e = event_pool_.back();
    event_pool_.pop_back();
    return e;
}

void Model::prof_begin() {
    if (!prof_) return;
    if (event_pool_.size() < 2) {
        for (int i = 0; i < 64; i++) {
            cudaEvent_t e;
            N3D_CUDA(cudaEventCreate(&e));
            event_pool_.push_back(e);
        }
    }
    cur_begin_ = event_pool_.back();
    event_pool_.pop_back();
    N3D_CUDA(cudaEventRecord(cur_begin_, stream_));
}

void Model::prof_end(int cls, double flops, double bytes) {
    if (!prof_ || !cur_begin_) return;
    cudaEvent_t b = event_pool_.back();
    event_pool_.pop_back();
    N3D_CUDA(cudaEventRecord(b, stream_));
    pending_.push_back(ProfRec{cls, cur_begin_, b, flops, bytes});
    cur_begin_ = nullptr;
    if (pending_.size() > 4096) {
        N3D_CUDA(cudaStreamSynchronize(stream_));
        prof_collect();
    }
}

// Resolve recorded event pairs (the stream must be idle).
void Model::prof_collect() {
    for (const auto& pr : step_ev_) {
        float ms = 0.0f;
        N3D_CUDA(cudaEventElapsedTime(&ms, pr.first, pr.second));
        step_ms_.push_back(ms);
        event_pool_.push_back(pr.first);
        event_pool_.push_back(pr.second);
    }
    step_ev_.clear();
    for (const ProfRec& r : pending_) {
        float ms = 0.0f;
        N3D_CUDA(cudaEventElapsedTime(&ms, r.a, r.b));
        ProfTotals& t = totals_[r.cls];
        t.launches++;
        t.ms += ms;
        t.flops += r.flops;
        t.bytes += r.bytes;
        event_pool_.push_back(r.a);
        event_pool_.push_back(r.b);
    }
    pending_.clear();
}

// The 31-layer tower on B sequences of stride S rows (S a multiple of 8) held in
// ws "win".  Output: the final LayerNorm in the fp16 split in ws "n" (and
// plain in enc_plain when given).  Residual adds are fused into the LayerNorm
// that follows them, so every GEMM epilogue is a pure (TMA) store.
void Model::tower(int B, int S, const int* d_seq_len, const int* d_valid, float* enc_plain) {
    const Config& c = cfg_;
    const long long M = (long long)B * S, h = c.hidden;
    float* win = (float*)ws("win", M * h * 4);
    float* x = (float*)ws("x", M * h * 4);
    const SplitBuf n = ws2("n", M, h);  // LayerNorm output, fp16 split
    // attention operands in the fp16 split: Q, K [M, h]; V^T [h, M] (column = global row)
    AttnOperands ao;
    ao.q_h = ws("q_h", M * h * 2);
    ao.q_l = ws("q_l", M * h * 2);
    ao.k_h = ws("k_h", M * h * 2);
    ao.k_l = ws("k_l", M * h * 2);
    ao.vt_ld = M;
    ao.vt_h = ws("vt_h", h * M * 2);
    ao.vt_l = ws("vt_l", h * M * 2);
    ao.rows_cap = (long long)(ws_["q_h"].bytes / (h * 2));
    const SplitBuf ctx = ws2("ctx", M, h);     // attention context
    const SplitBuf f = ws2("f", M, c.inter);   // GELU(fc1)

    Epi e;  // QKV: Q/K pairs with RoPE, V^T pair
    e.mode = EPI_QKV_ATTN;
    e.tma = 1;
    e.map_h = make_f16_map(ao.q_h, M, h, h, 64, 32, true);
    e.map_l = make_f16_map(ao.q_l, M, h, h, 64, 32, true);
    e.map_k_h = make_f16_map(ao.k_h, M, h, h, 64, 32, true);
    e.map_k_l = make_f16_map(ao.k_l, M, h, h, 64, 32, true);
    e.map_vt_h = make_f16_map(ao.vt_h, h, M, ao.vt_ld, 32, 64, false);
    e.map_vt_l = make_f16_map(ao.vt_l, h, M, ao.vt_ld, 32, 64, false);
    e.cos_t = rope_cos_;
    e.sin_t = rope_sin_;
    e.rope_seq = S;
    e.head_dim = (int)(h / c.heads);
    e.q_cols = (int)h;
    e.k_cols = (int)h;
    Epi eo;  // o_proj / fc2: x += acc + bias, the residual adds of src/encoder.rs:262-276
    eo.mode = EPI_STORE;
    eo.tma = 1;
    eo.reduce = 1;
    eo.map_out = make_store_map(x, M, h, h);
    eo.out = x;
    eo.ldo = h;
    if (M <= 2048) {  // small launches may split K (gemm_split): 4 partial [M rounded to 128, h] tiles
        const long long mp = (M + 127) / 128 * 128;
        eo.split_ws = (float*)ws("split_ws", (size_t)4 * mp * h * 4);
        eo.split_ws_floats = 4 * mp * h;
    }
    Epi e1;  // fc1: GELU(acc + bias) -> fp16 split
    e1.mode = EPI_GELU_SPLIT;
    e1.tma = 1;
    e1.map_h = make_store_map_f16(f.h, M, c.inter, c.inter);
    e1.map_l = make_store_map_f16(f.l, M, c.inter, c.inter);

    const double ln_bytes = (double)M * h * 8;  // read x, write h, l
    prof_begin();
    launch_layer_norm(stream_, win, M, (int)h, in_ln_w_, in_ln_b_, plain_out(x));
    prof_end(K_LN, 0, (double)M * h * 8);
    for (int l = 0; l < c.layers; l++) {
        const DevLayer& L = layers_[l];
        prof_begin();
        launch_layer_norm(stream_, x, M, (int)h, L.ln1_w, L.ln1_b, n.out(L.s_ln1));
        prof_end(K_LN, 0, ln_bytes);
        e.sec_scale[0] = ao.q_scale = L.s_q;
        e.sec_scale[1] = ao.k_scale = L.s_k;
        e.sec_scale[2] = ao.v_scale = L.s_ctx;
        prof_begin();
        gemm_split(stream_, n.op(L.s_ln1), L.qkv.op(), (int)M, (int)(3 * h), (int)h, 0, e, dev_err_);
        prof_end(K_GEMM_QKV, 2.0 * M * 3 * h * h, 0);
        prof_begin();
        launch_attention_tc(stream_, ao, B, S, d_valid, c.heads, (int)(h / c.heads), ctx.out(L.s_ctx), dev_err_);
        prof_end(K_ATTN, 4.0 * B * (double)S * S * h, 0);
        eo.bias = L.o.bias;
        prof_begin();
        gemm_split(stream_, ctx.op(L.s_ctx), L.o.op(), (int)M, (int)h, (int)h, 0, eo, dev_err_);
        prof_end(K_GEMM_O, 2.0 * M * h * h, 0);
        prof_begin();
        launch_layer_norm(stream_, x, M, (int)h, L.ln2_w, L.ln2_b, n.out(L.s_ln2));
        prof_end(K_LN, 0, ln_bytes);
        e1.bias = L.fc1.bias;
        e1.out_scale = L.s_ffn;
        prof_begin();
        gemm_split(stream_, n.op(L.s_ln2), L.fc1.op(), (int)M, c.inter, (int)h, 0, e1, dev_err_);
        prof_end(K_GEMM_FC1, 2.0 * M * c.inter * h, 0);
        eo.bias = L.fc2.bias;
        prof_begin();
        gemm_split(stream_, f.op(L.s_ffn), L.fc2.op(), (int)M, (int)h, c.inter, 0, eo, dev_err_);
        prof_end(K_GEMM_FC2, 2.0 * M * h * c.inter, 0);
    }
    prof_begin();
    launch_layer_norm(stream_, x, M, (int)h, fin_ln_w_, fin_ln_b_, n.out(s_fin_));
    prof_end(K_LN, 0, ln_bytes);
    if (enc_plain) launch_layer_norm(stream_, x, M, (int)h, fin_ln_w_, fin_ln_b_, plain_out(enc_plain));
    (void)d_seq_len;
}

// Classification head (src/head.rs:147-157) on the encoder output in ws "n":
// proj into a per-sequence zero-padded layout [B, S+2, hh] -> implicit-GEMM k=3
// conv over it (its output keeps that padded row layout; the sub-pixel reshape
// is free on row-major memory) -> dense + ReLU + out_proj fused.  Logits land
// in ws "logits" with sequence i at rows i * (S + 2) * sub.
void Model::head(int B, int S, const int* d_seq_len, float widen) {
    const Config& c = cfg_;
    const long long M = (long long)B * S, h = c.hidden, hh = c.head_hidden, up = c.sub;
    const long long PR = (long long)B * (S + 2), MC = PR - 2;
    const SplitBuf n = ws2("n", M, h);
    const SplitBuf pb = ws2("p", PR, hh);        // proj output, zero-padded per sequence
    const SplitBuf u = ws2("u", PR * up, hh);    // conv output as [8 rows per frame, hh]
    float* logits = (float*)ws("logits", PR * up * c.num_speakers * 4);
    N3D_CUDA(cudaMemsetAsync(pb.h, 0, PR * hh * 2, stream_));
    N3D_CUDA(cudaMemsetAsync(pb.l, 0, PR * hh * 2, stream_));
    Epi ep;
    ep.mode = EPI_SPLIT;
    ep.out_h = pb.h;
    ep.out_l = pb.l;
    // the input's scale is s_fin_ / widen; proj's and the conv's output bounds grow with it
    const float s_in = s_fin_ / widen, s_p = s_proj_ / widen, s_u = s_conv_ / widen;
    ep.out_scale = s_p;
    ep.ldo = hh;
    ep.bias = proj_.bias;
    ep.rdiv = S;
    ep.rkeep = S;
    ep.rmul = S + 2;
    ep.roff = 1;
    ep.seq_len = d_seq_len;
    prof_begin();
    gemm_split(stream_, n.op(s_in), proj_.op(), (int)M, (int)hh, (int)h, 0, ep, dev_err_);
    prof_end(K_GEMM_PROJ, 2.0 * M * hh * h, 0);
    Epi ec;
    ec.mode = EPI_RELU_SPLIT;
    ec.tma = 1;
    ec.bias = conv_.bias;
    ec.out_scale = s_u;
    ec.map_h = make_store_map_f16(u.h, MC, up * hh, up * hh);
    ec.map_l = make_store_map_f16(u.l, MC, up * hh, up * hh);
    prof_begin();
    // k=3 conv: k-block kb (of 64) reads tap kb / (hh / 64), i.e. rows shifted by 0, 1, 2
    gemm_split(stream_, pb.op(s_p), conv_.op(), (int)MC, (int)(up * hh), (int)(3 * hh), (int)(hh / 64), ec,
               dev_err_);
    prof_end(K_GEMM_CONV, 2.0 * M * up * hh * 3 * hh, 0);
    Epi ed;
    ed.mode = EPI_DENSE_OUT;
    ed.out = logits;
    ed.ldo = c.num_speakers;
    ed.bias = dense_.bias;
    ed.w2 = out_w_;
    ed.b2 = out_b_;
    ed.n2 = c.num_speakers;
    prof_begin();
    gemm_split(stream_, u.op(s_u), dense_.op(), (int)(MC * up), (int)hh, (int)hh, 0, ed, dev_err_);
    prof_end(K_GEMM_DENSE, 2.0 * M * up * hh * hh + 2.0 * M * up * hh * c.num_speakers, 0);
}

float* Model::host_stage(size_t bytes) {
    if (bytes > host_stage_bytes_) {
        if (host_stage_) N3D_CUDA(cudaFreeHost(host_stage_));
        host_stage_ = nullptr;
        host_stage_bytes_ = 0;
        N3D_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&host_stage_), bytes, cudaHostAllocDefault));
        host_stage_bytes_ = bytes;
    }
    return host_stage_;
}

void Model::run_batch(int mode, const std::vector<const float*>& host_audio, const float* d_audio_in,
                      const std::vector<long long>& offsets_in, const std::vector<long long>& lens,
                      const HostSink* host_out, float* d_logits,
                      const std::vector<long long>* out_offsets, std::vector<ClipPlan>* plans_out) {
    const Config& c = cfg_;
    N3D_CUDA(cudaSetDevice(device_));
    const int nclips = (int)lens.size();
    std::vector<ClipPlan> plans(nclips);
    for (int i = 0; i < nclips; i++)
        plans[i] = mode == 3 ? plan_offline(c, lens[i]) : plan_streaming(c, lens[i], mode);
    if (plans_out) *plans_out = plans;
    const int ns = c.num_speakers, h = c.hidden;
    const int B_CAP = 128;

    for (int c0 = 0; c0 < nclips; c0 += B_CAP) {
        const int c1 = std::min(nclips, c0 + B_CAP), nb = c1 - c0;
        // ---- audio.  Host audio goes up on the copy stream in two phases: the samples
        // that chunk step 0 of every clip needs, then the rest, which arrives while step 0
        // computes.  Each phase is cut into parts of kUploadClips clips, and the mel of a
        // part waits only for that part's upload.
        std::vector<long long> aoff(nb);
        long long total_samples = 0;
        const float* d_audio = d_audio_in;
        const int nphase = d_audio_in ? 1 : 2;
        const int nparts = d_audio_in ? 0 : (nb + kUploadClips - 1) / kUploadClips;
        if (!d_audio_in) {
            for (int i = 0; i < nb; i++) {
                aoff[i] = total_samples;
                total_samples += lens[c0 + i];
            }
        } else {
            for (int i = 0; i < nb; i++) aoff[i] = offsets_in[c0 + i];
        }
        // ---- mel parts per phase: the groups of each segment that the phase's steps read
        // (device audio: one phase with every group of every segment)
        struct PartRef {
            long long base = -1, lo = 0;  // group base in the phase's embeddings, first group
        };
        std::vector<std::vector<std::array<PartRef, 2>>> ref(nb);
        std::vector<std::vector<MelSeg>> pseg(nphase);
        std::vector<std::vector<long long>> pbase(nphase);
        std::vector<long long> ptot_groups(nphase, 0), ptot_frames(nphase, 0);
        std::vector<std::vector<std::pair<long long, cudaEvent_t>>> pparts(nphase);
        std::vector<long long> end0(nb, 0);  // host audio: samples uploaded in phase 0
        if (!d_audio_in)
            while ((int)upload_ev_.size() < nphase * nparts) {
                cudaEvent_t e;
                N3D_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
                upload_ev_.push_back(e);
            }
        // A step reuses the previous step's embedding rows only when both embed in the
        // same phase (host audio: step 0 embeds in phase 0, the rest in phase 1); step 1
        // of a two-phase batch embeds its whole chunk instead.
        if (nphase == 2)
            for (int i = 0; i < nb; i++) {
                std::vector<StepPlan>& st = plans[c0 + i].steps;
                if (st.size() > 1 && st[1].reuse > 0) {
                    st[1].group_lo -= st[1].reuse;
                    st[1].n_new += st[1].reuse;
                    st[1].reuse = 0;
                }
            }
        for (int i = 0; i < nb; i++) {
            const ClipPlan& p = plans[c0 + i];
            const int nseg = (int)p.segs.size();
            ref[i].assign(nseg, {});
            std::vector<std::array<long long, 4>> rng(nseg, {LLONG_MAX, -1, LLONG_MAX, -1});  // lo0, hi0, lo1, hi1
            if (nphase == 1) {
                for (int sg = 0; sg < nseg; sg++) rng[sg] = {0, p.segs[sg].groups, LLONG_MAX, -1};
            } else {
                for (size_t w = 0; w < p.steps.size(); w++) {
                    const StepPlan& sp = p.steps[w];
                    const int ph = w == 0 ? 0 : 1;
                    long long& lo = rng[sp.seg][2 * ph];
                    long long& hi = rng[sp.seg][2 * ph + 1];
                    lo = std::min(lo, (long long)sp.group_lo);
                    hi = std::max(hi, (long long)(sp.group_lo + sp.n_new));
                }
            }
            for (int ph = 0; ph < nphase; ph++) {
                for (int sg = 0; sg < nseg; sg++) {
                    const long long lo = rng[sg][2 * ph], hi = rng[sg][2 * ph + 1];
                    if (hi <= lo) continue;
                    MelSeg m = p.segs[sg];
                    m.frame_lo = (int)(lo * c.sub);
                    m.groups = (int)(hi - lo);
                    m.group_base = ptot_groups[ph];
                    ref[i][sg][ph] = PartRef{ptot_groups[ph], lo};
                    ptot_groups[ph] += m.groups;
                    const int nf = mel_frames(m, c.sub);
                    ptot_frames[ph] += nf;
                    pseg[ph].push_back(m);
                    pbase[ph].push_back(aoff[i] + m.audio_off);
                    if (ph == 0 && nf > 0) {  // last sample phase 0's frames read, plus one
                        const long long t = m.frame_lo + nf - 1;
                        const long long e = m.audio_off + t * c.hop - (m.centered ? c.n_fft / 2 : 0) + c.n_fft;
                        end0[i] = std::max(end0[i], std::min(e, m.audio_off + m.len));
                    }
                }
                if (nparts && ((i + 1) % kUploadClips == 0 || i + 1 == nb))
                    pparts[ph].emplace_back(ptot_frames[ph], upload_ev_[ph * nparts + i / kUploadClips]);
            }
        }
        if (!d_audio_in) {
            float* buf = (float*)ws("audio", (size_t)std::max(total_samples, 1LL) * 4);
            // the previous batch's mel has read the buffer before the upload overwrites it
            N3D_CUDA(cudaEventRecord(upload_start_, stream_));
            N3D_CUDA(cudaStreamWaitEvent(copy_stream_, upload_start_, 0));
            for (int ph = 0; ph < 2; ph++)
                for (int k = 0; k < nparts; k++) {
                    for (int i = k * kUploadClips; i < std::min(nb, (k + 1) * kUploadClips); i++) {
                        const long long n = lens[c0 + i], e = std::min(std::max(end0[i], 0LL), n);
                        const long long s0 = ph == 0 ? 0 : e, s1 = ph == 0 ? e : n;
                        if (s1 > s0)
                            N3D_CUDA(cudaMemcpyAsync(buf + aoff[i] + s0, host_audio[c0 + i] + s0, (s1 - s0) * 4,
                                                     cudaMemcpyHostToDevice, copy_stream_));
                    }
                    N3D_CUDA(cudaEventRecord(upload_ev_[ph * nparts + k], copy_stream_));
                }
            d_audio = buf;
        }
        std::vector<MelJob> jobs;
        for (int ph = 0; ph < nphase; ph++)
            jobs.push_back(mel_prepare(pbase[ph], pseg[ph], ptot_groups[ph], ptot_frames[ph], ph ? "1" : ""));
        const float* emb_phase[2] = {nullptr, nullptr};
        emb_phase[0] = mel_launch(d_audio, jobs[0], nparts ? &pparts[0] : nullptr);
        // ---- per-clip state and outputs
        int max_steps = 0;
        long long out_total = 0;
        std::vector<long long> out_base(nb);
        for (int i = 0; i < nb; i++) {
            max_steps = std::max(max_steps, (int)plans[c0 + i].steps.size());
            out_base[i] = out_total;
            out_total += plans[c0 + i].emitted_rows;
        }
        const long long pre_rows = s_cap_;
        float* pre = (float*)ws("pre", (size_t)2 * nb * pre_rows * h * 4);
        float* cprob = (float*)ws("cprob", (size_t)2 * nb * pre_rows * ns * 4);
        float* outl = (float*)ws("out_logits", std::max(out_total, 1LL) * ns * 4);
        // ---- step table (all steps, compact per step)
        std::vector<SeqStep> table;
        std::vector<int> seq_len, valid;
        std::vector<int> step_first(max_steps + 1), step_S(max_steps);
        std::vector<long long> out_cursor(out_base);
        for (int w = 0; w < max_steps; w++) {
            step_first[w] = (int)table.size();
            int Smax = 0;
            for (int i = 0; i < nb; i++) {
                const ClipPlan& p = plans[c0 + i];
                if (w >= (int)p.steps.size()) continue;
                const StepPlan& sp = p.steps[w];
                if (sp.S == 0) continue;  // an empty final chunk changes nothing
                SeqStep q{};
                q.S = sp.S;
                q.valid = sp.valid;
                q.ncache = sp.ncache;
                q.nfifo = sp.nfifo;
                q.nchunk = sp.nchunk;
                q.popped = sp.popped;
                q.compress = sp.compress;
                q.was_compressed = sp.was_compressed;
                q.keep_rows = sp.keep_rows;
                const PartRef& pr = ref[i][sp.seg][nphase == 2 && w > 0 ? 1 : 0];
                // reused rows: the previous step's last rows, which end where this
                // step's segment begins in the same phase
                q.emb_row = pr.base + (sp.group_lo - pr.lo) - sp.reuse;
                const int cur = w & 1, nxt = cur ^ 1;
                q.pre_in = pre + ((size_t)cur * nb + i) * pre_rows * h;
                q.pre_out = pre + ((size_t)nxt * nb + i) * pre_rows * h;
                q.cp_in = cprob + ((size_t)cur * nb + i) * pre_rows * ns;
                q.cp_out = cprob + ((size_t)nxt * nb + i) * pre_rows * ns;
                q.out_logits = outl + out_cursor[i] * ns;
                out_cursor[i] += sp.keep_rows;
                if (sp.S > s_cap_) throw Error(kStatusGpu, "window of " + std::to_string(sp.S) + " frames exceeds 1024");
                table.push_back(q);
                seq_len.push_back(sp.S);
                valid.push_back(sp.valid);
                Smax = std::max(Smax, sp.S);
            }
            step_S[w] = (Smax + 7) / 8 * 8;  // row stride: a multiple of 8 keeps TMA coordinates 16-byte aligned
        }
        step_first[max_steps] = (int)table.size();
        // Clips whose plans skip a step (S == 0) must still carry state forward:
        // that can only happen on a final empty chunk, after which nothing reads it.
        if (!table.empty()) {
            SeqStep* d_table = (SeqStep*)ws("steps", table.size() * sizeof(SeqStep));
            int* d_len = (int*)ws("seq_len", table.size() * 4);
            int* d_valid = (int*)ws("valid", table.size() * 4);
            N3D_CUDA(cudaMemcpyAsync(d_table, table.data(), table.size() * sizeof(SeqStep), cudaMemcpyHostToDevice,
                                     stream_));
            N3D_CUDA(cudaMemcpyAsync(d_len, seq_len.data(), seq_len.size() * 4, cudaMemcpyHostToDevice, stream_));
            N3D_CUDA(cudaMemcpyAsync(d_valid, valid.data(), valid.size() * 4, cudaMemcpyHostToDevice, stream_));
            for (int w = 0; w < max_steps; w++) {
                if (w == 1 && nphase == 2)  // the later steps' groups, once their audio is up
                    emb_phase[1] = mel_launch(d_audio, jobs[1], nparts ? &pparts[1] : nullptr);
                const int B = step_first[w + 1] - step_first[w];
                if (B == 0) continue;
                run_step(d_table + step_first[w], B, step_S[w], d_len + step_first[w], d_valid + step_first[w],
                         emb_phase[nphase == 2 && w > 0 ? 1 : 0]);
            }
        }
        // the caller may release its audio once this returns: every upload has finished
        if (nparts) N3D_CUDA(cudaStreamSynchronize(copy_stream_));
        // ---- results
        if (host_out) {
            // one copy into pinned staging, then into the caller's buffers (a few host
            // threads share the copies of a large batch)
            float* stage = host_stage((size_t)std::max(out_total, 1LL) * ns * 4);
            if (out_total)
                N3D_CUDA(cudaMemcpyAsync(stage, outl, out_total * ns * 4, cudaMemcpyDeviceToHost, stream_));
            N3D_CUDA(cudaStreamSynchronize(stream_));
            std::vector<float*> dst(nb);
            for (int i = 0; i < nb; i++) dst[i] = (*host_out)(c0 + i, (size_t)plans[c0 + i].out_rows * ns);
            auto copy_range = [&](int i0, int i1) {
                for (int i = i0; i < i1; i++)
                    if (plans[c0 + i].out_rows)
                        std::memcpy(dst[i], stage + out_base[i] * ns, (size_t)plans[c0 + i].out_rows * ns * 4);
            };
            const int nthreads = (size_t)out_total * ns * 4 >= (4u << 20) ? std::min(8, nb) : 1;
            if (nthreads <= 1) {
                copy_range(0, nb);
            } else {
                std::vector<std::thread> pool;
                for (int t = 0; t < nthreads; t++)
                    pool.emplace_back(copy_range, nb * t / nthreads, nb * (t + 1) / nthreads);
                for (std::thread& th : pool) th.join();
            }
        } else {
            for (int i = 0; i < nb; i++) {
                const ClipPlan& p = plans[c0 + i];
                if (p.out_rows)
                    N3D_CUDA(cudaMemcpyAsync(d_logits + (*out_offsets)[c0 + i] * ns, outl + out_base[i] * ns,
                                             p.out_rows * ns * 4, cudaMemcpyDeviceToDevice, stream_));
            }
            N3D_CUDA(cudaStreamSynchronize(stream_));
        }
        prof_collect();
        check_dev_error();
    }
}

// Log-mel of every segment (segment i's samples start at d_audio[base[i]]) into one
// split [groups·sub, n_mels] array, then one embedder GEMM over all groups ->
// [total_groups, hidden] (src/mel.rs:160-225, src/encoder.rs:126-146).
Model::MelJob Model::mel_prepare(const std::vector<long long>& base, const std::vector<MelSeg>& segs,
                                 long long total_groups, long long total_frames, const char* tag) {
    const Config& c = cfg_;
    const int sub = c.sub;
    MelJob job;
    job.groups = total_groups;
    job.frames = total_frames;
    job.tag = tag;
    if (total_frames <= 0) return job;
    std::vector<MelSegDev> table;
    table.reserve(segs.size());
    long long f = 0;
    for (size_t i = 0; i < segs.size(); i++) {
        const MelSeg& s = segs[i];
        const int nf = mel_frames(s, sub);
        if (nf == 0) continue;
        if (s.len > INT_MAX) throw Error(kStatusArg, "mel segment longer than 2^31 samples");
        table.push_back(MelSegDev{base[i], s.group_base * sub, f, (int)s.len, s.frame_lo, s.centered, 0});
        f += nf;
    }
    if (f != total_frames) throw Error(kStatusGpu, "mel_prepare: frame count mismatch");
    MelSegDev* d_segs = (MelSegDev*)ws(("melseg" + job.tag).c_str(), table.size() * sizeof(MelSegDev));
    N3D_CUDA(cudaMemcpyAsync(d_segs, table.data(), table.size() * sizeof(MelSegDev), cudaMemcpyHostToDevice, stream_));
    job.segs = d_segs;
    job.nsegs = (int)table.size();
    return job;
}

const float* Model::mel_launch(const float* d_audio, const MelJob& job,
                               const std::vector<std::pair<long long, cudaEvent_t>>* parts) {
    const Config& c = cfg_;
    const int h = c.hidden, sub = c.sub;
    const long long mel_rows = std::max(job.groups * sub, 1LL);
    const SplitBuf mel = ws2("mel" + job.tag, mel_rows, c.n_mels);  // rows past a segment's frames stay zero
    N3D_CUDA(cudaMemsetAsync(mel.h, 0, mel_rows * c.n_mels * 2, stream_));
    N3D_CUDA(cudaMemsetAsync(mel.l, 0, mel_rows * c.n_mels * 2, stream_));
    if (job.frames > 0) {
        prof_begin();
        if (parts) {
            long long f0 = 0;
            for (const auto& pt : *parts) {
                N3D_CUDA(cudaStreamWaitEvent(stream_, pt.second, 0));
                launch_mel(stream_, d_audio, job.segs, job.nsegs, f0, pt.first - f0, c.hop, mel_tab_, c.preemph,
                           mel.out(s_mel_), nullptr);
                f0 = pt.first;
            }
        } else {
            launch_mel(stream_, d_audio, job.segs, job.nsegs, 0, job.frames, c.hop, mel_tab_, c.preemph, mel.out(s_mel_),
                       nullptr);
        }
        prof_end(K_MEL, 0, (double)job.frames * (c.hop * 4 + c.n_mels * 4));
    }
    const long long K_emb = (long long)sub * c.n_mels;
    float* embeds = (float*)ws(("embeds" + job.tag).c_str(), std::max(job.groups, 1LL) * h * 4);
    if (job.groups > 0) {
        Epi e;
        e.mode = EPI_STORE;
        e.out = embeds;
        e.ldo = h;
        // the [rows, 128] mel viewed as [groups, 8 * 128]: 8 stacked frames per row
        const SplitOperand A{mel.h, mel.l, mel.rows_cap / sub, K_emb, K_emb, s_mel_};
        prof_begin();
        gemm_split(stream_, A, embed_.op(), (int)job.groups, h, (int)K_emb, 0, e, dev_err_);
        prof_end(K_GEMM_EMBED, 2.0 * job.groups * h * K_emb, 0);
    }
    return embeds;
}

void Model::tower_step(int B, int S, const int* d_len, const int* d_valid) {
    if (B > kGraphMaxSeqs || prof_) {
        tower(B, S, d_len, d_valid, nullptr);
        return;
    }
    int* len_slot = (int*)ws("graph_len", (size_t)B * 4);
    int* valid_slot = (int*)ws("graph_valid", (size_t)B * 4);
    N3D_CUDA(cudaMemcpyAsync(len_slot, d_len, (size_t)B * 4, cudaMemcpyDeviceToDevice, stream_));
    N3D_CUDA(cudaMemcpyAsync(valid_slot, d_valid, (size_t)B * 4, cudaMemcpyDeviceToDevice, stream_));
    const std::pair<int, int> key{B, S};
    auto it = tower_graphs_.find(key);
    if (it == tower_graphs_.end()) {  // first step of this shape: eager
        tower(B, S, len_slot, valid_slot, nullptr);
        tower_graphs_.emplace(key, TowerGraph{});
        return;
    }
    TowerGraph& g = it->second;
    if (!g.exec || g.gen != ws_gen_) {
        if (g.exec) N3D_CUDA(cudaGraphExecDestroy(g.exec));
        g.exec = nullptr;
        // bound the host memory of cached graphs (~220 kernel nodes each): past
        // kGraphCacheMax captured shapes, drop them all and start over
        int captured = 0;
        for (const auto& kv : tower_graphs_) captured += kv.second.exec != nullptr;
        if (captured >= kGraphCacheMax) {
            N3D_CUDA(cudaStreamSynchronize(stream_));
            for (auto& kv : tower_graphs_)
                if (kv.second.exec) {
                    N3D_CUDA(cudaGraphExecDestroy(kv.second.exec));
                    kv.second.exec = nullptr;
                }
        }
        // capture on a private stream (the caller's stream may be the legacy default
        // stream); every workspace buffer already has its size, so nothing allocates
        const uint64_t gen = ws_gen_;
        cudaStream_t caller = stream_;
        cudaGraph_t graph = nullptr;
        N3D_CUDA(cudaStreamBeginCapture(capture_stream_, cudaStreamCaptureModeThreadLocal));
        stream_ = capture_stream_;
        try {
            tower(B, S, len_slot, valid_slot, nullptr);
        } catch (...) {
            stream_ = caller;
            cudaStreamEndCapture(capture_stream_, &graph);
            if (graph) cudaGraphDestroy(graph);
            throw;
        }
        stream_ = caller;
        N3D_CUDA(cudaStreamEndCapture(capture_stream_, &graph));
        const cudaError_t e = cudaGraphInstantiate(&g.exec, graph, 0);
        cudaGraphDestroy(graph);
        N3D_CUDA(e);
        if (ws_gen_ != gen) throw Error(kStatusGpu, "tower graph: the workspace changed during capture");
        g.gen = gen;
    }
    N3D_CUDA(cudaGraphLaunch(g.exec, stream_));
}

void Model::run_step(const SeqStep* d_st, int B, int S, const int* d_len, const int* d_valid, const float* embeds) {
    const Config& c = cfg_;
    const int h = c.hidden;
    float* win = (float*)ws("win", (size_t)B * S * h * 4);
    cudaEvent_t step_begin = nullptr;
    if (step_timing_) {
        step_begin = pool_event();
        N3D_CUDA(cudaEventRecord(step_begin, stream_));
    }
    prof_begin();
    launch_assemble(stream_, d_st, B, embeds, win, S, h);
    prof_end(K_ASSEMBLE, 0, 2.0 * B * S * h * 4);
    tower_step(B, S, d_len, d_valid);
    head(B, S, d_len);
    const CacheConst cc{h, c.num_speakers, c.sub, c.cache_len, c.n_sil, c.min_pos, c.k_strong, c.k_weak, c.thr,
                        c.latest_boost};
    prof_begin();
    launch_cache_update(stream_, d_st, B, (float*)ws("win", 0), (float*)ws("logits", 0), S, cc, silence_);
    prof_end(K_CACHE, 0, 0);
    if (step_timing_) {
        cudaEvent_t step_end = pool_event();
        N3D_CUDA(cudaEventRecord(step_end, stream_));
        step_ev_.emplace_back(step_begin, step_end);
    }
}

// ------------------------------------------------------------ sessions

struct Model::SessionChunk {
    Session* s;
    int idx;             // position in the caller's list
    long long off, len;  // samples, absolute
    int centered, la;
    bool last;
};

namespace {

// The next chunk of `s` whose samples are all present: plan_streaming's chunk list,
// decided as audio arrives (`final`: no more audio will come).
bool next_session_chunk(const Config& c, const Session& s, bool final, Model::SessionChunk& ch) {
    if (s.done) return false;
    const int cl = c.modes[s.mode][0], rc = c.modes[s.mode][1];
    const long long mel_chunk = (long long)(cl + rc) * c.sub, mel_step = (long long)cl * c.sub;
    const long long first = (mel_chunk - 1) * c.hop + c.win / 2;
    const long long per_chunk = mel_chunk * c.hop + c.win;
    const long long n = s.received;
    if (s.next_chunk == 0) {
        if (n < first && !final) return false;
        ch.off = 0, ch.len = std::min(first, n), ch.centered = 1, ch.la = rc, ch.last = false;
        return true;
    }
    const long long start = (long long)s.next_chunk * mel_step * c.hop - c.n_fft / 2;
    if (start + per_chunk <= n) {
        ch.off = start, ch.len = per_chunk, ch.centered = 0, ch.la = rc, ch.last = false;
        return true;
    }
    if (!final) return false;
    ch.off = std::min(start, n), ch.len = n - ch.off, ch.centered = 1, ch.la = 0, ch.last = true;
    return true;
}

}  // namespace

Session* Model::session_open(int mode) {
    if (mode < 0 || mode > 2) throw Error(kStatusArg, "streaming mode must be low, very low or ultra low latency");
    N3D_CUDA(cudaSetDevice(device_));
    auto s = std::make_unique<Session>();
    s->model = this;
    s->mode = mode;
    const size_t pre_bytes = (size_t)2 * s_cap_ * cfg_.hidden * 4, cp_bytes = (size_t)2 * s_cap_ * cfg_.num_speakers * 4;
    N3D_CUDA(cudaMalloc(&s->pre, pre_bytes));
    if (cudaMalloc(&s->cprob, cp_bytes) != cudaSuccess) {
        cudaFree(s->pre);
        throw Error(kStatusCuda, "CUDA error in session state allocation: out of device memory");
    }
    return s.release();
}

void Model::session_free(Session* s) {
    if (!s) return;
    cudaSetDevice(device_);
    cudaStreamSynchronize(stream_);  // no step of this session is still in flight
    cudaFree(s->pre);
    cudaFree(s->cprob);
    delete s;
}

void Model::sessions_push(const std::vector<Session*>& ss, const std::vector<const float*>& samples,
                          const std::vector<long long>& lens, bool close, std::vector<std::vector<float>>& rows) {
    N3D_CUDA(cudaSetDevice(device_));
    const int n = (int)ss.size();
    for (int i = 0; i < n; i++) {
        const Session* s = ss[i];
        if (!s || s->model != this) throw Error(kStatusArg, "session does not belong to this model");
        if (s->failed) throw Error(kStatusArg, "session failed in an earlier call; free it");
        if (s->closed) throw Error(kStatusArg, "session is closed");
        for (int j = 0; j < i; j++)
            if (ss[j] == s) throw Error(kStatusArg, "a session appears twice in one call");
    }
    rows.assign(n, {});
    try {
        for (int i = 0; i < n; i++) {
            if (lens[i] > 0) ss[i]->audio.insert(ss[i]->audio.end(), samples[i], samples[i] + lens[i]);
            ss[i]->received += lens[i];
        }
        for (;;) {  // one round = the next ready chunk of every session
            std::vector<SessionChunk> items;
            for (int i = 0; i < n; i++) {
                SessionChunk ch{};
                ch.s = ss[i];
                ch.idx = i;
                if (next_session_chunk(cfg_, *ss[i], close, ch)) items.push_back(ch);
            }
            if (items.empty()) break;
            session_round(items, rows);
        }
        if (close)
            for (Session* s : ss) s->closed = true;
    } catch (...) {
        for (Session* s : ss) s->failed = true;
        throw;
    }
}

void Model::session_round(std::vector<SessionChunk>& items, std::vector<std::vector<float>>& rows) {
    const Config& c = cfg_;
    const int ns = c.num_speakers, h = c.hidden, sub = c.sub;
    const int nb = (int)items.size();
    // ---- step plans; the cache counts advance exactly as in plan_streaming
    std::vector<MelSeg> segs(nb);
    std::vector<StepPlan> sps(nb);
    std::vector<long long> aoff(nb);
    long long total_samples = 0, total_groups = 0, total_frames = 0;
    for (int i = 0; i < nb; i++) {
        const SessionChunk& it = items[i];
        Session& s = *it.s;
        const long long nm = frame_count(c, it.len, it.centered != 0);
        const long long groups = ceil_div(nm, sub);
        if (groups < it.la)
            throw Error(kStatusAudio, "unsupported audio: a streaming chunk holds " + std::to_string(groups) +
                                          " encoder frames, fewer than the look-ahead of " + std::to_string(it.la));
        segs[i] = MelSeg{0, it.len, it.centered, (int)nm, (int)groups, total_groups};
        aoff[i] = total_samples;
        total_samples += it.len;
        total_groups += groups;
        total_frames += nm;
        StepPlan sp{};
        sp.n_new = (int)groups;
        sp.nchunk = (int)(groups - it.la);
        sp.S = s.ncache + s.nfifo + sp.n_new;
        sp.valid = sp.S;
        sp.keep_rows = (int)std::min((long long)sp.nchunk * sub, nm);
        if (sp.S > s_cap_) throw Error(kStatusGpu, "window of " + std::to_string(sp.S) + " frames exceeds 1024");
        CacheSim cs{c.s_fifo, c.s_period, c.cache_len};
        cs.ncache = s.ncache;
        cs.nfifo = s.nfifo;
        cs.compressed = s.compressed;
        cs.step(sp);
        s.ncache = cs.ncache;
        s.nfifo = cs.nfifo;
        s.compressed = cs.compressed;
        sps[i] = sp;
    }
    // ---- the chunks' audio, log-mel, embedder
    float* d_audio = (float*)ws("s_audio", (size_t)std::max(total_samples, 1LL) * 4);
    for (int i = 0; i < nb; i++) {
        const SessionChunk& it = items[i];
        if (it.len > 0)  // pageable source: returns once the samples are staged, so trimming below is safe
            N3D_CUDA(cudaMemcpyAsync(d_audio + aoff[i], it.s->audio.data() + (it.off - it.s->base), it.len * 4,
                                     cudaMemcpyHostToDevice, stream_));
    }
    const float* embeds = mel_embed(d_audio, aoff, segs, total_groups, total_frames);
    // ---- one step per session
    long long out_total = 0;
    std::vector<long long> out_base(nb);
    for (int i = 0; i < nb; i++) {
        out_base[i] = out_total;
        out_total += sps[i].keep_rows;
    }
    float* outl = (float*)ws("s_out", (size_t)std::max(out_total, 1LL) * ns * 4);
    std::vector<SeqStep> table;
    std::vector<int> seq_len, valid;
    int Smax = 0;
    for (int i = 0; i < nb; i++) {
        const StepPlan& sp = sps[i];
        if (sp.S == 0) continue;  // nothing cached and no new frames: the step changes nothing
        Session& s = *items[i].s;
        const int cur = (int)(s.steps & 1), nxt = cur ^ 1;
        SeqStep q{};
        q.S = sp.S;
        q.valid = sp.valid;
        q.ncache = sp.ncache;
        q.nfifo = sp.nfifo;
        q.nchunk = sp.nchunk;
        q.popped = sp.popped;
        q.compress = sp.compress;
        q.was_compressed = sp.was_compressed;
        q.keep_rows = sp.keep_rows;
        q.emb_row = segs[i].group_base;
        q.pre_in = s.pre + (size_t)cur * s_cap_ * h;
        q.pre_out = s.pre + (size_t)nxt * s_cap_ * h;
        q.cp_in = s.cprob + (size_t)cur * s_cap_ * ns;
        q.cp_out = s.cprob + (size_t)nxt * s_cap_ * ns;
        q.out_logits = outl + out_base[i] * ns;
        table.push_back(q);
        seq_len.push_back(sp.S);
        valid.push_back(sp.valid);
        Smax = std::max(Smax, sp.S);
        s.steps++;
    }
    if (!table.empty()) {
        SeqStep* d_table = (SeqStep*)ws("s_steps", table.size() * sizeof(SeqStep));
        int* d_len = (int*)ws("s_seq_len", table.size() * 4);
        int* d_valid = (int*)ws("s_valid", table.size() * 4);
        N3D_CUDA(cudaMemcpyAsync(d_table, table.data(), table.size() * sizeof(SeqStep), cudaMemcpyHostToDevice,
                                 stream_));
        N3D_CUDA(cudaMemcpyAsync(d_len, seq_len.data(), seq_len.size() * 4, cudaMemcpyHostToDevice, stream_));
        N3D_CUDA(cudaMemcpyAsync(d_valid, valid.data(), valid.size() * 4, cudaMemcpyHostToDevice, stream_));
        run_step(d_table, (int)table.size(), (Smax + 7) / 8 * 8, d_len, d_valid, embeds);
    }
    // ---- new rows
    std::vector<float> out((size_t)out_total * ns);
    if (out_total)
        N3D_CUDA(cudaMemcpyAsync(out.data(), outl, out.size() * 4, cudaMemcpyDeviceToHost, stream_));
    N3D_CUDA(cudaStreamSynchronize(stream_));
    prof_collect();
    check_dev_error();
    for (int i = 0; i < nb; i++) {
        std::vector<float>& r = rows[items[i].idx];
        r.insert(r.end(), out.begin() + out_base[i] * ns, out.begin() + (out_base[i] + sps[i].keep_rows) * ns);
    }
    // ---- advance the schedules; drop the samples no later chunk reads
    for (int i = 0; i < nb; i++) {
        Session& s = *items[i].s;
        s.next_chunk++;
        s.num_chunks++;
        if (items[i].last) {
            s.done = true;
            s.audio.clear();
            s.audio.shrink_to_fit();
            s.base = s.received;
            continue;
        }
        const long long mel_step = (long long)c.modes[s.mode][0] * sub;
        const long long keep_from = std::min((long long)s.next_chunk * mel_step * c.hop - c.n_fft / 2, s.received);
        if (keep_from > s.base) {
            s.audio.erase(s.audio.begin(), s.audio.begin() + (keep_from - s.base));
            s.base = keep_from;
        }
    }
}

// ------------------------------------------------------------ stage APIs

int Model::log_mel(const float* samples, long long n, bool centered, std::vector<float>& out) {
    const Config& c = cfg_;
    N3D_CUDA(cudaSetDevice(device_));
    const long long frames = frame_count(c, n, centered);
    out.assign((size_t)frames * c.n_mels, 0.0f);
    if (frames == 0) return 0;
    float* a = (float*)ws("audio", n * 4);
    N3D_CUDA(cudaMemcpyAsync(a, samples, n * 4, cudaMemcpyHostToDevice, stream_));
    if (n > INT_MAX) throw Error(kStatusArg, "log_mel: more than 2^31 samples");
    const MelSegDev seg{0, 0, 0, (int)n, 0, centered ? 1 : 0, 0};
    MelSegDev* d_seg = (MelSegDev*)ws("melseg", sizeof(MelSegDev));
    float* pl = (float*)ws("mel_plain", frames * c.n_mels * 4);
    N3D_CUDA(cudaMemcpyAsync(d_seg, &seg, sizeof(MelSegDev), cudaMemcpyHostToDevice, stream_));
    launch_mel(stream_, a, d_seg, 1, 0, frames, c.hop, mel_tab_, c.preemph,
               SplitOut{}, pl);
    N3D_CUDA(cudaMemcpyAsync(out.data(), pl, frames * c.n_mels * 4, cudaMemcpyDeviceToHost, stream_));
    N3D_CUDA(cudaStreamSynchronize(stream_));
    return (int)frames;
}

void Model::embed_range(const float* mel, long long num_frames, long long lo, long long hi, float* out) {
    const Config& c = cfg_;
    N3D_CUDA(cudaSetDevice(device_));
    const long long groups = hi - lo, K = (long long)c.sub * c.n_mels;
    if (groups <= 0) return;
    std::vector<float> buf((size_t)groups * K, 0.0f);
    const long long end = std::min(hi * c.sub, num_frames);
    if (lo * c.sub < end) std::memcpy(buf.data(), mel + lo * c.sub * c.n_mels, (end - lo * c.sub) * c.n_mels * 4);
    float* plain = (float*)ws("stage_in", groups * K * 4);
    const SplitBuf sp = ws2("stage_split", groups, K);
    float* o = (float*)ws("embeds", groups * c.hidden * 4);
    N3D_CUDA(cudaMemcpyAsync(plain, buf.data(), groups * K * 4, cudaMemcpyHostToDevice, stream_));
    const float sc = dyn_scale(plain, groups * K);  // caller data: scaled by its own max
    launch_split(stream_, plain, groups * K, sp.out(sc));
    Epi e;
    e.mode = EPI_STORE;
    e.out = o;
    e.ldo = c.hidden;
    gemm_split(stream_, sp.op(sc), embed_.op(), (int)groups, c.hidden, (int)K, 0, e, dev_err_);
    N3D_CUDA(cudaMemcpyAsync(out, o, groups * c.hidden * 4, cudaMemcpyDeviceToHost, stream_));
    N3D_CUDA(cudaStreamSynchronize(stream_));
    check_dev_error();
}

void Model::forward_window(const float* embeds, int frames, int valid, float* enc_out, float* logits) {
    const Config& c = cfg_;
    N3D_CUDA(cudaSetDevice(device_));
    if (frames <= 0 || frames > s_cap_)
        throw Error(kStatusGpu, "seq " + std::to_string(frames) + " outside 1..=1024");
    valid = std::min(valid, frames);
    const int S = (frames + 7) / 8 * 8;  // row stride (multiple of 8), rows past `frames` are zero
    const long long M = frames, h = c.hidden;
    float* win = (float*)ws("win", (long long)S * h * 4);
    N3D_CUDA(cudaMemsetAsync(win, 0, (long long)S * h * 4, stream_));
    N3D_CUDA(cudaMemcpyAsync(win, embeds, M * h * 4, cudaMemcpyHostToDevice, stream_));
    int* d_len = (int*)ws("seq_len", 4);
    int* d_valid = (int*)ws("valid", 4);
    N3D_CUDA(cudaMemcpyAsync(d_len, &frames, 4, cudaMemcpyHostToDevice, stream_));
    N3D_CUDA(cudaMemcpyAsync(d_valid, &valid, 4, cudaMemcpyHostToDevice, stream_));
    float* enc = enc_out ? (float*)ws("enc_plain", (long long)S * h * 4) : nullptr;
    tower(1, S, d_len, d_valid, enc);
    if (enc_out) N3D_CUDA(cudaMemcpyAsync(enc_out, enc, M * h * 4, cudaMemcpyDeviceToHost, stream_));
    if (logits) {
        head(1, S, d_len);
        N3D_CUDA(cudaMemcpyAsync(logits, ws("logits", 0), M * c.sub * c.num_speakers * 4, cudaMemcpyDeviceToHost,
                                 stream_));
    }
    N3D_CUDA(cudaStreamSynchronize(stream_));
    check_dev_error();
}

void Model::head_forward(const float* enc, int frames, float* logits) {
    const Config& c = cfg_;
    N3D_CUDA(cudaSetDevice(device_));
    if (frames <= 0 || frames > s_cap_)
        throw Error(kStatusGpu, "head frames " + std::to_string(frames) + " outside 1..=1024");
    const int S = (frames + 7) / 8 * 8;
    const long long M = frames, h = c.hidden;
    float* plain = (float*)ws("enc_plain", (long long)S * h * 4);
    const SplitBuf n = ws2("n", S, h);
    N3D_CUDA(cudaMemsetAsync(plain, 0, (long long)S * h * 4, stream_));
    N3D_CUDA(cudaMemcpyAsync(plain, enc, M * h * 4, cudaMemcpyHostToDevice, stream_));
    // caller data: scaled like the final LayerNorm's output when it respects that
    // bound, else by a power of two more (and proj's and the conv's outputs with it)
    const float sc = dyn_scale(plain, (long long)S * h);
    const float widen = sc < s_fin_ ? s_fin_ / sc : 1.0f;
    launch_split(stream_, plain, (long long)S * h, n.out(s_fin_ / widen));
    int* d_len = (int*)ws("seq_len", 4);
    N3D_CUDA(cudaMemcpyAsync(d_len, &frames, 4, cudaMemcpyHostToDevice, stream_));
    head(1, S, d_len, widen);
    N3D_CUDA(cudaMemcpyAsync(logits, ws("logits", 0), M * c.sub * c.num_speakers * 4, cudaMemcpyDeviceToHost,
                             stream_));
    N3D_CUDA(cudaStreamSynchronize(stream_));
    check_dev_error();
}

}  // namespace n3d
