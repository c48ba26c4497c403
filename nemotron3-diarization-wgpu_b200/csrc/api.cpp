// extern "C" boundary (include/n3d.h): status codes, thread-local error
// messages, ownership of returned buffers, and the host-only pieces of the
// reference API (extract_speaker_dict, activity_stats).

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
#include <memory>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/n3d.h"
#include "model.h"

struct n3d_model {
    std::unique_ptr<n3d::Model> m;
    std::string describe;  // n3d_model_describe's last answer
};

struct n3d_session {
    n3d_model* owner;
    n3d::Session* s;
};

struct n3d_config {
    n3d::Config c;
};

namespace {

thread_local std::string g_last_error;

template <class F>
n3d_status guarded(F&& f) {
    try {
        f();
        g_last_error.clear();
        return N3D_OK;
    } catch (const n3d::Error& e) {
        g_last_error = e.what();
        return (n3d_status)e.status;
    } catch (const std::bad_alloc&) {
        g_last_error = "out of host memory";
        return N3D_ERR_GPU;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return N3D_ERR_GPU;
    }
}

void arg_check(bool ok, const char* what) {
    if (!ok) throw n3d::Error(N3D_ERR_INVALID_ARGUMENT, what);
}

void fill_output(n3d_run_output* out, std::vector<float>& logits, const n3d::ClipPlan& p, size_t ns) {
    out->num_speakers = ns;
    out->num_frames = logits.size() / ns;
    out->logits = (float*)std::malloc(std::max<size_t>(logits.size(), 1) * sizeof(float));
    if (!out->logits) throw std::bad_alloc();
    if (!logits.empty()) std::memcpy(out->logits, logits.data(), logits.size() * sizeof(float));
    out->num_chunks = (size_t)p.num_chunks;
    out->cache_compressed = p.cache_compressed;
    out->cache_frames = (size_t)p.cache_frames;
    out->fifo_frames = (size_t)p.fifo_frames;
}

// Run outputs whose logits run_batch writes in place: the sink allocates each clip's
// array in its n3d_run_output; the remaining fields come from the plans afterwards.
// On an exception every array allocated so far is freed.
void run_batch_to_outputs(n3d::Model& m, int mode, const std::vector<const float*>& audio,
                          const std::vector<long long>& lens, n3d_run_output* outs) {
    const size_t n = lens.size(), ns = (size_t)m.cfg().num_speakers;
    for (size_t i = 0; i < n; i++) std::memset(&outs[i], 0, sizeof(outs[i]));
    std::vector<n3d::ClipPlan> plans;
    const n3d::Model::HostSink sink = [&](int clip, size_t count) {
        float* p = (float*)std::malloc(std::max<size_t>(count, 1) * sizeof(float));
        if (!p) throw std::bad_alloc();
        outs[clip].logits = p;
        outs[clip].num_frames = count / ns;
        return p;
    };
    try {
        m.run_batch(mode, audio, nullptr, std::vector<long long>(n, 0), lens, &sink, nullptr, nullptr, &plans);
    } catch (...) {
        for (size_t i = 0; i < n; i++) {
            std::free(outs[i].logits);
            outs[i].logits = nullptr;
        }
        throw;
    }
    for (size_t i = 0; i < n; i++) {
        outs[i].num_speakers = ns;
        outs[i].num_chunks = (size_t)plans[i].num_chunks;
        outs[i].cache_compressed = plans[i].cache_compressed;
        outs[i].cache_frames = (size_t)plans[i].cache_frames;
        outs[i].fifo_frames = (size_t)plans[i].fifo_frames;
    }
}

// torch.sigmoid in fp32 (src/segments.rs:41-43)
float sigmoidf(float x) { return 1.0f / (1.0f + std::exp(-x)); }

// Python round(x, 2), half to even (src/segments.rs:51-62)
float round2(float v) {
    const double scaled = (double)v * 100.0;
    double r = std::round(scaled);
    if (std::fabs(scaled - std::trunc(scaled)) == 0.5) {
        const double t = std::trunc(scaled);
        r = ((long long)t % 2 == 0) ? t : t + 1.0;
    }
    return (float)(r / 100.0);
}

// Per-device stream and error word of the single-kernel entry points.  A call holds
// `call` from its first launch to its last check, so calls on one device from several
// threads take turns instead of mixing their launches and error reports.
struct KernelCtx {
    std::mutex call;
    cudaStream_t stream = nullptr;
    int* err = nullptr;
};
KernelCtx& kctx(int device) {
    static std::mutex mu;
    static KernelCtx ctxs[64];
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0 || device >= 64) throw n3d::Error(N3D_ERR_NO_DEVICE, "bad device index");
    KernelCtx& k = ctxs[device];
    if (!k.stream) {
        N3D_CUDA(cudaSetDevice(device));
        N3D_CUDA(cudaStreamCreateWithFlags(&k.stream, cudaStreamNonBlocking));
        N3D_CUDA(cudaMalloc(&k.err, sizeof(int)));
        N3D_CUDA(cudaMemset(k.err, 0, sizeof(int)));
    }
    return k;
}
void kcheck(KernelCtx& k) {
    N3D_CUDA(cudaStreamSynchronize(k.stream));
    int e = 0;
    N3D_CUDA(cudaMemcpy(&e, k.err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) {
        N3D_CUDA(cudaMemset(k.err, 0, sizeof(int)));
        throw n3d::Error(N3D_ERR_TIMEOUT, "a device-side wait timed out (site " + std::to_string(e) + ")");
    }
}

struct DevScratch {
    std::vector<void*> ptrs;
    float* get(size_t n) {
        void* p = nullptr;
        N3D_CUDA(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(float) + 256));
        ptrs.push_back(p);
        return (float*)p;
    }
    ~DevScratch() {
        for (void* p : ptrs) cudaFree(p);
    }
};

// The fp16-split scales of up to four device operands from their max |x| (one
// readback); grow[i] widens operand i's bound (RoPE may double a Q or K element).
void operand_scales(KernelCtx& k, DevScratch& sc, std::initializer_list<std::pair<const float*, size_t>> ops,
                    float* out, const double* grow = nullptr) {
    float* m = sc.get(4);
    N3D_CUDA(cudaMemsetAsync(m, 0, 16, k.stream));
    int i = 0;
    for (const auto& o : ops) n3d::launch_absmax(k.stream, o.first, (long long)o.second, m + i++);
    float hm[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    N3D_CUDA(cudaMemcpyAsync(hm, m, 16, cudaMemcpyDeviceToHost, k.stream));
    N3D_CUDA(cudaStreamSynchronize(k.stream));
    for (int j = 0; j < i; j++) out[j] = n3d::split_scale((double)hm[j] * (grow ? grow[j] : 1.0));
}

}  // namespace

extern "C" {

const char* n3d_last_error(void) { return g_last_error.c_str(); }
const char* n3d_version(void) { return "n3d-b200 0.4 (sm_100a, tcgen05: fp16-split GEMMs and attention (h*h + h*l + l*h))"; }

n3d_status n3d_model_load_gpu(const char* dir, int device, n3d_model** out) {
    return guarded([&] {
        arg_check(dir && out, "n3d_model_load_gpu: null argument");
        *out = nullptr;
        auto* h = new n3d_model;
        try {
            h->m = std::make_unique<n3d::Model>(dir, device);
        } catch (...) {
            delete h;
            throw;
        }
        *out = h;
    });
}

void n3d_model_free(n3d_model* model) { delete model; }

n3d_status n3d_model_set_stream(n3d_model* model, void* stream) {
    return guarded([&] {
        arg_check(model != nullptr, "n3d_model_set_stream: null model");
        model->m->set_stream((cudaStream_t)stream);
    });
}

size_t n3d_num_speakers(const n3d_model* model) { return model ? (size_t)model->m->cfg().num_speakers : 0; }
size_t n3d_hidden_size(const n3d_model* model) { return model ? (size_t)model->m->cfg().hidden : 0; }

const char* n3d_model_describe(n3d_model* model) {
    if (!model) return nullptr;
    const int dev = model->m->device();
    cudaDeviceProp prop{};
    std::string d;
    if (cudaGetDeviceProperties(&prop, dev) == cudaSuccess) {
        d = std::string(prop.name) + " (device " + std::to_string(dev) + ", sm_" + std::to_string(prop.major) +
            std::to_string(prop.minor) + ", " + std::to_string(prop.multiProcessorCount) + " SMs, " +
            std::to_string(prop.totalGlobalMem >> 30) + " GiB)";
    } else {
        cudaGetLastError();  // the failed query's error is not sticky: clear it for later calls
        d = "CUDA device " + std::to_string(dev);
    }
    model->describe = d + " | " + n3d_version();
    return model->describe.c_str();
}

static n3d_status run_one(n3d_model* model, const float* samples, size_t n, int mode, n3d_run_output* out) {
    return guarded([&] {
        arg_check(model && out && (samples || n == 0), "null argument");
        run_batch_to_outputs(*model->m, mode, {samples}, {(long long)n}, out);
    });
}

n3d_status n3d_run_offline(n3d_model* model, const float* samples, size_t n, n3d_run_output* out) {
    return run_one(model, samples, n, 3, out);
}

n3d_status n3d_run_streaming(n3d_model* model, const float* samples, size_t n, n3d_mode mode, n3d_run_output* out) {
    if (mode == N3D_MODE_OFFLINE || (int)mode < 0 || (int)mode > 3) {
        g_last_error = "n3d_run_streaming: mode must be a streaming mode";
        return N3D_ERR_INVALID_ARGUMENT;
    }
    return run_one(model, samples, n, (int)mode, out);
}

void n3d_run_output_free(n3d_run_output* out) {
    if (!out) return;
    std::free(out->logits);
    out->logits = nullptr;
}

n3d_status n3d_session_open(n3d_model* model, n3d_mode mode, n3d_session** out) {
    return guarded([&] {
        arg_check(model && out, "n3d_session_open: null argument");
        arg_check((int)mode >= 0 && (int)mode <= 2, "n3d_session_open: mode must be a streaming mode");
        *out = nullptr;
        n3d::Session* s = model->m->session_open((int)mode);
        auto* h = new (std::nothrow) n3d_session{model, s};
        if (!h) {
            model->m->session_free(s);
            throw std::bad_alloc();
        }
        *out = h;
    });
}

void n3d_session_free(n3d_session* session) {
    if (!session) return;
    session->owner->m->session_free(session->s);
    delete session;
}

n3d_status n3d_sessions_push(n3d_session* const* sessions, const float* const* samples, const size_t* lens,
                             size_t count, int close, n3d_run_output* outs) {
    return guarded([&] {
        if (count == 0) return;
        arg_check(sessions && lens && outs, "n3d_sessions_push: null argument");
        for (size_t i = 0; i < count; i++) outs[i] = n3d_run_output{};
        std::vector<n3d::Session*> ss(count);
        std::vector<const float*> a(count);
        std::vector<long long> l(count);
        n3d_model* owner = nullptr;
        for (size_t i = 0; i < count; i++) {
            arg_check(sessions[i] != nullptr, "n3d_sessions_push: null session");
            arg_check(lens[i] == 0 || (samples && samples[i]), "n3d_sessions_push: null samples");
            if (!owner) owner = sessions[i]->owner;
            arg_check(sessions[i]->owner == owner, "n3d_sessions_push: sessions of different models");
            ss[i] = sessions[i]->s;
            a[i] = lens[i] ? samples[i] : nullptr;
            l[i] = (long long)lens[i];
        }
        std::vector<std::vector<float>> rows;
        owner->m->sessions_push(ss, a, l, close != 0, rows);
        const size_t ns = (size_t)owner->m->cfg().num_speakers;
        try {
            for (size_t i = 0; i < count; i++) {
                n3d::ClipPlan totals;
                totals.num_chunks = ss[i]->num_chunks;
                totals.cache_compressed = ss[i]->compressed;
                totals.cache_frames = ss[i]->ncache;
                totals.fifo_frames = ss[i]->nfifo;
                fill_output(&outs[i], rows[i], totals, ns);
            }
        } catch (...) {
            for (size_t i = 0; i < count; i++) n3d_run_output_free(&outs[i]);
            throw;
        }
    });
}

n3d_status n3d_session_push(n3d_session* session, const float* samples, size_t n, n3d_run_output* out) {
    return n3d_sessions_push(&session, &samples, &n, 1, 0, out);
}

n3d_status n3d_session_close(n3d_session* session, n3d_run_output* out) {
    const float* none = nullptr;
    size_t zero = 0;
    return n3d_sessions_push(&session, &none, &zero, 1, 1, out);
}

n3d_status n3d_run_batch(n3d_model* model, n3d_mode mode, const float* const* samples, const size_t* lens,
                         size_t n_clips, n3d_run_output* outs) {
    return guarded([&] {
        arg_check(model && (n_clips == 0 || (samples && lens && outs)), "n3d_run_batch: null argument");
        arg_check((int)mode >= 0 && (int)mode <= 3, "n3d_run_batch: bad mode");
        std::vector<const float*> a(samples, samples + n_clips);
        std::vector<long long> l(lens, lens + n_clips);
        run_batch_to_outputs(*model->m, (int)mode, a, l, outs);
    });
}

n3d_status n3d_batch_out_frames(const n3d_model* model, n3d_mode mode, const size_t* lens, size_t n_clips,
                                size_t* frames_out) {
    return guarded([&] {
        arg_check(model && (n_clips == 0 || (lens && frames_out)), "n3d_batch_out_frames: null argument");
        arg_check((int)mode >= 0 && (int)mode <= 3, "n3d_batch_out_frames: bad mode");
        for (size_t i = 0; i < n_clips; i++) {
            arg_check(lens[i] <= (size_t)INT_MAX, "n3d_batch_out_frames: a clip of more than 2^31 samples");
            n3d::ClipPlan p = mode == N3D_MODE_OFFLINE ? n3d::plan_offline(model->m->cfg(), (long long)lens[i])
                                                       : n3d::plan_streaming(model->m->cfg(), (long long)lens[i], (int)mode);
            frames_out[i] = (size_t)p.out_rows;
        }
    });
}

n3d_status n3d_run_batch_device(n3d_model* model, n3d_mode mode, const float* d_audio, const size_t* offsets,
                                const size_t* lens, size_t n_clips, float* d_logits, const size_t* out_offsets) {
    return guarded([&] {
        arg_check(model && (n_clips == 0 || (d_audio && offsets && lens && d_logits && out_offsets)),
                  "n3d_run_batch_device: null argument");
        arg_check((int)mode >= 0 && (int)mode <= 3, "n3d_run_batch_device: bad mode");
        std::vector<long long> off(offsets, offsets + n_clips), l(lens, lens + n_clips),
            oo(out_offsets, out_offsets + n_clips);
        model->m->run_batch((int)mode, {}, d_audio, off, l, nullptr, d_logits, &oo, nullptr);
    });
}

n3d_status n3d_log_mel(n3d_model* model, const float* samples, size_t n, int centered, float* out, size_t out_cap,
                       size_t* frames) {
    return guarded([&] {
        arg_check(model && (samples || n == 0) && frames, "n3d_log_mel: null argument");
        std::vector<float> mel;
        const int f = model->m->log_mel(samples, (long long)n, centered != 0, mel);
        *frames = (size_t)f;
        arg_check(out_cap >= mel.size() && (out || mel.empty()), "n3d_log_mel: output buffer too small");
        if (!mel.empty()) std::memcpy(out, mel.data(), mel.size() * sizeof(float));
    });
}

n3d_status n3d_embed_range(n3d_model* model, const float* mel, size_t num_frames, size_t lo, size_t hi, float* out) {
    return guarded([&] {
        arg_check(model && out && (mel || num_frames == 0) && hi >= lo, "n3d_embed_range: bad argument");
        // one call embeds at most MAX_SEQ groups (src/gpu_engine.rs:1328-1334), and the
        // frame arithmetic stays inside 64-bit range
        arg_check(hi - lo <= 1024 && hi <= (size_t)INT_MAX && num_frames <= (size_t)INT_MAX,
                  "n3d_embed_range: at most 1024 groups per call, indices below 2^31");
        model->m->embed_range(mel, (long long)num_frames, (long long)lo, (long long)hi, out);
    });
}

n3d_status n3d_forward_embeds(n3d_model* model, const float* embeds, size_t frames, size_t valid, float* out) {
    return guarded([&] {
        arg_check(model && embeds && out, "n3d_forward_embeds: null argument");
        arg_check(frames <= (size_t)INT_MAX, "n3d_forward_embeds: frames beyond 2^31");
        model->m->forward_window(embeds, (int)frames, (int)std::min(valid, frames), out, nullptr);
    });
}

n3d_status n3d_head_forward(n3d_model* model, const float* encoder_out, size_t frames, float* logits) {
    return guarded([&] {
        arg_check(model && encoder_out && logits, "n3d_head_forward: null argument");
        arg_check(frames <= (size_t)INT_MAX, "n3d_head_forward: frames beyond 2^31");
        model->m->head_forward(encoder_out, (int)frames, logits);
    });
}

n3d_status n3d_forward_window(n3d_model* model, const float* embeds, size_t frames, size_t valid, float* logits) {
    return guarded([&] {
        arg_check(model && embeds && logits, "n3d_forward_window: null argument");
        arg_check(frames <= (size_t)INT_MAX, "n3d_forward_window: frames beyond 2^31");
        model->m->forward_window(embeds, (int)frames, (int)std::min(valid, frames), nullptr, logits);
    });
}

n3d_status n3d_extract_speaker_dict(const float* logits, size_t num_frames, size_t ns, float duration,
                                    const uint8_t* mask, float threshold, n3d_segment** out, size_t* count) {
    return guarded([&] {
        arg_check(out && count && (logits || num_frames == 0 || ns == 0), "n3d_extract_speaker_dict: null argument");
        std::vector<n3d_segment> segs;
        for (size_t s = 0; s < ns; s++) {
            long long start = -1;
            for (size_t t = 0; t <= num_frames; t++) {
                const bool active = t < num_frames && sigmoidf(logits[t * ns + s]) > threshold && (!mask || mask[t]);
                if (active && start < 0) {
                    start = (long long)t;
                } else if (!active && start >= 0) {
                    segs.push_back(n3d_segment{round2((float)start * duration), round2((float)t * duration), s});
                    start = -1;
                }
            }
        }
        std::stable_sort(segs.begin(), segs.end(), [](const n3d_segment& a, const n3d_segment& b) {
            if (a.start != b.start) return a.start < b.start;
            return a.speaker < b.speaker;
        });
        *count = segs.size();
        *out = (n3d_segment*)std::malloc(std::max<size_t>(segs.size(), 1) * sizeof(n3d_segment));
        if (!*out) throw std::bad_alloc();
        if (!segs.empty()) std::memcpy(*out, segs.data(), segs.size() * sizeof(n3d_segment));
    });
}

void n3d_segments_free(n3d_segment* segments) { std::free(segments); }

float n3d_activity_stats(const float* logits, size_t num_frames, size_t ns, const uint8_t* mask, float threshold,
                         size_t* per_speaker) {
    size_t any = 0, total = 0;
    if (per_speaker)
        for (size_t s = 0; s < ns; s++) per_speaker[s] = 0;
    for (size_t t = 0; t < num_frames; t++) {
        if (mask && !mask[t]) continue;
        total++;
        bool hot = false;
        for (size_t s = 0; s < ns; s++)
            if (sigmoidf(logits[t * ns + s]) > threshold) {
                if (per_speaker) per_speaker[s]++;
                hot = true;
            }
        any += hot;
    }
    return total == 0 ? 0.0f : (float)any * 100.0f / (float)total;
}

float n3d_frame_duration(size_t hop_length, uint32_t sampling_rate) {
    return (float)hop_length / (float)sampling_rate;
}

n3d_status n3d_profile_enable(n3d_model* model, int on) {
    return guarded([&] {
        arg_check(model != nullptr, "n3d_profile_enable: null model");
        model->m->profile_enable(on != 0);
    });
}

size_t n3d_profile_read(const n3d_model* model, n3d_kernel_stats* out, size_t cap) {
    static const char* names[n3d::K_NCLASS] = {"gemm_other",   "attention",  "layer_norm", "mel",
                                               "cache_update", "assemble",   "other",      "gemm_qkv",
                                               "gemm_o",       "gemm_fc1",   "gemm_fc2",   "gemm_head_proj",
                                               "gemm_head_conv", "gemm_head_dense", "gemm_embed"};
    if (!model) return 0;
    const n3d::ProfTotals* t = model->m->profile_totals();
    size_t n = 0;
    for (int i = 0; i < n3d::K_NCLASS && n < cap; i++, n++)
        out[n] = n3d_kernel_stats{names[i], (size_t)t[i].launches, t[i].ms, t[i].flops, t[i].bytes};
    return n;
}

n3d_status n3d_step_timing_enable(n3d_model* model, int on) {
    return guarded([&] {
        arg_check(model != nullptr, "n3d_step_timing_enable: null model");
        model->m->step_timing_enable(on != 0);
    });
}

size_t n3d_step_times(const n3d_model* model, double* ms, size_t cap) {
    if (!model) return 0;
    const std::vector<float>& t = model->m->step_times();
    for (size_t i = 0; i < t.size() && i < cap; i++) ms[i] = t[i];
    return t.size();
}

n3d_status n3d_config_load(const char* dir, n3d_config** out) {
    return guarded([&] {
        arg_check(dir && out, "n3d_config_load: null argument");
        *out = nullptr;
        auto h = std::make_unique<n3d_config>();
        h->c = n3d::load_config(dir);
        *out = h.release();
    });
}

void n3d_config_free(n3d_config* cfg) { delete cfg; }

n3d_status n3d_mode_params_resolve(const n3d_config* cfg, n3d_mode mode, n3d_mode_params* out) {
    return guarded([&] {
        arg_check(cfg && out, "n3d_mode_params_resolve: null argument");
        arg_check((int)mode >= 0 && (int)mode <= 3, "n3d_mode_params_resolve: bad mode");
        const n3d::Config& c = cfg->c;
        n3d_mode_params p{};
        p.hop_length = (size_t)c.hop;
        p.n_fft = (size_t)c.n_fft;
        p.subsampling = (size_t)c.proc_sub;
        if (mode == N3D_MODE_OFFLINE) {
            p.latency_ms = (size_t)(c.chunk_length + c.chunk_rc) * 80;
        } else {
            const size_t cl = (size_t)c.modes[mode][0], rc = (size_t)c.modes[mode][1];
            p.mel_frames_per_chunk = (cl + rc) * p.subsampling;
            p.mel_frames_per_step = cl * p.subsampling;
            p.lookahead_encoder_frames = rc;
            p.first_chunk_samples = (p.mel_frames_per_chunk - 1) * p.hop_length + (size_t)c.win / 2;
            p.samples_per_chunk = p.mel_frames_per_chunk * p.hop_length + (size_t)c.win;
            p.latency_ms = (cl + rc) * 80;
        }
        *out = p;
    });
}

n3d_status n3d_streaming_chunks(const n3d_config* cfg, size_t n_samples, n3d_mode mode, n3d_chunk* out, size_t cap,
                                size_t* count) {
    return guarded([&] {
        arg_check(cfg && count && (out || cap == 0), "n3d_streaming_chunks: null argument");
        arg_check((int)mode >= 0 && (int)mode <= 2, "n3d_streaming_chunks: mode must be a streaming mode");
        arg_check(n_samples <= (size_t)INT_MAX, "n3d_streaming_chunks: more than 2^31 samples");
        const std::vector<n3d::StreamChunk> ch = n3d::streaming_chunks(cfg->c, (long long)n_samples, (int)mode);
        for (size_t i = 0; i < ch.size() && i < cap; i++)
            out[i] = n3d_chunk{(size_t)ch[i].start, (size_t)ch[i].len, ch[i].centered, (size_t)ch[i].mel_frames,
                               (size_t)ch[i].lookahead};
        *count = ch.size();
    });
}

n3d_status n3d_schedule(const n3d_config* cfg, n3d_mode mode, size_t n_samples, n3d_step_plan* steps, size_t cap,
                        size_t* count, n3d_run_output* totals) {
    return guarded([&] {
        arg_check(cfg && count && (steps || cap == 0), "n3d_schedule: null argument");
        arg_check((int)mode >= 0 && (int)mode <= 3, "n3d_schedule: bad mode");
        arg_check(n_samples <= (size_t)INT_MAX, "n3d_schedule: more than 2^31 samples");
        const n3d::ClipPlan p = mode == N3D_MODE_OFFLINE ? n3d::plan_offline(cfg->c, (long long)n_samples)
                                                         : n3d::plan_streaming(cfg->c, (long long)n_samples, (int)mode);
        const size_t n = p.steps.size();
        for (size_t i = 0; i < n && i < cap; i++) {
            const n3d::StepPlan& sp = p.steps[i];
            // the cache after step i is what step i + 1 starts from
            const bool last = i + 1 == n;
            steps[i] = n3d_step_plan{(size_t)(sp.ncache + sp.nfifo),
                                     (size_t)sp.S,
                                     (size_t)sp.valid,
                                     (size_t)sp.nchunk,
                                     (size_t)(last ? p.cache_frames : p.steps[i + 1].ncache),
                                     (size_t)(last ? p.fifo_frames : p.steps[i + 1].nfifo),
                                     last ? p.cache_compressed : p.steps[i + 1].was_compressed};
        }
        *count = n;
        if (totals) {
            *totals = n3d_run_output{};
            totals->num_frames = (size_t)p.out_rows;
            totals->num_speakers = (size_t)cfg->c.num_speakers;
            totals->num_chunks = (size_t)p.num_chunks;
            totals->cache_compressed = p.cache_compressed;
            totals->cache_frames = (size_t)p.cache_frames;
            totals->fifo_frames = (size_t)p.fifo_frames;
        }
    });
}

n3d_status n3d_linear(int device, const float* d_x, size_t rows, size_t cols, const float* d_w, size_t out,
                      const float* d_bias, float* d_y) {
    return guarded([&] {
        arg_check(d_x && d_w && d_y, "n3d_linear: null argument");
        arg_check(cols % 32 == 0 && cols > 0, "n3d_linear: cols must be a positive multiple of 32");
        arg_check(rows <= (size_t)INT_MAX && cols <= (size_t)INT_MAX && out <= (size_t)INT_MAX,
                  "n3d_linear: sizes beyond 2^31");
        N3D_CUDA(cudaSetDevice(device));
        KernelCtx& k = kctx(device);
        std::lock_guard<std::mutex> turn(k.call);
        DevScratch sc;
        float scale[2];
        operand_scales(k, sc, {{d_x, rows * cols}, {d_w, out * cols}}, scale);
        const n3d::SplitOut x{sc.get(rows * cols / 2), sc.get(rows * cols / 2), scale[0], nullptr};
        const n3d::SplitOut w{sc.get(out * cols / 2), sc.get(out * cols / 2), scale[1], nullptr};
        n3d::launch_split(k.stream, d_x, (long long)(rows * cols), x);
        n3d::launch_split(k.stream, d_w, (long long)(out * cols), w);
        n3d::Epi e;
        e.mode = n3d::EPI_STORE;
        e.bias = d_bias;
        e.out = d_y;
        e.ldo = (long long)out;
        n3d::gemm_split(k.stream, n3d::SplitOperand{x.h, x.l, (long long)rows, (long long)cols, (long long)cols, x.scale},
                        n3d::SplitOperand{w.h, w.l, (long long)out, (long long)cols, (long long)cols, w.scale},
                        (int)rows, (int)out, (int)cols, 0, e, k.err);
        kcheck(k);
    });
}

n3d_status n3d_linear_noalloc(int device, const float* d_x, size_t rows, size_t cols, const float* d_w, size_t out,
                              const float* d_bias, float* d_y, void* stream) {
    return guarded([&] {
        n3d::linear_noalloc(device, d_x, rows, cols, d_w, out, d_bias, d_y, (cudaStream_t)stream);
    });
}

n3d_status n3d_layer_norm(int device, const float* d_x, size_t rows, size_t cols, const float* d_w, const float* d_b,
                          float* d_y) {
    return guarded([&] {
        arg_check(d_x && d_w && d_b && d_y, "n3d_layer_norm: null argument");
        arg_check(cols == 512 || cols == 1024, "n3d_layer_norm: cols must be 512 or 1024");
        arg_check(rows <= (size_t)INT_MAX, "n3d_layer_norm: rows beyond 2^31");
        N3D_CUDA(cudaSetDevice(device));
        KernelCtx& k = kctx(device);
        std::lock_guard<std::mutex> turn(k.call);
        n3d::launch_layer_norm(k.stream, d_x, (long long)rows, (int)cols, d_w, d_b, n3d::plain_out(d_y));
        kcheck(k);
    });
}

n3d_status n3d_attention(int device, const float* d_q, const float* d_k, const float* d_v, size_t seq, size_t heads,
                         size_t head_dim, size_t valid, int rope, double rope_theta, float* d_out) {
    return guarded([&] {
        arg_check(d_q && d_k && d_v && d_out, "n3d_attention: null argument");
        arg_check(head_dim == 64 || head_dim == 128, "n3d_attention: head_dim must be 64 or 128");
        arg_check(seq <= (size_t)INT_MAX && heads >= 1 && heads <= 65535, "n3d_attention: seq beyond 2^31 or heads "
                                                                           "outside 1..65535");
        N3D_CUDA(cudaSetDevice(device));
        KernelCtx& k = kctx(device);
        std::lock_guard<std::mutex> turn(k.call);
        DevScratch sc;
        float *cs = nullptr, *sn = nullptr;
        if (rope) {
            // rope_tables (src/encoder.rs:163-185), positions 0..seq-1
            const size_t half = head_dim / 2;
            std::vector<float> inv(half), hc(seq * head_dim), hs(seq * head_dim);
            for (size_t i = 0; i < half; i++)
                inv[i] = (float)(1.0 / std::pow(rope_theta, 2.0 * (double)i / (double)head_dim));
            for (size_t p = 0; p < seq; p++)
                for (size_t i = 0; i < half; i++) {
                    const float a = (float)p * inv[i];
                    hc[p * head_dim + i] = hc[p * head_dim + half + i] = std::cos(a);
                    hs[p * head_dim + i] = hs[p * head_dim + half + i] = std::sin(a);
                }
            cs = sc.get(seq * head_dim);
            sn = sc.get(seq * head_dim);
            N3D_CUDA(cudaMemcpyAsync(cs, hc.data(), hc.size() * 4, cudaMemcpyHostToDevice, k.stream));
            N3D_CUDA(cudaMemcpyAsync(sn, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice, k.stream));
        }
        int v = (int)std::min(valid, seq);
        int* dv = (int*)sc.get(1);
        N3D_CUDA(cudaMemcpyAsync(dv, &v, 4, cudaMemcpyHostToDevice, k.stream));
        // tcgen05 path: operands in the fp16 split with scales from their maxima, V transposed
        const size_t W = heads * head_dim, vt_ld = (seq + 7) / 8 * 8;
        n3d::AttnOperands op;
        op.q_h = sc.get(seq * W / 2);
        op.q_l = sc.get(seq * W / 2);
        op.k_h = sc.get(seq * W / 2);
        op.k_l = sc.get(seq * W / 2);
        op.rows_cap = (long long)seq;
        op.vt_h = sc.get(W * vt_ld / 2);
        op.vt_l = sc.get(W * vt_ld / 2);
        op.vt_ld = (long long)vt_ld;
        {
            const size_t n = seq * W;
            const double grow[3] = {rope ? 2.0 : 1.0, rope ? 2.0 : 1.0, 1.0};
            float sc3[3];
            operand_scales(k, sc, {{d_q, n}, {d_k, n}, {d_v, n}}, sc3, grow);
            op.q_scale = sc3[0];
            op.k_scale = sc3[1];
            op.v_scale = sc3[2];
        }
        n3d::launch_pack_attn(k.stream, d_q, d_k, d_v, (long long)seq, (int)heads, (int)head_dim, cs, sn, op);
        n3d::launch_attention_tc(k.stream, op, 1, (int)seq, dv, (int)heads, (int)head_dim, n3d::plain_out(d_out),
                                 k.err);
        kcheck(k);
    });
}

n3d_status n3d_selftest_wait_timeout(int device, double limit_ms, double* waited_ms) {
    return guarded([&] {
        arg_check(limit_ms >= 0.001 && limit_ms <= 2000.0, "n3d_selftest_wait_timeout: limit_ms outside 0.001..2000");
        N3D_CUDA(cudaSetDevice(device));
        KernelCtx& k = kctx(device);
        std::lock_guard<std::mutex> turn(k.call);
        DevScratch sc;
        unsigned long long* d_waited = (unsigned long long*)sc.get(2);
        N3D_CUDA(cudaMemsetAsync(d_waited, 0, 8, k.stream));
        n3d::launch_wait_probe(k.stream, k.err, (unsigned long long)(limit_ms * 1e6), d_waited);
        N3D_CUDA(cudaStreamSynchronize(k.stream));
        unsigned long long ns = 0;
        N3D_CUDA(cudaMemcpy(&ns, d_waited, 8, cudaMemcpyDeviceToHost));
        if (waited_ms) *waited_ms = (double)ns / 1e6;
        kcheck(k);  // the expired wait's status: N3D_ERR_TIMEOUT, and the word is cleared
    });
}

n3d_status n3d_cache_compress(int device, const n3d_cache_config* cfg, const float* probs, size_t frames,
                              const float* embeds, size_t hidden, const float* silence, size_t* picked,
                              size_t* sentinel, size_t* count, float* out_embeds, float* out_probs) {
    return guarded([&] {
        arg_check(cfg && probs && picked && sentinel && count, "n3d_cache_compress: null argument");
        arg_check(!embeds || (silence && out_embeds && out_probs), "n3d_cache_compress: null gather argument");
        arg_check(frames >= 1 && frames <= 65536, "n3d_cache_compress: frames outside 1..65536");
        arg_check(cfg->num_speakers >= 1 && cfg->num_speakers <= 16, "n3d_cache_compress: num_speakers outside 1..16");
        arg_check(cfg->num_silence_frames <= 65536 && cfg->speaker_cache_length <= (size_t)INT_MAX &&
                      cfg->min_positive_scores <= (size_t)INT_MAX && cfg->num_strong_boosted_frames <= (size_t)INT_MAX &&
                      cfg->num_weak_boosted_frames <= (size_t)INT_MAX,
                  "n3d_cache_compress: cache sizes beyond 2^31");
        arg_check(!embeds || (hidden >= 4 && hidden % 4 == 0 && hidden <= 65536),
                  "n3d_cache_compress: hidden must be a positive multiple of 4");
        const int ne = (int)frames, ns = (int)cfg->num_speakers, n_sil = (int)cfg->num_silence_frames;
        if (n3d::cache_compress_smem(ne, ns, n_sil) > 227 * 1024)
            throw n3d::Error(N3D_ERR_INVALID_ARGUMENT, "n3d_cache_compress: frames * speakers too large for one CTA");
        const n3d::CacheConst cc{embeds ? (int)hidden : 0, ns, (int)cfg->subsampling_factor,
                                 (int)cfg->speaker_cache_length, n_sil, (int)cfg->min_positive_scores,
                                 (int)cfg->num_strong_boosted_frames, (int)cfg->num_weak_boosted_frames,
                                 cfg->score_threshold, cfg->latest_frames_score_boost};
        const size_t total = (size_t)ns * (frames + (size_t)n_sil);
        const size_t L = std::min(cfg->speaker_cache_length, total);
        N3D_CUDA(cudaSetDevice(device));
        KernelCtx& k = kctx(device);
        std::lock_guard<std::mutex> turn(k.call);
        DevScratch sc;
        float* d_probs = sc.get(frames * ns);
        int* d_picked = (int*)sc.get(L);
        int* d_counts = (int*)sc.get(2);
        float *d_rows = nullptr, *d_sil = nullptr, *d_oe = nullptr, *d_op = nullptr;
        N3D_CUDA(cudaMemcpyAsync(d_probs, probs, frames * ns * 4, cudaMemcpyHostToDevice, k.stream));
        if (embeds) {
            d_rows = sc.get(frames * hidden);
            d_sil = sc.get(hidden);
            d_oe = sc.get(L * hidden);
            d_op = sc.get(L * ns);
            N3D_CUDA(cudaMemcpyAsync(d_rows, embeds, frames * hidden * 4, cudaMemcpyHostToDevice, k.stream));
            N3D_CUDA(cudaMemcpyAsync(d_sil, silence, hidden * 4, cudaMemcpyHostToDevice, k.stream));
        }
        n3d::launch_cache_compress(k.stream, d_probs, ne, d_rows, d_sil, cc, d_picked, d_counts, d_oe, d_op);
        kcheck(k);
        int counts[2] = {0, 0};
        N3D_CUDA(cudaMemcpy(counts, d_counts, sizeof(counts), cudaMemcpyDeviceToHost));
        const size_t n_real = (size_t)counts[0];
        if ((size_t)counts[1] != L || n_real > L) throw n3d::Error(N3D_ERR_GPU, "n3d_cache_compress: bad pick count");
        std::vector<int> got(n_real);
        if (n_real) N3D_CUDA(cudaMemcpy(got.data(), d_picked, n_real * 4, cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < n_real; i++) picked[i] = (size_t)got[i];
        for (size_t i = n_real; i < L; i++) picked[i] = total;  // the -inf picks, remapped and sorted last
        *sentinel = total;
        *count = L;
        if (embeds) {
            N3D_CUDA(cudaMemcpy(out_embeds, d_oe, L * hidden * 4, cudaMemcpyDeviceToHost));
            N3D_CUDA(cudaMemcpy(out_probs, d_op, L * ns * 4, cudaMemcpyDeviceToHost));
        }
    });
}

}  // extern "C"

namespace {

// Times `launch` (3 untimed calls, then `iters` between two events on k's stream).
template <class F>
double time_launches(KernelCtx& k, int iters, F&& launch) {
    for (int i = 0; i < 3; i++) launch();
    cudaEvent_t e0, e1;
    N3D_CUDA(cudaEventCreate(&e0));
    N3D_CUDA(cudaEventCreate(&e1));
    N3D_CUDA(cudaEventRecord(e0, k.stream));
    for (int i = 0; i < iters; i++) launch();
    N3D_CUDA(cudaEventRecord(e1, k.stream));
    kcheck(k);
    float ms = 0.0f;
    N3D_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return (double)ms / iters;
}

}  // namespace

extern "C" {

n3d_status n3d_bench_linear(int device, size_t rows, size_t cols, size_t out, int iters, double* ms) {
    return guarded([&] {
        arg_check(ms != nullptr && iters >= 1, "n3d_bench_linear: null ms or iters < 1");
        arg_check(cols % 32 == 0 && cols > 0 && rows > 0 && out > 0, "n3d_bench_linear: cols must be a positive "
                                                                     "multiple of 32, rows and out positive");
        arg_check(rows <= (size_t)INT_MAX && cols <= (size_t)INT_MAX && out <= (size_t)INT_MAX &&
                      rows * cols <= ((size_t)1 << 33) && out * cols <= ((size_t)1 << 33) &&
                      rows * out <= ((size_t)1 << 33),
                  "n3d_bench_linear: sizes beyond 2^31 or operands beyond 2^33 elements");
        N3D_CUDA(cudaSetDevice(device));
        KernelCtx& k = kctx(device);
        std::lock_guard<std::mutex> turn(k.call);
        DevScratch sc;
        float* x = sc.get(rows * cols);
        float* w = sc.get(out * cols);
        float* bias = sc.get(out);
        float* y = sc.get(rows * out);
        n3d::launch_fill_random(k.stream, x, (long long)(rows * cols), 1, 1.0f);
        n3d::launch_fill_random(k.stream, w, (long long)(out * cols), 2, 1.0f / std::sqrt((float)cols));
        n3d::launch_fill_random(k.stream, bias, (long long)out, 3, 1.0f);
        float scale[2];
        operand_scales(k, sc, {{x, rows * cols}, {w, out * cols}}, scale);
        const n3d::SplitOut xs{sc.get(rows * cols / 2), sc.get(rows * cols / 2), scale[0], nullptr};
        const n3d::SplitOut ws{sc.get(out * cols / 2), sc.get(out * cols / 2), scale[1], nullptr};
        n3d::launch_split(k.stream, x, (long long)(rows * cols), xs);
        n3d::launch_split(k.stream, w, (long long)(out * cols), ws);
        n3d::Epi e;
        e.mode = n3d::EPI_STORE;
        e.bias = bias;
        e.out = y;
        e.ldo = (long long)out;
        *ms = time_launches(k, iters, [&] {
            n3d::gemm_split(k.stream, n3d::SplitOperand{xs.h, xs.l, (long long)rows, (long long)cols, (long long)cols, xs.scale},
                            n3d::SplitOperand{ws.h, ws.l, (long long)out, (long long)cols, (long long)cols, ws.scale},
                            (int)rows, (int)out, (int)cols, 0, e, k.err);
        });
    });
}

n3d_status n3d_bench_attention(int device, size_t seq, size_t heads, size_t head_dim, int iters, double* ms) {
    return guarded([&] {
        arg_check(ms != nullptr && iters >= 1, "n3d_bench_attention: null ms or iters < 1");
        arg_check(head_dim == 64 || head_dim == 128, "n3d_bench_attention: head_dim must be 64 or 128");
        arg_check(seq >= 1 && seq <= 65536 && heads >= 1 && heads <= 64,
                  "n3d_bench_attention: seq outside 1..65536 or heads outside 1..64");
        N3D_CUDA(cudaSetDevice(device));
        KernelCtx& k = kctx(device);
        std::lock_guard<std::mutex> turn(k.call);
        DevScratch sc;
        const size_t W = heads * head_dim;
        float* q = sc.get(seq * W);
        float* kk = sc.get(seq * W);
        float* v = sc.get(seq * W);
        float* ctx = sc.get(seq * W);
        n3d::launch_fill_random(k.stream, q, (long long)(seq * W), 4, 1.0f);
        n3d::launch_fill_random(k.stream, kk, (long long)(seq * W), 5, 1.0f);
        n3d::launch_fill_random(k.stream, v, (long long)(seq * W), 6, 1.0f);
        int vv = (int)seq;
        int* dv = (int*)sc.get(1);
        N3D_CUDA(cudaMemcpyAsync(dv, &vv, 4, cudaMemcpyHostToDevice, k.stream));
        const size_t vt_ld = (seq + 7) / 8 * 8;
        n3d::AttnOperands op;
        op.q_h = sc.get(seq * W / 2);
        op.q_l = sc.get(seq * W / 2);
        op.k_h = sc.get(seq * W / 2);
        op.k_l = sc.get(seq * W / 2);
        op.rows_cap = (long long)seq;
        op.vt_h = sc.get(W * vt_ld / 2);
        op.vt_l = sc.get(W * vt_ld / 2);
        op.vt_ld = (long long)vt_ld;
        {
            float sc3[3];
            operand_scales(k, sc, {{q, seq * W}, {kk, seq * W}, {v, seq * W}}, sc3);
            op.q_scale = sc3[0];
            op.k_scale = sc3[1];
            op.v_scale = sc3[2];
        }
        n3d::launch_pack_attn(k.stream, q, kk, v, (long long)seq, (int)heads, (int)head_dim, nullptr, nullptr, op);
        *ms = time_launches(k, iters, [&] {
            n3d::launch_attention_tc(k.stream, op, 1, (int)seq, dv, (int)heads, (int)head_dim, n3d::plain_out(ctx),
                                     k.err);
        });
    });
}

n3d_status n3d_bench_layer_norm(int device, size_t rows, size_t cols, int iters, double* ms) {
    return guarded([&] {
        arg_check(ms != nullptr && iters >= 1, "n3d_bench_layer_norm: null ms or iters < 1");
        arg_check(cols == 512 || cols == 1024, "n3d_bench_layer_norm: cols must be 512 or 1024");
        arg_check(rows >= 1 && rows <= ((size_t)1 << 24), "n3d_bench_layer_norm: rows outside 1..2^24");
        N3D_CUDA(cudaSetDevice(device));
        KernelCtx& k = kctx(device);
        std::lock_guard<std::mutex> turn(k.call);
        DevScratch sc;
        float* x = sc.get(rows * cols);
        float* y = sc.get(rows * cols);
        float* w = sc.get(cols);
        float* b = sc.get(cols);
        n3d::launch_fill_random(k.stream, x, (long long)(rows * cols), 7, 3.0f);
        n3d::launch_fill_random(k.stream, w, (long long)cols, 8, 1.0f);
        n3d::launch_fill_random(k.stream, b, (long long)cols, 9, 0.1f);
        *ms = time_launches(k, iters, [&] {
            n3d::launch_layer_norm(k.stream, x, (long long)rows, (int)cols, w, b, n3d::plain_out(y));
        });
    });
}

}  // extern "C"
