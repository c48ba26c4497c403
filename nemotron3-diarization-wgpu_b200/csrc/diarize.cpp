// diarize: the command-line diarizer of the reference (src/bin/diarize.rs) over the
// C ABI of this backend.
//
//   diarize <audio.wav|audio.npy> [--mode MODE] [--model DIR] [--out FILE]
//           [--threshold T] [--device N] [--gpu]
//
// Reads 16 kHz mono audio (WAV: 16-bit PCM or 32-bit float, channels averaged; .npy:
// <f4 or <i8, as the reference's reader), runs the model on a B200 (n3d_run_offline or
// n3d_run_streaming), extracts the speaker segments (n3d_extract_speaker_dict) and
// writes the reference's JSON report: the same fields, keys in sorted order and 2-space
// indentation as serde_json's pretty printer, segments as {End, Speaker, Start} rounded
// to hundredths.  Like the reference, it never resamples.  `--gpu` is accepted for
// command-line compatibility (this backend always runs on the GPU).

#include <algorithm>
#include <cctype>
#include <charconv>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/n3d.h"
#include "json.h"
#include "report_json.h"

namespace {

struct ModeName {
    const char* arg;     // --mode value
    const char* report;  // the reference's format!("{mode:?}").to_lowercase()
    n3d_mode mode;
};
const ModeName kModes[] = {{"offline", "offline", N3D_MODE_OFFLINE},
                           {"low_latency", "lowlatency", N3D_MODE_LOW_LATENCY},
                           {"very_low_latency", "verylowlatency", N3D_MODE_VERY_LOW_LATENCY},
                           {"ultra_low_latency", "ultralowlatency", N3D_MODE_ULTRA_LOW_LATENCY}};

std::string read_bytes(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot open " + path);
    std::ostringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

uint32_t le32(const std::string& b, size_t o) {
    return (uint32_t)(uint8_t)b[o] | (uint32_t)(uint8_t)b[o + 1] << 8 | (uint32_t)(uint8_t)b[o + 2] << 16 |
           (uint32_t)(uint8_t)b[o + 3] << 24;
}
uint16_t le16(const std::string& b, size_t o) { return (uint16_t)((uint8_t)b[o] | (uint8_t)b[o + 1] << 8); }

// The value of `key` in a .npy header dict ("'descr': '<f4', 'fortran_order': False, ...").
std::string npy_field(const std::string& hdr, const std::string& key) {
    const size_t k = hdr.find("'" + key + "':");
    if (k == std::string::npos) return "";
    size_t i = k + key.size() + 3;
    while (i < hdr.size() && hdr[i] == ' ') i++;
    if (i < hdr.size() && hdr[i] == '\'') i++;
    size_t j = i;
    if (key == "shape") {
        j = hdr.find(')', i);
        return hdr.substr(i, j == std::string::npos ? std::string::npos : j - i + 1);
    }
    while (j < hdr.size() && hdr[j] != '\'' && hdr[j] != ',' && hdr[j] != '}') j++;
    return hdr.substr(i, j - i);
}

// .npy (src/npy.rs:30-117): little-endian <f4 or <i8, any shape, flattened in C order.
std::vector<float> read_npy(const std::string& path) {
    const std::string b = read_bytes(path);
    if (b.size() < 10 || b.compare(0, 6, "\x93NUMPY") != 0) throw std::runtime_error(path + ": not a .npy file");
    const int major = (uint8_t)b[6];
    if (major != 1 && b.size() < 12) throw std::runtime_error(path + ": truncated .npy header");
    const size_t hlen = major == 1 ? le16(b, 8) : le32(b, 8), off = major == 1 ? 10 : 12;
    if (off + hlen > b.size()) throw std::runtime_error(path + ": truncated .npy header");
    const std::string hdr = b.substr(off, hlen);
    const std::string descr = npy_field(hdr, "descr");
    const bool fortran = npy_field(hdr, "fortran_order").find("True") == 0;
    std::vector<size_t> shape;
    {
        const std::string s = npy_field(hdr, "shape");
        size_t i = 0;
        while (i < s.size()) {
            if (std::isdigit((unsigned char)s[i])) {
                size_t j = i;
                while (j < s.size() && std::isdigit((unsigned char)s[j])) j++;
                shape.push_back(std::stoull(s.substr(i, j - i)));
                i = j;
            } else {
                i++;
            }
        }
    }
    const size_t data = off + hlen, bytes = b.size() - data;
    std::vector<float> out;
    if (descr == "<f4") {
        out.resize(bytes / 4);
        std::memcpy(out.data(), b.data() + data, out.size() * 4);
    } else if (descr == "<i8") {
        out.resize(bytes / 8);
        for (size_t i = 0; i < out.size(); i++) {
            int64_t v;
            std::memcpy(&v, b.data() + data + 8 * i, 8);
            out[i] = (float)(double)v;
        }
    } else {
        throw std::runtime_error(path + ": expected <f4 or <i8, got " + descr);
    }
    if (fortran && shape.size() == 2) {  // to row-major, as the reference's reader
        const size_t rows = shape[0], cols = shape[1];
        if (rows * cols != out.size()) throw std::runtime_error(path + ": .npy data does not match its shape");
        std::vector<float> t(out.size());
        for (size_t r = 0; r < rows; r++)
            for (size_t c = 0; c < cols; c++) t[r * cols + c] = out[c * rows + r];
        out.swap(t);
    }
    return out;
}

// WAV: 16-bit PCM (scaled by 1/32768) or 32-bit float, channels averaged in fp32 order.
std::vector<float> read_wav(const std::string& path) {
    const std::string b = read_bytes(path);
    if (b.size() < 12 || b.compare(0, 4, "RIFF") != 0 || b.compare(8, 4, "WAVE") != 0)
        throw std::runtime_error(path + ": not a RIFF/WAVE file");
    int fmt = 0, ch = 0, bits = 0;
    bool have_fmt = false, have_data = false;
    size_t data = 0, data_len = 0;
    for (size_t o = 12; o + 8 <= b.size();) {
        const std::string id = b.substr(o, 4);
        const size_t len = le32(b, o + 4);
        if (id == "fmt ") {
            if (len < 16 || o + 8 + 16 > b.size()) throw std::runtime_error(path + ": truncated fmt chunk");
            fmt = le16(b, o + 8);
            ch = le16(b, o + 10);
            bits = le16(b, o + 22);
            if (fmt == 0xFFFE) {  // WAVE_FORMAT_EXTENSIBLE: the sub-format's first two bytes
                if (len < 40 || o + 8 + 26 > b.size()) throw std::runtime_error(path + ": truncated fmt chunk");
                fmt = le16(b, o + 8 + 24);
            }
            have_fmt = true;
        } else if (id == "data") {
            data = o + 8;
            data_len = std::min(len, b.size() - data);
            have_data = true;
        }
        o += 8 + len + (len & 1);
    }
    if (!have_fmt) throw std::runtime_error(path + ": no fmt chunk");
    if (!have_data) throw std::runtime_error(path + ": no data chunk");
    if (ch < 1) throw std::runtime_error(path + " has no channels");
    const bool flt = fmt == 3 && bits == 32, pcm16 = fmt == 1 && bits == 16;
    if (!flt && !pcm16) throw std::runtime_error(path + " must be 16-bit PCM or float32");
    const size_t width = bits / 8, n = data_len / width;
    std::vector<float> s(n);
    for (size_t i = 0; i < n; i++) {
        if (flt) {
            std::memcpy(&s[i], b.data() + data + 4 * i, 4);
        } else {
            int16_t v;
            std::memcpy(&v, b.data() + data + 2 * i, 2);
            s[i] = (float)v / 32768.0f;
        }
    }
    if (n % ch) throw std::runtime_error(path + " is not a whole number of frames");
    if (ch == 1) return s;
    std::vector<float> mono(n / ch);
    for (size_t f = 0; f < mono.size(); f++) {
        float acc = 0.0f;
        for (int c = 0; c < ch; c++) acc += s[f * ch + c];
        mono[f] = acc / (float)ch;
    }
    return mono;
}

using n3d::report::number;
using n3d::report::quote;

double round_to(double v, double scale) { return std::round(v * scale) / scale; }

int usage(int rc) {
    std::printf("usage: diarize <audio.wav|audio.npy> [--mode MODE] [--model DIR] [--out FILE] [--threshold T] "
                "[--device N]\n");
    std::printf("modes: offline, low_latency, very_low_latency, ultra_low_latency\n");
    return rc;
}

}  // namespace

// Where to look for the checkpoint when --model is not given: a sibling checkout of
// the project that owns the weights, then an in-tree models/ (src/bin/diarize.rs:33-45).
std::string default_model_dir() {
    const char* cands[] = {"../nemotron3-diarization/models/Nemotron-3-Diarization",
                           "../models/Nemotron-3-Diarization"};
    for (const char* c : cands)
        if (std::ifstream(std::string(c) + "/model.safetensors")) return c;
    return cands[1];
}

int main(int argc, char** argv) {
    std::string audio, model_dir = default_model_dir(), out;
    const ModeName* mode = &kModes[0];
    float threshold = 0.5f;
    int device = 0;
    try {
        for (int i = 1; i < argc; i++) {
            const std::string a = argv[i];
            auto value = [&](const char* flag) -> std::string {
                if (i + 1 >= argc) throw std::runtime_error(std::string(flag) + " needs a value");
                return argv[++i];
            };
            if (a == "--mode") {
                const std::string m = value("--mode");
                mode = nullptr;
                for (const ModeName& k : kModes)
                    if (m == k.arg) mode = &k;
                if (!mode) throw std::runtime_error("unknown mode " + m);
            } else if (a == "--model") {
                model_dir = value("--model");
            } else if (a == "--out") {
                out = value("--out");
            } else if (a == "--threshold") {
                const std::string v = value("--threshold");
                const auto r = std::from_chars(v.data(), v.data() + v.size(), threshold);
                if (r.ec != std::errc() || r.ptr != v.data() + v.size() || !std::isfinite(threshold))
                    throw std::runtime_error("--threshold needs a finite number, got " + v);
            } else if (a == "--device") {
                const std::string v = value("--device");
                const auto r = std::from_chars(v.data(), v.data() + v.size(), device);
                if (r.ec != std::errc() || r.ptr != v.data() + v.size() || device < 0)
                    throw std::runtime_error("--device needs a non-negative integer, got " + v);
            } else if (a == "--gpu") {
            } else if (a == "-h" || a == "--help") {
                return usage(0);
            } else if (a.rfind("--", 0) == 0) {
                throw std::runtime_error("unknown flag " + a);
            } else {
                audio = a;
            }
        }
        if (audio.empty()) throw std::runtime_error("no audio file given (try --help)");

        const auto t0 = std::chrono::steady_clock::now();
        const bool npy = audio.size() >= 4 && audio.compare(audio.size() - 4, 4, ".npy") == 0;
        const std::vector<float> samples = npy ? read_npy(audio) : read_wav(audio);
        n3d_model* model = nullptr;
        if (n3d_model_load_gpu(model_dir.c_str(), device, &model) != N3D_OK)
            throw std::runtime_error(std::string("model load: ") + n3d_last_error());
        const double loaded = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();

        const auto t1 = std::chrono::steady_clock::now();
        n3d_run_output r{};
        const n3d_status st = mode->mode == N3D_MODE_OFFLINE
                                  ? n3d_run_offline(model, samples.data(), samples.size(), &r)
                                  : n3d_run_streaming(model, samples.data(), samples.size(), mode->mode, &r);
        if (st != N3D_OK) throw std::runtime_error(std::string("run: ") + n3d_last_error());
        const double infer = std::chrono::duration<double>(std::chrono::steady_clock::now() - t1).count();

        // frame duration from the model's feature extractor (src/bin/diarize.rs:117-118)
        const n3d::json::Value proc = n3d::json::parse(read_bytes(model_dir + "/processor_config.json"));
        const n3d::json::Value* fe = proc.get("feature_extractor");
        if (!fe || !fe->get("hop_length") || !fe->get("sampling_rate"))
            throw std::runtime_error("processor_config.json: feature_extractor.hop_length / sampling_rate missing");
        const size_t hop = (size_t)fe->get("hop_length")->num;
        const uint32_t sr = (uint32_t)fe->get("sampling_rate")->num;
        const float dur = n3d_frame_duration(hop, sr);
        n3d_segment* segs = nullptr;
        size_t nseg = 0;
        if (n3d_extract_speaker_dict(r.logits, r.num_frames, r.num_speakers, dur, nullptr, threshold, &segs, &nseg) !=
            N3D_OK)
            throw std::runtime_error(std::string("segments: ") + n3d_last_error());
        std::vector<size_t> speakers;
        for (size_t s = 0; s < r.num_speakers; s++)
            for (size_t g = 0; g < nseg; g++)
                if (segs[g].speaker == s) {
                    speakers.push_back(s);
                    break;
                }
        const double duration_s = (double)samples.size() / (double)sr;
        const double rtfx = infer > 0.0 ? duration_s / infer : INFINITY;

        // keys in serde_json's (sorted) order, 2-space pretty printing
        std::ostringstream j;
        j << "{\n";
        j << "  \"audio\": " << quote(audio) << ",\n";
        j << "  \"cache_compressed\": " << (r.cache_compressed ? "true" : "false") << ",\n";
        j << "  \"cache_frames\": " << r.cache_frames << ",\n";
        j << "  \"duration_s\": " << number(round_to(duration_s, 1000.0)) << ",\n";
        j << "  \"fifo_frames\": " << r.fifo_frames << ",\n";
        j << "  \"forward_s\": " << number(round_to(infer, 1000.0)) << ",\n";
        j << "  \"load_s\": " << number(round_to(loaded, 1000.0)) << ",\n";
        j << "  \"mode\": " << quote(mode->report) << ",\n";
        j << "  \"num_chunks\": " << r.num_chunks << ",\n";
        j << "  \"num_frames\": " << r.num_frames << ",\n";
        j << "  \"num_segments\": " << nseg << ",\n";
        j << "  \"num_speakers\": " << speakers.size() << ",\n";
        j << "  \"rtfx\": " << number(round_to(rtfx, 100.0)) << ",\n";
        if (nseg == 0) {
            j << "  \"segments\": [],\n";
        } else {
            j << "  \"segments\": [\n";
            for (size_t g = 0; g < nseg; g++) {
                j << "    {\n";
                j << "      \"End\": " << number(round_to((double)segs[g].end, 100.0)) << ",\n";
                j << "      \"Speaker\": " << segs[g].speaker << ",\n";
                j << "      \"Start\": " << number(round_to((double)segs[g].start, 100.0)) << "\n";
                j << "    }" << (g + 1 < nseg ? "," : "") << "\n";
            }
            j << "  ],\n";
        }
        if (speakers.empty()) {
            j << "  \"speakers\": []\n";
        } else {
            j << "  \"speakers\": [\n";
            for (size_t s = 0; s < speakers.size(); s++)
                j << "    " << speakers[s] << (s + 1 < speakers.size() ? "," : "") << "\n";
            j << "  ]\n";
        }
        j << "}";
        n3d_segments_free(segs);
        n3d_run_output_free(&r);
        n3d_model_free(model);

        if (out.empty()) {
            std::printf("%s\n", j.str().c_str());
        } else {
            std::ofstream f(out);
            if (!f) throw std::runtime_error("cannot write " + out);
            f << j.str() << "\n";
            std::fprintf(stderr, "%.2fs audio, %s mode: %zu segments, %zu speakers in %.2fs (RTFx %.1f) -> %s\n",
                         duration_s, mode->report, nseg, speakers.size(), infer, rtfx, out.c_str());
        }
    } catch (const std::exception& e) {
        std::fprintf(stderr, "Error: %s\n", e.what());
        return 1;
    }
    return 0;
}
