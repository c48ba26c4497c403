// Reader of .safetensors checkpoints, the format the reference loads its weights from
// (src/weights.rs, safetensors 0.4.5): an 8-byte little-endian header length, a JSON
// header {name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": ...},
// then the tensor bytes, offsets counted from the end of the header.  Host only.
//
// A damaged file is an error with a message, never a read outside the file: every
// shape dimension and offset must be a non-negative integer, the element count must
// match the byte range without overflowing, and the range must lie inside the file.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>
#include <string>
#include <vector>

#include "json.h"
#include "n3d_internal.h"

namespace n3d {

struct Tensor {
    std::vector<long long> shape;
    const float* data;
};

struct SafeTensors {
    std::string raw;
    std::map<std::string, Tensor> tensors;

    explicit SafeTensors(const std::string& path) {
        {
            std::ifstream f(path, std::ios::binary);
            if (!f) throw Error(1 /*N3D_ERR_IO*/, "io error at " + path + ": cannot open");
            std::ostringstream ss;
            ss << f.rdbuf();
            raw = ss.str();
        }
        if (raw.size() < 8) fail("file too short");
        uint64_t hlen = 0;
        std::memcpy(&hlen, raw.data(), 8);
        if (hlen > raw.size() - 8) fail("header out of range");
        json::Value h;
        try {
            h = json::parse(raw.substr(8, hlen));
        } catch (const std::exception& e) {
            fail(e.what());
        }
        if (h.kind != json::Value::Obj) fail("the header is not an object");
        const uint64_t base = 8 + hlen, body = raw.size() - base;
        for (const auto& kv : h.obj) {
            if (kv.first == "__metadata__") continue;
            const json::Value& t = kv.second;
            const json::Value* dt = t.get("dtype");
            const json::Value* sh = t.get("shape");
            const json::Value* off = t.get("data_offsets");
            if (t.kind != json::Value::Obj || !dt || !sh || !off || dt->kind != json::Value::Str ||
                sh->kind != json::Value::Arr || off->kind != json::Value::Arr || off->arr.size() != 2)
                fail("bad entry " + kv.first);
            if (dt->str != "F32")
                throw Error(4 /*N3D_ERR_TENSOR_DTYPE*/,
                            "tensor `" + kv.first + "` has dtype " + dt->str + ", this port only reads F32");
            uint64_t s = 0, e = 0;
            if (!index(off->arr[0], body, s) || !index(off->arr[1], body, e) || e < s)
                fail("bad data offsets for " + kv.first);
            // element count, checked against the byte range as it grows (no overflow)
            Tensor tt;
            uint64_t numel = 1;
            for (const auto& d : sh->arr) {
                uint64_t n = 0;
                if (!index(d, body, n)) fail("bad shape for " + kv.first);
                tt.shape.push_back((long long)n);
                numel = n == 0 ? 0 : numel;
                if (numel && n > (e - s) / 4 / numel) fail("bad data offsets for " + kv.first);
                numel *= n;
            }
            if (numel * 4 != e - s) fail("bad data offsets for " + kv.first);
            if ((base + s) % 4) fail("misaligned tensor " + kv.first);
            tt.data = reinterpret_cast<const float*>(raw.data() + base + s);
            tensors[kv.first] = tt;
        }
    }

    // Weights::tensor (src/weights.rs:78-93): fetch with a shape check.
    const float* get(const std::string& name, std::vector<long long> shape) const {
        auto it = tensors.find(name);
        if (it == tensors.end())
            throw Error(5 /*N3D_ERR_MISSING_TENSOR*/, "tensor `" + name + "` is missing from the checkpoint");
        if (it->second.shape != shape) {
            auto fmt = [](const std::vector<long long>& v) {
                std::string s = "[";
                for (size_t i = 0; i < v.size(); i++) s += (i ? ", " : "") + std::to_string(v[i]);
                return s + "]";
            };
            throw Error(6 /*N3D_ERR_TENSOR_SHAPE*/,
                        "tensor `" + name + "` has shape " + fmt(it->second.shape) + ", expected " + fmt(shape));
        }
        return it->second.data;
    }

  private:
    [[noreturn]] static void fail(const std::string& what) {
        throw Error(3 /*N3D_ERR_SAFETENSORS*/, "safetensors error: " + what);
    }
    // A header number used as a size or offset: an integer in [0, limit].
    static bool index(const json::Value& v, uint64_t limit, uint64_t& out) {
        if (v.kind != json::Value::Num || v.num < 0 || v.num != std::floor(v.num) || v.num > (double)limit)
            return false;
        out = (uint64_t)v.num;
        return true;
    }
};

}  // namespace n3d
