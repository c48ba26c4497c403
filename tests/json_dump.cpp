// Test helper for tests/test_config_parse.py: parses a JSON document (or, with
// --safetensors, the header of a .safetensors file) with the library's reader
// (csrc/json.h) and prints it back in a canonical form that Python can compare:
// objects in file order, numbers with 17 significant digits.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>

#include "../nemotron3-diarization-wgpu_b200/csrc/json.h"

static void dump(const n3d::json::Value& v, std::string& o) {
    using V = n3d::json::Value;
    char buf[64];
    switch (v.kind) {
        case V::Null: o += "null"; break;
        case V::Bool: o += v.b ? "true" : "false"; break;
        case V::Num: std::snprintf(buf, sizeof buf, "%.17g", v.num); o += buf; break;
        case V::Str: o += "\"" + v.str + "\""; break;
        case V::Arr:
            o += "[";
            for (size_t i = 0; i < v.arr.size(); i++) {
                if (i) o += ",";
                dump(v.arr[i], o);
            }
            o += "]";
            break;
        case V::Obj:
            o += "{";
            for (size_t i = 0; i < v.obj.size(); i++) {
                if (i) o += ",";
                o += "\"" + v.obj[i].first + "\":";
                dump(v.obj[i].second, o);
            }
            o += "}";
            break;
    }
}

int main(int argc, char** argv) {
    const bool st = argc > 2 && std::strcmp(argv[1], "--safetensors") == 0;
    std::ifstream f(argv[st ? 2 : 1], std::ios::binary);
    std::ostringstream ss;
    ss << f.rdbuf();
    std::string text = ss.str();
    if (st) {
        uint64_t n = 0;
        std::memcpy(&n, text.data(), 8);
        text = text.substr(8, n);
    }
    try {
        std::string o;
        dump(n3d::json::parse(text), o);
        std::printf("%s\n", o.c_str());
    } catch (const std::exception& e) {
        std::printf("error: %s\n", e.what());
        return 1;
    }
    return 0;
}
