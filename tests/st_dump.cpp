// Test helper for tests/test_safetensors.py: opens a .safetensors file with the
// library's checkpoint reader (csrc/safetensors.h) and prints, per tensor, its name,
// shape and the double-precision sum of its values; or the error status and message.
// Exit code 0 when the file was read, 1 for a reported error.
#include <cstdio>

#include "../nemotron3-diarization-wgpu_b200/csrc/safetensors.h"

int main(int argc, char** argv) {
    try {
        const n3d::SafeTensors st(argv[1]);
        for (const auto& kv : st.tensors) {
            long long numel = 1;
            std::printf("%s [", kv.first.c_str());
            for (size_t i = 0; i < kv.second.shape.size(); i++) {
                std::printf(i ? ",%lld" : "%lld", kv.second.shape[i]);
                numel *= kv.second.shape[i];
            }
            double sum = 0.0;
            for (long long i = 0; i < numel; i++) sum += kv.second.data[i];
            std::printf("] %.17g\n", sum);
        }
    } catch (const n3d::Error& e) {
        std::printf("error %d %s\n", e.status, e.what());
        return 1;
    }
    return 0;
}
