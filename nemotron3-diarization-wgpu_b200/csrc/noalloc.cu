// Allocation-free variant of tensor::linear (src/tensor.rs:22-57) on the GPU.
//
// n3d_linear needs temporary device memory for the fp16 split (h, l) of
// its operands and gets it from cudaMalloc.  Some callers cannot allocate device
// memory at the point where they call: a real-time audio thread that must not
// block in the driver's allocator, a host framework that has reserved all of
// the GPU's memory for its own pool and hands out only its own buffers, or a
// process whose allocation budget is fixed after start-up.  For them this
// file keeps the scratch in a fixed array that is part of the library's GPU
// image, so a call allocates nothing: no cudaMalloc, no cudaFree, no
// allocating library routine, no host-heap map cache.
//
// Limits and sharing rules:
//  * the scratch holds kScratchFloats 4-byte words (16 MiB).  The first 64 hold the
//    two operands' max |x| (which set their fp16-split scales); the split of each
//    operand takes n fp16 values twice, i.e. n words rounded up to 64, so
//    rows * cols + out * cols may be at most 4 Mi - 64; larger requests are
//    rejected with N3D_ERR_INVALID_ARGUMENT.
//  * every GPU that loads the library holds these 16 MiB until the process
//    exits.
//  * all calls on a device share the one array and it keeps the last call's
//    contents; calls whose GPU work overlaps (different streams, different
//    host threads) race on it and must be serialised by the caller.
//  * the first call on each device does the set-up: it resolves the device
//    address of the array (which also loads the library's GPU code onto that
//    device).  Make that first call before any stream capture.

#include <climits>
#include <mutex>

#include "n3d_device.cuh"
#include "n3d_internal.h"

namespace n3d {

namespace {

constexpr size_t kScratchFloats = size_t(4) << 20;  // 16 MiB
__device__ __align__(256) float g_linear_scratch[kScratchFloats];
__device__ int g_linear_status;  // bounded-wait status word of the GEMM

struct DeviceSymbols {
    float* scratch = nullptr;
    int* status = nullptr;
};

// Host copies of the two symbols' device addresses, resolved once per device.
DeviceSymbols g_symbols[128];
std::mutex g_symbols_mu;

DeviceSymbols symbols_for(int device) {
    if (device < 0 || device >= 128) throw Error(12, "n3d_linear_noalloc: bad device index");
    std::lock_guard<std::mutex> lock(g_symbols_mu);
    DeviceSymbols& s = g_symbols[device];
    if (!s.scratch) {
        cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.scratch), g_linear_scratch);
        if (e != cudaSuccess) {
            s.scratch = nullptr;
            throw Error(10, std::string("n3d_linear_noalloc set-up: cudaGetSymbolAddress(scratch): ") +
                                cudaGetErrorString(e));
        }
        e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.status), g_linear_status);
        if (e != cudaSuccess) {
            s.scratch = nullptr;
            throw Error(10, std::string("n3d_linear_noalloc set-up: cudaGetSymbolAddress(status): ") +
                                cudaGetErrorString(e));
        }
    }
    return s;
}

size_t round64(size_t n) { return (n + 63) & ~size_t(63); }

// One operand's fp16 split carved out of the scratch: h and l (n fp16 each), each
// part starting on a 256-byte boundary; n words in all, rounded up to 64.
struct Carve {
    void* h;
    void* l;
    float* next;
};
Carve carve(float* p, size_t n) {
    const size_t nf = round64(n);  // words, a multiple of 64 (256 bytes)
    Carve c;
    c.h = p;
    c.l = p + nf / 2;
    c.next = p + nf;
    return c;
}

}  // namespace

size_t linear_noalloc_capacity() { return kScratchFloats; }

void linear_noalloc(int device, const float* d_x, size_t rows, size_t cols, const float* d_w, size_t out,
                    const float* d_bias, float* d_y, cudaStream_t stream) {
    if (!d_x || !d_w || !d_y) throw Error(13, "n3d_linear_noalloc: null argument");
    if (cols == 0 || cols % 32) throw Error(13, "n3d_linear_noalloc: cols must be a positive multiple of 32");
    // the same limits as n3d_linear: the kernels count rows, columns and outputs in int
    if (rows > (size_t)INT_MAX || cols > (size_t)INT_MAX || out > (size_t)INT_MAX)
        throw Error(13, "n3d_linear_noalloc: sizes beyond 2^31");
    if (rows == 0 || out == 0) return;
    // each operand on its own first (rows * cols < 2^62 cannot wrap), so the sum below cannot wrap either
    const bool fits = rows * cols <= kScratchFloats && out * cols <= kScratchFloats;
    const size_t need = fits ? 64 + round64(rows * cols) + round64(out * cols) : 0;  // maxima, then h + l per operand
    if (!fits || need > kScratchFloats)
        throw Error(13, "n3d_linear_noalloc: the request needs more scratch than the fixed " +
                            std::to_string(kScratchFloats) +
                            " words (rows*cols + out*cols must stay within 4194240)");
    N3D_CUDA(cudaSetDevice(device));
    const DeviceSymbols sym = symbols_for(device);
    float* maxima = sym.scratch;  // [0]: max |x|, [1]: max |w|
    const Carve x = carve(sym.scratch + 64, rows * cols);
    const Carve w = carve(x.next, out * cols);
    // the status word and the maxima start at zero for every call; the split arrays are
    // fully overwritten
    N3D_CUDA(cudaMemsetAsync(sym.status, 0, sizeof(int), stream));
    N3D_CUDA(cudaMemsetAsync(maxima, 0, 2 * sizeof(float), stream));
    launch_absmax(stream, d_x, (long long)(rows * cols), maxima);
    launch_absmax(stream, d_w, (long long)(out * cols), maxima + 1);
    float hm[2] = {0.0f, 0.0f};
    N3D_CUDA(cudaMemcpyAsync(hm, maxima, sizeof(hm), cudaMemcpyDeviceToHost, stream));
    N3D_CUDA(cudaStreamSynchronize(stream));
    const float sx = split_scale(hm[0]), sw = split_scale(hm[1]);
    launch_split(stream, d_x, (long long)(rows * cols), SplitOut{x.h, x.l, sx, nullptr});
    launch_split(stream, d_w, (long long)(out * cols), SplitOut{w.h, w.l, sw, nullptr});
    Epi e;
    e.mode = EPI_STORE;
    e.bias = d_bias;
    e.out = d_y;
    e.ldo = (long long)out;
    gemm_split_stack_maps(stream, SplitOperand{x.h, x.l, (long long)rows, (long long)cols, (long long)cols, sx},
                          SplitOperand{w.h, w.l, (long long)out, (long long)cols, (long long)cols, sw},
                          (int)rows, (int)out, (int)cols, e, sym.status);
    // read the status word back on the caller's stream only (one plain copy), so the call
    // waits for its own work and not for other streams of the device
    int status = 0;
    N3D_CUDA(cudaMemcpyAsync(&status, sym.status, sizeof(int), cudaMemcpyDeviceToHost, stream));
    N3D_CUDA(cudaStreamSynchronize(stream));
    if (status) throw Error(11, "n3d_linear_noalloc: a device-side wait timed out (site " + std::to_string(status) + ")");
}

}  // namespace n3d
