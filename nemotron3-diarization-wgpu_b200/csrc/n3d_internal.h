// Internal host/device interfaces of the diarization path (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>

namespace n3d {

// Error carrying an n3d_status code (include/n3d.h) up to the C ABI.
struct Error : std::runtime_error {
    int status;
    Error(int s, const std::string& m) : std::runtime_error(m), status(s) {}
};

void cuda_check(cudaError_t e, const char* what);
#define N3D_CUDA(x) ::n3d::cuda_check((x), #x)

// Per-device tables below hold this many devices.
constexpr int kMaxDevices = 64;

// The current CUDA device, checked against kMaxDevices.
inline int current_device() {
    int dev = 0;
    N3D_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) throw Error(12 /*N3D_ERR_NO_DEVICE*/, "CUDA device index beyond 63");
    return dev;
}

// Runs `set_up` once on each device for the call site that owns `done`.  A kernel's
// attributes (its dynamic shared-memory limit, for one) belong to the current device,
// so a process that drives several GPUs must set them on every one; concurrent first
// calls wait for each other.
template <class F>
void once_per_device(std::atomic<unsigned long long>& done, F&& set_up) {
    const unsigned long long bit = 1ull << current_device();
    if (done.load(std::memory_order_acquire) & bit) return;
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (done.load(std::memory_order_relaxed) & bit) return;
    set_up();
    done.fetch_or(bit, std::memory_order_release);
}

// Launch with programmatic stream serialization: the kernel may become resident and
// run its set-up while the previous kernel of the stream drains.  Every kernel launched
// this way calls griddep_wait() (n3d_device.cuh) before it touches global memory that
// another kernel writes or reads, and griddep_launch_dependents() right after, so at
// most two such kernels are in flight.
template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    N3D_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// ------------------------------------------------------------------ GEMM

// Epilogue applied to each accumulator tile of C = A * B^T.
// Every mode first forms v = acc * acc_scale + bias, where acc_scale = 1 / (s_A s_B)
// undoes the operands' power-of-two scales (exact).
enum EpiMode : int {
    EPI_STORE = 0,       // out[r, c] = v                               (fp32)
    EPI_SPLIT = 1,       // fp16 split of v * out_scale -> out_h, out_l
    EPI_GELU_SPLIT = 2,  // fp16 split of gelu(v) * out_scale
    EPI_RELU_SPLIT = 4,  // fp16 split of relu(v) * out_scale
    EPI_DENSE_OUT = 6,   // r = relu(v); out[r, 0:ns] = r . w2^T + b2
    EPI_QKV_ATTN = 7,    // Q, K rotated by RoPE -> fp16 splits [rows, heads*64] (map_h / map_l,
                         // map_k_*); V -> transposed fp16 split V^T[head*64 + d][row] (map_vt_*), with
                         // the scales sec_scale[0..2]; TMA only
};

struct Epi {
    int mode = EPI_STORE;
    const float* bias = nullptr;
    float acc_scale = 1.0f;  // set by gemm_split from the operands' scales
    float out_scale = 1.0f;  // the split modes' output scale (the consumer operand's s)
    float sec_scale[3] = {1.0f, 1.0f, 1.0f};  // EPI_QKV_ATTN: the Q, K and V scales
    // Direct stores: out (fp32, EPI_STORE and EPI_DENSE_OUT), out_h and out_l (the
    // fp16 arrays of the split modes).
    float* out = nullptr;
    void* out_h = nullptr;
    void* out_l = nullptr;
    long long ldo = 0;
    // Row remap: q = r / rdiv, t = r % rdiv; rows with t >= rkeep are skipped;
    // the output row is q * rmul + t + roff.
    int rdiv = 0x7fffffff, rkeep = 0x7fffffff;
    long long rmul = 0, roff = 0;
    // Rows with t >= seq_len[q] are written as zeros (needs rdiv = sequence stride).
    const int* seq_len = nullptr;
    // RoPE tables [max_pos, head_dim]; position = r % rope_seq.
    const float* cos_t = nullptr;
    const float* sin_t = nullptr;
    int rope_seq = 1;
    int head_dim = 64;
    int q_cols = 0, k_cols = 0;  // [0,q_cols) is Q, [q_cols,q_cols+k_cols) is K
    // Stores through TMA (tma != 0), box 32 columns x 32 rows: map_out fp32 (128-byte
    // swizzle, make_store_map), map_h / map_l fp16 (64-byte swizzle,
    // make_store_map_f16).  EPI_QKV_ATTN: fp16 maps from make_f16_map -- map_h /
    // map_l (Q) and map_k_* with box 64 x 32 and the 128-byte swizzle, map_vt_* over
    // V^T [heads*64, rows] with box 32 x 64 and no swizzle.
    int tma = 0;
    // EPI_STORE through TMA only: add the tile into map_out's fp32 destination
    // (cp.reduce.async.bulk.tensor .add; each element is added exactly once).
    int reduce = 0;
    // Optional split-K scratch for such reduce-add GEMMs (destination `out`, row
    // stride `ldo`): when a launch would leave most SMs idle, K is split over up to 4
    // CTAs per tile, each writing its partial tile here, and a second kernel adds
    // ((p0 + p1 + ...) + bias) into the destination in split order (deterministic).
    float* split_ws = nullptr;
    long long split_ws_floats = 0;
    CUtensorMap map_out, map_h, map_l, map_k_h, map_k_l, map_vt_h, map_vt_l;
    // EPI_DENSE_OUT second projection
    const float* w2 = nullptr;
    const float* b2 = nullptr;
    int n2 = 0;
};

// A K-major GEMM operand [rows, cols] in the fp16 split, row stride ld (elements,
// shared by both arrays): for the logical fp32 values x and the operand's power-of-two
// scale s, h = RN-fp16(x s) and l = RN-fp16(x s - h).
struct SplitOperand {
    const void* h = nullptr;
    const void* l = nullptr;
    long long rows = 0, cols = 0, ld = 0;
    float scale = 1.0f;
};

// The power-of-two scale for a tensor whose magnitudes are at most `bound`:
// bound * s <= 2^15 (half the fp16 range), s as large as that allows, within
// [2^-60, 2^60]; 1 for a zero or non-finite bound.
float split_scale(double bound);

// TMA-store maps (box 32 x 32) over a row-major fp32 matrix (128-byte swizzle) or
// fp16 matrix (64-byte swizzle).
// Streaming multiprocessors of the current device.
int sm_count();
CUtensorMap make_store_map(const float* p, long long rows, long long cols, long long ld);
CUtensorMap make_store_map_f16(const void* p, long long rows, long long cols, long long ld);
// 2-D map over a row-major fp16 matrix [rows, cols] with row stride ld elements;
// box box_cols x box_rows, 128-byte swizzle when `swizzle` (box_cols must then be 64).
CUtensorMap make_f16_map(const void* p, long long rows, long long cols, long long ld, int box_cols, int box_rows,
                         bool swizzle);

// C[M, N] = A[M, K] * B[N, K]^T with the fp16 split on tcgen05 (gemm.cu).  K % 32 == 0
// (k-blocks of 64; a last half block reads zeros past K).  `kb_per_tap` > 0 turns on
// the shifted-row (implicit k=3 conv) mode: k-block kb (of 64) reads A at column
// (kb % kb_per_tap) * 64 and row m0 + kb / kb_per_tap.
void gemm_split(cudaStream_t s, const SplitOperand& A, const SplitOperand& B, int M, int N, int K, int kb_per_tap,
                const Epi& epi, int* dev_err);
// Same with tensor maps encoded on the stack (no host allocation), 128 x 128 tiles.
void gemm_split_stack_maps(cudaStream_t s, const SplitOperand& A, const SplitOperand& B, int M, int N, int K,
                           const Epi& epi, int* dev_err);

// --------------------------------------------------------------- other kernels
// Destination of a producer of GEMM operands: the two fp16 arrays of the split of
// x * scale (row stride = the producer's row length), or plain fp32 into `plain` when
// h == nullptr.
struct SplitOut {
    void* h = nullptr;
    void* l = nullptr;
    float scale = 1.0f;
    float* plain = nullptr;
};
inline SplitOut plain_out(float* p) {
    SplitOut o;
    o.plain = p;
    return o;
}
void launch_layer_norm(cudaStream_t s, const float* x, long long rows, int cols, const float* w, const float* b,
                       SplitOut out);
// One mel segment of a launch: global frames [f_begin, next segment's f_begin) are
// frames frame_lo.. of a segment whose `len` samples start at audio[base]; frame t
// reads samples t * hop - (centered ? 256 : 0) + [0, 512) (zeros outside [0, len))
// and writes mel row out_row0 + (f - f_begin).  Segments are sorted by f_begin.
struct MelSegDev {
    long long base, out_row0, f_begin;
    int len, frame_lo, centered, pad;
};
// The log-mel's constant tables (device pointers): the centred Hann window [512], the
// 256 twiddles as (cos, sin) pairs, and the slaney filterbank in its sparse, transposed
// form: filter m's weights for bins filt_lo[m] + i at fbank_t[i * 128 + m] for
// i < filt_w[m] (zeros up to fb_w rows), group_w[q] = the widest filter of mels
// 32q..32q+31.
struct MelTables {
    const float* window = nullptr;
    const float* twiddle = nullptr;
    const float* fbank_t = nullptr;
    const int* filt_lo = nullptr;
    const int* filt_w = nullptr;
    int fb_w = 0;
    int group_w[4] = {0, 0, 0, 0};
};
constexpr int MEL_FB_MAX_W = 64;  // widest filter the kernel's shared table holds
// Log-mel of global frames [f_first, f_first + n_frames) of the segment table into
// [rows, 128] outputs (fp16 split, plain optional).
void launch_mel(cudaStream_t s, const float* audio, const MelSegDev* segs, int nsegs, long long f_first,
                long long n_frames, int hop, const MelTables& tab, float preemph, SplitOut mel, float* mel_plain);
// x -> the fp16 split of x * out.scale, elementwise (n % 4 == 0).
void launch_split(cudaStream_t s, const float* x, long long n, SplitOut out);
// max |x| over n floats (n % 4 == 0) into *d_max (a float the caller zeroes first).
void launch_absmax(cudaStream_t s, const float* x, long long n, float* d_max);
// Operands of the tcgen05 attention (head_dim hd = 64 or 128), all in the fp16 split
// (h, l) of the values times their power-of-two scale: Q, K [rows_cap, heads*hd] with
// sequence b at rows b*S..; V^T [heads*hd, vt_ld] whose column is the global row.
struct AttnOperands {
    const void *q_h = nullptr, *q_l = nullptr, *k_h = nullptr, *k_l = nullptr;
    long long rows_cap = 0;
    const void *vt_h = nullptr, *vt_l = nullptr;
    long long vt_ld = 0;
    float q_scale = 1.0f, k_scale = 1.0f, v_scale = 1.0f;
};
// tcgen05 attention (attention_tc.cu), head_dim 64 or 128; S (when seqs > 1) and
// vt_ld must be multiples of 8.  Context [seqs*S, heads*hd] in the fp16 split (or
// plain fp32).
void launch_attention_tc(cudaStream_t s, const AttnOperands& op, int seqs, int S, const int* valid, int heads,
                         int hd, SplitOut ctx, int* err);
// q, k, v [seq, heads*hd] -> the attention operands (RoPE on q, k when cos_t != nullptr).
void launch_pack_attn(cudaStream_t s, const float* q, const float* k, const float* v, long long seq, int heads,
                      int hd, const float* cos_t, const float* sin_t, const AttnOperands& op);
// The bounded-wait self-test kernel: a wait on a flag that nothing sets, limited to
// limit_ns; it records its timeout in *err and writes the time waited (ns) to *waited.
void launch_wait_probe(cudaStream_t s, int* err, unsigned long long limit_ns, unsigned long long* waited);
// Synthetic benchmark operands: p[i] ~ scale * (sum of 4 hashed uniforms in [-1, 1)).
void launch_fill_random(cudaStream_t s, float* p, long long n, uint32_t seed, float scale);
// tensor::linear without any allocation: scratch is a fixed device array (noalloc.cu).
void linear_noalloc(int device, const float* d_x, size_t rows, size_t cols, const float* d_w, size_t out,
                    const float* d_bias, float* d_y, cudaStream_t stream);
size_t linear_noalloc_capacity();

}  // namespace n3d
