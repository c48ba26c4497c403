// Memory-bound and small kernels of the diarization path: LayerNorm, the fused
// log-mel front-end, the operand split and the attention operand packing.

#include <algorithm>
#include <cfloat>
#include <cmath>

#include "n3d_device.cuh"
#include "n3d_internal.h"

namespace n3d {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------- LayerNorm
// torch LayerNorm, eps 1e-5, two-pass population variance (src/tensor.rs:97-110).
// One warp per RPW rows, VPL values per lane and row held in registers (128-bit
// loads, all of a warp's rows issued before any reduction, so each warp keeps RPW
// rows of loads in flight; VPL a multiple of 8).  Writes either a plain fp32 row (out.h == nullptr) or the
// fp16 split of row * out.scale.
template <int VPL, int RPW>
__global__ void layer_norm_kernel(const float* __restrict__ x, long long rows, const float* __restrict__ w,
                                  const float* __restrict__ b, SplitOut out) {
    griddep_wait();
    griddep_launch_dependents();
    constexpr int COLS = VPL * 32;
    const long long row0 = ((long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW;
    const int lane = threadIdx.x & 31;
    if (row0 >= rows) return;
    // lane L holds columns 256 c + 8 L .. + 7 of chunk c: two 16-byte loads, and the
    // split's 8 fp16 per array leave as one 16-byte store
    float v[RPW][VPL];
#pragma unroll
    for (int k = 0; k < RPW; k++) {
        if (row0 + k >= rows) break;
        const float* src = x + (row0 + k) * COLS;
#pragma unroll
        for (int i = 0; i < VPL; i += 8) {
            const float4 t0 = *reinterpret_cast<const float4*>(src + (i / 8) * 256 + lane * 8);
            const float4 t1 = *reinterpret_cast<const float4*>(src + (i / 8) * 256 + lane * 8 + 4);
            v[k][i] = t0.x, v[k][i + 1] = t0.y, v[k][i + 2] = t0.z, v[k][i + 3] = t0.w;
            v[k][i + 4] = t1.x, v[k][i + 5] = t1.y, v[k][i + 6] = t1.z, v[k][i + 7] = t1.w;
        }
    }
    float mean[RPW], inv[RPW];
#pragma unroll
    for (int k = 0; k < RPW; k++) {
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < VPL; i++) s += v[k][i];
        mean[k] = __fdiv_rn(warp_sum(s), (float)COLS);
    }
#pragma unroll
    for (int k = 0; k < RPW; k++) {
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < VPL; i++) {
            const float d = __fsub_rn(v[k][i], mean[k]);
            q = __fadd_rn(q, __fmul_rn(d, d));
        }
        const float var = __fdiv_rn(warp_sum(q), (float)COLS);
        inv[k] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
    }
#pragma unroll
    for (int k = 0; k < RPW; k++) {
        const long long row = row0 + k;
        if (row >= rows) break;
        float* dst = out.h ? nullptr : out.plain + row * COLS;
        uint16_t* dh = out.h ? static_cast<uint16_t*>(out.h) + row * COLS : nullptr;
        uint16_t* dl = out.h ? static_cast<uint16_t*>(out.l) + row * COLS : nullptr;
#pragma unroll
        for (int i = 0; i < VPL; i += 8) {
            const int c = (i / 8) * 256 + lane * 8;
            float y[8];
#pragma unroll
            for (int j4 = 0; j4 < 8; j4 += 4) {
                const float4 w4 = __ldg(reinterpret_cast<const float4*>(w + c + j4));
                const float4 b4 = __ldg(reinterpret_cast<const float4*>(b + c + j4));
                const float ww[4] = {w4.x, w4.y, w4.z, w4.w}, bb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
                for (int j = 0; j < 4; j++)
                    y[j4 + j] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[k][i + j4 + j], mean[k]), inv[k]), ww[j]),
                                          bb[j]);
            }
            if (dh) {
                uint2 h0, l0, h1, l1;
                split2x4(y, out.scale, h0, l0);
                split2x4(y + 4, out.scale, h1, l1);
                *reinterpret_cast<uint4*>(dh + c) = make_uint4(h0.x, h0.y, h1.x, h1.y);
                *reinterpret_cast<uint4*>(dl + c) = make_uint4(l0.x, l0.y, l1.x, l1.y);
            } else {
                *reinterpret_cast<float4*>(dst + c) = make_float4(y[0], y[1], y[2], y[3]);
                *reinterpret_cast<float4*>(dst + c + 4) = make_float4(y[4], y[5], y[6], y[7]);
            }
        }
    }
}

// ------------------------------------------------------------------- log-mel
// One warp per frame, 8 frames per CTA: preemphasis on the fly, centred 400-tap
// Hann in the 512 frame, radix-2 DIT FFT in registers, power, sparse slaney
// filterbank, ln(x + 2^-24) (src/mel.rs:160-225).  The butterflies (pairs,
// twiddles, operation order) and the filterbank accumulation order are the CPU
// restatement's exactly and every operation is explicitly rounded, so the spectrum
// is bit-identical to it; only the assignment of butterflies to lanes is this
// kernel's own.
//   layout A: lane L holds bit-reversed positions 16L + s (s = 0..15): stages with
//             half 1, 2, 4, 8 in registers; half 16 pairs lanes L and L ^ 1 (shuffles)
//   layout B: lane L holds positions L + 32t (t = 0..15), reached through shared
//             memory (padded: no bank conflicts either way): halves 32..256 in registers
// Shared-memory reads are conflict-free: the stages of layout A read one twiddle for
// the whole warp; those of layout B read per-stage copies of their twiddles, indexed
// by lane (stage h: twiddle (lane + 32u) * 256 / h at position lane + 32u); the
// filterbank reads its weights transposed (lane m reads word i * 128 + m).
constexpr int NFFT = 512;
constexpr int NBINS = NFFT / 2 + 1;
constexpr int MEL_WARPS = 8;
constexpr int MEL_PAD = NFFT + NFFT / 32;  // padded index p + p / 32
constexpr int TWB = 32 + 64 + 128 + 256;   // layout B's per-stage twiddle copies
__host__ __device__ constexpr int twb_offset(int h) { return h - 32; }  // 32 -> 0, 64 -> 32, 128 -> 96, 256 -> 224

// One radix-2 butterfly with twiddle (wr, wi): (u, x) -> (u + x w, u - x w).
__device__ __forceinline__ void butterfly(float& ur, float& ui, float& xr, float& xi, float wr, float wi) {
    const float vr = __fsub_rn(__fmul_rn(xr, wr), __fmul_rn(xi, wi));
    const float vi = __fadd_rn(__fmul_rn(xr, wi), __fmul_rn(xi, wr));
    xr = __fsub_rn(ur, vr);
    xi = __fsub_rn(ui, vi);
    ur = __fadd_rn(ur, vr);
    ui = __fadd_rn(ui, vi);
}

__global__ void __launch_bounds__(MEL_WARPS * 32) mel_kernel(
    const float* __restrict__ audio, const MelSegDev* __restrict__ segs, int nsegs, long long f_first,
    long long n_frames, int hop, const MelTables tab, float preemph, SplitOut mel, float* __restrict__ mel_plain) {
    __shared__ float tw_s[NFFT];  // (cos, sin) pairs of the 256 twiddles
    __shared__ float win_s[NFFT];
    __shared__ float twb_re[TWB], twb_im[TWB];
    __shared__ float xs[MEL_WARPS][2][MEL_PAD];
    extern __shared__ float fb_s[];  // [fb_w][128]
    for (int i = threadIdx.x; i < NFFT; i += blockDim.x) {
        tw_s[i] = tab.twiddle[i];
        win_s[i] = tab.window[i];
    }
    for (int i = threadIdx.x; i < TWB; i += blockDim.x) {
        const int h = i < 32 ? 32 : i < 96 ? 64 : i < 224 ? 128 : 256;
        const int t = (i - twb_offset(h)) * (NFFT / 2 / h);
        twb_re[i] = tab.twiddle[2 * t];
        twb_im[i] = tab.twiddle[2 * t + 1];
    }
    for (int i = threadIdx.x; i < tab.fb_w * 128; i += blockDim.x) fb_s[i] = tab.fbank_t[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long f = f_first + (long long)blockIdx.x * MEL_WARPS + warp;
    if (f >= f_first + n_frames) return;
    int lo = 0, hi = nsegs - 1;  // the segment holding frame f: last f_begin <= f
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (segs[mid].f_begin <= f) lo = mid;
        else hi = mid - 1;
    }
    const MelSegDev sg = segs[lo];
    const long long base = sg.base;
    const int p0 = (sg.frame_lo + (int)(f - sg.f_begin)) * hop - (sg.centered ? NFFT / 2 : 0), n = sg.len;
    float re[16], im[16];
    // ---- input at bit-reversed positions (layout A): position 16L + s <- sample
    // j = brev9(16L + s) = brev4(s) * 32 + brev5(L)
    const int jl = __brev(lane) >> 27;
#pragma unroll
    for (int s = 0; s < 16; s++) {
        const int j = ((__brev(s) >> 28) << 5) | jl;
        const int p = p0 + j;
        float x = 0.0f;
        if (p >= 0 && p < n) {
            const float cur = audio[base + p];
            x = p >= 1 ? __fsub_rn(cur, __fmul_rn(preemph, audio[base + p - 1])) : cur;
        }
        re[s] = __fmul_rn(x, win_s[j]);
        im[s] = 0.0f;
    }
    // ---- halves 1, 2, 4, 8 inside the lane: pair (s, s + h), twiddle (s % h) * 256 / h
#pragma unroll
    for (int h = 1; h <= 8; h <<= 1) {
#pragma unroll
        for (int s = 0; s < 16; s++) {
            if (s & h) continue;
            const int t = (s & (h - 1)) * (NFFT / 2 / h);
            butterfly(re[s], im[s], re[s + h], im[s + h], tw_s[2 * t], tw_s[2 * t + 1]);
        }
    }
    // ---- half 16: positions 16L + s pair with lane L ^ 1; twiddle s * 16.  Both
    // lanes form v = x w from the upper value with the same operations.
    {
        const bool upper = lane & 1;
#pragma unroll
        for (int s = 0; s < 16; s++) {
            const float pr = __shfl_xor_sync(0xffffffffu, re[s], 1), pi = __shfl_xor_sync(0xffffffffu, im[s], 1);
            float ur = upper ? pr : re[s], ui = upper ? pi : im[s];
            float xr = upper ? re[s] : pr, xi = upper ? im[s] : pi;
            butterfly(ur, ui, xr, xi, tw_s[2 * (s * 16)], tw_s[2 * (s * 16) + 1]);
            re[s] = upper ? xr : ur;
            im[s] = upper ? xi : ui;
        }
    }
    // ---- layout A -> B through shared memory
    float* xr_s = xs[warp][0];
    float* xi_s = xs[warp][1];
#pragma unroll
    for (int s = 0; s < 16; s++) {
        const int p = 16 * lane + s;
        xr_s[p + (p >> 5)] = re[s];
        xi_s[p + (p >> 5)] = im[s];
    }
    __syncwarp();
#pragma unroll
    for (int t = 0; t < 16; t++) {
        const int p = lane + 32 * t;
        re[t] = xr_s[p + (p >> 5)];
        im[t] = xi_s[p + (p >> 5)];
    }
    __syncwarp();
    // ---- halves 32..256 inside the lane: position lane + 32t pairs with t + h / 32;
    // twiddle ((lane + 32t) % h) * 256 / h
#pragma unroll
    for (int h = 32; h <= 256; h <<= 1) {
        const int hs = h / 32;
#pragma unroll
        for (int t = 0; t < 16; t++) {
            if (t & hs) continue;
            const int ix = twb_offset(h) + lane + 32 * (t & (hs - 1));  // twiddle (lane + 32u) * 256 / h
            butterfly(re[t], im[t], re[t + hs], im[t + hs], twb_re[ix], twb_im[ix]);
        }
    }
    // ---- power of bins 0..256 into shared memory (bin lane + 32t)
    float* pw = xr_s;
#pragma unroll
    for (int t = 0; t < 8; t++) pw[lane + 32 * t] = __fadd_rn(__fmul_rn(re[t], re[t]), __fmul_rn(im[t], im[t]));
    if (lane == 0) pw[256] = __fadd_rn(__fmul_rn(re[8], re[8]), __fmul_rn(im[8], im[8]));
    __syncwarp();
    // ---- filterbank (sequential over each filter's support, bins ascending) and log
    const long long orow = (sg.out_row0 + (f - sg.f_begin)) * 128;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int m = lane + 32 * q;
        const int lo = __ldg(tab.filt_lo + m), w = __ldg(tab.filt_w + m);
        float acc = 0.0f;
        for (int i = 0; i < tab.group_w[q]; i++) {  // the group's widest filter; lanes past their own skip
            const float prod = __fmul_rn(fb_s[i * 128 + m], pw[min(lo + i, NBINS - 1)]);
            if (i < w) acc = __fadd_rn(acc, prod);
        }
        const float v = (float)log((double)__fadd_rn(acc, 5.9604645e-8f));
        const long long o = orow + m;
        if (mel.h) {
            uint32_t hw, lw;
            split2x2(v, 0.0f, mel.scale, hw, lw);
            static_cast<uint16_t*>(mel.h)[o] = (uint16_t)(hw & 0xffffu);
            static_cast<uint16_t*>(mel.l)[o] = (uint16_t)(lw & 0xffffu);
        }
        if (mel_plain) mel_plain[o] = v;
    }
}

// Four elements per thread (n % 4 == 0, 16-byte aligned arrays).
__global__ void split_kernel(const float* __restrict__ x, long long n4, SplitOut out) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const float4 t = reinterpret_cast<const float4*>(x)[i];
        const float y[4] = {t.x, t.y, t.z, t.w};
        uint2 hw, lw;
        split2x4(y, out.scale, hw, lw);
        reinterpret_cast<uint2*>(out.h)[i] = hw;
        reinterpret_cast<uint2*>(out.l)[i] = lw;
    }
}

// max |x| (as its bit pattern: non-negative floats order like their bits; NaN above
// +inf) over n4 float4s into *d_max.
__global__ void absmax_kernel(const float* __restrict__ x, long long n4, unsigned* __restrict__ d_max) {
    unsigned m = 0;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const float4 t = reinterpret_cast<const float4*>(x)[i];
        m = max(m, max(max(__float_as_uint(t.x) & 0x7fffffffu, __float_as_uint(t.y) & 0x7fffffffu),
                       max(__float_as_uint(t.z) & 0x7fffffffu, __float_as_uint(t.w) & 0x7fffffffu)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(d_max, m);
}

// Kernel-level attention operands: RoPE'd Q and K, and V transposed, each as the fp16
// split (h, l) of the values times the operand's scale.
__device__ __forceinline__ void split16(float x, float s, uint16_t& h, uint16_t& l) {
    uint32_t hw, lw;
    split2x2(x, 0.0f, s, hw, lw);
    h = (uint16_t)(hw & 0xffffu);
    l = (uint16_t)(lw & 0xffffu);
}
__global__ void pack_attn_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                 const float* __restrict__ v, long long seq, int heads, int hd,
                                 const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                 uint16_t* __restrict__ q_h, uint16_t* __restrict__ q_l, uint16_t* __restrict__ k_h,
                                 uint16_t* __restrict__ k_l, uint16_t* __restrict__ vt_h, uint16_t* __restrict__ vt_l,
                                 long long vt_ld, float sq, float sk, float sv) {
    const int half = hd / 2;
    const long long W = (long long)heads * hd;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < seq * W;
         e += (long long)gridDim.x * blockDim.x) {
        const long long r = e / W;
        const int c = (int)(e % W), d = c % hd;
        float qo = q[e], ko = k[e];
        if (cos_t) {
            const float* cs = cos_t + r * hd;
            const float* sn = sin_t + r * hd;
            const long long pe = d < half ? e + half : e - half;
            if (d < half) {
                qo = __fsub_rn(__fmul_rn(q[e], cs[d]), __fmul_rn(q[pe], sn[d]));
                ko = __fsub_rn(__fmul_rn(k[e], cs[d]), __fmul_rn(k[pe], sn[d]));
            } else {
                qo = __fadd_rn(__fmul_rn(q[e], cs[d]), __fmul_rn(q[pe], sn[d]));
                ko = __fadd_rn(__fmul_rn(k[e], cs[d]), __fmul_rn(k[pe], sn[d]));
            }
        }
        split16(qo, sq, q_h[e], q_l[e]);
        split16(ko, sk, k_h[e], k_l[e]);
        split16(v[e], sv, vt_h[(long long)c * vt_ld + r], vt_l[(long long)c * vt_ld + r]);
    }
}

// Synthetic operands for the probe benchmarks: x[i] = scale * (sum of 4 uniforms in
// [-1, 1) from a hash of (seed, i)), roughly N(0, scale^2 * 4/3).
__global__ void fill_random_kernel(float* __restrict__ p, long long n, uint32_t seed, float scale) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        uint32_t h = (uint32_t)i * 2654435761u ^ (uint32_t)(i >> 32) * 40503u ^ seed * 2246822519u;
        float acc = 0.0f;
        for (int k = 0; k < 4; k++) {
            h ^= h >> 15;
            h *= 0x2c1b3c6du;
            h ^= h >> 12;
            h *= 0x297a2d39u;
            h ^= h >> 15;
            acc += (float)(h >> 8) * (1.0f / 8388608.0f) - 1.0f;
        }
        p[i] = acc * scale;
    }
}

// Self-test of the bounded waits (failure detection without a fault): one warp
// allocates TMEM as the tensor-core kernels do, arms an mbarrier for a 1 KB transfer
// that is never issued -- a flag nothing sets -- and waits on it with the production
// wait, limited to limit_ns.  The wait gives up, records DEV_TIMEOUT_PROBE in *err
// like any expired wait, the warp frees its TMEM and the kernel returns, leaving the
// context usable.  waited[0] receives the wait's duration in ns (globaltimer).
__global__ void __launch_bounds__(32) wait_probe_kernel(int* __restrict__ err, unsigned long long limit_ns,
                                                        unsigned long long* __restrict__ waited) {
    __shared__ uint64_t bar;
    __shared__ uint32_t tmem_slot;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
    }
    __syncwarp();
    tmem_alloc(&tmem_slot, 32);
    tc_fence_after();
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar, 1024);  // the phase completes only when 1 KB arrives: never
        const uint64_t t0 = globaltimer_ns();
        const bool ok = mbar_wait(&bar, 0, err, DEV_TIMEOUT_PROBE, limit_ns);
        *waited = ok ? 0ull : globaltimer_ns() - t0;
    }
    tc_fence_before();
    __syncwarp();
    tmem_dealloc(tmem_slot, 32);
}

}  // namespace

void launch_pack_attn(cudaStream_t s, const float* q, const float* k, const float* v, long long seq, int heads,
                      int hd, const float* cos_t, const float* sin_t, const AttnOperands& op) {
    using u16 = uint16_t;
    const long long n = seq * heads * hd;
    if (n <= 0) return;
    const long long blocks = std::min<long long>((n + 255) / 256, 148LL * 16);
    pack_attn_kernel<<<(unsigned)blocks, 256, 0, s>>>(q, k, v, seq, heads, hd, cos_t, sin_t, (u16*)op.q_h, (u16*)op.q_l,
                                                      (u16*)op.k_h, (u16*)op.k_l, (u16*)op.vt_h, (u16*)op.vt_l,
                                                      op.vt_ld, op.q_scale, op.k_scale, op.v_scale);
    N3D_CUDA(cudaGetLastError());
}

void launch_split(cudaStream_t s, const float* x, long long n, SplitOut out) {
    if (n <= 0) return;
    if (n % 4) throw Error(13, "split: the element count must be a multiple of 4");
    const long long n4 = n / 4;
    const long long blocks = std::min<long long>((n4 + 255) / 256, 148LL * 16);
    split_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, n4, out);
    N3D_CUDA(cudaGetLastError());
}

void launch_absmax(cudaStream_t s, const float* x, long long n, float* d_max) {
    if (n <= 0) return;
    if (n % 4) throw Error(13, "absmax: the element count must be a multiple of 4");
    const long long n4 = n / 4;
    const long long blocks = std::min<long long>((n4 + 255) / 256, 148LL * 8);
    absmax_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, n4, reinterpret_cast<unsigned*>(d_max));
    N3D_CUDA(cudaGetLastError());
}

void launch_layer_norm(cudaStream_t s, const float* x, long long rows, int cols, const float* w, const float* b,
                       SplitOut out) {
    if (rows <= 0) return;
    // two rows per warp at 512 columns (72 registers), one at 1024 (where two rows would
    // need 120 registers and halve the resident warps)
    const int warps = 8, rpw = cols == 512 ? 2 : 1;
    const unsigned grid = (unsigned)((rows + warps * rpw - 1) / (warps * rpw));
    if (cols == 512)
        launch_pdl(layer_norm_kernel<16, 2>, dim3(grid), dim3(warps * 32), 0, s, x, rows, w, b, out);
    else if (cols == 1024)
        launch_pdl(layer_norm_kernel<32, 1>, dim3(grid), dim3(warps * 32), 0, s, x, rows, w, b, out);
    else
        throw Error(13, "layer_norm supports 512 or 1024 columns");
    N3D_CUDA(cudaGetLastError());
}

void launch_mel(cudaStream_t s, const float* audio, const MelSegDev* segs, int nsegs, long long f_first,
                long long n_frames, int hop, const MelTables& tab, float preemph, SplitOut mel, float* mel_plain) {
    if (n_frames <= 0 || nsegs <= 0) return;
    if (tab.fb_w < 0 || tab.fb_w > MEL_FB_MAX_W) throw Error(13, "log-mel: a filter wider than the kernel's table");
    static std::atomic<unsigned long long> attr{0};
    once_per_device(attr, [] {
        N3D_CUDA(cudaFuncSetAttribute(mel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      MEL_FB_MAX_W * 128 * (int)sizeof(float)));
    });
    const long long blocks = (n_frames + MEL_WARPS - 1) / MEL_WARPS;
    mel_kernel<<<(unsigned)blocks, MEL_WARPS * 32, tab.fb_w * 128 * sizeof(float), s>>>(
        audio, segs, nsegs, f_first, n_frames, hop, tab, preemph, mel, mel_plain);
    N3D_CUDA(cudaGetLastError());
}

void launch_fill_random(cudaStream_t s, float* p, long long n, uint32_t seed, float scale) {
    if (n <= 0) return;
    const long long blocks = std::min<long long>((n + 255) / 256, 148LL * 16);
    fill_random_kernel<<<(unsigned)blocks, 256, 0, s>>>(p, n, seed, scale);
    N3D_CUDA(cudaGetLastError());
}

void launch_wait_probe(cudaStream_t s, int* err, unsigned long long limit_ns, unsigned long long* waited) {
    wait_probe_kernel<<<1, 32, 0, s>>>(err, limit_ns, waited);
    N3D_CUDA(cudaGetLastError());
}

}  // namespace n3d
