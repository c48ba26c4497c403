// C[M, N] = A[M, K] * B[N, K]^T on the sm_100a tensor cores (tcgen05) with fused
// epilogues.
//
// Replaces the reference's WGSL `gemm` pipeline (src/gpu.rs:1005-1611, wrapper
// src/gpu.rs:726-744) and the separate `add`, `unary` (GELU/ReLU), `rope` and
// `col3` dispatches that followed it (src/gpu.rs:1768-1838, 1973-1999): those
// become epilogue modes of this one kernel.  The reference arithmetic it must
// agree with is `tensor::linear` (src/tensor.rs:22-57) in fp32.
//
// Arithmetic (fp16 split): every operand x is stored as two fp16 arrays of x s (s a
// power of two per tensor): h = RN-fp16(x s), l = RN-fp16(x s - h).  Each k-step issues
// h·h, h·l and l·h on `kind::f16`, all into one fp32 TMEM accumulator, and the epilogue
// multiplies by 1 / (s_A s_B).  fp16's 11 significant bits make h + l good to ~2^-22,
// as accurate as 3xTF32, while all three products run at the 16-bit tensor rate and an
// operand costs 4 bytes per element.
//
// k-block = 64: per CTA and stage, A rows as [h: 128 B | l: 128 B] and the same for B,
// TMA-loaded with the 128-byte swizzle.  A K that is an odd multiple of 32 ends with a
// half block whose upper columns the TMA fills with zeros.
// Two kernels:
//   gemm_kernel<BN>        one CTA per 128 x BN tile, persistent (N = 192 head GEMMs,
//                          small M, the allocation-free entry point)
//   gemm_pair_kernel<BN, EW> CTA pairs on 256 x 256 tiles with M = 256
//                          `cta_group::2` MMAs: each CTA loads its 128 A rows and half
//                          the B tile, the leader issues, both own 128 accumulator rows;
//                          EW = 4 or 8 epilogue warps (8: two per lane quadrant, each
//                          storing half of the tile's columns)
// Both: warp 0 TMA, warp 1 TMEM owner + MMA issue, epilogue warps 2.. (TMEM lane
// quadrant = warp % 4); two TMEM accumulators so tile i's epilogue overlaps tile
// i + 1's main loop.  Every wait is bounded; an expired wait records its site.

#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <map>
#include <mutex>
#include <tuple>

#include "n3d_device.cuh"
#include "n3d_internal.h"

namespace n3d {

namespace {

constexpr int BM = 128;                 // rows per CTA
constexpr int BK = 64;                  // k-block (fp16 elements)
constexpr int ROW = BK * 2;             // bytes per row of one fp16 array (128: SW128)
constexpr int ROW_2 = 2 * ROW;          // both arrays of one row

// ------------------------------------------------------------------- GELU
// GELU(x) = 0.5 x (1 + erf(x/√2)) (src/tensor.rs:113-120), branch-free.
// h = Φ(-|x|) = erfc(|x|/√2)/2 is evaluated as t · 2^(Q(t) - x² log2(e)/2) with
// t = 1/(1 + C1 |x|): the Chebyshev-fitted erfc form of Numerical Recipes (§6.2) with
// coefficients fitted for this kernel by fit_gelu.py (relative error of erfc 2.3e-8 on
// [0, 6.5], ~1 ulp of the result in fp32 on average).  Φ(x) = 1/2 + copysign(1/2 - h, x)
// rounds like the reference's 1 + erf (cancellation included).  A library erff has two
// code paths per element, which diverge within a warp.
constexpr float GELU_C1 = 0.265165031f;   // 0.375 / √2
constexpr float GELU_KX = -0.721347511f;  // -log2(e) / 2
__host__ __device__ constexpr float gelu_q(int i) {  // Q(t) = sum gelu_q(i) t^i
    return i == 0 ? -3.24179554f : i == 1 ? 1.46152258f : i == 2 ? 0.468700767f : i == 3 ? 0.961769581f
         : i == 4 ? -1.82942355f : i == 5 ? 3.28494f : i == 6 ? -3.62900352f : i == 7 ? 1.90515316f
         : -0.381863475f;
}

__device__ __forceinline__ float copysign_bits(float mag, float sgn) {
    return __uint_as_float((__float_as_uint(mag) & 0x7fffffffu) | (__float_as_uint(sgn) & 0x80000000u));
}

// Two GELUs with packed arithmetic.
__device__ __forceinline__ void gelu2(float& a, float& b) {
    const float ta = rcp_approx(__fmaf_rn(GELU_C1, fabsf(a), 1.0f));
    const float tb = rcp_approx(__fmaf_rn(GELU_C1, fabsf(b), 1.0f));
    const uint64_t t = pack2(ta, tb), x = pack2(a, b);
    uint64_t q = fma2(t, pack2(gelu_q(8), gelu_q(8)), pack2(gelu_q(7), gelu_q(7)));
#pragma unroll
    for (int i = 6; i >= 0; i--) q = fma2(q, t, pack2(gelu_q(i), gelu_q(i)));
    const uint64_t y = fma2(mul2(x, pack2(GELU_KX, GELU_KX)), x, q);
    float ya, yb;
    unpack2(y, ya, yb);
    const uint64_t h = mul2(t, pack2(ex2_approx(ya), ex2_approx(yb)));
    float da, db;  // 1/2 - h
    unpack2(fma2(h, pack2(-1.0f, -1.0f), pack2(0.5f, 0.5f)), da, db);
    const uint64_t phi = add2(pack2(0.5f, 0.5f), pack2(copysign_bits(da, a), copysign_bits(db, b)));
    unpack2(mul2(x, phi), a, b);
}

// The same arithmetic for one value (identical results to a half of gelu2).
__device__ __forceinline__ float gelu1(float x) {
    const float t = rcp_approx(__fmaf_rn(GELU_C1, fabsf(x), 1.0f));
    float q = __fmaf_rn(t, gelu_q(8), gelu_q(7));
#pragma unroll
    for (int i = 6; i >= 0; i--) q = __fmaf_rn(q, t, gelu_q(i));
    const float y = __fmaf_rn(__fmul_rn(x, GELU_KX), x, q);
    const float h = __fmul_rn(t, ex2_approx(y));
    const float d = __fmaf_rn(h, -1.0f, 0.5f);
    return __fmul_rn(x, __fadd_rn(0.5f, copysign_bits(d, x)));
}

// Store 32 consecutive fp32 values of one output row.
__device__ __forceinline__ void store_row32(float* dst, const float* v, int ncols_left) {
    if (ncols_left >= 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (i < ncols_left) dst[i] = v[i];
    }
}
// 32 16-bit values of one row (16 packed words).
__device__ __forceinline__ void store_row32_16(uint16_t* dst, const uint32_t* w, int ncols_left) {
    if (ncols_left >= 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
        for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<uint4*>(dst + 2 * i) = make_uint4(w[i], w[i + 1], w[i + 2], w[i + 3]);
    } else {
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (i < ncols_left) dst[i] = (uint16_t)(w[i / 2] >> (16 * (i & 1)));
    }
}

// Epilogue value of accumulator column i: operand scales undone, bias, activation.
__device__ __forceinline__ float epi_value(int mode, float acc, float scale, float bias) {
    float x = __fadd_rn(__fmul_rn(acc, scale), bias);
    if (mode == EPI_GELU_SPLIT) x = gelu1(x);
    if (mode == EPI_RELU_SPLIT) x = fmaxf(x, 0.0f);
    return x;
}

// 32 bias values for columns col0.. (zeros past N or without bias).
__device__ __forceinline__ void load_bias32(const float* bias, int col0, int N, float* b) {
    if (bias != nullptr && col0 + 32 <= N) {
#pragma unroll
        for (int i4 = 0; i4 < 8; i4++) {
            const float4 b4 = __ldg(reinterpret_cast<const float4*>(bias + col0) + i4);
            b[4 * i4] = b4.x;
            b[4 * i4 + 1] = b4.y;
            b[4 * i4 + 2] = b4.z;
            b[4 * i4 + 3] = b4.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; i++) b[i] = (bias != nullptr && col0 + i < N) ? bias[col0 + i] : 0.0f;
    }
}

// ------------------------------------------------------ direct-store epilogue
// For the modes with a row remap (head proj into its padded layout), the fused
// dense + out_proj, and plain stores without a tensor map.  Tile rows
// r = m0 + 32 q + lane.
// `w2s` (EPI_DENSE_OUT): w2 [n2, N] and the dense bias [N] staged in shared memory.
template <int BN>
__device__ __forceinline__ void epilogue_tile(const Epi& epi, uint32_t tl, int m0, int n0, int M, int N, int q,
                                              int lane, const float* w2s = nullptr, int ncols = BN) {
    const int r = m0 + q * 32 + lane;
    const bool row_ok = r < M;
    const int qq = r / epi.rdiv, t = r - qq * epi.rdiv;
    const bool keep = row_ok && t < epi.rkeep;
    const long long orow = (long long)qq * epi.rmul + t + epi.roff;
    const bool zero_row = epi.seq_len != nullptr && keep && t >= epi.seq_len[qq];
    if (epi.mode == EPI_DENSE_OUT) {
        // relu(dense) then the out projection, sequential over the hidden
        // index with separate multiply and add (src/tensor.rs:33-43)
        float acc[8];
#pragma unroll
        for (int o = 0; o < 8; o++) acc[o] = 0.0f;
        const float* bs = w2s + 8 * N;  // N = 192 = BN: one column tile
        for (int c = 0; c < BN; c += 32) {
            float v[32];
            tmem_ld32(tl + c, v);
            if (!keep) continue;
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const int col = n0 + c + i;
                const float rr = fmaxf(__fadd_rn(__fmul_rn(v[i], epi.acc_scale), bs[col]), 0.0f);
#pragma unroll
                for (int o = 0; o < 8; o++) acc[o] = __fadd_rn(acc[o], __fmul_rn(rr, w2s[o * N + col]));
            }
        }
        if (keep)
            for (int o = 0; o < epi.n2; o++) epi.out[orow * epi.ldo + o] = __fadd_rn(acc[o], epi.b2[o]);
        return;
    }
    for (int c = 0; c < ncols; c += 32) {
        float v[32];
        tmem_ld32(tl + c, v);
        const int col0 = n0 + c;
        if (!keep || col0 >= N) continue;
        float bias[32];
        load_bias32(epi.bias, col0, N, bias);
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = zero_row ? 0.0f : epi_value(epi.mode, v[i], epi.acc_scale, bias[i]);
        const int left = N - col0;
        if (epi.mode == EPI_STORE) {
            store_row32(epi.out + orow * epi.ldo + col0, v, left);
        } else {  // fp16 split of the output
            uint32_t hw[16], lw[16];
#pragma unroll
            for (int i = 0; i < 16; i++) split2x2(v[2 * i], v[2 * i + 1], epi.out_scale, hw[i], lw[i]);
            store_row32_16(static_cast<uint16_t*>(epi.out_h) + orow * epi.ldo + col0, hw, left);
            store_row32_16(static_cast<uint16_t*>(epi.out_l) + orow * epi.ldo + col0, lw, left);
        }
    }
}

// ------------------------------------------------------- TMA-store epilogue
// Element-wise add of the box into global memory (the L2 performs the read-modify-write).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map),
                 "r"(x), "r"(y), "r"(smem_u32(src))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// One warp's 32 x 32 fp32 block into a 4 KB 128-byte-swizzled staging box: lane = box row.
__device__ __forceinline__ void stage_rows(uint8_t* box, int lane, const float* v) {
#pragma unroll
    for (int i = 0; i < 8; i++)
        *reinterpret_cast<float4*>(box + lane * 128 + ((i ^ (lane & 7)) << 4)) =
            make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}
// 32 x 32 16-bit values (16 packed words per lane) into a 2 KB 64-byte-swizzled box.
__device__ __forceinline__ void stage_rows_16(uint8_t* box, int lane, const uint32_t* w) {
#pragma unroll
    for (int i = 0; i < 4; i++)
        *reinterpret_cast<uint4*>(box + lane * 64 + ((i ^ ((lane >> 1) & 3)) << 4)) =
            make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}
// The staging area is double-buffered: consecutive store groups of a warp alternate
// between its two halves, so before a half is overwritten only the group before the
// latest -- the last one that used this half -- must have finished reading it.
template <bool DB = true>
__device__ __forceinline__ void stage_begin(int lane) {
    if (lane == 0) {
        if (DB)
            bulk_wait_read1();
        else  // one 4 KB area: every earlier group must have read it
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    }
    __syncwarp();
}
// Make the staged boxes visible to the TMA unit and store them (up to three maps);
// `add0`: the first box is added into its destination instead of stored.
__device__ __forceinline__ void stage_issue(int lane, const CUtensorMap* m0, const void* b0, const CUtensorMap* m1,
                                            const void* b1, const CUtensorMap* m2, const void* b2, int x, int y,
                                            bool add0 = false) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
        if (add0)
            tma_reduce_add_2d(m0, b0, x, y);
        else
            tma_store_2d(m0, b0, x, y);
        if (m1) tma_store_2d(m1, b1, x, y);
        if (m2) tma_store_2d(m2, b2, x, y);
        bulk_commit();
    }
}

// Epilogue with TMA stores, for modes whose output rows are the tile's rows:
// EPI_STORE, EPI_SPLIT, EPI_GELU_SPLIT, EPI_RELU_SPLIT, EPI_QKV_ATTN, over accumulator
// columns [c_begin, c_end).  `stg` is this warp's 8 KB staging area, two 4 KB halves
// that consecutive store groups alternate between (`sbuf` counts the warp's groups
// across tiles).
template <int BN, bool DB = true>
__device__ __forceinline__ void epilogue_tile_tma(const Epi& epi, uint32_t tl, int m0, int n0, int M, int N, int q,
                                                  int lane, uint8_t* stg, uint32_t& sbuf, int c_begin = 0,
                                                  int c_end = BN) {
    const int mode = epi.mode;
    const int rowbase = m0 + q * 32;
    if (rowbase >= M) return;  // whole warp past the end: nothing to load or store
    const int r = rowbase + lane;
    if (mode == EPI_QKV_ATTN) {
        uint8_t* bhi = stg;
        uint8_t* blo = DB ? stg + 4096 : stg;
        for (int c = c_begin; c < c_end; c += 64) {
            float v[64];
            tmem_ld32(tl + c, v);
            tmem_ld32(tl + c + 32, v + 32);
            const int col0 = n0 + c;
            if (col0 >= N) break;
#pragma unroll
            for (int i = 0; i < 64; i += 2) unpack2(mul2(pack2(v[i], v[i + 1]), pack2(epi.acc_scale, epi.acc_scale)), v[i], v[i + 1]);
            const int sec = col0 / epi.q_cols, hcol = col0 - sec * epi.q_cols;
            if (sec < 2) {
                // rotate-half RoPE (src/encoder.rs:281-296); the tables repeat their first
                // half (cat(freqs, freqs)), so one float4 of cos and of sin serves four pairs
                const int pos = r % epi.rope_seq;
                const float4* cs = reinterpret_cast<const float4*>(epi.cos_t + (long long)pos * epi.head_dim);
                const float4* sn = reinterpret_cast<const float4*>(epi.sin_t + (long long)pos * epi.head_dim);
#pragma unroll
                for (int i4 = 0; i4 < 8; i4++) {
                    const float4 c4 = __ldg(cs + i4), s4 = __ldg(sn + i4);
                    const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int i = 4 * i4 + j;
                        const float x1 = v[i], x2 = v[32 + i];
                        v[i] = __fsub_rn(__fmul_rn(x1, cc[j]), __fmul_rn(x2, ss[j]));
                        v[32 + i] = __fadd_rn(__fmul_rn(x2, cc[j]), __fmul_rn(x1, ss[j]));
                    }
                }
            }
            // fp16 splits with the section's scale: Q / K rows (64 values = one 128-byte
            // swizzled box row), V transposed (box row = d, 32 rows of the tile = 64
            // bytes, unswizzled)
            const float sc = epi.sec_scale[sec < 3 ? sec : 2];
            uint32_t hi[32], lo[32];
#pragma unroll
            for (int i = 0; i < 32; i++) split2x2(v[2 * i], v[2 * i + 1], sc, hi[i], lo[i]);
            // h goes out from the first half, then l from the second, each as its own group
            if (sec < 2) {
                stage_begin<DB>(lane);
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int o = lane * 128 + ((i ^ (lane & 7)) << 4);
                    *reinterpret_cast<uint4*>(bhi + o) = make_uint4(hi[4 * i], hi[4 * i + 1], hi[4 * i + 2], hi[4 * i + 3]);
                }
                stage_issue(lane, sec == 0 ? &epi.map_h : &epi.map_k_h, bhi, nullptr, nullptr, nullptr, nullptr, hcol,
                            rowbase);
                stage_begin<DB>(lane);
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int o = lane * 128 + ((i ^ (lane & 7)) << 4);
                    *reinterpret_cast<uint4*>(blo + o) = make_uint4(lo[4 * i], lo[4 * i + 1], lo[4 * i + 2], lo[4 * i + 3]);
                }
                stage_issue(lane, sec == 0 ? &epi.map_l : &epi.map_k_l, blo, nullptr, nullptr, nullptr, nullptr, hcol,
                            rowbase);
            } else {
                // transpose by lane pairs: word i of lane L holds d = 2i, 2i + 1 of token L;
                // an even lane stores row 2i for tokens L, L + 1 and an odd lane row 2i + 1
                // for tokens L - 1, L, one 32-bit store each (rows 2i and 2i + 1 fall in
                // disjoint banks)
                const bool odd = lane & 1;
                const int tok = (lane & ~1) * 2;
                stage_begin<DB>(lane);
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const uint32_t ph = __shfl_xor_sync(0xffffffffu, hi[i], 1);
                    const int row = (2 * i + (odd ? 1 : 0)) * 64 + tok;
                    *reinterpret_cast<uint32_t*>(bhi + row) = odd ? __byte_perm(ph, hi[i], 0x7632) : __byte_perm(hi[i], ph, 0x5410);
                }
                stage_issue(lane, &epi.map_vt_h, bhi, nullptr, nullptr, nullptr, nullptr, rowbase, hcol);
                stage_begin<DB>(lane);
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const uint32_t pl = __shfl_xor_sync(0xffffffffu, lo[i], 1);
                    const int row = (2 * i + (odd ? 1 : 0)) * 64 + tok;
                    *reinterpret_cast<uint32_t*>(blo + row) = odd ? __byte_perm(pl, lo[i], 0x7632) : __byte_perm(lo[i], pl, 0x5410);
                }
                stage_issue(lane, &epi.map_vt_l, blo, nullptr, nullptr, nullptr, nullptr, rowbase, hcol);
            }
        }
        return;
    }
    const bool split = mode != EPI_STORE;
    const uint64_t sc2 = pack2(epi.acc_scale, epi.acc_scale);
    for (int c = c_begin; c < c_end; c += 32) {
        float v[32];
        tmem_ld32(tl + c, v);
        const int col0 = n0 + c;
        if (col0 >= N) break;
        float bias[32];
        load_bias32(epi.bias, col0, N, bias);
        if (mode == EPI_GELU_SPLIT) {
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
                unpack2(fma2(pack2(v[i], v[i + 1]), sc2, pack2(bias[i], bias[i + 1])), v[i], v[i + 1]);
                gelu2(v[i], v[i + 1]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = epi_value(mode, v[i], epi.acc_scale, bias[i]);
        }
        uint8_t* half = DB ? stg + (sbuf++ & 1u) * 4096 : stg;
        uint8_t* bst = half;         // 4 KB fp32 box (EPI_STORE)
        uint8_t* bh = half;          // 2 KB fp16 box (split modes)
        uint8_t* bl = half + 2048;   // 2 KB fp16 box
        stage_begin<DB>(lane);
        if (split) {
            uint32_t hw[16], lw[16];
#pragma unroll
            for (int i = 0; i < 16; i++) split2x2(v[2 * i], v[2 * i + 1], epi.out_scale, hw[i], lw[i]);
            stage_rows_16(bh, lane, hw);
            stage_rows_16(bl, lane, lw);
            stage_issue(lane, &epi.map_h, bh, &epi.map_l, bl, nullptr, nullptr, col0, rowbase);
        } else {
            stage_rows(bst, lane, v);
            stage_issue(lane, &epi.map_out, bst, nullptr, nullptr, nullptr, nullptr, col0, rowbase, epi.reduce != 0);
        }
    }
}

// ------------------------------------------------------------- main loops
// Shared-memory stage of one CTA: [A: h | l][B: h | l] with `ra` and `rb` rows of
// 128 bytes.  MMAs of one k-block (4 steps of 16) into accumulator `d`.
template <bool PAIR>
__device__ __forceinline__ void mma_kblock(uint32_t d, uint32_t st, int ra, int rb, uint32_t idesc, bool first) {
    const uint32_t ah = st, al = ah + ra * ROW, bh = al + ra * ROW, bl = bh + rb * ROW;
#pragma unroll
    for (int k = 0; k < BK / 16; k++) {  // 16 fp16 = 32 bytes along the 128-byte rows
        const uint64_t a_h = desc_k_sw128(ah + 32 * k), a_l = desc_k_sw128(al + 32 * k);
        const uint64_t b_h = desc_k_sw128(bh + 32 * k), b_l = desc_k_sw128(bl + 32 * k);
        if (PAIR) {
            umma_f16_pair(d, a_h, b_h, idesc, !(first && k == 0));
            umma_f16_pair(d, a_h, b_l, idesc, 1);
            umma_f16_pair(d, a_l, b_h, idesc, 1);
        } else {
            umma_f16(d, a_h, b_h, idesc, !(first && k == 0));
            umma_f16(d, a_h, b_l, idesc, 1);
            umma_f16(d, a_l, b_h, idesc, 1);
        }
    }
}

// TMA loads of one stage: rows [ya, ya + ra) of A at column xa and [yb, yb + rb) of B
// at column xb, completion on `bar` (pair: the leader's barrier, `bar_cluster`).
template <bool PAIR>
__device__ __forceinline__ void load_stage(uint8_t* st, int ra, int rb, const CUtensorMap* m, uint64_t* bar,
                                           uint32_t bar_cluster, int xa, int ya, int xb, int yb) {
    uint8_t* p[4] = {st, st + ra * ROW, st + ra * ROW_2, st + ra * ROW_2 + rb * ROW};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int x = i < 2 ? xa : xb, y = i < 2 ? ya : yb;
        if (PAIR)
            tma_load_2d_pair(p[i], &m[i], bar_cluster, x, y);
        else
            tma_load_2d(p[i], &m[i], bar, x, y);
    }
}

struct Maps4 {
    CUtensorMap m[4];  // A h, l; B h, l
};

// ------------------------------------------------------------ one-CTA kernel
template <int BN>
struct GemmCfg {
    static constexpr int STAGE_BYTES = (BM + BN) * ROW_2;
    static constexpr int STAGING = 4 * 8192;
    static constexpr int STAGES_FIT = (232448 - STAGING - 2048) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 6 ? 6 : STAGES_FIT;
    static constexpr int ACC_COLS = BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
    static constexpr int TMEM_COLS = 2 * ACC_COLS;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 1024 + STAGING;
    static_assert(STAGES >= 2, "need two pipeline stages");
};

template <int BN>
__global__ void __launch_bounds__(192, 1)
    gemm_kernel(const __grid_constant__ Maps4 maps, int M, int N, int K, int kb_per_tap,
                const __grid_constant__ Epi epi, int* err, int ksplit, int Mp) {
    using Cfg = GemmCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty = full + Cfg::STAGES;
    uint64_t* acc_full = empty + Cfg::STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_n = (N + BN - 1) / BN;
    // tile t = (output tile, k split): split ks covers k-blocks [ks nkb / ksplit,
    // (ks + 1) nkb / ksplit) and stores its partial tile at row offset ks * Mp
    const int tiles = ((M + BM - 1) / BM) * tiles_n * ksplit;
    const int nkb = (K + BK - 1) / BK;

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < Cfg::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        mbar_fence_init();
        for (int i = 0; i < 4; i++) tma_prefetch_desc(&maps.m[i]);
    }
    if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    griddep_wait();  // operands written by the previous kernel
    griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
                const int tmn = t / ksplit, ks = t - tmn * ksplit;
                const int m0 = (tmn / tiles_n) * BM, n0 = (tmn % tiles_n) * BN;
                for (int kb = ks * nkb / ksplit; kb < (ks + 1) * nkb / ksplit; kb++, g++) {
                    const int s = g % Cfg::STAGES;
                    if (g >= (uint32_t)Cfg::STAGES &&
                        !mbar_wait(&empty[s], ((g / Cfg::STAGES) - 1) & 1, err, DEV_TIMEOUT_TMA_EMPTY)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
                    const int tap = kb_per_tap > 0 ? kb / kb_per_tap : 0;
                    const int ka = kb_per_tap > 0 ? (kb % kb_per_tap) * BK : kb * BK;
                    load_stage<false>(smem + s * Cfg::STAGE_BYTES, BM, BN, maps.m, &full[s], 0, ka, m0 + tap, kb * BK,
                                      n0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(BN);
            uint32_t g = 0;
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, it++) {
                const int buf = it & 1;
                if (it >= 2 && !mbar_wait(&acc_empty[buf], ((it >> 1) - 1) & 1, err, DEV_TIMEOUT_ACC)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * Cfg::ACC_COLS;
                const int ks = t % ksplit, kb0 = ks * nkb / ksplit;
                for (int kb = kb0; kb < (ks + 1) * nkb / ksplit; kb++, g++) {
                    const int s = g % Cfg::STAGES;
                    if (!mbar_wait(&full[s], (g / Cfg::STAGES) & 1, err, DEV_TIMEOUT_TMA_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    mma_kblock<false>(d, smem_u32(smem + s * Cfg::STAGE_BYTES), BM, BN, idesc, kb == kb0);
                    umma_commit(&empty[s]);
                }
                if (ok) umma_commit(&acc_full[buf]);
            }
        }
    } else {
        const int q = warp & 3;
        float* w2s = reinterpret_cast<float*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES + 1024);
        if (epi.mode == EPI_DENSE_OUT) {
            // the out_proj weights [8, N] (rows past n2 zero) and the dense bias [N], once
            // per CTA into the staging area, which direct-store epilogues do not use
            for (int i = threadIdx.x - 64; i < 9 * N; i += 128)
                w2s[i] = i < 8 * N ? (i / N < epi.n2 ? epi.w2[i] : 0.0f) : epi.bias[i - 8 * N];
            asm volatile("bar.sync 1, 128;" ::: "memory");  // the 4 epilogue warps
        }
        int it = 0;
        uint32_t sbuf = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, it++) {
            const int buf = it & 1;
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (it >> 1) & 1, err, DEV_TIMEOUT_ACC));
            if (!ok) break;
            tc_fence_after();
            const int tmn = t / ksplit, ks = t - tmn * ksplit;
            const int m0 = (tmn / tiles_n) * BM, n0 = (tmn % tiles_n) * BN;
            const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * Cfg::ACC_COLS;
            if (epi.tma)  // a k split's partial rows start at ks * Mp (rows past M land in padding)
                epilogue_tile_tma<BN>(epi, tl, m0 + ks * Mp, n0, ksplit > 1 ? ksplit * Mp : M, N, q, lane,
                                      smem + Cfg::STAGES * Cfg::STAGE_BYTES + 1024 + (warp - 2) * 8192, sbuf);
            else
                epilogue_tile<BN>(epi, tl, m0, n0, M, N, q, lane, w2s);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
        if (lane == 0) bulk_wait0();
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, Cfg::TMEM_COLS);
}

// ------------------------------------------------------------ CTA-pair kernel
// A cluster of two CTAs walks 256 x BN output tiles.  CTA r of the pair loads A rows
// m0 + 128 r and B rows n0 + r BN / 2, so each SM streams half the B tile of the
// one-CTA kernel for the same work; its TMEM receives output rows m0 + 128 r, which
// its own epilogue warps store.  Barriers: full[s] lives in the leader (both CTAs'
// loads complete on it), empty[s] and acc_full[b] in both (arrived by the leader's
// multicast commits), acc_empty[b] in the leader (the 8 epilogue warps of the pair).
// Tile t of a launch.  The first `full` tiles are 256 x BN in m-major order; the
// tiles of the last, partial wave are each split along N into `split` sub-tiles of
// BN / split columns, so that wave ends sooner (same dot products in the same k
// order, so the results do not depend on the split).
struct PairTile {
    int mt, n0, nw;  // 256-row tile index, first column, width
};
template <int BN>
__device__ __forceinline__ PairTile pair_tile(int t, int tiles_n, int full, int split) {
    if (t < full) return PairTile{t / tiles_n, (t % tiles_n) * BN, BN};
    const int u = t - full, base = full + u / split, nw = BN / split;
    return PairTile{base / tiles_n, (base % tiles_n) * BN + (u % split) * nw, nw};
}

// EW epilogue warps: 4 (one per TMEM lane quadrant, each with a double-buffered 8 KB
// staging area) or 8 (two per quadrant, each storing half of the tile's columns
// through a single 4 KB box, so that three 64 KB stages still fit).  8 suits the
// epilogues with arithmetic per element (GELU, ReLU, plain stores); 4 those whose
// stores dominate (the attention operands' hi/lo pairs, the reduce-adds).
template <int BN, int EW>
struct PairCfg {
    static_assert(EW == 4 || EW == 8, "4 or 8 epilogue warps");
    static constexpr int STAGE_BYTES = (BM + BN / 2) * ROW_2;
    static constexpr int EPI_WARPS = EW;
    static constexpr int STAGE_BOX = EW == 8 ? 4096 : 8192;
    static constexpr int STAGING = EPI_WARPS * STAGE_BOX;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int STAGES_FIT = (232448 - STAGING - 2048) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 6 ? 6 : STAGES_FIT;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 1024 + STAGING;
    static_assert(BN == 128 || BN == 256, "pair tiles are 256 x 128 or 256 x 256");
    static_assert(STAGES >= 2, "need two pipeline stages");
};

template <int BN, int EW>
__global__ void __launch_bounds__(PairCfg<BN, EW>::THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ Maps4 maps, int M, int N, int K, int kb_per_tap,
                     const __grid_constant__ Epi epi, int* err, int full, int split) {
    using Cfg = PairCfg<BN, EW>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty = full_bar + Cfg::STAGES;
    uint64_t* acc_full = empty + Cfg::STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rank = static_cast<int>(cluster_rank());
    const bool leader = rank == 0;
    const int cid = static_cast<int>(cluster_id_x()), ncl = static_cast<int>(cluster_count_x());
    const int tiles_n = (N + BN - 1) / BN;
    const int tiles = full + (((M + 2 * BM - 1) / (2 * BM)) * tiles_n - full) * split;
    const int nkb = (K + BK - 1) / BK;

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < Cfg::STAGES; s++) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 2 * Cfg::EPI_WARPS);
        }
        mbar_fence_init();
        for (int i = 0; i < 4; i++) tma_prefetch_desc(&maps.m[i]);
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrive
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    griddep_wait();  // operands written by the previous kernel
    griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            for (int t = cid; ok && t < tiles; t += ncl) {
                const PairTile tile = pair_tile<BN>(t, tiles_n, full, split);
                // B rows of this CTA: its half of the tile's width (a full BN / 2-row box
                // is loaded; rows past the sub-tile are not read by the MMA)
                const int m0 = tile.mt * 2 * BM + rank * BM, n0 = tile.n0 + rank * (tile.nw / 2);
                for (int kb = 0; kb < nkb; kb++, g++) {
                    const int s = g % Cfg::STAGES;
                    if (g >= (uint32_t)Cfg::STAGES &&
                        !mbar_wait_cluster(&empty[s], ((g / Cfg::STAGES) - 1) & 1, err, DEV_TIMEOUT_TMA_EMPTY)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * Cfg::STAGE_BYTES);
                    const int tap = kb_per_tap > 0 ? kb / kb_per_tap : 0;
                    const int ka = kb_per_tap > 0 ? (kb % kb_per_tap) * BK : kb * BK;
                    load_stage<true>(smem + s * Cfg::STAGE_BYTES, BM, BN / 2, maps.m, nullptr,
                                     leader_addr(&full_bar[s]), ka, m0 + tap, kb * BK, n0);
                }
            }
        }
    } else if (warp == 1) {
        if (leader && lane == 0) {
            uint32_t g = 0;
            int it = 0;
            bool ok = true;
            for (int t = cid; ok && t < tiles; t += ncl, it++) {
                const int nw = pair_tile<BN>(t, tiles_n, full, split).nw;
                const uint32_t idesc = idesc_f16_pair(nw);
                const int buf = it & 1;
                if (it >= 2 && !mbar_wait_cluster(&acc_empty[buf], ((it >> 1) - 1) & 1, err, DEV_TIMEOUT_ACC)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * BN;
                for (int kb = 0; kb < nkb; kb++, g++) {
                    const int s = g % Cfg::STAGES;
                    if (!mbar_wait_cluster(&full_bar[s], (g / Cfg::STAGES) & 1, err, DEV_TIMEOUT_TMA_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    mma_kblock<true>(d, smem_u32(smem + s * Cfg::STAGE_BYTES), BM, BN / 2, idesc, kb == 0);
                    umma_commit_pair(&empty[s]);
                }
                if (ok) umma_commit_pair(&acc_full[buf]);
            }
        }
    } else {
        const int q = warp & 3, half = (warp - 2) / 4;  // TMEM lane quadrant, column half
        const uint32_t acc_empty_leader = leader_addr(&acc_empty[0]);
        int it = 0;
        uint32_t sbuf = 0;
        for (int t = cid; t < tiles; t += ncl, it++) {
            const int buf = it & 1;
            const bool ok =
                __all_sync(0xffffffffu, mbar_wait_cluster(&acc_full[buf], (it >> 1) & 1, err, DEV_TIMEOUT_ACC));
            if (!ok) break;
            tc_fence_after();
            const PairTile tile = pair_tile<BN>(t, tiles_n, full, split);
            const int m0 = tile.mt * 2 * BM + rank * BM;
            const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
            if (epi.tma) {
                // this warp's columns: half of the tile, in the mode's chunks (64 columns for
                // the attention operands, else 32)
                const int chunk = epi.mode == EPI_QKV_ATTN ? 64 : 32;
                const int cw = Cfg::EPI_WARPS == 8 ? ((tile.nw / 2 + chunk - 1) / chunk) * chunk : tile.nw;
                const int c0 = half * cw, c1 = min(tile.nw, c0 + cw);
                if (c0 < c1)
                    epilogue_tile_tma<BN, Cfg::STAGE_BOX == 8192>(
                        epi, tl, m0, tile.n0, M, N, q, lane,
                        smem + Cfg::STAGES * Cfg::STAGE_BYTES + 1024 + (warp - 2) * Cfg::STAGE_BOX, sbuf, c0, c1);
            } else if (half == 0) {  // direct stores, one warp per quadrant
                epilogue_tile<BN>(epi, tl, m0, tile.n0, M, N, q, lane, nullptr, tile.nw);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(acc_empty_leader + 8u * buf);
        }
        if (lane == 0) bulk_wait0();
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // the peer's TMEM reads and remote arrives are done
    if (warp == 1) tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
}

// ------------------------------------------------------ split-K reduction
// dst[r, c] += ((p_0 + p_1 + ...) + bias[c]) over the ks partial tiles (rows r of
// split s at parts[(s * Mp + r) * N + c]), in split order: the same bits every run.
__global__ void split_reduce_kernel(const float* __restrict__ parts, int ks, long long Mp, int M, int N,
                                    const float* __restrict__ bias, float* __restrict__ dst, long long ldd) {
    griddep_wait();
    griddep_launch_dependents();
    const long long n4 = (long long)M * (N / 4);
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / (N / 4);
        const int c = (int)(i - r * (N / 4)) * 4;
        float4 a = *reinterpret_cast<const float4*>(parts + r * N + c);
        for (int sp = 1; sp < ks; sp++) {
            const float4 b = *reinterpret_cast<const float4*>(parts + ((long long)sp * Mp + r) * N + c);
            a = make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
        }
        if (bias) a = make_float4(__fadd_rn(a.x, bias[c]), __fadd_rn(a.y, bias[c + 1]), __fadd_rn(a.z, bias[c + 2]),
                                  __fadd_rn(a.w, bias[c + 3]));
        float4* d = reinterpret_cast<float4*>(dst + r * ldd + c);
        const float4 x = *d;
        *d = make_float4(__fadd_rn(x.x, a.x), __fadd_rn(x.y, a.y), __fadd_rn(x.z, a.z), __fadd_rn(x.w, a.w));
    }
}

// ------------------------------------------------------------ tensor maps

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    if (!fn) throw Error(9 /*N3D_ERR_GPU*/, "cuTensorMapEncodeTiled is unavailable");
    return fn;
}

// Element types of the maps: fp32 and fp16 (the split operands).
enum MapType : int { MAP_F32 = 4, MAP_F16 = 2 };

// 2-D map over a row-major matrix [rows, cols] of `type` elements (row stride ld
// elements), box = box_cols x box_rows, swizzle = box_cols * element size bytes (32,
// 64, 128) or none, zero fill out of bounds.
CUtensorMap encode_map(const void* ptr, int type, long long rows, long long cols, long long ld, int box_cols,
                       int box_rows, bool swizzle) {
    const int esize = type == MAP_F32 ? 4 : 2;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * esize) % 16)
        throw Error(9, "GEMM operand or output is not 16-byte aligned");
    CUtensorMap m;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * esize};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    const int span = box_cols * esize;
    const CUtensorMapSwizzle sw = !swizzle      ? CU_TENSOR_MAP_SWIZZLE_NONE
                                  : span == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : span == 64  ? CU_TENSOR_MAP_SWIZZLE_64B
                                                : CU_TENSOR_MAP_SWIZZLE_32B;
    const CUtensorMapDataType dt = type == MAP_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = encode_fn()(&m, dt, 2,
                             const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(9, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return m;
}

CUtensorMap cached_map(const void* ptr, int type, long long rows, long long cols, long long ld, int box_cols,
                       int box_rows, bool swizzle) {
    using Key = std::tuple<const void*, int, long long, long long, long long, int, int, bool>;
    static std::map<Key, CUtensorMap> cache;
    static std::mutex mu;
    const Key key{ptr, type, rows, cols, ld, box_cols, box_rows, swizzle};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    const CUtensorMap m = encode_map(ptr, type, rows, cols, ld, box_cols, box_rows, swizzle);
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, m);
    return m;
}

// The four operand maps: A with box rows ra, B with box rows rb, BK columns each.
Maps4 operand_maps(const SplitOperand& A, const SplitOperand& B, int ra, int rb, bool cache) {
    auto mk = cache ? cached_map : encode_map;
    Maps4 m;
    const SplitOperand* ops[2] = {&A, &B};
    for (int i = 0; i < 2; i++) {
        const SplitOperand& o = *ops[i];
        const int rows = i == 0 ? ra : rb;
        m.m[2 * i] = mk(o.h, MAP_F16, o.rows, o.cols, o.ld, BK, rows, true);
        m.m[2 * i + 1] = mk(o.l, MAP_F16, o.rows, o.cols, o.ld, BK, rows, true);
    }
    return m;
}


template <int BN>
void launch_one(cudaStream_t s, const Maps4& maps, int M, int N, int K, int kb_per_tap, const Epi& epi, int* err,
                int ksplit = 1, int Mp = 0) {
    using Cfg = GemmCfg<BN>;
    static std::atomic<unsigned long long> attr{0};
    once_per_device(attr, [] {
        N3D_CUDA(cudaFuncSetAttribute(gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    });
    const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN) * ksplit;
    const int grid = tiles < sm_count() ? tiles : sm_count();
    launch_pdl(gemm_kernel<BN>, dim3(grid), dim3(192), Cfg::SMEM, s, maps, M, N, K, kb_per_tap, epi, err, ksplit,
               Mp);
}

template <int BN, int EW>
void launch_pair(cudaStream_t s, const SplitOperand& A, const SplitOperand& B, int M, int N, int K, int kb_per_tap,
                 const Epi& epi, int* err) {
    using Cfg = PairCfg<BN, EW>;
    static std::atomic<int> clusters_per_device[kMaxDevices];  // 0 until measured on that device
    const int dev = current_device();
    int max_clusters = clusters_per_device[dev].load(std::memory_order_acquire);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see launch_pdl
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.blockDim = dim3(Cfg::THREADS);
    cfg.dynamicSmemBytes = Cfg::SMEM;
    cfg.stream = s;
    if (!max_clusters) {
        N3D_CUDA(cudaFuncSetAttribute(gemm_pair_kernel<BN, EW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      Cfg::SMEM));
        cfg.gridDim = dim3(2 * (sm_count() / 2));
        N3D_CUDA(cudaOccupancyMaxActiveClusters(&max_clusters, gemm_pair_kernel<BN, EW>, &cfg));
        if (max_clusters <= 0) throw Error(9, "no CTA pair of the GEMM fits on this device");
        clusters_per_device[dev].store(max_clusters, std::memory_order_release);
    }
    const Maps4 maps = operand_maps(A, B, BM, BN / 2, true);
    const int tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + BN - 1) / BN);
    const int clusters = tiles < max_clusters ? tiles : max_clusters;
    // tail split: the R tiles of a partial last wave become R * split narrower tiles
    // (split 2 or 4, with R * split <= clusters; widths stay multiples of 64 columns)
    const int waves = tiles / clusters, rem = tiles - waves * clusters;
    int split = 1;
    if (waves >= 1 && rem > 0) split = clusters / rem >= 4 && BN / 4 >= 64 ? 4 : clusters / rem >= 2 ? 2 : 1;
    const int full = tiles - rem;
    cfg.gridDim = dim3(2 * clusters);
    cfg.numAttrs = 2;
    N3D_CUDA(cudaLaunchKernelEx(&cfg, gemm_pair_kernel<BN, EW>, maps, M, N, K, kb_per_tap, epi, err, full, split));
}

void check_shape(const SplitOperand& A, const SplitOperand& B, int K, int kb_per_tap, const Epi& epi, int bn) {
    if (K % 32) throw Error(13, "GEMM K must be a multiple of 32");
    if (kb_per_tap > 0 && K % BK) throw Error(13, "the implicit-conv GEMM needs K and its taps in blocks of 64");
    if (!A.h || !A.l || !B.h || !B.l) throw Error(13, "GEMM operand without both fp16 parts");
    if (epi.mode == EPI_DENSE_OUT && (bn != 192 || epi.n2 > 8 || epi.tma))
        throw Error(9, "the fused dense+out_proj epilogue needs N == 192, at most 8 outputs and direct stores");
    if (epi.reduce && (epi.mode != EPI_STORE || !epi.tma))
        throw Error(9, "the reduce-add epilogue stores plain fp32 through TMA");
    if (epi.mode == EPI_QKV_ATTN && (bn % 64 || !epi.tma))
        throw Error(9, "the attention-operand epilogue needs 64-column chunks and TMA stores");
}

}  // namespace

// Streaming multiprocessors of the current device (queried once per device).
int sm_count() {
    static std::atomic<int> count[kMaxDevices];  // per device, 0 until queried
    const int dev = current_device();
    int n = count[dev].load(std::memory_order_relaxed);
    if (!n) {
        N3D_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        count[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

float split_scale(double bound) {
    if (!(bound > 0.0) || !std::isfinite(bound)) return 1.0f;
    int e = (int)std::floor(std::log2(32768.0 / bound));
    while (e > -60 && std::ldexp(bound, e) > 32768.0) e--;  // guard the log2 rounding
    e = std::max(-60, std::min(60, e));
    return (float)std::ldexp(1.0, e);
}

CUtensorMap make_store_map(const float* p, long long rows, long long cols, long long ld) {
    return cached_map(p, MAP_F32, rows, cols, ld, 32, 32, true);
}

CUtensorMap make_store_map_f16(const void* p, long long rows, long long cols, long long ld) {
    return cached_map(p, MAP_F16, rows, cols, ld, 32, 32, true);
}

CUtensorMap make_f16_map(const void* p, long long rows, long long cols, long long ld, int box_cols, int box_rows,
                         bool swizzle) {
    if (swizzle && box_cols != 64) throw Error(9, "fp16 map: the 128-byte swizzle needs 64-column boxes");
    return cached_map(p, MAP_F16, rows, cols, ld, box_cols, box_rows, swizzle);
}

// A plain fp32 output (EPI_STORE without a reduce) whose rows start on 16-byte
// boundaries leaves through the TMA epilogue: 32 x 32 boxes staged in shared memory,
// instead of each thread writing its own row.  The values are the same either way.
void store_via_tma(Epi& epi, int M, int N, bool cache) {
    if (epi.mode != EPI_STORE || epi.tma || epi.reduce || !epi.out || epi.ldo < N || epi.ldo % 4 ||
        (reinterpret_cast<uintptr_t>(epi.out) & 15))
        return;
    epi.map_out = cache ? make_store_map(epi.out, M, N, epi.ldo)
                        : encode_map(epi.out, MAP_F32, M, N, epi.ldo, 32, 32, true);
    epi.tma = 1;
}

void gemm_split(cudaStream_t s, const SplitOperand& A, const SplitOperand& B, int M, int N, int K, int kb_per_tap,
                const Epi& epi_in, int* err) {
    if (M <= 0 || N <= 0) return;
    Epi epi = epi_in;
    epi.acc_scale = (float)(1.0 / ((double)A.scale * (double)B.scale));
    store_via_tma(epi, M, N, true);
    int bn;
    if (epi.mode == EPI_DENSE_OUT || N == 192) {
        bn = 192;
    } else if (N % 256 == 0 && M >= 4096) {
        bn = 512;  // 256 x 256 tiles on CTA pairs
    } else if (N % 128 == 0 || N > 64) {
        bn = 128;
        // small launches (a single long clip's windows): 128 x 64 tiles when 128 x 128
        // ones would leave more than half the SMs idle
        const long long tiles = (long long)((M + BM - 1) / BM) * ((N + 127) / 128);
        if (N % 64 == 0 && tiles < sm_count() / 2) bn = 64;
    } else {
        bn = 64;
    }
    check_shape(A, B, K, kb_per_tap, epi, bn == 512 ? 256 : bn);
    if ((bn == 64 || bn == 128) && epi.mode == EPI_STORE && epi.tma && epi.reduce && epi.split_ws && kb_per_tap == 0 &&
        N % 4 == 0 && epi.out && epi.ldo > 0) {
        // split K (2..4 ways, >= 4 k-blocks each) while the tiles still fit one wave
        const int mt = (M + BM - 1) / BM, tiles = mt * ((N + bn - 1) / bn), nkb = (K + BK - 1) / BK, sms = sm_count();
        int ks = 1;
        while (ks < 4 && tiles * (ks + 1) <= sms && nkb / (ks + 1) >= 4) ks++;
        const long long Mp = (long long)mt * BM;
        if (ks > 1 && (long long)ks * Mp * N <= epi.split_ws_floats) {
            Epi ep = epi;  // partial tiles: plain TMA stores, no bias
            ep.reduce = 0;
            ep.bias = nullptr;
            ep.map_out = make_store_map(epi.split_ws, ks * Mp, N, N);
            if (bn == 64)
                launch_one<64>(s, operand_maps(A, B, BM, 64, true), M, N, K, 0, ep, err, ks, (int)Mp);
            else
                launch_one<128>(s, operand_maps(A, B, BM, 128, true), M, N, K, 0, ep, err, ks, (int)Mp);
            const long long n4 = (long long)M * (N / 4);
            const int blocks = (int)std::min<long long>((n4 + 255) / 256, 4LL * sms);
            launch_pdl(split_reduce_kernel, dim3(blocks), dim3(256), 0, s, (const float*)epi.split_ws, ks, Mp, M, N,
                       epi.bias, epi.out, epi.ldo);
            return;
        }
    }
    switch (bn) {
        case 64: launch_one<64>(s, operand_maps(A, B, BM, 64, true), M, N, K, kb_per_tap, epi, err); break;
        case 128: launch_one<128>(s, operand_maps(A, B, BM, 128, true), M, N, K, kb_per_tap, epi, err); break;
        case 192: launch_one<192>(s, operand_maps(A, B, BM, 192, true), M, N, K, kb_per_tap, epi, err); break;
        default:
            if (epi.mode == EPI_QKV_ATTN || epi.reduce)
                launch_pair<256, 4>(s, A, B, M, N, K, kb_per_tap, epi, err);
            else
                launch_pair<256, 8>(s, A, B, M, N, K, kb_per_tap, epi, err);
            break;
    }
}

// Same kernel (128-column tiles) with tensor maps encoded on the stack: no map cache,
// so nothing is allocated on the host heap either (the allocation-free entry point).
void gemm_split_stack_maps(cudaStream_t s, const SplitOperand& A, const SplitOperand& B, int M, int N, int K,
                           const Epi& epi_in, int* err) {
    if (M <= 0 || N <= 0) return;
    Epi epi = epi_in;
    epi.acc_scale = (float)(1.0 / ((double)A.scale * (double)B.scale));
    store_via_tma(epi, M, N, false);
    check_shape(A, B, K, 0, epi, 128);
    launch_one<128>(s, operand_maps(A, B, BM, 128, false), M, N, K, 0, epi, err);
}

}  // namespace n3d
