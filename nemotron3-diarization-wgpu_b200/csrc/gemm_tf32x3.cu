// C[M, N] = A[M, K] * B[N, K]^T on the sm_100a tensor cores (tcgen05, kind::tf32)
// with 3xTF32 error compensation and fused epilogues.
//
// Replaces the reference's WGSL `gemm` pipeline (src/gpu.rs:1005-1611, wrapper
// src/gpu.rs:726-744) and the separate `add`, `unary` (GELU/ReLU), `rope` and
// `col3` dispatches that followed it (src/gpu.rs:1768-1838, 1973-1999): those
// become epilogue modes of this one kernel.  The reference arithmetic it must
// agree with is `tensor::linear` (src/tensor.rs:22-57) in fp32; every operand
// is a TF32 hi/lo pair and each k-step issues lo*hi + hi*lo + hi*hi, which
// keeps the products at fp32 grade (a plain TF32 GEMM flips sigmoid>0.5
// decisions on this model, see the design notes).
//
// CTA = 6 warps, one 128 x BN output tile:
//   warp 0      one thread issues TMA loads of A_hi, A_lo, B_hi, B_lo per k-block
//   warp 1      allocates TMEM; one thread issues the UMMAs and the commits
//   warps 2..5  epilogue: tcgen05.ld the accumulator (warp w owns TMEM lanes
//               32*(w%4) .. +31, i.e. output rows), apply the mode, store.
// Shared memory holds STAGES k-blocks of 32 fp32 (128 B rows, 128-byte swizzle).
// Every wait is bounded; a wait that expires records its site in *err.

#include <cstdio>
#include <map>
#include <mutex>
#include <tuple>

#include "n3d_device.cuh"
#include "n3d_internal.h"

namespace n3d {

namespace {

constexpr int BM = 128;
constexpr int BK = 32;

template <int BN>
struct GemmCfg {
    static constexpr int A_BYTES = BM * BK * 4;
    static constexpr int B_BYTES = BN * BK * 4;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int STAGES = (200 * 1024) / STAGE_BYTES;
    static constexpr int TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
    static_assert(STAGES >= 2, "need at least two pipeline stages");
};

__device__ __forceinline__ float gelu_erf(float x) {
    // 0.5 * x * (1 + erf(x / sqrt(2))), the exact form of src/tensor.rs:113-120
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

// Store 32 consecutive fp32 values of one output row.
__device__ __forceinline__ void store_row32(float* dst, const float* v, int ncols_left) {
    if (ncols_left >= 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
        for (int i = 0; i < 32 && i < ncols_left; i++) dst[i] = v[i];
    }
}

// Epilogue of one 128 x BN accumulator tile held in TMEM at `tl` (this warp's
// lane quadrant and the tile's first column): row r = m0 + 32 * q + lane.
template <int BN>
__device__ __forceinline__ void epilogue_tile(const Epi& epi, uint32_t tl, int m0, int n0, int M, int N, int q,
                                              int lane) {
    const int r = m0 + q * 32 + lane;
    const bool row_ok = r < M;
    const int qq = r / epi.rdiv, t = r - qq * epi.rdiv;
    const bool keep = row_ok && t < epi.rkeep;
    const long long orow = (long long)qq * epi.rmul + t + epi.roff;
    const bool zero_row = epi.seq_len != nullptr && keep && t >= epi.seq_len[qq];
    
    if (epi.mode == EPI_QKV_ROPE) {
        // 64-column chunks = one head; rotate-half RoPE (src/encoder.rs:281-296)
        for (int c = 0; c < BN; c += 64) {
            float v[64];
            tmem_ld32(tl + c, v);
            tmem_ld32(tl + c + 32, v + 32);
            const int col0 = n0 + c;
            if (!keep || col0 >= N) continue;
            if (col0 < epi.q_cols + epi.k_cols) {
                const int pos = r % epi.rope_seq;
                const float* cs = epi.cos_t + (long long)pos * epi.head_dim;
                const float* sn = epi.sin_t + (long long)pos * epi.head_dim;
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const float x1 = v[i], x2 = v[32 + i];
                    v[i] = __fsub_rn(__fmul_rn(x1, cs[i]), __fmul_rn(x2, sn[i]));
                    v[32 + i] = __fadd_rn(__fmul_rn(x2, cs[32 + i]), __fmul_rn(x1, sn[32 + i]));
                }
            }
            float* dst = epi.out + orow * epi.ldo + col0;
            store_row32(dst, v, N - col0);
            store_row32(dst + 32, v + 32, N - col0 - 32);
        }
    } else if (epi.mode == EPI_DENSE_OUT) {
        // relu(dense) then the out projection, sequential over the hidden
        // index with separate multiply and add (src/tensor.rs:33-43)
        float acc[8];
#pragma unroll
        for (int o = 0; o < 8; o++) acc[o] = 0.0f;
        for (int c = 0; c < BN; c += 32) {
            float v[32];
            tmem_ld32(tl + c, v);
            if (!keep) continue;
            for (int i = 0; i < 32; i++) {
                const int col = n0 + c + i;
                if (col >= N) break;
                const float rr = fmaxf(__fadd_rn(v[i], epi.bias[col]), 0.0f);
#pragma unroll
                for (int o = 0; o < 8; o++)
                    if (o < epi.n2) acc[o] = __fadd_rn(acc[o], __fmul_rn(rr, epi.w2[o * N + col]));
            }
        }
        if (keep)
            for (int o = 0; o < epi.n2; o++) epi.out[orow * epi.ldo + o] = __fadd_rn(acc[o], epi.b2[o]);
    } else {
        for (int c = 0; c < BN; c += 32) {
            float v[32];
            tmem_ld32(tl + c, v);
            const int col0 = n0 + c;
            if (!keep || col0 >= N) continue;
            const int left = N - col0;
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const float b = (epi.bias != nullptr && col0 + i < N) ? epi.bias[col0 + i] : 0.0f;
                v[i] = __fadd_rn(v[i], b);
            }
            float* dst = epi.out + orow * epi.ldo + col0;
            switch (epi.mode) {
                case EPI_STORE:
                    store_row32(dst, v, left);
                    break;
                case EPI_RESID: {
                    for (int i = 0; i < 32 && i < left; i++) dst[i] = __fadd_rn(dst[i], v[i]);
                    break;
                }
                default: {
                    float lo[32];
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        float x = v[i];
                        if (epi.mode == EPI_GELU_SPLIT) x = gelu_erf(x);
                        if (epi.mode == EPI_RELU_SPLIT) x = fmaxf(x, 0.0f);
                        if (zero_row) x = 0.0f;
                        split_tf32(x, v[i], lo[i]);
                    }
                    store_row32(dst, v, left);
                    store_row32(epi.out_lo + orow * epi.ldo + col0, lo, left);
                }
            }
        }
    }
}

template <int BN>
__global__ void __launch_bounds__(192, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tA_hi, const __grid_constant__ CUtensorMap tA_lo,
                       const __grid_constant__ CUtensorMap tB_hi, const __grid_constant__ CUtensorMap tB_lo, int M,
                       int N, int K, int kb_per_tap, const __grid_constant__ Epi epi, int* err) {
    using Cfg = GemmCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty = full + Cfg::STAGES;
    uint64_t* acc_full = empty + Cfg::STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int nkb = K / BK;

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < Cfg::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_fence_init();
        tma_prefetch_desc(&tA_hi);
        tma_prefetch_desc(&tA_lo);
        tma_prefetch_desc(&tB_hi);
        tma_prefetch_desc(&tB_lo);
    }
    if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            for (int kb = 0; kb < nkb; kb++) {
                const int s = kb % Cfg::STAGES;
                const uint32_t ph = (kb / Cfg::STAGES) & 1;
                if (kb >= Cfg::STAGES && !mbar_wait(&empty[s], ph ^ 1, err, DEV_TIMEOUT_TMA_EMPTY)) break;
                uint8_t* st = smem + s * Cfg::STAGE_BYTES;
                mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
                const int tap = kb_per_tap > 0 ? kb / kb_per_tap : 0;
                const int ka = kb_per_tap > 0 ? (kb % kb_per_tap) * BK : kb * BK;
                tma_load_2d(st, &tA_hi, &full[s], ka, m0 + tap);
                tma_load_2d(st + Cfg::A_BYTES, &tA_lo, &full[s], ka, m0 + tap);
                tma_load_2d(st + 2 * Cfg::A_BYTES, &tB_hi, &full[s], kb * BK, n0);
                tma_load_2d(st + 2 * Cfg::A_BYTES + Cfg::B_BYTES, &tB_lo, &full[s], kb * BK, n0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32(BN);
            bool ok = true;
            for (int kb = 0; kb < nkb; kb++) {
                const int s = kb % Cfg::STAGES;
                const uint32_t ph = (kb / Cfg::STAGES) & 1;
                if (!mbar_wait(&full[s], ph, err, DEV_TIMEOUT_TMA_FULL)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a_hi = smem_u32(smem + s * Cfg::STAGE_BYTES);
                const uint32_t a_lo = a_hi + Cfg::A_BYTES;
                const uint32_t b_hi = a_hi + 2 * Cfg::A_BYTES;
                const uint32_t b_lo = b_hi + Cfg::B_BYTES;
#pragma unroll
                for (int k = 0; k < BK / 8; k++) {
                    const uint32_t off = k * 32;  // 8 tf32 = 32 bytes along the swizzled row
                    const uint64_t dah = desc_k_sw128(a_hi + off), dal = desc_k_sw128(a_lo + off);
                    const uint64_t dbh = desc_k_sw128(b_hi + off), dbl = desc_k_sw128(b_lo + off);
                    umma_tf32(tmem, dal, dbh, idesc, (kb | k) != 0);
                    umma_tf32(tmem, dah, dbl, idesc, 1);
                    umma_tf32(tmem, dah, dbh, idesc, 1);
                }
                umma_commit(&empty[s]);
            }
            if (ok) umma_commit(acc_full);
        }
    } else {
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        // warp-uniform result: the TMEM loads below are .sync.aligned
        const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, err, DEV_TIMEOUT_ACC));
        tc_fence_after();
        if (ok) {
            epilogue_tile<BN>(epi, tmem + (static_cast<uint32_t>(q * 32) << 16), m0, n0, M, N, q, lane);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, Cfg::TMEM_COLS);
}

// ------------------------------------------------------- TMA-store epilogue
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(x),
                 "r"(y), "r"(smem_u32(src))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// One warp's 32 x 32 fp32 block into a 4 KB 128-byte-swizzled staging box:
// lane = box row, v = its 32 columns.
__device__ __forceinline__ void stage_rows(uint8_t* box, int lane, const float* v) {
#pragma unroll
    for (int i = 0; i < 8; i++)
        *reinterpret_cast<float4*>(box + lane * 128 + ((i ^ (lane & 7)) << 4)) =
            make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

// Hand the staged boxes to TMA: wait until the previous boxes have been read,
// which the caller does before staging; here fence and issue.
__device__ __forceinline__ void stage_begin(int lane) {
    if (lane == 0) bulk_wait_read0();
    __syncwarp();
}
__device__ __forceinline__ void stage_issue(int lane, const CUtensorMap* m0, const void* b0, const CUtensorMap* m1,
                                            const void* b1, int x, int y) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(m0, b0, x, y);
        if (m1) tma_store_2d(m1, b1, x, y);
        bulk_commit();
    }
}

// Epilogue with TMA stores, for modes whose output rows are the tile's rows:
// EPI_STORE, EPI_SPLIT, EPI_GELU_SPLIT, EPI_RELU_SPLIT, EPI_QKV_ATTN.
// `stg` is this warp's 8 KB staging area (hi box, lo box).
template <int BN>
__device__ __forceinline__ void epilogue_tile_tma(const Epi& epi, uint32_t tl, int m0, int n0, int M, int N, int q,
                                                  int lane, uint8_t* stg, int c_begin = 0, int c_end = BN) {
    const int rowbase = m0 + q * 32;
    if (rowbase >= M) return;  // whole warp past the end: nothing to load or store
    const int r = rowbase + lane;
    uint8_t* bhi = stg;
    uint8_t* blo = stg + 4096;
    if (epi.mode == EPI_QKV_ATTN) {
        for (int c = c_begin; c < c_end; c += 64) {
            float v[64];
            tmem_ld32(tl + c, v);
            tmem_ld32(tl + c + 32, v + 32);
            const int col0 = n0 + c;
            if (col0 >= N) break;
            const int sec = col0 / epi.q_cols, hcol = col0 - sec * epi.q_cols;
            if (sec < 2) {
                // the tables repeat their first half (cat(freqs, freqs)), so one float4 of
                // cos and of sin serves four rotation pairs
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
            // bf16 pairs: Q / K rows (64 values = one 128-byte swizzled box row), V
            // transposed (box row = d, 32 rows of the tile = 64 bytes, unswizzled)
            uint32_t hi[32], lo[32];
#pragma unroll
            for (int i = 0; i < 32; i++) split_bf16x2(v[2 * i], v[2 * i + 1], hi[i], lo[i]);
            stage_begin(lane);
            if (sec < 2) {
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int o = lane * 128 + ((i ^ (lane & 7)) << 4);
                    *reinterpret_cast<uint4*>(bhi + o) = make_uint4(hi[4 * i], hi[4 * i + 1], hi[4 * i + 2], hi[4 * i + 3]);
                    *reinterpret_cast<uint4*>(blo + o) = make_uint4(lo[4 * i], lo[4 * i + 1], lo[4 * i + 2], lo[4 * i + 3]);
                }
                stage_issue(lane, sec == 0 ? &epi.map_out : &epi.map_k_hi, bhi,
                            sec == 0 ? &epi.map_out_lo : &epi.map_k_lo, blo, hcol, rowbase);
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    *reinterpret_cast<uint16_t*>(bhi + (2 * i) * 64 + lane * 2) = (uint16_t)(hi[i] & 0xffffu);
                    *reinterpret_cast<uint16_t*>(bhi + (2 * i + 1) * 64 + lane * 2) = (uint16_t)(hi[i] >> 16);
                    *reinterpret_cast<uint16_t*>(blo + (2 * i) * 64 + lane * 2) = (uint16_t)(lo[i] & 0xffffu);
                    *reinterpret_cast<uint16_t*>(blo + (2 * i + 1) * 64 + lane * 2) = (uint16_t)(lo[i] >> 16);
                }
                stage_issue(lane, &epi.map_vt_hi, bhi, &epi.map_vt_lo, blo, rowbase, hcol);
            }
        }
    } else {
        const bool pair = epi.mode != EPI_STORE;
        for (int c = c_begin; c < c_end; c += 32) {
            float v[32];
            tmem_ld32(tl + c, v);
            const int col0 = n0 + c;
            if (col0 >= N) break;
            float lo[32], bias[32];
            if (epi.bias != nullptr && col0 + 32 <= N) {
#pragma unroll
                for (int i4 = 0; i4 < 8; i4++) {
                    const float4 b4 = __ldg(reinterpret_cast<const float4*>(epi.bias + col0) + i4);
                    bias[4 * i4] = b4.x;
                    bias[4 * i4 + 1] = b4.y;
                    bias[4 * i4 + 2] = b4.z;
                    bias[4 * i4 + 3] = b4.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) bias[i] = (epi.bias != nullptr && col0 + i < N) ? epi.bias[col0 + i] : 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 32; i++) {
                float x = __fadd_rn(v[i], bias[i]);
                if (epi.mode == EPI_GELU_SPLIT) x = gelu_erf(x);
                if (epi.mode == EPI_RELU_SPLIT) x = fmaxf(x, 0.0f);
                if (pair)
                    split_tf32(x, v[i], lo[i]);
                else
                    v[i] = x;
            }
            stage_begin(lane);
            stage_rows(bhi, lane, v);
            if (pair) stage_rows(blo, lane, lo);
            stage_issue(lane, &epi.map_out, bhi, pair ? &epi.map_out_lo : nullptr, blo, col0, rowbase);
        }
    }
}

// Persistent variant: one CTA per SM walks the output tiles (t = blockIdx.x,
// + gridDim.x, ...), k-blocks of 16 fp32 (64 B rows, 64-byte swizzle) so that
// even BN = 256 gets 4 shared-memory stages, and two TMEM accumulators so the
// epilogue of tile i overlaps the main loop of tile i + 1.
constexpr int PBK = 16;

template <int BN>
struct PCfg {
    static constexpr int A_BYTES = BM * PBK * 4;
    static constexpr int B_BYTES = BN * PBK * 4;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int STAGING = 4 * 8192;  // per epilogue warp: hi + lo 32 x 32 boxes
    static constexpr int STAGES_FIT = (232448 - STAGING - 2048) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
    static constexpr int ACC_COLS = BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
    static constexpr int TMEM_COLS = 2 * ACC_COLS;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 1024 + STAGING;
    static_assert(STAGES >= 3, "persistent GEMM wants at least three stages");
};

template <int BN>
__global__ void __launch_bounds__(192, 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tA_hi, const __grid_constant__ CUtensorMap tA_lo,
                           const __grid_constant__ CUtensorMap tB_hi, const __grid_constant__ CUtensorMap tB_lo,
                           int M, int N, int K, int kb_per_tap, const __grid_constant__ Epi epi, int* err) {
    using Cfg = PCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty = full + Cfg::STAGES;
    uint64_t* acc_full = empty + Cfg::STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_n = (N + BN - 1) / BN;
    const int tiles = ((M + BM - 1) / BM) * tiles_n;
    const int nkb = K / PBK;

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
        tma_prefetch_desc(&tA_hi);
        tma_prefetch_desc(&tA_lo);
        tma_prefetch_desc(&tB_hi);
        tma_prefetch_desc(&tB_lo);
    }
    if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
                const int m0 = (t / tiles_n) * BM, n0 = (t % tiles_n) * BN;
                for (int kb = 0; kb < nkb; kb++, g++) {
                    const int s = g % Cfg::STAGES;
                    if (g >= (uint32_t)Cfg::STAGES &&
                        !mbar_wait(&empty[s], ((g / Cfg::STAGES) - 1) & 1, err, DEV_TIMEOUT_TMA_EMPTY)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + s * Cfg::STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
                    const int tap = kb_per_tap > 0 ? kb / kb_per_tap : 0;
                    const int ka = kb_per_tap > 0 ? (kb % kb_per_tap) * PBK : kb * PBK;
                    tma_load_2d(st, &tA_hi, &full[s], ka, m0 + tap);
                    tma_load_2d(st + Cfg::A_BYTES, &tA_lo, &full[s], ka, m0 + tap);
                    tma_load_2d(st + 2 * Cfg::A_BYTES, &tB_hi, &full[s], kb * PBK, n0);
                    tma_load_2d(st + 2 * Cfg::A_BYTES + Cfg::B_BYTES, &tB_lo, &full[s], kb * PBK, n0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32(BN);
            uint32_t g = 0;
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, it++) {
                const int buf = it & 1;
                if (it >= 2 && !mbar_wait(&acc_empty[buf], ((it >> 1) - 1) & 1, err, DEV_TIMEOUT_ACC)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * Cfg::ACC_COLS;
                for (int kb = 0; kb < nkb; kb++, g++) {
                    const int s = g % Cfg::STAGES;
                    if (!mbar_wait(&full[s], (g / Cfg::STAGES) & 1, err, DEV_TIMEOUT_TMA_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_hi = smem_u32(smem + s * Cfg::STAGE_BYTES);
                    const uint32_t a_lo = a_hi + Cfg::A_BYTES;
                    const uint32_t b_hi = a_hi + 2 * Cfg::A_BYTES;
                    const uint32_t b_lo = b_hi + Cfg::B_BYTES;
#pragma unroll
                    for (int k = 0; k < PBK / 8; k++) {
                        const uint32_t off = k * 32;
                        const uint64_t dah = desc_k_sw64(a_hi + off), dal = desc_k_sw64(a_lo + off);
                        const uint64_t dbh = desc_k_sw64(b_hi + off), dbl = desc_k_sw64(b_lo + off);
                        umma_tf32(d, dal, dbh, idesc, (kb | k) != 0);
                        umma_tf32(d, dah, dbl, idesc, 1);
                        umma_tf32(d, dah, dbh, idesc, 1);
                    }
                    umma_commit(&empty[s]);
                }
                if (ok) umma_commit(&acc_full[buf]);
            }
        }
    } else {
        const int q = warp & 3;
        int it = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, it++) {
            const int buf = it & 1;
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (it >> 1) & 1, err, DEV_TIMEOUT_ACC));
            if (!ok) break;
            tc_fence_after();
            const int m0 = (t / tiles_n) * BM, n0 = (t % tiles_n) * BN;
            const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * Cfg::ACC_COLS;
            if (epi.tma)
                epilogue_tile_tma<BN>(epi, tl, m0, n0, M, N, q, lane,
                                      smem + Cfg::STAGES * Cfg::STAGE_BYTES + 1024 + (warp - 2) * 8192);
            else
                epilogue_tile<BN>(epi, tl, m0, n0, M, N, q, lane);
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

// CTA-pair variant: a cluster of two CTAs walks 256 x BN output tiles with
// M = 256 UMMAs (cta_group::2).  CTA r of the pair loads A rows m0 + 128 r and
// B rows n0 + r * BN / 2, so each SM streams half the B tile of the one-CTA
// kernel for the same work; its TMEM receives output rows m0 + 128 r, which its
// own epilogue warps store.  Barriers: full[s] lives in the leader (both CTAs'
// loads complete on it), empty[s] and acc_full[b] in both (arrived by the
// leader's multicast commits), acc_empty[b] in the leader (8 epilogue warps).
template <int BN, int EW>
struct PairCfg {
    static constexpr int A_BYTES = BM * PBK * 4;
    static constexpr int B_BYTES = (BN / 2) * PBK * 4;
    static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
    static constexpr int STAGING = EW * 8192;  // per epilogue warp: hi + lo boxes
    static constexpr int THREADS = 64 + 32 * EW;
    static constexpr int STAGES_FIT = (232448 - STAGING - 2048) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 1024 + STAGING;
    static_assert(BN == 128 || BN == 256, "pair tiles are 256 x 128 or 256 x 256");
    static_assert(EW == 4 || EW == 8, "4 or 8 epilogue warps");
};

// EW epilogue warps per CTA: with 8, warps w and w + 4 share TMEM lane quadrant w % 4
// and take half of the tile's columns each (two warps per SM sub-partition hide the
// latency of heavy epilogues such as GELU + split).
template <int BN, int EW>
__global__ void __launch_bounds__(64 + 32 * EW, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tA_hi, const __grid_constant__ CUtensorMap tA_lo,
                     const __grid_constant__ CUtensorMap tB_hi, const __grid_constant__ CUtensorMap tB_lo, int M,
                     int N, int K, int kb_per_tap, const __grid_constant__ Epi epi, int* err) {
    using Cfg = PairCfg<BN, EW>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty = full + Cfg::STAGES;
    uint64_t* acc_full = empty + Cfg::STAGES;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rank = static_cast<int>(cluster_rank());
    const bool leader = rank == 0;
    const int cid = static_cast<int>(cluster_id_x()), ncl = static_cast<int>(cluster_count_x());
    const int tiles_n = (N + BN - 1) / BN;
    const int tiles = ((M + 2 * BM - 1) / (2 * BM)) * tiles_n;
    const int nkb = K / PBK;

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < Cfg::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 2 * EW);
        }
        mbar_fence_init();
        tma_prefetch_desc(&tA_hi);
        tma_prefetch_desc(&tA_lo);
        tma_prefetch_desc(&tB_hi);
        tma_prefetch_desc(&tB_lo);
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrive
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t g = 0;
            bool ok = true;
            for (int t = cid; ok && t < tiles; t += ncl) {
                const int m0 = (t / tiles_n) * 2 * BM + rank * BM, n0 = (t % tiles_n) * BN + rank * (BN / 2);
                for (int kb = 0; kb < nkb; kb++, g++) {
                    const int s = g % Cfg::STAGES;
                    if (g >= (uint32_t)Cfg::STAGES &&
                        !mbar_wait_cluster(&empty[s], ((g / Cfg::STAGES) - 1) & 1, err, DEV_TIMEOUT_TMA_EMPTY)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + s * Cfg::STAGE_BYTES;
                    if (leader) mbar_arrive_expect_tx(&full[s], 2 * Cfg::STAGE_BYTES);
                    const uint32_t fb = leader_addr(&full[s]);
                    const int tap = kb_per_tap > 0 ? kb / kb_per_tap : 0;
                    const int ka = kb_per_tap > 0 ? (kb % kb_per_tap) * PBK : kb * PBK;
                    tma_load_2d_pair(st, &tA_hi, fb, ka, m0 + tap);
                    tma_load_2d_pair(st + Cfg::A_BYTES, &tA_lo, fb, ka, m0 + tap);
                    tma_load_2d_pair(st + 2 * Cfg::A_BYTES, &tB_hi, fb, kb * PBK, n0);
                    tma_load_2d_pair(st + 2 * Cfg::A_BYTES + Cfg::B_BYTES, &tB_lo, fb, kb * PBK, n0);
                }
            }
        }
    } else if (warp == 1) {
        if (leader && lane == 0) {
            constexpr uint32_t idesc = idesc_tf32_pair(BN);
            uint32_t g = 0;
            int it = 0;
            bool ok = true;
            for (int t = cid; ok && t < tiles; t += ncl, it++) {
                const int buf = it & 1;
                if (it >= 2 && !mbar_wait_cluster(&acc_empty[buf], ((it >> 1) - 1) & 1, err, DEV_TIMEOUT_ACC)) break;
                tc_fence_after();
                const uint32_t d = tmem + buf * BN;
                for (int kb = 0; kb < nkb; kb++, g++) {
                    const int s = g % Cfg::STAGES;
                    if (!mbar_wait_cluster(&full[s], (g / Cfg::STAGES) & 1, err, DEV_TIMEOUT_TMA_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_hi = smem_u32(smem + s * Cfg::STAGE_BYTES);
                    const uint32_t a_lo = a_hi + Cfg::A_BYTES;
                    const uint32_t b_hi = a_hi + 2 * Cfg::A_BYTES;
                    const uint32_t b_lo = b_hi + Cfg::B_BYTES;
#pragma unroll
                    for (int k = 0; k < PBK / 8; k++) {
                        const uint32_t off = k * 32;
                        const uint64_t dah = desc_k_sw64(a_hi + off), dal = desc_k_sw64(a_lo + off);
                        const uint64_t dbh = desc_k_sw64(b_hi + off), dbl = desc_k_sw64(b_lo + off);
                        umma_tf32_pair(d, dal, dbh, idesc, (kb | k) != 0);
                        umma_tf32_pair(d, dah, dbl, idesc, 1);
                        umma_tf32_pair(d, dah, dbh, idesc, 1);
                    }
                    umma_commit_pair(&empty[s]);
                }
                if (ok) umma_commit_pair(&acc_full[buf]);
            }
        }
    } else {
        const int q = warp & 3, part = (warp - 2) >> 2;
        constexpr int CW = BN / (EW / 4);  // columns per epilogue warp
        const uint32_t acc_empty_leader = leader_addr(&acc_empty[0]);
        int it = 0;
        for (int t = cid; t < tiles; t += ncl, it++) {
            const int buf = it & 1;
            const bool ok =
                __all_sync(0xffffffffu, mbar_wait_cluster(&acc_full[buf], (it >> 1) & 1, err, DEV_TIMEOUT_ACC));
            if (!ok) break;
            tc_fence_after();
            const int m0 = (t / tiles_n) * 2 * BM + rank * BM, n0 = (t % tiles_n) * BN;
            const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
            if (epi.tma)
                epilogue_tile_tma<BN>(epi, tl, m0, n0, M, N, q, lane,
                                      smem + Cfg::STAGES * Cfg::STAGE_BYTES + 1024 + (warp - 2) * 8192, part * CW,
                                      part * CW + CW);
            else if (part == 0)  // direct stores: one warp per quadrant takes the whole tile
                epilogue_tile<BN>(epi, tl, m0, n0, M, N, q, lane);
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

// 2-D map over a row-major fp32 matrix [rows, cols] (row stride ld elements),
// box = 32 columns x box_rows rows, 128-byte swizzle, zero fill out of bounds.
CUtensorMap make_map(const float* ptr, long long rows, long long cols, long long ld, int box_rows, int box_cols = BK) {
    using Key = std::tuple<const float*, long long, long long, long long, int, int>;
    static std::map<Key, CUtensorMap> cache;
    static std::mutex mu;
    const Key key{ptr, rows, cols, ld, box_rows, box_cols};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * 4) % 16)
        throw Error(9, "GEMM operand or output is not 16-byte aligned");
    CUtensorMap m;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box,
                             estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             box_cols == 16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(9, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, m);
    return m;
}

template <int BN>
void launch(cudaStream_t s, const SplitOperand& A, const SplitOperand& B, int M, int N, int K, int kb_per_tap,
            const Epi& epi, int* err) {
    using Cfg = GemmCfg<BN>;
    static bool attr = false;
    if (!attr) {
        N3D_CUDA(cudaFuncSetAttribute(gemm_tf32x3_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      Cfg::SMEM));
        attr = true;
    }
    const CUtensorMap a_hi = make_map(A.hi, A.rows, A.cols, A.ld, BM);
    const CUtensorMap a_lo = make_map(A.lo, A.rows, A.cols, A.ld, BM);
    const CUtensorMap b_hi = make_map(B.hi, B.rows, B.cols, B.ld, BN);
    const CUtensorMap b_lo = make_map(B.lo, B.rows, B.cols, B.ld, BN);
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    gemm_tf32x3_kernel<BN><<<grid, 192, Cfg::SMEM, s>>>(a_hi, a_lo, b_hi, b_lo, M, N, K, kb_per_tap, epi, err);
    N3D_CUDA(cudaGetLastError());
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        N3D_CUDA(cudaGetDevice(&dev));
        N3D_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    }
    return n;
}

template <int BN>
void launch_persistent(cudaStream_t s, const SplitOperand& A, const SplitOperand& B, int M, int N, int K,
                       int kb_per_tap, const Epi& epi, int* err) {
    using Cfg = PCfg<BN>;
    static bool attr = false;
    if (!attr) {
        N3D_CUDA(cudaFuncSetAttribute(gemm_persistent_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      Cfg::SMEM));
        attr = true;
    }
    const CUtensorMap a_hi = make_map(A.hi, A.rows, A.cols, A.ld, BM, PBK);
    const CUtensorMap a_lo = make_map(A.lo, A.rows, A.cols, A.ld, BM, PBK);
    const CUtensorMap b_hi = make_map(B.hi, B.rows, B.cols, B.ld, BN, PBK);
    const CUtensorMap b_lo = make_map(B.lo, B.rows, B.cols, B.ld, BN, PBK);
    const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const int grid = tiles < sm_count() ? tiles : sm_count();
    gemm_persistent_kernel<BN><<<grid, 192, Cfg::SMEM, s>>>(a_hi, a_lo, b_hi, b_lo, M, N, K,
                                                             kb_per_tap > 0 ? kb_per_tap * (BK / PBK) : 0, epi, err);
    N3D_CUDA(cudaGetLastError());
}

template <int BN, int EW>
void launch_pair(cudaStream_t s, const SplitOperand& A, const SplitOperand& B, int M, int N, int K, int kb_per_tap,
                 const Epi& epi, int* err) {
    using Cfg = PairCfg<BN, EW>;
    static int max_clusters = 0;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.blockDim = dim3(Cfg::THREADS);
    cfg.dynamicSmemBytes = Cfg::SMEM;
    cfg.stream = s;
    if (!max_clusters) {
        N3D_CUDA(cudaFuncSetAttribute(gemm_pair_kernel<BN, EW>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
        cfg.gridDim = dim3(2 * (sm_count() / 2));
        N3D_CUDA(cudaOccupancyMaxActiveClusters(&max_clusters, gemm_pair_kernel<BN, EW>, &cfg));
        if (max_clusters <= 0) throw Error(9, "no CTA pair of the GEMM fits on this device");
    }
    const CUtensorMap a_hi = make_map(A.hi, A.rows, A.cols, A.ld, BM, PBK);
    const CUtensorMap a_lo = make_map(A.lo, A.rows, A.cols, A.ld, BM, PBK);
    const CUtensorMap b_hi = make_map(B.hi, B.rows, B.cols, B.ld, BN / 2, PBK);
    const CUtensorMap b_lo = make_map(B.lo, B.rows, B.cols, B.ld, BN / 2, PBK);
    const int tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + BN - 1) / BN);
    cfg.gridDim = dim3(2 * (tiles < max_clusters ? tiles : max_clusters));
    N3D_CUDA(cudaLaunchKernelEx(&cfg, gemm_pair_kernel<BN, EW>, a_hi, a_lo, b_hi, b_lo, M, N, K,
                                kb_per_tap > 0 ? kb_per_tap * (BK / PBK) : 0, epi, err));
}

}  // namespace

CUtensorMap make_store_map(const float* p, long long rows, long long cols, long long ld) {
    return make_map(p, rows, cols, ld, 32, 32);
}

CUtensorMap make_bf16_map(const void* p, long long rows, long long cols, long long ld, int box_cols, int box_rows,
                          bool swizzle) {
    using Key = std::tuple<const void*, long long, long long, long long, int, int, bool>;
    static std::map<Key, CUtensorMap> cache;
    static std::mutex mu;
    const Key key{p, rows, cols, ld, box_cols, box_rows, swizzle};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    if ((reinterpret_cast<uintptr_t>(p) & 15) || (ld * 2) % 16 || (swizzle && box_cols != 64))
        throw Error(9, "bf16 operand is not 16-byte aligned");
    CUtensorMap m;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(p), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE,
                             swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(9, "cuTensorMapEncodeTiled failed (bf16, " + std::to_string(int(r)) + ")");
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, m);
    return m;
}

void gemm_tf32x3(cudaStream_t s, const SplitOperand& A, const SplitOperand& B, int M, int N, int K,
                 int kb_per_tap, const Epi& epi, int* err) {
    if (M <= 0 || N <= 0) return;
    if (K % BK) throw Error(9, "GEMM K must be a multiple of 32");
    int bn;
    if (epi.mode == EPI_DENSE_OUT) {
        if (N != 192) throw Error(9, "the fused dense+out_proj epilogue needs N == 192");
        bn = 192;
    } else if (N == 192) {
        bn = 192;
    } else if (N % 256 == 0 && M >= 4096) {
        bn = 512;  // 256 x 256 tiles on CTA pairs
    } else if (N % 128 == 0 || N > 64) {
        bn = 128;
    } else {
        bn = 64;
    }
    if ((epi.mode == EPI_QKV_ROPE || epi.mode == EPI_QKV_ATTN) && (bn % 64))
        throw Error(9, "QKV epilogue needs 64-column chunks");
    if (epi.mode == EPI_QKV_ATTN && !epi.tma) throw Error(9, "the attention-operand epilogue stores through TMA only");
    switch (bn) {
        case 64: launch_persistent<64>(s, A, B, M, N, K, kb_per_tap, epi, err); break;
        case 128: launch_persistent<128>(s, A, B, M, N, K, kb_per_tap, epi, err); break;
        case 192: launch_persistent<192>(s, A, B, M, N, K, kb_per_tap, epi, err); break;
        default:
            // the erf-GELU + split epilogue is latency bound on one warp per sub-partition:
            // 8 epilogue warps (measured: FC1 177 -> 217 TFLOP/s; the lighter epilogues lose
            // more to the smaller pipeline than they gain)
            if (epi.tma && epi.mode == EPI_GELU_SPLIT)
                launch_pair<256, 8>(s, A, B, M, N, K, kb_per_tap, epi, err);
            else
                launch_pair<256, 4>(s, A, B, M, N, K, kb_per_tap, epi, err);
            break;
    }
}

// Same kernel with tensor maps encoded on the stack: no map cache, so nothing
// is allocated on the host heap either (used by the allocation-free entry point).
void gemm_tf32x3_stack_maps(cudaStream_t s, const SplitOperand& A, const SplitOperand& B, int M, int N, int K,
                            const Epi& epi, int* err) {
    if (M <= 0 || N <= 0) return;
    if (K % BK) throw Error(13, "GEMM K must be a multiple of 32");
    if ((reinterpret_cast<uintptr_t>(A.hi) | reinterpret_cast<uintptr_t>(A.lo) | reinterpret_cast<uintptr_t>(B.hi) |
         reinterpret_cast<uintptr_t>(B.lo)) & 15)
        throw Error(13, "GEMM operands must be 16-byte aligned");
    using Cfg = GemmCfg<128>;
    static bool attr = false;
    if (!attr) {
        N3D_CUDA(cudaFuncSetAttribute(gemm_tf32x3_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      Cfg::SMEM));
        attr = true;
    }
    CUtensorMap maps[4];
    const SplitOperand* ops[2] = {&A, &B};
    for (int i = 0; i < 4; i++) {
        const SplitOperand& o = *ops[i / 2];
        cuuint64_t dims[2] = {static_cast<cuuint64_t>(o.cols), static_cast<cuuint64_t>(o.rows)};
        cuuint64_t strides[1] = {static_cast<cuuint64_t>(o.ld) * 4};
        cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(i < 2 ? BM : 128)};
        cuuint32_t estr[2] = {1, 1};
        const float* p = (i % 2) ? o.lo : o.hi;
        CUresult r = encode_fn()(&maps[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p), dims, strides,
                                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) throw Error(9, "cuTensorMapEncodeTiled failed");
    }
    dim3 grid((N + 127) / 128, (M + BM - 1) / BM);
    gemm_tf32x3_kernel<128><<<grid, 192, Cfg::SMEM, s>>>(maps[0], maps[1], maps[2], maps[3], M, N, K, 0, epi, err);
    N3D_CUDA(cudaGetLastError());
}

// Explicit tile choice, for the kernel tests and tile sweeps.
void gemm_tf32x3_bn(cudaStream_t s, const SplitOperand& A, const SplitOperand& B, int M, int N, int K,
                    int kb_per_tap, const Epi& epi, int* err, int bn) {
    switch (bn) {
        case 64: launch<64>(s, A, B, M, N, K, kb_per_tap, epi, err); break;
        case 128: launch<128>(s, A, B, M, N, K, kb_per_tap, epi, err); break;
        case 192: launch<192>(s, A, B, M, N, K, kb_per_tap, epi, err); break;
        case 256: launch<256>(s, A, B, M, N, K, kb_per_tap, epi, err); break;
        default: throw Error(13, "unsupported GEMM tile width");
    }
}

}  // namespace n3d
