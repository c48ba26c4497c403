// Softmax attention on the sm_100a tensor cores (tcgen05, 3xTF32), head_dim 64.
//
// Replaces the reference's three attention dispatches -- `gemm_strided` QK^T,
// `attn_sm` softmax with the key-padding mask, `gemm_n64` PV (src/gpu.rs:390-396,
// 1914-1971; src/gpu_engine.rs:162-211) -- and must agree with the CPU
// `attention` (src/encoder.rs:302-329): scores q.k * hd^-1/2 over the first
// `valid` keys, softmax, context = sum p v.  No S x S scores buffer exists.
//
// CTA = 128 queries of one (sequence, head); 6 warps:
//   warp 0      TMA: the Q pair once, then per block of 64 keys the K pair and
//               the V^T pair into a 2-stage ring
//   warp 1      TMEM owner; one thread issues S_j = Q K_j^T (into one of two S
//               buffers, so block j+1's QK^T overlaps block j's softmax) and
//               O_j = P_j V_j with P_j read straight from TMEM
//   warps 2..9  softmax, two warps per query row (TMEM lane): each takes half of
//               the block's keys and half of the output columns; online max/sum,
//               P_j as a TF32 pair written back to TMEM, O folded in registers
// TMEM columns: S[2] 0..127, P_hi/P_lo[2] 128..383, O[2] 384..511.
// Every wait is bounded; an expired wait records its site in *err.

#include "n3d_device.cuh"
#include "n3d_internal.h"

namespace n3d {

namespace {

constexpr int HD = 64;       // head dim
constexpr int QT = 128;      // queries per CTA
constexpr int KB = 64;       // keys per block
constexpr int Q_ATOM = QT * 128;         // [128 rows x 128 B] = 16 KB
constexpr int KV_ATOM = KB * 128;        // [64 rows x 128 B] = 8 KB
constexpr int Q_BYTES = 2 * Q_ATOM;      // one of hi / lo: 32 KB
constexpr int KV_BYTES = 2 * KV_ATOM;    // one of K_hi / K_lo / V_hi / V_lo: 16 KB
constexpr int STAGE_BYTES = 4 * KV_BYTES;
constexpr int SMEM_BYTES = 2 * Q_BYTES + 2 * STAGE_BYTES + 1024 + 256 + 6 * QT * 4;
constexpr int THREADS = 320;  // TMA warp, MMA warp, 8 softmax warps
constexpr uint32_t COL_S = 0, COL_PHI = 128, COL_PLO = 192, COL_O = 384;  // P buffers: +128 per buffer
constexpr int DEV_TIMEOUT_ATTN = 5;

__device__ __forceinline__ uint32_t col_p_hi(int b) { return COL_PHI + 128u * b; }
__device__ __forceinline__ uint32_t col_p_lo(int b) { return COL_PLO + 128u * b; }

__global__ void __launch_bounds__(THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tQh, const __grid_constant__ CUtensorMap tQl,
                        const __grid_constant__ CUtensorMap tKh, const __grid_constant__ CUtensorMap tKl,
                        const __grid_constant__ CUtensorMap tVh, const __grid_constant__ CUtensorMap tVl, int S,
                        const int* __restrict__ valid_arr, int heads, float* __restrict__ ctx_hi,
                        float* __restrict__ ctx_lo, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQh = smem;
    uint8_t* sQl = smem + Q_BYTES;
    uint8_t* stages = smem + 2 * Q_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(stages + 2 * STAGE_BYTES);
    uint64_t* q_full = bars;        // 1
    uint64_t* kv_full = bars + 1;   // 2
    uint64_t* kv_empty = bars + 3;  // 2
    uint64_t* s_full = bars + 5;    // 2
    uint64_t* s_free = bars + 7;    // 2
    uint64_t* p_full = bars + 9;    // 2
    uint64_t* o_full = bars + 11;   // 2
    uint64_t* o_free = bars + 13;   // 2
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
    float* red_max = reinterpret_cast<float*>(bars + 32);  // [2 blocks][2 halves][QT]
    float* red_sum = red_max + 4 * QT;                      // [2 halves][QT]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * QT;
    const int valid = min(valid_arr[b], S);
    const int nblk = (valid + KB - 1) / KB;
    const int row0 = b * S;  // first row of this sequence in Q / K

    if (warp == 0 && lane == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&kv_full[i], 1);
            mbar_init(&kv_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 8);
            mbar_init(&p_full[i], 8);
            mbar_init(&o_full[i], 1);
            mbar_init(&o_free[i], 8);
        }
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0 && nblk > 0) {
            mbar_arrive_expect_tx(q_full, 2 * Q_BYTES);
            for (int a = 0; a < 2; a++) {
                tma_load_2d(sQh + a * Q_ATOM, &tQh, q_full, h * HD + 32 * a, row0 + q0);
                tma_load_2d(sQl + a * Q_ATOM, &tQl, q_full, h * HD + 32 * a, row0 + q0);
            }
            for (int j = 0; j < nblk; j++) {
                const int st = j & 1;
                if (j >= 2 && !mbar_wait(&kv_empty[st], ((j >> 1) - 1) & 1, err, DEV_TIMEOUT_ATTN)) break;
                uint8_t* sb = stages + st * STAGE_BYTES;
                mbar_arrive_expect_tx(&kv_full[st], STAGE_BYTES);
                for (int a = 0; a < 2; a++) {
                    tma_load_2d(sb + a * KV_ATOM, &tKh, &kv_full[st], h * HD + 32 * a, row0 + j * KB);
                    tma_load_2d(sb + KV_BYTES + a * KV_ATOM, &tKl, &kv_full[st], h * HD + 32 * a, row0 + j * KB);
                    tma_load_2d(sb + 2 * KV_BYTES + a * KV_ATOM, &tVh, &kv_full[st], row0 + j * KB + 32 * a, h * HD);
                    tma_load_2d(sb + 3 * KV_BYTES + a * KV_ATOM, &tVl, &kv_full[st], row0 + j * KB + 32 * a, h * HD);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && nblk > 0) {
            constexpr uint32_t idesc = idesc_tf32(64);
            bool ok = mbar_wait(q_full, 0, err, DEV_TIMEOUT_ATTN);
            const uint32_t qh = smem_u32(sQh), ql = smem_u32(sQl);
            auto issue_qk = [&](int j) {
                const uint32_t kb = smem_u32(stages + (j & 1) * STAGE_BYTES);
                const uint32_t d = tmem + COL_S + 64u * (j & 1);
#pragma unroll
                for (int k = 0; k < HD / 8; k++) {
                    const uint32_t qa = (k >> 2) * Q_ATOM + (k & 3) * 32, ka = (k >> 2) * KV_ATOM + (k & 3) * 32;
                    umma_tf32(d, desc_k_sw128(ql + qa), desc_k_sw128(kb + ka), idesc, k != 0);
                    umma_tf32(d, desc_k_sw128(qh + qa), desc_k_sw128(kb + KV_BYTES + ka), idesc, 1);
                    umma_tf32(d, desc_k_sw128(qh + qa), desc_k_sw128(kb + ka), idesc, 1);
                }
                umma_commit(&s_full[j & 1]);
            };
            if (ok) ok = mbar_wait(&kv_full[0], 0, err, DEV_TIMEOUT_ATTN);
            if (ok) {
                tc_fence_after();
                issue_qk(0);
            }
            for (int j = 0; ok && j < nblk; j++) {
                if (j + 1 < nblk) {
                    ok = mbar_wait(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1, err, DEV_TIMEOUT_ATTN);
                    if (ok && j + 1 >= 2)
                        ok = mbar_wait(&s_free[(j + 1) & 1], (((j + 1) >> 1) - 1) & 1, err, DEV_TIMEOUT_ATTN);
                    if (!ok) break;
                    tc_fence_after();
                    issue_qk(j + 1);
                }
                ok = mbar_wait(&p_full[j & 1], (j >> 1) & 1, err, DEV_TIMEOUT_ATTN);
                if (ok && j >= 2) ok = mbar_wait(&o_free[j & 1], ((j >> 1) - 1) & 1, err, DEV_TIMEOUT_ATTN);
                if (!ok) break;
                tc_fence_after();
                const uint32_t vb = smem_u32(stages + (j & 1) * STAGE_BYTES + 2 * KV_BYTES);
                const uint32_t d = tmem + COL_O + 64u * (j & 1);
                const uint32_t ph = tmem + col_p_hi(j & 1), pl = tmem + col_p_lo(j & 1);
#pragma unroll
                for (int k = 0; k < KB / 8; k++) {
                    const uint32_t va = (k >> 2) * KV_ATOM + (k & 3) * 32;
                    umma_tf32_ts(d, pl + 8 * k, desc_k_sw128(vb + va), idesc, k != 0);
                    umma_tf32_ts(d, ph + 8 * k, desc_k_sw128(vb + KV_BYTES + va), idesc, 1);
                    umma_tf32_ts(d, ph + 8 * k, desc_k_sw128(vb + va), idesc, 1);
                }
                umma_commit(&o_full[j & 1]);
                umma_commit(&kv_empty[j & 1]);
            }
        }
    } else {
        // ---- softmax warps 2..9: warp w owns TMEM lane quadrant w % 4 (query rows) and
        // half hf of each 64-key block and of the 64 output columns; the two warps of
        // a quadrant exchange row maxima and sums through shared memory.
        const int qd = warp & 3, hf = (warp - 2) >> 2;
        const int r = qd * 32 + lane;
        const uint32_t lb = tmem + (static_cast<uint32_t>(qd * 32) << 16);
        const uint32_t bar_id = 1 + qd;  // named barrier of this quadrant's two warps
        const float scaling = 0.125f;    // 1 / sqrt(64)
        float o[32];
#pragma unroll
        for (int d = 0; d < 32; d++) o[d] = 0.0f;
        float m = -INFINITY, l = 0.0f, c_prev = 0.0f;
        bool ok = true;
        auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory"); };
        auto fold = [&](int jj, float c) {  // O <- O * c + PV_jj, this warp's 32 columns
            float v[32];
            tmem_ld32(lb + COL_O + 64u * (jj & 1) + 32 * hf, v);
#pragma unroll
            for (int i = 0; i < 32; i++) o[i] = fmaf(o[i], c, v[i]);
        };
        for (int j = 0; j < nblk; j++) {
            const int bf = j & 1;
            // after an expired wait the loop keeps running (work skipped, results unused)
            // so both warps of the pair reach every pair_sync
            ok = __all_sync(0xffffffffu, ok && mbar_wait(&s_full[bf], (j >> 1) & 1, err, DEV_TIMEOUT_ATTN));
            tc_fence_after();
            float s[32];
            tmem_ld32(lb + COL_S + 64u * bf + 32 * hf, s);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[bf]);
            float mloc = -INFINITY;
#pragma unroll
            for (int c = 0; c < 32; c++) {
                s[c] = (j * KB + 32 * hf + c < valid) ? s[c] * scaling : -INFINITY;
                mloc = fmaxf(mloc, s[c]);
            }
            red_max[(bf * 2 + hf) * QT + r] = mloc;
            pair_sync();
            const float mx = fmaxf(m, fmaxf(mloc, red_max[(bf * 2 + (hf ^ 1)) * QT + r]));
            const float corr = (m == -INFINITY) ? 0.0f : expf(m - mx);
            float sum = 0.0f;
#pragma unroll
            for (int c = 0; c < 32; c++) {
                s[c] = (s[c] == -INFINITY) ? 0.0f : expf(s[c] - mx);
                sum += s[c];
            }
            l = l * corr + sum;  // this half's partial row sum, at the common running max
            m = mx;
            // PV_{j-1} done => P buffer bf (read by PV_{j-2}) is free and O_{j-1} is ready
            if (j >= 1) {
                ok = __all_sync(0xffffffffu, ok && mbar_wait(&o_full[(j - 1) & 1], ((j - 1) >> 1) & 1, err,
                                                             DEV_TIMEOUT_ATTN));
                tc_fence_after();
            }
            {
                float hi[32], lo[32];
#pragma unroll
                for (int i = 0; i < 32; i++) split_tf32(s[i], hi[i], lo[i]);
                tmem_st32(lb + col_p_hi(bf) + 32 * hf, hi);
                tmem_st32(lb + col_p_lo(bf) + 32 * hf, lo);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[bf]);
            if (j >= 1) {
                fold(j - 1, c_prev);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&o_free[(j - 1) & 1]);
            }
            c_prev = corr;
        }
        if (ok && nblk > 0) {
            ok = __all_sync(0xffffffffu,
                            mbar_wait(&o_full[(nblk - 1) & 1], ((nblk - 1) >> 1) & 1, err, DEV_TIMEOUT_ATTN));
            if (ok) {
                tc_fence_after();
                fold(nblk - 1, c_prev);
            }
        }
        red_sum[hf * QT + r] = l;
        pair_sync();
        const float ltot = l + red_sum[(hf ^ 1) * QT + r];
        // ---- context row, this warp's 32 columns (TF32 pair, or plain fp32 when ctx_lo is null)
        if (q0 + r < S) {
            const float inv = ltot > 0.0f ? 1.0f / ltot : 0.0f;
            const long long off = (long long)(row0 + q0 + r) * (heads * HD) + h * HD + 32 * hf;
            float* dh = ctx_hi + off;
#pragma unroll
            for (int d = 0; d < 32; d += 4) {
                float x[4], lo[4];
#pragma unroll
                for (int i = 0; i < 4; i++) x[i] = o[d + i] * inv;
                if (ctx_lo) {
#pragma unroll
                    for (int i = 0; i < 4; i++) split_tf32(x[i], x[i], lo[i]);
                    *reinterpret_cast<float4*>(ctx_lo + off + d) = make_float4(lo[0], lo[1], lo[2], lo[3]);
                }
                *reinterpret_cast<float4*>(dh + d) = make_float4(x[0], x[1], x[2], x[3]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

CUtensorMap map2d(const float* p, long long rows, long long cols, long long ld, int box_rows) {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            throw Error(9, "cuTensorMapEncodeTiled is unavailable");
        fn = reinterpret_cast<EncodeTiledFn>(f);
    }
    if ((reinterpret_cast<uintptr_t>(p) & 15) || (ld * 4) % 16) throw Error(9, "attention operand misaligned");
    CUtensorMap m;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        throw Error(9, "cuTensorMapEncodeTiled failed (attention)");
    return m;
}

}  // namespace

// Q, K: TF32 pairs [rows_cap, heads*64] (sequence b at rows b*S ..), RoPE applied.
// V^T: TF32 pair [heads*64, vt_ld]; row h*64 + d holds v[r, h, d] at column r (global row).
void launch_attention_tc(cudaStream_t s, const float* q_hi, const float* q_lo, const float* k_hi,
                         const float* k_lo, long long rows_cap, const float* vt_hi, const float* vt_lo,
                         long long vt_ld, int seqs, int S, const int* valid, int heads, float* ctx_hi,
                         float* ctx_lo, int* err) {
    if (seqs <= 0 || S <= 0) return;
    if ((seqs > 1 && S % 4) || vt_ld % 4)
        throw Error(9, "attention: the sequence stride and V^T row stride must be multiples of 4");
    static bool attr = false;
    if (!attr) {
        N3D_CUDA(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        attr = true;
    }
    const long long W = (long long)heads * HD;
    const CUtensorMap qh = map2d(q_hi, rows_cap, W, W, QT), ql = map2d(q_lo, rows_cap, W, W, QT);
    const CUtensorMap kh = map2d(k_hi, rows_cap, W, W, KB), kl = map2d(k_lo, rows_cap, W, W, KB);
    const CUtensorMap vh = map2d(vt_hi, W, (long long)seqs * S, vt_ld, HD);
    const CUtensorMap vl = map2d(vt_lo, W, (long long)seqs * S, vt_ld, HD);
    dim3 grid((S + QT - 1) / QT, heads, seqs);
    attention_tc_kernel<<<grid, THREADS, SMEM_BYTES, s>>>(qh, ql, kh, kl, vh, vl, S, valid, heads, ctx_hi, ctx_lo, err);
    N3D_CUDA(cudaGetLastError());
}

}  // namespace n3d
