// Softmax attention on the sm_100a tensor cores (tcgen05, kind::f16), head_dim 64.
//
// Replaces the reference's three attention dispatches -- `gemm_strided` QK^T,
// `attn_sm` softmax with the key-padding mask, `gemm_n64` PV (src/gpu.rs:390-396,
// 1914-1971; src/gpu_engine.rs:162-211) -- and must agree with the CPU
// `attention` (src/encoder.rs:302-329): scores q.k * hd^-1/2 over the first
// `valid` keys, softmax, context = sum p v.  No S x S scores buffer exists.
//
// Arithmetic ("3xBF16"): Q, K, V^T and P are bfloat16 pairs x = hi + lo; each
// k-step issues lo*hi + hi*lo + hi*hi into an fp32 accumulator.  On the encoder
// this keeps the model's logits as close to the fp32 CPU path as 3xTF32 does
// (max |diff| 5e-8 either way, measured by emulation on the synthetic
// checkpoint), at half the tensor time and half the operand bytes, which lets
// two CTAs share an SM.
//
// CTA = 128 queries of one (sequence, head); 10 warps, two CTAs per SM:
//   warp 0      TMA: the Q pair once, then per block of 64 keys the K pair and
//               the V^T pair into a 2-stage ring
//   warp 1      TMEM owner; one thread issues S_j = Q K_j^T into TMEM buffer
//               j % 2 (block j+1's QK^T overlaps block j's softmax) and
//               O_j = P_j V_j with P_j read from TMEM, into O buffer j % 2
//   warps 2..9  softmax, two warps per query row (TMEM lane): each takes half of
//               the block's keys and half of the output columns; online max/sum;
//               P_j as bf16 pairs written over the S_j columns it read (QK_{j+2}
//               is issued once PV_j has completed); O folded into registers.
//               exp is 2^x on the special-function unit after one FMA folds the
//               1/sqrt(hd) scale, log2 e and the running max together; sums and the
//               O fold use packed f32x2 FMA/add.
// TMEM (256 columns): S/P[2] 0..127, O[2] 128..255.
// Every wait is bounded; an expired wait records its site in *err.

#include "n3d_device.cuh"
#include "n3d_internal.h"

namespace n3d {

namespace {

constexpr int HD = 64;                    // head dim
constexpr int QT = 128;                   // queries per CTA
constexpr int KB = 64;                    // keys per block
constexpr int Q_TILE = QT * 128;          // [128 rows x 64 bf16]: 16 KB (hi or lo)
constexpr int KV_TILE = KB * 128;         // [64 rows x 64 bf16]: 8 KB
constexpr int STAGE_BYTES = 4 * KV_TILE;  // K_hi, K_lo, V^T_hi, V^T_lo
constexpr int THREADS = 320;
constexpr int SMEM_BYTES = 2 * Q_TILE + 2 * STAGE_BYTES + 1024 + 256 + 6 * QT * 4;
constexpr uint32_t COL_S = 0, COL_O = 128, TMEM_COLS = 256;
constexpr int DEV_TIMEOUT_ATTN = 5;

// f32 pairs in one 64-bit register: Blackwell's packed FMA / add issue two lanes' worth
// of work per instruction.
__device__ __forceinline__ uint64_t pack2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void unpack2(uint64_t r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
// 2^x on the special-function unit (relative error ~2^-22; results below 2^-126 flush to 0).
__device__ __forceinline__ float ex2_approx(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

__global__ void __launch_bounds__(THREADS, 2)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tQh, const __grid_constant__ CUtensorMap tQl,
                        const __grid_constant__ CUtensorMap tKh, const __grid_constant__ CUtensorMap tKl,
                        const __grid_constant__ CUtensorMap tVh, const __grid_constant__ CUtensorMap tVl, int S,
                        const int* __restrict__ valid_arr, int heads, Split3Out ctx, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQh = smem;
    uint8_t* sQl = smem + Q_TILE;
    uint8_t* stages = smem + 2 * Q_TILE;
    uint64_t* bars = reinterpret_cast<uint64_t*>(stages + 2 * STAGE_BYTES);
    uint64_t* q_full = bars;        // 1
    uint64_t* kv_full = bars + 1;   // 2
    uint64_t* kv_empty = bars + 3;  // 2
    uint64_t* s_full = bars + 5;    // 2: QK_j committed
    uint64_t* p_full = bars + 7;    // 2: P_j in TMEM (8 warps)
    uint64_t* o_full = bars + 9;    // 2: PV_j committed
    uint64_t* o_free = bars + 11;   // 2: O_j folded (8 warps)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
    float* red_max = reinterpret_cast<float*>(bars + 32);  // [2 blocks][2 halves][QT]
    float* red_sum = red_max + 4 * QT;                      // [2 halves][QT]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * QT;
    const int valid = min(valid_arr[b], S);
    const int nblk = (valid + KB - 1) / KB;
    const int row0 = b * S;  // first row of this sequence in Q / K, first column in V^T

    if (warp == 0 && lane == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&kv_full[i], 1);
            mbar_init(&kv_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 8);
            mbar_init(&o_full[i], 1);
            mbar_init(&o_free[i], 8);
        }
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0 && nblk > 0) {
            mbar_arrive_expect_tx(q_full, 2 * Q_TILE);
            tma_load_2d(sQh, &tQh, q_full, h * HD, row0 + q0);
            tma_load_2d(sQl, &tQl, q_full, h * HD, row0 + q0);
            int issued = 0;
            for (int j = 0; j < nblk; j++) {
                const int st = j & 1;
                if (j >= 2 && !mbar_wait(&kv_empty[st], ((j >> 1) - 1) & 1, err, DEV_TIMEOUT_ATTN)) break;
                uint8_t* sb = stages + st * STAGE_BYTES;
                mbar_arrive_expect_tx(&kv_full[st], STAGE_BYTES);
                tma_load_2d(sb, &tKh, &kv_full[st], h * HD, row0 + j * KB);
                tma_load_2d(sb + KV_TILE, &tKl, &kv_full[st], h * HD, row0 + j * KB);
                tma_load_2d(sb + 2 * KV_TILE, &tVh, &kv_full[st], row0 + j * KB, h * HD);
                tma_load_2d(sb + 3 * KV_TILE, &tVl, &kv_full[st], row0 + j * KB, h * HD);
                issued = j + 1;
            }
            // the last loads of each stage have landed before the CTA may exit
            // (already true unless a wait above or in the MMA warp expired)
            mbar_wait(q_full, 0, err, DEV_TIMEOUT_ATTN);
            for (int j = max(0, issued - 2); j < issued; j++) mbar_wait(&kv_full[j & 1], (j >> 1) & 1, err, DEV_TIMEOUT_ATTN);
        }
    } else if (warp == 1) {
        if (lane == 0 && nblk > 0) {
            constexpr uint32_t idesc = idesc_bf16(64);
            bool ok = mbar_wait(q_full, 0, err, DEV_TIMEOUT_ATTN);
            const uint32_t qh = smem_u32(sQh), ql = smem_u32(sQl);
            auto issue_qk = [&](int j) {
                const uint32_t kb = smem_u32(stages + (j & 1) * STAGE_BYTES);
                const uint32_t d = tmem + COL_S + 64u * (j & 1);
#pragma unroll
                for (int k = 0; k < HD / 16; k++) {  // 16 bf16 = 32 bytes along the swizzled row
                    const uint32_t off = k * 32;
                    umma_bf16(d, desc_k_sw128(ql + off), desc_k_sw128(kb + off), idesc, k != 0);
                    umma_bf16(d, desc_k_sw128(qh + off), desc_k_sw128(kb + KV_TILE + off), idesc, 1);
                    umma_bf16(d, desc_k_sw128(qh + off), desc_k_sw128(kb + off), idesc, 1);
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
                    // S buffer (j+1)%2 holds P_{j-1}: MMAs into different accumulators are not
                    // ordered, so PV_{j-1} must have completed before QK_{j+1} overwrites it
                    ok = mbar_wait(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1, err, DEV_TIMEOUT_ATTN);
                    if (ok && j >= 1) ok = mbar_wait(&o_full[(j - 1) & 1], ((j - 1) >> 1) & 1, err, DEV_TIMEOUT_ATTN);
                    if (!ok) break;
                    tc_fence_after();
                    issue_qk(j + 1);
                }
                ok = mbar_wait(&p_full[j & 1], (j >> 1) & 1, err, DEV_TIMEOUT_ATTN);
                if (ok && j >= 2) ok = mbar_wait(&o_free[j & 1], ((j >> 1) - 1) & 1, err, DEV_TIMEOUT_ATTN);
                if (!ok) break;
                tc_fence_after();
                const uint32_t vb = smem_u32(stages + (j & 1) * STAGE_BYTES + 2 * KV_TILE);
                const uint32_t d = tmem + COL_O + 64u * (j & 1);
                const uint32_t pb = tmem + COL_S + 64u * (j & 1);
#pragma unroll
                for (int k = 0; k < KB / 16; k++) {
                    // keys 16k..16k+15 were written by softmax half k/2: P_hi at its
                    // columns 0..15, P_lo at 16..31 (8 columns per 16 keys)
                    const uint32_t ph = pb + 32 * (k >> 1) + 8 * (k & 1), pl = ph + 16;
                    const uint32_t off = k * 32;
                    umma_bf16_ts(d, pl, desc_k_sw128(vb + off), idesc, k != 0);
                    umma_bf16_ts(d, ph, desc_k_sw128(vb + KV_TILE + off), idesc, 1);
                    umma_bf16_ts(d, ph, desc_k_sw128(vb + off), idesc, 1);
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
        // exp(x) = 2^(x log2 e): p = 2^(s * k - m * k) with k = hd^-1/2 * log2 e, one FMA and
        // one ex2 per score; m is the running row maximum of the raw scores
        const float k2 = 0.125f * 1.4426950408889634f;
        uint64_t o[16];  // this warp's 32 output columns as f32 pairs
#pragma unroll
        for (int d = 0; d < 16; d++) o[d] = 0;
        float m = -INFINITY, l = 0.0f, c_prev = 0.0f;
        bool ok = true;
        auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory"); };
        auto fold = [&](int jj, float c) {  // O <- O * c + PV_jj, this warp's 32 columns
            float v[32];
            tmem_ld32(lb + COL_O + 64u * (jj & 1) + 32 * hf, v);
            const uint64_t c2 = pack2(c, c);
#pragma unroll
            for (int i = 0; i < 16; i++) o[i] = fma2(o[i], c2, pack2(v[2 * i], v[2 * i + 1]));
        };
        for (int j = 0; j < nblk; j++) {
            const int bf = j & 1;
            const uint32_t sp = lb + COL_S + 64u * bf + 32 * hf;  // this warp's S_j / P_j columns
            // after an expired wait the loop keeps running (work skipped, results unused)
            // so both warps of the pair reach every pair_sync
            ok = __all_sync(0xffffffffu, ok && mbar_wait(&s_full[bf], (j >> 1) & 1, err, DEV_TIMEOUT_ATTN));
            tc_fence_after();
            float s[32];
            tmem_ld32(sp, s);
            if (j * KB + 32 * hf + 32 > valid) {  // the block holding the last valid key
#pragma unroll
                for (int c = 0; c < 32; c++)
                    if (j * KB + 32 * hf + c >= valid) s[c] = -INFINITY;
            }
            float mloc = s[0];
#pragma unroll
            for (int c = 1; c < 32; c++) mloc = fmaxf(mloc, s[c]);
            red_max[(bf * 2 + hf) * QT + r] = mloc;
            pair_sync();
            // the row maximum is finite: key 0 is valid and the running max carries it
            const float mx = fmaxf(m, fmaxf(mloc, red_max[(bf * 2 + (hf ^ 1)) * QT + r]));
            const float corr = ex2_approx((m - mx) * k2);  // 0 on the first block (m = -inf)
            const uint64_t k22 = pack2(k2, k2), nmk = pack2(-mx * k2, -mx * k2);
            uint64_t sum2 = 0;
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
                float t0, t1;
                unpack2(fma2(pack2(s[c], s[c + 1]), k22, nmk), t0, t1);  // masked keys: -inf -> p = 0
                s[c] = ex2_approx(t0);
                s[c + 1] = ex2_approx(t1);
                sum2 = add2(sum2, pack2(s[c], s[c + 1]));
            }
            float sa, sb;
            unpack2(sum2, sa, sb);
            l = l * corr + (sa + sb);  // this half's partial row sum, at the common running max
            m = mx;
            {
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int i = 0; i < 16; i++) split_bf16x2(s[2 * i], s[2 * i + 1], hi[i], lo[i]);
                tmem_st16(sp, hi);
                tmem_st16(sp + 16, lo);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[bf]);
            if (j >= 1) {
                ok = __all_sync(0xffffffffu, ok && mbar_wait(&o_full[(j - 1) & 1], ((j - 1) >> 1) & 1, err,
                                                             DEV_TIMEOUT_ATTN));
                tc_fence_after();
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
        // ---- context row, this warp's 32 columns (3-term split, or plain fp32 when ctx.hb is null)
        if (q0 + r < S) {
            const float inv = ltot > 0.0f ? 1.0f / ltot : 0.0f;
            const long long off = (long long)(row0 + q0 + r) * (heads * HD) + h * HD + 32 * hf;
#pragma unroll
            for (int d = 0; d < 32; d += 4) {
                float x[4];
                unpack2(o[d / 2], x[0], x[1]);
                unpack2(o[d / 2 + 1], x[2], x[3]);
#pragma unroll
                for (int i = 0; i < 4; i++) x[i] *= inv;
                if (ctx.hb) {
                    float hh[4];
                    uint2 hb, lb;
                    split3x4(x, hh, hb, lb);
                    *reinterpret_cast<float4*>(ctx.hi + off + d) = make_float4(hh[0], hh[1], hh[2], hh[3]);
                    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(ctx.hb) + off + d) = hb;
                    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(ctx.lb) + off + d) = lb;
                } else {
                    *reinterpret_cast<float4*>(ctx.hi + off + d) = make_float4(x[0], x[1], x[2], x[3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace

void launch_attention_tc(cudaStream_t s, const AttnOperands& op, int seqs, int S, const int* valid, int heads,
                         Split3Out ctx, int* err) {
    if (seqs <= 0 || S <= 0) return;
    if ((seqs > 1 && S % 8) || op.vt_ld % 8)
        throw Error(9, "attention: the sequence stride and the V^T row stride must be multiples of 8");
    static bool attr = false;
    if (!attr) {
        N3D_CUDA(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        attr = true;
    }
    const long long W = (long long)heads * HD;
    const CUtensorMap qh = make_bf16_map(op.q_hi, op.rows_cap, W, W, 64, QT, true);
    const CUtensorMap ql = make_bf16_map(op.q_lo, op.rows_cap, W, W, 64, QT, true);
    const CUtensorMap kh = make_bf16_map(op.k_hi, op.rows_cap, W, W, 64, KB, true);
    const CUtensorMap kl = make_bf16_map(op.k_lo, op.rows_cap, W, W, 64, KB, true);
    const CUtensorMap vh = make_bf16_map(op.vt_hi, W, (long long)seqs * S, op.vt_ld, 64, HD, true);
    const CUtensorMap vl = make_bf16_map(op.vt_lo, W, (long long)seqs * S, op.vt_ld, 64, HD, true);
    dim3 grid((S + QT - 1) / QT, heads, seqs);
    attention_tc_kernel<<<grid, THREADS, SMEM_BYTES, s>>>(qh, ql, kh, kl, vh, vl, S, valid, heads, ctx, err);
    N3D_CUDA(cudaGetLastError());
}

}  // namespace n3d
