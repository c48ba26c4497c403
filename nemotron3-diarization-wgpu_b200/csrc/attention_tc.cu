// Softmax attention on the sm_100a tensor cores (tcgen05, kind::f16), head_dim 64
// (the model's) or 128 (BASELINE config 1's kernel sweep).
//
// Replaces the reference's three attention dispatches -- `gemm_strided` QK^T,
// `attn_sm` softmax with the key-padding mask, `gemm_n64` PV (src/gpu.rs:390-396,
// 1914-1971; src/gpu_engine.rs:162-211) -- and must agree with the CPU
// `attention` (src/encoder.rs:302-329): scores q.k * hd^-1/2 over the first
// `valid` keys, softmax, context = sum p v.  No S x S scores buffer exists.
//
// Arithmetic (the fp16 split, as the GEMMs): Q, K, V^T and P are each two fp16 arrays
// h + l of the values times a power-of-two scale; each k-step issues l*h + h*l + h*h
// into an fp32 accumulator, ~2^-22 per product, at the 16-bit tensor rate.  Q, K and
// V carry the scales the QKV epilogue gave them (from load-time bounds); P <= 2^8
// (the lazy rescale below) is kept as P * 2^7, the 7 added to its exponent.  The score
// scale 1/sqrt(hd) log2 e is divided by s_Q s_K, and the context by s_V (the row sum l
// carries P's 2^7), exactly (powers of two).
//
// Persistent CTAs: each resident CTA (two per SM at head_dim 64, one at 128) takes
// items blockIdx.x, + gridDim.x, ...; an item is 128 queries of one (sequence, head).
// Key blocks of 64 are numbered g across the CTA's items, and the rings and the S, P
// and O columns run on g.  6 warps; two threads issue the tensor-core work, so that
// neither waits for the other's MMAs:
//   warp 0      the next item's Q pair (TMA into the Q buffer) and the K pairs into a
//               2-stage K ring; issues S_g = Q K_g^T once the softmax has read S_{g-1}
//   warp 1      TMEM owner; the V^T pairs into a 2-stage V ring; issues O += P_g V_g
//               once the softmax has written P_g
//   warps 2..5  softmax, one thread per query row (TMEM lane): per block the row's 64
//               scores, exp as 2^x on the special-function unit after one FMA folds the
//               1/sqrt(hd) scale, log2 e and the reference max together; then, once
//               PV_{g-1} has read the P buffer, P_g as fp16 splits; after an item's last
//               block the next item's Q pair from the Q buffer into TMEM, then the
//               item's context.
// Both MMAs take their A operand (Q, P) from TMEM, so only K / V^T are read from
// shared memory.  QK_{g+1} computes while the softmax works on S_g and PV_{g-1}
// alongside it; the next item's first QK computes during the epilogue.  K_{g+2} loads
// once QK_g has completed, V_{g+2} once PV_g has.  (Writing P over S in two alternating
// buffers, so that the softmax need not wait for PV_{g-1}, measured slower: the QK
// issue then waits for PV completion instead.)
// Lazy rescaling: exponents use a per-row reference max m that is raised only when
// a block's max exceeds it by more than 2^8 in the exponent; only then is O
// (in TMEM) multiplied by the correction, after PV_{g-1} has completed and before
// P_g is released.  P values stay below 2^8; O / l is unchanged mathematically.
// Context rows leave through shared memory (the Q buffer, once the next Q has moved
// to TMEM) and TMA stores, a warp's 32 rows at a time.
// TMEM: S 0..63, P 64..127 (hi 64.., lo 96..), O 128..128+HD-1, Q 128+HD..128+2HD-1
// (h first, then l); 16-bit operands two per 32-bit column.  256 columns at head_dim
// 64, 512 at 128.  A K block [64 keys, HD] is HD/64 TMA boxes of 64 columns (the
// 128-byte swizzle's limit), as is the Q tile.
// Every waiter is at most one phase behind its barrier (argued at each wait).  Every
// wait is bounded; an expired wait records its site in *err.

#include <algorithm>
#include <climits>
#include <cmath>

#include "n3d_device.cuh"
#include "n3d_internal.h"

namespace n3d {

namespace {

constexpr int QT = 128;                   // queries per CTA
constexpr int KB = 64;                    // keys per block
constexpr int BOX = KB * 128;             // one 64-column TMA box of 64 rows: 8 KB
constexpr int THREADS = 192;
constexpr uint32_t COL_S = 0, COL_P = 64, COL_O = 128;
constexpr int DEV_TIMEOUT_ATTN = 5;

template <int HD>
struct AttnCfg {
    static_assert(HD == 64 || HD == 128, "head_dim 64 or 128");
    static constexpr int KTILE = KB * HD * 2;                  // K block [64 keys x HD] fp16
    static constexpr int VTILE = HD * KB * 2;                  // V^T block [HD x 64 keys] fp16
    static constexpr int KSTAGE = 2 * KTILE, VSTAGE = 2 * VTILE;  // hi + lo
    static constexpr int QBUF = 2 * QT * HD * 2;                  // the next item's Q pair, or the context staging
    static constexpr int RING_BYTES = 2 * KSTAGE + 2 * VSTAGE + QBUF;
    static constexpr int SMEM_BYTES = RING_BYTES + 1024 + 256;
    static constexpr uint32_t COL_Q = COL_O + HD, TMEM_COLS = HD == 64 ? 256 : 512;
    static constexpr int CTAS_PER_SM = HD == 64 ? 2 : 1;
    static_assert(4 * 32 * HD * 4 == QBUF, "the context staging of the 4 softmax warps fills the Q buffer");
};
constexpr float RESCALE_LOG2 = 8.0f;      // raise the reference max when exponents would exceed 2^8
constexpr float P_LOG2_SCALE = 7.0f;      // P <= 2^8 is kept as P * 2^7 <= 2^15, inside fp16's range

// Two scaled probabilities x = P * 2^7 in [0, 2^15] -> their fp16 split words (a in the
// low half).  h = x rounded to 11 significant bits; its fp16 bits are
// (bits(x) + 2^12 - (112 << 23)) >> 13 (rebias the exponent, drop 13 mantissa bits),
// formed as the high half of bits(x) * 8 + 0x40008000 (the same sum shifted left by 3,
// modulo 2^32; it stays below 2^29 before the shift for x in [2^-14, 2^15]), and one
// byte permute packs the two high halves.  x below fp16's normal range takes
// h = 2^-14 and a negative l.  Only l goes through the conversion pipe.
__device__ __forceinline__ void split_p2(float a, float b, uint32_t& h, uint32_t& l) {
    const uint32_t ba = __float_as_uint(fmaxf(a, 6.103515625e-05f)), bb = __float_as_uint(fmaxf(b, 6.103515625e-05f));
    h = __byte_perm(ba * 8u + 0x40008000u, bb * 8u + 0x40008000u, 0x7632);
    const uint32_t ua = (ba + 0x1000u) & 0xffffe000u, ub = (bb + 0x1000u) & 0xffffe000u;
    uint64_t d;  // (a, b) - (h_a, h_b), both lanes rounded to nearest (exact here)
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pack2(a, b)), "l"(pack2(__uint_as_float(ua), __uint_as_float(ub))));
    float la, lb;
    unpack2(d, la, lb);
    l = f16x2_rn(la, lb);
}

// max(a, b, c) in one instruction
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// 64 consecutive TMEM columns of this thread's lane: two loads, one wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
    uint32_t r[64];
#pragma unroll
    for (int h = 0; h < 2; h++)
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
            "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(r[32 * h + 0]), "=r"(r[32 * h + 1]), "=r"(r[32 * h + 2]), "=r"(r[32 * h + 3]),
              "=r"(r[32 * h + 4]), "=r"(r[32 * h + 5]), "=r"(r[32 * h + 6]), "=r"(r[32 * h + 7]),
              "=r"(r[32 * h + 8]), "=r"(r[32 * h + 9]), "=r"(r[32 * h + 10]), "=r"(r[32 * h + 11]),
              "=r"(r[32 * h + 12]), "=r"(r[32 * h + 13]), "=r"(r[32 * h + 14]), "=r"(r[32 * h + 15]),
              "=r"(r[32 * h + 16]), "=r"(r[32 * h + 17]), "=r"(r[32 * h + 18]), "=r"(r[32 * h + 19]),
              "=r"(r[32 * h + 20]), "=r"(r[32 * h + 21]), "=r"(r[32 * h + 22]), "=r"(r[32 * h + 23]),
              "=r"(r[32 * h + 24]), "=r"(r[32 * h + 25]), "=r"(r[32 * h + 26]), "=r"(r[32 * h + 27]),
              "=r"(r[32 * h + 28]), "=r"(r[32 * h + 29]), "=r"(r[32 * h + 30]), "=r"(r[32 * h + 31])
            : "r"(taddr + 32 * h));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    reg_fence32(r);
    reg_fence32(r + 32);
#pragma unroll
    for (int i = 0; i < 64; i++) v[i] = __uint_as_float(r[i]);
}
// 32 consecutive TMEM columns from 32-bit words; completes with tmem_wait_st().
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

struct AttnMaps {
    CUtensorMap qh, ql;      // Q split [rows, heads*hd] fp16, box 64 x 128, 128-byte swizzle
    CUtensorMap kh, kl;      // K split, box 64 x 64
    CUtensorMap vh, vl;      // V^T split [heads*hd, rows], box 64 x hd
    CUtensorMap ch, cl;      // context fp16 split h / l [rows, heads*64], box 64 x 32, 128-byte swizzle
};

template <int HD>
__global__ void __launch_bounds__(THREADS, AttnCfg<HD>::CTAS_PER_SM)
    attention_tc_kernel(const __grid_constant__ AttnMaps maps, int S, const int* __restrict__ valid_arr, int heads,
                        int qblocks, int items, SplitOut ctx, int ctx_tma, float k2, float out_unscale, int* err) {
    using Cfg = AttnCfg<HD>;
    constexpr int KTILE = Cfg::KTILE, VTILE = Cfg::VTILE, KSTAGE = Cfg::KSTAGE, VSTAGE = Cfg::VSTAGE;
    constexpr uint32_t COL_Q = Cfg::COL_Q, TMEM_COLS = Cfg::TMEM_COLS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* kring = smem;                             // K pair of block g in stage g % 2
    uint8_t* vring = smem + 2 * KSTAGE;                // V^T pair of block g in stage g % 2
    uint8_t* qbuf = smem + 2 * KSTAGE + 2 * VSTAGE;    // Q hi [HD/64 boxes of 128 rows x 128 B], then Q lo
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::RING_BYTES);
    uint64_t* q_full = bars;        // 1: phase k = item k's Q pair landed in the Q buffer
    uint64_t* q_ready = bars + 1;   // 1: phase k = item k's Q pair in TMEM, Q buffer free (4 warps)
    uint64_t* k_full = bars + 2;    // 2: K_g landed (stage g % 2)
    uint64_t* k_empty = bars + 4;   // 2: QK_g completed
    uint64_t* v_full = bars + 6;    // 2: V_g landed
    uint64_t* v_empty = bars + 8;   // 2: PV_g completed
    uint64_t* s_full = bars + 10;   // 1: phase g = QK_g completed
    uint64_t* s_free = bars + 11;   // 1: phase g = S_g read by the softmax (4 warps)
    uint64_t* p_full = bars + 12;   // 1: phase g = P_g in TMEM, any rescale of O done (4 warps)
    uint64_t* o_full = bars + 13;   // 1: phase g = PV_g completed
    uint64_t* ctx_done = bars + 14; // 1: phase k = item k's context has left the Q buffer (4 warps)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == 0 && lane == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_ready, 4);
        for (int i = 0; i < 2; i++) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 4);
        mbar_init(p_full, 4);
        mbar_init(o_full, 1);
        mbar_init(ctx_done, 4);
        mbar_fence_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    griddep_wait();  // Q / K / V^T and the key counts written by earlier kernels
    griddep_launch_dependents();
    // The two CTAs that share an SM (the scheduler fills the second slot with the upper
    // half of the grid) would otherwise start in step and stay there: both in softmax
    // while the tensor pipe idles, then both issuing MMAs.  Starting the second one
    // ~1.6 us late (about a key block) staggers them: +2 % attention throughput measured
    // at C4's shapes on one box, results unchanged.
    if (Cfg::CTAS_PER_SM == 2 && blockIdx.x >= gridDim.x / 2) __nanosleep(1600);

    // This CTA's items: blockIdx.x + k * gridDim.x, k = 0.. ; item = (b * heads + h) *
    // qblocks + qb covers queries qb*128.. of head h of sequence b, and its key blocks
    // are numbered g = 0, 1, ... across the CTA's items (the rings, S, P and O run on g)
    const int n_items = items > (int)blockIdx.x ? (items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    struct Item {
        int qb, h, b, valid, nblk;
    };
    auto item = [&](int k) {
        const int it = (int)blockIdx.x + k * (int)gridDim.x, t = it / qblocks;
        Item r;
        r.qb = it - t * qblocks;
        r.h = t % heads;
        r.b = t / heads;
        r.valid = min(valid_arr[r.b], S);
        r.nblk = (r.valid + KB - 1) / KB;
        return r;
    };
    // the next key block a ring loads: item ck, block cj of sequence cb, head ch (items
    // without keys skipped; ck = n_items once every block is loaded)
    auto settle = [&](int& ck, int& cj, int& cb, int& ch) {
        for (; ck < n_items; ck++, cj = 0) {
            const Item it = item(ck);
            cb = it.b;
            ch = it.h;
            if (cj < it.nblk) break;
        }
    };

    if (warp == 0) {
        // ---- Q and K loads, S_g = Q K_g^T
        if (lane == 0 && n_items > 0) {
            auto load_q = [&](int k) {
                const Item it = item(k);
                // Q rows past S belong to the next sequence (or lie past the buffer:
                // zeros); their context is never stored
                mbar_arrive_expect_tx(q_full, Cfg::QBUF);
#pragma unroll
                for (int i = 0; i < HD / 64; i++) {
                    const int x = it.h * HD + 64 * i, y = it.b * S + it.qb * QT;
                    tma_load_2d(qbuf + i * QT * 128, &maps.qh, q_full, x, y);
                    tma_load_2d(qbuf + QT * HD * 2 + i * QT * 128, &maps.ql, q_full, x, y);
                }
            };
            int kk_ = 0, kj = 0, kb_ = 0, kh = 0;
            settle(kk_, kj, kb_, kh);
            int gk = 0;  // K blocks issued
            auto load_k = [&] {
                uint8_t* sb = kring + (gk & 1) * KSTAGE;
                uint64_t* bar = &k_full[gk & 1];
                mbar_arrive_expect_tx(bar, KSTAGE);
#pragma unroll
                for (int i = 0; i < HD / 64; i++) {
                    const int x = kh * HD + 64 * i, y = kb_ * S + kj * KB;
                    tma_load_2d(sb + i * BOX, &maps.kh, bar, x, y);
                    tma_load_2d(sb + KTILE + i * BOX, &maps.kl, bar, x, y);
                }
                gk++;
                kj++;
                settle(kk_, kj, kb_, kh);
            };
            load_q(0);
            int q_loaded = 1;
            for (int t = 0; t < 2 && kk_ < n_items; t++) load_k();
            constexpr uint32_t idesc_qk = idesc_f16(KB);
            bool ok = true;
            int g = 0;  // QK blocks issued
            for (int k = 0; ok && k < n_items; k++) {
                // item k's Q in TMEM (q_ready phase k: phase k+1 needs Q_{k+1}, loaded below)
                ok = mbar_wait(q_ready, k & 1, err, DEV_TIMEOUT_ATTN);
                if (!ok) break;
                tc_fence_after();
                // the next item's Q goes into the Q buffer once item k-1's context has left
                // it (ctx_done phase k-1: phase k needs this item's P, hence its QKs, or, for
                // an item without keys, the Q loaded here).  Done after this item's first
                // QK, which then computes during item k-1's epilogue.
                auto load_next_q = [&] {
                    if (k + 1 < n_items) {
                        if (k >= 1) ok = mbar_wait(ctx_done, (k - 1) & 1, err, DEV_TIMEOUT_ATTN);
                        if (ok) {
                            load_q(k + 1);
                            q_loaded = k + 2;
                        }
                    }
                };
                const int nblk = item(k).nblk;
                if (nblk == 0) load_next_q();
                for (int j = 0; ok && j < nblk; j++, g++) {
                    if (g > 0) {
                        // S_{g-1} read (s_free phase g-1: phase g needs QK_g, issued below)
                        ok = mbar_wait(s_free, (g - 1) & 1, err, DEV_TIMEOUT_ATTN);
                        if (!ok) break;
                    }
                    if (gk == g + 1 && kk_ < n_items) {
                        // K_{g+1}: its stage frees when QK_{g-1} completes (k_empty phase
                        // (g-1)/2; implied by s_free, and K_{g+1} is not issued yet)
                        ok = mbar_wait(&k_empty[(g - 1) & 1], ((g - 1) >> 1) & 1, err, DEV_TIMEOUT_ATTN);
                        if (!ok) break;
                        load_k();
                    }
                    // K_g landed (k_full phase g/2: K_{g+2} waits for this QK)
                    ok = mbar_wait(&k_full[g & 1], (g >> 1) & 1, err, DEV_TIMEOUT_ATTN);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t kb = smem_u32(kring + (g & 1) * KSTAGE);
#pragma unroll
                    for (int kk = 0; kk < HD / 16; kk++) {  // d 16kk..: Q_hi at column 8kk, Q_lo at HD/2 + 8kk
                        // 16 fp16 = 32 bytes along the swizzled K rows, in box kk / 4
                        const uint32_t off = (kk / 4) * BOX + (kk % 4) * 32;
                        const uint32_t qh = tmem + COL_Q + 8 * kk, ql = qh + HD / 2;
                        umma_f16_ts(tmem + COL_S, ql, desc_k_sw128(kb + off), idesc_qk, kk != 0);
                        umma_f16_ts(tmem + COL_S, qh, desc_k_sw128(kb + KTILE + off), idesc_qk, 1);
                        umma_f16_ts(tmem + COL_S, qh, desc_k_sw128(kb + off), idesc_qk, 1);
                    }
                    umma_commit(s_full);
                    umma_commit(&k_empty[g & 1]);
                    if (j == 0) load_next_q();
                }
            }
            // every load has landed before the CTA may exit (already true unless a wait
            // here or elsewhere expired)
            mbar_wait(q_full, (q_loaded - 1) & 1, err, DEV_TIMEOUT_ATTN);
            for (int x = max(0, gk - 2); x < gk; x++) mbar_wait(&k_full[x & 1], (x >> 1) & 1, err, DEV_TIMEOUT_ATTN);
        }
    } else if (warp == 1) {
        // ---- V loads, O += P_g V_g
        if (lane == 0 && n_items > 0) {
            int vk = 0, vj = 0, vb_ = 0, vh = 0;
            settle(vk, vj, vb_, vh);
            int gv = 0;  // V blocks issued
            auto load_v = [&] {
                uint8_t* sb = vring + (gv & 1) * VSTAGE;
                uint64_t* bar = &v_full[gv & 1];
                mbar_arrive_expect_tx(bar, VSTAGE);
                const int x = vb_ * S + vj * KB, y = vh * HD;
                tma_load_2d(sb, &maps.vh, bar, x, y);
                tma_load_2d(sb + VTILE, &maps.vl, bar, x, y);
                gv++;
                vj++;
                settle(vk, vj, vb_, vh);
            };
            for (int t = 0; t < 2 && vk < n_items; t++) load_v();
            constexpr uint32_t idesc_pv = idesc_f16(HD);
            bool ok = true;
            int g = 0;  // PV blocks issued
            for (int k = 0; ok && k < n_items; k++) {
                const int nblk = item(k).nblk;
                for (int j = 0; ok && j < nblk; j++, g++) {
                    // P_g (p_full phase g: phase g+1 needs PV_g) and V_g (v_full phase g/2)
                    ok = mbar_wait(p_full, g & 1, err, DEV_TIMEOUT_ATTN) &&
                         mbar_wait(&v_full[g & 1], (g >> 1) & 1, err, DEV_TIMEOUT_ATTN);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t vb = smem_u32(vring + (g & 1) * VSTAGE);
                    const uint32_t pb = tmem + COL_P;
#pragma unroll
                    for (int kk = 0; kk < KB / 16; kk++) {  // keys 16kk..: P_hi at column 8kk, P_lo at 32 + 8kk
                        const uint32_t off = kk * 32;
                        // the item's first PV starts O afresh
                        umma_f16_ts(tmem + COL_O, pb + 32 + 8 * kk, desc_k_sw128(vb + off), idesc_pv, j > 0 || kk != 0);
                        umma_f16_ts(tmem + COL_O, pb + 8 * kk, desc_k_sw128(vb + VTILE + off), idesc_pv, 1);
                        umma_f16_ts(tmem + COL_O, pb + 8 * kk, desc_k_sw128(vb + off), idesc_pv, 1);
                    }
                    umma_commit(o_full);
                    umma_commit(&v_empty[g & 1]);
                    if (gv == g + 1 && vk < n_items) {
                        // V_{g+1}: its stage frees when PV_{g-1} completes (v_empty phase
                        // (g-1)/2: issued a block ago; V_{g+1} is not issued yet)
                        ok = mbar_wait(&v_empty[(g - 1) & 1], ((g - 1) >> 1) & 1, err, DEV_TIMEOUT_ATTN);
                        if (!ok) break;
                        load_v();
                    }
                }
            }
            for (int x = max(0, gv - 2); x < gv; x++) mbar_wait(&v_full[x & 1], (x >> 1) & 1, err, DEV_TIMEOUT_ATTN);
        }
    } else {
        // ---- softmax warps 2..5: warp w owns TMEM lane quadrant w % 4; thread = query row
        const int qd = warp & 3;
        const int r = qd * 32 + lane;
        const uint32_t lb = tmem + (static_cast<uint32_t>(qd * 32) << 16);
        bool ok = true;
        // item k's Q split (HD fp16 each, RoPE applied) from the Q buffer (boxes of
        // 128-byte rows, 16-byte chunk c at c ^ (row % 8)) into TMEM columns COL_Q..
        auto copy_q = [&](int k) {
            ok = __all_sync(0xffffffffu, ok && mbar_wait(q_full, k & 1, err, DEV_TIMEOUT_ATTN));
#pragma unroll
            for (int part = 0; part < 2; part++) {  // hi, then lo
#pragma unroll
                for (int box = 0; box < HD / 64; box++) {
                    uint32_t qw[32];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const int o = part * QT * HD * 2 + box * QT * 128 + r * 128 + ((i ^ (r & 7)) << 4);
                        const uint4 a = *reinterpret_cast<const uint4*>(qbuf + o);
                        qw[4 * i] = a.x, qw[4 * i + 1] = a.y, qw[4 * i + 2] = a.z, qw[4 * i + 3] = a.w;
                    }
                    tmem_st32u(lb + COL_Q + part * (HD / 2) + 32 * box, qw);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(q_ready);
        };
        if (n_items > 0) copy_q(0);
        int g = 0;  // key blocks done
        for (int k = 0; k < n_items; k++) {
            int valid, nblk;
            {
                const Item it = item(k);
                valid = it.valid;
                nblk = it.nblk;
            }
            // the next item's Q moves into TMEM once this item's last QK has completed
            // (after its last block; at once for an item without keys: every earlier QK has)
            if (nblk == 0 && k + 1 < n_items) copy_q(k + 1);
            // k2 = hd^-1/2 log2 e / (s_Q s_K): p = 2^(s k2 - m k2) for raw accumulator scores s
            float m = -INFINITY, l = 0.0f;  // reference max (raw score units), row sum
            for (int j = 0; j < nblk; j++, g++) {
                // S_g (s_full phase g: QK_{g+1} waits for this block's s_free).  After an
                // expired wait the loop keeps running (work skipped, results unused).
                ok = __all_sync(0xffffffffu, ok && mbar_wait(s_full, g & 1, err, DEV_TIMEOUT_ATTN));
                tc_fence_after();
                float s[64];
                tmem_ld64(lb + COL_S, s);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(s_free);  // QK_{g+1} may now overwrite S_g
                if (j * KB + KB > valid) {  // the block holding the last valid key
#pragma unroll
                    for (int c = 0; c < 64; c++)
                        if (j * KB + c >= valid) s[c] = -INFINITY;
                }
                // block max by three-input maxima: 64 -> 22 -> 8 -> 3 -> 1 (31 instructions)
                float m22[22];
#pragma unroll
                for (int c = 0; c < 21; c++) m22[c] = max3f(s[c], s[c + 21], s[c + 42]);
                m22[21] = s[63];
                float m8[8];
#pragma unroll
                for (int c = 0; c < 7; c++) m8[c] = max3f(m22[c], m22[c + 7], m22[c + 14]);
                m8[7] = m22[21];
                const float mb = max3f(max3f(m8[0], m8[1], m8[2]), max3f(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
                // (finite: the block has a valid key)
                const bool raise = (mb - m) * k2 > RESCALE_LOG2;              // always on the first block (m = -inf)
                const float corr = raise ? ex2_approx((m - mb) * k2) : 1.0f;  // 0 on the first block
                if (raise) m = mb;
                // exponents carry the 2^7 scale of P: s = 2^(t + 7) = P * 2^7, and l sums those
                const float off = P_LOG2_SCALE - m * k2;
                const uint64_t k22 = pack2(k2, k2), nmk = pack2(off, off);
                uint64_t sum2[4] = {0, 0, 0, 0};  // four independent packed partial sums
#pragma unroll
                for (int c = 0; c < 64; c += 2) {
                    float t0, t1;
                    unpack2(fma2(pack2(s[c], s[c + 1]), k22, nmk), t0, t1);  // masked keys: -inf -> p = 0
                    s[c] = ex2_approx(t0);
                    s[c + 1] = ex2_approx(t1);
                    sum2[(c >> 1) & 3] = add2(sum2[(c >> 1) & 3], pack2(s[c], s[c + 1]));
                }
                float sa, sb;
                unpack2(add2(add2(sum2[0], sum2[1]), add2(sum2[2], sum2[3])), sa, sb);
                l = l * corr + (sa + sb);
                uint32_t hi[32], lo[32];
#pragma unroll
                for (int i = 0; i < 32; i++) split_p2(s[2 * i], s[2 * i + 1], hi[i], lo[i]);
                if (j > 0) {
                    // PV_{g-1} has read the P buffer and finished O up to block j-1 (o_full
                    // phase g-1: this loop waited for phase g-2 a block ago, and PV_g needs P_g)
                    ok = __all_sync(0xffffffffu, ok && mbar_wait(o_full, (g - 1) & 1, err, DEV_TIMEOUT_ATTN));
                    tc_fence_after();
                }
                if (j > 0 && __any_sync(0xffffffffu, raise)) {  // bring O to the new reference max
                    const uint64_t c2 = pack2(corr, corr);
#pragma unroll 1
                    for (int cb = 0; cb < HD; cb += 32) {  // 32 columns at a time, not unrolled: hi / lo stay live
                        float o[32];
                        tmem_ld32(lb + COL_O + cb, o);
#pragma unroll
                        for (int d = 0; d < 32; d += 2) {
                            uint64_t t = fma2(pack2(o[d], o[d + 1]), c2, 0);
                            unpack2(t, o[d], o[d + 1]);
                        }
                        tmem_st32(lb + COL_O + cb, o);
                    }
                }
                tmem_st32u(lb + COL_P, hi);
                tmem_st32u(lb + COL_P + 32, lo);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(p_full);
                // the item's last QK has completed (S_g was read): the next item's Q may
                // take its TMEM columns, and its first QK computes during this epilogue
                if (j == nblk - 1 && k + 1 < n_items) copy_q(k + 1);
            }
            if (nblk > 0) {
                // the item's last PV (o_full phase g-1; phase g-2 was waited for above, or
                // at the end of the previous item)
                ok = __all_sync(0xffffffffu, ok && mbar_wait(o_full, (g - 1) & 1, err, DEV_TIMEOUT_ATTN));
                tc_fence_after();
            }
            // ---- context rows, 64 columns at a time: the fp16 split through TMA stores when
            // all 32 rows of the warp belong to this sequence; otherwise (and for a plain
            // fp32 context) per row
            const Item it = item(k);  // recomputed: fewer registers live across the key loop
            const int q0 = it.qb * QT, row0 = it.b * S, wrow0 = q0 + qd * 32;
            // 1 / l, and O's scales undone (a power of two: exact)
            const float inv = (nblk > 0 && l > 0.0f) ? (1.0f / l) * out_unscale : 0.0f;
            const bool via_tma = ctx_tma && wrow0 + 32 <= S;
            // staging in the Q buffer, once every warp has copied the next item's Q out of
            // it (q_ready phase k+1: phase k+2 needs Q_{k+2}, loaded after ctx_done of this
            // item): per warp HD/64 pairs of 4 KB boxes (h, l), 128-byte rows of 64 fp16
            if (via_tma && k + 1 < n_items)
                ok = __all_sync(0xffffffffu, ok && mbar_wait(q_ready, (k + 1) & 1, err, DEV_TIMEOUT_ATTN));
            uint8_t* stg = qbuf + (warp - 2) * (HD * 128);
#pragma unroll 1
            for (int cb = 0; cb < HD; cb += 32) {  // 32 columns: half a 128-byte staging row (not unrolled: registers)
                float o[32];
                if (nblk > 0) tmem_ld32(lb + COL_O + cb, o);
                if (via_tma) {
                    uint32_t hw[16], lw[16];
#pragma unroll
                    for (int d = 0; d < 32; d += 2) {
                        const float x0 = nblk > 0 ? o[d] * inv : 0.0f, x1 = nblk > 0 ? o[d + 1] * inv : 0.0f;
                        split2x2(x0, x1, ctx.scale, hw[d / 2], lw[d / 2]);
                    }
                    uint8_t* bx = stg + (cb / 64) * 8192;
                    const int c0 = (cb % 64) / 8;  // first 16-byte chunk of the row
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int sw = (((c0 + i) ^ (lane & 7)) << 4) + lane * 128;
                        *reinterpret_cast<uint4*>(bx + sw) =
                            make_uint4(hw[4 * i], hw[4 * i + 1], hw[4 * i + 2], hw[4 * i + 3]);
                        *reinterpret_cast<uint4*>(bx + 4096 + sw) =
                            make_uint4(lw[4 * i], lw[4 * i + 1], lw[4 * i + 2], lw[4 * i + 3]);
                    }
                } else if (q0 + r < S) {
                    const long long off = (long long)(row0 + q0 + r) * (heads * HD) + it.h * HD + cb;
#pragma unroll
                    for (int d = 0; d < 32; d += 4) {
                        float x[4];
#pragma unroll
                        for (int i = 0; i < 4; i++) x[i] = nblk > 0 ? o[d + i] * inv : 0.0f;
                        if (ctx.h) {
                            uint2 hw, lw;
                            split2x4(x, ctx.scale, hw, lw);
                            *reinterpret_cast<uint2*>(static_cast<uint16_t*>(ctx.h) + off + d) = hw;
                            *reinterpret_cast<uint2*>(static_cast<uint16_t*>(ctx.l) + off + d) = lw;
                        } else {
                            *reinterpret_cast<float4*>(ctx.plain + off + d) = make_float4(x[0], x[1], x[2], x[3]);
                        }
                    }
                }
            }
            if (via_tma) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    const int y = row0 + wrow0;
#pragma unroll
                    for (int cb = 0; cb < HD; cb += 64) {
                        tma_store_2d(&maps.ch, stg + (cb / 64) * 8192, it.h * HD + cb, y);
                        tma_store_2d(&maps.cl, stg + (cb / 64) * 8192 + 4096, it.h * HD + cb, y);
                    }
                    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // staging read
                }
            }
            // O is read (the next item's first PV may overwrite it once P is released) and
            // the staging is free for the item after next's Q
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(ctx_done);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

template <int HD>
void launch_attention_hd(cudaStream_t s, const AttnOperands& op, int seqs, int S, const int* valid, int heads,
                         SplitOut ctx, int* err) {
    using Cfg = AttnCfg<HD>;
    static std::atomic<unsigned long long> attr{0};
    once_per_device(attr, [] {
        N3D_CUDA(cudaFuncSetAttribute(attention_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      Cfg::SMEM_BYTES));
    });
    const long long W = (long long)heads * HD, rows = (long long)seqs * S;
    AttnMaps m;
    m.qh = make_f16_map(op.q_h, op.rows_cap, W, W, 64, QT, true);
    m.ql = make_f16_map(op.q_l, op.rows_cap, W, W, 64, QT, true);
    m.kh = make_f16_map(op.k_h, op.rows_cap, W, W, 64, KB, true);
    m.kl = make_f16_map(op.k_l, op.rows_cap, W, W, 64, KB, true);
    m.vh = make_f16_map(op.vt_h, W, rows, op.vt_ld, 64, HD, true);
    m.vl = make_f16_map(op.vt_l, W, rows, op.vt_ld, 64, HD, true);
    const int ctx_tma = ctx.h != nullptr;
    if (ctx_tma) {
        m.ch = make_f16_map(ctx.h, rows, W, W, 64, 32, true);
        m.cl = make_f16_map(ctx.l, rows, W, W, 64, 32, true);
    } else {
        m.ch = m.cl = m.qh;  // unused
    }
    // persistent CTAs: every resident slot takes items blockIdx.x, + gridDim.x, ...
    const int qblocks = (S + QT - 1) / QT;
    const long long items = (long long)qblocks * heads * seqs;
    if (items > INT_MAX) throw Error(9, "attention: more than 2^31 query blocks");
    const int grid = (int)std::min<long long>(items, (long long)Cfg::CTAS_PER_SM * sm_count());
    const float k2 = (float)((1.0 / std::sqrt((double)HD)) * 1.4426950408889634 / ((double)op.q_scale * op.k_scale));
    const float out_unscale = (float)(1.0 / (double)op.v_scale);  // l already carries P's 2^7
    launch_pdl(attention_tc_kernel<HD>, dim3(grid), dim3(THREADS), Cfg::SMEM_BYTES, s, m, S, valid, heads, qblocks,
               (int)items, ctx, ctx_tma, k2, out_unscale, err);
}

}  // namespace

void launch_attention_tc(cudaStream_t s, const AttnOperands& op, int seqs, int S, const int* valid, int heads, int hd,
                         SplitOut ctx, int* err) {
    if (seqs <= 0 || S <= 0) return;
    if ((seqs > 1 && S % 8) || op.vt_ld % 8)
        throw Error(9, "attention: the sequence stride and the V^T row stride must be multiples of 8");
    if (hd == 64)
        launch_attention_hd<64>(s, op, seqs, S, valid, heads, ctx, err);
    else if (hd == 128)
        launch_attention_hd<128>(s, op, seqs, S, valid, heads, ctx, err);
    else
        throw Error(13, "attention: head_dim must be 64 or 128");
}

}  // namespace n3d
