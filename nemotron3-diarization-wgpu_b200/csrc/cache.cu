// Device-resident speaker cache (AOSC + FIFO) and encoder-window assembly.
//
// Replaces the reference's CPU `SpeakerCache` (src/streaming.rs:130-482) and the
// host-side window concatenation of `Model::step` (src/model.rs:383-391,
// 444-461).  All bookkeeping counts (cache/FIFO sizes, pops, whether a step
// compresses) depend only on the chunk schedule, never on data, so the host
// precomputes them per step and these kernels only move and rank data.
//
// Per sequence, the state carried between steps is its *prefix*: the rows
// `[cache ++ fifo]` that open the next window, plus the probabilities stored
// with a compressed cache.  Both live in ping-pong buffers.

#include <cmath>

#include "n3d_device.cuh"
#include "n3d_internal.h"
#include "n3d_cache.h"

namespace n3d {

namespace {

constexpr float kLn2 = 0.69314718055994531f;

// Rust `f32::ln` / `f32::exp` call the platform libm; evaluating in double and
// rounding once lands on the correctly rounded float, which is what that libm
// returns for these arguments.
__device__ __forceinline__ float ln_f(float x) { return (float)log((double)x); }
__device__ __forceinline__ float exp_f(float x) { return (float)exp((double)x); }

// window row t of sequence i: prefix rows from the previous step, then this
// step's new embeddings, then zeros up to the batch stride.
__global__ void assemble_kernel(const SeqStep* __restrict__ steps, const float* __restrict__ embeds,
                                float* __restrict__ win, int stride, int hidden) {
    griddep_wait();
    griddep_launch_dependents();
    const int i = blockIdx.y, t = blockIdx.x;
    const SeqStep st = steps[i];
    const int prefix = st.ncache + st.nfifo;
    const float4* src = nullptr;
    if (t < prefix)
        src = reinterpret_cast<const float4*>(st.pre_in + (long long)t * hidden);
    else if (t < st.S)
        src = reinterpret_cast<const float4*>(embeds + (st.emb_row + t - prefix) * hidden);
    float4* dst = reinterpret_cast<float4*>(win + ((long long)i * stride + t) * hidden);
    for (int c = threadIdx.x; c < hidden / 4; c += blockDim.x) dst[c] = src ? src[c] : make_float4(0.f, 0.f, 0.f, 0.f);
}

// Order-preserving unsigned image of a float: a > b iff key(a) > key(b) (-inf lowest,
// +inf highest; the scores here are never NaN).  -0 and +0 compare equal in the
// reference's sort, so -0 is first mapped to +0 (adding +0 in round-to-nearest).
__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t u = __float_as_uint(__fadd_rn(v, 0.0f));
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// _compress's ranking (src/streaming.rs:410-463) of `ne` candidate frames whose
// probabilities are cand[ne * ns]: frame scores (into sc), the latest-frames boost,
// the strong and weak per-speaker top-k boosts, then the flat speaker-major pick of
// the first L = min(cache_len, ns * (ne + n_sil)) in (score desc, flat index asc)
// order.  Leaves the picked flat indices ascending in idx[0, n_real) -- the -inf
// picks are dropped, they become the sentinel -- and returns n_real in every thread,
// with L in *L_out.  Every thread of the block calls it (it synchronises).
// "The first k in (score descending, index ascending) order" -- Rust's stable sort
// followed by a truncation -- is computed as a selection: an MSB-first radix select
// of the k-th key, then the elements above it plus the lowest-index ties.
__device__ int compress_select(const float* __restrict__ cand, float* __restrict__ sc, uint32_t* __restrict__ fkey,
                               int* __restrict__ idx, int* __restrict__ aux, int ne, const CacheConst& cp,
                               int* L_out) {
    const int ns = cp.ns;
    const int tid = threadIdx.x, nt = blockDim.x;
    // ---- _get_frame_scores (src/streaming.rs:294-330)
    for (int f = tid; f < ne; f += nt) {
        const float* row = cand + f * ns;
        float lp[16], lc[16];
        float sum_lc = 0.0f;
        for (int s = 0; s < ns; s++) {
            lp[s] = ln_f(fmaxf(row[s], cp.thr));
            lc[s] = ln_f(fmaxf(__fsub_rn(1.0f, row[s]), cp.thr));
        }
        for (int s = 0; s < ns; s++) sum_lc = __fadd_rn(sum_lc, lc[s]);
        for (int s = 0; s < ns; s++) {
            const float v = __fadd_rn(__fadd_rn(__fsub_rn(lp[s], lc[s]), sum_lc), kLn2);
            sc[f * ns + s] = row[s] > 0.5f ? v : -INFINITY;
        }
    }
    if (tid < ns) aux[tid] = 0;
    __syncthreads();
    for (int e = tid; e < ne * ns; e += nt)
        if (sc[e] > 0.0f) atomicAdd(&aux[e % ns], 1);
    __syncthreads();
    for (int e = tid; e < ne * ns; e += nt) {
        const int s = e % ns;
        if (aux[s] >= cp.min_pos && sc[e] <= 0.0f && cand[e] > 0.5f) sc[e] = -INFINITY;
    }
    __syncthreads();
    // ---- latest-frames boost: frames past the cache capacity were just popped
    for (int e = tid; e < ne * ns; e += nt)
        if (e / ns >= cp.cache_len) sc[e] = __fadd_rn(sc[e], cp.latest_boost);
    __syncthreads();
    // ---- _boost_scores twice (src/streaming.rs:333-346): per speaker, the k best frames
    // (one warp per speaker selects them)
    const int warp = tid >> 5, lane = tid & 31, nwarps = nt >> 5;
    for (int pass = 0; pass < 2; pass++) {
        const int kk = min(pass == 0 ? cp.k_strong : cp.k_weak, ne);
        const float boost = pass == 0 ? 2.0f * kLn2 : kLn2;
        for (int s = warp; s < ns; s += nwarps) {
            uint32_t prefix = 0, mask = 0;
            int need = kk;
            for (int bit = 31; kk > 0 && bit >= 0; bit--) {
                const uint32_t b = 1u << bit;
                int c = 0;
                for (int f0 = 0; f0 < ne; f0 += 32) {
                    const int f = f0 + lane;
                    const uint32_t kf = f < ne ? order_key(sc[f * ns + s]) : 0u;
                    c += __popc(__ballot_sync(0xffffffffu, f < ne && (kf & mask) == prefix && (kf & b)));
                }
                if (c >= need) prefix |= b;
                else need -= c;
                mask |= b;
            }
            // above the k-th key, or equal to it and among the first `need` such frames
            int ties = 0;
            for (int f0 = 0; f0 < ne; f0 += 32) {
                const int f = f0 + lane;
                const uint32_t kf = f < ne ? order_key(sc[f * ns + s]) : 0u;
                const bool eq = kk > 0 && f < ne && kf == prefix;
                const unsigned m = __ballot_sync(0xffffffffu, eq);
                const int rank_eq = ties + __popc(m & ((1u << lane) - 1u));
                if (f < ne) aux[f * ns + s] = kk > 0 && (kf > prefix || (eq && rank_eq < need));
                ties += __popc(m);
            }
        }
        __syncthreads();
        for (int e = tid; e < ne * ns; e += nt)
            if (aux[e]) sc[e] = __fadd_rn(sc[e], boost);
        __syncthreads();
    }
    // ---- flat speaker-major scores with +inf silence slots; keep the first cache_len in
    // (score desc, flat index asc) order, except -inf ones (src/streaming.rs:436-463)
    const int nsc = ne + cp.n_sil;
    const int total = ns * nsc;
    const int L = min(cp.cache_len, total);
    for (int e = tid; e < total; e += nt) {
        const int sp = e / nsc, f = e % nsc;
        fkey[e] = order_key(f < ne ? sc[f * ns + sp] : INFINITY);
    }
    __syncthreads();
    __shared__ int part[16];
    __shared__ int carry, warp_tot[16];
    uint32_t prefix = 0, mask = 0;
    int need = L;
    for (int bit = 31; L > 0 && bit >= 0; bit--) {
        const uint32_t b = 1u << bit;
        int c = 0;
        for (int e = tid; e < total; e += nt) c += (fkey[e] & mask) == prefix && (fkey[e] & b);
        c = __reduce_add_sync(0xffffffffu, c);
        if (lane == 0) part[warp] = c;
        __syncthreads();
        int sum = 0;
        for (int q = 0; q < nwarps; q++) sum += part[q];
        __syncthreads();
        if (sum >= need) prefix |= b;
        else need -= sum;
        mask |= b;
    }
    // flags: above the L-th key, or equal to it among the first `need` in flat order
    // (block scan of the ties); -inf picks become the sentinel, i.e. are dropped
    const uint32_t ninf = order_key(-INFINITY);
    if (tid == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < total; base += nt) {
        const int e = base + tid;
        const bool in = e < total && L > 0;
        const uint32_t ke = e < total ? fkey[e] : 0u;
        const int eq = in && ke == prefix;
        int x = eq;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_tot[warp] = x;
        __syncthreads();
        int woff = 0;
        for (int q = 0; q < warp; q++) woff += warp_tot[q];
        const int rank_eq = carry + woff + x - eq;
        if (e < total) aux[e] = in && ke != ninf && (ke > prefix || (eq && rank_eq < need));
        __syncthreads();
        if (tid == nt - 1) carry = rank_eq + eq;
        __syncthreads();
    }
    // exclusive scan of aux over [0, total) -> position of each kept index (block scan in chunks)
    if (tid == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < total; base += nt) {
        const int e = base + tid;
        const int flag = e < total ? aux[e] : 0;
        int x = flag;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_tot[warp] = x;
        __syncthreads();
        int woff = 0;
        for (int q = 0; q < warp; q++) woff += warp_tot[q];
        const int pos = carry + woff + x - flag;
        __syncthreads();
        if (e < total && flag) idx[pos] = e;  // the picked list (sorted ascending)
        if (tid == nt - 1) carry = pos + flag;
        __syncthreads();
    }
    *L_out = L;
    return carry;
}

// The gather of src/streaming.rs:464-481: output row p is candidate frame
// idx[p] % nsc for p < n_real and that slot is a frame; silence slots and the
// sentinels get `silence` and a zero probability row.
__device__ void compress_gather(const int* __restrict__ idx, int n_real, int L, int ne, int nsc,
                                const float* __restrict__ rows, const float* __restrict__ cand,
                                const float* __restrict__ silence, int hidden, int ns, float* __restrict__ out_rows,
                                float* __restrict__ out_probs) {
    const int tid = threadIdx.x, nt = blockDim.x;
    for (long long e = tid; e < (long long)L * (hidden / 4); e += nt) {
        const int p = (int)(e / (hidden / 4)), c = (int)(e % (hidden / 4));
        int frame = ne;
        if (p < n_real) {
            const int f = idx[p] % nsc;
            frame = f < ne ? f : ne;
        }
        const float4* src = frame < ne ? reinterpret_cast<const float4*>(rows + (long long)frame * hidden)
                                       : reinterpret_cast<const float4*>(silence);
        reinterpret_cast<float4*>(out_rows + (long long)p * hidden)[c] = src[c];
    }
    for (int e = tid; e < L * ns; e += nt) {
        const int p = e / ns, s = e % ns;
        int frame = ne;
        if (p < n_real) {
            const int f = idx[p] % nsc;
            frame = f < ne ? f : ne;
        }
        out_probs[e] = frame < ne ? cand[frame * ns + s] : 0.0f;
    }
}

// One CTA per sequence.  Shared layout (floats unless noted):
//   probs [S*ns]      pooled step probabilities (_pool_probs)
//   cand  [ne*ns]     probabilities of the compression candidates
//   sc    [ne*ns]     frame scores
//   key   [P] (uint)  order keys of the flat speaker-major scores (P >= ns*(ne+n_sil))
//   idx   [P] (int)   the picked flat indices, ascending
//   aux   [P] (int)   selection flags
__global__ void __launch_bounds__(512) cache_update_kernel(const SeqStep* __restrict__ steps,
                                                           const float* __restrict__ win,
                                                           const float* __restrict__ logits, int stride,
                                                           long long logit_rows, CacheConst cp,
                                                           const float* __restrict__ silence, int P_max) {
    griddep_wait();
    griddep_launch_dependents();
    extern __shared__ float sm[];
    const int i = blockIdx.x;
    const SeqStep st = steps[i];
    const int ns = cp.ns, sub = cp.sub, hidden = cp.hidden;
    const int S = st.S;
    const int tid = threadIdx.x, nt = blockDim.x;
    const float* wrow = win + (long long)i * stride * hidden;
    const float* lrow = logits + (long long)i * logit_rows * ns;  // head output keeps 2 pad rows per sequence

    float* probs = sm;
    float* cand = probs + stride * ns;
    float* sc = cand + stride * ns;
    float* key = sc + stride * ns;
    int* idx = reinterpret_cast<int*>(key + P_max);
    int* aux = idx + P_max;

    // ---- _pool_probs (src/streaming.rs:202-217): sigmoid averaged over sub-frames, mask after
    for (int e = tid; e < S * ns; e += nt) {
        const int g = e / ns, c = e % ns;
        float acc = 0.0f;
        for (int k = 0; k < sub; k++) {
            const float l = lrow[((long long)g * sub + k) * ns + c];
            acc = __fadd_rn(acc, __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_f(-l))));
        }
        probs[e] = g < st.valid ? __fdiv_rn(acc, (float)sub) : 0.0f;
    }
    // ---- scored logit rows [cached*sub, (cached+nchunk)*sub), capped (src/model.rs:455-461)
    {
        const long long s0 = (long long)(st.ncache + st.nfifo) * sub * ns;
        const long long n = (long long)st.keep_rows * ns;
        for (long long e = tid; e < n; e += nt) st.out_logits[e] = lrow[s0 + e];
    }
    __syncthreads();

    const int ne = st.ncache + st.popped;
    // ---- candidates' probabilities: stored (compressed cache) or this step's, then popped FIFO frames
    for (int e = tid; e < ne * ns; e += nt) {
        const int f = e / ns;
        cand[e] = (f < st.ncache && st.was_compressed) ? st.cp_in[e] : probs[e];
    }
    __syncthreads();

    // ---- new FIFO: window rows [ncache + popped, ncache + nfifo + nchunk)
    const int cf_new = st.popped > 0 ? (st.compress ? cp.cache_len : ne) : st.ncache;
    const int ff_new = st.nfifo + st.nchunk - st.popped;
    for (long long e = tid; e < (long long)ff_new * (hidden / 4); e += nt) {
        const int r = (int)(e / (hidden / 4)), c = (int)(e % (hidden / 4));
        reinterpret_cast<float4*>(st.pre_out + (long long)(cf_new + r) * hidden)[c] =
            reinterpret_cast<const float4*>(wrow + (long long)(st.ncache + st.popped + r) * hidden)[c];
    }

    if (!st.compress) {
        // cache rows = window rows [0, cf_new); stored probs follow them
        for (long long e = tid; e < (long long)cf_new * (hidden / 4); e += nt) {
            const int r = (int)(e / (hidden / 4)), c = (int)(e % (hidden / 4));
            reinterpret_cast<float4*>(st.pre_out + (long long)r * hidden)[c] =
                reinterpret_cast<const float4*>(wrow + (long long)r * hidden)[c];
        }
        if (st.popped > 0)
            for (int e = tid; e < ne * ns; e += nt) st.cp_out[e] = cand[e];
        else if (st.was_compressed)
            for (int e = tid; e < st.ncache * ns; e += nt) st.cp_out[e] = st.cp_in[e];
        return;
    }

    // ================= _compress (src/streaming.rs:410-482) =================
    int L = 0;
    const int n_real = compress_select(cand, sc, reinterpret_cast<uint32_t*>(key), idx, aux, ne, cp, &L);
    compress_gather(idx, n_real, L, ne, ne + cp.n_sil, wrow, cand, silence, hidden, ns, st.pre_out, st.cp_out);
}

// SpeakerCache::compress / trace_compress (src/streaming.rs:353-482) alone, for the
// stage entry point: one CTA runs compress_select and compress_gather -- the code the
// chunk loop's cache_update_kernel runs -- on `ne` given candidate frames.  Shared
// layout as cache_update_kernel's: cand [ne*ns], sc [ne*ns], key/idx/aux [P_max].
__global__ void __launch_bounds__(512) cache_compress_kernel(const float* __restrict__ probs, int ne,
                                                             const float* __restrict__ rows,
                                                             const float* __restrict__ silence, CacheConst cp,
                                                             int P_max, int* __restrict__ picked,
                                                             int* __restrict__ counts, float* __restrict__ out_rows,
                                                             float* __restrict__ out_probs) {
    extern __shared__ float sm[];
    const int ns = cp.ns;
    float* cand = sm;
    float* sc = cand + ne * ns;
    float* key = sc + ne * ns;
    int* idx = reinterpret_cast<int*>(key + P_max);
    int* aux = idx + P_max;
    for (int e = threadIdx.x; e < ne * ns; e += blockDim.x) cand[e] = probs[e];
    __syncthreads();
    int L = 0;
    const int n_real = compress_select(cand, sc, reinterpret_cast<uint32_t*>(key), idx, aux, ne, cp, &L);
    for (int p = threadIdx.x; p < n_real; p += blockDim.x) picked[p] = idx[p];
    if (threadIdx.x == 0) {
        counts[0] = n_real;
        counts[1] = L;
    }
    if (rows) compress_gather(idx, n_real, L, ne, ne + cp.n_sil, rows, cand, silence, cp.hidden, ns, out_rows, out_probs);
}

}  // namespace

void launch_assemble(cudaStream_t s, const SeqStep* steps, int nseq, const float* embeds, float* win, int stride,
                     int hidden) {
    if (nseq <= 0 || stride <= 0) return;
    launch_pdl(assemble_kernel, dim3(stride, nseq), dim3(128), 0, s, steps, embeds, win, stride, hidden);
}

size_t cache_update_smem(int stride, int ns, int P_max) {
    return (size_t)3 * stride * ns * 4 + (size_t)P_max * 4 * 3;
}

void launch_cache_update(cudaStream_t s, const SeqStep* steps, int nseq, const float* win, const float* logits,
                         int stride, const CacheConst& c, const float* silence) {
    if (nseq <= 0) return;
    int P = 1;
    while (P < c.ns * (stride + c.n_sil)) P <<= 1;
    const size_t smem = cache_update_smem(stride, c.ns, P);
    {
        // the limit set so far on each device; raised when a longer window needs more
        static size_t attr[kMaxDevices];
        static std::mutex mu;
        const int dev = current_device();
        std::lock_guard<std::mutex> lock(mu);
        if (smem > attr[dev]) {
            N3D_CUDA(cudaFuncSetAttribute(cache_update_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            attr[dev] = smem;
        }
    }
    launch_pdl(cache_update_kernel, dim3(nseq), dim3(512), smem, s, steps, win, logits, stride,
               (long long)(stride + 2) * c.sub, c, silence, P);
}

size_t cache_compress_smem(int ne, int ns, int n_sil) {
    const long long P = ((long long)ns * (ne + n_sil) + 3) / 4 * 4;
    return (size_t)2 * ne * ns * 4 + (size_t)P * 4 * 3;
}

void launch_cache_compress(cudaStream_t s, const float* probs, int ne, const float* rows, const float* silence,
                           const CacheConst& c, int* picked, int* counts, float* out_rows, float* out_probs) {
    const int P = (c.ns * (ne + c.n_sil) + 3) / 4 * 4;
    const size_t smem = cache_compress_smem(ne, c.ns, c.n_sil);
    N3D_CUDA(cudaFuncSetAttribute(cache_compress_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cache_compress_kernel<<<1, 512, smem, s>>>(probs, ne, rows, silence, c, P, picked, counts, out_rows, out_probs);
    N3D_CUDA(cudaGetLastError());
}

}  // namespace n3d
