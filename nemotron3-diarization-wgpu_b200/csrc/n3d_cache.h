// Per-step, per-sequence schedule entries shared by the host runner and the
// window-assembly / speaker-cache kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

namespace n3d {

// One sequence's view of one chunk-loop step (src/model.rs:371-475).  Every
// count is data-independent and precomputed on the host.
struct SeqStep {
    int S;               // window frames = ncache + nfifo + new embeddings
    int valid;           // frames the attention mask lets through (a true prefix)
    int ncache, nfifo;   // prefix split at step start
    int nchunk;          // scored frames appended to the FIFO
    int popped;          // FIFO frames promoted to the cache (_num_popped_frames)
    int compress;        // 1 when ncache + popped exceeds speaker_cache_length
    int was_compressed;  // the cache held compressed frames at step start
    int keep_rows;       // 10 ms logit rows emitted = min(nchunk * sub, cap)
    int pad_;
    long long emb_row;   // first row of this step's new embeddings in the embeds buffer
    const float* pre_in;   // prefix rows [ncache + nfifo, hidden] from the previous step
    float* pre_out;        // prefix for the next step
    const float* cp_in;    // probabilities stored with a compressed cache [ncache, ns]
    float* cp_out;
    float* out_logits;     // destination of this step's emitted logit rows
};

// Cache policy constants (CacheConfig, src/streaming.rs:39-72).
struct CacheConst {
    int hidden, ns, sub, cache_len, n_sil, min_pos, k_strong, k_weak;
    float thr, latest_boost;
};

void launch_assemble(cudaStream_t s, const SeqStep* steps, int nseq, const float* embeds, float* win, int stride,
                     int hidden);
void launch_cache_update(cudaStream_t s, const SeqStep* steps, int nseq, const float* win, const float* logits,
                         int stride, const CacheConst& c, const float* silence);

}  // namespace n3d
