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
// SpeakerCache::compress alone (one CTA, the selection and gather code of
// cache_update_kernel): probs [ne, ns]; rows [ne, hidden] and silence [hidden], or
// rows == nullptr for the ranking only.  Writes the n_real picked flat indices
// (ascending, -inf picks dropped) to picked, counts[0] = n_real, counts[1] = L =
// min(cache_len, ns * (ne + n_sil)), and the gathered [L, hidden] rows and [L, ns]
// probabilities.  cache_compress_smem() is its shared memory (at most 227 KB).
size_t cache_compress_smem(int ne, int ns, int n_sil);
void launch_cache_compress(cudaStream_t s, const float* probs, int ne, const float* rows, const float* silence,
                           const CacheConst& c, int* picked, int* counts, float* out_rows, float* out_probs);

}  // namespace n3d
