/* Test helper for tests/test_c_abi.py: a plain C99 caller of include/n3d.h, as a cgo or
 * other FFI binding would be.  It uses only entry points that need no GPU: version,
 * frame duration, the chunk schedule of a checkpoint, and speaker segments.  It prints
 * what it gets so the test can compare it with the Python binding; on a machine without
 * a GPU it also checks that model load reports N3D_ERR_NO_DEVICE. */
#include <stdio.h>
#include <stdlib.h>

#include "n3d.h"

int main(int argc, char **argv) {
    n3d_config *cfg = NULL;
    n3d_mode_params mp;
    n3d_step_plan steps[64];
    n3d_run_output totals;
    n3d_segment *segs = NULL;
    size_t n = 0, i;
    float logits[12];
    n3d_model *model = NULL;
    n3d_status st;

    if (argc < 2) return 2;
    printf("version %s\n", n3d_version());
    printf("frame_duration %.9g\n", (double)n3d_frame_duration(160, 16000));
    if (n3d_config_load(argv[1], &cfg) != N3D_OK) {
        printf("config error %s\n", n3d_last_error());
        return 1;
    }
    if (n3d_mode_params_resolve(cfg, N3D_MODE_ULTRA_LOW_LATENCY, &mp) != N3D_OK) return 1;
    printf("ultra first_chunk_samples %zu samples_per_chunk %zu latency_ms %zu\n", mp.first_chunk_samples,
           mp.samples_per_chunk, mp.latency_ms);
    if (n3d_schedule(cfg, N3D_MODE_OFFLINE, 480000, steps, 64, &n, &totals) != N3D_OK) return 1;
    printf("offline steps %zu frames %zu chunks %zu", n, totals.num_frames, totals.num_chunks);
    for (i = 0; i < n && i < 64; i++) printf(" [%zu %zu %zu]", steps[i].window_frames, steps[i].valid_frames,
                                             steps[i].scored_frames);
    printf("\n");
    if (n3d_schedule(cfg, N3D_MODE_LOW_LATENCY, 100, steps, 64, &n, NULL) != N3D_ERR_UNSUPPORTED_AUDIO) return 1;
    printf("short streaming audio: %s\n", n3d_last_error());
    n3d_config_free(cfg);

    /* speaker 0 active in frames 1-2, speaker 1 in frame 3 (src/segments.rs) */
    for (i = 0; i < 12; i++) logits[i] = -4.0f;
    logits[1 * 2 + 0] = logits[2 * 2 + 0] = logits[3 * 2 + 1] = 4.0f;
    if (n3d_extract_speaker_dict(logits, 6, 2, 0.01f, NULL, 0.5f, &segs, &n) != N3D_OK) return 1;
    for (i = 0; i < n; i++) printf("segment %.2f %.2f %zu\n", (double)segs[i].start, (double)segs[i].end, segs[i].speaker);
    n3d_segments_free(segs);

    if (argc > 2) {
        st = n3d_model_load_gpu(argv[1], 0, &model);
        printf("load status %d\n", (int)st);
        n3d_model_free(model);
    }
    return 0;
}
