/* Prints sizeof / offsetof of every field of the C ABI's structs, one "name value" per line. The test suite
 * compiles this file twice, once against this repository's include/flyhigh.h and once against the reference's own
 * header, and requires the two listings to be identical (byte-for-byte struct layout of the drop-in). */
#include <stddef.h>
#include <stdio.h>

#include "flyhigh.h"

#define F(S, m) printf(#S "." #m " %zu %zu\n", offsetof(S, m), sizeof(((S*)0)->m))

int main(void) {
    printf("FhEngineOptions %zu %zu\n", sizeof(FhEngineOptions), _Alignof(FhEngineOptions));
    F(FhEngineOptions, backend);
    F(FhEngineOptions, tensor_cores);
    F(FhEngineOptions, autotune);
    F(FhEngineOptions, adapter);
    F(FhEngineOptions, precision);
    F(FhEngineOptions, tune_cache);
    F(FhEngineOptions, compact_memory);
    F(FhEngineOptions, dxc_path);
    printf("FhSessionOptions %zu %zu\n", sizeof(FhSessionOptions), _Alignof(FhSessionOptions));
    F(FhSessionOptions, width);
    F(FhSessionOptions, height);
    F(FhSessionOptions, internal_w);
    F(FhSessionOptions, internal_h);
    F(FhSessionOptions, k);
    F(FhSessionOptions, repair);
    F(FhSessionOptions, render);
    F(FhSessionOptions, keep_static);
    F(FhSessionOptions, static_frames);
    F(FhSessionOptions, static_tolerance);
    F(FhSessionOptions, fast_render);
    F(FhSessionOptions, linear_t);
    F(FhSessionOptions, keep_maps);
    F(FhSessionOptions, protection_mask);
    F(FhSessionOptions, tune);
    printf("FhStreamOptions %zu %zu\n", sizeof(FhStreamOptions), _Alignof(FhStreamOptions));
    F(FhStreamOptions, mode);
    F(FhStreamOptions, cadence);
    F(FhStreamOptions, scene_cut);
    F(FhStreamOptions, held_frames);
    F(FhStreamOptions, held_mean);
    F(FhStreamOptions, held_max);
    F(FhStreamOptions, inputs);
    F(FhStreamOptions, outputs);
    printf("FhClassification %zu %zu\n", sizeof(FhClassification), _Alignof(FhClassification));
    F(FhClassification, kind);
    F(FhClassification, mean);
    F(FhClassification, max);
    F(FhClassification, black);
    F(FhClassification, motion);
    printf("FhPush %zu %zu\n", sizeof(FhPush), _Alignof(FhPush));
    F(FhPush, ready);
    F(FhPush, base_slot);
    F(FhPush, stats_pending);
    F(FhPush, start_pts);
    F(FhPush, end_pts);
    return 0;
}
