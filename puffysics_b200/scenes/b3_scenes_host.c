/*
 * b3_scenes_host.c -- host entry points of the seeded scene / action
 * generators (b3_scenes.h) for one capacity configuration, compiled by
 * puffysics_b200/build.py into _lib/libb3scenes_<cfg>.so.  The benchmark
 * builds its synthetic worlds with these; the GPU generates the same action
 * and reset streams with b3x_scene_actions_gpu / b3x_scene_reset_gpu.
 */
#include <stdint.h>
#include "puffysics_b200.h"
#include "b3_scenes.h"

#define EXPORT __attribute__((visibility("default")))

EXPORT size_t b3s_world_bytes(void) { return sizeof(B3World); }
EXPORT unsigned long long b3s_signature(void) { return B3_CONFIG_SIGNATURE; }

/* Build n worlds (global indices first..first+n-1) at `stride` bytes apart. */
EXPORT int b3s_build_batch(void* data, size_t stride, int n, int scene, unsigned long long seed,
        unsigned long long first) {
    for (int i = 0; i < n; i++) {
        B3World* w = (B3World*)((unsigned char*)data + (size_t)i * stride);
        if (b3s_build(w, scene, seed, first + (uint64_t)i) != 0) return -1 - i;
    }
    return 0;
}

/* Action values (values_per_world floats per world) for one step. */
EXPORT int b3s_actions_batch(float* out, int n, int scene, unsigned long long seed, unsigned long long first,
        unsigned long long step) {
    int kind, index, nv;
    b3s_action_layout(scene, &kind, &index, &nv);
    for (int i = 0; i < n && nv > 0; i++) b3s_actions(scene, seed, first + (uint64_t)i, step, out + (size_t)i * nv);
    return nv;
}

/* Reset mask of the scale-out configuration for one step. */
EXPORT void b3s_reset_batch(unsigned char* out, int n, unsigned long long seed, unsigned long long first,
        unsigned long long step) {
    for (int i = 0; i < n; i++) out[i] = (unsigned char)b3s_reset_selected(seed, first + (uint64_t)i, step);
}
