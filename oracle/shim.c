/*
 * shim.c -- C entry points of the two CPU oracles, loaded by the tests and by
 * the benchmark's CPU-baseline leg through ctypes.
 *
 * TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * Built twice per capacity configuration by oracle/Makefile:
 *   -DSHIM_REF  : against the reference's own headers (b3_batch.cuh ->
 *                 puffysics.cuh, compiled from the reference checkout), symbols
 *                 prefixed ref_, output oracle/_ref/libb3ref_<cfg>.so;
 *   -DSHIM_PORT : against include/puffysics_b200.h and the restatement in
 *                 oracle/port/b3port.c, symbols prefixed port_, output
 *                 oracle/_build/libb3port_<cfg>.so.
 * Both compile with -ffp-contract=off so their float results are exactly the
 * IEEE single-precision results of the source expressions.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#if defined(SHIM_REF)
#include "b3_batch.cuh"
#define SHIM(name) ref_##name
#elif defined(SHIM_PORT)
#include "puffysics_b200.h"
#include "b3port.h"
#define SHIM(name) port_##name
#ifndef PORT_JOINT_ITERS
#define PORT_JOINT_ITERS B3_JOINT_ITERS
#endif
#ifndef PORT_RELAX_ITERS
#define PORT_RELAX_ITERS B3_RELAX_ITERS
#endif
#else
#error "define SHIM_REF or SHIM_PORT"
#endif

#include "b3_scenes.h"

#define EXPORT __attribute__((visibility("default")))

static int shim_batch_step(B3Batch b, float dt, int subs, const unsigned char* active) {
#if defined(SHIM_REF)
    return b3_batch_step(b, dt, subs, active);
#else
    return b3port_batch_step(b, dt, subs, active, PORT_JOINT_ITERS, PORT_RELAX_ITERS);
#endif
}

static void shim_step_world(B3World* w, float dt, int subs) {
#if defined(SHIM_REF)
    b3_step(w, dt, subs);
#else
    b3port_step(w, dt, subs, PORT_JOINT_ITERS, PORT_RELAX_ITERS);
#endif
}

EXPORT size_t SHIM(world_bytes)(void) { return sizeof(B3World); }
EXPORT unsigned long long SHIM(config_signature)(void) { return b3_config_signature(); }
EXPORT int SHIM(joint_iters)(void) { return B3_JOINT_ITERS; }
EXPORT int SHIM(relax_iters)(void) { return B3_RELAX_ITERS; }

/* Build n contiguous worlds of `scene`, global indices first .. first+n-1. */
EXPORT int SHIM(build)(void* worlds, int n, int scene, unsigned long long seed, unsigned long long first) {
    B3World* w = (B3World*)worlds;
    for (int i = 0; i < n; i++)
        if (b3s_build(&w[i], scene, seed, first + (uint64_t)i) != 0) return -1 - i;
    return 0;
}

EXPORT int SHIM(batch_step)(void* data, size_t stride, size_t offset, int count, float dt, int subs,
        const unsigned char* active) {
    B3Batch b;
    b.data = data; b.stride = stride; b.world_offset = offset; b.count = count;
    return shim_batch_step(b, dt, subs, active);
}

EXPORT int SHIM(batch_restore)(void* data, size_t stride, size_t offset, int count, const void* initial,
        const unsigned char* reset) {
    B3Batch b;
    b.data = data; b.stride = stride; b.world_offset = offset; b.count = count;
#if defined(SHIM_REF)
    return b3_batch_restore(b, (const B3World*)initial, reset);
#else
    return b3port_batch_restore(b, (const B3World*)initial, reset);
#endif
}

EXPORT void SHIM(step_world)(void* world, float dt, int subs) { shim_step_world((B3World*)world, dt, subs); }

/* Apply the scene's generated actions for `step` through the per-world API. */
EXPORT void SHIM(apply)(void* data, size_t stride, size_t offset, int count, int scene, unsigned long long seed,
        unsigned long long first, unsigned long long step, const unsigned char* active) {
    int kind, index, nv;
    b3s_action_layout(scene, &kind, &index, &nv);
    if (kind < 0) return;
    float v[16];
    B3Batch b;
    b.data = data; b.stride = stride; b.world_offset = offset; b.count = count;
    for (int i = 0; i < count; i++) {
        if (active && !active[i]) continue;
        b3s_actions(scene, seed, first + (uint64_t)i, step, v);
        b3s_apply(b3_batch_world(b, i), kind, index, nv, v);
    }
}

/* Apply explicit action values (values_per_world floats per world). */
EXPORT void SHIM(apply_values)(void* data, size_t stride, size_t offset, int count, int kind, int index,
        const float* values, int values_per_world, const unsigned char* active) {
    B3Batch b;
    b.data = data; b.stride = stride; b.world_offset = offset; b.count = count;
    for (int i = 0; i < count; i++) {
        if (active && !active[i]) continue;
        b3s_apply(b3_batch_world(b, i), kind, index, values_per_world, values + (size_t)i * values_per_world);
    }
}

EXPORT int SHIM(collide)(const void* world, int sa, int sb, float* normal, float* pa, float* pb, float* sep,
        unsigned* feature) {
    const B3World* w = (const B3World*)world;
#if defined(SHIM_REF)
    B3Mani m;
    b3_collide_shapes(&m, w, &w->shapes[sa], &w->shapes[sb]);
    normal[0] = m.normal.x; normal[1] = m.normal.y; normal[2] = m.normal.z;
    for (int i = 0; i < m.count; i++) {
        pa[3 * i] = m.p_a[i].x; pa[3 * i + 1] = m.p_a[i].y; pa[3 * i + 2] = m.p_a[i].z;
        pb[3 * i] = m.p_b[i].x; pb[3 * i + 1] = m.p_b[i].y; pb[3 * i + 2] = m.p_b[i].z;
        sep[i] = m.sep[i];
        feature[i] = m.feature[i];
    }
    return m.count;
#else
    return b3port_collide(w, sa, sb, normal, pa, pb, sep, feature);
#endif
}

/* ---- multi-threaded CPU baseline: one pthread per core, contiguous world
 * partitions, each thread applies the step's actions and steps its worlds. */
typedef struct RunArgs {
    B3World* worlds;
    int begin, end;
    int scene;
    uint64_t seed, first, step0;
    int steps;
    float dt;
    int subs;
} RunArgs;

static void* run_part(void* p) {
    RunArgs* a = (RunArgs*)p;
    int kind, index, nv;
    b3s_action_layout(a->scene, &kind, &index, &nv);
    float v[16];
    for (int s = 0; s < a->steps; s++) {
        uint64_t step = a->step0 + (uint64_t)s;
        for (int i = a->begin; i < a->end; i++) {
            if (kind >= 0) {
                b3s_actions(a->scene, a->seed, a->first + (uint64_t)i, step, v);
                b3s_apply(&a->worlds[i], kind, index, nv, v);
            }
            shim_step_world(&a->worlds[i], a->dt, a->subs);
        }
    }
    return NULL;
}

/* Returns wall seconds for `steps` steps of `count` contiguous worlds on
 * `threads` threads (<= 0: all online CPUs), or a negative value on error. */
EXPORT double SHIM(run_mt)(void* worlds, int count, int scene, unsigned long long seed, unsigned long long first,
        unsigned long long step0, int steps, float dt, int subs, int threads) {
    if (threads <= 0) threads = 1;
    if (threads > count) threads = count > 0 ? count : 1;
    pthread_t* tid = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    RunArgs* args = (RunArgs*)calloc((size_t)threads, sizeof(RunArgs));
    if (!tid || !args) { free(tid); free(args); return -1.0; }
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for (int t = 0; t < threads; t++) {
        args[t].worlds = (B3World*)worlds;
        args[t].begin = (int)((long long)count * t / threads);
        args[t].end = (int)((long long)count * (t + 1) / threads);
        args[t].scene = scene; args[t].seed = seed; args[t].first = first; args[t].step0 = step0;
        args[t].steps = steps; args[t].dt = dt; args[t].subs = subs;
        if (pthread_create(&tid[t], NULL, run_part, &args[t]) != 0) {
            for (int k = 0; k < t; k++) pthread_join(tid[k], NULL);
            free(tid); free(args);
            return -2.0;
        }
    }
    for (int t = 0; t < threads; t++) pthread_join(tid[t], NULL);
    clock_gettime(CLOCK_MONOTONIC, &t1);
    free(tid); free(args);
    return (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
}
