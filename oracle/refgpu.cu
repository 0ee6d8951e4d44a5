/*
 * refgpu.cu -- the reference's own GPU batch step, compiled from the
 * reference checkout: b3_batch_step_gpu (b3_batch.cuh:63-89), one thread per
 * world stepping its AoS B3World with b3_step (09_step.inl:262-264).
 *
 * TEST AND BENCHMARK INFRASTRUCTURE, NOT PRODUCT CODE.  oracle/Makefile builds
 * it per capacity configuration into _ref/libb3refgpu_<cfg>.so with the
 * reference's stock nvcc flags (-O3, default floating-point contraction);
 * bench.py's reference arm times it as the GPU kernel the batched engine
 * replaces.
 */
#include <cuda_runtime.h>

#include "b3_batch.cuh"
#include "b3_scenes.h"

#define EXPORT extern "C" __attribute__((visibility("default")))

/* The benchmark scenes' per-step actions, applied per world with the
 * reference's own b3_apply_* / joint setters (as the CPU shim does). */
static __global__ void refgpu_apply_kernel(B3Batch b, int scene, unsigned long long seed,
                                           unsigned long long first, unsigned long long step) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= b.count) return;
    int kind, index, nv;
    b3s_action_layout(scene, &kind, &index, &nv);
    if (nv <= 0) return;
    float v[16];
    b3s_actions(scene, seed, first + (unsigned long long)i, step, v);
    b3s_apply(b3_batch_world(b, i), kind, index, nv, v);
}

EXPORT int refgpu_apply(void* data, size_t stride, size_t offset, int count, int scene, unsigned long long seed,
                        unsigned long long first, unsigned long long step, void* stream) {
    B3Batch b;
    b.data = data;
    b.stride = stride;
    b.world_offset = offset;
    b.count = count;
    if (!b3_batch_valid(b)) return (int)cudaErrorInvalidValue;
    if (!count) return (int)cudaSuccess;
    refgpu_apply_kernel<<<(count + 31) / 32, 32, 0, (cudaStream_t)stream>>>(b, scene, seed, first, step);
    return (int)cudaGetLastError();
}

EXPORT size_t refgpu_world_bytes(void) { return sizeof(B3World); }
EXPORT unsigned long long refgpu_signature(void) { return b3_config_signature(); }

EXPORT int refgpu_batch_step(void* data, size_t stride, size_t offset, int count, float dt, int substeps,
                             const unsigned char* active, void* stream) {
    B3Batch b;
    b.data = data;
    b.stride = stride;
    b.world_offset = offset;
    b.count = count;
    return (int)b3_batch_step_gpu(b, dt, substeps, active, (cudaStream_t)stream);
}
