// b3x_thread_step.cu -- launchers of the header's per-thread device b3_step
// (include/puffysics.cuh), built once per capacity configuration into
// libb3thread_<config>.so.
//
// These are the entry points of the compatibility path: one thread steps one
// world in place (the reference's own GPU form, b3_batch.cuh:63-89, with this
// library's device step).  They exist so that the per-thread step can be
// checked against the reference on the GPU and timed beside the batched
// kernel; the capacities (B3_MAX_*) and solver iteration counts
// (B3_JOINT_ITERS, B3_RELAX_ITERS) are those this file is compiled with.
#include <cmath>

#include <cuda_runtime.h>

#include "puffysics.cuh"
#include "b3_scenes.h"

#define B3T_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr int kThreads = 32;   // one warp per block, as the reference launches

__global__ void B3X_THREAD_BOUNDS thread_batch_kernel(B3Batch batch, float dt, int substeps, const unsigned char* active) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (size_t)batch.count && (!active || active[i])) b3_step(b3_batch_world(batch, (int)i), dt, substeps);
}

// The benchmark scene's actions of one step, generated and applied per
// world with the header's b3_apply_* (one launch, as the reference arm's
// action kernel does).
__global__ void thread_scene_apply_kernel(B3Batch batch, int scene, unsigned long long seed, unsigned long long first,
        unsigned long long step) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)batch.count) return;
    int kind, index, nv;
    b3s_action_layout(scene, &kind, &index, &nv);
    if (nv <= 0) return;
    float v[16];
    b3s_actions(scene, seed, first + (unsigned long long)i, step, v);
    b3s_apply(b3_batch_world(batch, (int)i), kind, index, nv, v);
}

}  // namespace

// Capacity signature the library was compiled for (B3_CONFIG_SIGNATURE).
B3T_API unsigned long long b3x_thread_signature(void) { return B3_CONFIG_SIGNATURE; }
B3T_API int b3x_thread_joint_iters(void) { return B3_JOINT_ITERS; }
B3T_API int b3x_thread_relax_iters(void) { return B3_RELAX_ITERS; }

// b3_batch_step_gpu semantics (b3_batch.cuh:81-89): invalid batch, dt not
// finite or negative, or substeps < 1 -> cudaErrorInvalidValue with no
// launch; count == 0 or dt == 0 -> no-op; otherwise one thread per world on
// `stream`, no allocation, no synchronisation.
B3T_API int b3x_thread_step_gpu(B3Batch batch, float dt, int substeps, const unsigned char* active, void* stream) {
    if (!b3_batch_valid(batch) || !std::isfinite(dt) || dt < 0.0f || substeps < 1) return (int)cudaErrorInvalidValue;
    if (batch.count == 0 || dt == 0.0f) return (int)cudaSuccess;
    unsigned blocks = ((unsigned)batch.count + kThreads - 1) / kThreads;
    thread_batch_kernel<<<blocks, kThreads, 0, (cudaStream_t)stream>>>(batch, dt, substeps, active);
    return (int)cudaGetLastError();
}

// The header's own b3_batch_step_gpu (the inline shim an adapter compiles):
// a call into libpuffysics_b200.so, or, with a force hook or
// B3_ART_CONTACTS=1, this translation unit's per-thread step.  Exported only
// where it stays inside this library (hook and articulation builds), so that
// the route an adapter gets can be checked on the GPU.
#if B3_HAS_USER_FORCES || B3_ART_CONTACTS
B3T_API int b3x_thread_shim_step_gpu(B3Batch batch, float dt, int substeps, const unsigned char* active,
        void* stream) {
    return (int)b3_batch_step_gpu(batch, dt, substeps, active, (cudaStream_t)stream);
}
#endif

// Benchmark input: the scene's actions of `step` applied to every world of
// the batch in one launch (no launch for scenes without actions).
B3T_API int b3x_thread_scene_apply_gpu(B3Batch batch, int scene, unsigned long long seed, unsigned long long first,
        unsigned long long step, void* stream) {
    if (!b3_batch_valid(batch)) return (int)cudaErrorInvalidValue;
    int kind, index, nv;
    b3s_action_layout(scene, &kind, &index, &nv);
    if (batch.count == 0 || nv <= 0) return (int)cudaSuccess;
    unsigned blocks = ((unsigned)batch.count + kThreads - 1) / kThreads;
    thread_scene_apply_kernel<<<blocks, kThreads, 0, (cudaStream_t)stream>>>(batch, scene, seed, first, step);
    return (int)cudaGetLastError();
}

// b3_step_kernel (reference 09_step.inl:325-333) over contiguous worlds.
B3T_API int b3x_thread_step_worlds_gpu(B3World* worlds, int n, float dt, int substeps, void* stream) {
    if (n < 0 || (n > 0 && !worlds)) return (int)cudaErrorInvalidValue;
    if (n == 0) return (int)cudaSuccess;
    b3_step_kernel<<<(n + kThreads - 1) / kThreads, kThreads, 0, (cudaStream_t)stream>>>(worlds, n, dt, substeps);
    return (int)cudaGetLastError();
}
