/* Compatibility name: adapters written against the reference include
 * "puffysics.cuh"; it resolves to this library's public header.
 *
 * Compiled by nvcc it also provides the per-world device step of the
 * reference, for adapters that step their worlds from their own kernels, one
 * thread per world:
 *   __device__ void b3_step(B3World* w, float dt, int substeps);
 *       (reference src/puffysics/09_step.inl:262-264)
 *   static __global__ void b3_step_kernel(B3World* worlds, int n, float dt,
 *       int substeps);   (reference 09_step.inl:325-333)
 * with the capacities and B3_JOINT_ITERS / B3_RELAX_ITERS of the including
 * translation unit.  The batched b3_batch_step_gpu (b3_batch.cuh) is the
 * fast path for the same step. */
#pragma once
#include "puffysics_b200.h"

#if defined(__CUDACC__)
#include "../puffysics_b200/csrc/b3x_world_step.cuh"

/* The reference's step-mode switches of the including translation unit. */
#if defined(B3_INTERLEAVE_CONTACTS)
#define B3X_MODE_INTERLEAVE b3x::kStepInterleaveContacts
#else
#define B3X_MODE_INTERLEAVE 0
#endif
#if defined(B3_SKIP_RESTITUTION)
#define B3X_MODE_SKIP_RESTITUTION b3x::kStepSkipRestitution
#else
#define B3X_MODE_SKIP_RESTITUTION 0
#endif

/* Per-thread launches run one warp per block (as the reference launches);
 * 16 resident blocks per SM cap the step at 128 registers per thread, which
 * keeps large worlds' local-memory latency covered (pile: +31% over the
 * uncapped 150 registers). */
#define B3X_THREAD_BOUNDS __launch_bounds__(32, 16)

__device__ inline void b3_step(B3World* w, float dt, int substeps) {
    b3x::one::step_world<(B3_ART_CONTACTS != 0)>(w, dt, substeps, B3_JOINT_ITERS, B3_RELAX_ITERS,
                                                 B3X_MODE_INTERLEAVE | B3X_MODE_SKIP_RESTITUTION);
}

static __global__ void B3X_THREAD_BOUNDS b3_step_kernel(B3World* worlds, int n, float dt, int substeps) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) b3_step(&worlds[i], dt, substeps);
}

#if B3_HAS_USER_FORCES || B3_ART_CONTACTS
/* With a per-substep force hook, or with the articulated contact response
 * of B3_ART_CONTACTS=1, the batch step runs this translation unit's
 * per-thread b3_step, which has them (reference b3_batch.cuh:63-89
 * semantics: same validation, no-ops, mask, stream; no allocation). */
static __global__ void B3X_THREAD_BOUNDS b3x_user_force_batch_kernel(B3Batch batch, float dt, int substeps,
        const unsigned char* active) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (size_t)batch.count && (!active || active[i])) b3_step(b3_batch_world(batch, (int)i), dt, substeps);
}

B3_INL cudaError_t b3_batch_step_gpu(B3Batch batch, float dt, int substeps, const unsigned char* active,
        cudaStream_t stream) {
    if (!b3_batch_valid(batch) || !isfinite(dt) || dt < 0 || substeps < 1) return cudaErrorInvalidValue;
    if (!batch.count || dt == 0) return cudaSuccess;
    b3x_user_force_batch_kernel<<<((unsigned)batch.count + 31u) / 32u, 32, 0, stream>>>(batch, dt, substeps,
                                                                                         active);
    return cudaGetLastError();
}
#endif
#endif
