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

__device__ inline void b3_step(B3World* w, float dt, int substeps) {
    b3x::one::step_world(w, dt, substeps, B3_JOINT_ITERS, B3_RELAX_ITERS);
}

static __global__ void b3_step_kernel(B3World* worlds, int n, float dt, int substeps) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) b3_step(&worlds[i], dt, substeps);
}
#endif
