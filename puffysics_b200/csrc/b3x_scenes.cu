// b3x_scenes.cu -- device generators of the benchmark's per-step inputs:
// action values and reset masks (puffysics_b200/scenes/b3_scenes.h).  They
// use integer hashing and exactly representable float arithmetic only, so
// they produce the same bits as the host generators.
#include <cuda_runtime.h>

#include "puffysics_b200.h"
#include "b3_scenes.h"

namespace b3x {

__global__ void scene_actions_kernel(float* out, int n, int scene, unsigned long long seed,
        unsigned long long first, unsigned long long step, int nv) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v[16];
    b3s_actions(scene, seed, first + (uint64_t)i, step, v);
    for (int k = 0; k < nv && k < 16; k++) out[(size_t)i * nv + k] = v[k];
}

__global__ void scene_reset_kernel(unsigned char* out, int n, unsigned long long seed, unsigned long long first,
        unsigned long long step) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = (unsigned char)b3s_reset_selected(seed, first + (uint64_t)i, step);
}

}  // namespace b3x

extern "C" {

// Writes values_per_world floats per world; returns values_per_world (0: the
// scene has no actions), or -1 on invalid arguments.
B3X_API int b3x_scene_actions_gpu(float* out, int n, int scene, unsigned long long seed, unsigned long long first,
        unsigned long long step, void* stream) {
    int kind, index, nv;
    b3s_action_layout(scene, &kind, &index, &nv);
    if (n < 0 || (n > 0 && nv > 0 && !out)) return -1;
    if (n == 0 || nv == 0) return nv;
    b3x::scene_actions_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(out, n, scene, seed, first, step,
        nv);
    return cudaGetLastError() == cudaSuccess ? nv : -1;
}

B3X_API int b3x_scene_reset_gpu(unsigned char* out, int n, unsigned long long seed, unsigned long long first,
        unsigned long long step, void* stream) {
    if (n < 0 || (n > 0 && !out)) return cudaErrorInvalidValue;
    if (n == 0) return cudaSuccess;
    b3x::scene_reset_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(out, n, seed, first, step);
    return cudaGetLastError();
}

}  // extern "C"
