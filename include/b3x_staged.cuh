/* b3x_staged.cuh -- staged per-element launches for adapters' fused kernels.
 *
 * An environment adapter that steps its worlds from its own kernel (action,
 * b3_step, reward, observation, reset: reference
 * examples/pufferlib/puffysics_hover/puffysics_hover.cu:40-43) runs one
 * thread per environment over an array of caller structs in global memory.
 * For environments whose struct is small (a world of a few bodies, shapes and
 * contacts, a few KB), this header provides the B200 form of that launch:
 * blocks of 32 threads copy kPerBlock consecutive elements into shared memory
 * with coalesced asynchronous 8-byte copies, call fn(element, index) on one
 * thread per element -- the element's world is then stepped in shared memory
 * by the device b3_step of puffysics.cuh -- and copy the elements back.
 * Fewer elements than threads per block spread the work over every SM and let
 * several warps of an SM share the instruction fetches of the long per-element
 * program (8 per block measured best for the hover world).
 *
 * Requirements: sizeof(T) a multiple of 8, the array 8-byte aligned,
 * kPerBlock * sizeof(T) within the shared memory a block may use (the launch
 * helper raises the kernel's limit when needed).  fn must not keep pointers
 * into its element past the call; pointers stored inside an element are copied
 * as values and keep pointing where they did.
 */
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "puffysics.cuh"

namespace b3x {

// Words (8 bytes) between staged elements: 2 x odd, so that consecutive
// threads' elements fall in different shared-memory bank pairs.
template <class T>
__host__ __device__ constexpr unsigned staged_stride_words() {
    return (unsigned)(sizeof(T) / 8) % 2 == 0 ? (unsigned)(sizeof(T) / 8) + 1 : (unsigned)(sizeof(T) / 8);
}

template <int kPerBlock, class T, class Fn>
__global__ void __launch_bounds__(32) staged_kernel(T* items, int n, Fn fn) {
    static_assert(sizeof(T) % 8 == 0, "staged elements must be a multiple of 8 bytes");
    static_assert(kPerBlock >= 1 && kPerBlock <= 32, "one thread per element, at most one warp");
    extern __shared__ __align__(16) unsigned char b3x_staged_smem[];
    uint64_t* sw = reinterpret_cast<uint64_t*>(b3x_staged_smem);
    constexpr unsigned kWords = sizeof(T) / 8;
    constexpr unsigned kStride = staged_stride_words<T>();
    const int lane = threadIdx.x;
    const long long first = (long long)blockIdx.x * kPerBlock;
    const int here = n - first < kPerBlock ? (int)(n - first) : kPerBlock;
    const uint64_t* src = reinterpret_cast<const uint64_t*>(items + first);
    for (int e = 0; e < here; e++) {
        for (unsigned w = lane; w < kWords; w += 32) {
            const uint32_t dst = (uint32_t)__cvta_generic_to_shared(sw + (size_t)e * kStride + w);
            asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src + (size_t)e * kWords + w)
                         : "memory");
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
    if (lane < here) fn(*reinterpret_cast<T*>(sw + (size_t)lane * kStride), (int)(first + lane));
    __syncwarp();
    uint64_t* dst = reinterpret_cast<uint64_t*>(items + first);
    for (int e = 0; e < here; e++)
        for (unsigned w = lane; w < kWords; w += 32) dst[(size_t)e * kWords + w] = sw[(size_t)e * kStride + w];
}

// Shared memory of one block of staged_kernel<kPerBlock, T>.
template <int kPerBlock, class T>
__host__ __device__ constexpr size_t staged_smem_bytes() {
    return (size_t)kPerBlock * staged_stride_words<T>() * 8;
}

// Enqueue fn over items[0, n) on `stream`: no allocation, no synchronisation.
// Returns cudaErrorInvalidValue (nothing launched) for n < 0, a null or
// misaligned array with n > 0, or elements too large to stage.
template <int kPerBlock, class T, class Fn>
cudaError_t staged_launch(T* items, int n, Fn fn, cudaStream_t stream) {
    if (n < 0 || (n > 0 && (items == nullptr || ((uintptr_t)items % 8) != 0))) return cudaErrorInvalidValue;
    if (n == 0) return cudaSuccess;
    const size_t smem = staged_smem_bytes<kPerBlock, T>();
    if (smem > 48 * 1024) {
        int dev = 0, optin = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e != cudaSuccess) return e;
        if (smem > (size_t)optin) return cudaErrorInvalidValue;
        e = cudaFuncSetAttribute(staged_kernel<kPerBlock, T, Fn>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e != cudaSuccess) return e;
    }
    const unsigned blocks = (unsigned)((n + kPerBlock - 1) / kPerBlock);
    staged_kernel<kPerBlock, T, Fn><<<blocks, 32, smem, stream>>>(items, n, fn);
    return cudaGetLastError();
}

}  // namespace b3x
