// b3x_step.cu -- batched rigid-body step on B200 (sm_100a) and the exported
// C-ABI of libpuffysics_b200.so.
//
// Mapping.  A tile is 32 consecutive worlds.  A step launches step_kernel
// once per chunk of tiles (as many tiles as the device keeps resident), one
// 128-thread block per tile, which runs three phases:
//   collide (all warps)  reads the caller's AoS worlds with coalesced row
//       transfers, builds the per-lane solver columns of the tile's
//       workspace slot, runs broadphase and narrowphase spread over
//       (pair, world) and (candidate, world), and prepares contacts and
//       joints (b3x_phases.cuh);
//   solve (warp 0, lane = world)  warm starts and runs the substeps:
//       Gauss-Seidel sweeps over contacts / joints streamed through shared
//       memory with TMA bulk copies, body state in shared memory
//       (b3x_solver.cuh);
//   write-back (all warps)  finalizes the bodies and writes bodies,
//       contacts, joints and header counts back to the AoS worlds, again as
//       coalesced rows (b3x_phases.cuh).
// Every loop is bounded by the world's capacities; the solver's pipeline
// waits are bounded and report through b3x_fault_flags().
//
// Small worlds (a few bodies, shapes and contacts: the hover task) have too
// little work per world for the tile phases to pay for their barriers; their
// step is small_step_kernel: 32 worlds per block staged whole into shared
// memory with asynchronous copies, one thread stepping one world there with
// the per-world step of b3x_world_step.cuh, then copied back.
//
// Arithmetic.  The per-world work follows the reference's default
// b3_step (src/puffysics/09_step.inl:183-258) operation by operation; the
// library is compiled with -fmad=false and IEEE division / square root so
// the results equal the reference CPU build (-ffp-contract=off) bit for bit,
// atan2f (revolute twist) excepted.  Reordering is limited to hoisting pure
// values (shape world poses, gated inverse masses, step softness) and to
// evaluating the side-effect-free broadphase filters in a cheaper order.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "puffysics_b200.h"
#include "b3x_layout.cuh"
#include "b3x_solver.cuh"
#include "b3x_phases.cuh"
#include "b3x_world_step.cuh"

namespace b3x {

// Set (never cleared by the kernels) when a pipeline wait gave up; read with
// b3x_fault_flags().  Not expected to happen: it would mean a bulk copy never
// completed.
__device__ int g_fault;

// Block-wide phase runner: every thread runs the phase, then the block meets.
struct DevExec {
    template <class F>
    __host__ __device__ __forceinline__ void each(F&& f) {
#if defined(__CUDA_ARCH__)
        f((int)threadIdx.x);
        __syncthreads();
#else
        (void)f;
#endif
    }
};

// Shared memory of a step block: the collide and write-back phases use it
// as their block state; the solve phase as the streaming stages, their
// mbarriers, then the body columns that live on chip, most-used first: the
// velocities (every contact and joint row reads and writes them), the pose
// deltas, the constants.  What stays off chip is read from the workspace
// (through L1 for the constants, which the solve does not write).
constexpr size_t kStageBytes = (size_t)kStages * kStreamWords * kLanes * sizeof(float);
constexpr size_t kBarBytes = 64;
enum BodyPlace : int { kBodyNone = 0, kBodyVel = 1, kBodyState = 2, kBodyAll = 3 };

// Warp 0's part of the step: warm start and substeps of the tile's 32 worlds.
// Returns false when a pipeline wait gave up (nothing of the tile is then
// written back: the step is abandoned for these worlds).
template <int kBody, bool kInterleave>
__device__ bool solve_tile(const Args& a, unsigned char* smem_raw) {
    const int lane = threadIdx.x & 31;
    float* slot = slot_of(a, blockIdx.x);
    Pipe P;
    P.buf = reinterpret_cast<float*>(smem_raw);
    P.bar = reinterpret_cast<uint64_t*>(smem_raw + kStageBytes);
    pipe_init(P);
    float* gv = slot + a.SP.body;
    float* gp = slot + a.SP.bodyp;
    const float* gk = slot + a.SP.bodyk;
    float* sv = reinterpret_cast<float*>(smem_raw + kStageBytes + kBarBytes);
    float* sp = sv + (size_t)a.L.B * NBF * kLanes;
    float* sk = sp + (size_t)a.L.B * NBP * kLanes;
    const int nb = warp_max(ldi(slot + a.SP.rec + lane, RNB));
    // each lane copies its own columns
    if (kBody >= kBodyVel)
        for (int idx = lane; idx < nb * NBF * kLanes; idx += kLanes) sv[idx] = gv[idx];
    if (kBody >= kBodyState)
        for (int idx = lane; idx < nb * NBP * kLanes; idx += kLanes) sp[idx] = gp[idx];
    if (kBody == kBodyAll)
        for (int idx = lane; idx < nb * NBC * kLanes; idx += kLanes) sk[idx] = gk[idx];
    float* bc = (kBody >= kBodyVel ? sv : gv) + lane;
    float* bp = (kBody >= kBodyState ? sp : gp) + lane;
    const float* bk = (kBody == kBodyAll ? sk : gk) + lane;
    const bool ok = solve_world<kInterleave>(a, slot, lane, bc, bp, bk, P);
    if (ok && kBody >= kBodyVel)
        for (int idx = lane; idx < nb * NBF * kLanes; idx += kLanes) gv[idx] = sv[idx];
    if (ok && kBody >= kBodyState)
        for (int idx = lane; idx < nb * NBP * kLanes; idx += kLanes) gp[idx] = sp[idx];
    __syncwarp();
    if (lane == 0) {
        // the barriers' memory is reused by the write-back
        for (int s = 0; s < kStages; s++)
            asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_addr(&P.bar[s])) : "memory");
        if (!ok) atomicExch(&g_fault, 1);
    }
    return ok;
}

// One block per tile: collide (all warps), solve (warp 0), write-back (all
// warps).  kRes: the worlds are the resident world columns (a.res) instead
// of the caller's AoS array.
template <int kBody, bool kInterleave = false, bool kRes = false>
__global__ void __launch_bounds__(kCta, 4) step_kernel(Args a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ int solved;
    DevExec x;
    collide_tile<kRes>(x, a, blockIdx.x, *reinterpret_cast<CollideShared*>(smem_raw));
    // the solve's bulk copies (async proxy) read workspace data every thread
    // wrote and reuse shared memory the collide phase accessed, both through
    // the generic proxy: each thread orders its accesses before the barrier
    asm volatile("fence.proxy.async;" ::: "memory");
    __syncthreads();
    if (threadIdx.x < kLanes) {
        const bool ok = solve_tile<kBody, kInterleave>(a, smem_raw);
        if (threadIdx.x == 0) solved = ok;
    } else if constexpr (kRes) {
        // the other warps write the contact and joint words the solve does not change
        if (!(a.flags & kStepStateOnly)) o_rows_early(a, a.tile0 + blockIdx.x, slot_of(a, blockIdx.x),
                                                          threadIdx.x - kLanes);
    }
    __syncthreads();
    if (!solved) return;
    out_tile<kRes>(x, a, blockIdx.x, *reinterpret_cast<OutShared*>(smem_raw));
}

// ---- small worlds -----------------------------------------------------------------
// Capacity bounds of the small-world step (its per-world scratch is sized by
// them) and the shared memory its 32 staged worlds may take.
constexpr int kSmallB = 8, kSmallS = 8, kSmallC = 8;
constexpr size_t kSmallSmemMax = 112 * 1024;
#ifndef SMALL_WORLDS_PER_BLOCK
#define SMALL_WORLDS_PER_BLOCK 8
#endif
using SmallView = one::WorldView<kSmallB, kSmallS, kSmallC>;

// 8-byte words between staged worlds: the world rounded up so that
// consecutive threads' worlds start in different bank pairs (the word stride
// is 2 x odd, the least conflict an 8-byte aligned stride allows).
static inline unsigned small_stride_words(const Layout& L) {
    unsigned w = L.size / 8;
    if (w % 2 == 0) w++;
    return w;
}

__device__ __forceinline__ void async_copy8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

// One block of 32 threads per group of kSmallWorlds worlds: stage the
// group's selected worlds, step each on its own thread, write them back
// (unselected worlds are neither read nor written).  Groups smaller than a
// warp spread the worlds over more SMs and let several warps of one SM share
// the instruction fetches of this long per-world program.
constexpr int kSmallWorlds = SMALL_WORLDS_PER_BLOCK;
static_assert(kLanes % kSmallWorlds == 0, "a small-world group lies inside one tile");
template <bool kRes = false>
__global__ void __launch_bounds__(kLanes) small_step_kernel(Args a, unsigned stride_words) {
    extern __shared__ __align__(16) unsigned char small_smem[];
    uint64_t* sw = reinterpret_cast<uint64_t*>(small_smem);
    const int lane = threadIdx.x;
    const long long first = (long long)blockIdx.x * kSmallWorlds;
    const unsigned words = a.L.size / 8;
    const long long wi = first + lane;
    const bool live = lane < kSmallWorlds && wi < a.count && (!a.active || a.active[wi]);
    const unsigned live_mask = __ballot_sync(0xffffffffu, live);
    auto world_ptr = [&](int l) {
        return reinterpret_cast<uint64_t*>(a.data + (size_t)(first + l) * a.stride + a.offset);
    };
    // resident columns: the group's worlds are lanes [lt, lt + kSmallWorlds)
    // of one tile; thread t moves 4-byte word t / kSmallWorlds (+ 4 per round)
    // of group world t % kSmallWorlds, so each round reads or writes four
    // 32-byte runs
    const int tile = (int)(first / kLanes), lt = (int)(first % kLanes);
    const int rg = lane % kSmallWorlds, rw = lane / kSmallWorlds;
    constexpr int kRoundWords = kLanes / kSmallWorlds;
    if constexpr (kRes) {
        if ((live_mask >> rg) & 1u) {
            float* dst = reinterpret_cast<float*>(sw + (size_t)rg * stride_words);
            for (unsigned w = rw; w < 2 * words; w += kRoundWords)
                async_copy4_world(dst + w, res_word(a, tile, w, lt + rg));
        }
    } else {
        for (int l = 0; l < kSmallWorlds; l++) {
            if (!((live_mask >> l) & 1u)) continue;
            const uint64_t* src = world_ptr(l);
            uint64_t* dst = sw + (size_t)l * stride_words;
            for (unsigned idx = lane; idx < words; idx += kLanes) async_copy8(dst + idx, src + idx);
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
    if (live) {
        unsigned char* base = small_smem + (size_t)lane * stride_words * 8;
        SmallView v;
        v.h = reinterpret_cast<B3World*>(base);
        v.bodies = reinterpret_cast<B3Body*>(base + B3X_WORLD_HEADER_BYTES);
        v.shapes = reinterpret_cast<B3Shape*>(base + a.L.shape_off);
        v.contacts = reinterpret_cast<B3Contact*>(base + a.L.contact_off);
        v.joints = reinterpret_cast<B3Joint*>(base + a.L.joint_off);
        v.cap_b = a.L.B;
        v.cap_s = a.L.S;
        v.cap_c = a.L.C;
        v.cap_j = a.L.J;
        one::step_view(v, a.dt, a.substeps, a.joint_iters, a.relax_iters, a.flags);
    }
    __syncwarp();
    if constexpr (kRes) {
        if ((live_mask >> rg) & 1u) {
            const float* src = reinterpret_cast<const float*>(sw + (size_t)rg * stride_words);
            for (unsigned w = rw; w < 2 * words; w += kRoundWords) store_world(res_word(a, tile, w, lt + rg), src[w]);
        }
    } else {
        for (int l = 0; l < kSmallWorlds; l++) {
            if (!((live_mask >> l) & 1u)) continue;
            uint64_t* dst = world_ptr(l);
            const uint64_t* src = sw + (size_t)l * stride_words;
            for (unsigned idx = lane; idx < words; idx += kLanes) dst[idx] = src[idx];
        }
    }
}

// ---- restore, actions --------------------------------------------------------
// One warp per world, 8-byte words, coalesced on both sides.
__global__ void restore_kernel(unsigned char* data, unsigned long long stride, unsigned long long offset, int count,
        const unsigned long long* initial, const unsigned char* reset, unsigned words) {
    const int lane = threadIdx.x & 31;
    const int warps = (int)(gridDim.x * (blockDim.x >> 5));
    for (int wi = (int)(blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)); wi < count; wi += warps) {
        if (reset && !reset[wi]) continue;
        unsigned long long* dst = reinterpret_cast<unsigned long long*>(data + (size_t)wi * stride + offset);
        const unsigned long long* src = initial + (size_t)wi * words;
        for (unsigned w = lane; w < words; w += 32) dst[w] = src[w];
    }
}

// A world's 4-byte words, in the caller's AoS array or in the resident
// columns (word w of lane l of a tile at base[w * 32]).
struct AosAt {
    unsigned char* base;
    __device__ __forceinline__ float& operator()(size_t w) const { return reinterpret_cast<float*>(base)[w]; }
};
struct ColAt {
    float* base;
    __device__ __forceinline__ float& operator()(size_t w) const { return base[w * kLanes]; }
};
__device__ __forceinline__ AosAt aos_at(unsigned char* data, unsigned long long stride, unsigned long long offset,
        int wi) {
    return {data + (size_t)wi * stride + offset};
}
__device__ __forceinline__ ColAt col_at(float* res, unsigned long long W, int wi) {
    return {res + (size_t)(wi / kLanes) * W * kLanes + (wi % kLanes)};
}

// Actions of one world (b3_apply_force / b3_apply_torque /
// b3_apply_linear_impulse, 09_step.inl:132-146, and the spring target of
// b3_joint_set_spring) on its words.
template <class At>
__device__ void apply_world(const At& w, const Layout& L, int kind, int index, const float* v, int vpw) {
    if (kind == B3X_ACTION_JOINT_TARGET) {
        const int nj = clampi(b3x_f2i(w(HNJ)), 0, L.J);
        for (int k = 0; k < vpw; k++)
            if (index + k >= 0 && index + k < nj)
                w(L.joint_off / 4 + (size_t)(index + k) * NVW + VTA) = b3_clamp(v[k], -B3_PI, B3_PI);
        return;
    }
    const int nb = clampi(b3x_f2i(w(HNB)), 0, L.B);
    for (int k = 0; 3 * k + 2 < vpw; k++) {
        const int bi = index + k;
        if (bi < 0 || bi >= nb) continue;
        const size_t b = B3X_WORLD_HEADER_BYTES / 4 + (size_t)bi * NYW;
        const float x[3] = {v[3 * k], v[3 * k + 1], v[3 * k + 2]};
        if (kind == B3X_ACTION_FORCE) {
            for (int c = 0; c < 3; c++) w(b + YF + c) = w(b + YF + c) + x[c];
        } else if (kind == B3X_ACTION_TORQUE) {
            for (int c = 0; c < 3; c++) w(b + YT + c) = w(b + YT + c) + x[c];
        } else if (b3x_f2i(w(b + YTYPE)) == B3_DYNAMIC) {
            const float im = w(b + YIM);
            for (int c = 0; c < 3; c++) w(b + YLV + c) = w(b + YLV + c) + im * x[c];
        }
    }
}

__global__ void apply_kernel(unsigned char* data, unsigned long long stride, unsigned long long offset, int count,
        Layout L, int kind, int index, const float* values, int vpw, const unsigned char* active) {
    int wi = blockIdx.x * blockDim.x + threadIdx.x;
    if (wi >= count || (active && !active[wi])) return;
    apply_world(aos_at(data, stride, offset, wi), L, kind, index, values + (size_t)wi * vpw, vpw);
}

__global__ void apply_columns_kernel(float* res, unsigned long long W, int count, Layout L, int kind, int index,
        const float* values, int vpw, const unsigned char* active) {
    int wi = blockIdx.x * blockDim.x + threadIdx.x;
    if (wi >= count || (active && !active[wi])) return;
    apply_world(col_at(res, W, wi), L, kind, index, values + (size_t)wi * vpw, vpw);
}

// Position, rotation (x y z s), lin_vel, ang_vel of one body (NaN past the
// world's bodies).
template <class At>
__device__ void observe_world(const At& w, int body, float* o) {
    if (body < 0 || body >= b3x_f2i(w(HNB))) {
        for (int k = 0; k < 13; k++) o[k] = NAN;
        return;
    }
    const size_t b = B3X_WORLD_HEADER_BYTES / 4 + (size_t)body * NYW;
    for (int k = 0; k < 7; k++) o[k] = w(b + YPOS + k);    // position, rotation
    for (int k = 0; k < 3; k++) o[7 + k] = w(b + YLV + k);
    for (int k = 0; k < 3; k++) o[10 + k] = w(b + YAV + k);
}

// One thread per world.
__global__ void observe_kernel(const unsigned char* data, unsigned long long stride, unsigned long long offset,
        int count, int body, float* out) {
    int wi = blockIdx.x * blockDim.x + threadIdx.x;
    if (wi >= count) return;
    observe_world(aos_at(const_cast<unsigned char*>(data), stride, offset, wi), body, out + (size_t)wi * 13);
}

__global__ void observe_columns_kernel(const float* res, unsigned long long W, int count, int body, float* out) {
    int wi = blockIdx.x * blockDim.x + threadIdx.x;
    if (wi >= count) return;
    observe_world(col_at(const_cast<float*>(res), W, wi), body, out + (size_t)wi * 13);
}

// ---- resident world columns: transposes between the AoS worlds and the
// columns, one block per tile, kTrChunk words of its 32 worlds per round
// through shared memory (AoS side: consecutive lanes read or write
// consecutive words of one world; column side: one word of the 32 worlds,
// one 128-byte line).  Only selected worlds move; a tile without any is
// skipped.
constexpr int kTrChunk = 64;
template <bool kIn>
__global__ void __launch_bounds__(kCta) columns_kernel(float* res, unsigned long long W, unsigned char* data,
        unsigned long long stride, unsigned long long offset, int count, const unsigned char* select) {
    __shared__ float buf[kLanes][kTrChunk + 1];
    __shared__ unsigned sel;
    const int tile = blockIdx.x, t = threadIdx.x;
    if (t < kLanes) {
        const int wi = tile * kLanes + t;
        const unsigned m = __ballot_sync(0xffffffffu, wi < count && (!select || select[wi]));
        if (t == 0) sel = m;
    }
    __syncthreads();
    const unsigned m = sel;
    if (m == 0) return;
    for (unsigned long long w0 = 0; w0 < W; w0 += kTrChunk) {
        const int n = W - w0 < (unsigned long long)kTrChunk ? (int)(W - w0) : kTrChunk;
        if (kIn) {
            for (int l = t >> 5; l < kLanes; l += kCtaWarps) {
                if (!((m >> l) & 1u)) continue;
                const float* src = reinterpret_cast<const float*>(data + (size_t)(tile * kLanes + l) * stride
                                                                  + offset) + w0;
                for (int i = t & 31; i < n; i += kLanes) buf[l][i] = src[i];
            }
            __syncthreads();
            for (int idx = t; idx < n * kLanes; idx += kCta) {
                const int l = idx & 31, i = idx >> 5;
                if ((m >> l) & 1u) res[((size_t)tile * W + w0 + i) * kLanes + l] = buf[l][i];
            }
        } else {
            for (int idx = t; idx < n * kLanes; idx += kCta) {
                const int l = idx & 31, i = idx >> 5;
                if ((m >> l) & 1u) buf[l][i] = res[((size_t)tile * W + w0 + i) * kLanes + l];
            }
            __syncthreads();
            for (int l = t >> 5; l < kLanes; l += kCtaWarps) {
                if (!((m >> l) & 1u)) continue;
                float* dst = reinterpret_cast<float*>(data + (size_t)(tile * kLanes + l) * stride + offset) + w0;
                for (int i = t & 31; i < n; i += kLanes) dst[i] = buf[l][i];
            }
        }
        __syncthreads();
    }
}

// ---- host side --------------------------------------------------------------
struct Plan {
    bool small;              // the small-world step (no workspace)
    size_t small_smem;       // its dynamic shared memory per block
    unsigned small_stride;   // its staged world stride (8-byte words)
    int body;                // BodyPlace of the solve
    Space SP;
    size_t smem_bytes;       // dynamic shared memory of a step block
    size_t tile_bytes;       // one tile's workspace slot
    int chunk_tiles;         // tiles per launch with the default workspace
    size_t ws_bytes;         // the default workspace (chunk_tiles slots)
};

static std::mutex g_mutex;
static std::map<std::pair<int, unsigned long long>, Plan> g_plans;

// ---- workspaces ------------------------------------------------------------------
// A step never allocates.  Its workspace is, in order of preference:
//  * the caller's (b3x_batch_step_gpu_ws);
//  * the one reserved for the calling stream by b3x_reserve_workspace, an
//    explicit set-up call (the only place the library allocates device
//    memory), freed by b3x_release_workspaces;
//  * the library's fixed array g_step_scratch, which every device that loads
//    the library holds until exit.  Steps on it run as many tiles per launch
//    as its slots hold.  Calls from different streams are ordered on the GPU
//    through an event, so they cannot overlap on the array; a call made while
//    its stream is being captured into a CUDA graph is ordered only by that
//    stream (reserve a workspace for capture streams).
struct Reserved {
    void* ptr;
    size_t bytes;
};
static std::mutex g_ws_mutex;
static std::map<std::pair<int, void*>, Reserved> g_reserved;   // (device, stream)

constexpr size_t kStepScratchBytes = 128ull << 20;
static __device__ __align__(256) unsigned char g_step_scratch[kStepScratchBytes];
struct FixedUse {
    cudaEvent_t done = nullptr;   // recorded after the last launch on the array
    void* last = nullptr;         // the stream of that launch
    bool pending = false;         // `done` has been recorded
};
static std::mutex g_fixed_mutex;  // held across a call's launches on the array
static std::map<int, FixedUse> g_fixed;   // per device

// The allocation-free entry's own array (b3x_batch_step_gpu_noalloc).
constexpr size_t kNoAllocScratchBytes = 64ull << 20;   // 64 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Resident blocks per SM the default chunk and the shared memory budget are
// sized for.
static constexpr int kChunkBlocksPerSM = 4;

static cudaError_t make_plan(int dev, unsigned long long sig, const Layout& L, Plan* out) {
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_plans.find({dev, sig});
    if (it != g_plans.end()) {
        *out = it->second;
        return cudaSuccess;
    }
    Plan p;
    p.SP = space_from_layout(L);
    p.tile_bytes = (size_t)p.SP.tile_words * sizeof(float);
    int sms = 0, per_sm = 0, reserved = 0;
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    if (e != cudaSuccess) return e;
    // The dynamic shared memory cap is a property of the kernel function, not
    // of a plan: raise it once to the device's opt-in maximum so plans of
    // different capacity configurations never lower it under one another.
    int optin = 0;
    e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    // (the cap excludes the kernel's static shared memory)
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, step_kernel<kBodyAll>);
    if (e != cudaSuccess) return e;
    const int cap = optin - (int)fa.sharedSizeBytes;
    // Body columns go on chip as far as kChunkBlocksPerSM blocks still fit
    // on an SM: velocities, then pose deltas, then constants.
    const size_t budget = (size_t)(per_sm / kChunkBlocksPerSM - reserved) - fa.sharedSizeBytes;
    const size_t col = (size_t)L.B * kLanes * sizeof(float);
    const size_t base = kStageBytes + kBarBytes;
    const size_t upto[4] = {base, base + NBF * col, base + (NBF + NBP) * col, base + (NBF + NBP + NBC) * col};
    p.body = kBodyNone;
    for (int m = kBodyAll; m > kBodyNone; m--)
        if (upto[m] <= budget) {
            p.body = m;
            break;
        }
    p.smem_bytes = upto[p.body];
    if (p.smem_bytes < sizeof(CollideShared)) p.smem_bytes = sizeof(CollideShared);
    if (p.smem_bytes < sizeof(OutShared)) p.smem_bytes = sizeof(OutShared);
    if (p.smem_bytes > (size_t)cap) return cudaErrorInvalidValue;
    for (auto fn : {step_kernel<kBodyNone>, step_kernel<kBodyVel>, step_kernel<kBodyState>, step_kernel<kBodyAll>,
                    step_kernel<kBodyNone, true>, step_kernel<kBodyVel, true>, step_kernel<kBodyState, true>,
                    step_kernel<kBodyAll, true>,
                    step_kernel<kBodyNone, false, true>, step_kernel<kBodyVel, false, true>,
                    step_kernel<kBodyState, false, true>, step_kernel<kBodyAll, false, true>,
                    step_kernel<kBodyNone, true, true>, step_kernel<kBodyVel, true, true>,
                    step_kernel<kBodyState, true, true>, step_kernel<kBodyAll, true, true>}) {
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
        if (e != cudaSuccess) return e;
    }
    p.chunk_tiles = sms * kChunkBlocksPerSM;
    p.ws_bytes = (size_t)p.chunk_tiles * p.tile_bytes;
    p.small_stride = small_stride_words(L);
    p.small_smem = (size_t)kSmallWorlds * p.small_stride * 8;
    p.small = L.B <= kSmallB && L.S <= kSmallS && L.C <= kSmallC && p.small_smem <= kSmallSmemMax
              && p.small_smem <= (size_t)optin;
    if (p.small) {
        e = cudaFuncSetAttribute(small_step_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)p.small_smem);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(small_step_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)p.small_smem);
        if (e != cudaSuccess) return e;
    }
    g_plans[{dev, sig}] = p;
    *out = p;
    return cudaSuccess;
}

static bool batch_ok(const B3Batch& b, size_t world_bytes) {
    if (b.count < 0) return false;
    if (b.count == 0) return true;
    return b.data != nullptr && b.stride >= world_bytes && b.world_offset <= b.stride - world_bytes
        && (size_t)b.count <= SIZE_MAX / b.stride;
}

static bool aligned8(const B3Batch& b) {
    return (((uintptr_t)b.data + b.world_offset) % 8 == 0) && (b.stride % 8 == 0);
}

// The worlds a step runs on: the caller's AoS batch, or resident world
// columns (res != null, the b3x_engine_* entry points).
struct Worlds {
    unsigned char* data;
    size_t stride, offset;
    int count;
    float* res;
};

static Worlds aos_worlds(const B3Batch& b) { return {(unsigned char*)b.data, b.stride, b.world_offset, b.count, nullptr}; }

static Args step_args(const Worlds& w, float dt, int substeps, const unsigned char* active, const Layout& L, int ji,
        int ri, int flags, const Plan& p) {
    Args a;
    a.data = w.data;
    a.stride = w.stride;
    a.offset = w.offset;
    a.count = w.count;
    a.active = active;
    a.dt = dt;
    a.substeps = substeps;
    a.joint_iters = ji;
    a.relax_iters = ri;
    a.flags = flags;
    a.L = L;
    a.SP = p.SP;
    a.ws = nullptr;
    a.tile0 = 0;
    a.res = w.res;
    a.resW = L.size / 4;
    return a;
}

template <bool kI, bool kR>
static void launch_tiles(const Plan& p, int nt, cudaStream_t stream, const Args& a) {
    if (p.body == kBodyAll) step_kernel<kBodyAll, kI, kR><<<nt, kCta, p.smem_bytes, stream>>>(a);
    else if (p.body == kBodyState) step_kernel<kBodyState, kI, kR><<<nt, kCta, p.smem_bytes, stream>>>(a);
    else if (p.body == kBodyVel) step_kernel<kBodyVel, kI, kR><<<nt, kCta, p.smem_bytes, stream>>>(a);
    else step_kernel<kBodyNone, kI, kR><<<nt, kCta, p.smem_bytes, stream>>>(a);
}

// The step over chunks of `chunk` tiles, one step_kernel launch per chunk.
static cudaError_t launch_step(const Worlds& w, float dt, int substeps, const unsigned char* active,
        cudaStream_t stream, const Layout& L, int ji, int ri, int flags, const Plan& p, void* ws, int chunk) {
    Args a = step_args(w, dt, substeps, active, L, ji, ri, flags, p);
    a.ws = (float*)ws;
    const bool il = (flags & kStepInterleaveContacts) != 0, res = w.res != nullptr;
    const int ntiles = (w.count + kLanes - 1) / kLanes;
    for (int t0 = 0; t0 < ntiles; t0 += chunk) {
        const int nt = ntiles - t0 < chunk ? ntiles - t0 : chunk;
        a.tile0 = t0;
        if (il) res ? launch_tiles<true, true>(p, nt, stream, a) : launch_tiles<true, false>(p, nt, stream, a);
        else res ? launch_tiles<false, true>(p, nt, stream, a) : launch_tiles<false, false>(p, nt, stream, a);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace b3x

using namespace b3x;

extern "C" {

B3X_API const char* b3x_version(void) { return "puffysics_b200 0.1 (sm_100a)"; }

B3X_API size_t b3x_world_bytes(unsigned long long sig) {
    Layout L;
    return layout_from_signature(sig, &L) ? L.size : 0;
}

B3X_API size_t b3x_workspace_bytes(unsigned long long sig, int device) {
    Layout L;
    if (!layout_from_signature(sig, &L)) return 0;
    Plan p;
    if (make_plan(device, sig, L, &p) != cudaSuccess) return 0;
    return p.ws_bytes;
}

B3X_API size_t b3x_workspace_slot_bytes(unsigned long long sig) {
    Layout L;
    if (!layout_from_signature(sig, &L)) return 0;
    return (size_t)space_from_layout(L).tile_words * sizeof(float);
}

B3X_API int b3x_step_launches(unsigned long long sig, int count, int device) {
    Layout L;
    if (!layout_from_signature(sig, &L) || count < 0) return 0;
    Plan p;
    if (make_plan(device, sig, L, &p) != cudaSuccess) return 0;
    const int ntiles = (count + kLanes - 1) / kLanes;
    if (p.small) return ntiles > 0 ? 1 : 0;
    return (ntiles + p.chunk_tiles - 1) / p.chunk_tiles;
}

// Where a step's workspace comes from (see "workspaces" above).
enum class WsFrom { kLibrary, kCaller, kNoAlloc };

// Chunked launches on the library's fixed array, ordered after the previous
// user of the array when that was another stream.
static cudaError_t step_on_fixed(int dev, const Worlds& batch, float dt, int substeps,
        const unsigned char* active, void* stream, const Layout& L, int ji, int ri, int flags, const Plan& p) {
    void* ws = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ws, g_step_scratch);
    if (e != cudaSuccess) return e;
    const long long slots = (long long)(kStepScratchBytes / p.tile_bytes);
    if (slots < 1) return cudaErrorMemoryAllocation;   // a reserved workspace is needed
    const int chunk = (int)(slots < p.chunk_tiles ? slots : p.chunk_tiles);
    std::lock_guard<std::mutex> lock(g_fixed_mutex);
    FixedUse& f = g_fixed[dev];
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing((cudaStream_t)stream, &cs) != cudaSuccess) {
        (void)cudaGetLastError();
        cs = cudaStreamCaptureStatusActive;
    }
    const bool ordered = cs == cudaStreamCaptureStatusNone;
    if (ordered) {
        if (!f.done) {
            e = cudaEventCreateWithFlags(&f.done, cudaEventDisableTiming);
            if (e != cudaSuccess) return e;
        }
        if (f.pending && f.last != stream) {
            e = cudaStreamWaitEvent((cudaStream_t)stream, f.done, 0);
            if (e != cudaSuccess) return e;
        }
    }
    e = launch_step(batch, dt, substeps, active, (cudaStream_t)stream, L, ji, ri, flags, p, ws, chunk);
    if (e != cudaSuccess || !ordered) return e;
    e = cudaEventRecord(f.done, (cudaStream_t)stream);
    if (e != cudaSuccess) return e;
    f.last = stream;
    f.pending = true;
    return cudaSuccess;
}

// The step of validated worlds: the small-world kernel, or the tile kernel on
// the workspace `from` names.
static int run_step(const Worlds& w, float dt, int substeps, const unsigned char* active, void* stream,
        unsigned long long sig, const Layout& L, int ji, int ri, WsFrom from, void* ws, size_t ws_bytes, int flags) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    Plan p;
    e = make_plan(dev, sig, L, &p);
    if (e != cudaSuccess) return e;
    if (p.small) {
        // no workspace: the worlds are stepped in shared memory
        Args a = step_args(w, dt, substeps, active, L, ji, ri, flags, p);
        const unsigned groups = (unsigned)((w.count + kSmallWorlds - 1) / kSmallWorlds);
        if (w.res) small_step_kernel<true><<<groups, kLanes, p.small_smem, (cudaStream_t)stream>>>(a, p.small_stride);
        else small_step_kernel<false><<<groups, kLanes, p.small_smem, (cudaStream_t)stream>>>(a, p.small_stride);
        return (int)cudaGetLastError();
    }
    if (from == WsFrom::kLibrary) {
        {
            std::lock_guard<std::mutex> lock(g_ws_mutex);
            auto it = g_reserved.find({dev, stream});
            if (it != g_reserved.end() && it->second.bytes >= p.tile_bytes) {
                ws = it->second.ptr;
                ws_bytes = it->second.bytes;
            }
        }
        if (ws == nullptr)
            return step_on_fixed(dev, w, dt, substeps, active, stream, L, ji, ri, flags, p);
    } else if (from == WsFrom::kNoAlloc) {
        // looked up on every call: the address is per device and per context
        e = cudaGetSymbolAddress(&ws, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        ws_bytes = kNoAllocScratchBytes;
        if (p.tile_bytes > kNoAllocScratchBytes) return cudaErrorInvalidValue;
    }
    if (ws == nullptr || ((uintptr_t)ws % 256) != 0) return cudaErrorInvalidValue;
    // A smaller caller workspace simply runs fewer tiles per launch.
    long long slots = (long long)(ws_bytes / p.tile_bytes);
    if (slots < 1) return cudaErrorInvalidValue;
    int chunk = (int)(slots < p.chunk_tiles ? slots : p.chunk_tiles);
    return launch_step(w, dt, substeps, active, (cudaStream_t)stream, L, ji, ri, flags, p, ws, chunk);
}

static bool step_params_ok(float dt, int substeps, int ji, int ri, int flags,
        int allowed = kStepInterleaveContacts | kStepSkipRestitution) {
    return std::isfinite(dt) && dt >= 0 && substeps >= 1 && ji >= 1 && ri >= 1 && (flags & ~allowed) == 0;
}

static int step_common(B3Batch batch, float dt, int substeps, const unsigned char* active, void* stream,
        unsigned long long sig, int ji, int ri, WsFrom from, void* ws, size_t ws_bytes, int flags = 0) {
    Layout L;
    if (!layout_from_signature(sig, &L)) return cudaErrorInvalidValue;
    if (!batch_ok(batch, L.size) || !step_params_ok(dt, substeps, ji, ri, flags)) return cudaErrorInvalidValue;
    if (batch.count == 0 || dt == 0) return cudaSuccess;
    if (!aligned8(batch)) return cudaErrorInvalidValue;
    return run_step(aos_worlds(batch), dt, substeps, active, stream, sig, L, ji, ri, from, ws, ws_bytes, flags);
}

B3X_API int b3x_batch_step_gpu(B3Batch batch, float dt, int substeps, const unsigned char* active, void* stream,
        unsigned long long sig, int ji, int ri) {
    return step_common(batch, dt, substeps, active, stream, sig, ji, ri, WsFrom::kLibrary, nullptr, 0);
}

B3X_API int b3x_batch_step_gpu_flags(B3Batch batch, float dt, int substeps, const unsigned char* active,
        void* stream, unsigned long long sig, int ji, int ri, int flags) {
    return step_common(batch, dt, substeps, active, stream, sig, ji, ri, WsFrom::kLibrary, nullptr, 0, flags);
}

B3X_API int b3x_batch_step_gpu_ws(B3Batch batch, float dt, int substeps, const unsigned char* active, void* stream,
        unsigned long long sig, int ji, int ri, void* ws, size_t ws_bytes) {
    return step_common(batch, dt, substeps, active, stream, sig, ji, ri, WsFrom::kCaller, ws, ws_bytes);
}

// Set-up call: a workspace for steps of this capacity configuration on
// `stream` (current device), large enough for one launch per resident wave.
// Grows an existing reservation of the stream (synchronising, as cudaFree
// does); a large enough one is kept.
B3X_API int b3x_reserve_workspace(void* stream, unsigned long long sig) {
    Layout L;
    if (!layout_from_signature(sig, &L)) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    Plan p;
    e = make_plan(dev, sig, L, &p);
    if (e != cudaSuccess) return e;
    if (p.small) return cudaSuccess;   // stepped in shared memory, no workspace
    std::lock_guard<std::mutex> lock(g_ws_mutex);
    auto key = std::make_pair(dev, stream);
    auto it = g_reserved.find(key);
    if (it != g_reserved.end()) {
        if (it->second.bytes >= p.ws_bytes) return cudaSuccess;
        e = cudaFree(it->second.ptr);
        g_reserved.erase(it);
        if (e != cudaSuccess) return e;
    }
    void* mem = nullptr;
    e = cudaMalloc(&mem, p.ws_bytes);
    if (e != cudaSuccess) return e;
    g_reserved[key] = {mem, p.ws_bytes};
    return cudaSuccess;
}

// Frees every workspace reserved on the current device (synchronising, as
// cudaFree does); steps on those streams fall back to the library's array.
B3X_API int b3x_release_workspaces(void) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    cudaError_t first = cudaSuccess;
    std::lock_guard<std::mutex> lock(g_ws_mutex);
    for (auto it = g_reserved.begin(); it != g_reserved.end();) {
        if (it->first.first != dev) {
            ++it;
            continue;
        }
        e = cudaFree(it->second.ptr);
        if (e != cudaSuccess && first == cudaSuccess) first = e;
        it = g_reserved.erase(it);
    }
    return first;
}

// Bytes reserved for `stream` on the current device (0 if none).
B3X_API size_t b3x_reserved_bytes(void* stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lock(g_ws_mutex);
    auto it = g_reserved.find({dev, stream});
    return it == g_reserved.end() ? 0 : it->second.bytes;
}

B3X_API int b3x_batch_restore_gpu(B3Batch batch, const void* initial, const unsigned char* reset, void* stream,
        unsigned long long sig) {
    Layout L;
    if (!layout_from_signature(sig, &L)) return cudaErrorInvalidValue;
    if (!batch_ok(batch, L.size) || (batch.count && !initial)) return cudaErrorInvalidValue;
    if (!batch.count) return cudaSuccess;
    if (!aligned8(batch) || ((uintptr_t)initial % 8) != 0) return cudaErrorInvalidValue;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int warps_needed = batch.count;
    int blocks = (warps_needed + 7) / 8;
    int cap = sms * 16;
    if (blocks > cap) blocks = cap;
    restore_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((unsigned char*)batch.data, batch.stride,
        batch.world_offset, batch.count, (const unsigned long long*)initial, reset, L.size / 8);
    return cudaGetLastError();
}

B3X_API int b3x_batch_apply_gpu(B3Batch batch, int kind, int index, const float* values, int vpw,
        const unsigned char* active, void* stream, unsigned long long sig) {
    Layout L;
    if (!layout_from_signature(sig, &L)) return cudaErrorInvalidValue;
    if (!batch_ok(batch, L.size) || kind < 0 || kind > 3 || vpw < 1 || (batch.count && !values))
        return cudaErrorInvalidValue;
    if (kind != B3X_ACTION_JOINT_TARGET && vpw % 3 != 0) return cudaErrorInvalidValue;
    if (!batch.count) return cudaSuccess;
    if (!aligned8(batch)) return cudaErrorInvalidValue;
    int blocks = (batch.count + 127) / 128;
    apply_kernel<<<blocks, 128, 0, (cudaStream_t)stream>>>((unsigned char*)batch.data, batch.stride,
        batch.world_offset, batch.count, L, kind, index, values, vpw, active);
    return cudaGetLastError();
}

// Nonzero if a step kernel on the current device ever abandoned a step
// because a pipeline wait gave up; `clear` resets the flag.  Synchronises.
B3X_API int b3x_fault_flags(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_fault, sizeof(int)) != cudaSuccess) return -1;
    if (clear) {
        int z = 0;
        cudaMemcpyToSymbol(g_fault, &z, sizeof(int));
    }
    return v;
}

B3X_API int b3x_batch_observe_gpu(B3Batch batch, int body, float* out, void* stream, unsigned long long sig) {
    Layout L;
    if (!layout_from_signature(sig, &L)) return cudaErrorInvalidValue;
    if (!batch_ok(batch, L.size) || body < 0 || body >= L.B || (batch.count && !out)) return cudaErrorInvalidValue;
    if (!batch.count) return cudaSuccess;
    if (!aligned8(batch)) return cudaErrorInvalidValue;
    observe_kernel<<<(batch.count + 127) / 128, 128, 0, (cudaStream_t)stream>>>((const unsigned char*)batch.data,
        batch.stride, batch.world_offset, batch.count, body, out);
    return cudaGetLastError();
}

// ---- resident world columns (b3x_engine_*) ----------------------------------------
// The worlds live in HBM as structure-of-arrays across worlds: word w of the
// B3World of world i at engine[((i / 32) * W + w) * 32 + i % 32], W =
// sizeof(B3World) / 4.  Steps read and write these columns (one word of a
// tile's 32 worlds is one 128-byte line) instead of the caller's AoS array;
// bind and sync move worlds between the two layouts.

static bool engine_ok(const void* engine, int count) {
    return count >= 0 && (count == 0 || (engine != nullptr && ((uintptr_t)engine % 16) == 0));
}

B3X_API size_t b3x_engine_bytes(unsigned long long sig, int count) {
    Layout L;
    if (!layout_from_signature(sig, &L) || count < 0) return 0;
    const size_t tiles = ((size_t)count + kLanes - 1) / kLanes;
    return tiles * (size_t)L.size * kLanes;
}

static int engine_move(void* engine, int count, B3Batch worlds, const unsigned char* select, void* stream,
        unsigned long long sig, bool in) {
    Layout L;
    if (!layout_from_signature(sig, &L)) return cudaErrorInvalidValue;
    if (!engine_ok(engine, count) || !batch_ok(worlds, L.size) || worlds.count != count) return cudaErrorInvalidValue;
    if (count == 0) return cudaSuccess;
    if (!aligned8(worlds)) return cudaErrorInvalidValue;
    const unsigned tiles = (unsigned)((count + kLanes - 1) / kLanes);
    if (in)
        columns_kernel<true><<<tiles, kCta, 0, (cudaStream_t)stream>>>((float*)engine, L.size / 4,
            (unsigned char*)worlds.data, worlds.stride, worlds.world_offset, count, select);
    else
        columns_kernel<false><<<tiles, kCta, 0, (cudaStream_t)stream>>>((float*)engine, L.size / 4,
            (unsigned char*)worlds.data, worlds.stride, worlds.world_offset, count, select);
    return cudaGetLastError();
}

B3X_API int b3x_engine_bind(void* engine, int count, B3Batch worlds, const unsigned char* select, void* stream,
        unsigned long long sig) {
    return engine_move(engine, count, worlds, select, stream, sig, true);
}

B3X_API int b3x_engine_sync_to_aos(const void* engine, int count, B3Batch worlds, const unsigned char* select,
        void* stream, unsigned long long sig) {
    return engine_move(const_cast<void*>(engine), count, worlds, select, stream, sig, false);
}

B3X_API int b3x_engine_step(void* engine, int count, float dt, int substeps, const unsigned char* active,
        void* stream, unsigned long long sig, int ji, int ri, int flags) {
    Layout L;
    if (!layout_from_signature(sig, &L)) return cudaErrorInvalidValue;
    if (!engine_ok(engine, count)
            || !step_params_ok(dt, substeps, ji, ri, flags,
                               kStepInterleaveContacts | kStepSkipRestitution | kStepStateOnly))
        return cudaErrorInvalidValue;
    if (count == 0 || dt == 0) return cudaSuccess;
    Worlds w{nullptr, 0, 0, count, (float*)engine};
    return run_step(w, dt, substeps, active, stream, sig, L, ji, ri, WsFrom::kLibrary, nullptr, 0, flags);
}

B3X_API int b3x_engine_apply(void* engine, int count, int kind, int index, const float* values, int vpw,
        const unsigned char* active, void* stream, unsigned long long sig) {
    Layout L;
    if (!layout_from_signature(sig, &L)) return cudaErrorInvalidValue;
    if (!engine_ok(engine, count) || kind < 0 || kind > 3 || vpw < 1 || (count && !values))
        return cudaErrorInvalidValue;
    if (kind != B3X_ACTION_JOINT_TARGET && vpw % 3 != 0) return cudaErrorInvalidValue;
    if (!count) return cudaSuccess;
    apply_columns_kernel<<<(count + 127) / 128, 128, 0, (cudaStream_t)stream>>>((float*)engine, L.size / 4, count, L,
        kind, index, values, vpw, active);
    return cudaGetLastError();
}

B3X_API int b3x_engine_observe(const void* engine, int count, int body, float* out, void* stream,
        unsigned long long sig) {
    Layout L;
    if (!layout_from_signature(sig, &L)) return cudaErrorInvalidValue;
    if (!engine_ok(engine, count) || body < 0 || body >= L.B || (count && !out)) return cudaErrorInvalidValue;
    if (!count) return cudaSuccess;
    observe_columns_kernel<<<(count + 127) / 128, 128, 0, (cudaStream_t)stream>>>((const float*)engine, L.size / 4,
        count, body, out);
    return cudaGetLastError();
}

// ---- allocation-free variant ---------------------------------------------------
// Some callers cannot allocate device memory at the moment they step: code
// whose device memory is entirely owned by a framework's caching allocator or
// a plugin host that forbids raw cudaMalloc, and real-time loops that cannot
// afford the implicit synchronisation an allocation may bring.  For them,
// b3x_batch_step_gpu_noalloc takes its workspace from g_noalloc_scratch, a
// fixed 64 MiB array reserved on every device that loads the library until
// the process exits.
//
// Same step as b3x_batch_step_gpu with that array as the workspace; it calls
// no cudaMalloc, cudaFree or other allocating routine.  Every call looks up
// the array's device address on the current device (cudaGetSymbolAddress);
// the first call on a device also loads the library's kernels there, so make
// it before any stream capture.  Every call on a device shares the array, and
// its contents are left over from the previous call (the step writes every
// word of it that it reads, so nothing needs clearing); calls whose launches
// overlap on the GPU (different streams, no ordering between them) race on it
// and must not be issued.  A capacity configuration whose per-CTA workspace
// slot exceeds 64 MiB is rejected with cudaErrorInvalidValue (configurations
// small enough to be stepped in shared memory use no workspace and are never
// rejected); smaller ones run as many tiles per launch as slots fit (at most
// the device's resident blocks), so any batch size is accepted.
B3X_API int b3x_batch_step_gpu_noalloc(B3Batch batch, float dt, int substeps, const unsigned char* active,
        void* stream, unsigned long long sig, int ji, int ri) {
    return step_common(batch, dt, substeps, active, stream, sig, ji, ri, WsFrom::kNoAlloc, nullptr, 0);
}

}  // extern "C"

