/*
 * hover_shim.c -- the reference's hover task (examples/pufferlib/
 * puffysics_hover/hover_task.h, compiled from the reference checkout) behind
 * C entry points over arrays of its HoverTask, for the hover-environment
 * parity tests and the benchmark's reference arm.
 *
 * TEST AND BENCHMARK INFRASTRUCTURE, NOT PRODUCT CODE.  Built by
 * oracle/Makefile with -ffp-contract=off (CPU, _ref/libb3ref_hoverenv.so)
 * and, as refhover_gpu.cu, by nvcc with the reference's stock flags
 * (_ref/libb3refgpu_hoverenv.so).  The adapter's environment wrapper
 * (puffysics_hover.h:32-58, whose header also needs PufferLib's pufferenv.h)
 * is restated here over flat action / observation / reward / terminal arrays
 * and a per-environment log of five floats.
 */
#include <stddef.h>
#include <stdint.h>

#include "hover_task.h"

#if defined(__CUDACC__)
#define HS_EXPORT extern "C" __attribute__((visibility("default")))
#define HS_FN __host__ __device__
#else
#define HS_EXPORT __attribute__((visibility("default")))
#define HS_FN
#endif

typedef struct HoverShimLog {
    float perf, score, episode_return, episode_length, n;
} HoverShimLog;

/* puffysics_hover.h:39-58 */
HS_FN static inline void shim_env_step(HoverTask* task, HoverShimLog* log, float action, float* obs, float* reward_out,
        float* terminal_out) {
    hover_step(task, action);
    float reward = hover_reward(task);
    int done = hover_terminal(task);
    task->episode_return += reward;
    if (done) {
        log->perf += task->tick >= task->config.horizon;
        log->score += task->episode_return;
        log->episode_return += task->episode_return;
        log->episode_length += (float)task->tick;
        log->n += 1;
        hover_reset(task);
    }
    hover_observe(task, obs);
    *reward_out = reward;
    *terminal_out = (float)done;
}

HS_FN static inline HoverConfig shim_config(float target, float thrust, float dt, int substeps, int horizon) {
    HoverConfig c = hover_default_config();
    c.target_height = target;
    c.thrust = thrust;
    c.dt = dt;
    c.substeps = substeps;
    c.horizon = horizon;
    return c;
}

HS_EXPORT size_t refhover_task_bytes(void) { return sizeof(HoverTask); }

#if !defined(__CUDACC__)
/* puffysics_hover.cu:21-34 (the initialisation part), on the host */
HS_EXPORT void refhover_init(HoverTask* tasks, int n, float target, float thrust, float dt, int substeps,
        int horizon, unsigned seed) {
    HoverConfig c = shim_config(target, thrust, dt, substeps, horizon);
    for (int i = 0; i < n; i++) hover_init(&tasks[i], c, seed + (uint32_t)i * 747796405u);
}

HS_EXPORT void refhover_step(HoverTask* tasks, HoverShimLog* logs, int n, const float* actions, float* obs,
        float* rewards, float* terminals) {
    for (int i = 0; i < n; i++)
        shim_env_step(&tasks[i], &logs[i], actions[i], obs + (size_t)i * HOVER_OBS_SIZE, rewards + i, terminals + i);
}
#else
/* The reference adapter's step kernel shape (puffysics_hover.cu:40-43,
 * launched <<<ceil(n/32), 32>>>): one thread per environment in place. */
static __global__ void refhover_init_kernel(HoverTask* tasks, int n, HoverConfig c, unsigned seed) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) hover_init(&tasks[i], c, seed + (uint32_t)i * 747796405u);
}

static __global__ void refhover_step_kernel(HoverTask* tasks, HoverShimLog* logs, int n, const float* actions,
        float* obs, float* rewards, float* terminals) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n)
        shim_env_step(&tasks[i], &logs[i], actions[i], obs + (size_t)i * HOVER_OBS_SIZE, rewards + i,
                      terminals + i);
}

HS_EXPORT int refhover_gpu_init(HoverTask* tasks, int n, float target, float thrust, float dt, int substeps,
        int horizon, unsigned seed, void* stream) {
    if (n <= 0) return 0;
    refhover_init_kernel<<<(n + 31) / 32, 32, 0, (cudaStream_t)stream>>>(
        tasks, n, shim_config(target, thrust, dt, substeps, horizon), seed);
    return (int)cudaGetLastError();
}

HS_EXPORT int refhover_gpu_step(HoverTask* tasks, HoverShimLog* logs, int n, const float* actions, float* obs,
        float* rewards, float* terminals, void* stream) {
    if (n <= 0) return 0;
    refhover_step_kernel<<<(n + 31) / 32, 32, 0, (cudaStream_t)stream>>>(tasks, logs, n, actions, obs, rewards,
                                                                          terminals);
    return (int)cudaGetLastError();
}
#endif
