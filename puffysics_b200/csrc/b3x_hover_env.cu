// b3x_hover_env.cu -- the PufferLib hover environment, fused into one launch
// per environment step (libb3hover.so).
//
// The reference ships this task as an example adapter that steps each
// environment on its own thread in global memory
// (examples/pufferlib/puffysics_hover/hover_task.h, puffysics_hover.h:39-58,
// puffysics_hover.cu:40-43).  Here one launch does the whole environment step
// -- action, b3_step, reward, terminal test, episode log, automatic reset,
// observation -- on environments staged in shared memory (b3x_staged.cuh):
// the hover world is 3 KB, so eight environments per block fit with room to
// spare and the world is stepped on chip.  Actions, observations, rewards and
// terminals are flat arrays indexed by environment (the trainer's buffers).
//
// The task is the reference's, operation for operation, with its capacities
// (2 bodies, 2 shapes, 4 contacts, 2 joints); HoverTask has the reference's
// field order so its bytes compare directly.  Built with the library's parity
// flags, so the worlds match the reference's CPU step bit for bit.
#define B3_MAX_BODIES 2
#define B3_MAX_SHAPES 2
#define B3_MAX_CONTACTS 4
#define B3_MAX_JOINTS 2
#include <cmath>
#include <cstddef>

#include <cuda_runtime.h>

#include "b3x_staged.cuh"

#define B3H_API extern "C" __attribute__((visibility("default")))

namespace {

enum { kObs = 3 };

// hover_task.h:24-39
struct HoverConfig {
    float target_height;
    float thrust;     // acceleration per action level: 0, thrust, 2 * thrust
    float dt;
    int substeps;
    int horizon;
};

struct HoverTask {
    B3World world;
    HoverConfig config;
    uint32_t rng;     // per-environment state, kept across episode resets
    int tick;
    int body;
    float episode_return;
};

// Episode statistics of one environment (puffysics_hover.h:12-18).
struct HoverLog {
    float perf, score, episode_return, episode_length, n;
};

struct HoverEnv {
    HoverTask task;
    HoverLog log;
    float pad_;       // 8-byte multiple for the staged copies
};
static_assert(sizeof(HoverEnv) % 8 == 0, "staged element size");

// hover_task.h:45-59
__device__ void hover_reset(HoverTask& t) {
    b3_world_init(&t.world);
    t.rng = t.rng * 1664525u + 1013904223u;
    const float jitter = (float)(t.rng >> 8) * (1.0f / 16777216.0f) - 0.5f;
    B3BodyDef body = b3_default_body();
    body.type = B3_DYNAMIC;
    body.position = b3_v(0.0f, t.config.target_height + jitter, 0.0f);
    body.linear_damping = 0.0f;
    t.body = b3_create_body(&t.world, &body);
    B3ShapeDef shape = b3_default_shape();
    b3_create_sphere(&t.world, t.body, b3_v(0.0f, 0.0f, 0.0f), 0.25f, &shape);
    b3_finalize_mass(&t.world, t.body);
    t.tick = 0;
    t.episode_return = 0.0f;
}

// hover_task.h:68-73
__device__ void hover_apply_action(HoverTask& t, float action) {
    const float level = action >= 1.5f ? 2.0f : (action >= 0.5f ? 1.0f : 0.0f);
    const B3Body& b = t.world.bodies[t.body];
    b3_apply_force(&t.world, t.body, b3_v(0.0f, level * t.config.thrust / b.inv_mass, 0.0f));
}

// hover_task.h:75-80
__device__ void hover_observe(const HoverTask& t, float* obs) {
    const B3Body& b = t.world.bodies[t.body];
    obs[0] = b.position.y - t.config.target_height;
    obs[1] = b.lin_vel.y;
    obs[2] = (float)t.tick / (float)t.config.horizon;
}

// hover_task.h:82-86
__device__ float hover_reward(const HoverTask& t) {
    const B3Body& b = t.world.bodies[t.body];
    const float error = fabsf(b.position.y - t.config.target_height);
    return 1.0f - b3_minf(error + 0.1f * fabsf(b.lin_vel.y), 2.0f);
}

// hover_task.h:88-92
__device__ int hover_terminal(const HoverTask& t) {
    const float height = t.world.bodies[t.body].position.y;
    return !isfinite(height) || fabsf(height - t.config.target_height) > 3.0f || t.tick >= t.config.horizon;
}

// One environment step with automatic reset (hover_task.h:95-99,
// puffysics_hover.h:39-58): terminal reward and done, then the next
// episode's first observation.
__device__ void hover_env_step(HoverEnv& e, float action, float* obs, float* reward_out, float* terminal_out) {
    HoverTask& t = e.task;
    hover_apply_action(t, action);
    b3_step(&t.world, t.config.dt, t.config.substeps);
    t.tick++;
    const float reward = hover_reward(t);
    const int done = hover_terminal(t);
    t.episode_return += reward;
    if (done) {
        e.log.perf += t.tick >= t.config.horizon;
        e.log.score += t.episode_return;
        e.log.episode_return += t.episode_return;
        e.log.episode_length += (float)t.tick;
        e.log.n += 1.0f;
        hover_reset(t);
    }
    hover_observe(t, obs);
    *reward_out = reward;
    *terminal_out = (float)done;
}

// puffysics_hover.h:32-37
__device__ void hover_env_reset(HoverEnv& e, float* obs, float* reward_out, float* terminal_out) {
    hover_reset(e.task);
    hover_observe(e.task, obs);
    *reward_out = 0.0f;
    *terminal_out = 0.0f;
}

struct StepFn {
    const float* actions;
    float *obs, *rewards, *terminals;
    __device__ void operator()(HoverEnv& e, int i) const {
        hover_env_step(e, actions[i], obs + (size_t)i * kObs, rewards + i, terminals + i);
    }
};

struct ResetFn {
    float *obs, *rewards, *terminals;
    __device__ void operator()(HoverEnv& e, int i) const {
        hover_env_reset(e, obs + (size_t)i * kObs, rewards + i, terminals + i);
    }
};

struct InitFn {
    HoverConfig config;
    uint32_t seed;
    __device__ void operator()(HoverEnv& e, int i) const {
        e.log = HoverLog{0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        e.pad_ = 0.0f;
        e.task.config = config;
        e.task.rng = seed + (uint32_t)i * 747796405u;   // puffysics_hover.cu:33
        hover_reset(e.task);
    }
};

// The reference's launch shape: one thread per environment in global memory.
__global__ void step_in_place_kernel(HoverEnv* envs, int n, StepFn fn) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) fn(envs[i], i);
}

constexpr int kPerBlock = 8;

bool arrays_ok(int n, const void* envs, const void* a, const void* b, const void* c) {
    if (n < 0) return false;
    if (n == 0) return true;
    return envs && a && b && c && ((uintptr_t)envs % 8) == 0;
}

}  // namespace

B3H_API size_t b3x_hover_env_bytes(void) { return sizeof(HoverEnv); }
B3H_API size_t b3x_hover_task_offset(void) { return offsetof(HoverEnv, task); }
B3H_API size_t b3x_hover_task_bytes(void) { return sizeof(HoverTask); }
B3H_API size_t b3x_hover_log_offset(void) { return offsetof(HoverEnv, log); }
B3H_API unsigned long long b3x_hover_signature(void) { return B3_CONFIG_SIGNATURE; }

// Initialise n environments (puffysics_hover.cu:21-34): configuration, the
// per-environment seed, first episode.
B3H_API int b3x_hover_init_gpu(void* envs, int n, float target_height, float thrust, float dt, int substeps,
        int horizon, unsigned seed, void* stream) {
    if (n < 0 || (n > 0 && (!envs || ((uintptr_t)envs % 8) != 0)) || !(dt > 0.0f) || substeps < 1 || horizon < 1)
        return (int)cudaErrorInvalidValue;
    InitFn fn{HoverConfig{target_height, thrust, dt, substeps, horizon}, seed};
    return (int)b3x::staged_launch<kPerBlock>((HoverEnv*)envs, n, fn, (cudaStream_t)stream);
}

// Reset every environment and write its first observation.
B3H_API int b3x_hover_reset_gpu(void* envs, int n, float* obs, float* rewards, float* terminals, void* stream) {
    if (!arrays_ok(n, envs, obs, rewards, terminals)) return (int)cudaErrorInvalidValue;
    ResetFn fn{obs, rewards, terminals};
    return (int)b3x::staged_launch<kPerBlock>((HoverEnv*)envs, n, fn, (cudaStream_t)stream);
}

// One fused environment step of every environment, staged in shared memory.
B3H_API int b3x_hover_step_gpu(void* envs, int n, const float* actions, float* obs, float* rewards, float* terminals,
        void* stream) {
    if (!arrays_ok(n, envs, actions, obs, rewards) || (n > 0 && !terminals)) return (int)cudaErrorInvalidValue;
    StepFn fn{actions, obs, rewards, terminals};
    return (int)b3x::staged_launch<kPerBlock>((HoverEnv*)envs, n, fn, (cudaStream_t)stream);
}

// The same step with the reference adapter's launch shape (one thread per
// environment, 32-thread blocks, environments read and written in place).
B3H_API int b3x_hover_step_in_place_gpu(void* envs, int n, const float* actions, float* obs, float* rewards,
        float* terminals, void* stream) {
    if (!arrays_ok(n, envs, actions, obs, rewards) || (n > 0 && !terminals)) return (int)cudaErrorInvalidValue;
    if (n == 0) return (int)cudaSuccess;
    StepFn fn{actions, obs, rewards, terminals};
    step_in_place_kernel<<<(n + 31) / 32, 32, 0, (cudaStream_t)stream>>>((HoverEnv*)envs, n, fn);
    return (int)cudaGetLastError();
}
