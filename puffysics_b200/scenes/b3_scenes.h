/*
 * b3_scenes.h -- seeded synthetic scenes and per-step actions for the five
 * benchmark configurations (hover, box stack, capsule chain, pile, and the
 * stack reused for the scale-out run).
 *
 * Header-only and written against the public world-building API only
 * (b3_world_init, b3_create_*, b3_finalize_mass, b3_create_revolute, ...), so
 * the same source builds identical worlds whether it is compiled against
 * include/puffysics_b200.h or against the reference's own puffysics.cuh.
 * Include one of those headers first.
 *
 * Randomness is a counter hash of (seed, world index, step, slot): worlds do
 * not depend on how a batch is split across threads or GPUs.  Scene building
 * runs on the host (it calls sinf/cosf through b3_q_axis_angle).  The action
 * and reset-mask generators use integer hashing and exactly representable
 * float arithmetic only, so host and device produce the same bits.
 */
#ifndef B3_SCENES_H
#define B3_SCENES_H

#include <stdint.h>

#ifndef B3_HD
#error "include puffysics_b200.h (or the reference puffysics.cuh) before b3_scenes.h"
#endif

#define B3S_HOVER 1
#define B3S_STACK 2
#define B3S_CHAIN 3
#define B3S_PILE 4
#define B3S_BOUNCE 5
#define B3S_CAPSULE 6

/* Action kinds (same numbering as the b3x_batch_apply_gpu C-ABI). */
#define B3S_ACT_NONE (-1)
#define B3S_ACT_FORCE 0
#define B3S_ACT_TORQUE 1
#define B3S_ACT_LINEAR_IMPULSE 2
#define B3S_ACT_JOINT_TARGET 3

#define B3S_CHAIN_LINKS 10
#define B3S_STACK_BOXES 8
#define B3S_PILE_BOXES 16
#define B3S_PILE_SPHERES 16
#define B3S_CAPSULE_SHAPES 12

/* splitmix64 finaliser over a combined counter. */
B3_HD B3_INL uint64_t b3s_mix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

B3_HD B3_INL uint64_t b3s_hash(uint64_t seed, uint64_t world, uint64_t step, uint64_t slot) {
    uint64_t h = b3s_mix(seed ^ 0x5EEDull);
    h = b3s_mix(h ^ world);
    h = b3s_mix(h ^ (step * 0x100000001B3ull));
    return b3s_mix(h ^ (slot * 0xC2B2AE3D27D4EB4Full));
}

/* Uniform in [0, 1) with 24 bits: exact in float. */
B3_HD B3_INL float b3s_unit(uint64_t h) { return (float)(uint32_t)(h >> 40) * (1.0f / 16777216.0f); }

B3_HD B3_INL float b3s_uniform(uint64_t seed, uint64_t world, uint64_t step, uint64_t slot, float lo, float hi) {
    return lo + (hi - lo) * b3s_unit(b3s_hash(seed, world, step, slot));
}

/* Approximately standard normal: Irwin-Hall sum of twelve 16-bit uniforms
 * minus 6.  Every intermediate is an exactly representable float, so the
 * value does not depend on the platform. */
B3_HD B3_INL float b3s_normal(uint64_t seed, uint64_t world, uint64_t step, uint64_t slot) {
    uint32_t sum = 0;
    for (int k = 0; k < 12; k++) {
        uint64_t h = b3s_hash(seed, world, step, slot * 16u + (uint64_t)k);
        sum += (uint32_t)(h >> 48);
    }
    return (float)sum * (1.0f / 65536.0f) - 6.0f;
}

/* ---------------------------------------------------------------- scenes */

B3_HD B3_INL int b3s_ground(B3World* w) {
    B3BodyDef gd = b3_default_body();
    gd.position = b3_v(0.0f, -0.5f, 0.0f);
    int g = b3_create_body(w, &gd);
    B3ShapeDef sd = b3_default_shape();
    sd.friction = 0.6f;
    b3_create_box(w, g, b3_v(50.0f, 0.5f, 50.0f), &sd);
    return g;
}

/* C1: ground + one dynamic sphere (r 0.5, mass 1), y0 ~ U[0.5, 3],
 * v0 ~ N(0, 0.5) per axis. */
static inline int b3s_build_hover(B3World* w, uint64_t seed, uint64_t index) {
    b3_world_init(w);
    w->gravity = b3_v(0.0f, -9.81f, 0.0f);
    b3s_ground(w);
    B3BodyDef bd = b3_default_body();
    bd.type = B3_DYNAMIC;
    bd.position = b3_v(0.0f, b3s_uniform(seed, index, 0, 1, 0.5f, 3.0f), 0.0f);
    bd.lin_vel = b3_v(0.5f * b3s_normal(seed, index, 0, 2), 0.5f * b3s_normal(seed, index, 0, 3),
        0.5f * b3s_normal(seed, index, 0, 4));
    int b = b3_create_body(w, &bd);
    B3ShapeDef sd = b3_default_shape();
    sd.density = 1.0f / ((4.0f / 3.0f) * B3_PI * 0.125f);
    b3_create_sphere(w, b, b3_v(0.0f, 0.0f, 0.0f), 0.5f, &sd);
    b3_finalize_mass(w, b);
    return b3_world_error(w) ? -1 : 0;
}

/* C2 / C5: ground + 8 unit boxes (half 0.5, mass 1, friction 0.6) stacked at
 * y = 0.5 + k with x/z jitter U[-0.05, 0.05] and yaw U[-0.2, 0.2]. */
static inline int b3s_build_stack(B3World* w, uint64_t seed, uint64_t index) {
    b3_world_init(w);
    w->gravity = b3_v(0.0f, -9.81f, 0.0f);
    b3s_ground(w);
    for (int k = 0; k < B3S_STACK_BOXES; k++) {
        B3BodyDef bd = b3_default_body();
        bd.type = B3_DYNAMIC;
        bd.position = b3_v(b3s_uniform(seed, index, 0, 10u + 3u * (uint64_t)k, -0.05f, 0.05f),
            0.5f + (float)k,
            b3s_uniform(seed, index, 0, 11u + 3u * (uint64_t)k, -0.05f, 0.05f));
        bd.rotation = b3_q_axis_angle(b3_v(0.0f, 1.0f, 0.0f),
            b3s_uniform(seed, index, 0, 12u + 3u * (uint64_t)k, -0.2f, 0.2f));
        int b = b3_create_body(w, &bd);
        B3ShapeDef sd = b3_default_shape();
        sd.density = 1.0f;
        sd.friction = 0.6f;
        sd.restitution = 0.0f;
        b3_create_box(w, b, b3_v(0.5f, 0.5f, 0.5f), &sd);
        b3_finalize_mass(w, b);
    }
    return b3_world_error(w) ? -1 : 0;
}

/* C3: static shapeless anchor near y = 2; 10 capsule links (r 0.05, half
 * length 0.2, mass 0.5) laid out horizontally from it along a yawed x axis;
 * link 0 welded to the anchor; 9 revolutes about the links' local z axis
 * (horizontal, so the chain swings down under gravity and its tail reaches
 * the ground), limits +-1.2, spring (4 Hz, zeta 0.7) toward the action
 * target, and an enabled speed-0 motor that bounds the spring impulse
 * (5 N m). */
static inline int b3s_build_chain(B3World* w, uint64_t seed, uint64_t index) {
    b3_world_init(w);
    w->gravity = b3_v(0.0f, -9.81f, 0.0f);
    b3s_ground(w);
    float yaw = b3s_uniform(seed, index, 0, 20, -0.3f, 0.3f);
    float h = 2.0f + b3s_uniform(seed, index, 0, 21, -0.1f, 0.1f);
    B3Quat qyaw = b3_q_axis_angle(b3_v(0.0f, 1.0f, 0.0f), yaw);
    B3Quat qlink = b3_qmul(qyaw, b3_q_axis_angle(b3_v(0.0f, 0.0f, 1.0f), -0.5f * B3_PI));
    B3Vec3 dir = b3_rotate(qyaw, b3_v(1.0f, 0.0f, 0.0f));
    B3BodyDef ad = b3_default_body();
    ad.position = b3_v(0.0f, h, 0.0f);
    int anchor = b3_create_body(w, &ad);
    const float r = 0.05f, half_len = 0.2f, seg = 0.5f;
    float vol = B3_PI * r * r * (2.0f * half_len) + (4.0f / 3.0f) * B3_PI * r * r * r;
    int links[B3S_CHAIN_LINKS];
    for (int k = 0; k < B3S_CHAIN_LINKS; k++) {
        B3BodyDef bd = b3_default_body();
        bd.type = B3_DYNAMIC;
        bd.position = b3_add(ad.position, b3_mul(dir, 0.5f * seg + seg * (float)k));
        bd.rotation = qlink;
        links[k] = b3_create_body(w, &bd);
        B3ShapeDef sd = b3_default_shape();
        sd.density = 0.5f / vol;
        b3_create_capsule(w, links[k], half_len, r, &sd);
        b3_finalize_mass(w, links[k]);
    }
    b3_create_weld(w, anchor, links[0], b3_v(0.0f, 0.0f, 0.0f), b3_v(0.0f, -0.5f * seg, 0.0f));
    for (int k = 1; k < B3S_CHAIN_LINKS; k++) {
        B3Vec3 axis = b3_v(0.0f, 0.0f, 1.0f);
        int j = b3_create_revolute(w, links[k - 1], links[k], b3_v(0.0f, 0.5f * seg, 0.0f),
            b3_v(0.0f, -0.5f * seg, 0.0f), axis);
        if (j < 0) return -1;
        b3_joint_enable_limit(w, j, 1);
        b3_joint_set_limits(w, j, -1.2f, 1.2f);
        b3_joint_enable_spring(w, j, 1);
        b3_joint_set_spring(w, j, 0.0f, 4.0f, 0.7f);
        b3_joint_enable_motor(w, j, 1);
        b3_joint_set_motor(w, j, 0.0f, 5.0f);
    }
    return b3_world_error(w) ? -1 : 0;
}

/* C4: ground + 4 walls around x, z in [-2, 2] + 16 boxes (half U[0.1,0.4]^3,
 * random orientation) and 16 spheres (r U[0.1, 0.4]), densities U[500, 2000],
 * placed without overlap (bounding spheres, seeded rejection sampling) in
 * the 4 x 4 x 6 m region above the ground. */
static inline int b3s_build_pile(B3World* w, uint64_t seed, uint64_t index) {
    b3_world_init(w);
    w->gravity = b3_v(0.0f, -9.81f, 0.0f);
    b3s_ground(w);
    B3ShapeDef wsd = b3_default_shape();
    wsd.friction = 0.6f;
    for (int k = 0; k < 4; k++) {
        B3BodyDef wd = b3_default_body();
        float s = (k & 1) ? 1.0f : -1.0f;
        wd.position = (k < 2) ? b3_v(2.25f * s, 3.0f, 0.0f) : b3_v(0.0f, 3.0f, 2.25f * s);
        int b = b3_create_body(w, &wd);
        b3_create_box(w, b, (k < 2) ? b3_v(0.25f, 3.5f, 2.5f) : b3_v(2.5f, 3.5f, 0.25f), &wsd);
    }
    float px[B3S_PILE_BOXES + B3S_PILE_SPHERES];
    float py[B3S_PILE_BOXES + B3S_PILE_SPHERES];
    float pz[B3S_PILE_BOXES + B3S_PILE_SPHERES];
    float pr[B3S_PILE_BOXES + B3S_PILE_SPHERES];
    int n = B3S_PILE_BOXES + B3S_PILE_SPHERES;
    for (int i = 0; i < n; i++) {
        int is_box = (i & 1) == 0;
        uint64_t base = 100u + 64u * (uint64_t)i;
        B3Vec3 half = b3_v(b3s_uniform(seed, index, 0, base + 0, 0.1f, 0.4f),
            b3s_uniform(seed, index, 0, base + 1, 0.1f, 0.4f),
            b3s_uniform(seed, index, 0, base + 2, 0.1f, 0.4f));
        float rad = b3s_uniform(seed, index, 0, base + 3, 0.1f, 0.4f);
        float bound = is_box ? b3_len(half) : rad;
        float x = 0.0f, y = 0.0f, z = 0.0f;
        int placed = 0;
        for (int t = 0; t < 48 && !placed; t++) {
            uint64_t sl = 10000u + 1000u * (uint64_t)i + 3u * (uint64_t)t;
            x = b3s_uniform(seed, index, 0, sl + 0, -2.0f + bound, 2.0f - bound);
            y = b3s_uniform(seed, index, 0, sl + 1, bound + 0.05f, 6.0f - bound);
            z = b3s_uniform(seed, index, 0, sl + 2, -2.0f + bound, 2.0f - bound);
            placed = 1;
            for (int k = 0; k < i; k++) {
                float dx = x - px[k], dy = y - py[k], dz = z - pz[k];
                float rr = bound + pr[k] + 0.01f;
                if (dx * dx + dy * dy + dz * dz < rr * rr) { placed = 0; break; }
            }
        }
        if (!placed) {            /* deterministic fallback: a column above the bin */
            x = -1.5f + 1.0f * (float)(i % 4);
            z = -1.5f + 1.0f * (float)((i / 4) % 4);
            y = 7.0f + 1.0f * (float)i;
        }
        px[i] = x; py[i] = y; pz[i] = z; pr[i] = bound;
        B3BodyDef bd = b3_default_body();
        bd.type = B3_DYNAMIC;
        bd.position = b3_v(x, y, z);
        if (is_box) {
            B3Vec3 axis = b3_v(b3s_uniform(seed, index, 0, base + 4, -1.0f, 1.0f),
                b3s_uniform(seed, index, 0, base + 5, -1.0f, 1.0f),
                b3s_uniform(seed, index, 0, base + 6, -1.0f, 1.0f));
            bd.rotation = b3_q_axis_angle(axis, b3s_uniform(seed, index, 0, base + 7, 0.0f, B3_PI));
        }
        int b = b3_create_body(w, &bd);
        B3ShapeDef sd = b3_default_shape();
        sd.density = b3s_uniform(seed, index, 0, base + 8, 500.0f, 2000.0f);
        sd.friction = 0.6f;
        if (is_box) b3_create_box(w, b, half, &sd);
        else b3_create_sphere(w, b, b3_v(0.0f, 0.0f, 0.0f), rad, &sd);
        b3_finalize_mass(w, b);
    }
    return b3_world_error(w) ? -1 : 0;
}

/* Bounce (parity coverage of restitution and rolling resistance, which the
 * benchmark scenes leave at 0): ground + 4 spheres (r U[0.2, 0.45]) and 4
 * boxes (half U[0.15, 0.34], random orientation) on a 2 x 2 x 2 lattice of
 * 1.2 m cells, thrown down with spin; per shape restitution U[0.3, 0.9],
 * rolling resistance U[0.02, 0.2], friction U[0.2, 1]. */
static inline int b3s_build_bounce(B3World* w, uint64_t seed, uint64_t index) {
    b3_world_init(w);
    w->gravity = b3_v(0.0f, -9.81f, 0.0f);
    b3s_ground(w);
    for (int i = 0; i < 8; i++) {
        int is_box = (i & 1) != 0;
        uint64_t base = 200u + 32u * (uint64_t)i;
        B3BodyDef bd = b3_default_body();
        bd.type = B3_DYNAMIC;
        bd.position = b3_v((i & 2) ? 0.6f : -0.6f, 1.2f + 1.2f * (float)(i >> 2), (i & 4) ? 0.6f : -0.6f);
        bd.lin_vel = b3_v(b3s_uniform(seed, index, 0, base + 0, -1.0f, 1.0f),
            b3s_uniform(seed, index, 0, base + 1, -4.0f, 0.0f), b3s_uniform(seed, index, 0, base + 2, -1.0f, 1.0f));
        bd.ang_vel = b3_v(b3s_uniform(seed, index, 0, base + 3, -6.0f, 6.0f),
            b3s_uniform(seed, index, 0, base + 4, -6.0f, 6.0f), b3s_uniform(seed, index, 0, base + 5, -6.0f, 6.0f));
        if (is_box) {
            B3Vec3 axis = b3_v(b3s_uniform(seed, index, 0, base + 6, -1.0f, 1.0f),
                b3s_uniform(seed, index, 0, base + 7, -1.0f, 1.0f),
                b3s_uniform(seed, index, 0, base + 8, -1.0f, 1.0f));
            bd.rotation = b3_q_axis_angle(axis, b3s_uniform(seed, index, 0, base + 9, 0.0f, B3_PI));
        }
        int b = b3_create_body(w, &bd);
        B3ShapeDef sd = b3_default_shape();
        sd.density = b3s_uniform(seed, index, 0, base + 10, 500.0f, 2000.0f);
        sd.friction = b3s_uniform(seed, index, 0, base + 11, 0.2f, 1.0f);
        sd.restitution = b3s_uniform(seed, index, 0, base + 12, 0.3f, 0.9f);
        sd.rolling = b3s_uniform(seed, index, 0, base + 13, 0.02f, 0.2f);
        if (is_box) {
            B3Vec3 half = b3_v(b3s_uniform(seed, index, 0, base + 14, 0.15f, 0.34f),
                b3s_uniform(seed, index, 0, base + 15, 0.15f, 0.34f),
                b3s_uniform(seed, index, 0, base + 16, 0.15f, 0.34f));
            b3_create_box(w, b, half, &sd);
        } else {
            b3_create_sphere(w, b, b3_v(0.0f, 0.0f, 0.0f), b3s_uniform(seed, index, 0, base + 17, 0.2f, 0.45f), &sd);
        }
        b3_finalize_mass(w, b);
    }
    return b3_world_error(w) ? -1 : 0;
}

/* Capsules (parity coverage of the sphere-capsule and capsule-capsule
 * manifolds, which no benchmark scene makes): ground + 4 walls around x, z in
 * [-1, 1] + 6 capsules (radius U[0.08, 0.2], half length U[0.15, 0.35],
 * random orientation) and 6 spheres (r U[0.1, 0.25]), densities
 * U[500, 2000], placed without overlap (bounding spheres, seeded rejection
 * sampling) in the 2 x 2 x 4 m region above the ground, so they fall into a
 * tangle. */
static inline int b3s_build_capsule(B3World* w, uint64_t seed, uint64_t index) {
    b3_world_init(w);
    w->gravity = b3_v(0.0f, -9.81f, 0.0f);
    b3s_ground(w);
    B3ShapeDef wsd = b3_default_shape();
    wsd.friction = 0.5f;
    for (int k = 0; k < 4; k++) {
        B3BodyDef wd = b3_default_body();
        float s = (k & 1) ? 1.0f : -1.0f;
        wd.position = (k < 2) ? b3_v(1.2f * s, 1.5f, 0.0f) : b3_v(0.0f, 1.5f, 1.2f * s);
        int b = b3_create_body(w, &wd);
        b3_create_box(w, b, (k < 2) ? b3_v(0.2f, 1.5f, 1.4f) : b3_v(1.4f, 1.5f, 0.2f), &wsd);
    }
    float px[B3S_CAPSULE_SHAPES], py[B3S_CAPSULE_SHAPES], pz[B3S_CAPSULE_SHAPES], pr[B3S_CAPSULE_SHAPES];
    for (int i = 0; i < B3S_CAPSULE_SHAPES; i++) {
        int is_capsule = (i & 1) == 0;
        uint64_t base = 300u + 32u * (uint64_t)i;
        float rad = is_capsule ? b3s_uniform(seed, index, 0, base + 0, 0.08f, 0.2f)
                               : b3s_uniform(seed, index, 0, base + 0, 0.1f, 0.25f);
        float half_len = b3s_uniform(seed, index, 0, base + 1, 0.15f, 0.35f);
        float bound = is_capsule ? rad + half_len : rad;
        float x = 0.0f, y = 0.0f, z = 0.0f;
        int placed = 0;
        for (int t = 0; t < 48 && !placed; t++) {
            uint64_t sl = 20000u + 1000u * (uint64_t)i + 3u * (uint64_t)t;
            x = b3s_uniform(seed, index, 0, sl + 0, -1.0f + bound, 1.0f - bound);
            y = b3s_uniform(seed, index, 0, sl + 1, bound + 0.05f, 4.0f - bound);
            z = b3s_uniform(seed, index, 0, sl + 2, -1.0f + bound, 1.0f - bound);
            placed = 1;
            for (int k = 0; k < i; k++) {
                float dx = x - px[k], dy = y - py[k], dz = z - pz[k];
                float rr = bound + pr[k] + 0.01f;
                if (dx * dx + dy * dy + dz * dz < rr * rr) { placed = 0; break; }
            }
        }
        if (!placed) {            /* deterministic fallback: a column above the bin */
            x = -0.5f + 1.0f * (float)(i % 2);
            z = -0.5f + 1.0f * (float)((i / 2) % 2);
            y = 5.0f + 0.8f * (float)i;
        }
        px[i] = x; py[i] = y; pz[i] = z; pr[i] = bound;
        B3BodyDef bd = b3_default_body();
        bd.type = B3_DYNAMIC;
        bd.position = b3_v(x, y, z);
        if (is_capsule) {
            B3Vec3 axis = b3_v(b3s_uniform(seed, index, 0, base + 2, -1.0f, 1.0f),
                b3s_uniform(seed, index, 0, base + 3, -1.0f, 1.0f),
                b3s_uniform(seed, index, 0, base + 4, -1.0f, 1.0f));
            bd.rotation = b3_q_axis_angle(axis, b3s_uniform(seed, index, 0, base + 5, 0.0f, B3_PI));
        }
        bd.ang_vel = b3_v(b3s_uniform(seed, index, 0, base + 6, -2.0f, 2.0f),
            b3s_uniform(seed, index, 0, base + 7, -2.0f, 2.0f), b3s_uniform(seed, index, 0, base + 8, -2.0f, 2.0f));
        int b = b3_create_body(w, &bd);
        B3ShapeDef sd = b3_default_shape();
        sd.density = b3s_uniform(seed, index, 0, base + 9, 500.0f, 2000.0f);
        sd.friction = b3s_uniform(seed, index, 0, base + 10, 0.3f, 0.9f);
        if (is_capsule) b3_create_capsule(w, b, half_len, rad, &sd);
        else b3_create_sphere(w, b, b3_v(0.0f, 0.0f, 0.0f), rad, &sd);
        b3_finalize_mass(w, b);
    }
    return b3_world_error(w) ? -1 : 0;
}

static inline int b3s_build(B3World* w, int kind, uint64_t seed, uint64_t index) {
    switch (kind) {
    case B3S_HOVER: return b3s_build_hover(w, seed, index);
    case B3S_STACK: return b3s_build_stack(w, seed, index);
    case B3S_CHAIN: return b3s_build_chain(w, seed, index);
    case B3S_PILE: return b3s_build_pile(w, seed, index);
    case B3S_BOUNCE: return b3s_build_bounce(w, seed, index);
    case B3S_CAPSULE: return b3s_build_capsule(w, seed, index);
    default: return -1;
    }
}

/* --------------------------------------------------------------- actions */

/* Action layout per scene: kind, first body / joint index, values per world. */
B3_HD B3_INL void b3s_action_layout(int scene, int* kind, int* index, int* values) {
    switch (scene) {
    case B3S_HOVER: *kind = B3S_ACT_FORCE; *index = 1; *values = 3; break;
    case B3S_STACK: *kind = B3S_ACT_LINEAR_IMPULSE; *index = B3S_STACK_BOXES; *values = 3; break;
    case B3S_CHAIN: *kind = B3S_ACT_JOINT_TARGET; *index = 1; *values = B3S_CHAIN_LINKS - 1; break;
    default: *kind = B3S_ACT_NONE; *index = 0; *values = 0; break;
    }
}

/* Action values of world `index` for step `step` (step counts from 1):
 * hover: thrust force (U[-2,2], U[0,20], U[-2,2]) N on the sphere;
 * stack: impulse N(0,1) per axis on the top box;
 * chain: spring targets U[-1,1] rad for revolutes 1..9. */
B3_HD B3_INL void b3s_actions(int scene, uint64_t seed, uint64_t index, uint64_t step, float* out) {
    switch (scene) {
    case B3S_HOVER:
        out[0] = b3s_uniform(seed, index, step, 1, -2.0f, 2.0f);
        out[1] = b3s_uniform(seed, index, step, 2, 0.0f, 20.0f);
        out[2] = b3s_uniform(seed, index, step, 3, -2.0f, 2.0f);
        break;
    case B3S_STACK:
        out[0] = b3s_normal(seed, index, step, 1);
        out[1] = b3s_normal(seed, index, step, 2);
        out[2] = b3s_normal(seed, index, step, 3);
        break;
    case B3S_CHAIN:
        for (int k = 0; k < B3S_CHAIN_LINKS - 1; k++)
            out[k] = b3s_uniform(seed, index, step, 1u + (uint64_t)k, -1.0f, 1.0f);
        break;
    default:
        break;
    }
}

/* Apply action values to one world through the public per-world API
 * (b3_apply_force / b3_apply_linear_impulse / b3_joint_set_spring target). */
B3_HD B3_INL void b3s_apply(B3World* w, int kind, int index, int nvalues, const float* v) {
    if (kind == B3S_ACT_FORCE || kind == B3S_ACT_TORQUE || kind == B3S_ACT_LINEAR_IMPULSE) {
        for (int k = 0; 3 * k + 2 < nvalues; k++) {
            B3Vec3 a = b3_v(v[3 * k], v[3 * k + 1], v[3 * k + 2]);
            if (kind == B3S_ACT_FORCE) b3_apply_force(w, index + k, a);
            else if (kind == B3S_ACT_TORQUE) b3_apply_torque(w, index + k, a);
            else b3_apply_linear_impulse(w, index + k, a);
        }
    } else if (kind == B3S_ACT_JOINT_TARGET) {
        for (int k = 0; k < nvalues; k++)
            w->joints[index + k].target_angle = b3_clamp(v[k], -B3_PI, B3_PI);
    }
}

/* Reset mask of the scale-out run: about 1% of worlds per step. */
B3_HD B3_INL int b3s_reset_selected(uint64_t seed, uint64_t index, uint64_t step) {
    return (b3s_hash(seed ^ 0xA5A5ull, index, step, 7) >> 40) < (uint64_t)(0.01 * 16777216.0);
}

#endif /* B3_SCENES_H */
