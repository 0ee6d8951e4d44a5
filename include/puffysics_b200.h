/*
 * puffysics_b200.h -- public C header of the B200 batched rigid-body engine.
 *
 * Drop-in for the Puffysics C API on its batched stepping path:
 *   - the B3World / B3Body / B3Shape / B3Contact / B3Joint structs, byte-for-byte
 *     the layout of puffysics.cuh for the same B3_MAX_* capacities
 *     (reference src/puffysics/02_types.inl:23-367), so an environment adapter
 *     that embeds B3World in its Env keeps working unchanged;
 *   - the world-building API (b3_world_init, b3_create_*, b3_finalize_mass,
 *     b3_create_weld/revolute, b3_joint_*, b3_apply_*), host- and
 *     device-callable, producing bit-identical worlds
 *     (reference src/puffysics/04_world.inl, 06_joints.inl:5-159,
 *     09_step.inl:132-146);
 *   - B3Batch and b3_batch_step_gpu / b3_batch_restore_gpu with the reference
 *     signatures (reference b3_batch.cuh:12-99).  Those two are thin inline
 *     shims over the exported C-ABI entry points b3x_* (declared at the end),
 *     which carry the caller's capacity configuration across the library
 *     boundary: a precompiled library cannot see the B3_MAX_* macros of the
 *     translation unit that calls it.
 *
 * Capacities (B3_MAX_*) and solver iteration counts (B3_JOINT_ITERS,
 * B3_RELAX_ITERS) are set before including this header, exactly as with the
 * reference.  The library reads them at run time from each call.
 *
 * Not supported (compile error): the reference's experimental layout flags
 * B3_REVOLUTE_ONLY, B3_CACHE_JOINTS and B3_PACKED_GS.  B3_ART_CONTACTS=1 is
 * supported by the device b3_step of puffysics.cuh (see below).
 */
#ifndef PUFFYSICS_B200_H
#define PUFFYSICS_B200_H

#include <float.h>
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define B3_HD __host__ __device__
#define B3_INL __forceinline__
#elif defined(__cplusplus)
#define B3_HD
#define B3_INL inline
#else
#define B3_HD
#define B3_INL static inline
#endif

#ifdef __cplusplus
#define B3X_EXTERN_C extern "C"
#else
#define B3X_EXTERN_C
#endif
#define B3X_API B3X_EXTERN_C __attribute__((visibility("default")))

/* ---------------------------------------------------------------------------
 * Configuration (same macro names and defaults as reference
 * src/puffysics/01_config.inl:53-104).
 * ------------------------------------------------------------------------- */
#ifndef B3_MAX_BODIES
#define B3_MAX_BODIES 80
#endif
#ifndef B3_MAX_SHAPES
#define B3_MAX_SHAPES 128
#endif
#ifndef B3_MAX_CONTACTS
#define B3_MAX_CONTACTS 128
#endif
#ifndef B3_MAX_JOINTS
#define B3_MAX_JOINTS 32
#endif
#ifndef B3_JOINT_ITERS
#define B3_JOINT_ITERS 2
#endif
#ifndef B3_RELAX_ITERS
#define B3_RELAX_ITERS B3_JOINT_ITERS
#endif
#if B3_JOINT_ITERS < 1 || B3_RELAX_ITERS < 1
#error "Solver iteration counts must be positive"
#endif
#if defined(B3_REVOLUTE_ONLY) || defined(B3_CACHE_JOINTS) || defined(B3_PACKED_GS)
#error "puffysics_b200 implements the default joint layout only"
#endif
/* B3_ART_CONTACTS=1 (reference 01_config.inl:43, 185-187): contacts of
 * worlds with joints are resolved through the articulation of their
 * revolute joints.  Run by the device b3_step of puffysics.cuh (built in
 * when the macro is 1); b3_batch_step_gpu then steps with that per-thread
 * b3_step, as with a force hook. */
#ifndef B3_ART_CONTACTS
#define B3_ART_CONTACTS 0
#endif
/* Optional per-substep force hook (reference 01_config.inl:186-198): code the
 * including translation unit runs on a B3World* w and substep h before each
 * velocity integration; its force / torque additions last one substep.  Run
 * by the device b3_step of puffysics.cuh; with a hook, b3_batch_step_gpu steps
 * with that per-thread b3_step (a precompiled library cannot run the hook). */
#ifndef B3_USER_FORCES
#define B3_USER_FORCES(w, h) ((void)0)
#define B3_HAS_USER_FORCES 0
#else
#define B3_HAS_USER_FORCES 1
#endif
#define B3_CONNECT_WORDS ((B3_MAX_BODIES + 63) / 64)

/* 16 bits per capacity, bodies in the low word (reference 01_config.inl:70-74). */
#define B3_CONFIG_SIGNATURE ( \
    ((unsigned long long)(B3_MAX_BODIES) & 0xffffull) \
  | (((unsigned long long)(B3_MAX_SHAPES) & 0xffffull) << 16) \
  | (((unsigned long long)(B3_MAX_CONTACTS) & 0xffffull) << 32) \
  | (((unsigned long long)(B3_MAX_JOINTS) & 0xffffull) << 48))

#define B3_PI 3.14159265359f
#define B3_LINEAR_SLOP 0.005f
#define B3_SPECULATIVE 0.020f
#define B3_MAX_MANIFOLD 4
#define B3_MAX_ROTATION (0.25f * B3_PI)
#define B3_MIN_FRICTION_W 1.0e-10f

#define B3_STATIC 0
#define B3_KINEMATIC 1
#define B3_DYNAMIC 2

#define B3_SPHERE 0
#define B3_CAPSULE 1
#define B3_BOX 2

#define B3_JOINT_WELD 0
#define B3_JOINT_REVOLUTE 1

#define B3_FLAG_DYNAMIC 0x00001000u
#define B3_LOCK_LIN_X 0x00000001u
#define B3_LOCK_LIN_Y 0x00000002u
#define B3_LOCK_LIN_Z 0x00000004u
#define B3_LOCK_ANG_X 0x00000008u
#define B3_LOCK_ANG_Y 0x00000010u
#define B3_LOCK_ANG_Z 0x00000020u

/* ---------------------------------------------------------------------------
 * Types.  Member names, order and widths are the ABI (reference
 * src/puffysics/02_types.inl:23-367); sizes are checked below.
 * ------------------------------------------------------------------------- */
typedef struct B3Vec3 { float x, y, z; } B3Vec3;
typedef struct B3Vec2 { float x, y; } B3Vec2;
typedef struct B3Quat { B3Vec3 v; float s; } B3Quat;
typedef struct B3Mat3 { B3Vec3 cx, cy, cz; } B3Mat3;
typedef struct B3Mat2 { B3Vec2 cx, cy; } B3Mat2;
typedef struct B3AABB { B3Vec3 lo, hi; } B3AABB;
typedef struct B3Soft { float bias_rate, mass_scale, impulse_scale; } B3Soft;

typedef struct B3Body {
    B3Vec3 position;
    B3Quat rotation;
    B3Vec3 center;
    B3Vec3 local_center;
    B3Vec3 lin_vel;
    B3Vec3 ang_vel;
    B3Vec3 force;
    B3Vec3 torque;
    B3Vec3 delta_pos;
    B3Quat delta_rot;
    float inv_mass;
    B3Vec3 inv_inertia;
    B3Mat3 inv_i_world;
    float linear_damping;
    float angular_damping;
    float gravity_scale;
    int type;
    uint32_t flags;
} B3Body;

typedef struct B3Shape {
    int body;
    int type;
    B3Vec3 local_pos;
    B3Quat local_rot;
    float radius;
    B3Vec3 half;
    float friction;
    float restitution;
    float rolling;
    float density;
    uint64_t category;
    uint64_t mask;
} B3Shape;

typedef struct B3Point {
    B3Vec3 r_a;
    B3Vec3 r_b;
    float base_sep;
    float rel_vel;
    float normal_impulse;
    float total_normal;
    float normal_mass;
    float lever;
    uint32_t feature;
} B3Point;

typedef struct B3Contact {
    int shape_a;
    int shape_b;
    int body_a;
    int body_b;
    int point_count;
    int static_contact;
    B3Vec3 normal;
    B3Vec3 tangent1;
    B3Vec3 tangent2;
    B3Point points[B3_MAX_MANIFOLD];
    B3Vec3 center_a;
    B3Vec3 center_b;
    float friction;
    float restitution;
    float rolling;
    float twist_mass;
    float twist_impulse;
    B3Vec2 friction_impulse;
    B3Vec3 rolling_impulse;
    B3Mat2 tangent_mass;
    B3Mat3 rolling_mass;
    float inv_mass_a;
    float inv_mass_b;
    B3Mat3 inv_i_a;
    B3Mat3 inv_i_b;
    B3Soft softness;
} B3Contact;

typedef struct B3Joint {
    int type;
    int body_a;
    int body_b;
    int collide_connected;
    int fixed_rotation;
    B3Vec3 local_anchor_a;
    B3Vec3 local_anchor_b;
    B3Quat local_rot_a;
    B3Quat local_rot_b;
    float constraint_hertz;
    float constraint_damping;
    B3Soft softness;
    float inv_mass_a;
    float inv_mass_b;
    B3Mat3 inv_i_a;
    B3Mat3 inv_i_b;
    B3Vec3 frame_p_a;
    B3Vec3 frame_p_b;
    B3Quat frame_q_a;
    B3Quat frame_q_b;
    B3Vec3 delta_center;
    B3Vec3 linear_impulse;
    B3Vec3 angular_impulse;
    B3Mat3 angular_mass;
    float linear_hertz;
    float linear_damping;
    float angular_hertz;
    float angular_damping;
    B3Soft linear_spring;
    B3Soft angular_spring;
    B3Vec2 perp_impulse;
    float spring_impulse;
    float motor_impulse;
    float lower_impulse;
    float upper_impulse;
    float hertz;
    float damping_ratio;
    float max_motor_torque;
    float motor_speed;
    float target_angle;
    float lower_angle;
    float upper_angle;
    int enable_spring;
    int enable_motor;
    int enable_limit;
    B3Vec3 rotation_axis;
    B3Vec3 perp_x;
    B3Vec3 perp_y;
    float axial_mass;
    B3Soft spring_softness;
} B3Joint;

typedef struct B3World {
    B3Vec3 gravity;
    float contact_hertz;
    float contact_damping;
    float contact_speed;
    float restitution_threshold;
    float max_linear_speed;
    int body_count;
    int shape_count;
    int contact_count;
    int joint_count;
    int body_overflow;
    int shape_overflow;
    int joint_overflow;
    int contact_overflow;
    int contacts_dropped;
    B3Body bodies[B3_MAX_BODIES];
    B3Shape shapes[B3_MAX_SHAPES];
    B3Contact contacts[B3_MAX_CONTACTS];
    B3Joint joints[B3_MAX_JOINTS];
} B3World;

typedef struct B3StepStats {
    int body_count;
    int shape_count;
    int contact_count;
    int joint_count;
    int body_overflow;
    int shape_overflow;
    int joint_overflow;
    int contact_overflow;
    int contacts_dropped;
} B3StepStats;

typedef struct B3BodyDef {
    int type;
    B3Vec3 position;
    B3Quat rotation;
    B3Vec3 lin_vel;
    B3Vec3 ang_vel;
    float linear_damping;
    float angular_damping;
    float gravity_scale;
    uint32_t flags;
} B3BodyDef;

typedef struct B3ShapeDef {
    float density;
    float friction;
    float restitution;
    float rolling;
    uint64_t category;
    uint64_t mask;
} B3ShapeDef;

/* Non-owning strided view of count worlds (reference b3_batch.cuh:12-17). */
typedef struct B3Batch {
    void* data;
    size_t stride;
    size_t world_offset;
    int count;
} B3Batch;

/* Byte sizes the kernels assume when they decode a world at run time. */
#define B3X_WORLD_HEADER_BYTES 68
#define B3X_BODY_BYTES 200
#define B3X_SHAPE_BYTES 88
#define B3X_POINT_BYTES 52
#define B3X_CONTACT_BYTES 476
#define B3X_JOINT_BYTES 460

#if defined(__cplusplus)
#define B3X_STATIC_ASSERT(c, m) static_assert(c, m)
#else
#define B3X_STATIC_ASSERT(c, m) _Static_assert(c, m)
#endif
B3X_STATIC_ASSERT(sizeof(B3Body) == B3X_BODY_BYTES, "B3Body layout");
B3X_STATIC_ASSERT(sizeof(B3Shape) == B3X_SHAPE_BYTES, "B3Shape layout");
B3X_STATIC_ASSERT(sizeof(B3Point) == B3X_POINT_BYTES, "B3Point layout");
B3X_STATIC_ASSERT(sizeof(B3Contact) == B3X_CONTACT_BYTES, "B3Contact layout");
B3X_STATIC_ASSERT(sizeof(B3Joint) == B3X_JOINT_BYTES, "B3Joint layout");
B3X_STATIC_ASSERT(offsetof(B3World, bodies) == B3X_WORLD_HEADER_BYTES, "B3World header");

/* ---------------------------------------------------------------------------
 * Small vector / quaternion helpers (the public names adapters use; the
 * arithmetic order of each matches reference src/puffysics/03_math.inl).
 * ------------------------------------------------------------------------- */
B3_HD B3_INL B3Vec3 b3_v(float x, float y, float z) { B3Vec3 r; r.x = x; r.y = y; r.z = z; return r; }
B3_HD B3_INL B3Vec3 b3_add(B3Vec3 a, B3Vec3 b) { return b3_v(a.x + b.x, a.y + b.y, a.z + b.z); }
B3_HD B3_INL B3Vec3 b3_sub(B3Vec3 a, B3Vec3 b) { return b3_v(a.x - b.x, a.y - b.y, a.z - b.z); }
B3_HD B3_INL B3Vec3 b3_neg(B3Vec3 a) { return b3_v(-a.x, -a.y, -a.z); }
B3_HD B3_INL B3Vec3 b3_mul(B3Vec3 a, float s) { return b3_v(a.x * s, a.y * s, a.z * s); }
B3_HD B3_INL B3Vec3 b3_madd(B3Vec3 a, float s, B3Vec3 b) { return b3_v(a.x + s * b.x, a.y + s * b.y, a.z + s * b.z); }
B3_HD B3_INL B3Vec3 b3_msub(B3Vec3 a, float s, B3Vec3 b) { return b3_v(a.x - s * b.x, a.y - s * b.y, a.z - s * b.z); }
B3_HD B3_INL float b3_dot(B3Vec3 a, B3Vec3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
B3_HD B3_INL B3Vec3 b3_cross(B3Vec3 a, B3Vec3 b) {
    return b3_v(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x);
}
B3_HD B3_INL float b3_len2(B3Vec3 a) { return b3_dot(a, a); }
B3_HD B3_INL float b3_len(B3Vec3 a) { return sqrtf(b3_len2(a)); }
B3_HD B3_INL float b3_maxf(float a, float b) { return a > b ? a : b; }
B3_HD B3_INL float b3_minf(float a, float b) { return a < b ? a : b; }
B3_HD B3_INL float b3_clamp(float x, float lo, float hi) { return x < lo ? lo : (x > hi ? hi : x); }
B3_HD B3_INL B3Vec3 b3_norm(B3Vec3 a) {
    float l2 = b3_len2(a);
    if (l2 > 0.0f) {
        float k = 1.0f / sqrtf(l2);
        return b3_mul(a, k);
    }
    return b3_v(0.0f, 1.0f, 0.0f);
}
B3_HD B3_INL B3Quat b3_q(float x, float y, float z, float s) { B3Quat q; q.v = b3_v(x, y, z); q.s = s; return q; }
B3_HD B3_INL B3Quat b3_q_id(void) { return b3_q(0.0f, 0.0f, 0.0f, 1.0f); }
B3_HD B3_INL float b3_qdot(B3Quat a, B3Quat b) { return b3_dot(a.v, b.v) + a.s * b.s; }
B3_HD B3_INL B3Quat b3_qnorm(B3Quat q) {
    float d2 = b3_qdot(q, q);
    if (d2 <= 0.0f) return b3_q_id();
    float k = 1.0f / sqrtf(d2);
    return b3_q(q.v.x * k, q.v.y * k, q.v.z * k, q.s * k);
}
B3_HD B3_INL B3Quat b3_qmul(B3Quat a, B3Quat b) {
    B3Quat r;
    r.v = b3_add(b3_add(b3_mul(b.v, a.s), b3_mul(a.v, b.s)), b3_cross(a.v, b.v));
    r.s = a.s * b.s - b3_dot(a.v, b.v);
    return r;
}
B3_HD B3_INL B3Quat b3_qconj(B3Quat q) { return b3_q(-q.v.x, -q.v.y, -q.v.z, q.s); }
B3_HD B3_INL B3Quat b3_qneg(B3Quat q) { return b3_q(-q.v.x, -q.v.y, -q.v.z, -q.s); }
B3_HD B3_INL B3Vec3 b3_rotate(B3Quat q, B3Vec3 v) {
    B3Vec3 t = b3_mul(b3_cross(q.v, v), 2.0f);
    return b3_add(v, b3_add(b3_mul(t, q.s), b3_cross(q.v, t)));
}
B3_HD B3_INL B3Vec3 b3_inv_rotate(B3Quat q, B3Vec3 v) { return b3_rotate(b3_qconj(q), v); }
/* conj(a) * b, expanded (reference 03_math.inl:273-278). */
B3_HD B3_INL B3Quat b3_qinv_mul(B3Quat a, B3Quat b) {
    B3Vec3 t = b3_msub(b3_madd(b3_cross(b.v, a.v), a.s, b.v), b.s, a.v);
    return b3_q(t.x, t.y, t.z, a.s * b.s + b3_dot(a.v, b.v));
}
B3_HD B3_INL B3Vec3 b3_xf_point(B3Vec3 p, B3Quat q, B3Vec3 local) { return b3_add(p, b3_rotate(q, local)); }
B3_HD B3_INL void b3_axes(B3Quat q, B3Vec3* x, B3Vec3* y, B3Vec3* z) {
    *x = b3_rotate(q, b3_v(1.0f, 0.0f, 0.0f));
    *y = b3_rotate(q, b3_v(0.0f, 1.0f, 0.0f));
    *z = b3_rotate(q, b3_v(0.0f, 0.0f, 1.0f));
}
B3_HD B3_INL B3Vec3 b3_mv(B3Mat3 m, B3Vec3 v) {
    return b3_add(b3_add(b3_mul(m.cx, v.x), b3_mul(m.cy, v.y)), b3_mul(m.cz, v.z));
}
/* Diagonal body inverse inertia rotated to world (reference 03_math.inl:187-198). */
B3_HD B3_INL B3Mat3 b3_world_inv_i(B3Quat q, B3Vec3 inv) {
    B3Vec3 ax, ay, az;
    b3_axes(q, &ax, &ay, &az);
    B3Mat3 r;
    r.cx = b3_add(b3_add(b3_mul(ax, inv.x * ax.x), b3_mul(ay, inv.y * ay.x)), b3_mul(az, inv.z * az.x));
    r.cy = b3_add(b3_add(b3_mul(ax, inv.x * ax.y), b3_mul(ay, inv.y * ay.y)), b3_mul(az, inv.z * az.y));
    r.cz = b3_add(b3_add(b3_mul(ax, inv.x * ax.z), b3_mul(ay, inv.y * ay.z)), b3_mul(az, inv.z * az.z));
    return r;
}
B3_HD B3_INL B3Vec3 b3_perp(B3Vec3 n) {
    if (fabsf(n.x) >= 0.57735027f) return b3_norm(b3_v(-n.y, n.x, 0.0f));
    return b3_norm(b3_v(0.0f, -n.z, n.y));
}
B3_HD B3_INL B3Quat b3_q_axis_angle(B3Vec3 axis, float radians) {
    B3Vec3 u = b3_norm(axis);
    float half = 0.5f * radians;
    float s = sinf(half);
    return b3_q(s * u.x, s * u.y, s * u.z, cosf(half));
}
/* Shortest rotation taking +z to z (reference 03_math.inl:328-341). */
B3_HD B3_INL B3Quat b3_q_from_z(B3Vec3 z) {
    B3Vec3 u = b3_norm(z);
    float d = b3_dot(b3_v(0.0f, 0.0f, 1.0f), u);
    if (d > 0.999999f) return b3_q_id();
    if (d < -0.999999f) {
        B3Vec3 a = b3_perp(b3_v(0.0f, 0.0f, 1.0f));
        return b3_q(a.x, a.y, a.z, 0.0f);
    }
    B3Vec3 a = b3_cross(b3_v(0.0f, 0.0f, 1.0f), u);
    return b3_qnorm(b3_q(a.x, a.y, a.z, 1.0f + d));
}

/* ---------------------------------------------------------------------------
 * World construction (reference src/puffysics/04_world.inl).
 * ------------------------------------------------------------------------- */
B3_HD B3_INL B3BodyDef b3_default_body(void) {
    B3BodyDef d;
    memset(&d, 0, sizeof(d));
    d.type = B3_STATIC;
    d.rotation = b3_q_id();
    d.gravity_scale = 1.0f;
    return d;
}

B3_HD B3_INL B3ShapeDef b3_default_shape(void) {
    B3ShapeDef d;
    d.density = 1000.0f;
    d.friction = 0.6f;
    d.restitution = 0.0f;
    d.rolling = 0.0f;
    d.category = ~0ull;
    d.mask = ~0ull;
    return d;
}

B3_HD B3_INL void b3_world_init(B3World* w) {
    memset(w, 0, sizeof(*w));
    w->gravity = b3_v(0.0f, -10.0f, 0.0f);
    w->contact_hertz = 30.0f;
    w->contact_damping = 10.0f;
    w->contact_speed = 3.0f;
    w->restitution_threshold = 1.0f;
    w->max_linear_speed = 400.0f;
}

B3_HD B3_INL int b3_body_capacity(void) { return B3_MAX_BODIES; }
B3_HD B3_INL int b3_shape_capacity(void) { return B3_MAX_SHAPES; }
B3_HD B3_INL int b3_contact_capacity(void) { return B3_MAX_CONTACTS; }
B3_HD B3_INL int b3_joint_capacity(void) { return B3_MAX_JOINTS; }
B3_HD B3_INL unsigned long long b3_config_signature(void) { return B3_CONFIG_SIGNATURE; }
B3_HD B3_INL int b3_config_matches(unsigned long long sig) { return sig == B3_CONFIG_SIGNATURE; }

B3_HD B3_INL void b3_clear_errors(B3World* w) {
    w->body_overflow = 0;
    w->shape_overflow = 0;
    w->joint_overflow = 0;
    w->contact_overflow = 0;
    w->contacts_dropped = 0;
}

B3_HD B3_INL int b3_world_error(const B3World* w) {
    return (w->body_overflow || w->shape_overflow || w->joint_overflow || w->contact_overflow);
}

B3_HD B3_INL int b3_step_stats(const B3World* w, B3StepStats* out) {
    out->body_count = w->body_count;
    out->shape_count = w->shape_count;
    out->contact_count = w->contact_count;
    out->joint_count = w->joint_count;
    out->body_overflow = w->body_overflow;
    out->shape_overflow = w->shape_overflow;
    out->joint_overflow = w->joint_overflow;
    out->contact_overflow = w->contact_overflow;
    out->contacts_dropped = w->contacts_dropped;
    return b3_world_error(w);
}

B3_HD B3_INL int b3_create_body(B3World* w, const B3BodyDef* def) {
    if (w->body_count >= B3_MAX_BODIES) {
        w->body_overflow = 1;
        return -1;
    }
    int id = w->body_count++;
    B3Body* b = &w->bodies[id];
    memset(b, 0, sizeof(*b));
    b->position = def->position;
    b->rotation = b3_qnorm(def->rotation);
    b->center = def->position;
    b->lin_vel = def->lin_vel;
    b->ang_vel = def->ang_vel;
    b->delta_rot = b3_q_id();
    b->linear_damping = def->linear_damping;
    b->angular_damping = def->angular_damping;
    b->gravity_scale = def->gravity_scale;
    b->type = def->type;
    b->flags = def->flags | (def->type == B3_DYNAMIC ? B3_FLAG_DYNAMIC : 0u);
    return id;
}

B3_HD B3_INL int b3_add_shape(B3World* w, int body, int type, B3Vec3 local_pos,
        B3Quat local_rot, float radius, B3Vec3 half, const B3ShapeDef* def) {
    if (w->shape_count >= B3_MAX_SHAPES || body < 0 || body >= w->body_count
            || type < B3_SPHERE || type > B3_BOX) {
        w->shape_overflow = 1;
        return -1;
    }
    int id = w->shape_count++;
    B3Shape* s = &w->shapes[id];
    s->body = body;
    s->type = type;
    s->local_pos = local_pos;
    s->local_rot = b3_qnorm(local_rot);
    s->radius = radius;
    s->half = half;
    s->friction = def->friction;
    s->restitution = def->restitution;
    s->rolling = def->rolling;
    s->density = def->density;
    s->category = def->category;
    s->mask = def->mask;
    return id;
}

B3_HD B3_INL int b3_create_sphere(B3World* w, int body, B3Vec3 c, float r, const B3ShapeDef* def) {
    return b3_add_shape(w, body, B3_SPHERE, c, b3_q_id(), r, b3_v(0.0f, 0.0f, 0.0f), def);
}
B3_HD B3_INL int b3_create_capsule(B3World* w, int body, float half_len, float r, const B3ShapeDef* def) {
    return b3_add_shape(w, body, B3_CAPSULE, b3_v(0.0f, 0.0f, 0.0f), b3_q_id(), r,
        b3_v(0.0f, half_len, 0.0f), def);
}
B3_HD B3_INL int b3_create_box(B3World* w, int body, B3Vec3 half, const B3ShapeDef* def) {
    return b3_add_shape(w, body, B3_BOX, b3_v(0.0f, 0.0f, 0.0f), b3_q_id(), 0.0f, half, def);
}
B3_HD B3_INL int b3_create_box_local(B3World* w, int body, B3Vec3 half, B3Vec3 local_pos,
        B3Quat local_rot, const B3ShapeDef* def) {
    return b3_add_shape(w, body, B3_BOX, local_pos, local_rot, 0.0f, half, def);
}

B3_HD B3_INL void b3x_write_inv_mass(B3Body* b, float inv_mass, B3Vec3 inertia) {
    b->inv_mass = inv_mass;
    b->inv_inertia = b3_v(inertia.x > 0.0f ? 1.0f / inertia.x : 0.0f,
        inertia.y > 0.0f ? 1.0f / inertia.y : 0.0f,
        inertia.z > 0.0f ? 1.0f / inertia.z : 0.0f);
    b->inv_i_world = b3_world_inv_i(b->rotation, b->inv_inertia);
}

B3_HD B3_INL void b3_set_inertial(B3World* w, int body, float mass, B3Vec3 local_com, B3Vec3 inertia) {
    B3Body* b = &w->bodies[body];
    b->local_center = local_com;
    b->center = b3_xf_point(b->position, b->rotation, local_com);
    if (b->type != B3_DYNAMIC || mass <= 0.0f) {
        b3x_write_inv_mass(b, 0.0f, b3_v(0.0f, 0.0f, 0.0f));
        return;
    }
    b3x_write_inv_mass(b, 1.0f / mass, inertia);
}

/* Mass, centre and principal inertia of one shape (reference 04_world.inl:193-231). */
B3_HD B3_INL void b3_shape_mass(const B3Shape* s, float* mass, B3Vec3* com, B3Vec3* inertia) {
    *com = s->local_pos;
    if (s->type == B3_SPHERE) {
        float r = s->radius;
        float m = (4.0f / 3.0f) * B3_PI * r * r * r * s->density;
        float i = 0.4f * m * r * r;
        *mass = m;
        *inertia = b3_v(i, i, i);
    } else if (s->type == B3_BOX) {
        float hx = s->half.x, hy = s->half.y, hz = s->half.z;
        float m = 8.0f * hx * hy * hz * s->density;
        float k = m / 3.0f;
        *mass = m;
        *inertia = b3_v(k * (hy * hy + hz * hz), k * (hx * hx + hz * hz), k * (hx * hx + hy * hy));
    } else {
        float r = s->radius;
        float h = 2.0f * s->half.y;
        float cyl_m = (B3_PI * r * r * h) * s->density;
        float sph_m = ((4.0f / 3.0f) * B3_PI * r * r * r) * s->density;
        float m = cyl_m + sph_m;
        float ix = 0.5f * cyl_m * r * r + 0.4f * sph_m * r * r;
        float iy = (1.0f / 12.0f) * cyl_m * (3.0f * r * r + h * h)
            + 0.4f * sph_m * r * r + 0.125f * sph_m * (3.0f * r + 2.0f * h) * h;
        *mass = m;
        *inertia = b3_v(iy, ix, iy);
    }
}

/* Combined mass, centre and diagonal inertia of all shapes on a body
 * (reference 04_world.inl:233-287; off-diagonal terms dropped there too). */
B3_HD B3_INL void b3_finalize_mass_of(B3Body* b, B3Shape* shapes, int n, int body) {
    if (b->type != B3_DYNAMIC) {
        b3x_write_inv_mass(b, 0.0f, b3_v(0.0f, 0.0f, 0.0f));
        b->center = b->position;
        return;
    }
    float mass = 0.0f;
    B3Vec3 com = b3_v(0.0f, 0.0f, 0.0f);
    for (int i = 0; i < n; i++) {
        const B3Shape* s = &shapes[i];
        if (s->body != body || s->density <= 0.0f) continue;
        float sm; B3Vec3 sc, si;
        b3_shape_mass(s, &sm, &sc, &si);
        mass += sm;
        com = b3_madd(com, sm, sc);
    }
    if (mass <= 0.0f) {
        b->inv_mass = 0.0f;
        b->inv_inertia = b3_v(0.0f, 0.0f, 0.0f);
        return;
    }
    com = b3_mul(com, 1.0f / mass);
    b->local_center = com;
    b->center = b3_xf_point(b->position, b->rotation, com);
    B3Vec3 diag = b3_v(0.0f, 0.0f, 0.0f);
    for (int i = 0; i < n; i++) {
        const B3Shape* s = &shapes[i];
        if (s->body != body || s->density <= 0.0f) continue;
        float sm; B3Vec3 sc, si, ax, ay, az;
        b3_shape_mass(s, &sm, &sc, &si);
        b3_axes(s->local_rot, &ax, &ay, &az);
        B3Vec3 d = b3_sub(sc, com);
        float d2 = b3_dot(d, d);
        diag.x += si.x * ax.x * ax.x + si.y * ay.x * ay.x + si.z * az.x * az.x + sm * (d2 - d.x * d.x);
        diag.y += si.x * ax.y * ax.y + si.y * ay.y * ay.y + si.z * az.y * az.y + sm * (d2 - d.y * d.y);
        diag.z += si.x * ax.z * ax.z + si.y * ay.z * ay.z + si.z * az.z * az.z + sm * (d2 - d.z * d.z);
    }
    b3x_write_inv_mass(b, 1.0f / mass, diag);
}

B3_HD B3_INL void b3_finalize_mass(B3World* w, int body) {
    b3_finalize_mass_of(&w->bodies[body], w->shapes, w->shape_count, body);
}

/* ---------------------------------------------------------------------------
 * Joints (reference src/puffysics/06_joints.inl:5-159).
 * ------------------------------------------------------------------------- */
B3_HD B3_INL B3Joint* b3_add_joint(B3World* w, int type, int body_a, int body_b,
        B3Vec3 anchor_a, B3Vec3 anchor_b, B3Quat rot_a, B3Quat rot_b) {
    if (w->joint_count >= B3_MAX_JOINTS || body_a < 0 || body_a >= w->body_count
            || body_b < 0 || body_b >= w->body_count) {
        w->joint_overflow = 1;
        return NULL;
    }
    B3Joint* j = &w->joints[w->joint_count++];
    memset(j, 0, sizeof(*j));
    j->type = type;
    j->body_a = body_a;
    j->body_b = body_b;
    j->local_anchor_a = anchor_a;
    j->local_anchor_b = anchor_b;
    j->local_rot_a = b3_qnorm(rot_a);
    j->local_rot_b = b3_qnorm(rot_b);
    j->constraint_hertz = 90.0f;
    j->constraint_damping = 2.0f;
    return j;
}

B3_HD B3_INL int b3_create_weld(B3World* w, int body_a, int body_b, B3Vec3 local_anchor_a,
        B3Vec3 local_anchor_b) {
    if (body_a < 0 || body_a >= w->body_count || body_b < 0 || body_b >= w->body_count) {
        w->joint_overflow = 1;
        return -1;
    }
    B3Quat rot_b = b3_qinv_mul(w->bodies[body_b].rotation, w->bodies[body_a].rotation);
    B3Joint* j = b3_add_joint(w, B3_JOINT_WELD, body_a, body_b, local_anchor_a, local_anchor_b,
        b3_q_id(), rot_b);
    return j ? (int)(j - w->joints) : -1;
}

B3_HD B3_INL int b3_create_revolute(B3World* w, int body_a, int body_b, B3Vec3 local_anchor_a,
        B3Vec3 local_anchor_b, B3Vec3 local_axis_a) {
    if (body_a < 0 || body_a >= w->body_count || body_b < 0 || body_b >= w->body_count) {
        w->joint_overflow = 1;
        return -1;
    }
    B3Quat rot_a = b3_q_from_z(local_axis_a);
    B3Quat frame = b3_qmul(w->bodies[body_a].rotation, rot_a);
    B3Quat rot_b = b3_qinv_mul(w->bodies[body_b].rotation, frame);
    B3Joint* j = b3_add_joint(w, B3_JOINT_REVOLUTE, body_a, body_b, local_anchor_a, local_anchor_b,
        rot_a, rot_b);
    return j ? (int)(j - w->joints) : -1;
}

B3_HD B3_INL void b3_joint_enable_motor(B3World* w, int joint, int enable) {
    B3Joint* j = &w->joints[joint];
    if (j->enable_motor != enable) j->motor_impulse = 0.0f;
    j->enable_motor = enable;
}
B3_HD B3_INL void b3_joint_set_motor(B3World* w, int joint, float speed, float max_torque) {
    B3Joint* j = &w->joints[joint];
    j->motor_speed = speed;
    j->max_motor_torque = b3_maxf(max_torque, 0.0f);
}
B3_HD B3_INL void b3_joint_enable_limit(B3World* w, int joint, int enable) {
    B3Joint* j = &w->joints[joint];
    if (j->enable_limit != enable) {
        j->lower_impulse = 0.0f;
        j->upper_impulse = 0.0f;
    }
    j->enable_limit = enable;
}
B3_HD B3_INL void b3_joint_set_limits(B3World* w, int joint, float lower, float upper) {
    B3Joint* j = &w->joints[joint];
    float lo = b3_minf(lower, upper), hi = b3_maxf(lower, upper);
    j->lower_angle = b3_clamp(lo, -0.99f * B3_PI, 0.99f * B3_PI);
    j->upper_angle = b3_clamp(hi, -0.99f * B3_PI, 0.99f * B3_PI);
}
B3_HD B3_INL void b3_joint_enable_spring(B3World* w, int joint, int enable) {
    B3Joint* j = &w->joints[joint];
    if (j->enable_spring != enable) j->spring_impulse = 0.0f;
    j->enable_spring = enable;
}
B3_HD B3_INL void b3_joint_set_spring(B3World* w, int joint, float target, float hertz, float damping) {
    B3Joint* j = &w->joints[joint];
    j->target_angle = b3_clamp(target, -B3_PI, B3_PI);
    j->hertz = b3_maxf(hertz, 0.0f);
    j->damping_ratio = b3_maxf(damping, 0.0f);
}

/* Hinge twist: twice the angle of the z-axis part of q, with q taken in the
 * hemisphere s >= 0 (reference 03_math.inl:293-309, default atan2f path). */
B3_HD B3_INL float b3_twist(B3Quat q) {
    float t = q.s < 0.0f ? atan2f(-q.v.z, -q.s) : atan2f(q.v.z, q.s);
    return 2.0f * t;
}

B3_HD B3_INL float b3_joint_angle(const B3World* w, int joint) {
    const B3Joint* j = &w->joints[joint];
    B3Quat qa = b3_qmul(w->bodies[j->body_a].rotation, j->local_rot_a);
    B3Quat qb = b3_qmul(w->bodies[j->body_b].rotation, j->local_rot_b);
    if (b3_qdot(qa, qb) < 0.0f) qb = b3_qneg(qb);
    return b3_twist(b3_qinv_mul(qa, qb));
}

B3_HD B3_INL float b3_joint_speed(const B3World* w, int joint) {
    const B3Joint* j = &w->joints[joint];
    B3Vec3 axis = b3_rotate(b3_qmul(w->bodies[j->body_a].rotation, j->local_rot_a), b3_v(0.0f, 0.0f, 1.0f));
    return b3_dot(b3_sub(w->bodies[j->body_b].ang_vel, w->bodies[j->body_a].ang_vel), axis);
}

/* ---------------------------------------------------------------------------
 * Actions (reference src/puffysics/09_step.inl:132-146).  Forces and torques
 * act over the whole next step and are cleared by it.
 * ------------------------------------------------------------------------- */
B3_HD B3_INL void b3_apply_force(B3World* w, int body, B3Vec3 force) {
    w->bodies[body].force = b3_add(w->bodies[body].force, force);
}
B3_HD B3_INL void b3_apply_torque(B3World* w, int body, B3Vec3 torque) {
    w->bodies[body].torque = b3_add(w->bodies[body].torque, torque);
}
B3_HD B3_INL void b3_apply_linear_impulse(B3World* w, int body, B3Vec3 impulse) {
    B3Body* b = &w->bodies[body];
    if (b->type == B3_DYNAMIC) b->lin_vel = b3_madd(b->lin_vel, b->inv_mass, impulse);
}

/* ---------------------------------------------------------------------------
 * Batches (reference b3_batch.cuh:19-33).
 * ------------------------------------------------------------------------- */
B3_HD B3_INL int b3_batch_valid(B3Batch batch) {
    if (batch.count < 0) return 0;
    if (batch.count == 0) return 1;
    return batch.data != NULL && batch.stride >= sizeof(B3World)
        && batch.world_offset <= batch.stride - sizeof(B3World)
        && (size_t)batch.count <= SIZE_MAX / batch.stride;
}
B3_HD B3_INL B3World* b3_batch_world(B3Batch batch, int index) {
    return (B3World*)((unsigned char*)batch.data + (size_t)index * batch.stride + batch.world_offset);
}

/* ---------------------------------------------------------------------------
 * Exported C-ABI of libpuffysics_b200.so.  Return values are cudaError_t
 * codes (0 = cudaSuccess, 1 = cudaErrorInvalidValue, ...).  `stream` is a
 * cudaStream_t.  `config_signature` is B3_CONFIG_SIGNATURE of the caller.
 * ------------------------------------------------------------------------- */

/* Step every selected world once on the GPU.  Replaces b3_batch_step_gpu
 * (reference b3_batch.cuh:81-89): same validation (invalid batch, non-finite
 * or negative dt, substeps < 1 -> 1, nothing launched or written), same no-op
 * cases (count == 0 or dt == 0 -> 0), same mask meaning (NULL = all worlds,
 * nonzero byte = selected; unselected worlds are not written).  Additionally
 * rejects world addresses or strides that are not 8-byte aligned.  Like the
 * reference (b3_batch.cuh:77-80) it only enqueues on `stream`: no allocation,
 * no synchronisation.  Its workspace is the one b3x_reserve_workspace made
 * for `stream` (set-up), else a fixed 128 MiB array inside the library, on
 * which it runs as many tiles per launch as fit (slower for large batches);
 * calls on the array from different streams are ordered on the GPU with an
 * event, except while the stream is being captured into a CUDA graph (reserve
 * a workspace for capture streams).  A capacity configuration whose tile slot
 * exceeds the array needs a reservation: 2 (cudaErrorMemoryAllocation)
 * without one.  The library's kernels load on a device at its first call:
 * make that call before any stream capture. */
B3X_API int b3x_batch_step_gpu(B3Batch batch, float dt, int substeps, const unsigned char* active,
    void* stream, unsigned long long config_signature, int joint_iters, int relax_iters);

/* The same step in the reference's alternative step modes, selected there by
 * compile-time macros of the translation unit (reference 01_config.inl:50-52):
 *   B3X_STEP_INTERLEAVE_CONTACTS  (B3_INTERLEAVE_CONTACTS) contacts are swept
 *       at the start of every joint iteration, bias and relax phases, instead
 *       of once per phase (07_packed.inl:61-65, 09_step.inl:169-177);
 *   B3X_STEP_SKIP_RESTITUTION     (B3_SKIP_RESTITUTION) no restitution pass
 *       (09_step.inl:178-180).
 * Unknown flag bits -> 1 (invalid), nothing launched. */
#define B3X_STEP_INTERLEAVE_CONTACTS 1
#define B3X_STEP_SKIP_RESTITUTION 2
B3X_API int b3x_batch_step_gpu_flags(B3Batch batch, float dt, int substeps, const unsigned char* active,
    void* stream, unsigned long long config_signature, int joint_iters, int relax_iters, int flags);

/* Same step with a caller-owned device workspace of at least
 * b3x_workspace_bytes(...) bytes (256-byte aligned): never allocates.
 * Work queued on different streams must use different workspaces. */
B3X_API int b3x_batch_step_gpu_ws(B3Batch batch, float dt, int substeps, const unsigned char* active,
    void* stream, unsigned long long config_signature, int joint_iters, int relax_iters,
    void* workspace, size_t workspace_bytes);

/* No counterpart in the reference.  The step of b3x_batch_step_gpu for
 * callers that cannot allocate device memory when they step (memory owned by
 * a framework allocator or plugin host that forbids cudaMalloc, real-time
 * loops that cannot risk an allocation's synchronisation): the workspace is a
 * fixed 64 MiB array inside the library, reserved on every device that loads
 * it, never a reservation.  Calls nothing that allocates.  Every call looks
 * up the array's device address on the current device; the first call on a
 * device loads the library's kernels there (make it before any stream
 * capture).  All calls on a device share the array: calls that overlap on
 * the GPU race.  Capacity configurations needing a workspace slot above
 * 64 MiB return cudaErrorInvalidValue (configurations stepped whole in shared
 * memory need none); batch size is not limited. */
B3X_API int b3x_batch_step_gpu_noalloc(B3Batch batch, float dt, int substeps, const unsigned char* active,
    void* stream, unsigned long long config_signature, int joint_iters, int relax_iters);

/* Bytes of workspace a step needs on `device` for this capacity configuration
 * to run one launch per wave of resident tiles (independent of the batch
 * size; what b3x_reserve_workspace allocates); 0 if the configuration is
 * invalid. */
B3X_API size_t b3x_workspace_bytes(unsigned long long config_signature, int device);

/* No counterpart in the reference.  Bytes of one tile's slot of the
 * workspace (32 worlds); a workspace of k slots runs up to k tiles per
 * launch.  0 if the configuration is invalid. */
B3X_API size_t b3x_workspace_slot_bytes(unsigned long long config_signature);

/* No counterpart in the reference (whose per-thread step needs no
 * workspace).  Set-up call, the library's only device allocation: reserve
 * b3x_workspace_bytes(...) of device memory for steps of this capacity
 * configuration on `stream` (current device).  Later b3x_batch_step_gpu /
 * b3_batch_step_gpu calls on that stream use it.  A reservation that is
 * large enough is kept; a smaller one is replaced (cudaFree synchronises).
 * Configurations stepped in shared memory need none (returns 0).  Batches
 * stepped concurrently on several streams should each have one. */
B3X_API int b3x_reserve_workspace(void* stream, unsigned long long config_signature);

/* Free every workspace reserved on the current device (synchronises, as
 * cudaFree does).  Later steps on those streams use the library's array. */
B3X_API int b3x_release_workspaces(void);

/* Bytes reserved for `stream` on the current device, 0 if none. */
B3X_API size_t b3x_reserved_bytes(void* stream);

/* No counterpart in the reference.  Number of kernel launches one
 * b3x_batch_step_gpu call of `count` worlds makes on `device` with a
 * reserved workspace (one per chunk of resident tiles; one for configurations small
 * enough to be stepped whole in shared memory, at most 8 bodies, 8 shapes
 * and 8 contacts, which use no workspace); 0 if the configuration is
 * invalid.  For launch accounting by callers and benchmarks. */
B3X_API int b3x_step_launches(unsigned long long config_signature, int count, int device);

/* Replaces b3_batch_restore_gpu (reference b3_batch.cuh:91-99): copy
 * initial[i] (contiguous snapshots of sizeof(B3World) bytes) over world i for
 * every world selected by `reset` (NULL = all).  Never allocates. */
B3X_API int b3x_batch_restore_gpu(B3Batch batch, const void* initial, const unsigned char* reset,
    void* stream, unsigned long long config_signature);

/* Batched actions on device-resident worlds (the reference applies these per
 * world with b3_apply_force / b3_apply_torque / b3_apply_linear_impulse /
 * b3_joint_set_spring inside the adapter's own kernel):
 *   kind 0: force  += values[3*i..]      on body `index` of world i
 *   kind 1: torque += values[3*i..]      on body `index`
 *   kind 2: linear impulse values[3*i..] on body `index` (dynamic bodies only)
 *   kind 3: spring target_angle = clamp(values[i], -pi, pi) of joint `index`
 * `values` is device-accessible; `active` as in b3x_batch_step_gpu. */
#define B3X_ACTION_FORCE 0
#define B3X_ACTION_TORQUE 1
#define B3X_ACTION_LINEAR_IMPULSE 2
#define B3X_ACTION_JOINT_TARGET 3
B3X_API int b3x_batch_apply_gpu(B3Batch batch, int kind, int index, const float* values, int values_per_world,
    const unsigned char* active, void* stream, unsigned long long config_signature);

/* Observation gather: out[13*i ..] = position(3), rotation(4: x y z s),
 * lin_vel(3), ang_vel(3) of body `body` of world i (NaN when the world has
 * fewer bodies).  What an adapter reads after b3_step (reference
 * examples/pufferlib/puffysics_hover/hover_task.h:79-84), batched. */
B3X_API int b3x_batch_observe_gpu(B3Batch batch, int body, float* out, void* stream,
    unsigned long long config_signature);

/* ---------------------------------------------------------------------------
 * Resident world columns.  No counterpart in the reference, whose worlds
 * always stay in the caller's AoS array (src/puffysics/02_types.inl:306-332,
 * stepped in place by b3_batch.cuh:63-68).  Here the worlds of a batch can
 * live in HBM as structure-of-arrays across worlds ("columns"): word w of the
 * B3World of world i at engine[((i / 32) * W + w) * 32 + i % 32] (4-byte
 * words, W = sizeof(B3World) / 4), so one word of 32 consecutive worlds is
 * one 128-byte line.  Steps on the columns read and write only them: no AoS
 * row gathers or scatters.  The memory is the caller's (device, 16-byte
 * aligned, b3x_engine_bytes long); world i of the columns is world i of the
 * batches bound to or synced from them.  Results are the same bytes as
 * b3x_batch_step_gpu on the AoS worlds.
 * ------------------------------------------------------------------------- */

/* Bytes of the columns of `count` worlds (whole tiles of 32); 0 if invalid. */
B3X_API size_t b3x_engine_bytes(unsigned long long config_signature, int count);

/* Copy the selected worlds (NULL = all; nonzero byte = selected) of the AoS
 * batch into the columns; the batch must hold `count` worlds (stride and
 * embedding offset as in b3_batch_step_gpu).  Binding the initial snapshots
 * with a reset mask is the columns' b3_batch_restore_gpu. */
B3X_API int b3x_engine_bind(void* engine, int count, B3Batch worlds, const unsigned char* select,
    void* stream, unsigned long long config_signature);

/* Copy the selected worlds of the columns back into the AoS batch. */
B3X_API int b3x_engine_sync_to_aos(const void* engine, int count, B3Batch worlds, const unsigned char* select,
    void* stream, unsigned long long config_signature);

/* b3x_batch_step_gpu_flags on the columns: same validation, no-op cases,
 * mask, modes, workspace (reservation or the library's array) and results.
 * One more flag: B3X_STEP_STATE_ONLY writes back only the world state later
 * steps read -- bodies, header counts, each contact's warm-start cache (pair,
 * point count, features, impulses) and joint impulses -- and skips the words
 * a step merely outputs (a contact's anchors, masses, tangents, softness; a
 * joint's prepared frames, masses and softness), which keep the bytes of the
 * last step without the flag.  Trajectories are unchanged.  After a step
 * without the flag every word the reference defines is again byte-equal to
 * the AoS path; contact slots past a world's contact count and point slots
 * past a contact's point count (whose bytes the reference leaves over from
 * earlier steps) may then hold bytes of an earlier step than there. */
#define B3X_STEP_STATE_ONLY 4
B3X_API int b3x_engine_step(void* engine, int count, float dt, int substeps, const unsigned char* active,
    void* stream, unsigned long long config_signature, int joint_iters, int relax_iters, int flags);

/* b3x_batch_apply_gpu and b3x_batch_observe_gpu on the columns. */
B3X_API int b3x_engine_apply(void* engine, int count, int kind, int index, const float* values,
    int values_per_world, const unsigned char* active, void* stream, unsigned long long config_signature);
B3X_API int b3x_engine_observe(const void* engine, int count, int body, float* out, void* stream,
    unsigned long long config_signature);

/* Device generators of the benchmark inputs (seeded scenes of
 * puffysics_b200/scenes/b3_scenes.h): per-step action values of world
 * first+i (returns values per world, 0 when the scene has none, -1 on error)
 * and the 1%-per-step reset mask of the scale-out configuration. */
B3X_API int b3x_scene_actions_gpu(float* out, int n, int scene, unsigned long long seed, unsigned long long first,
    unsigned long long step, void* stream);
B3X_API int b3x_scene_reset_gpu(unsigned char* out, int n, unsigned long long seed, unsigned long long first,
    unsigned long long step, void* stream);

/* Nonzero if a step on the current device was abandoned because one of its
 * bounded waits for a bulk copy into shared memory gave up (not expected).
 * The 32 worlds of the tile whose wait gave up are then left as they were
 * before the call (nothing of that tile is written back), except on resident
 * world columns (b3x_engine_step without B3X_STEP_STATE_ONLY), whose contact
 * rows may already hold the step's new contacts with their previous
 * impulses; the other tiles are stepped.  clear != 0 resets it.  Synchronises
 * the device; -1 on error. */
B3X_API int b3x_fault_flags(int clear);

/* Capacity configuration helpers (host). */
B3X_API size_t b3x_world_bytes(unsigned long long config_signature);
B3X_API const char* b3x_version(void);

/* Inline shims with the exact reference signatures (reference
 * b3_batch.cuh:81-99), available wherever the CUDA runtime types are. */
#if (defined(__CUDACC__) || defined(CUDART_VERSION)) && !B3_HAS_USER_FORCES && !B3_ART_CONTACTS
B3_INL cudaError_t b3_batch_step_gpu(B3Batch batch, float dt, int substeps,
        const unsigned char* active, cudaStream_t stream) {
#if defined(B3_INTERLEAVE_CONTACTS) || defined(B3_SKIP_RESTITUTION)
    int flags = 0;
#if defined(B3_INTERLEAVE_CONTACTS)
    flags |= B3X_STEP_INTERLEAVE_CONTACTS;
#endif
#if defined(B3_SKIP_RESTITUTION)
    flags |= B3X_STEP_SKIP_RESTITUTION;
#endif
    return (cudaError_t)b3x_batch_step_gpu_flags(batch, dt, substeps, active, (void*)stream,
        B3_CONFIG_SIGNATURE, B3_JOINT_ITERS, B3_RELAX_ITERS, flags);
#else
    return (cudaError_t)b3x_batch_step_gpu(batch, dt, substeps, active, (void*)stream,
        B3_CONFIG_SIGNATURE, B3_JOINT_ITERS, B3_RELAX_ITERS);
#endif
}
#endif
#if defined(__CUDACC__) || defined(CUDART_VERSION)
B3_INL cudaError_t b3_batch_restore_gpu(B3Batch batch, const B3World* initial,
        const unsigned char* reset, cudaStream_t stream) {
    return (cudaError_t)b3x_batch_restore_gpu(batch, (const void*)initial, reset, (void*)stream,
        B3_CONFIG_SIGNATURE);
}
#endif

#endif /* PUFFYSICS_B200_H */
