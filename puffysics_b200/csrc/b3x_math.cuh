// b3x_math.cuh -- device math beyond the public header's helpers.
//
// Every function keeps the floating-point operation order of the reference
// helper it replaces (file:line cited, paths relative to the reference
// repository root).  The library is compiled with -fmad=false and IEEE
// division / square root, so each expression rounds exactly as the
// reference's CPU build (-ffp-contract=off) does.
#pragma once
#include <cstring>

#include "puffysics_b200.h"

#if defined(__CUDACC__)
#define B3X_HD __host__ __device__
#define B3X_HDI __host__ __device__ __forceinline__
#else
#define B3X_HD
#define B3X_HDI inline
#endif

namespace b3x {

// Step modes of the reference's compile-time switches (01_config.inl:50-52,
// 07_packed.inl:63-65, 09_step.inl:169-181): contacts swept inside every
// joint iteration instead of once per phase (B3_INTERLEAVE_CONTACTS), and no
// restitution pass (B3_SKIP_RESTITUTION).
enum : int { kStepInterleaveContacts = 1, kStepSkipRestitution = 2, kStepStateOnly = 4 };

// Bit casts between 32-bit words (ints and flags share the float columns).
B3X_HDI int b3x_f2i(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_int(f);
#else
    int i; std::memcpy(&i, &f, 4); return i;
#endif
}
B3X_HDI float b3x_i2f(int i) {
#if defined(__CUDA_ARCH__)
    return __int_as_float(i);
#else
    float f; std::memcpy(&f, &i, 4); return f;
#endif
}
B3X_HDI uint32_t b3x_f2u(float f) { return (uint32_t)b3x_f2i(f); }
B3X_HDI float b3x_u2f(uint32_t u) { return b3x_i2f((int)u); }

B3X_HDI B3Mat3 m3_zero() {
    B3Mat3 m;
    m.cx = b3_v(0.0f, 0.0f, 0.0f);
    m.cy = b3_v(0.0f, 0.0f, 0.0f);
    m.cz = b3_v(0.0f, 0.0f, 0.0f);
    return m;
}

B3X_HDI B3Mat3 m3_add(B3Mat3 a, B3Mat3 b) {
    B3Mat3 r;
    r.cx = b3_add(a.cx, b.cx);
    r.cy = b3_add(a.cy, b.cy);
    r.cz = b3_add(a.cz, b.cz);
    return r;
}

// Cofactor inverse; zero matrix when |det| < 1e-12 (03_math.inl:200-215).
B3X_HDI B3Mat3 m3_inv(B3Mat3 m) {
    B3Vec3 c0 = b3_cross(m.cy, m.cz);
    float det = b3_dot(m.cx, c0);
    B3Mat3 r = m3_zero();
    if (fabsf(det) < 1.0e-12f) return r;
    float inv = 1.0f / det;
    B3Vec3 r0 = b3_mul(c0, inv);
    B3Vec3 r1 = b3_mul(b3_cross(m.cz, m.cx), inv);
    B3Vec3 r2 = b3_mul(b3_cross(m.cx, m.cy), inv);
    r.cx = b3_v(r0.x, r1.x, r2.x);
    r.cy = b3_v(r0.y, r1.y, r2.y);
    r.cz = b3_v(r0.z, r1.z, r2.z);
    return r;
}

// 2x2 inverse (03_math.inl:217-231).
B3X_HDI B3Mat2 m2_inv(B3Mat2 k) {
    float det = k.cx.x * k.cy.y - k.cx.y * k.cy.x;
    B3Mat2 r;
    r.cx.x = 0.0f; r.cx.y = 0.0f; r.cy.x = 0.0f; r.cy.y = 0.0f;
    if (fabsf(det) < 1.0e-12f) return r;
    float inv = 1.0f / det;
    r.cx.x = k.cy.y * inv;
    r.cx.y = -k.cx.y * inv;
    r.cy.x = -k.cy.x * inv;
    r.cy.y = k.cx.x * inv;
    return r;
}

B3X_HDI B3Vec2 m2_mv(B3Mat2 m, B3Vec2 v) {
    B3Vec2 r;
    r.x = m.cx.x * v.x + m.cy.x * v.y;
    r.y = m.cx.y * v.x + m.cy.y * v.y;
    return r;
}

// Normalized explicit Euler step of a rotation (03_math.inl:152-157).
B3X_HDI B3Quat q_integrate(B3Quat q, B3Vec3 dw) {
    B3Quat qd = b3_qmul(b3_q(0.5f * dw.x, 0.5f * dw.y, 0.5f * dw.z, 0.0f), q);
    return b3_qnorm(b3_q(q.v.x + qd.v.x, q.v.y + qd.v.y, q.v.z + qd.v.z, q.s + qd.s));
}

// Soft-step spring coefficients (03_math.inl:247-263).
B3X_HDI B3Soft make_soft(float hertz, float zeta, float h) {
    B3Soft s;
    s.bias_rate = 0.0f;
    s.mass_scale = 0.0f;
    s.impulse_scale = 0.0f;
    if (hertz == 0.0f) return s;
    float omega = 2.0f * B3_PI * hertz;
    float a1 = 2.0f * zeta + h * omega;
    float a2 = h * omega * a1;
    float a3 = 1.0f / (1.0f + a2);
    s.bias_rate = omega / a1;
    s.mass_scale = a2 * a3;
    s.impulse_scale = a3;
    return s;
}

// Hinge perpendicular rows (03_math.inl:311-319).
B3X_HDI void hinge_perps(B3Quat qa, B3Quat rel, B3Vec3* px, B3Vec3* py) {
    B3Vec3 ex = b3_v(1.0f, 0.0f, 0.0f);
    B3Vec3 ey = b3_v(0.0f, 1.0f, 0.0f);
    *px = b3_mul(b3_rotate(qa, b3_add(b3_mul(ex, rel.s), b3_cross(rel.v, ex))), 0.5f);
    *py = b3_mul(b3_rotate(qa, b3_add(b3_mul(ey, rel.s), b3_cross(rel.v, ey))), 0.5f);
}

// 2x2 solve with det <= 1e-12 -> 0 (03_math.inl:347-359).
B3X_HDI B3Vec2 solve2(B3Mat2 m, B3Vec2 b) {
    float det = m.cx.x * m.cy.y - m.cx.y * m.cy.x;
    B3Vec2 r;
    r.x = 0.0f;
    r.y = 0.0f;
    if (det <= 1.0e-12f) return r;
    float inv = 1.0f / det;
    r.x = inv * (m.cy.y * b.x - m.cy.x * b.y);
    r.y = inv * (-m.cx.y * b.x + m.cx.x * b.y);
    return r;
}

}  // namespace b3x
