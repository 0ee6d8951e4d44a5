// b3x_narrow.cuh -- per-pair contact manifolds on the device.
//
// Sphere / capsule / box pairs, up to four points, normal pointing from shape
// A to shape B, feature ids as in the reference (sphere 1, capsule-capsule 2,
// sphere-box 3, sphere-capsule 4, capsule-box 5, box edge 6-14, box face
// 16+i / 20+i).  Shapes arrive with their world pose already composed
// (body pose x shape local pose), which the reference recomputes for every
// pair; the values are bit-identical.  Float operation order follows
// reference src/puffysics/05_collision.inl line by line.
#pragma once
#include "puffysics_b200.h"
#include "b3x_math.cuh"

// Linkage of the out-of-line narrowphase functions (external in the library).
#ifndef B3X_NARROW
#define B3X_NARROW B3X_HD
#endif

namespace b3x {

struct Mani {
    int count;
    B3Vec3 normal;
    B3Vec3 pa[B3_MAX_MANIFOLD];
    B3Vec3 pb[B3_MAX_MANIFOLD];
    float sep[B3_MAX_MANIFOLD];
    uint32_t feat[B3_MAX_MANIFOLD];
};

struct Geo {             // world-space shape
    B3Vec3 p;
    B3Quat q;
    int type;
    float radius;
    B3Vec3 half;
};

B3X_HDI void m_clear(Mani& m) {
    m.count = 0;
    m.normal = b3_v(0.0f, 1.0f, 0.0f);
}

// Append a point (dropped when the manifold is full).  The slot is selected
// with constant indices so the manifold stays in registers.
B3X_HDI void m_put(Mani& m, int i, B3Vec3 pa, B3Vec3 pb, float sep, uint32_t f) {
    m.pa[i] = pa;
    m.pb[i] = pb;
    m.sep[i] = sep;
    m.feat[i] = f;
}
B3X_HDI void m_push(Mani& m, B3Vec3 pa, B3Vec3 pb, float sep, uint32_t f) {
    switch (m.count) {
    case 0: m_put(m, 0, pa, pb, sep, f); break;
    case 1: m_put(m, 1, pa, pb, sep, f); break;
    case 2: m_put(m, 2, pa, pb, sep, f); break;
    case 3: m_put(m, 3, pa, pb, sep, f); break;
    default: return;
    }
    m.count++;
}

// Clip polygon scratch: vertex v, component c at base[(3 * v + c) * stride]
// (shared memory, interleaved across the threads of a block).  Two polygons
// of up to 8 vertices each.
struct Poly {
    float* base;
    int stride;
    B3X_HDI B3Vec3 get(int v) const {
        return b3_v(base[(3 * v) * stride], base[(3 * v + 1) * stride], base[(3 * v + 2) * stride]);
    }
    B3X_HDI void put(int v, B3Vec3 p) const {
        base[(3 * v) * stride] = p.x;
        base[(3 * v + 1) * stride] = p.y;
        base[(3 * v + 2) * stride] = p.z;
    }
    B3X_HDI Poly second() const { Poly q; q.base = base + 24 * stride; q.stride = stride; return q; }
};
static_assert(B3_MAX_MANIFOLD == 4, "manifold slots");

B3X_HDI float rsq(float x) { return 1.0f / sqrtf(x); }

// 05_collision.inl:5-13
B3X_NARROW B3Vec3 closest_on_segment(B3Vec3 a, B3Vec3 b, B3Vec3 p) {
    B3Vec3 ab = b3_sub(b, a);
    float d = b3_len2(ab);
    if (d <= 1.0e-12f) return a;
    float t = b3_clamp(b3_dot(b3_sub(p, a), ab) / d, 0.0f, 1.0f);
    return b3_madd(a, t, ab);
}

// 05_collision.inl:15-55
B3X_NARROW void closest_between_segments(B3Vec3 a1, B3Vec3 a2, B3Vec3 b1, B3Vec3 b2, B3Vec3* pa, B3Vec3* pb) {
    B3Vec3 d1 = b3_sub(a2, a1);
    B3Vec3 d2 = b3_sub(b2, b1);
    B3Vec3 r = b3_sub(a1, b1);
    float a = b3_len2(d1);
    float e = b3_len2(d2);
    float f = b3_dot(d2, r);
    float s, t;
    if (a <= 1.0e-12f && e <= 1.0e-12f) {
        *pa = a1;
        *pb = b1;
        return;
    }
    if (a <= 1.0e-12f) {
        s = 0.0f;
        t = b3_clamp(f / e, 0.0f, 1.0f);
    } else {
        float c = b3_dot(d1, r);
        if (e <= 1.0e-12f) {
            t = 0.0f;
            s = b3_clamp(-c / a, 0.0f, 1.0f);
        } else {
            float b = b3_dot(d1, d2);
            float den = a * e - b * b;
            s = den != 0.0f ? b3_clamp((b * f - c * e) / den, 0.0f, 1.0f) : 0.0f;
            t = (b * s + f) / e;
            if (t < 0.0f) {
                t = 0.0f;
                s = b3_clamp(-c / a, 0.0f, 1.0f);
            } else if (t > 1.0f) {
                t = 1.0f;
                s = b3_clamp((b - c) / a, 0.0f, 1.0f);
            }
        }
    }
    *pa = b3_madd(a1, s, d1);
    *pb = b3_madd(b1, t, d2);
}

// 05_collision.inl:83-98
B3X_NARROW void sphere_sphere(Mani& m, B3Vec3 ca, float ra, B3Vec3 cb, float rb, uint32_t f) {
    m_clear(m);
    B3Vec3 d = b3_sub(cb, ca);
    float dist2 = b3_len2(d);
    float rad = ra + rb;
    if (dist2 > rad * rad) return;
    float dist = sqrtf(dist2);
    B3Vec3 n = dist > 1.0e-8f ? b3_mul(d, rsq(dist2)) : b3_v(0.0f, 1.0f, 0.0f);
    m.normal = n;
    m_push(m, b3_madd(ca, ra, n), b3_msub(cb, rb, n), dist - rad, f);
}

// 05_collision.inl:100-129
B3X_NARROW B3Vec3 closest_on_box(B3Vec3 c, B3Quat q, B3Vec3 half, B3Vec3 p, int* inside, int* face) {
    B3Vec3 local = b3_inv_rotate(q, b3_sub(p, c));
    B3Vec3 cl = b3_v(b3_clamp(local.x, -half.x, half.x), b3_clamp(local.y, -half.y, half.y),
        b3_clamp(local.z, -half.z, half.z));
    int in = fabsf(local.x) <= half.x && fabsf(local.y) <= half.y && fabsf(local.z) <= half.z;
    *inside = in;
    if (in) {
        float dx = half.x - fabsf(local.x);
        float dy = half.y - fabsf(local.y);
        float dz = half.z - fabsf(local.z);
        if (dx <= dy && dx <= dz) {
            cl.x = local.x >= 0.0f ? half.x : -half.x;
            *face = 0;
        } else if (dy <= dz) {
            cl.y = local.y >= 0.0f ? half.y : -half.y;
            *face = 1;
        } else {
            cl.z = local.z >= 0.0f ? half.z : -half.z;
            *face = 2;
        }
    } else {
        *face = -1;
    }
    return b3_xf_point(c, q, cl);
}

// 05_collision.inl:131-150
B3X_NARROW void ball_vs_point(Mani& m, B3Vec3 p, float r, B3Vec3 q, int inside, B3Vec3 n_fb, uint32_t f) {
    B3Vec3 d = b3_sub(p, q);
    float dist2 = b3_len2(d);
    if (!inside && dist2 > r * r) return;
    B3Vec3 n;
    float sep;
    if (inside) {
        n = dist2 > 1.0e-12f ? b3_norm(d) : n_fb;
        sep = -b3_len(d) - r;
    } else {
        float dist = sqrtf(dist2);
        n = b3_mul(d, rsq(dist2));
        sep = dist - r;
    }
    m.normal = n;
    m_push(m, b3_msub(p, r, n), q, sep, f);
}

// 05_collision.inl:152-162
B3X_NARROW void sphere_box(Mani& m, B3Vec3 sc, float r, B3Vec3 bc, B3Quat bq, B3Vec3 half) {
    m_clear(m);
    int inside, face;
    B3Vec3 q = closest_on_box(bc, bq, half, sc, &inside, &face);
    B3Vec3 ax, ay, az;
    b3_axes(bq, &ax, &ay, &az);
    B3Vec3 n_fb = face == 0 ? ax : (face == 1 ? ay : az);
    ball_vs_point(m, sc, r, q, inside, n_fb, 3u);
}

// 05_collision.inl:164-175
B3X_NARROW void capsule_box(Mani& m, B3Vec3 c1, B3Vec3 c2, float r, B3Vec3 bc, B3Quat bq, B3Vec3 half) {
    m_clear(m);
    B3Vec3 mid = b3_mul(b3_add(c1, c2), 0.5f);
    int inside, face;
    B3Vec3 q = closest_on_box(bc, bq, half, mid, &inside, &face);
    B3Vec3 p = closest_on_segment(c1, c2, q);
    q = closest_on_box(bc, bq, half, p, &inside, &face);
    p = closest_on_segment(c1, c2, q);
    ball_vs_point(m, p, r, q, inside, b3_v(0.0f, 1.0f, 0.0f), 5u);
}

struct Obb {
    B3Vec3 c;
    B3Vec3 ax[3];
    B3Vec3 h;
};

B3X_HDI float hcomp(B3Vec3 h, int i) { return i == 0 ? h.x : (i == 1 ? h.y : h.z); }
// axis i of a box, selected without dynamic indexing
B3X_HDI B3Vec3 oax(const Obb& o, int i) { return i == 0 ? o.ax[0] : (i == 1 ? o.ax[1] : o.ax[2]); }

// 05_collision.inl:195-201
B3X_HDI B3Vec3 obb_support(const Obb& o, B3Vec3 dir) {
    float sx = b3_dot(o.ax[0], dir) < 0.0f ? -o.h.x : o.h.x;
    float sy = b3_dot(o.ax[1], dir) < 0.0f ? -o.h.y : o.h.y;
    float sz = b3_dot(o.ax[2], dir) < 0.0f ? -o.h.z : o.h.z;
    return b3_add(o.c, b3_add(b3_mul(o.ax[0], sx), b3_add(b3_mul(o.ax[1], sy), b3_mul(o.ax[2], sz))));
}

// 05_collision.inl:253-258
B3X_HDI void support_pair(Mani& m, const Obb& a, const Obb& b, B3Vec3 n, int f) {
    B3Vec3 pa = obb_support(a, n);
    B3Vec3 pb = obb_support(b, b3_neg(n));
    m_push(m, pa, pb, b3_dot(b3_sub(pb, pa), n), (uint32_t)f);
}

// 05_collision.inl:260-271; returns false when the axis separates.
B3X_HDI bool sat_face(float s, B3Vec3 axis, float side, float& best, B3Vec3& n, int f, int& of) {
    if (s > B3_SPECULATIVE) return false;
    if (s > best) {
        best = s;
        n = side < 0.0f ? b3_neg(axis) : axis;
        of = f;
    }
    return true;
}

// 05_collision.inl:273-293; returns false when the axis separates.
B3X_HDI bool sat_edge(float e, float ra, float rb, B3Vec3 cr, float& best, B3Vec3& n, int f,
        int& of) {
    float cl2 = b3_len2(cr);
    if (cl2 <= 1.0e-3f) return true;
    float inv = rsq(cl2);
    float s = (fabsf(e) - ra - rb) * inv;
    if (s > B3_SPECULATIVE && cl2 > 0.05f) return false;
    if (s > B3_SPECULATIVE) return true;
    if (s > best + 0.002f) {
        best = s;
        n = e < 0.0f ? b3_mul(cr, -inv) : b3_mul(cr, inv);
        of = f;
    }
    return true;
}

// Sutherland-Hodgman step against one plane, at most 8 output vertices
// (05_collision.inl:203-228).
B3X_NARROW int clip_against(const Poly& in, int n, const Poly& out, B3Vec3 pn, float po) {
    if (n <= 0) return 0;
    int c = 0;
    B3Vec3 prev = in.get(n - 1);
    float pd = b3_dot(prev, pn) - po;
    int pin = pd <= 0.0f;
    for (int i = 0; i < n; i++) {
        B3Vec3 cur = in.get(i);
        float cd = b3_dot(cur, pn) - po;
        int cin = cd <= 0.0f;
        if (cin != pin && c < 8) {
            float t = pd / (pd - cd);
            out.put(c++, b3_madd(prev, t, b3_sub(cur, prev)));
        }
        if (cin && c < 8) out.put(c++, cur);
        prev = cur;
        pd = cd;
        pin = cin;
    }
    return c;
}

// Separating-axis box-box with reference-face clipping (05_collision.inl:295-461).
B3X_NARROW void box_box(Mani& m, const Obb& a, const Obb& b, const Poly& P) {
    m_clear(m);
    B3Vec3 d = b3_sub(b.c, a.c);
    float t0 = b3_dot(d, a.ax[0]), t1 = b3_dot(d, a.ax[1]), t2 = b3_dot(d, a.ax[2]);
    float r00 = b3_dot(a.ax[0], b.ax[0]), r01 = b3_dot(a.ax[0], b.ax[1]), r02 = b3_dot(a.ax[0], b.ax[2]);
    float r10 = b3_dot(a.ax[1], b.ax[0]), r11 = b3_dot(a.ax[1], b.ax[1]), r12 = b3_dot(a.ax[1], b.ax[2]);
    float r20 = b3_dot(a.ax[2], b.ax[0]), r21 = b3_dot(a.ax[2], b.ax[1]), r22 = b3_dot(a.ax[2], b.ax[2]);
    float q00 = fabsf(r00), q01 = fabsf(r01), q02 = fabsf(r02);
    float q10 = fabsf(r10), q11 = fabsf(r11), q12 = fabsf(r12);
    float q20 = fabsf(r20), q21 = fabsf(r21), q22 = fabsf(r22);
    float ax = a.h.x, ay = a.h.y, az = a.h.z, bx = b.h.x, by = b.h.y, bz = b.h.z;
    float best = -FLT_MAX;
    B3Vec3 n = a.ax[0];
    int f = 0;
    if (!sat_face(fabsf(t0) - ax - (bx * q00 + by * q01 + bz * q02), a.ax[0], t0, best, n, 0, f)) return;
    if (!sat_face(fabsf(t1) - ay - (bx * q10 + by * q11 + bz * q12), a.ax[1], t1, best, n, 1, f)) return;
    if (!sat_face(fabsf(t2) - az - (bx * q20 + by * q21 + bz * q22), a.ax[2], t2, best, n, 2, f)) return;
    float u0 = t0 * r00 + t1 * r10 + t2 * r20;
    float u1 = t0 * r01 + t1 * r11 + t2 * r21;
    float u2 = t0 * r02 + t1 * r12 + t2 * r22;
    if (!sat_face(fabsf(u0) - bx - (ax * q00 + ay * q10 + az * q20), b.ax[0], u0, best, n, 3, f)) return;
    if (!sat_face(fabsf(u1) - by - (ax * q01 + ay * q11 + az * q21), b.ax[1], u1, best, n, 4, f)) return;
    if (!sat_face(fabsf(u2) - bz - (ax * q02 + ay * q12 + az * q22), b.ax[2], u2, best, n, 5, f)) return;
    if (!sat_edge(t2 * r10 - t1 * r20, ay * q20 + az * q10, by * q02 + bz * q01, b3_cross(a.ax[0], b.ax[0]),
            best, n, 6, f)) return;
    if (!sat_edge(t2 * r11 - t1 * r21, ay * q21 + az * q11, bz * q00 + bx * q02, b3_cross(a.ax[0], b.ax[1]),
            best, n, 7, f)) return;
    if (!sat_edge(t2 * r12 - t1 * r22, ay * q22 + az * q12, bx * q01 + by * q00, b3_cross(a.ax[0], b.ax[2]),
            best, n, 8, f)) return;
    if (!sat_edge(t0 * r20 - t2 * r00, az * q00 + ax * q20, by * q12 + bz * q11, b3_cross(a.ax[1], b.ax[0]),
            best, n, 9, f)) return;
    if (!sat_edge(t0 * r21 - t2 * r01, az * q01 + ax * q21, bz * q10 + bx * q12, b3_cross(a.ax[1], b.ax[1]),
            best, n, 10, f)) return;
    if (!sat_edge(t0 * r22 - t2 * r02, az * q02 + ax * q22, bx * q11 + by * q10, b3_cross(a.ax[1], b.ax[2]),
            best, n, 11, f)) return;
    if (!sat_edge(t1 * r00 - t0 * r10, ax * q10 + ay * q00, by * q22 + bz * q21, b3_cross(a.ax[2], b.ax[0]),
            best, n, 12, f)) return;
    if (!sat_edge(t1 * r01 - t0 * r11, ax * q11 + ay * q01, bz * q20 + bx * q22, b3_cross(a.ax[2], b.ax[1]),
            best, n, 13, f)) return;
    if (!sat_edge(t1 * r02 - t0 * r12, ax * q12 + ay * q02, bx * q21 + by * q20, b3_cross(a.ax[2], b.ax[2]),
            best, n, 14, f)) return;

    if (b3_dot(n, d) < 0.0f) n = b3_neg(n);
    m.normal = n;
    if (f >= 6) {
        support_pair(m, a, b, n, f);
        return;
    }
    const Obb ref = f < 3 ? a : b;
    const Obb inc = f < 3 ? b : a;
    int rax = f < 3 ? f : f - 3;
    float rd = b3_dot(oax(ref, rax), n);
    float rsign = (f < 3 ? rd < 0.0f : rd > 0.0f) ? -1.0f : 1.0f;
    B3Vec3 rn = b3_mul(oax(ref, rax), rsign);
    // incident face: the face of inc most anti-parallel to rn (05_collision.inl:243-251, 422-426)
    float b0 = fabsf(b3_dot(inc.ax[0], rn)), b1 = fabsf(b3_dot(inc.ax[1], rn)), b2 = fabsf(b3_dot(inc.ax[2], rn));
    int iax = (b0 >= b1 && b0 >= b2) ? 0 : (b1 >= b2 ? 1 : 2);
    float isign = b3_dot(oax(inc, iax), rn) > 0.0f ? -1.0f : 1.0f;
    // the polygon alternates between the two scratch buffers
    Poly cur = P, nxt = P.second();
    {
        int ta = (iax + 1) % 3, tb = (iax + 2) % 3;
        B3Vec3 c = b3_madd(inc.c, isign * hcomp(inc.h, iax), oax(inc, iax));
        B3Vec3 ea = b3_mul(oax(inc, ta), hcomp(inc.h, ta));
        B3Vec3 eb = b3_mul(oax(inc, tb), hcomp(inc.h, tb));
        cur.put(0, b3_sub(b3_sub(c, ea), eb));
        cur.put(1, b3_add(b3_sub(c, ea), eb));
        cur.put(2, b3_add(b3_add(c, ea), eb));
        cur.put(3, b3_sub(b3_add(c, ea), eb));
    }
    int count = 4;
    int ta = (rax + 1) % 3, tb = (rax + 2) % 3;
    B3Vec3 face_c = b3_madd(ref.c, rsign * hcomp(ref.h, rax), oax(ref, rax));
    for (int i = 0; i < 4; i++) {
        int t = i < 2 ? ta : tb;
        float s = (i & 1) ? 1.0f : -1.0f;
        B3Vec3 cn = b3_mul(oax(ref, t), s);
        float co = b3_dot(cn, ref.c) + hcomp(ref.h, t);
        count = clip_against(cur, count, nxt, cn, co);
        Poly sw = cur;
        cur = nxt;
        nxt = sw;
        if (count == 0) {
            support_pair(m, a, b, n, f);
            return;
        }
    }
    float ro = b3_dot(rn, face_c);
    for (int i = 0; i < count && m.count < B3_MAX_MANIFOLD; i++) {
        B3Vec3 pi = cur.get(i);
        float ps = b3_dot(pi, rn) - ro;
        if (ps <= B3_SPECULATIVE) {
            B3Vec3 on_ref = b3_msub(pi, ps, rn);
            B3Vec3 pa = f < 3 ? on_ref : pi;
            B3Vec3 pb = f < 3 ? pi : on_ref;
            m_push(m, pa, pb, b3_dot(b3_sub(pb, pa), n), (f < 3 ? 16u : 20u) + (uint32_t)i);
        }
    }
    if (m.count == 0) support_pair(m, a, b, n, f);
}

B3X_HDI void m_flip(Mani& m) {
    m.normal = b3_neg(m.normal);
#pragma unroll
    for (int i = 0; i < B3_MAX_MANIFOLD; i++) {
        if (i < m.count) {
            B3Vec3 t = m.pa[i];
            m.pa[i] = m.pb[i];
            m.pb[i] = t;
        }
    }
}

// Pair dispatch by type with the A->B normal convention (05_collision.inl:472-534).
B3X_NARROW void collide(Mani& m, Geo a, Geo b, const Poly& P) {
    B3Vec3 center_a = a.p, center_b = b.p;
    bool flip = false;
    if (a.type > b.type) {
        Geo t = a;
        a = b;
        b = t;
        flip = true;
    }
    if (a.type == B3_SPHERE && b.type == B3_SPHERE) {
        sphere_sphere(m, a.p, a.radius, b.p, b.radius, 1u);
    } else if (a.type == B3_SPHERE && b.type == B3_CAPSULE) {
        B3Vec3 y = b3_rotate(b.q, b3_v(0.0f, b.half.y, 0.0f));
        sphere_sphere(m, closest_on_segment(b3_sub(b.p, y), b3_add(b.p, y), a.p), b.radius, a.p, a.radius, 4u);
        m_flip(m);
    } else if (a.type == B3_SPHERE && b.type == B3_BOX) {
        sphere_box(m, a.p, a.radius, b.p, b.q, b.half);
    } else if (a.type == B3_CAPSULE && b.type == B3_CAPSULE) {
        B3Vec3 ya = b3_rotate(a.q, b3_v(0.0f, a.half.y, 0.0f));
        B3Vec3 yb = b3_rotate(b.q, b3_v(0.0f, b.half.y, 0.0f));
        B3Vec3 ca, cb;
        closest_between_segments(b3_sub(a.p, ya), b3_add(a.p, ya), b3_sub(b.p, yb), b3_add(b.p, yb), &ca, &cb);
        sphere_sphere(m, ca, a.radius, cb, b.radius, 2u);
    } else if (a.type == B3_CAPSULE && b.type == B3_BOX) {
        B3Vec3 y = b3_rotate(a.q, b3_v(0.0f, a.half.y, 0.0f));
        capsule_box(m, b3_sub(a.p, y), b3_add(a.p, y), a.radius, b.p, b.q, b.half);
    } else {
        Obb oa, ob;
        oa.c = a.p;
        oa.h = a.half;
        b3_axes(a.q, &oa.ax[0], &oa.ax[1], &oa.ax[2]);
        ob.c = b.p;
        ob.h = b.half;
        b3_axes(b.q, &ob.ax[0], &ob.ax[1], &ob.ax[2]);
        box_box(m, oa, ob, P);
    }
    if (flip && m.count > 0) m_flip(m);
    if (m.count > 0) {
        if (b3_dot(m.normal, b3_sub(center_b, center_a)) < 0.0f) m.normal = b3_neg(m.normal);
#pragma unroll
        for (int i = 0; i < B3_MAX_MANIFOLD; i++)
            if (i < m.count) m.sep[i] = b3_dot(b3_sub(m.pb[i], m.pa[i]), m.normal);
    }
}

}  // namespace b3x
