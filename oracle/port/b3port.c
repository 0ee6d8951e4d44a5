/*
 * b3port.c -- CPU restatement of the Puffysics default stepping path
 * (b3_step with B3_ART_CONTACTS=0 and no experimental flags).
 *
 * TEST INFRASTRUCTURE, NOT PRODUCT CODE.  This file is the parity oracle
 * ("port"): tests and the benchmark's CPU-baseline leg call it to check and
 * time the CUDA engine.  Nothing in puffysics_b200/ links or includes it.
 *
 * Every function restates one reference function (file:line cited; paths
 * are relative to the reference repository root) with the same floating
 * point operation order, so that with -ffp-contract=off it reproduces the
 * reference bit for bit.  It operates in place on the AoS B3World of
 * include/puffysics_b200.h, compiled with the capacity macros of the build.
 * Solver iteration counts are run-time arguments here (compile-time
 * B3_JOINT_ITERS / B3_RELAX_ITERS in the reference, 01_config.inl:96-104).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "puffysics_b200.h"
#include "b3port.h"

typedef B3Vec3 V;
typedef B3Quat Q;
typedef B3Mat3 M;

/* ------------------------------------------------------------ math ---- */
/* reference src/puffysics/03_math.inl:5-369 */
static inline V pv(float x, float y, float z) { V r; r.x = x; r.y = y; r.z = z; return r; }
static inline V padd(V a, V b) { return pv(a.x + b.x, a.y + b.y, a.z + b.z); }
static inline V psub(V a, V b) { return pv(a.x - b.x, a.y - b.y, a.z - b.z); }
static inline V pneg(V a) { return pv(-a.x, -a.y, -a.z); }
static inline V pscale(V a, float s) { return pv(a.x * s, a.y * s, a.z * s); }
static inline V pmadd(V a, float s, V b) { return pv(a.x + s * b.x, a.y + s * b.y, a.z + s * b.z); }
static inline V pmsub(V a, float s, V b) { return pv(a.x - s * b.x, a.y - s * b.y, a.z - s * b.z); }
static inline float pdot(V a, V b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
static inline V pcross(V a, V b) { return pv(a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x); }
static inline float plen2(V a) { return pdot(a, a); }
static inline float plen(V a) { return sqrtf(plen2(a)); }
static inline float prsqrt(float x) { return 1.0f / sqrtf(x); }
static inline V pnorm(V a) { float l2 = plen2(a); return l2 > 0.0f ? pscale(a, prsqrt(l2)) : pv(0.0f, 1.0f, 0.0f); }
static inline float pclamp(float x, float lo, float hi) { return x < lo ? lo : (x > hi ? hi : x); }
static inline float pmax(float a, float b) { return a > b ? a : b; }
static inline float pmin(float a, float b) { return a < b ? a : b; }
static inline Q pq(float x, float y, float z, float s) { Q q; q.v = pv(x, y, z); q.s = s; return q; }
static inline Q pqid(void) { return pq(0.0f, 0.0f, 0.0f, 1.0f); }
static inline float pqdot(Q a, Q b) { return pdot(a.v, b.v) + a.s * b.s; }
static inline Q pqnorm(Q q) {
    float d2 = pqdot(q, q);
    if (d2 <= 0.0f) return pqid();
    float inv = prsqrt(d2);
    return pq(q.v.x * inv, q.v.y * inv, q.v.z * inv, q.s * inv);
}
static inline Q pqmul(Q a, Q b) {
    Q r;
    r.v = padd(padd(pscale(b.v, a.s), pscale(a.v, b.s)), pcross(a.v, b.v));
    r.s = a.s * b.s - pdot(a.v, b.v);
    return r;
}
static inline V prot(Q q, V v) {
    V t = pscale(pcross(q.v, v), 2.0f);
    return padd(v, padd(pscale(t, q.s), pcross(q.v, t)));
}
static inline V pinvrot(Q q, V v) { return prot(pq(-q.v.x, -q.v.y, -q.v.z, q.s), v); }
/* normalized explicit Euler (03_math.inl:132-158, B3_POLY_ROTATION == 0) */
static inline Q pqint(Q q, V dw) {
    Q qd = pq(0.5f * dw.x, 0.5f * dw.y, 0.5f * dw.z, 0.0f);
    qd = pqmul(qd, q);
    return pqnorm(pq(q.v.x + qd.v.x, q.v.y + qd.v.y, q.v.z + qd.v.z, q.s + qd.s));
}
static inline void paxes(Q q, V* x, V* y, V* z) {
    *x = prot(q, pv(1.0f, 0.0f, 0.0f));
    *y = prot(q, pv(0.0f, 1.0f, 0.0f));
    *z = prot(q, pv(0.0f, 0.0f, 1.0f));
}
static inline V pmv(M m, V v) { return padd(padd(pscale(m.cx, v.x), pscale(m.cy, v.y)), pscale(m.cz, v.z)); }
static inline M pmaddm(M a, M b) { M r; r.cx = padd(a.cx, b.cx); r.cy = padd(a.cy, b.cy); r.cz = padd(a.cz, b.cz); return r; }
static inline M pmat0(void) { M m; m.cx = pv(0, 0, 0); m.cy = pv(0, 0, 0); m.cz = pv(0, 0, 0); return m; }
static inline M pwinvi(Q q, V inv) {                      /* 03_math.inl:187-198 */
    V ax, ay, az;
    paxes(q, &ax, &ay, &az);
    M r;
    r.cx = padd(padd(pscale(ax, inv.x * ax.x), pscale(ay, inv.y * ay.x)), pscale(az, inv.z * az.x));
    r.cy = padd(padd(pscale(ax, inv.x * ax.y), pscale(ay, inv.y * ay.y)), pscale(az, inv.z * az.y));
    r.cz = padd(padd(pscale(ax, inv.x * ax.z), pscale(ay, inv.y * ay.z)), pscale(az, inv.z * az.z));
    return r;
}
static inline M pinv3(M m) {                              /* 03_math.inl:200-215 */
    V c0 = pcross(m.cy, m.cz);
    float det = pdot(m.cx, c0);
    M r = pmat0();
    if (fabsf(det) < 1.0e-12f) return r;
    float inv = 1.0f / det;
    V r0 = pscale(c0, inv);
    V r1 = pscale(pcross(m.cz, m.cx), inv);
    V r2 = pscale(pcross(m.cx, m.cy), inv);
    r.cx = pv(r0.x, r1.x, r2.x);
    r.cy = pv(r0.y, r1.y, r2.y);
    r.cz = pv(r0.z, r1.z, r2.z);
    return r;
}
static inline B3Mat2 pinv2(B3Mat2 k) {                    /* 03_math.inl:217-231 */
    float det = k.cx.x * k.cy.y - k.cx.y * k.cy.x;
    B3Mat2 r;
    r.cx.x = r.cx.y = r.cy.x = r.cy.y = 0.0f;
    if (fabsf(det) < 1.0e-12f) return r;
    float inv = 1.0f / det;
    r.cx.x = k.cy.y * inv;
    r.cx.y = -k.cx.y * inv;
    r.cy.x = -k.cy.x * inv;
    r.cy.y = k.cx.x * inv;
    return r;
}
static inline B3Vec2 pmv2(B3Mat2 m, B3Vec2 v) {
    B3Vec2 r;
    r.x = m.cx.x * v.x + m.cy.x * v.y;
    r.y = m.cx.y * v.x + m.cy.y * v.y;
    return r;
}
static inline V pperp(V n) {                              /* 03_math.inl:240-245 */
    if (fabsf(n.x) >= 0.57735027f) return pnorm(pv(-n.y, n.x, 0.0f));
    return pnorm(pv(0.0f, -n.z, n.y));
}
static inline B3Soft psoft(float hertz, float zeta, float h) {   /* 03_math.inl:247-263 */
    B3Soft s;
    s.bias_rate = 0.0f; s.mass_scale = 0.0f; s.impulse_scale = 0.0f;
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
static inline Q pqneg(Q q) { return pq(-q.v.x, -q.v.y, -q.v.z, -q.s); }
static inline Q pqconj(Q q) { return pq(-q.v.x, -q.v.y, -q.v.z, q.s); }
static inline Q pqinvmul(Q a, Q b) {                      /* 03_math.inl:273-278 */
    V t1 = pcross(b.v, a.v);
    V t2 = pmadd(t1, a.s, b.v);
    V t3 = pmsub(t2, b.s, a.v);
    return pq(t3.x, t3.y, t3.z, a.s * b.s + pdot(a.v, b.v));
}
static inline float ptwist(Q q) {                         /* 03_math.inl:293-309 */
    float t = q.s < 0.0f ? atan2f(-q.v.z, -q.s) : atan2f(q.v.z, q.s);
    return 2.0f * t;
}
static inline void phperps(Q qa, Q rel, V* px, V* py) {   /* 03_math.inl:311-319 */
    V ex = pv(1.0f, 0.0f, 0.0f), ey = pv(0.0f, 1.0f, 0.0f);
    *px = pscale(prot(qa, padd(pscale(ex, rel.s), pcross(rel.v, ex))), 0.5f);
    *py = pscale(prot(qa, padd(pscale(ey, rel.s), pcross(rel.v, ey))), 0.5f);
}
static inline B3Vec2 psolve2(B3Mat2 m, B3Vec2 b) {        /* 03_math.inl:347-359 */
    float det = m.cx.x * m.cy.y - m.cx.y * m.cy.x;
    B3Vec2 r; r.x = 0.0f; r.y = 0.0f;
    if (det <= 1.0e-12f) return r;
    float inv = 1.0f / det;
    r.x = inv * (m.cy.y * b.x - m.cy.x * b.y);
    r.y = inv * (-m.cx.y * b.x + m.cx.x * b.y);
    return r;
}
static inline V pxf(V p, Q q, V local) { return padd(p, prot(q, local)); }

/* ------------------------------------------------------- narrowphase -- */
typedef struct PMani {
    int count;
    V normal;
    V pa[B3_MAX_MANIFOLD];
    V pb[B3_MAX_MANIFOLD];
    float sep[B3_MAX_MANIFOLD];
    uint32_t feat[B3_MAX_MANIFOLD];
} PMani;

static inline void mclear(PMani* m) { m->count = 0; m->normal = pv(0.0f, 1.0f, 0.0f); }
static inline void mpush(PMani* m, V pa, V pb, float sep, uint32_t f) {
    if (m->count >= B3_MAX_MANIFOLD) return;
    int i = m->count++;
    m->pa[i] = pa; m->pb[i] = pb; m->sep[i] = sep; m->feat[i] = f;
}

static V seg_closest(V a, V b, V p) {                     /* 05_collision.inl:5-13 */
    V ab = psub(b, a);
    float d = plen2(ab);
    if (d <= 1.0e-12f) return a;
    float t = pclamp(pdot(psub(p, a), ab) / d, 0.0f, 1.0f);
    return pmadd(a, t, ab);
}

static void segs_closest(V a1, V a2, V b1, V b2, V* pa, V* pb) {   /* 05_collision.inl:15-55 */
    V d1 = psub(a2, a1), d2 = psub(b2, b1), r = psub(a1, b1);
    float a = plen2(d1), e = plen2(d2), f = pdot(d2, r);
    float s, t;
    if (a <= 1.0e-12f && e <= 1.0e-12f) { *pa = a1; *pb = b1; return; }
    if (a <= 1.0e-12f) {
        s = 0.0f;
        t = pclamp(f / e, 0.0f, 1.0f);
    } else {
        float c = pdot(d1, r);
        if (e <= 1.0e-12f) {
            t = 0.0f;
            s = pclamp(-c / a, 0.0f, 1.0f);
        } else {
            float b = pdot(d1, d2);
            float den = a * e - b * b;
            s = den != 0.0f ? pclamp((b * f - c * e) / den, 0.0f, 1.0f) : 0.0f;
            t = (b * s + f) / e;
            if (t < 0.0f) {
                t = 0.0f;
                s = pclamp(-c / a, 0.0f, 1.0f);
            } else if (t > 1.0f) {
                t = 1.0f;
                s = pclamp((b - c) / a, 0.0f, 1.0f);
            }
        }
    }
    *pa = pmadd(a1, s, d1);
    *pb = pmadd(b1, t, d2);
}

static void balls(PMani* m, V ca, float ra, V cb, float rb, uint32_t f) {   /* 05_collision.inl:83-98 */
    mclear(m);
    V d = psub(cb, ca);
    float dist2 = plen2(d);
    float rad = ra + rb;
    if (dist2 > rad * rad) return;
    float dist = sqrtf(dist2);
    V n = dist > 1.0e-8f ? pscale(d, prsqrt(dist2)) : pv(0.0f, 1.0f, 0.0f);
    m->normal = n;
    mpush(m, pmadd(ca, ra, n), pmsub(cb, rb, n), dist - rad, f);
}

static V obb_closest(V c, Q q, V half, V p, int* inside, int* face) {    /* 05_collision.inl:100-129 */
    V local = pinvrot(q, psub(p, c));
    V cl = pv(pclamp(local.x, -half.x, half.x), pclamp(local.y, -half.y, half.y),
        pclamp(local.z, -half.z, half.z));
    int in = fabsf(local.x) <= half.x && fabsf(local.y) <= half.y && fabsf(local.z) <= half.z;
    *inside = in;
    if (in) {
        float dx = half.x - fabsf(local.x), dy = half.y - fabsf(local.y), dz = half.z - fabsf(local.z);
        if (dx <= dy && dx <= dz) { cl.x = local.x >= 0.0f ? half.x : -half.x; *face = 0; }
        else if (dy <= dz) { cl.y = local.y >= 0.0f ? half.y : -half.y; *face = 1; }
        else { cl.z = local.z >= 0.0f ? half.z : -half.z; *face = 2; }
    } else {
        *face = -1;
    }
    return pxf(c, q, cl);
}

static void ball_point(PMani* m, V p, float r, V q, int inside, V nfb, uint32_t f) {  /* 05_collision.inl:131-150 */
    V d = psub(p, q);
    float dist2 = plen2(d);
    if (!inside && dist2 > r * r) return;
    V n;
    float sep;
    if (inside) {
        n = dist2 > 1.0e-12f ? pnorm(d) : nfb;
        sep = -plen(d) - r;
    } else {
        float dist = sqrtf(dist2);
        n = pscale(d, prsqrt(dist2));
        sep = dist - r;
    }
    m->normal = n;
    mpush(m, pmsub(p, r, n), q, sep, f);
}

static void sphere_box(PMani* m, V sc, float r, V bc, Q bq, V half) {   /* 05_collision.inl:152-162 */
    mclear(m);
    int inside, face;
    V q = obb_closest(bc, bq, half, sc, &inside, &face);
    V ax, ay, az;
    paxes(bq, &ax, &ay, &az);
    V nfb = face == 0 ? ax : (face == 1 ? ay : az);
    ball_point(m, sc, r, q, inside, nfb, 3u);
}

static void capsule_box(PMani* m, V c1, V c2, float r, V bc, Q bq, V half) {   /* 05_collision.inl:164-175 */
    mclear(m);
    V mid = pscale(padd(c1, c2), 0.5f);
    int inside, face;
    V q = obb_closest(bc, bq, half, mid, &inside, &face);
    V p = seg_closest(c1, c2, q);
    q = obb_closest(bc, bq, half, p, &inside, &face);
    p = seg_closest(c1, c2, q);
    ball_point(m, p, r, q, inside, pv(0.0f, 1.0f, 0.0f), 5u);
}

typedef struct PObb { V c; V ax[3]; V h; } PObb;

static inline float hcomp(V h, int i) { return i == 0 ? h.x : (i == 1 ? h.y : h.z); }

static V obb_support(const PObb* o, V dir) {              /* 05_collision.inl:195-201 */
    float sx = pdot(o->ax[0], dir) < 0.0f ? -o->h.x : o->h.x;
    float sy = pdot(o->ax[1], dir) < 0.0f ? -o->h.y : o->h.y;
    float sz = pdot(o->ax[2], dir) < 0.0f ? -o->h.z : o->h.z;
    return padd(o->c, padd(pscale(o->ax[0], sx), padd(pscale(o->ax[1], sy), pscale(o->ax[2], sz))));
}

static int clip_poly(const V* in, int n, V* out, V pn, float po) {   /* 05_collision.inl:203-228 */
    if (n <= 0) return 0;
    int c = 0;
    V prev = in[n - 1];
    float pd = pdot(prev, pn) - po;
    int pin = pd <= 0.0f;
    for (int i = 0; i < n; i++) {
        V cur = in[i];
        float cd = pdot(cur, pn) - po;
        int cin = cd <= 0.0f;
        if (cin != pin && c < 8) {
            float t = pd / (pd - cd);
            out[c++] = pmadd(prev, t, psub(cur, prev));
        }
        if (cin && c < 8) out[c++] = cur;
        prev = cur; pd = cd; pin = cin;
    }
    return c;
}

static void face_quad(const PObb* o, int axis, float sign, V out[4]) {   /* 05_collision.inl:230-241 */
    int ta = (axis + 1) % 3, tb = (axis + 2) % 3;
    V c = pmadd(o->c, sign * hcomp(o->h, axis), o->ax[axis]);
    V a = pscale(o->ax[ta], hcomp(o->h, ta));
    V b = pscale(o->ax[tb], hcomp(o->h, tb));
    out[0] = psub(psub(c, a), b);
    out[1] = padd(psub(c, a), b);
    out[2] = padd(padd(c, a), b);
    out[3] = psub(padd(c, a), b);
}

static int most_aligned(const PObb* o, V n) {             /* 05_collision.inl:243-251 */
    float b0 = fabsf(pdot(o->ax[0], n)), b1 = fabsf(pdot(o->ax[1], n)), b2 = fabsf(pdot(o->ax[2], n));
    if (b0 >= b1 && b0 >= b2) return 0;
    return b1 >= b2 ? 1 : 2;
}

static void support_point(PMani* m, const PObb* a, const PObb* b, V n, int f) {   /* 05_collision.inl:253-258 */
    V pa = obb_support(a, n);
    V pb = obb_support(b, pneg(n));
    mpush(m, pa, pb, pdot(psub(pb, pa), n), (uint32_t)f);
}

static int sat_face(float s, V axis, float side, float* best, V* n, int f, int* of) {   /* 05_collision.inl:260-271 */
    if (s > B3_SPECULATIVE) return -1;
    if (s > *best) { *best = s; *n = side < 0.0f ? pneg(axis) : axis; *of = f; }
    return 0;
}

static int sat_edge(float e, float ra, float rb, V cr, float* best, V* n, int f, int* of) {   /* 05_collision.inl:273-293 */
    float cl2 = plen2(cr);
    if (cl2 <= 1.0e-3f) return 0;
    float inv = prsqrt(cl2);
    float s = (fabsf(e) - ra - rb) * inv;
    if (s > B3_SPECULATIVE && cl2 > 0.05f) return -1;
    if (s > B3_SPECULATIVE) return 0;
    if (s > *best + 0.002f) { *best = s; *n = e < 0.0f ? pscale(cr, -inv) : pscale(cr, inv); *of = f; }
    return 0;
}

static void box_box(PMani* m, const PObb* a, const PObb* b) {   /* 05_collision.inl:295-461 */
    mclear(m);
    V d = psub(b->c, a->c);
    float t0 = pdot(d, a->ax[0]), t1 = pdot(d, a->ax[1]), t2 = pdot(d, a->ax[2]);
    float R[3][3], A[3][3];
    for (int i = 0; i < 3; i++)
        for (int k = 0; k < 3; k++) { R[i][k] = pdot(a->ax[i], b->ax[k]); A[i][k] = fabsf(R[i][k]); }
    float ax = a->h.x, ay = a->h.y, az = a->h.z, bx = b->h.x, by = b->h.y, bz = b->h.z;
    float best = -FLT_MAX;
    V n = a->ax[0];
    int f = 0;
    if (sat_face(fabsf(t0) - ax - (bx * A[0][0] + by * A[0][1] + bz * A[0][2]), a->ax[0], t0, &best, &n, 0, &f) < 0) return;
    if (sat_face(fabsf(t1) - ay - (bx * A[1][0] + by * A[1][1] + bz * A[1][2]), a->ax[1], t1, &best, &n, 1, &f) < 0) return;
    if (sat_face(fabsf(t2) - az - (bx * A[2][0] + by * A[2][1] + bz * A[2][2]), a->ax[2], t2, &best, &n, 2, &f) < 0) return;
    float u0 = t0 * R[0][0] + t1 * R[1][0] + t2 * R[2][0];
    float u1 = t0 * R[0][1] + t1 * R[1][1] + t2 * R[2][1];
    float u2 = t0 * R[0][2] + t1 * R[1][2] + t2 * R[2][2];
    if (sat_face(fabsf(u0) - bx - (ax * A[0][0] + ay * A[1][0] + az * A[2][0]), b->ax[0], u0, &best, &n, 3, &f) < 0) return;
    if (sat_face(fabsf(u1) - by - (ax * A[0][1] + ay * A[1][1] + az * A[2][1]), b->ax[1], u1, &best, &n, 4, &f) < 0) return;
    if (sat_face(fabsf(u2) - bz - (ax * A[0][2] + ay * A[1][2] + az * A[2][2]), b->ax[2], u2, &best, &n, 5, &f) < 0) return;
    if (sat_edge(t2 * R[1][0] - t1 * R[2][0], ay * A[2][0] + az * A[1][0], by * A[0][2] + bz * A[0][1],
            pcross(a->ax[0], b->ax[0]), &best, &n, 6, &f) < 0) return;
    if (sat_edge(t2 * R[1][1] - t1 * R[2][1], ay * A[2][1] + az * A[1][1], bz * A[0][0] + bx * A[0][2],
            pcross(a->ax[0], b->ax[1]), &best, &n, 7, &f) < 0) return;
    if (sat_edge(t2 * R[1][2] - t1 * R[2][2], ay * A[2][2] + az * A[1][2], bx * A[0][1] + by * A[0][0],
            pcross(a->ax[0], b->ax[2]), &best, &n, 8, &f) < 0) return;
    if (sat_edge(t0 * R[2][0] - t2 * R[0][0], az * A[0][0] + ax * A[2][0], by * A[1][2] + bz * A[1][1],
            pcross(a->ax[1], b->ax[0]), &best, &n, 9, &f) < 0) return;
    if (sat_edge(t0 * R[2][1] - t2 * R[0][1], az * A[0][1] + ax * A[2][1], bz * A[1][0] + bx * A[1][2],
            pcross(a->ax[1], b->ax[1]), &best, &n, 10, &f) < 0) return;
    if (sat_edge(t0 * R[2][2] - t2 * R[0][2], az * A[0][2] + ax * A[2][2], bx * A[1][1] + by * A[1][0],
            pcross(a->ax[1], b->ax[2]), &best, &n, 11, &f) < 0) return;
    if (sat_edge(t1 * R[0][0] - t0 * R[1][0], ax * A[1][0] + ay * A[0][0], by * A[2][2] + bz * A[2][1],
            pcross(a->ax[2], b->ax[0]), &best, &n, 12, &f) < 0) return;
    if (sat_edge(t1 * R[0][1] - t0 * R[1][1], ax * A[1][1] + ay * A[0][1], bz * A[2][0] + bx * A[2][2],
            pcross(a->ax[2], b->ax[1]), &best, &n, 13, &f) < 0) return;
    if (sat_edge(t1 * R[0][2] - t0 * R[1][2], ax * A[1][2] + ay * A[0][2], bx * A[2][1] + by * A[2][0],
            pcross(a->ax[2], b->ax[2]), &best, &n, 14, &f) < 0) return;

    if (pdot(n, d) < 0.0f) n = pneg(n);
    m->normal = n;
    if (f >= 6) { support_point(m, a, b, n, f); return; }

    const PObb* ref = f < 3 ? a : b;
    const PObb* inc = f < 3 ? b : a;
    int rax = f < 3 ? f : f - 3;
    float rd = pdot(ref->ax[rax], n);
    float rsign = (f < 3 ? rd < 0.0f : rd > 0.0f) ? -1.0f : 1.0f;
    V rn = pscale(ref->ax[rax], rsign);
    int iax = most_aligned(inc, rn);
    float isign = pdot(inc->ax[iax], rn) > 0.0f ? -1.0f : 1.0f;
    V poly[8], tmp[8];
    face_quad(inc, iax, isign, poly);
    int count = 4;
    int ta = (rax + 1) % 3, tb = (rax + 2) % 3;
    V face_c = pmadd(ref->c, rsign * hcomp(ref->h, rax), ref->ax[rax]);
    for (int i = 0; i < 4; i++) {
        int t = i < 2 ? ta : tb;
        float s = (i & 1) ? 1.0f : -1.0f;
        V cn = pscale(ref->ax[t], s);
        float co = pdot(cn, ref->c) + hcomp(ref->h, t);
        count = clip_poly(poly, count, tmp, cn, co);
        for (int k = 0; k < count; k++) poly[k] = tmp[k];
        if (count == 0) { support_point(m, a, b, n, f); return; }
    }
    float ro = pdot(rn, face_c);
    for (int i = 0; i < count && m->count < B3_MAX_MANIFOLD; i++) {
        float ps = pdot(poly[i], rn) - ro;
        if (ps <= B3_SPECULATIVE) {
            V on_ref = pmsub(poly[i], ps, rn);
            V pa = f < 3 ? on_ref : poly[i];
            V pb = f < 3 ? poly[i] : on_ref;
            mpush(m, pa, pb, pdot(psub(pb, pa), n), (f < 3 ? 16u : 20u) + (uint32_t)i);
        }
    }
    if (m->count == 0) support_point(m, a, b, n, f);
}

static void mflip(PMani* m) {
    m->normal = pneg(m->normal);
    for (int i = 0; i < m->count; i++) { V t = m->pa[i]; m->pa[i] = m->pb[i]; m->pb[i] = t; }
}

/* Pair dispatch with A->B normal orientation (05_collision.inl:472-534). */
static void collide(PMani* m, const B3Body* ba, const B3Shape* sa, const B3Body* bb, const B3Shape* sb) {
    V pa = pxf(ba->position, ba->rotation, sa->local_pos);
    V pb = pxf(bb->position, bb->rotation, sb->local_pos);
    V center_a = pa, center_b = pb;
    Q qa = pqmul(ba->rotation, sa->local_rot);
    Q qb = pqmul(bb->rotation, sb->local_rot);
    int ta = sa->type, tb = sb->type, flip = 0;
    if (ta > tb) {
        const B3Shape* ts = sa; sa = sb; sb = ts;
        V tp = pa; pa = pb; pb = tp;
        Q tq = qa; qa = qb; qb = tq;
        int tt = ta; ta = tb; tb = tt;
        flip = 1;
    }
    if (ta == B3_SPHERE && tb == B3_SPHERE) {
        balls(m, pa, sa->radius, pb, sb->radius, 1u);
    } else if (ta == B3_SPHERE && tb == B3_CAPSULE) {
        V y = prot(qb, pv(0.0f, sb->half.y, 0.0f));
        balls(m, seg_closest(psub(pb, y), padd(pb, y), pa), sb->radius, pa, sa->radius, 4u);
        mflip(m);
    } else if (ta == B3_SPHERE && tb == B3_BOX) {
        sphere_box(m, pa, sa->radius, pb, qb, sb->half);
    } else if (ta == B3_CAPSULE && tb == B3_CAPSULE) {
        V ya = prot(qa, pv(0.0f, sa->half.y, 0.0f));
        V yb = prot(qb, pv(0.0f, sb->half.y, 0.0f));
        V ca, cb;
        segs_closest(psub(pa, ya), padd(pa, ya), psub(pb, yb), padd(pb, yb), &ca, &cb);
        balls(m, ca, sa->radius, cb, sb->radius, 2u);
    } else if (ta == B3_CAPSULE && tb == B3_BOX) {
        V y = prot(qa, pv(0.0f, sa->half.y, 0.0f));
        capsule_box(m, psub(pa, y), padd(pa, y), sa->radius, pb, qb, sb->half);
    } else {
        PObb oa, ob;
        oa.c = pa; oa.h = sa->half; paxes(qa, &oa.ax[0], &oa.ax[1], &oa.ax[2]);
        ob.c = pb; ob.h = sb->half; paxes(qb, &ob.ax[0], &ob.ax[1], &ob.ax[2]);
        box_box(m, &oa, &ob);
    }
    if (flip && m->count > 0) mflip(m);
    if (m->count > 0) {
        if (pdot(m->normal, psub(center_b, center_a)) < 0.0f) m->normal = pneg(m->normal);
        for (int i = 0; i < m->count; i++) m->sep[i] = pdot(psub(m->pb[i], m->pa[i]), m->normal);
    }
}

/* Shape AABB (04_world.inl:301-336). */
static B3AABB shape_box(const B3Body* b, const B3Shape* s) {
    V p = pxf(b->position, b->rotation, s->local_pos);
    Q q = pqmul(b->rotation, s->local_rot);
    B3AABB a;
    if (s->type == B3_SPHERE) {
        V e = pv(s->radius, s->radius, s->radius);
        a.lo = psub(p, e); a.hi = padd(p, e);
        return a;
    }
    if (s->type == B3_CAPSULE) {
        V y = prot(q, pv(0.0f, s->half.y, 0.0f));
        V c1 = psub(p, y), c2 = padd(p, y);
        V e = pv(s->radius, s->radius, s->radius);
        a.lo = pv(pmin(c1.x, c2.x), pmin(c1.y, c2.y), pmin(c1.z, c2.z));
        a.hi = pv(pmax(c1.x, c2.x), pmax(c1.y, c2.y), pmax(c1.z, c2.z));
        a.lo = psub(a.lo, e); a.hi = padd(a.hi, e);
        return a;
    }
    V ax, ay, az;
    paxes(q, &ax, &ay, &az);
    V e = pv(fabsf(ax.x) * s->half.x + fabsf(ay.x) * s->half.y + fabsf(az.x) * s->half.z,
        fabsf(ax.y) * s->half.x + fabsf(ay.y) * s->half.y + fabsf(az.y) * s->half.z,
        fabsf(ax.z) * s->half.x + fabsf(ay.z) * s->half.y + fabsf(az.z) * s->half.z);
    a.lo = psub(p, e); a.hi = padd(p, e);
    return a;
}

/* --------------------------------------------------------- contacts --- */
typedef struct PWarm {
    int sa, sb, n;
    uint32_t feat[B3_MAX_MANIFOLD];
    float ni[B3_MAX_MANIFOLD];
    B3Vec2 fi;
    float ti;
    V ri;
} PWarm;

/* Contact generation with warm-cache carry (08_contacts.inl:5-39, 45-62, 64-173). */
static void find_contacts(B3World* w) {
    static __thread PWarm old[B3_MAX_CONTACTS];
    static __thread B3AABB box[B3_MAX_SHAPES];
    static __thread uint64_t conn[B3_MAX_BODIES][B3_CONNECT_WORDS];
    int old_n = w->contact_count;
    for (int i = 0; i < old_n; i++) {
        const B3Contact* c = &w->contacts[i];
        old[i].sa = c->shape_a; old[i].sb = c->shape_b; old[i].n = c->point_count;
        old[i].fi = c->friction_impulse; old[i].ti = c->twist_impulse; old[i].ri = c->rolling_impulse;
        for (int p = 0; p < c->point_count; p++) {
            old[i].feat[p] = c->points[p].feature;
            old[i].ni[p] = c->points[p].normal_impulse;
        }
    }
    w->contact_count = 0;
    for (int i = 0; i < w->body_count; i++)
        for (int k = 0; k < B3_CONNECT_WORDS; k++) conn[i][k] = 0;
    for (int i = 0; i < w->joint_count; i++) {
        const B3Joint* j = &w->joints[i];
        if (j->collide_connected) continue;
        conn[j->body_a][j->body_b >> 6] |= 1ull << (j->body_b & 63);
        conn[j->body_b][j->body_a >> 6] |= 1ull << (j->body_a & 63);
    }
    V pad = pv(B3_SPECULATIVE, B3_SPECULATIVE, B3_SPECULATIVE);
    for (int i = 0; i < w->shape_count; i++) {
        box[i] = shape_box(&w->bodies[w->shapes[i].body], &w->shapes[i]);
        box[i].lo = psub(box[i].lo, pad);
        box[i].hi = padd(box[i].hi, pad);
    }
    for (int i = 0; i < w->shape_count; i++) {
        const B3Shape* sa = &w->shapes[i];
        const B3Body* ba = &w->bodies[sa->body];
        for (int j = i + 1; j < w->shape_count; j++) {
            const B3Shape* sb = &w->shapes[j];
            const B3Body* bb = &w->bodies[sb->body];
            if (sa->body == sb->body
                    || (conn[sa->body][sb->body >> 6] & (1ull << (sb->body & 63))) != 0
                    || (ba->type == B3_STATIC && bb->type == B3_STATIC)
                    || (sa->category & sb->mask) == 0 || (sb->category & sa->mask) == 0
                    || !(box[i].lo.x <= box[j].hi.x && box[i].hi.x >= box[j].lo.x
                        && box[i].lo.y <= box[j].hi.y && box[i].hi.y >= box[j].lo.y
                        && box[i].lo.z <= box[j].hi.z && box[i].hi.z >= box[j].lo.z))
                continue;
            PMani mani;
            collide(&mani, ba, sa, bb, sb);
            if (mani.count == 0) continue;
            if (w->contact_count >= B3_MAX_CONTACTS) {
                w->contact_overflow = 1;
                w->contacts_dropped++;
                continue;
            }
            B3Contact* c = &w->contacts[w->contact_count++];
            c->shape_a = i; c->shape_b = j;
            c->body_a = sa->body; c->body_b = sb->body;
            c->point_count = mani.count;
            c->normal = mani.normal;
            c->tangent1 = pperp(mani.normal);
            c->tangent2 = pcross(c->tangent1, mani.normal);
            c->friction = sqrtf(sa->friction * sb->friction);
            c->restitution = sa->restitution > sb->restitution ? sa->restitution : sb->restitution;
            c->rolling = pmax(sa->rolling, sb->rolling);
            c->static_contact = ba->type != B3_DYNAMIC || bb->type != B3_DYNAMIC;
            c->friction_impulse.x = 0.0f; c->friction_impulse.y = 0.0f;
            c->twist_impulse = 0.0f;
            c->rolling_impulse = pv(0.0f, 0.0f, 0.0f);
            for (int p = 0; p < mani.count; p++) {
                B3Point* cp = &c->points[p];
                cp->r_a = psub(mani.pa[p], ba->center);
                cp->r_b = psub(mani.pb[p], bb->center);
                cp->base_sep = mani.sep[p] - pdot(psub(cp->r_b, cp->r_a), mani.normal);
                cp->feature = mani.feat[p];
                cp->normal_impulse = 0.0f; cp->total_normal = 0.0f; cp->rel_vel = 0.0f;
                cp->normal_mass = 0.0f; cp->lever = 0.0f;
            }
            for (int k = 0; k < old_n; k++) {
                if (old[k].sa != i || old[k].sb != j) continue;
                for (int p = 0; p < c->point_count; p++)
                    for (int q = 0; q < old[k].n; q++)
                        if (c->points[p].feature == old[k].feat[q]) c->points[p].normal_impulse = old[k].ni[q];
                c->friction_impulse = old[k].fi;
                c->twist_impulse = old[k].ti;
                c->rolling_impulse = old[k].ri;
            }
        }
    }
}

/* 08_contacts.inl:234-291 */
static void prepare_contact(B3Contact* c, const B3Body* ba, const B3Body* bb, B3Soft cs, B3Soft ss) {
    float ma = ba->type == B3_DYNAMIC ? ba->inv_mass : 0.0f;
    float mb = bb->type == B3_DYNAMIC ? bb->inv_mass : 0.0f;
    M ia = ba->type == B3_DYNAMIC ? ba->inv_i_world : pmat0();
    M ib = bb->type == B3_DYNAMIC ? bb->inv_i_world : pmat0();
    c->inv_mass_a = ma; c->inv_mass_b = mb;
    c->inv_i_a = ia; c->inv_i_b = ib;
    c->rolling_mass = pinv3(pmaddm(ia, ib));
    c->softness = c->static_contact ? ss : cs;
    V n = c->normal;
    V center_a = pv(0.0f, 0.0f, 0.0f), center_b = pv(0.0f, 0.0f, 0.0f);
    float wsum = 0.0f;
    float inv_tau = 1.0f / B3_SPECULATIVE;
    for (int p = 0; p < c->point_count; p++) {
        B3Point* cp = &c->points[p];
        V rn_a = pcross(cp->r_a, n), rn_b = pcross(cp->r_b, n);
        float kn = ma + mb + pdot(rn_a, pmv(ia, rn_a)) + pdot(rn_b, pmv(ib, rn_b));
        cp->normal_mass = kn > 0.0f ? 1.0f / kn : 0.0f;
        V vra = padd(ba->lin_vel, pcross(ba->ang_vel, cp->r_a));
        V vrb = padd(bb->lin_vel, pcross(bb->ang_vel, cp->r_b));
        cp->rel_vel = pdot(n, psub(vrb, vra));
        cp->total_normal = 0.0f;
        float sep = cp->base_sep + pdot(psub(cp->r_b, cp->r_a), n);
        float wgt = pclamp(2.0f - sep * inv_tau, B3_MIN_FRICTION_W, 1.0f);
        center_a = pmadd(center_a, wgt, cp->r_a);
        center_b = pmadd(center_b, wgt, cp->r_b);
        wsum += wgt;
    }
    float invw = wsum > 0.0f ? 1.0f / wsum : 0.0f;
    c->center_a = pscale(center_a, invw);
    c->center_b = pscale(center_b, invw);
    for (int p = 0; p < c->point_count; p++) c->points[p].lever = plen(psub(c->points[p].r_a, c->center_a));
    V rta1 = pcross(c->center_a, c->tangent1), rta2 = pcross(c->center_a, c->tangent2);
    V rtb1 = pcross(c->center_b, c->tangent1), rtb2 = pcross(c->center_b, c->tangent2);
    B3Mat2 k;
    k.cx.x = ma + mb + pdot(rta1, pmv(ia, rta1)) + pdot(rtb1, pmv(ib, rtb1));
    k.cy.y = ma + mb + pdot(rta2, pmv(ia, rta2)) + pdot(rtb2, pmv(ib, rtb2));
    k.cx.y = k.cy.x = pdot(rta1, pmv(ia, rta2)) + pdot(rtb1, pmv(ib, rtb2));
    c->tangent_mass = pinv2(k);
    float kt = pdot(n, pmv(pmaddm(ia, ib), n));
    c->twist_mass = kt > 0.0f ? 1.0f / kt : 0.0f;
}

/* 08_contacts.inl:184-192 */
static void push_impulse(B3Body* b, float m, M i, V r, V p, int sign) {
    if ((b->flags & B3_FLAG_DYNAMIC) == 0) return;
    float s = sign > 0 ? 1.0f : -1.0f;
    b->lin_vel = pmadd(b->lin_vel, s * m, p);
    b->ang_vel = padd(b->ang_vel, pmv(i, pscale(pcross(r, p), s)));
}

/* 08_contacts.inl:293-313 */
static void warm_contact(B3Contact* c, B3Body* ba, B3Body* bb) {
    V n = c->normal;
    for (int p = 0; p < c->point_count; p++) {
        B3Point* cp = &c->points[p];
        V P = pscale(n, cp->normal_impulse);
        push_impulse(ba, c->inv_mass_a, c->inv_i_a, cp->r_a, P, -1);
        push_impulse(bb, c->inv_mass_b, c->inv_i_b, cp->r_b, P, 1);
    }
    V f = padd(pscale(c->tangent1, c->friction_impulse.x), pscale(c->tangent2, c->friction_impulse.y));
    push_impulse(ba, c->inv_mass_a, c->inv_i_a, c->center_a, f, -1);
    push_impulse(bb, c->inv_mass_b, c->inv_i_b, c->center_b, f, 1);
    if (ba->flags & B3_FLAG_DYNAMIC)
        ba->ang_vel = psub(ba->ang_vel, pmv(c->inv_i_a, padd(pscale(n, c->twist_impulse), c->rolling_impulse)));
    if (bb->flags & B3_FLAG_DYNAMIC)
        bb->ang_vel = padd(bb->ang_vel, pmv(c->inv_i_b, padd(pscale(n, c->twist_impulse), c->rolling_impulse)));
}

/* Rolling disk (07_packed.inl:24-45). */
static void solve_rolling(V t1, V t2, float rolling, float total_n, M ia, M ib, V* impulse, V* wa, V* wb) {
    if (rolling <= 0.0f) return;
    M isum = pmaddm(ia, ib);
    B3Mat2 k;
    k.cx.x = pdot(t1, pmv(isum, t1));
    k.cy.y = pdot(t2, pmv(isum, t2));
    k.cx.y = k.cy.x = pdot(t1, pmv(isum, t2));
    V wr = psub(*wb, *wa);
    B3Vec2 rhs; rhs.x = pdot(wr, t1); rhs.y = pdot(wr, t2);
    B3Vec2 d = pmv2(pinv2(k), rhs);
    V next = psub(*impulse, padd(pscale(t1, d.x), pscale(t2, d.y)));
    float limit = rolling * total_n;
    float l2 = plen2(next);
    if (l2 > limit * limit && l2 > 0.0f) next = pscale(next, limit / sqrtf(l2));
    V delta = psub(next, *impulse);
    *impulse = next;
    *wa = psub(*wa, pmv(ia, delta));
    *wb = padd(*wb, pmv(ib, delta));
}

/* 08_contacts.inl:315-413 */
static void solve_contact(B3Contact* c, B3Body* ba, B3Body* bb, float inv_h, float speed, int use_bias) {
    V va = ba->lin_vel, wa = ba->ang_vel, vb = bb->lin_vel, wb = bb->ang_vel;
    Q dqa = ba->delta_rot, dqb = bb->delta_rot;
    V dp = psub(bb->delta_pos, ba->delta_pos);
    V n = c->normal;
    float total_n = 0.0f, twist_lim = 0.0f;
    for (int p = 0; p < c->point_count; p++) {
        B3Point* cp = &c->points[p];
        V ra = cp->r_a, rb = cp->r_b;
        V ds = padd(dp, psub(prot(dqb, rb), prot(dqa, ra)));
        float sep = pdot(ds, n) + cp->base_sep;
        float vbias = 0.0f, mscale = 1.0f, iscale = 0.0f;
        if (sep > 0.0f) {
            vbias = sep * inv_h;
        } else if (use_bias) {
            vbias = pmax(c->softness.mass_scale * c->softness.bias_rate * sep, -speed);
            mscale = c->softness.mass_scale;
            iscale = c->softness.impulse_scale;
        }
        V vra = padd(va, pcross(wa, ra)), vrb = padd(vb, pcross(wb, rb));
        float vn = pdot(psub(vrb, vra), n);
        float dimp = -cp->normal_mass * (mscale * vn + vbias) - iscale * cp->normal_impulse;
        float nimp = pmax(cp->normal_impulse + dimp, 0.0f);
        dimp = nimp - cp->normal_impulse;
        cp->normal_impulse = nimp;
        cp->total_normal += nimp;
        total_n += nimp;
        twist_lim += cp->lever * cp->normal_impulse;
        V P = pscale(n, dimp);
        va = pmsub(va, c->inv_mass_a, P);
        wa = psub(wa, pmv(c->inv_i_a, pcross(ra, P)));
        vb = pmadd(vb, c->inv_mass_b, P);
        wb = padd(wb, pmv(c->inv_i_b, pcross(rb, P)));
    }
    if (!use_bias) {
        float twist_s = pdot(n, psub(wb, wa));
        float max_t = c->friction * twist_lim;
        float dtw = -c->twist_mass * twist_s;
        float old_t = c->twist_impulse;
        c->twist_impulse = pclamp(old_t + dtw, -max_t, max_t);
        dtw = c->twist_impulse - old_t;
        wa = psub(wa, pmv(c->inv_i_a, pscale(n, dtw)));
        wb = padd(wb, pmv(c->inv_i_b, pscale(n, dtw)));
        V t1 = c->tangent1, t2 = c->tangent2, ra = c->center_a, rb = c->center_b;
        V vra = padd(va, pcross(wa, ra)), vrb = padd(vb, pcross(wb, rb));
        V vr = psub(vrb, vra);
        B3Vec2 vt; vt.x = pdot(vr, t1); vt.y = pdot(vr, t2);
        B3Vec2 tm = pmv2(c->tangent_mass, vt);
        B3Vec2 ni; ni.x = c->friction_impulse.x - tm.x; ni.y = c->friction_impulse.y - tm.y;
        float max_f = c->friction * total_n;
        float fl2 = ni.x * ni.x + ni.y * ni.y;
        if (fl2 > max_f * max_f && fl2 > 0.0f) {
            float sc = max_f / sqrtf(fl2);
            ni.x *= sc; ni.y *= sc;
        }
        B3Vec2 df; df.x = ni.x - c->friction_impulse.x; df.y = ni.y - c->friction_impulse.y;
        c->friction_impulse = ni;
        V P = padd(pscale(t1, df.x), pscale(t2, df.y));
        va = pmsub(va, c->inv_mass_a, P);
        wa = psub(wa, pmv(c->inv_i_a, pcross(ra, P)));
        vb = pmadd(vb, c->inv_mass_b, P);
        wb = padd(wb, pmv(c->inv_i_b, pcross(rb, P)));
        solve_rolling(c->tangent1, c->tangent2, c->rolling, total_n, c->inv_i_a, c->inv_i_b,
            &c->rolling_impulse, &wa, &wb);
    }
    if (ba->flags & B3_FLAG_DYNAMIC) { ba->lin_vel = va; ba->ang_vel = wa; }
    if (bb->flags & B3_FLAG_DYNAMIC) { bb->lin_vel = vb; bb->ang_vel = wb; }
}

/* 08_contacts.inl:439-480 */
static void restitution(B3World* w, float threshold) {
    for (int i = 0; i < w->contact_count; i++) {
        B3Contact* c = &w->contacts[i];
        if (c->restitution == 0.0f) continue;
        B3Body* ba = &w->bodies[c->body_a];
        B3Body* bb = &w->bodies[c->body_b];
        V va = ba->lin_vel, wa = ba->ang_vel, vb = bb->lin_vel, wb = bb->ang_vel;
        V n = c->normal;
        for (int p = 0; p < c->point_count; p++) {
            B3Point* cp = &c->points[p];
            if (cp->rel_vel > -threshold || cp->total_normal == 0.0f) continue;
            V vra = padd(va, pcross(wa, cp->r_a)), vrb = padd(vb, pcross(wb, cp->r_b));
            float vn = pdot(psub(vrb, vra), n);
            float imp = -cp->normal_mass * (vn + c->restitution * cp->rel_vel);
            float nimp = pmax(cp->normal_impulse + imp, 0.0f);
            imp = nimp - cp->normal_impulse;
            cp->normal_impulse = nimp;
            V P = pscale(n, imp);
            va = pmsub(va, c->inv_mass_a, P);
            wa = psub(wa, pmv(c->inv_i_a, pcross(cp->r_a, P)));
            vb = pmadd(vb, c->inv_mass_b, P);
            wb = padd(wb, pmv(c->inv_i_b, pcross(cp->r_b, P)));
        }
        if (ba->flags & B3_FLAG_DYNAMIC) { ba->lin_vel = va; ba->ang_vel = wa; }
        if (bb->flags & B3_FLAG_DYNAMIC) { bb->lin_vel = vb; bb->ang_vel = wb; }
    }
}

/* ------------------------------------------------------------ joints --- */
/* 06_joints.inl:161-202 */
static void prepare_joints(B3World* w, float h) {
    for (int i = 0; i < w->joint_count; i++) {
        B3Joint* j = &w->joints[i];
        const B3Body* ba = &w->bodies[j->body_a];
        const B3Body* bb = &w->bodies[j->body_b];
        j->inv_mass_a = ba->type == B3_DYNAMIC ? ba->inv_mass : 0.0f;
        j->inv_mass_b = bb->type == B3_DYNAMIC ? bb->inv_mass : 0.0f;
        j->inv_i_a = ba->type == B3_DYNAMIC ? ba->inv_i_world : pmat0();
        j->inv_i_b = bb->type == B3_DYNAMIC ? bb->inv_i_world : pmat0();
        M isum = pmaddm(j->inv_i_a, j->inv_i_b);
        j->fixed_rotation = pdot(isum.cx, pcross(isum.cy, isum.cz)) < 1.0e-20f;
        j->softness = psoft(j->constraint_hertz, j->constraint_damping, h);
        j->frame_q_a = pqmul(ba->rotation, j->local_rot_a);
        j->frame_q_b = pqmul(bb->rotation, j->local_rot_b);
        j->frame_p_a = prot(ba->rotation, psub(j->local_anchor_a, ba->local_center));
        j->frame_p_b = prot(bb->rotation, psub(j->local_anchor_b, bb->local_center));
        j->delta_center = psub(bb->center, ba->center);
        if (j->type == B3_JOINT_WELD) {
            j->angular_mass = pinv3(isum);
            j->linear_spring = j->linear_hertz == 0.0f ? j->softness
                : psoft(j->linear_hertz, j->linear_damping, h);
            j->angular_spring = j->angular_hertz == 0.0f ? j->softness
                : psoft(j->angular_hertz, j->angular_damping, h);
        } else {
            V axis = prot(j->frame_q_a, pv(0.0f, 0.0f, 1.0f));
            float k = pdot(axis, pmv(isum, axis));
            j->axial_mass = k > 0.0f ? 1.0f / k : 0.0f;
            j->rotation_axis = axis;
            Q rel = pqinvmul(j->frame_q_a, j->frame_q_b);
            phperps(j->frame_q_a, rel, &j->perp_x, &j->perp_y);
            j->spring_softness = psoft(j->hertz, j->damping_ratio, h);
        }
    }
}

/* 06_joints.inl:204-239 */
static void warm_joints(B3World* w) {
    for (int i = 0; i < w->joint_count; i++) {
        B3Joint* j = &w->joints[i];
        B3Body* ba = &w->bodies[j->body_a];
        B3Body* bb = &w->bodies[j->body_b];
        V ra = prot(ba->delta_rot, j->frame_p_a);
        V rb = prot(bb->delta_rot, j->frame_p_b);
        V ang = j->angular_impulse;
        if (j->type == B3_JOINT_REVOLUTE) {
            float axial = j->spring_impulse + j->motor_impulse + j->lower_impulse - j->upper_impulse;
            ang = padd(pscale(j->perp_x, j->perp_impulse.x), pscale(j->perp_y, j->perp_impulse.y));
            ang = pmadd(ang, axial, j->rotation_axis);
        }
        if (ba->flags & B3_FLAG_DYNAMIC) {
            ba->lin_vel = pmsub(ba->lin_vel, j->inv_mass_a, j->linear_impulse);
            ba->ang_vel = psub(ba->ang_vel, pmv(j->inv_i_a, padd(pcross(ra, j->linear_impulse), ang)));
        }
        if (bb->flags & B3_FLAG_DYNAMIC) {
            bb->lin_vel = pmadd(bb->lin_vel, j->inv_mass_b, j->linear_impulse);
            bb->ang_vel = padd(bb->ang_vel, pmv(j->inv_i_b, padd(pcross(rb, j->linear_impulse), ang)));
        }
    }
}

/* 06_joints.inl:241-255 */
static M point_k(float ma, float mb, M ia, M ib, V ra, V rb) {
    float msum = ma + mb;
    M k;
    k.cx = pv(msum, 0.0f, 0.0f);
    k.cy = pv(0.0f, msum, 0.0f);
    k.cz = pv(0.0f, 0.0f, msum);
    k.cx = psub(k.cx, pcross(ra, pmv(ia, pv(0.0f, ra.z, -ra.y))));
    k.cy = psub(k.cy, pcross(ra, pmv(ia, pv(-ra.z, 0.0f, ra.x))));
    k.cz = psub(k.cz, pcross(ra, pmv(ia, pv(ra.y, -ra.x, 0.0f))));
    k.cx = psub(k.cx, pcross(rb, pmv(ib, pv(0.0f, rb.z, -rb.y))));
    k.cy = psub(k.cy, pcross(rb, pmv(ib, pv(-rb.z, 0.0f, rb.x))));
    k.cz = psub(k.cz, pcross(rb, pmv(ib, pv(rb.y, -rb.x, 0.0f))));
    return k;
}

/* 06_joints.inl:257-282 */
static void solve_point(B3Joint* j, const B3Body* ba, const B3Body* bb, V* va, V* wa, V* vb, V* wb,
        B3Soft soft, int use_bias) {
    V ra = prot(ba->delta_rot, j->frame_p_a);
    V rb = prot(bb->delta_rot, j->frame_p_b);
    V cdot = psub(padd(*vb, pcross(*wb, rb)), padd(*va, pcross(*wa, ra)));
    V bias = pv(0.0f, 0.0f, 0.0f);
    float mscale = 1.0f, iscale = 0.0f;
    if (use_bias) {
        V sep = padd(padd(psub(bb->delta_pos, ba->delta_pos), psub(rb, ra)), j->delta_center);
        bias = pscale(sep, soft.bias_rate);
        mscale = soft.mass_scale;
        iscale = soft.impulse_scale;
    }
    V b = pmv(pinv3(point_k(j->inv_mass_a, j->inv_mass_b, j->inv_i_a, j->inv_i_b, ra, rb)), padd(cdot, bias));
    V impulse = pmsub(pscale(b, -mscale), iscale, j->linear_impulse);
    j->linear_impulse = padd(j->linear_impulse, impulse);
    *va = pmsub(*va, j->inv_mass_a, impulse);
    *wa = psub(*wa, pmv(j->inv_i_a, pcross(ra, impulse)));
    *vb = pmadd(*vb, j->inv_mass_b, impulse);
    *wb = padd(*wb, pmv(j->inv_i_b, pcross(rb, impulse)));
}

/* 06_joints.inl:285-332 */
static void solve_weld(B3Joint* j, B3Body* ba, B3Body* bb, int use_bias) {
    V va = ba->lin_vel, wa = ba->ang_vel, vb = bb->lin_vel, wb = bb->ang_vel;
    Q qa = pqmul(ba->delta_rot, j->frame_q_a);
    Q qb = pqmul(bb->delta_rot, j->frame_q_b);
    if (pqdot(qa, qb) < 0.0f) qb = pqneg(qb);
    Q rel = pqinvmul(qa, qb);
    if (!j->fixed_rotation) {
        V bias = pv(0.0f, 0.0f, 0.0f);
        float mscale = 1.0f, iscale = 0.0f;
        if (use_bias || j->angular_hertz > 0.0f) {
            Q s = rel;
            if (rel.s < 0.0f) s = pqneg(rel);
            Q diff = pq(-s.v.x, -s.v.y, -s.v.z, 1.0f - s.s);
            V c = pneg(prot(qa, pscale(pqmul(diff, pqconj(s)).v, 2.0f)));
            bias = pscale(c, j->angular_spring.bias_rate);
            mscale = j->angular_spring.mass_scale;
            iscale = j->angular_spring.impulse_scale;
        }
        V cdot = psub(wb, wa);
        V impulse = pmsub(pscale(pmv(j->angular_mass, padd(cdot, bias)), -mscale), iscale, j->angular_impulse);
        j->angular_impulse = padd(j->angular_impulse, impulse);
        wa = psub(wa, pmv(j->inv_i_a, impulse));
        wb = padd(wb, pmv(j->inv_i_b, impulse));
    }
    int lin_bias = use_bias || j->linear_hertz > 0.0f;
    solve_point(j, ba, bb, &va, &wa, &vb, &wb, j->linear_spring, lin_bias);
    if (ba->flags & B3_FLAG_DYNAMIC) { ba->lin_vel = va; ba->ang_vel = wa; }
    if (bb->flags & B3_FLAG_DYNAMIC) { bb->lin_vel = vb; bb->ang_vel = wb; }
}

/* 06_joints.inl:419-434 */
static float limit_row(float c, float cdot, float inv_h, int use_bias, B3Soft soft, float axial_mass, float old) {
    float bias = 0.0f, mscale = 1.0f, iscale = 0.0f;
    if (c > 0.0f) {
        bias = c * inv_h;
    } else if (use_bias) {
        bias = soft.bias_rate * c;
        mscale = soft.mass_scale;
        iscale = soft.impulse_scale;
    }
    float dimp = -mscale * axial_mass * (cdot + bias) - iscale * old;
    return pmax(old + dimp, 0.0f);
}

/* 06_joints.inl:436-642 (default, uncached path) */
static void solve_revolute(B3Joint* j, B3Body* ba, B3Body* bb, float h, float inv_h, int use_bias) {
    V va = ba->lin_vel, wa = ba->ang_vel, vb = bb->lin_vel, wb = bb->ang_vel;
    Q qa = pqmul(ba->delta_rot, j->frame_q_a);
    Q qb = pqmul(bb->delta_rot, j->frame_q_b);
    if (pqdot(qa, qb) < 0.0f) qb = pqneg(qb);
    Q rel = pqinvmul(qa, qb);
    V axis = j->rotation_axis;
    V ia_ax = pv(0.0f, 0.0f, 0.0f), ib_ax = pv(0.0f, 0.0f, 0.0f);
    float twist = 0.0f;
    int need_twist = (j->enable_spring || j->enable_limit || j->enable_motor) && !j->fixed_rotation;
    if (!j->fixed_rotation) {
        ia_ax = pmv(j->inv_i_a, axis);
        ib_ax = pmv(j->inv_i_b, axis);
    }
    if (need_twist) twist = ptwist(rel);
    if (j->enable_spring && !j->fixed_rotation) {
        float c = twist - j->target_angle;
        float bias = j->spring_softness.bias_rate * c;
        float mscale = j->spring_softness.mass_scale;
        float iscale = j->spring_softness.impulse_scale;
        float cdot = pdot(psub(wb, wa), axis);
        float dimp = -mscale * j->axial_mass * (cdot + bias) - iscale * j->spring_impulse;
        float old = j->spring_impulse;
        float nimp = old + dimp;
        if (j->max_motor_torque > 0.0f) {
            float maxp = j->max_motor_torque * h;
            nimp = pclamp(nimp, -maxp, maxp);
        }
        dimp = nimp - old;
        j->spring_impulse = nimp;
        wa = pmsub(wa, dimp, ia_ax);
        wb = pmadd(wb, dimp, ib_ax);
    }
    if (j->enable_motor && !j->fixed_rotation) {
        int blocked = 0;
        if (j->enable_limit) {
            if (twist >= j->upper_angle - 0.01f && j->motor_speed > 0.0f) blocked = 1;
            if (twist <= j->lower_angle + 0.01f && j->motor_speed < 0.0f) blocked = 1;
        }
        if (blocked) {
            j->motor_impulse = 0.0f;
        } else {
            float cdot = pdot(psub(wb, wa), axis) - j->motor_speed;
            float dimp = -j->axial_mass * cdot;
            float nimp = j->motor_impulse + dimp;
            float maxp = j->max_motor_torque * h;
            nimp = pclamp(nimp, -maxp, maxp);
            dimp = nimp - j->motor_impulse;
            j->motor_impulse = nimp;
            wa = pmsub(wa, dimp, ia_ax);
            wb = pmadd(wb, dimp, ib_ax);
        }
    }
    if (j->enable_limit && !j->fixed_rotation) {
        float old = j->lower_impulse;
        j->lower_impulse = limit_row(twist - j->lower_angle, pdot(psub(wb, wa), axis), inv_h, use_bias,
            j->softness, j->axial_mass, old);
        float dimp = j->lower_impulse - old;
        wa = pmsub(wa, dimp, ia_ax);
        wb = pmadd(wb, dimp, ib_ax);
        old = j->upper_impulse;
        j->upper_impulse = limit_row(j->upper_angle - twist, pdot(psub(wa, wb), axis), inv_h, use_bias,
            j->softness, j->axial_mass, old);
        dimp = j->upper_impulse - old;
        wa = pmadd(wa, dimp, ia_ax);
        wb = pmsub(wb, dimp, ib_ax);
    }
    if (!j->fixed_rotation) {
        B3Vec2 bias; bias.x = 0.0f; bias.y = 0.0f;
        float mscale = 1.0f, iscale = 0.0f;
        if (use_bias) {
            bias.x = j->softness.bias_rate * rel.v.x;
            bias.y = j->softness.bias_rate * rel.v.y;
            mscale = j->softness.mass_scale;
            iscale = j->softness.impulse_scale;
        }
        V px, py;
        phperps(qa, rel, &px, &py);
        j->perp_x = px;
        j->perp_y = py;
        M isum = pmaddm(j->inv_i_a, j->inv_i_b);
        B3Mat2 kang;
        kang.cx.x = pdot(px, pmv(isum, px));
        kang.cy.y = pdot(py, pmv(isum, py));
        kang.cx.y = kang.cy.x = pdot(px, pmv(isum, py));
        V wrel = psub(wb, wa);
        B3Vec2 rhs; rhs.x = pdot(wrel, px) + bias.x; rhs.y = pdot(wrel, py) + bias.y;
        B3Vec2 sol = psolve2(kang, rhs);
        B3Vec2 old = j->perp_impulse;
        B3Vec2 dimp;
        dimp.x = -mscale * sol.x - iscale * old.x;
        dimp.y = -mscale * sol.y - iscale * old.y;
        j->perp_impulse.x += dimp.x;
        j->perp_impulse.y += dimp.y;
        V ang = padd(pscale(px, dimp.x), pscale(py, dimp.y));
        wa = psub(wa, pmv(j->inv_i_a, ang));
        wb = padd(wb, pmv(j->inv_i_b, ang));
    }
    solve_point(j, ba, bb, &va, &wa, &vb, &wb, j->softness, use_bias);
    if (ba->flags & B3_FLAG_DYNAMIC) { ba->lin_vel = va; ba->ang_vel = wa; }
    if (bb->flags & B3_FLAG_DYNAMIC) { bb->lin_vel = vb; bb->ang_vel = wb; }
}

static void solve_contacts(B3World* w, float inv_h, int use_bias);

/* 07_packed.inl:48-81; with B3_INTERLEAVE_CONTACTS a contact sweep opens
 * every iteration (07_packed.inl:63-65) */
static void solve_joints(B3World* w, float h, float inv_h, int use_bias, int iters) {
    for (int it = 0; it < iters; it++) {
#ifdef B3_INTERLEAVE_CONTACTS
        solve_contacts(w, inv_h, use_bias);
#endif
        for (int i = 0; i < w->joint_count; i++) {
            B3Joint* j = &w->joints[i];
            B3Body* ba = &w->bodies[j->body_a];
            B3Body* bb = &w->bodies[j->body_b];
            if (j->type == B3_JOINT_WELD) solve_weld(j, ba, bb, use_bias);
            else solve_revolute(j, ba, bb, h, inv_h, use_bias);
        }
    }
}

/* -------------------------------------------------------------- step --- */
/* 09_step.inl:5-18, 41-53 */
static void integrate_velocities(B3World* w, float h) {
#ifdef B3_USER_FORCES
    /* the per-substep hook's contributions last one substep (09_step.inl:20-53) */
    V saved_f[B3_MAX_BODIES], saved_t[B3_MAX_BODIES];
    for (int i = 0; i < w->body_count; i++) {
        saved_f[i] = w->bodies[i].force;
        saved_t[i] = w->bodies[i].torque;
    }
    B3_USER_FORCES(w, h);
#endif
    for (int i = 0; i < w->body_count; i++) {
        B3Body* b = &w->bodies[i];
        if (b->type != B3_DYNAMIC) continue;
        float ld = 1.0f / (1.0f + h * b->linear_damping);
        float ad = 1.0f / (1.0f + h * b->angular_damping);
        float gs = b->inv_mass > 0.0f ? b->gravity_scale : 0.0f;
        V dv = padd(pscale(b->force, h * b->inv_mass), pscale(w->gravity, h * gs));
        b->lin_vel = pmadd(dv, ld, b->lin_vel);
        V dw = pscale(pmv(b->inv_i_world, b->torque), h);
        b->ang_vel = pmadd(dw, ad, b->ang_vel);
    }
#ifdef B3_USER_FORCES
    for (int i = 0; i < w->body_count; i++) {
        w->bodies[i].force = saved_f[i];
        w->bodies[i].torque = saved_t[i];
    }
#endif
}

/* 09_step.inl:55-107 */
static void integrate_positions(B3World* w, float h, float inv_dt, float max_lin) {
    float max_ang = B3_MAX_ROTATION * inv_dt;
    float max_lin2 = max_lin * max_lin, max_ang2 = max_ang * max_ang;
    for (int i = 0; i < w->body_count; i++) {
        B3Body* b = &w->bodies[i];
        if (b->type == B3_STATIC) continue;
        V v = b->lin_vel, av = b->ang_vel;
        if (b->flags & B3_LOCK_LIN_X) v.x = 0.0f;
        if (b->flags & B3_LOCK_LIN_Y) v.y = 0.0f;
        if (b->flags & B3_LOCK_LIN_Z) v.z = 0.0f;
        if (b->flags & B3_LOCK_ANG_X) av.x = 0.0f;
        if (b->flags & B3_LOCK_ANG_Y) av.y = 0.0f;
        if (b->flags & B3_LOCK_ANG_Z) av.z = 0.0f;
        float v2 = plen2(v);
        if (v2 > max_lin2 && v2 > 0.0f) v = pscale(v, max_lin / sqrtf(v2));
        float w2 = plen2(av);
        if (w2 > max_ang2 && w2 > 0.0f) av = pscale(av, max_ang / sqrtf(w2));
        b->lin_vel = v;
        b->ang_vel = av;
        b->delta_pos = pmadd(b->delta_pos, h, v);
        b->delta_rot = pqint(b->delta_rot, pscale(av, h));
    }
}

/* 09_step.inl:109-130 */
static void finalize(B3World* w) {
    for (int i = 0; i < w->body_count; i++) {
        B3Body* b = &w->bodies[i];
        if (b->type == B3_STATIC) continue;
        b->center = padd(b->center, b->delta_pos);
        b->rotation = pqnorm(pqmul(b->delta_rot, b->rotation));
        b->position = psub(b->center, prot(b->rotation, b->local_center));
        b->delta_pos = pv(0.0f, 0.0f, 0.0f);
        b->delta_rot = pqid();
        b->force = pv(0.0f, 0.0f, 0.0f);
        b->torque = pv(0.0f, 0.0f, 0.0f);
        if (b->type == B3_DYNAMIC) b->inv_i_world = pwinvi(b->rotation, b->inv_inertia);
    }
}

/* 08_contacts.inl:424-437 */
static void solve_contacts(B3World* w, float inv_h, int use_bias) {
    for (int i = 0; i < w->contact_count; i++) {
        B3Contact* c = &w->contacts[i];
        solve_contact(c, &w->bodies[c->body_a], &w->bodies[c->body_b], inv_h, w->contact_speed, use_bias);
    }
}

/* b3_step_indep (09_step.inl:148-258) with the default substep (167-181). */
void b3port_step(B3World* w, float dt, int substeps, int joint_iters, int relax_iters) {
    if (dt <= 0.0f) return;
    int subs = substeps < 1 ? 1 : substeps;
    float h = dt / (float)subs;
    float inv_dt = 1.0f / dt;
    float inv_h = (float)subs * inv_dt;
    float hertz = pmin(w->contact_hertz, 0.25f * inv_h);
    B3Soft cs = psoft(hertz, w->contact_damping, h);
    B3Soft ss = psoft(2.0f * hertz, 0.5f * w->contact_damping, h);
    find_contacts(w);
    for (int i = 0; i < w->contact_count; i++) {
        B3Contact* c = &w->contacts[i];
        prepare_contact(c, &w->bodies[c->body_a], &w->bodies[c->body_b], cs, ss);
    }
    prepare_joints(w, h);
    for (int i = 0; i < w->contact_count; i++) {
        B3Contact* c = &w->contacts[i];
        warm_contact(c, &w->bodies[c->body_a], &w->bodies[c->body_b]);
    }
    warm_joints(w);
    for (int s = 0; s < subs; s++) {
        integrate_velocities(w, h);
#ifndef B3_INTERLEAVE_CONTACTS
        solve_contacts(w, inv_h, 1);
#endif
        solve_joints(w, h, inv_h, 1, joint_iters);
        integrate_positions(w, h, inv_dt, w->max_linear_speed);
#ifndef B3_INTERLEAVE_CONTACTS
        solve_contacts(w, inv_h, 0);
#endif
        solve_joints(w, h, inv_h, 0, relax_iters);
#ifndef B3_SKIP_RESTITUTION
        restitution(w, w->restitution_threshold);
#endif
    }
    finalize(w);
}

/* b3_batch_step (b3_batch.cuh:39-48). */
int b3port_batch_step(B3Batch batch, float dt, int substeps, const unsigned char* active,
        int joint_iters, int relax_iters) {
    if (!b3_batch_valid(batch) || !isfinite(dt) || dt < 0 || substeps < 1) return 0;
    if (dt == 0) return 1;
    for (int i = 0; i < batch.count; i++)
        if (!active || active[i]) b3port_step(b3_batch_world(batch, i), dt, substeps, joint_iters, relax_iters);
    return 1;
}

/* b3_batch_restore (b3_batch.cuh:50-60). */
int b3port_batch_restore(B3Batch batch, const B3World* initial, const unsigned char* reset) {
    if (!b3_batch_valid(batch) || (batch.count && !initial)) return 0;
    for (int i = 0; i < batch.count; i++)
        if (!reset || reset[i]) *b3_batch_world(batch, i) = initial[i];
    return 1;
}

/* Narrowphase alone on two shapes of one world, for manifold known-answer
 * tests: fills count, normal[3], pa[12], pb[12], sep[4], feature[4]. */
int b3port_collide(const B3World* w, int shape_a, int shape_b, float* normal, float* pa, float* pb,
        float* sep, unsigned* feature) {
    PMani m;
    const B3Shape* sa = &w->shapes[shape_a];
    const B3Shape* sb = &w->shapes[shape_b];
    collide(&m, &w->bodies[sa->body], sa, &w->bodies[sb->body], sb);
    normal[0] = m.normal.x; normal[1] = m.normal.y; normal[2] = m.normal.z;
    for (int i = 0; i < m.count; i++) {
        pa[3 * i] = m.pa[i].x; pa[3 * i + 1] = m.pa[i].y; pa[3 * i + 2] = m.pa[i].z;
        pb[3 * i] = m.pb[i].x; pb[3 * i + 1] = m.pb[i].y; pb[3 * i + 2] = m.pb[i].z;
        sep[i] = m.sep[i];
        feature[i] = m.feat[i];
    }
    return m.count;
}
