// b3x_world_step.cuh -- b3_step for ONE world on ONE thread (device code).
//
// This is the per-world entry point of the reference (src/puffysics/
// 09_step.inl:262-264, b3_step -> b3_step_indep :183-258, default substep
// :167-181) for adapters that call b3_step from their own fused kernels, one
// thread per environment (examples/pufferlib/puffysics_hover/
// puffysics_hover.cu:40-43).  Semantics are unchanged: the world is stepped
// in place in its AoS B3World image, contacts are regenerated in (i, j)
// order with the warm-cache carry, then the reference's Gauss-Seidel order
// (contacts in index order, then joints in index order) runs per substep.
//
// It is the compatibility path, not the fast one: a thread walks a strided
// multi-kilobyte struct, as in the reference.  The batched step
// (b3x_batch_step_gpu, tiles of 32 worlds in lane-interleaved columns) is the
// throughput path; an adapter moves to it by calling b3_batch_step_gpu from
// the host instead of b3_step from its kernel.
//
// The narrowphase and the small matrix helpers are the batched kernel's own
// (b3x_narrow.cuh, b3x_math.cuh); what is here is the per-world driver around
// them.  Compiled with -fmad=false -prec-div=true -prec-sqrt=true, results
// are bit-identical to the reference's CPU b3_step built with
// -ffp-contract=off (atan2f of revolute twists aside, whose device and libm
// results may differ in the last bit).  Device only: the library ships no CPU
// implementation of the step.
#pragma once

#include "puffysics_b200.h"
#include "b3x_math.cuh"
// Narrowphase functions get internal linkage here, so that an adapter may
// include this header in several translation units.
#ifndef B3X_NARROW
#define B3X_NARROW static B3X_HD
#endif
#include "b3x_narrow.cuh"
#include "b3x_art.cuh"
#include <type_traits>

#if defined(__CUDACC__)
namespace b3x {
namespace one {

// Warm-start data of one contact of the previous step (08_contacts.inl:66-79).
struct Carry {
    int sa, sb, n;
    uint32_t feat[B3_MAX_MANIFOLD];
    float ni[B3_MAX_MANIFOLD];
    B3Vec2 fi;
    float ti;
    B3Vec3 ri;
};

__device__ __forceinline__ B3Vec3 zero3() { return b3_v(0.0f, 0.0f, 0.0f); }

__device__ __forceinline__ bool dynamic_flag(const B3Body& b) { return (b.flags & B3_FLAG_DYNAMIC) != 0u; }

// World pose of a shape: body pose composed with the shape's local pose
// (05_collision.inl:472-480).
__device__ __forceinline__ Geo shape_geo(const B3Body& b, const B3Shape& s) {
    Geo g;
    g.p = b3_xf_point(b.position, b.rotation, s.local_pos);
    g.q = b3_qmul(b.rotation, s.local_rot);
    g.type = s.type;
    g.radius = s.radius;
    g.half = s.half;
    return g;
}

// Shape AABB padded by the speculative distance (04_world.inl:301-336,
// 08_contacts.inl:92-97).
__device__ __forceinline__ B3AABB padded_box(const Geo& g) {
    B3AABB a;
    if (g.type == B3_SPHERE) {
        B3Vec3 e = b3_v(g.radius, g.radius, g.radius);
        a.lo = b3_sub(g.p, e);
        a.hi = b3_add(g.p, e);
    } else if (g.type == B3_CAPSULE) {
        B3Vec3 y = b3_rotate(g.q, b3_v(0.0f, g.half.y, 0.0f));
        B3Vec3 c1 = b3_sub(g.p, y), c2 = b3_add(g.p, y);
        B3Vec3 e = b3_v(g.radius, g.radius, g.radius);
        a.lo = b3_sub(b3_v(b3_minf(c1.x, c2.x), b3_minf(c1.y, c2.y), b3_minf(c1.z, c2.z)), e);
        a.hi = b3_add(b3_v(b3_maxf(c1.x, c2.x), b3_maxf(c1.y, c2.y), b3_maxf(c1.z, c2.z)), e);
    } else {
        B3Vec3 ax, ay, az;
        b3_axes(g.q, &ax, &ay, &az);
        B3Vec3 e = b3_v(fabsf(ax.x) * g.half.x + fabsf(ay.x) * g.half.y + fabsf(az.x) * g.half.z,
                        fabsf(ax.y) * g.half.x + fabsf(ay.y) * g.half.y + fabsf(az.y) * g.half.z,
                        fabsf(ax.z) * g.half.x + fabsf(ay.z) * g.half.y + fabsf(az.z) * g.half.z);
        a.lo = b3_sub(g.p, e);
        a.hi = b3_add(g.p, e);
    }
    B3Vec3 pad = b3_v(B3_SPECULATIVE, B3_SPECULATIVE, B3_SPECULATIVE);
    a.lo = b3_sub(a.lo, pad);
    a.hi = b3_add(a.hi, pad);
    return a;
}

__device__ __forceinline__ bool overlap(const B3AABB& a, const B3AABB& b) {
    return a.lo.x <= b.hi.x && a.hi.x >= b.lo.x && a.lo.y <= b.hi.y && a.hi.y >= b.lo.y && a.lo.z <= b.hi.z
        && a.hi.z >= b.lo.z;
}

__device__ __forceinline__ bool pair_less(int a0, int b0, int a1, int b1) {
    return a0 < a1 || (a0 == a1 && b0 < b1);
}

// Body velocity impulse (08_contacts.inl:184-192): dynamic bodies only.
__device__ __forceinline__ void push(B3Body& b, float m, const B3Mat3& i, B3Vec3 r, B3Vec3 p, float s) {
    if (!dynamic_flag(b)) return;
    b.lin_vel = b3_madd(b.lin_vel, s * m, p);
    b.ang_vel = b3_add(b.ang_vel, b3_mv(i, b3_mul(b3_cross(r, p), s)));
}

__device__ __forceinline__ void store_vel(B3Body& b, B3Vec3 v, B3Vec3 w) {
    if (dynamic_flag(b)) {
        b.lin_vel = v;
        b.ang_vel = w;
    }
}

// One world's arrays.  The element structs do not depend on the capacities,
// only the array lengths (and so the offsets of shapes, contacts and joints)
// do: a view addresses a world image of any capacity configuration through
// its header and four array bases.  kB / kS / kC bound the per-world scratch
// and must be at least the capacities.
template <int MB, int MS, int MC>
struct WorldView {
    static constexpr int kB = MB, kS = MS, kC = MC;
    B3World* h;            // header fields only (their offsets are fixed)
    B3Body* bodies;
    B3Shape* shapes;
    B3Contact* contacts;
    B3Joint* joints;
    int cap_b, cap_s, cap_c, cap_j;
};

// The view of a B3World of this translation unit's capacities.
__device__ __forceinline__ WorldView<B3_MAX_BODIES, B3_MAX_SHAPES, B3_MAX_CONTACTS> view_of(B3World* w) {
    WorldView<B3_MAX_BODIES, B3_MAX_SHAPES, B3_MAX_CONTACTS> v;
    v.h = w;
    v.bodies = w->bodies;
    v.shapes = w->shapes;
    v.contacts = w->contacts;
    v.joints = w->joints;
    v.cap_b = B3_MAX_BODIES;
    v.cap_s = B3_MAX_SHAPES;
    v.cap_c = B3_MAX_CONTACTS;
    v.cap_j = B3_MAX_JOINTS;
    return v;
}

__device__ __forceinline__ int clamp_count(int n, int cap) { return n < 0 ? 0 : (n > cap ? cap : n); }

// The per-world step.  Scratch (the previous step's warm cache, the padded
// shape boxes and the joint-connection bitset) lives in the thread's local
// memory, as in the reference.  Counts beyond the capacities are clamped and
// shapes or joints that name a body outside the world are inert (the
// reference would index past its arrays), so a corrupt world cannot fault.
// kArt: the articulated contact response of B3_ART_CONTACTS=1 for worlds
// with joints and contacts (b3x_art.cuh), built into the step only where it
// is asked for, since its tree takes several kilobytes of local memory.
struct NoTree {};
template <class V, bool kArt = false>
struct Stepper {
    V v;
    typename std::conditional<kArt, art::Tree<V::kB>, NoTree>::type tree;
    bool art_on;   // the articulated response resolves this step's contacts
    int nb, ns, nj;
    float h, inv_h, inv_dt;
    B3Soft cs, ss;
    int joint_iters, relax_iters;
    int flags;     // kStepInterleaveContacts | kStepSkipRestitution

    __device__ bool body_ok(int b) const { return b >= 0 && b < nb; }

    // ---- contacts: generation with warm carry (08_contacts.inl:5-39, 45-173)
    __device__ void find_contacts() {
        Carry old[V::kC];
        B3AABB box[V::kS];
        constexpr int kWords = (V::kB + 63) / 64;
        uint64_t conn[V::kB][kWords];
        const int old_n = clamp_count(v.h->contact_count, v.cap_c);
        bool sorted = true;   // strictly increasing (shape_a, shape_b): unique pairs
        for (int k = 0; k < old_n; k++) {
            const B3Contact& c = v.contacts[k];
            Carry& o = old[k];
            o.sa = c.shape_a;
            o.sb = c.shape_b;
            o.n = c.point_count;
            o.fi = c.friction_impulse;
            o.ti = c.twist_impulse;
            o.ri = c.rolling_impulse;
            for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
                if (p < o.n) {
                    o.feat[p] = c.points[p].feature;
                    o.ni[p] = c.points[p].normal_impulse;
                }
            }
            if (k > 0 && !pair_less(old[k - 1].sa, old[k - 1].sb, o.sa, o.sb)) sorted = false;
        }
        v.h->contact_count = 0;
        for (int i = 0; i < nb; i++)
            for (int k = 0; k < kWords; k++) conn[i][k] = 0ull;
        for (int i = 0; i < nj; i++) {
            const B3Joint& j = v.joints[i];
            if (j.collide_connected || !body_ok(j.body_a) || !body_ok(j.body_b)) continue;
            conn[j.body_a][j.body_b >> 6] |= 1ull << (j.body_b & 63);
            conn[j.body_b][j.body_a >> 6] |= 1ull << (j.body_a & 63);
        }
        for (int i = 0; i < ns; i++)
            if (body_ok(v.shapes[i].body)) box[i] = padded_box(shape_geo(v.bodies[v.shapes[i].body], v.shapes[i]));

        float clip[48];   // narrowphase polygon scratch (two 8-vertex polygons)
        Poly P;
        P.base = clip;
        P.stride = 1;
        int cursor = 0;   // merge cursor into the sorted old list
        for (int i = 0; i < ns; i++) {
            const B3Shape& sa = v.shapes[i];
            if (!body_ok(sa.body)) continue;
            const B3Body& ba = v.bodies[sa.body];
            for (int j = i + 1; j < ns; j++) {
                const B3Shape& sb = v.shapes[j];
                if (!body_ok(sb.body)) continue;
                const B3Body& bb = v.bodies[sb.body];
                if (sa.body == sb.body || (conn[sa.body][sb.body >> 6] >> (sb.body & 63) & 1ull)
                        || (ba.type == B3_STATIC && bb.type == B3_STATIC)
                        || (sa.category & sb.mask) == 0 || (sb.category & sa.mask) == 0 || !overlap(box[i], box[j]))
                    continue;
                Mani m;
                m_clear(m);
                collide(m, shape_geo(ba, sa), shape_geo(bb, sb), P);
                if (m.count == 0) continue;
                if (v.h->contact_count >= v.cap_c) {
                    v.h->contact_overflow = 1;
                    v.h->contacts_dropped++;
                    continue;
                }
                B3Contact& c = v.contacts[v.h->contact_count++];
                c.shape_a = i;
                c.shape_b = j;
                c.body_a = sa.body;
                c.body_b = sb.body;
                c.point_count = m.count;
                c.normal = m.normal;
                c.tangent1 = b3_perp(m.normal);
                c.tangent2 = b3_cross(c.tangent1, m.normal);
                c.friction = sqrtf(sa.friction * sb.friction);
                c.restitution = sa.restitution > sb.restitution ? sa.restitution : sb.restitution;
                c.rolling = b3_maxf(sa.rolling, sb.rolling);
                c.static_contact = ba.type != B3_DYNAMIC || bb.type != B3_DYNAMIC;
                c.friction_impulse.x = 0.0f;
                c.friction_impulse.y = 0.0f;
                c.twist_impulse = 0.0f;
                c.rolling_impulse = zero3();
                for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
                    if (p >= m.count) break;
                    B3Point& q = c.points[p];
                    q.r_a = b3_sub(m.pa[p], ba.center);
                    q.r_b = b3_sub(m.pb[p], bb.center);
                    q.base_sep = m.sep[p] - b3_dot(b3_sub(q.r_b, q.r_a), m.normal);
                    q.feature = m.feat[p];
                    q.normal_impulse = 0.0f;
                    q.total_normal = 0.0f;
                    q.rel_vel = 0.0f;
                    q.normal_mass = 0.0f;
                    q.lever = 0.0f;
                }
                // Warm carry: every old contact of the pair (the last one wins),
                // normal impulses matched by feature id (08_contacts.inl:136-171).
                // Old lists written by a step hold each pair once in increasing
                // order, so a merge cursor finds the one match.
                int k0 = 0, k1 = old_n;
                if (sorted) {
                    while (cursor < old_n && pair_less(old[cursor].sa, old[cursor].sb, i, j)) cursor++;
                    k0 = cursor;
                    k1 = cursor < old_n ? cursor + 1 : cursor;
                }
                for (int k = k0; k < k1; k++) {
                    const Carry& o = old[k];
                    if (o.sa != i || o.sb != j) continue;
                    for (int p = 0; p < c.point_count; p++)
                        for (int q = 0; q < o.n; q++)
                            if (c.points[p].feature == o.feat[q]) c.points[p].normal_impulse = o.ni[q];
                    c.friction_impulse = o.fi;
                    c.twist_impulse = o.ti;
                    c.rolling_impulse = o.ri;
                }
            }
        }
    }

    // 08_contacts.inl:234-291
    __device__ void prepare_contact(B3Contact& c) {
        const B3Body& ba = v.bodies[c.body_a];
        const B3Body& bb = v.bodies[c.body_b];
        bool da = ba.type == B3_DYNAMIC, db = bb.type == B3_DYNAMIC;
        float ma = da ? ba.inv_mass : 0.0f, mb = db ? bb.inv_mass : 0.0f;
        B3Mat3 ia = da ? ba.inv_i_world : m3_zero(), ib = db ? bb.inv_i_world : m3_zero();
        c.inv_mass_a = ma;
        c.inv_mass_b = mb;
        c.inv_i_a = ia;
        c.inv_i_b = ib;
        c.rolling_mass = m3_inv(m3_add(ia, ib));
        c.softness = c.static_contact ? ss : cs;
        const B3Vec3 n = c.normal;
        B3Vec3 ca = zero3(), cb = zero3();
        float wsum = 0.0f;
        const float inv_tau = 1.0f / B3_SPECULATIVE;
        for (int p = 0; p < c.point_count; p++) {
            B3Point& q = c.points[p];
            B3Vec3 rna = b3_cross(q.r_a, n), rnb = b3_cross(q.r_b, n);
            float kn = ma + mb + b3_dot(rna, b3_mv(ia, rna)) + b3_dot(rnb, b3_mv(ib, rnb));
            q.normal_mass = kn > 0.0f ? 1.0f / kn : 0.0f;
            B3Vec3 vra = b3_add(ba.lin_vel, b3_cross(ba.ang_vel, q.r_a));
            B3Vec3 vrb = b3_add(bb.lin_vel, b3_cross(bb.ang_vel, q.r_b));
            q.rel_vel = b3_dot(n, b3_sub(vrb, vra));
            q.total_normal = 0.0f;
            float sep = q.base_sep + b3_dot(b3_sub(q.r_b, q.r_a), n);
            float wgt = b3_clamp(2.0f - sep * inv_tau, B3_MIN_FRICTION_W, 1.0f);
            ca = b3_madd(ca, wgt, q.r_a);
            cb = b3_madd(cb, wgt, q.r_b);
            wsum += wgt;
        }
        float invw = wsum > 0.0f ? 1.0f / wsum : 0.0f;
        c.center_a = b3_mul(ca, invw);
        c.center_b = b3_mul(cb, invw);
        for (int p = 0; p < c.point_count; p++) c.points[p].lever = b3_len(b3_sub(c.points[p].r_a, c.center_a));
        B3Vec3 rta1 = b3_cross(c.center_a, c.tangent1), rta2 = b3_cross(c.center_a, c.tangent2);
        B3Vec3 rtb1 = b3_cross(c.center_b, c.tangent1), rtb2 = b3_cross(c.center_b, c.tangent2);
        B3Mat2 k;
        k.cx.x = ma + mb + b3_dot(rta1, b3_mv(ia, rta1)) + b3_dot(rtb1, b3_mv(ib, rtb1));
        k.cy.y = ma + mb + b3_dot(rta2, b3_mv(ia, rta2)) + b3_dot(rtb2, b3_mv(ib, rtb2));
        k.cx.y = k.cy.x = b3_dot(rta1, b3_mv(ia, rta2)) + b3_dot(rtb1, b3_mv(ib, rtb2));
        c.tangent_mass = m2_inv(k);
        float kt = b3_dot(n, b3_mv(m3_add(ia, ib), n));
        c.twist_mass = kt > 0.0f ? 1.0f / kt : 0.0f;
    }

    // 08_contacts.inl:293-313
    __device__ void warm_contact(const B3Contact& c) {
        B3Body& ba = v.bodies[c.body_a];
        B3Body& bb = v.bodies[c.body_b];
        const B3Vec3 n = c.normal;
        for (int p = 0; p < c.point_count; p++) {
            B3Vec3 P = b3_mul(n, c.points[p].normal_impulse);
            push(ba, c.inv_mass_a, c.inv_i_a, c.points[p].r_a, P, -1.0f);
            push(bb, c.inv_mass_b, c.inv_i_b, c.points[p].r_b, P, 1.0f);
        }
        B3Vec3 f = b3_add(b3_mul(c.tangent1, c.friction_impulse.x), b3_mul(c.tangent2, c.friction_impulse.y));
        push(ba, c.inv_mass_a, c.inv_i_a, c.center_a, f, -1.0f);
        push(bb, c.inv_mass_b, c.inv_i_b, c.center_b, f, 1.0f);
        B3Vec3 ang = b3_add(b3_mul(n, c.twist_impulse), c.rolling_impulse);
        if (dynamic_flag(ba)) ba.ang_vel = b3_sub(ba.ang_vel, b3_mv(c.inv_i_a, ang));
        if (dynamic_flag(bb)) bb.ang_vel = b3_add(bb.ang_vel, b3_mv(c.inv_i_b, ang));
    }

    // Soft-step contact rows; the relax sweep adds twist, Coulomb-disk
    // friction and rolling resistance (08_contacts.inl:315-413,
    // 07_packed.inl:24-45).
    __device__ void solve_contact(B3Contact& c, bool use_bias) {
        B3Body& ba = v.bodies[c.body_a];
        B3Body& bb = v.bodies[c.body_b];
        B3Vec3 va = ba.lin_vel, wa = ba.ang_vel, vb = bb.lin_vel, wb = bb.ang_vel;
        const B3Quat dqa = ba.delta_rot, dqb = bb.delta_rot;
        const B3Vec3 dp = b3_sub(bb.delta_pos, ba.delta_pos);
        const B3Vec3 n = c.normal;
        const float speed = v.h->contact_speed;
        float total_n = 0.0f, twist_lim = 0.0f;
        for (int p = 0; p < c.point_count; p++) {
            B3Point& q = c.points[p];
            B3Vec3 ra = q.r_a, rb = q.r_b;
            B3Vec3 ds = b3_add(dp, b3_sub(b3_rotate(dqb, rb), b3_rotate(dqa, ra)));
            float sep = b3_dot(ds, n) + q.base_sep;
            float vbias = 0.0f, mscale = 1.0f, iscale = 0.0f;
            if (sep > 0.0f) {
                vbias = sep * inv_h;
            } else if (use_bias) {
                vbias = b3_maxf(c.softness.mass_scale * c.softness.bias_rate * sep, -speed);
                mscale = c.softness.mass_scale;
                iscale = c.softness.impulse_scale;
            }
            B3Vec3 vra = b3_add(va, b3_cross(wa, ra)), vrb = b3_add(vb, b3_cross(wb, rb));
            float vn = b3_dot(b3_sub(vrb, vra), n);
            float dimp = -q.normal_mass * (mscale * vn + vbias) - iscale * q.normal_impulse;
            float nimp = b3_maxf(q.normal_impulse + dimp, 0.0f);
            dimp = nimp - q.normal_impulse;
            q.normal_impulse = nimp;
            q.total_normal += nimp;
            total_n += nimp;
            twist_lim += q.lever * q.normal_impulse;
            B3Vec3 P = b3_mul(n, dimp);
            va = b3_msub(va, c.inv_mass_a, P);
            wa = b3_sub(wa, b3_mv(c.inv_i_a, b3_cross(ra, P)));
            vb = b3_madd(vb, c.inv_mass_b, P);
            wb = b3_add(wb, b3_mv(c.inv_i_b, b3_cross(rb, P)));
        }
        if (!use_bias) {
            float max_t = c.friction * twist_lim;
            float dtw = -c.twist_mass * b3_dot(n, b3_sub(wb, wa));
            float old_t = c.twist_impulse;
            c.twist_impulse = b3_clamp(old_t + dtw, -max_t, max_t);
            dtw = c.twist_impulse - old_t;
            wa = b3_sub(wa, b3_mv(c.inv_i_a, b3_mul(n, dtw)));
            wb = b3_add(wb, b3_mv(c.inv_i_b, b3_mul(n, dtw)));

            const B3Vec3 t1 = c.tangent1, t2 = c.tangent2, ra = c.center_a, rb = c.center_b;
            B3Vec3 vr = b3_sub(b3_add(vb, b3_cross(wb, rb)), b3_add(va, b3_cross(wa, ra)));
            B3Vec2 vt;
            vt.x = b3_dot(vr, t1);
            vt.y = b3_dot(vr, t2);
            B3Vec2 tm = m2_mv(c.tangent_mass, vt);
            B3Vec2 fi;
            fi.x = c.friction_impulse.x - tm.x;
            fi.y = c.friction_impulse.y - tm.y;
            float max_f = c.friction * total_n;
            float fl2 = fi.x * fi.x + fi.y * fi.y;
            if (fl2 > max_f * max_f && fl2 > 0.0f) {
                float sc = max_f / sqrtf(fl2);
                fi.x *= sc;
                fi.y *= sc;
            }
            B3Vec2 df;
            df.x = fi.x - c.friction_impulse.x;
            df.y = fi.y - c.friction_impulse.y;
            c.friction_impulse = fi;
            B3Vec3 P = b3_add(b3_mul(t1, df.x), b3_mul(t2, df.y));
            va = b3_msub(va, c.inv_mass_a, P);
            wa = b3_sub(wa, b3_mv(c.inv_i_a, b3_cross(ra, P)));
            vb = b3_madd(vb, c.inv_mass_b, P);
            wb = b3_add(wb, b3_mv(c.inv_i_b, b3_cross(rb, P)));

            if (c.rolling > 0.0f) {
                B3Mat3 isum = m3_add(c.inv_i_a, c.inv_i_b);
                B3Mat2 k;
                k.cx.x = b3_dot(t1, b3_mv(isum, t1));
                k.cy.y = b3_dot(t2, b3_mv(isum, t2));
                k.cx.y = k.cy.x = b3_dot(t1, b3_mv(isum, t2));
                B3Vec3 wr = b3_sub(wb, wa);
                B3Vec2 rhs;
                rhs.x = b3_dot(wr, t1);
                rhs.y = b3_dot(wr, t2);
                B3Vec2 d = m2_mv(m2_inv(k), rhs);
                B3Vec3 next = b3_sub(c.rolling_impulse, b3_add(b3_mul(t1, d.x), b3_mul(t2, d.y)));
                float limit = c.rolling * total_n;
                float l2 = b3_len2(next);
                if (l2 > limit * limit && l2 > 0.0f) next = b3_mul(next, limit / sqrtf(l2));
                B3Vec3 delta = b3_sub(next, c.rolling_impulse);
                c.rolling_impulse = next;
                wa = b3_sub(wa, b3_mv(c.inv_i_a, delta));
                wb = b3_add(wb, b3_mv(c.inv_i_b, delta));
            }
        }
        store_vel(ba, va, wa);
        store_vel(bb, vb, wb);
    }

    // 08_contacts.inl:439-480
    __device__ void restitution() {
        const float threshold = v.h->restitution_threshold;
        for (int i = 0; i < v.h->contact_count; i++) {
            B3Contact& c = v.contacts[i];
            if (c.restitution == 0.0f) continue;
            B3Body& ba = v.bodies[c.body_a];
            B3Body& bb = v.bodies[c.body_b];
            B3Vec3 va = ba.lin_vel, wa = ba.ang_vel, vb = bb.lin_vel, wb = bb.ang_vel;
            const B3Vec3 n = c.normal;
            for (int p = 0; p < c.point_count; p++) {
                B3Point& q = c.points[p];
                if (q.rel_vel > -threshold || q.total_normal == 0.0f) continue;
                B3Vec3 vra = b3_add(va, b3_cross(wa, q.r_a)), vrb = b3_add(vb, b3_cross(wb, q.r_b));
                float vn = b3_dot(b3_sub(vrb, vra), n);
                float imp = -q.normal_mass * (vn + c.restitution * q.rel_vel);
                float nimp = b3_maxf(q.normal_impulse + imp, 0.0f);
                imp = nimp - q.normal_impulse;
                q.normal_impulse = nimp;
                B3Vec3 P = b3_mul(n, imp);
                va = b3_msub(va, c.inv_mass_a, P);
                wa = b3_sub(wa, b3_mv(c.inv_i_a, b3_cross(q.r_a, P)));
                vb = b3_madd(vb, c.inv_mass_b, P);
                wb = b3_add(wb, b3_mv(c.inv_i_b, b3_cross(q.r_b, P)));
            }
            store_vel(ba, va, wa);
            store_vel(bb, vb, wb);
        }
    }

    // ---- joints (06_joints.inl) ---------------------------------------------
    // 06_joints.inl:161-202
    __device__ void prepare_joint(B3Joint& j) {
        const B3Body& ba = v.bodies[j.body_a];
        const B3Body& bb = v.bodies[j.body_b];
        bool da = ba.type == B3_DYNAMIC, db = bb.type == B3_DYNAMIC;
        j.inv_mass_a = da ? ba.inv_mass : 0.0f;
        j.inv_mass_b = db ? bb.inv_mass : 0.0f;
        j.inv_i_a = da ? ba.inv_i_world : m3_zero();
        j.inv_i_b = db ? bb.inv_i_world : m3_zero();
        B3Mat3 isum = m3_add(j.inv_i_a, j.inv_i_b);
        j.fixed_rotation = b3_dot(isum.cx, b3_cross(isum.cy, isum.cz)) < 1.0e-20f;
        j.softness = make_soft(j.constraint_hertz, j.constraint_damping, h);
        j.frame_q_a = b3_qmul(ba.rotation, j.local_rot_a);
        j.frame_q_b = b3_qmul(bb.rotation, j.local_rot_b);
        j.frame_p_a = b3_rotate(ba.rotation, b3_sub(j.local_anchor_a, ba.local_center));
        j.frame_p_b = b3_rotate(bb.rotation, b3_sub(j.local_anchor_b, bb.local_center));
        j.delta_center = b3_sub(bb.center, ba.center);
        if (j.type == B3_JOINT_WELD) {
            j.angular_mass = m3_inv(isum);
            j.linear_spring = j.linear_hertz == 0.0f ? j.softness : make_soft(j.linear_hertz, j.linear_damping, h);
            j.angular_spring =
                j.angular_hertz == 0.0f ? j.softness : make_soft(j.angular_hertz, j.angular_damping, h);
        } else {
            B3Vec3 axis = b3_rotate(j.frame_q_a, b3_v(0.0f, 0.0f, 1.0f));
            float k = b3_dot(axis, b3_mv(isum, axis));
            j.axial_mass = k > 0.0f ? 1.0f / k : 0.0f;
            j.rotation_axis = axis;
            hinge_perps(j.frame_q_a, b3_qinv_mul(j.frame_q_a, j.frame_q_b), &j.perp_x, &j.perp_y);
            j.spring_softness = make_soft(j.hertz, j.damping_ratio, h);
        }
    }

    // 06_joints.inl:204-239
    __device__ void warm_joint(const B3Joint& j) {
        B3Body& ba = v.bodies[j.body_a];
        B3Body& bb = v.bodies[j.body_b];
        B3Vec3 ra = b3_rotate(ba.delta_rot, j.frame_p_a);
        B3Vec3 rb = b3_rotate(bb.delta_rot, j.frame_p_b);
        B3Vec3 ang = j.angular_impulse;
        if (j.type == B3_JOINT_REVOLUTE) {
            float axial = j.spring_impulse + j.motor_impulse + j.lower_impulse - j.upper_impulse;
            ang = b3_add(b3_mul(j.perp_x, j.perp_impulse.x), b3_mul(j.perp_y, j.perp_impulse.y));
            ang = b3_madd(ang, axial, j.rotation_axis);
        }
        if (dynamic_flag(ba)) {
            ba.lin_vel = b3_msub(ba.lin_vel, j.inv_mass_a, j.linear_impulse);
            ba.ang_vel = b3_sub(ba.ang_vel, b3_mv(j.inv_i_a, b3_add(b3_cross(ra, j.linear_impulse), ang)));
        }
        if (dynamic_flag(bb)) {
            bb.lin_vel = b3_madd(bb.lin_vel, j.inv_mass_b, j.linear_impulse);
            bb.ang_vel = b3_add(bb.ang_vel, b3_mv(j.inv_i_b, b3_add(b3_cross(rb, j.linear_impulse), ang)));
        }
    }

    // Three-row point constraint (06_joints.inl:241-282).
    __device__ void solve_point(B3Joint& j, const B3Body& ba, const B3Body& bb, B3Vec3& va, B3Vec3& wa,
                                B3Vec3& vb, B3Vec3& wb, B3Soft soft, bool use_bias) {
        B3Vec3 ra = b3_rotate(ba.delta_rot, j.frame_p_a);
        B3Vec3 rb = b3_rotate(bb.delta_rot, j.frame_p_b);
        B3Vec3 cdot = b3_sub(b3_add(vb, b3_cross(wb, rb)), b3_add(va, b3_cross(wa, ra)));
        B3Vec3 bias = zero3();
        float mscale = 1.0f, iscale = 0.0f;
        if (use_bias) {
            B3Vec3 sep = b3_add(b3_add(b3_sub(bb.delta_pos, ba.delta_pos), b3_sub(rb, ra)), j.delta_center);
            bias = b3_mul(sep, soft.bias_rate);
            mscale = soft.mass_scale;
            iscale = soft.impulse_scale;
        }
        const float msum = j.inv_mass_a + j.inv_mass_b;
        B3Mat3 k;
        k.cx = b3_v(msum, 0.0f, 0.0f);
        k.cy = b3_v(0.0f, msum, 0.0f);
        k.cz = b3_v(0.0f, 0.0f, msum);
        k.cx = b3_sub(k.cx, b3_cross(ra, b3_mv(j.inv_i_a, b3_v(0.0f, ra.z, -ra.y))));
        k.cy = b3_sub(k.cy, b3_cross(ra, b3_mv(j.inv_i_a, b3_v(-ra.z, 0.0f, ra.x))));
        k.cz = b3_sub(k.cz, b3_cross(ra, b3_mv(j.inv_i_a, b3_v(ra.y, -ra.x, 0.0f))));
        k.cx = b3_sub(k.cx, b3_cross(rb, b3_mv(j.inv_i_b, b3_v(0.0f, rb.z, -rb.y))));
        k.cy = b3_sub(k.cy, b3_cross(rb, b3_mv(j.inv_i_b, b3_v(-rb.z, 0.0f, rb.x))));
        k.cz = b3_sub(k.cz, b3_cross(rb, b3_mv(j.inv_i_b, b3_v(rb.y, -rb.x, 0.0f))));
        B3Vec3 b = b3_mv(m3_inv(k), b3_add(cdot, bias));
        B3Vec3 impulse = b3_msub(b3_mul(b, -mscale), iscale, j.linear_impulse);
        j.linear_impulse = b3_add(j.linear_impulse, impulse);
        va = b3_msub(va, j.inv_mass_a, impulse);
        wa = b3_sub(wa, b3_mv(j.inv_i_a, b3_cross(ra, impulse)));
        vb = b3_madd(vb, j.inv_mass_b, impulse);
        wb = b3_add(wb, b3_mv(j.inv_i_b, b3_cross(rb, impulse)));
    }

    // 06_joints.inl:285-332
    __device__ void solve_weld(B3Joint& j, bool use_bias) {
        B3Body& ba = v.bodies[j.body_a];
        B3Body& bb = v.bodies[j.body_b];
        B3Vec3 va = ba.lin_vel, wa = ba.ang_vel, vb = bb.lin_vel, wb = bb.ang_vel;
        B3Quat qa = b3_qmul(ba.delta_rot, j.frame_q_a);
        B3Quat qb = b3_qmul(bb.delta_rot, j.frame_q_b);
        if (b3_qdot(qa, qb) < 0.0f) qb = b3_qneg(qb);
        B3Quat rel = b3_qinv_mul(qa, qb);
        if (!j.fixed_rotation) {
            B3Vec3 bias = zero3();
            float mscale = 1.0f, iscale = 0.0f;
            if (use_bias || j.angular_hertz > 0.0f) {
                B3Quat s = rel.s < 0.0f ? b3_qneg(rel) : rel;
                B3Quat diff = b3_q(-s.v.x, -s.v.y, -s.v.z, 1.0f - s.s);
                B3Vec3 c = b3_neg(b3_rotate(qa, b3_mul(b3_qmul(diff, b3_qconj(s)).v, 2.0f)));
                bias = b3_mul(c, j.angular_spring.bias_rate);
                mscale = j.angular_spring.mass_scale;
                iscale = j.angular_spring.impulse_scale;
            }
            B3Vec3 cdot = b3_sub(wb, wa);
            B3Vec3 impulse =
                b3_msub(b3_mul(b3_mv(j.angular_mass, b3_add(cdot, bias)), -mscale), iscale, j.angular_impulse);
            j.angular_impulse = b3_add(j.angular_impulse, impulse);
            wa = b3_sub(wa, b3_mv(j.inv_i_a, impulse));
            wb = b3_add(wb, b3_mv(j.inv_i_b, impulse));
        }
        solve_point(j, ba, bb, va, wa, vb, wb, j.linear_spring, use_bias || j.linear_hertz > 0.0f);
        store_vel(ba, va, wa);
        store_vel(bb, vb, wb);
    }

    // One-sided limit row (06_joints.inl:419-434).
    __device__ static float limit_row(float c, float cdot, float inv_h, bool use_bias, B3Soft soft, float mass,
                                      float old) {
        float bias = 0.0f, mscale = 1.0f, iscale = 0.0f;
        if (c > 0.0f) {
            bias = c * inv_h;
        } else if (use_bias) {
            bias = soft.bias_rate * c;
            mscale = soft.mass_scale;
            iscale = soft.impulse_scale;
        }
        float dimp = -mscale * mass * (cdot + bias) - iscale * old;
        return b3_maxf(old + dimp, 0.0f);
    }

    // Spring, motor, limits, perpendicular rows, point (06_joints.inl:436-642).
    __device__ void solve_revolute(B3Joint& j, bool use_bias) {
        B3Body& ba = v.bodies[j.body_a];
        B3Body& bb = v.bodies[j.body_b];
        B3Vec3 va = ba.lin_vel, wa = ba.ang_vel, vb = bb.lin_vel, wb = bb.ang_vel;
        B3Quat qa = b3_qmul(ba.delta_rot, j.frame_q_a);
        B3Quat qb = b3_qmul(bb.delta_rot, j.frame_q_b);
        if (b3_qdot(qa, qb) < 0.0f) qb = b3_qneg(qb);
        B3Quat rel = b3_qinv_mul(qa, qb);
        const B3Vec3 axis = j.rotation_axis;
        const bool free_rot = !j.fixed_rotation;
        B3Vec3 ia_ax = zero3(), ib_ax = zero3();
        if (free_rot) {
            ia_ax = b3_mv(j.inv_i_a, axis);
            ib_ax = b3_mv(j.inv_i_b, axis);
        }
        float twist = 0.0f;
        if ((j.enable_spring || j.enable_limit || j.enable_motor) && free_rot) twist = b3_twist(rel);
        if (j.enable_spring && free_rot) {
            float c = twist - j.target_angle;
            float cdot = b3_dot(b3_sub(wb, wa), axis);
            float dimp = -j.spring_softness.mass_scale * j.axial_mass * (cdot + j.spring_softness.bias_rate * c)
                         - j.spring_softness.impulse_scale * j.spring_impulse;
            float old = j.spring_impulse;
            float nimp = old + dimp;
            if (j.max_motor_torque > 0.0f) {
                float maxp = j.max_motor_torque * h;
                nimp = b3_clamp(nimp, -maxp, maxp);
            }
            dimp = nimp - old;
            j.spring_impulse = nimp;
            wa = b3_msub(wa, dimp, ia_ax);
            wb = b3_madd(wb, dimp, ib_ax);
        }
        if (j.enable_motor && free_rot) {
            bool blocked = false;
            if (j.enable_limit) {
                if (twist >= j.upper_angle - 0.01f && j.motor_speed > 0.0f) blocked = true;
                if (twist <= j.lower_angle + 0.01f && j.motor_speed < 0.0f) blocked = true;
            }
            if (blocked) {
                j.motor_impulse = 0.0f;
            } else {
                float cdot = b3_dot(b3_sub(wb, wa), axis) - j.motor_speed;
                float dimp = -j.axial_mass * cdot;
                float maxp = j.max_motor_torque * h;
                float nimp = b3_clamp(j.motor_impulse + dimp, -maxp, maxp);
                dimp = nimp - j.motor_impulse;
                j.motor_impulse = nimp;
                wa = b3_msub(wa, dimp, ia_ax);
                wb = b3_madd(wb, dimp, ib_ax);
            }
        }
        if (j.enable_limit && free_rot) {
            float old = j.lower_impulse;
            j.lower_impulse = limit_row(twist - j.lower_angle, b3_dot(b3_sub(wb, wa), axis), inv_h, use_bias,
                                        j.softness, j.axial_mass, old);
            float dimp = j.lower_impulse - old;
            wa = b3_msub(wa, dimp, ia_ax);
            wb = b3_madd(wb, dimp, ib_ax);
            old = j.upper_impulse;
            j.upper_impulse = limit_row(j.upper_angle - twist, b3_dot(b3_sub(wa, wb), axis), inv_h, use_bias,
                                        j.softness, j.axial_mass, old);
            dimp = j.upper_impulse - old;
            wa = b3_madd(wa, dimp, ia_ax);
            wb = b3_msub(wb, dimp, ib_ax);
        }
        if (free_rot) {
            B3Vec2 bias;
            bias.x = 0.0f;
            bias.y = 0.0f;
            float mscale = 1.0f, iscale = 0.0f;
            if (use_bias) {
                bias.x = j.softness.bias_rate * rel.v.x;
                bias.y = j.softness.bias_rate * rel.v.y;
                mscale = j.softness.mass_scale;
                iscale = j.softness.impulse_scale;
            }
            B3Vec3 px, py;
            hinge_perps(qa, rel, &px, &py);
            j.perp_x = px;
            j.perp_y = py;
            B3Mat3 isum = m3_add(j.inv_i_a, j.inv_i_b);
            B3Mat2 k;
            k.cx.x = b3_dot(px, b3_mv(isum, px));
            k.cy.y = b3_dot(py, b3_mv(isum, py));
            k.cx.y = k.cy.x = b3_dot(px, b3_mv(isum, py));
            B3Vec3 wrel = b3_sub(wb, wa);
            B3Vec2 rhs;
            rhs.x = b3_dot(wrel, px) + bias.x;
            rhs.y = b3_dot(wrel, py) + bias.y;
            B3Vec2 sol = solve2(k, rhs);
            B3Vec2 d;
            d.x = -mscale * sol.x - iscale * j.perp_impulse.x;
            d.y = -mscale * sol.y - iscale * j.perp_impulse.y;
            j.perp_impulse.x += d.x;
            j.perp_impulse.y += d.y;
            B3Vec3 ang = b3_add(b3_mul(px, d.x), b3_mul(py, d.y));
            wa = b3_sub(wa, b3_mv(j.inv_i_a, ang));
            wb = b3_add(wb, b3_mv(j.inv_i_b, ang));
        }
        solve_point(j, ba, bb, va, wa, vb, wb, j.softness, use_bias);
        store_vel(ba, va, wa);
        store_vel(bb, vb, wb);
    }

    // Joint sweeps in joint index order (07_packed.inl:48-81).
    __device__ bool joint_ok(const B3Joint& j) const { return body_ok(j.body_a) && body_ok(j.body_b); }

    __device__ void solve_joints(bool use_bias, int iters, bool interleave) {
        for (int it = 0; it < iters; it++) {
            if (interleave) solve_contacts(use_bias);
            for (int i = 0; i < nj; i++) {
                B3Joint& j = v.joints[i];
                if (!joint_ok(j)) continue;
                if (j.type == B3_JOINT_WELD) solve_weld(j, use_bias);
                else solve_revolute(j, use_bias);
            }
        }
    }

    __device__ void solve_contacts(bool use_bias) {
        if constexpr (kArt) {
            if (art_on) {
                tree.solve_contacts(v.bodies, v.contacts, v.h->contact_count, inv_h, v.h->contact_speed, use_bias);
                return;
            }
        }
        for (int i = 0; i < v.h->contact_count; i++) solve_contact(v.contacts[i], use_bias);
    }

    // ---- integration (09_step.inl:5-130) ---------------------------------------
    __device__ void integrate_velocities() {
#if B3_HAS_USER_FORCES
        // the per-substep force hook of the including translation unit: its
        // contributions act for this substep only (09_step.inl:20-53)
        B3Vec3 saved_f[V::kB], saved_t[V::kB];
        for (int i = 0; i < nb; i++) {
            saved_f[i] = v.bodies[i].force;
            saved_t[i] = v.bodies[i].torque;
        }
        B3_USER_FORCES(v.h, h);
#endif
        for (int i = 0; i < nb; i++) {
            B3Body& b = v.bodies[i];
            if (b.type != B3_DYNAMIC) continue;
            float ld = 1.0f / (1.0f + h * b.linear_damping);
            float ad = 1.0f / (1.0f + h * b.angular_damping);
            float gs = b.inv_mass > 0.0f ? b.gravity_scale : 0.0f;
            B3Vec3 dv = b3_add(b3_mul(b.force, h * b.inv_mass), b3_mul(v.h->gravity, h * gs));
            b.lin_vel = b3_madd(dv, ld, b.lin_vel);
            b.ang_vel = b3_madd(b3_mul(b3_mv(b.inv_i_world, b.torque), h), ad, b.ang_vel);
        }
#if B3_HAS_USER_FORCES
        for (int i = 0; i < nb; i++) {
            v.bodies[i].force = saved_f[i];
            v.bodies[i].torque = saved_t[i];
        }
#endif
    }

    __device__ void integrate_positions() {
        const float max_lin = v.h->max_linear_speed;
        const float max_ang = B3_MAX_ROTATION * inv_dt;
        const float max_lin2 = max_lin * max_lin, max_ang2 = max_ang * max_ang;
        for (int i = 0; i < nb; i++) {
            B3Body& b = v.bodies[i];
            if (b.type == B3_STATIC) continue;
            B3Vec3 v = b.lin_vel, av = b.ang_vel;
            const uint32_t f = b.flags;
            if (f & B3_LOCK_LIN_X) v.x = 0.0f;
            if (f & B3_LOCK_LIN_Y) v.y = 0.0f;
            if (f & B3_LOCK_LIN_Z) v.z = 0.0f;
            if (f & B3_LOCK_ANG_X) av.x = 0.0f;
            if (f & B3_LOCK_ANG_Y) av.y = 0.0f;
            if (f & B3_LOCK_ANG_Z) av.z = 0.0f;
            float v2 = b3_len2(v);
            if (v2 > max_lin2 && v2 > 0.0f) v = b3_mul(v, max_lin / sqrtf(v2));
            float w2 = b3_len2(av);
            if (w2 > max_ang2 && w2 > 0.0f) av = b3_mul(av, max_ang / sqrtf(w2));
            b.lin_vel = v;
            b.ang_vel = av;
            b.delta_pos = b3_madd(b.delta_pos, h, v);
            b.delta_rot = q_integrate(b.delta_rot, b3_mul(av, h));
        }
    }

    __device__ void finalize() {
        for (int i = 0; i < nb; i++) {
            B3Body& b = v.bodies[i];
            if (b.type == B3_STATIC) continue;
            b.center = b3_add(b.center, b.delta_pos);
            b.rotation = b3_qnorm(b3_qmul(b.delta_rot, b.rotation));
            b.position = b3_sub(b.center, b3_rotate(b.rotation, b.local_center));
            b.delta_pos = zero3();
            b.delta_rot = b3_q_id();
            b.force = zero3();
            b.torque = zero3();
            if (b.type == B3_DYNAMIC) b.inv_i_world = b3_world_inv_i(b.rotation, b.inv_inertia);
        }
    }

    __device__ void run(int subs) {
        find_contacts();
        for (int i = 0; i < v.h->contact_count; i++) prepare_contact(v.contacts[i]);
        for (int i = 0; i < nj; i++)
            if (joint_ok(v.joints[i])) prepare_joint(v.joints[i]);
        // B3_ART_CONTACTS=1: worlds with joints and contacts whose revolute
        // joints span a tree warm start and solve contacts through it
        // (08_contacts.inl:194-232, 424-436)
        art_on = false;
        if constexpr (kArt) art_on = nj > 0 && v.h->contact_count > 0 && tree.build(v.bodies, nb, v.joints, nj);
        if constexpr (kArt) {
            if (art_on) tree.warm_start(v.bodies, v.contacts, v.h->contact_count);
        }
        if (!art_on)
            for (int i = 0; i < v.h->contact_count; i++) warm_contact(v.contacts[i]);
        for (int i = 0; i < nj; i++)
            if (joint_ok(v.joints[i])) warm_joint(v.joints[i]);
        const bool interleave = (flags & kStepInterleaveContacts) != 0;
        for (int s = 0; s < subs; s++) {
            // 09_step.inl:167-181; interleaved, a contact sweep opens every
            // joint iteration (07_packed.inl:61-65)
            integrate_velocities();
            if (!interleave) solve_contacts(true);
            solve_joints(true, joint_iters, interleave);
            integrate_positions();
            if (!interleave) solve_contacts(false);
            solve_joints(false, relax_iters, interleave);
            if (!(flags & kStepSkipRestitution)) restitution();
        }
        finalize();
    }
};

// b3_step_indep (09_step.inl:183-258) of the world a view addresses, with
// run-time solver iteration counts.
template <class V, bool kArt = false>
__device__ inline void step_view(const V& v, float dt, int substeps, int joint_iters, int relax_iters,
                                 int flags = 0) {
    if (dt <= 0.0f) return;
    const int subs = substeps < 1 ? 1 : substeps;
    Stepper<V, kArt> st;
    st.v = v;
    st.nb = clamp_count(v.h->body_count, v.cap_b < V::kB ? v.cap_b : V::kB);
    st.ns = clamp_count(v.h->shape_count, v.cap_s < V::kS ? v.cap_s : V::kS);
    st.nj = clamp_count(v.h->joint_count, v.cap_j);
    st.joint_iters = joint_iters;
    st.relax_iters = relax_iters;
    st.flags = flags;
    // b3_soft_step_params (09_step.inl:148-157)
    st.h = dt / (float)subs;
    st.inv_dt = 1.0f / dt;
    st.inv_h = (float)subs * st.inv_dt;
    float hertz = b3_minf(v.h->contact_hertz, 0.25f * st.inv_h);
    st.cs = make_soft(hertz, v.h->contact_damping, st.h);
    st.ss = make_soft(2.0f * hertz, 0.5f * v.h->contact_damping, st.h);
    st.run(subs);
}

// b3_step_indep on a B3World of this translation unit's capacities (kArt:
// with the B3_ART_CONTACTS=1 contact response).
template <bool kArt = false>
__device__ inline void step_world(B3World* w, float dt, int substeps, int joint_iters, int relax_iters,
                                  int flags = 0) {
    step_view<decltype(view_of(w)), kArt>(view_of(w), dt, substeps, joint_iters, relax_iters, flags);
}

}  // namespace one
}  // namespace b3x
#endif  // __CUDACC__
