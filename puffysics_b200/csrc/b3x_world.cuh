// b3x_world.cuh -- one world, one step: the per-thread body of the step
// kernel (b3x_step.cu), in lane-interleaved working columns.
//
// Mapping and arithmetic are described in b3x_step.cu.  Functions are
// __host__ __device__ only so that the same source can also be compiled for
// the host by development tools; the library runs them on the GPU alone.
#pragma once
#include <cstdint>
#include <cstring>

#include "puffysics_b200.h"
#include "b3x_math.cuh"
#include "b3x_narrow.cuh"

namespace b3x {

constexpr int kLanes = 32;

// ---- working-set field indices (words) -----------------------------------
// body columns
enum : int { BV = 0, BW = 3, BDP = 6, BDQ = 9, BMI = 13, BII = 14, BFLAGS = 23, BTYPE = 24, NBF = 25 };
// shape columns
enum : int { SPOS = 0, SROT = 3, SLO = 7, SHI = 10, NSF = 13 };
// contact columns; point p occupies CP + p * NPF ...
enum : int {
    CSA = 0, CSB = 1, CBA = 2, CBB = 3, CCNT = 4, CSTAT = 5, CN = 6, CT1 = 9, CT2 = 12, CCA = 15, CCB = 18,
    CFRIC = 21, CREST = 22, CROLL = 23, CTWM = 24, CTWI = 25, CFI = 26, CRI = 28, CTM = 31, CP = 35,
    PRA = 0, PRB = 3, PBSEP = 6, PRELV = 7, PNI = 8, PTOT = 9, PNM = 10, PLEV = 11, PFEAT = 12, NPF = 13,
    NCF = CP + B3_MAX_MANIFOLD * NPF
};
// joint columns
enum : int {
    JTYPE = 0, JBA = 1, JBB = 2, JFIX = 3, JENS = 4, JENM = 5, JENL = 6, JFPA = 7, JFPB = 10, JFQA = 13,
    JFQB = 17, JDC = 21, JSOFT = 24, JLI = 27, JAI = 30, JAM = 33, JLH = 42, JAH = 43, JLS = 44, JAS = 47,
    JPI = 50, JSI = 52, JMI = 53, JLOI = 54, JUPI = 55, JMMT = 56, JMS = 57, JTA = 58, JLA = 59, JUA = 60,
    JAX = 61, JPX = 64, JPY = 67, JAXM = 70, JSS = 71, JOK = 74, NJF = 75
};

// World header (the first 68 bytes of B3World, reference 02_types.inl:306-327).
struct Header {
    B3Vec3 gravity;
    float contact_hertz, contact_damping, contact_speed, restitution_threshold, max_linear_speed;
    int body_count, shape_count, contact_count, joint_count;
    int body_overflow, shape_overflow, joint_overflow, contact_overflow, contacts_dropped;
};
static_assert(sizeof(Header) == B3X_WORLD_HEADER_BYTES, "header layout");

// Run-time world layout decoded from the capacity signature.
struct Layout {
    int B, S, C, J;
    unsigned shape_off, contact_off, joint_off, size;
};

static bool layout_from_signature(unsigned long long sig, Layout* L) {
    long B = (long)(sig & 0xffff), S = (long)((sig >> 16) & 0xffff);
    long C = (long)((sig >> 32) & 0xffff), J = (long)((sig >> 48) & 0xffff);
    if (B < 1 || S < 1 || C < 1 || J < 1) return false;
    unsigned long shape_off = B3X_WORLD_HEADER_BYTES + (unsigned long)B3X_BODY_BYTES * B;
    shape_off = (shape_off + 7) & ~7ul;
    unsigned long contact_off = shape_off + (unsigned long)B3X_SHAPE_BYTES * S;
    unsigned long joint_off = contact_off + (unsigned long)B3X_CONTACT_BYTES * C;
    unsigned long size = (joint_off + (unsigned long)B3X_JOINT_BYTES * J + 7) & ~7ul;
    L->B = (int)B; L->S = (int)S; L->C = (int)C; L->J = (int)J;
    L->shape_off = (unsigned)shape_off; L->contact_off = (unsigned)contact_off;
    L->joint_off = (unsigned)joint_off; L->size = (unsigned)size;
    return true;
}

struct StepArgs {
    unsigned char* data;
    unsigned long long stride, offset;
    int count;
    const unsigned char* active;
    float dt;
    int substeps, joint_iters, relax_iters;
    Layout L;
    float* scratch;
    unsigned long long slot_words;    // words per CTA slot
    unsigned off_bodies, off_shapes, off_contacts, off_joints;   // word offsets inside a slot
};

// ---- lane-column accessors -------------------------------------------------
#define COL(c, i) ((c)[(size_t)(i) * kLanes])

B3X_HDI B3Vec3 ld3(const float* c, int i) { return b3_v(COL(c, i), COL(c, i + 1), COL(c, i + 2)); }
B3X_HDI void st3(float* c, int i, B3Vec3 v) { COL(c, i) = v.x; COL(c, i + 1) = v.y; COL(c, i + 2) = v.z; }
B3X_HDI B3Quat ldq(const float* c, int i) { return b3_q(COL(c, i), COL(c, i + 1), COL(c, i + 2), COL(c, i + 3)); }
B3X_HDI void stq(float* c, int i, B3Quat q) { st3(c, i, q.v); COL(c, i + 3) = q.s; }
B3X_HDI B3Mat3 ldm(const float* c, int i) {
    B3Mat3 m;
    m.cx = ld3(c, i); m.cy = ld3(c, i + 3); m.cz = ld3(c, i + 6);
    return m;
}
B3X_HDI void stm(float* c, int i, B3Mat3 m) { st3(c, i, m.cx); st3(c, i + 3, m.cy); st3(c, i + 6, m.cz); }
B3X_HDI B3Soft lds(const float* c, int i) { B3Soft s; s.bias_rate = COL(c, i); s.mass_scale = COL(c, i + 1); s.impulse_scale = COL(c, i + 2); return s; }
B3X_HDI void sts(float* c, int i, B3Soft s) { COL(c, i) = s.bias_rate; COL(c, i + 1) = s.mass_scale; COL(c, i + 2) = s.impulse_scale; }
B3X_HDI int ldi(const float* c, int i) { return b3x_f2i(COL(c, i)); }
B3X_HDI void sti(float* c, int i, int v) { COL(c, i) = b3x_i2f(v); }

B3X_HDI int BI(int k, int f) { return k * NBF + f; }
B3X_HDI int SI(int k, int f) { return k * NSF + f; }
B3X_HDI int CI(int k, int f) { return k * NCF + f; }
B3X_HDI int PI(int k, int p, int f) { return k * NCF + CP + p * NPF + f; }
B3X_HDI int JI(int k, int f) { return k * NJF + f; }

B3X_HDI int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Body velocity write-back gated by the dynamic flag (the reference writes a
// solved body only when flags has B3_FLAG_DYNAMIC, 08_contacts.inl:405-412).
B3X_HDI void put_vel(float* bc, int k, B3Vec3 v, B3Vec3 w) {
    if (b3x_f2u(COL(bc, BI(k, BFLAGS))) & B3_FLAG_DYNAMIC) {
        st3(bc, BI(k, BV), v);
        st3(bc, BI(k, BW), w);
    }
}

// 08_contacts.inl:184-192
B3X_HDI void apply_impulse(float* bc, int k, float m, const B3Mat3& i, B3Vec3 r, B3Vec3 p, int sign) {
    if ((b3x_f2u(COL(bc, BI(k, BFLAGS))) & B3_FLAG_DYNAMIC) == 0) return;
    float s = sign > 0 ? 1.0f : -1.0f;
    st3(bc, BI(k, BV), b3_madd(ld3(bc, BI(k, BV)), s * m, p));
    st3(bc, BI(k, BW), b3_add(ld3(bc, BI(k, BW)), b3_mv(i, b3_mul(b3_cross(r, p), s))));
}

// ---- contact sweep (08_contacts.inl:315-413, rolling 07_packed.inl:24-45) --
B3X_HD void solve_contact(float* bc, float* cc, int k, float inv_h, float speed, int use_bias, B3Soft cs,
        B3Soft ss) {
    int ba = ldi(cc, CI(k, CBA)), bb = ldi(cc, CI(k, CBB));
    int cnt = ldi(cc, CI(k, CCNT));
    B3Soft soft = ldi(cc, CI(k, CSTAT)) ? ss : cs;
    float ma = COL(bc, BI(ba, BMI)), mb = COL(bc, BI(bb, BMI));
    B3Mat3 ia = ldm(bc, BI(ba, BII)), ib = ldm(bc, BI(bb, BII));
    B3Vec3 va = ld3(bc, BI(ba, BV)), wa = ld3(bc, BI(ba, BW));
    B3Vec3 vb = ld3(bc, BI(bb, BV)), wb = ld3(bc, BI(bb, BW));
    B3Quat dqa = ldq(bc, BI(ba, BDQ)), dqb = ldq(bc, BI(bb, BDQ));
    B3Vec3 dp = b3_sub(ld3(bc, BI(bb, BDP)), ld3(bc, BI(ba, BDP)));
    B3Vec3 n = ld3(cc, CI(k, CN));
    float total_n = 0.0f, twist_lim = 0.0f;
    for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
        if (p >= cnt) break;
        B3Vec3 ra = ld3(cc, PI(k, p, PRA)), rb = ld3(cc, PI(k, p, PRB));
        B3Vec3 ds = b3_add(dp, b3_sub(b3_rotate(dqb, rb), b3_rotate(dqa, ra)));
        float sep = b3_dot(ds, n) + COL(cc, PI(k, p, PBSEP));
        float vbias = 0.0f, mscale = 1.0f, iscale = 0.0f;
        if (sep > 0.0f) {
            vbias = sep * inv_h;
        } else if (use_bias) {
            vbias = b3_maxf(soft.mass_scale * soft.bias_rate * sep, -speed);
            mscale = soft.mass_scale;
            iscale = soft.impulse_scale;
        }
        B3Vec3 vra = b3_add(va, b3_cross(wa, ra)), vrb = b3_add(vb, b3_cross(wb, rb));
        float vn = b3_dot(b3_sub(vrb, vra), n);
        float ni = COL(cc, PI(k, p, PNI));
        float dimp = -COL(cc, PI(k, p, PNM)) * (mscale * vn + vbias) - iscale * ni;
        float nimp = b3_maxf(ni + dimp, 0.0f);
        dimp = nimp - ni;
        COL(cc, PI(k, p, PNI)) = nimp;
        COL(cc, PI(k, p, PTOT)) = COL(cc, PI(k, p, PTOT)) + nimp;
        total_n += nimp;
        twist_lim += COL(cc, PI(k, p, PLEV)) * nimp;
        B3Vec3 P = b3_mul(n, dimp);
        va = b3_msub(va, ma, P);
        wa = b3_sub(wa, b3_mv(ia, b3_cross(ra, P)));
        vb = b3_madd(vb, mb, P);
        wb = b3_add(wb, b3_mv(ib, b3_cross(rb, P)));
    }
    if (!use_bias) {
        float fric = COL(cc, CI(k, CFRIC));
        float twist_s = b3_dot(n, b3_sub(wb, wa));
        float max_t = fric * twist_lim;
        float dtw = -COL(cc, CI(k, CTWM)) * twist_s;
        float old_t = COL(cc, CI(k, CTWI));
        float new_t = b3_clamp(old_t + dtw, -max_t, max_t);
        COL(cc, CI(k, CTWI)) = new_t;
        dtw = new_t - old_t;
        wa = b3_sub(wa, b3_mv(ia, b3_mul(n, dtw)));
        wb = b3_add(wb, b3_mv(ib, b3_mul(n, dtw)));

        B3Vec3 t1 = ld3(cc, CI(k, CT1)), t2 = ld3(cc, CI(k, CT2));
        B3Vec3 ra = ld3(cc, CI(k, CCA)), rb = ld3(cc, CI(k, CCB));
        B3Vec3 vra = b3_add(va, b3_cross(wa, ra)), vrb = b3_add(vb, b3_cross(wb, rb));
        B3Vec3 vr = b3_sub(vrb, vra);
        B3Vec2 vt;
        vt.x = b3_dot(vr, t1);
        vt.y = b3_dot(vr, t2);
        B3Mat2 tm;
        tm.cx.x = COL(cc, CI(k, CTM)); tm.cx.y = COL(cc, CI(k, CTM + 1));
        tm.cy.x = COL(cc, CI(k, CTM + 2)); tm.cy.y = COL(cc, CI(k, CTM + 3));
        B3Vec2 tv = m2_mv(tm, vt);
        B3Vec2 fi;
        fi.x = COL(cc, CI(k, CFI));
        fi.y = COL(cc, CI(k, CFI + 1));
        B3Vec2 ni;
        ni.x = fi.x - tv.x;
        ni.y = fi.y - tv.y;
        float max_f = fric * total_n;
        float fl2 = ni.x * ni.x + ni.y * ni.y;
        if (fl2 > max_f * max_f && fl2 > 0.0f) {
            float sc = max_f / sqrtf(fl2);
            ni.x *= sc;
            ni.y *= sc;
        }
        B3Vec2 df;
        df.x = ni.x - fi.x;
        df.y = ni.y - fi.y;
        COL(cc, CI(k, CFI)) = ni.x;
        COL(cc, CI(k, CFI + 1)) = ni.y;
        B3Vec3 P = b3_add(b3_mul(t1, df.x), b3_mul(t2, df.y));
        va = b3_msub(va, ma, P);
        wa = b3_sub(wa, b3_mv(ia, b3_cross(ra, P)));
        vb = b3_madd(vb, mb, P);
        wb = b3_add(wb, b3_mv(ib, b3_cross(rb, P)));

        float rolling = COL(cc, CI(k, CROLL));
        if (rolling > 0.0f) {
            B3Mat3 isum = m3_add(ia, ib);
            B3Mat2 kr;
            kr.cx.x = b3_dot(t1, b3_mv(isum, t1));
            kr.cy.y = b3_dot(t2, b3_mv(isum, t2));
            kr.cx.y = kr.cy.x = b3_dot(t1, b3_mv(isum, t2));
            B3Vec3 wr = b3_sub(wb, wa);
            B3Vec2 rhs;
            rhs.x = b3_dot(wr, t1);
            rhs.y = b3_dot(wr, t2);
            B3Vec2 dd = m2_mv(m2_inv(kr), rhs);
            B3Vec3 imp = ld3(cc, CI(k, CRI));
            B3Vec3 next = b3_sub(imp, b3_add(b3_mul(t1, dd.x), b3_mul(t2, dd.y)));
            float limit = rolling * total_n;
            float l2 = b3_len2(next);
            if (l2 > limit * limit && l2 > 0.0f) next = b3_mul(next, limit / sqrtf(l2));
            B3Vec3 delta = b3_sub(next, imp);
            st3(cc, CI(k, CRI), next);
            wa = b3_sub(wa, b3_mv(ia, delta));
            wb = b3_add(wb, b3_mv(ib, delta));
        }
    }
    put_vel(bc, ba, va, wa);
    put_vel(bc, bb, vb, wb);
}

// ---- joints (06_joints.inl:241-642) ---------------------------------------
B3X_HDI B3Mat3 point_k(float ma, float mb, const B3Mat3& ia, const B3Mat3& ib, B3Vec3 ra, B3Vec3 rb) {
    float msum = ma + mb;
    B3Mat3 k;
    k.cx = b3_v(msum, 0.0f, 0.0f);
    k.cy = b3_v(0.0f, msum, 0.0f);
    k.cz = b3_v(0.0f, 0.0f, msum);
    k.cx = b3_sub(k.cx, b3_cross(ra, b3_mv(ia, b3_v(0.0f, ra.z, -ra.y))));
    k.cy = b3_sub(k.cy, b3_cross(ra, b3_mv(ia, b3_v(-ra.z, 0.0f, ra.x))));
    k.cz = b3_sub(k.cz, b3_cross(ra, b3_mv(ia, b3_v(ra.y, -ra.x, 0.0f))));
    k.cx = b3_sub(k.cx, b3_cross(rb, b3_mv(ib, b3_v(0.0f, rb.z, -rb.y))));
    k.cy = b3_sub(k.cy, b3_cross(rb, b3_mv(ib, b3_v(-rb.z, 0.0f, rb.x))));
    k.cz = b3_sub(k.cz, b3_cross(rb, b3_mv(ib, b3_v(rb.y, -rb.x, 0.0f))));
    return k;
}

// 06_joints.inl:257-282
B3X_HDI void solve_point(float* bc, float* jc, int q, int ja, int jb, float ma, float mb,
        const B3Mat3& ia, const B3Mat3& ib, B3Vec3& va, B3Vec3& wa, B3Vec3& vb, B3Vec3& wb, B3Soft soft, int use_bias) {
    B3Vec3 ra = b3_rotate(ldq(bc, BI(ja, BDQ)), ld3(jc, JI(q, JFPA)));
    B3Vec3 rb = b3_rotate(ldq(bc, BI(jb, BDQ)), ld3(jc, JI(q, JFPB)));
    B3Vec3 cdot = b3_sub(b3_add(vb, b3_cross(wb, rb)), b3_add(va, b3_cross(wa, ra)));
    B3Vec3 bias = b3_v(0.0f, 0.0f, 0.0f);
    float mscale = 1.0f, iscale = 0.0f;
    if (use_bias) {
        B3Vec3 sep = b3_add(b3_add(b3_sub(ld3(bc, BI(jb, BDP)), ld3(bc, BI(ja, BDP))), b3_sub(rb, ra)),
            ld3(jc, JI(q, JDC)));
        bias = b3_mul(sep, soft.bias_rate);
        mscale = soft.mass_scale;
        iscale = soft.impulse_scale;
    }
    B3Vec3 b = b3_mv(m3_inv(point_k(ma, mb, ia, ib, ra, rb)), b3_add(cdot, bias));
    B3Vec3 li = ld3(jc, JI(q, JLI));
    B3Vec3 impulse = b3_msub(b3_mul(b, -mscale), iscale, li);
    st3(jc, JI(q, JLI), b3_add(li, impulse));
    va = b3_msub(va, ma, impulse);
    wa = b3_sub(wa, b3_mv(ia, b3_cross(ra, impulse)));
    vb = b3_madd(vb, mb, impulse);
    wb = b3_add(wb, b3_mv(ib, b3_cross(rb, impulse)));
}

// 06_joints.inl:419-434
B3X_HDI float limit_impulse(float c, float cdot, float inv_h, int use_bias, B3Soft soft,
        float axial_mass, float old) {
    float bias = 0.0f, mscale = 1.0f, iscale = 0.0f;
    if (c > 0.0f) {
        bias = c * inv_h;
    } else if (use_bias) {
        bias = soft.bias_rate * c;
        mscale = soft.mass_scale;
        iscale = soft.impulse_scale;
    }
    float dimp = -mscale * axial_mass * (cdot + bias) - iscale * old;
    return b3_maxf(old + dimp, 0.0f);
}

// One joint, either type (07_packed.inl:66-79 dispatch; weld 06_joints.inl:285-332,
// revolute 06_joints.inl:436-642 default uncached path).
B3X_HD void solve_joint(float* bc, float* jc, int q, float h, float inv_h, int use_bias) {
    int type = ldi(jc, JI(q, JTYPE));
    int ja = ldi(jc, JI(q, JBA)), jb = ldi(jc, JI(q, JBB));
    float ma = COL(bc, BI(ja, BMI)), mb = COL(bc, BI(jb, BMI));
    B3Mat3 ia = ldm(bc, BI(ja, BII)), ib = ldm(bc, BI(jb, BII));
    B3Vec3 va = ld3(bc, BI(ja, BV)), wa = ld3(bc, BI(ja, BW));
    B3Vec3 vb = ld3(bc, BI(jb, BV)), wb = ld3(bc, BI(jb, BW));
    int fixed = ldi(jc, JI(q, JFIX));
    B3Quat qa = b3_qmul(ldq(bc, BI(ja, BDQ)), ldq(jc, JI(q, JFQA)));
    B3Quat qb = b3_qmul(ldq(bc, BI(jb, BDQ)), ldq(jc, JI(q, JFQB)));
    if (b3_qdot(qa, qb) < 0.0f) qb = b3_qneg(qb);
    B3Quat rel = b3_qinv_mul(qa, qb);
    if (type == B3_JOINT_WELD) {
        float ah = COL(jc, JI(q, JAH));
        if (!fixed) {
            B3Vec3 bias = b3_v(0.0f, 0.0f, 0.0f);
            float mscale = 1.0f, iscale = 0.0f;
            if (use_bias || ah > 0.0f) {
                B3Quat s = rel;
                if (rel.s < 0.0f) s = b3_qneg(rel);
                B3Quat diff = b3_q(-s.v.x, -s.v.y, -s.v.z, 1.0f - s.s);
                B3Vec3 c = b3_neg(b3_rotate(qa, b3_mul(b3_qmul(diff, b3_qconj(s)).v, 2.0f)));
                B3Soft as = lds(jc, JI(q, JAS));
                bias = b3_mul(c, as.bias_rate);
                mscale = as.mass_scale;
                iscale = as.impulse_scale;
            }
            B3Vec3 cdot = b3_sub(wb, wa);
            B3Vec3 ai = ld3(jc, JI(q, JAI));
            B3Vec3 impulse = b3_msub(b3_mul(b3_mv(ldm(jc, JI(q, JAM)), b3_add(cdot, bias)), -mscale), iscale, ai);
            st3(jc, JI(q, JAI), b3_add(ai, impulse));
            wa = b3_sub(wa, b3_mv(ia, impulse));
            wb = b3_add(wb, b3_mv(ib, impulse));
        }
        int lin_bias = use_bias || COL(jc, JI(q, JLH)) > 0.0f;
        solve_point(bc, jc, q, ja, jb, ma, mb, ia, ib, va, wa, vb, wb, lds(jc, JI(q, JLS)), lin_bias);
        put_vel(bc, ja, va, wa);
        put_vel(bc, jb, vb, wb);
        return;
    }
    B3Vec3 axis = ld3(jc, JI(q, JAX));
    B3Vec3 ia_ax = b3_v(0.0f, 0.0f, 0.0f), ib_ax = b3_v(0.0f, 0.0f, 0.0f);
    float twist = 0.0f;
    int en_spring = ldi(jc, JI(q, JENS)), en_motor = ldi(jc, JI(q, JENM)), en_limit = ldi(jc, JI(q, JENL));
    int need_twist = (en_spring || en_limit || en_motor) && !fixed;
    if (!fixed) {
        ia_ax = b3_mv(ia, axis);
        ib_ax = b3_mv(ib, axis);
    }
    if (need_twist) twist = b3_twist(rel);
    float axial_mass = COL(jc, JI(q, JAXM));
    float mmt = COL(jc, JI(q, JMMT));
    if (en_spring && !fixed) {
        B3Soft ss = lds(jc, JI(q, JSS));
        float c = twist - COL(jc, JI(q, JTA));
        float bias = ss.bias_rate * c;
        float cdot = b3_dot(b3_sub(wb, wa), axis);
        float old = COL(jc, JI(q, JSI));
        float dimp = -ss.mass_scale * axial_mass * (cdot + bias) - ss.impulse_scale * old;
        float nimp = old + dimp;
        if (mmt > 0.0f) {
            float maxp = mmt * h;
            nimp = b3_clamp(nimp, -maxp, maxp);
        }
        dimp = nimp - old;
        COL(jc, JI(q, JSI)) = nimp;
        wa = b3_msub(wa, dimp, ia_ax);
        wb = b3_madd(wb, dimp, ib_ax);
    }
    if (en_motor && !fixed) {
        float speed = COL(jc, JI(q, JMS));
        int blocked = 0;
        if (en_limit) {
            if (twist >= COL(jc, JI(q, JUA)) - 0.01f && speed > 0.0f) blocked = 1;
            if (twist <= COL(jc, JI(q, JLA)) + 0.01f && speed < 0.0f) blocked = 1;
        }
        if (blocked) {
            COL(jc, JI(q, JMI)) = 0.0f;
        } else {
            float cdot = b3_dot(b3_sub(wb, wa), axis) - speed;
            float dimp = -axial_mass * cdot;
            float old = COL(jc, JI(q, JMI));
            float nimp = old + dimp;
            float maxp = mmt * h;
            nimp = b3_clamp(nimp, -maxp, maxp);
            dimp = nimp - old;
            COL(jc, JI(q, JMI)) = nimp;
            wa = b3_msub(wa, dimp, ia_ax);
            wb = b3_madd(wb, dimp, ib_ax);
        }
    }
    if (en_limit && !fixed) {
        B3Soft soft = lds(jc, JI(q, JSOFT));
        float old = COL(jc, JI(q, JLOI));
        float lo = limit_impulse(twist - COL(jc, JI(q, JLA)), b3_dot(b3_sub(wb, wa), axis), inv_h, use_bias, soft,
            axial_mass, old);
        COL(jc, JI(q, JLOI)) = lo;
        float dimp = lo - old;
        wa = b3_msub(wa, dimp, ia_ax);
        wb = b3_madd(wb, dimp, ib_ax);
        old = COL(jc, JI(q, JUPI));
        float up = limit_impulse(COL(jc, JI(q, JUA)) - twist, b3_dot(b3_sub(wa, wb), axis), inv_h, use_bias, soft,
            axial_mass, old);
        COL(jc, JI(q, JUPI)) = up;
        dimp = up - old;
        wa = b3_madd(wa, dimp, ia_ax);
        wb = b3_msub(wb, dimp, ib_ax);
    }
    B3Soft soft = lds(jc, JI(q, JSOFT));
    if (!fixed) {
        B3Vec2 bias;
        bias.x = 0.0f;
        bias.y = 0.0f;
        float mscale = 1.0f, iscale = 0.0f;
        if (use_bias) {
            bias.x = soft.bias_rate * rel.v.x;
            bias.y = soft.bias_rate * rel.v.y;
            mscale = soft.mass_scale;
            iscale = soft.impulse_scale;
        }
        B3Vec3 px, py;
        hinge_perps(qa, rel, &px, &py);
        st3(jc, JI(q, JPX), px);
        st3(jc, JI(q, JPY), py);
        B3Mat3 isum = m3_add(ia, ib);
        B3Mat2 kang;
        kang.cx.x = b3_dot(px, b3_mv(isum, px));
        kang.cy.y = b3_dot(py, b3_mv(isum, py));
        kang.cx.y = kang.cy.x = b3_dot(px, b3_mv(isum, py));
        B3Vec3 wrel = b3_sub(wb, wa);
        B3Vec2 rhs;
        rhs.x = b3_dot(wrel, px) + bias.x;
        rhs.y = b3_dot(wrel, py) + bias.y;
        B3Vec2 sol = solve2(kang, rhs);
        B3Vec2 old;
        old.x = COL(jc, JI(q, JPI));
        old.y = COL(jc, JI(q, JPI + 1));
        B3Vec2 dimp;
        dimp.x = -mscale * sol.x - iscale * old.x;
        dimp.y = -mscale * sol.y - iscale * old.y;
        COL(jc, JI(q, JPI)) = old.x + dimp.x;
        COL(jc, JI(q, JPI + 1)) = old.y + dimp.y;
        B3Vec3 ang = b3_add(b3_mul(px, dimp.x), b3_mul(py, dimp.y));
        wa = b3_sub(wa, b3_mv(ia, ang));
        wb = b3_add(wb, b3_mv(ib, ang));
    }
    solve_point(bc, jc, q, ja, jb, ma, mb, ia, ib, va, wa, vb, wb, soft, use_bias);
    put_vel(bc, ja, va, wa);
    put_vel(bc, jb, vb, wb);
}

// ---- one world, one step ----------------------------------------------------
B3X_HD void world_step(unsigned char* wp, const StepArgs& a, float* bc, float* sc, float* cc, float* jc) {
    const Layout& L = a.L;
    Header* hd = reinterpret_cast<Header*>(wp);
    B3Body* bodies = reinterpret_cast<B3Body*>(wp + B3X_WORLD_HEADER_BYTES);
    B3Shape* shapes = reinterpret_cast<B3Shape*>(wp + L.shape_off);
    B3Contact* contacts = reinterpret_cast<B3Contact*>(wp + L.contact_off);
    B3Joint* joints = reinterpret_cast<B3Joint*>(wp + L.joint_off);

    // Counts beyond the capacities would index past the arrays in the
    // reference; here they are clamped so a corrupt world cannot fault.
    const int nb = clampi(hd->body_count, 0, L.B);
    const int ns = clampi(hd->shape_count, 0, L.S);
    const int old_n = clampi(hd->contact_count, 0, L.C);
    const int nj = clampi(hd->joint_count, 0, L.J);

    // 09_step.inl:148-157
    const int subs = a.substeps;
    const float dt = a.dt;
    const float h = dt / (float)subs;
    const float inv_dt = 1.0f / dt;
    const float inv_h = (float)subs * inv_dt;
    const float hertz = b3_minf(hd->contact_hertz, 0.25f * inv_h);
    const float contact_damping = hd->contact_damping;
    const B3Soft cs = make_soft(hertz, contact_damping, h);
    const B3Soft ss = make_soft(2.0f * hertz, 0.5f * contact_damping, h);
    const float contact_speed = hd->contact_speed;

    // -- bodies into working columns (inverse mass / inertia gated by type as
    //    the contact and joint prepares do, 08_contacts.inl:236-239)
    for (int k = 0; k < nb; k++) {
        const B3Body* b = &bodies[k];
        int type = b->type;
        bool dyn = type == B3_DYNAMIC;
        st3(bc, BI(k, BV), b->lin_vel);
        st3(bc, BI(k, BW), b->ang_vel);
        st3(bc, BI(k, BDP), b->delta_pos);
        stq(bc, BI(k, BDQ), b->delta_rot);
        COL(bc, BI(k, BMI)) = dyn ? b->inv_mass : 0.0f;
        stm(bc, BI(k, BII), dyn ? b->inv_i_world : m3_zero());
        COL(bc, BI(k, BFLAGS)) = b3x_u2f(b->flags);
        sti(bc, BI(k, BTYPE), type);
    }

    // -- shape world poses and padded AABBs (04_world.inl:293-336,
    //    08_contacts.inl:109-114); a shape on an invalid body never overlaps
    for (int s = 0; s < ns; s++) {
        const B3Shape* sh = &shapes[s];
        int body = sh->body;
        if (body < 0 || body >= nb) {
            st3(sc, SI(s, SLO), b3_v(INFINITY, INFINITY, INFINITY));
            st3(sc, SI(s, SHI), b3_v(-INFINITY, -INFINITY, -INFINITY));
            continue;
        }
        B3Vec3 bp = bodies[body].position;
        B3Quat bq = bodies[body].rotation;
        B3Vec3 p = b3_xf_point(bp, bq, sh->local_pos);
        B3Quat q = b3_qmul(bq, sh->local_rot);
        B3Vec3 lo, hi;
        int type = sh->type;
        if (type == B3_SPHERE) {
            B3Vec3 e = b3_v(sh->radius, sh->radius, sh->radius);
            lo = b3_sub(p, e);
            hi = b3_add(p, e);
        } else if (type == B3_CAPSULE) {
            B3Vec3 y = b3_rotate(q, b3_v(0.0f, sh->half.y, 0.0f));
            B3Vec3 c1 = b3_sub(p, y), c2 = b3_add(p, y);
            B3Vec3 e = b3_v(sh->radius, sh->radius, sh->radius);
            lo = b3_sub(b3_v(b3_minf(c1.x, c2.x), b3_minf(c1.y, c2.y), b3_minf(c1.z, c2.z)), e);
            hi = b3_add(b3_v(b3_maxf(c1.x, c2.x), b3_maxf(c1.y, c2.y), b3_maxf(c1.z, c2.z)), e);
        } else {
            B3Vec3 ax, ay, az, hf = sh->half;
            b3_axes(q, &ax, &ay, &az);
            B3Vec3 e = b3_v(fabsf(ax.x) * hf.x + fabsf(ay.x) * hf.y + fabsf(az.x) * hf.z,
                fabsf(ax.y) * hf.x + fabsf(ay.y) * hf.y + fabsf(az.y) * hf.z,
                fabsf(ax.z) * hf.x + fabsf(ay.z) * hf.y + fabsf(az.z) * hf.z);
            lo = b3_sub(p, e);
            hi = b3_add(p, e);
        }
        B3Vec3 pad = b3_v(B3_SPECULATIVE, B3_SPECULATIVE, B3_SPECULATIVE);
        st3(sc, SI(s, SPOS), p);
        stq(sc, SI(s, SROT), q);
        st3(sc, SI(s, SLO), b3_sub(lo, pad));
        st3(sc, SI(s, SHI), b3_add(hi, pad));
    }

    // -- contact generation with warm-cache carry (08_contacts.inl:64-173).
    // The old cache is matched with a merge cursor when its (shape_a, shape_b)
    // keys are strictly increasing (always true for caches this step wrote),
    // otherwise with the reference's full scan; both pick the same entry.
    bool old_sorted = true;
    {
        int pa = -1, pb = -1;
        for (int k = 0; k < old_n; k++) {
            int sa = contacts[k].shape_a, sb = contacts[k].shape_b;
            if (sa < pa || (sa == pa && sb <= pb)) old_sorted = false;
            pa = sa;
            pb = sb;
        }
    }
    int n = 0, cursor = 0;
    int overflow = hd->contact_overflow, dropped = hd->contacts_dropped;
    for (int i = 0; i < ns; i++) {
        const B3Shape* si = &shapes[i];
        const int body_i = si->body;
        if (body_i < 0 || body_i >= nb) continue;
        const B3Vec3 lo_i = ld3(sc, SI(i, SLO)), hi_i = ld3(sc, SI(i, SHI));
        const int btype_i = ldi(bc, BI(body_i, BTYPE));
        for (int j = i + 1; j < ns; j++) {
            const B3Vec3 lo_j = ld3(sc, SI(j, SLO)), hi_j = ld3(sc, SI(j, SHI));
            if (!(lo_i.x <= hi_j.x && hi_i.x >= lo_j.x && lo_i.y <= hi_j.y && hi_i.y >= lo_j.y
                    && lo_i.z <= hi_j.z && hi_i.z >= lo_j.z))
                continue;
            const B3Shape* sj = &shapes[j];
            const int body_j = sj->body;
            if (body_i == body_j) continue;
            const int btype_j = ldi(bc, BI(body_j, BTYPE));
            if (btype_i == B3_STATIC && btype_j == B3_STATIC) continue;
            if ((si->category & sj->mask) == 0 || (sj->category & si->mask) == 0) continue;
            bool connected = false;
            for (int q = 0; q < nj; q++) {
                const B3Joint* jt = &joints[q];
                int ja = jt->body_a, jb = jt->body_b;
                if (!jt->collide_connected && ((ja == body_i && jb == body_j) || (ja == body_j && jb == body_i)))
                    connected = true;
            }
            if (connected) continue;
            Geo ga, gb;
            ga.p = ld3(sc, SI(i, SPOS)); ga.q = ldq(sc, SI(i, SROT)); ga.type = si->type;
            ga.radius = si->radius; ga.half = si->half;
            gb.p = ld3(sc, SI(j, SPOS)); gb.q = ldq(sc, SI(j, SROT)); gb.type = sj->type;
            gb.radius = sj->radius; gb.half = sj->half;
            Mani m;
            collide(m, ga, gb);
            if (m.count == 0) continue;
            if (n >= L.C) {
                overflow = 1;
                dropped++;
                continue;
            }
            // 08_contacts.inl:5-39
            B3Vec3 nrm = m.normal;
            B3Vec3 t1 = b3_perp(nrm);
            B3Vec3 t2 = b3_cross(t1, nrm);
            sti(cc, CI(n, CSA), i);
            sti(cc, CI(n, CSB), j);
            sti(cc, CI(n, CBA), body_i);
            sti(cc, CI(n, CBB), body_j);
            sti(cc, CI(n, CCNT), m.count);
            sti(cc, CI(n, CSTAT), btype_i != B3_DYNAMIC || btype_j != B3_DYNAMIC);
            st3(cc, CI(n, CN), nrm);
            st3(cc, CI(n, CT1), t1);
            st3(cc, CI(n, CT2), t2);
            COL(cc, CI(n, CFRIC)) = sqrtf(si->friction * sj->friction);
            COL(cc, CI(n, CREST)) = si->restitution > sj->restitution ? si->restitution : sj->restitution;
            COL(cc, CI(n, CROLL)) = b3_maxf(si->rolling, sj->rolling);
            B3Vec2 fi;
            fi.x = 0.0f;
            fi.y = 0.0f;
            float twi = 0.0f;
            B3Vec3 ri = b3_v(0.0f, 0.0f, 0.0f);
            B3Vec3 ca = bodies[body_i].center, cb = bodies[body_j].center;
            float ni[B3_MAX_MANIFOLD];
            for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
                ni[p] = 0.0f;
                if (p >= m.count) continue;
                B3Vec3 ra = b3_sub(m.pa[p], ca), rb = b3_sub(m.pb[p], cb);
                st3(cc, PI(n, p, PRA), ra);
                st3(cc, PI(n, p, PRB), rb);
                COL(cc, PI(n, p, PBSEP)) = m.sep[p] - b3_dot(b3_sub(rb, ra), nrm);
                sti(cc, PI(n, p, PFEAT), (int)m.feat[p]);
            }
            // warm-start carry by (shape_a, shape_b) and feature id (08_contacts.inl:136-171)
            int k_first = 0, k_end = old_n;
            if (old_sorted) {
                while (cursor < old_n && (contacts[cursor].shape_a < i
                        || (contacts[cursor].shape_a == i && contacts[cursor].shape_b < j)))
                    cursor++;
                k_first = cursor;
                k_end = cursor < old_n ? cursor + 1 : old_n;
            }
            for (int k = k_first; k < k_end; k++) {
                const B3Contact* oc = &contacts[k];
                if (oc->shape_a != i || oc->shape_b != j) continue;
                int ocnt = clampi(oc->point_count, 0, B3_MAX_MANIFOLD);
                for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
                    if (p >= m.count) continue;
                    for (int qq = 0; qq < ocnt; qq++)
                        if (m.feat[p] == oc->points[qq].feature) ni[p] = oc->points[qq].normal_impulse;
                }
                fi = oc->friction_impulse;
                twi = oc->twist_impulse;
                ri = oc->rolling_impulse;
            }
            for (int p = 0; p < B3_MAX_MANIFOLD; p++)
                if (p < m.count) COL(cc, PI(n, p, PNI)) = ni[p];
            COL(cc, CI(n, CFI)) = fi.x;
            COL(cc, CI(n, CFI + 1)) = fi.y;
            COL(cc, CI(n, CTWI)) = twi;
            st3(cc, CI(n, CRI), ri);
            n++;
        }
    }

    // -- prepare contacts (08_contacts.inl:234-291); the prepared fields are
    //    final for the step, so they go to the world now (the old cache is dead)
    const float inv_tau = 1.0f / B3_SPECULATIVE;
    for (int k = 0; k < n; k++) {
        B3Contact* oc = &contacts[k];
        int ba = ldi(cc, CI(k, CBA)), bb = ldi(cc, CI(k, CBB));
        int cnt = ldi(cc, CI(k, CCNT));
        int stat = ldi(cc, CI(k, CSTAT));
        float ma = COL(bc, BI(ba, BMI)), mb = COL(bc, BI(bb, BMI));
        B3Mat3 ia = ldm(bc, BI(ba, BII)), ib = ldm(bc, BI(bb, BII));
        B3Vec3 va = ld3(bc, BI(ba, BV)), wa = ld3(bc, BI(ba, BW));
        B3Vec3 vb = ld3(bc, BI(bb, BV)), wb = ld3(bc, BI(bb, BW));
        B3Vec3 nrm = ld3(cc, CI(k, CN));
        B3Vec3 t1 = ld3(cc, CI(k, CT1)), t2 = ld3(cc, CI(k, CT2));
        B3Vec3 center_a = b3_v(0.0f, 0.0f, 0.0f), center_b = b3_v(0.0f, 0.0f, 0.0f);
        float wsum = 0.0f;
        for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
            if (p >= cnt) break;
            B3Vec3 ra = ld3(cc, PI(k, p, PRA)), rb = ld3(cc, PI(k, p, PRB));
            B3Vec3 rn_a = b3_cross(ra, nrm), rn_b = b3_cross(rb, nrm);
            float kn = ma + mb + b3_dot(rn_a, b3_mv(ia, rn_a)) + b3_dot(rn_b, b3_mv(ib, rn_b));
            float nm = kn > 0.0f ? 1.0f / kn : 0.0f;
            B3Vec3 vra = b3_add(va, b3_cross(wa, ra)), vrb = b3_add(vb, b3_cross(wb, rb));
            float relv = b3_dot(nrm, b3_sub(vrb, vra));
            float base_sep = COL(cc, PI(k, p, PBSEP));
            float sep = base_sep + b3_dot(b3_sub(rb, ra), nrm);
            float wgt = b3_clamp(2.0f - sep * inv_tau, B3_MIN_FRICTION_W, 1.0f);
            center_a = b3_madd(center_a, wgt, ra);
            center_b = b3_madd(center_b, wgt, rb);
            wsum += wgt;
            COL(cc, PI(k, p, PNM)) = nm;
            COL(cc, PI(k, p, PRELV)) = relv;
            COL(cc, PI(k, p, PTOT)) = 0.0f;
            B3Point* op = &oc->points[p];
            op->r_a = ra;
            op->r_b = rb;
            op->base_sep = base_sep;
            op->rel_vel = relv;
            op->normal_mass = nm;
            op->feature = (uint32_t)ldi(cc, PI(k, p, PFEAT));
        }
        float invw = wsum > 0.0f ? 1.0f / wsum : 0.0f;
        B3Vec3 ca = b3_mul(center_a, invw), cb = b3_mul(center_b, invw);
        for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
            if (p >= cnt) break;
            float lev = b3_len(b3_sub(ld3(cc, PI(k, p, PRA)), ca));
            COL(cc, PI(k, p, PLEV)) = lev;
            oc->points[p].lever = lev;
        }
        B3Vec3 rta1 = b3_cross(ca, t1), rta2 = b3_cross(ca, t2);
        B3Vec3 rtb1 = b3_cross(cb, t1), rtb2 = b3_cross(cb, t2);
        B3Mat2 kt2;
        kt2.cx.x = ma + mb + b3_dot(rta1, b3_mv(ia, rta1)) + b3_dot(rtb1, b3_mv(ib, rtb1));
        kt2.cy.y = ma + mb + b3_dot(rta2, b3_mv(ia, rta2)) + b3_dot(rtb2, b3_mv(ib, rtb2));
        kt2.cx.y = kt2.cy.x = b3_dot(rta1, b3_mv(ia, rta2)) + b3_dot(rtb1, b3_mv(ib, rtb2));
        B3Mat2 tm = m2_inv(kt2);
        B3Mat3 isum = m3_add(ia, ib);
        float ktw = b3_dot(nrm, b3_mv(isum, nrm));
        float twm = ktw > 0.0f ? 1.0f / ktw : 0.0f;
        st3(cc, CI(k, CCA), ca);
        st3(cc, CI(k, CCB), cb);
        COL(cc, CI(k, CTM)) = tm.cx.x;
        COL(cc, CI(k, CTM + 1)) = tm.cx.y;
        COL(cc, CI(k, CTM + 2)) = tm.cy.x;
        COL(cc, CI(k, CTM + 3)) = tm.cy.y;
        COL(cc, CI(k, CTWM)) = twm;
        oc->shape_a = ldi(cc, CI(k, CSA));
        oc->shape_b = ldi(cc, CI(k, CSB));
        oc->body_a = ba;
        oc->body_b = bb;
        oc->point_count = cnt;
        oc->static_contact = stat;
        oc->normal = nrm;
        oc->tangent1 = t1;
        oc->tangent2 = t2;
        oc->center_a = ca;
        oc->center_b = cb;
        oc->friction = COL(cc, CI(k, CFRIC));
        oc->restitution = COL(cc, CI(k, CREST));
        oc->rolling = COL(cc, CI(k, CROLL));
        oc->twist_mass = twm;
        oc->tangent_mass = tm;
        oc->rolling_mass = m3_inv(isum);
        oc->inv_mass_a = ma;
        oc->inv_mass_b = mb;
        oc->inv_i_a = ia;
        oc->inv_i_b = ib;
        oc->softness = stat ? ss : cs;
    }

    // -- prepare joints (06_joints.inl:161-202); invalid body indices mark the
    //    joint inert (the reference would index out of bounds)
    for (int q = 0; q < nj; q++) {
        B3Joint* jt = &joints[q];
        int type = jt->type, ja = jt->body_a, jb = jt->body_b;
        if (ja < 0 || ja >= nb || jb < 0 || jb >= nb) {
            sti(jc, JI(q, JOK), 0);
            continue;
        }
        sti(jc, JI(q, JOK), 1);
        float ma = COL(bc, BI(ja, BMI)), mb = COL(bc, BI(jb, BMI));
        B3Mat3 ia = ldm(bc, BI(ja, BII)), ib = ldm(bc, BI(jb, BII));
        B3Mat3 isum = m3_add(ia, ib);
        int fixed = b3_dot(isum.cx, b3_cross(isum.cy, isum.cz)) < 1.0e-20f;
        B3Soft soft = make_soft(jt->constraint_hertz, jt->constraint_damping, h);
        const B3Body* ba = &bodies[ja];
        const B3Body* bb = &bodies[jb];
        B3Quat rot_a = ba->rotation, rot_b = bb->rotation;
        B3Quat fqa = b3_qmul(rot_a, jt->local_rot_a), fqb = b3_qmul(rot_b, jt->local_rot_b);
        B3Vec3 fpa = b3_rotate(rot_a, b3_sub(jt->local_anchor_a, ba->local_center));
        B3Vec3 fpb = b3_rotate(rot_b, b3_sub(jt->local_anchor_b, bb->local_center));
        B3Vec3 dc = b3_sub(bb->center, ba->center);
        jt->inv_mass_a = ma;
        jt->inv_mass_b = mb;
        jt->inv_i_a = ia;
        jt->inv_i_b = ib;
        jt->fixed_rotation = fixed;
        jt->softness = soft;
        jt->frame_q_a = fqa;
        jt->frame_q_b = fqb;
        jt->frame_p_a = fpa;
        jt->frame_p_b = fpb;
        jt->delta_center = dc;
        sti(jc, JI(q, JTYPE), type);
        sti(jc, JI(q, JBA), ja);
        sti(jc, JI(q, JBB), jb);
        sti(jc, JI(q, JFIX), fixed);
        st3(jc, JI(q, JFPA), fpa);
        st3(jc, JI(q, JFPB), fpb);
        stq(jc, JI(q, JFQA), fqa);
        stq(jc, JI(q, JFQB), fqb);
        st3(jc, JI(q, JDC), dc);
        sts(jc, JI(q, JSOFT), soft);
        st3(jc, JI(q, JLI), jt->linear_impulse);
        if (type == B3_JOINT_WELD) {
            float lh = jt->linear_hertz, ah = jt->angular_hertz;
            B3Mat3 am = m3_inv(isum);
            B3Soft ls = lh == 0.0f ? soft : make_soft(lh, jt->linear_damping, h);
            B3Soft as = ah == 0.0f ? soft : make_soft(ah, jt->angular_damping, h);
            jt->angular_mass = am;
            jt->linear_spring = ls;
            jt->angular_spring = as;
            stm(jc, JI(q, JAM), am);
            COL(jc, JI(q, JLH)) = lh;
            COL(jc, JI(q, JAH)) = ah;
            sts(jc, JI(q, JLS), ls);
            sts(jc, JI(q, JAS), as);
            st3(jc, JI(q, JAI), jt->angular_impulse);
        } else {
            B3Vec3 axis = b3_rotate(fqa, b3_v(0.0f, 0.0f, 1.0f));
            float kx = b3_dot(axis, b3_mv(isum, axis));
            float axm = kx > 0.0f ? 1.0f / kx : 0.0f;
            B3Quat rel = b3_qinv_mul(fqa, fqb);
            B3Vec3 px, py;
            hinge_perps(fqa, rel, &px, &py);
            B3Soft sps = make_soft(jt->hertz, jt->damping_ratio, h);
            jt->axial_mass = axm;
            jt->rotation_axis = axis;
            jt->perp_x = px;
            jt->perp_y = py;
            jt->spring_softness = sps;
            st3(jc, JI(q, JAX), axis);
            COL(jc, JI(q, JAXM)) = axm;
            st3(jc, JI(q, JPX), px);
            st3(jc, JI(q, JPY), py);
            sts(jc, JI(q, JSS), sps);
            sti(jc, JI(q, JENS), jt->enable_spring);
            sti(jc, JI(q, JENM), jt->enable_motor);
            sti(jc, JI(q, JENL), jt->enable_limit);
            COL(jc, JI(q, JPI)) = jt->perp_impulse.x;
            COL(jc, JI(q, JPI + 1)) = jt->perp_impulse.y;
            COL(jc, JI(q, JSI)) = jt->spring_impulse;
            COL(jc, JI(q, JMI)) = jt->motor_impulse;
            COL(jc, JI(q, JLOI)) = jt->lower_impulse;
            COL(jc, JI(q, JUPI)) = jt->upper_impulse;
            COL(jc, JI(q, JMMT)) = jt->max_motor_torque;
            COL(jc, JI(q, JMS)) = jt->motor_speed;
            COL(jc, JI(q, JTA)) = jt->target_angle;
            COL(jc, JI(q, JLA)) = jt->lower_angle;
            COL(jc, JI(q, JUA)) = jt->upper_angle;
            if (type != B3_JOINT_REVOLUTE) st3(jc, JI(q, JAI), jt->angular_impulse);
        }
    }

    // -- warm start contacts (08_contacts.inl:194-232, 293-313)
    for (int k = 0; k < n; k++) {
        int ba = ldi(cc, CI(k, CBA)), bb = ldi(cc, CI(k, CBB));
        int cnt = ldi(cc, CI(k, CCNT));
        float ma = COL(bc, BI(ba, BMI)), mb = COL(bc, BI(bb, BMI));
        B3Mat3 ia = ldm(bc, BI(ba, BII)), ib = ldm(bc, BI(bb, BII));
        B3Vec3 nrm = ld3(cc, CI(k, CN));
        for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
            if (p >= cnt) break;
            B3Vec3 P = b3_mul(nrm, COL(cc, PI(k, p, PNI)));
            apply_impulse(bc, ba, ma, ia, ld3(cc, PI(k, p, PRA)), P, -1);
            apply_impulse(bc, bb, mb, ib, ld3(cc, PI(k, p, PRB)), P, 1);
        }
        B3Vec3 f = b3_add(b3_mul(ld3(cc, CI(k, CT1)), COL(cc, CI(k, CFI))),
            b3_mul(ld3(cc, CI(k, CT2)), COL(cc, CI(k, CFI + 1))));
        apply_impulse(bc, ba, ma, ia, ld3(cc, CI(k, CCA)), f, -1);
        apply_impulse(bc, bb, mb, ib, ld3(cc, CI(k, CCB)), f, 1);
        B3Vec3 tr = b3_add(b3_mul(nrm, COL(cc, CI(k, CTWI))), ld3(cc, CI(k, CRI)));
        if (b3x_f2u(COL(bc, BI(ba, BFLAGS))) & B3_FLAG_DYNAMIC)
            st3(bc, BI(ba, BW), b3_sub(ld3(bc, BI(ba, BW)), b3_mv(ia, tr)));
        if (b3x_f2u(COL(bc, BI(bb, BFLAGS))) & B3_FLAG_DYNAMIC)
            st3(bc, BI(bb, BW), b3_add(ld3(bc, BI(bb, BW)), b3_mv(ib, tr)));
    }

    // -- warm start joints (06_joints.inl:204-239)
    for (int q = 0; q < nj; q++) {
        if (!ldi(jc, JI(q, JOK))) continue;
        int type = ldi(jc, JI(q, JTYPE));
        int ja = ldi(jc, JI(q, JBA)), jb = ldi(jc, JI(q, JBB));
        float ma = COL(bc, BI(ja, BMI)), mb = COL(bc, BI(jb, BMI));
        B3Mat3 ia = ldm(bc, BI(ja, BII)), ib = ldm(bc, BI(jb, BII));
        B3Vec3 ra = b3_rotate(ldq(bc, BI(ja, BDQ)), ld3(jc, JI(q, JFPA)));
        B3Vec3 rb = b3_rotate(ldq(bc, BI(jb, BDQ)), ld3(jc, JI(q, JFPB)));
        B3Vec3 li = ld3(jc, JI(q, JLI));
        B3Vec3 ang;
        if (type == B3_JOINT_REVOLUTE) {
            float axial = COL(jc, JI(q, JSI)) + COL(jc, JI(q, JMI)) + COL(jc, JI(q, JLOI)) - COL(jc, JI(q, JUPI));
            ang = b3_add(b3_mul(ld3(jc, JI(q, JPX)), COL(jc, JI(q, JPI))),
                b3_mul(ld3(jc, JI(q, JPY)), COL(jc, JI(q, JPI + 1))));
            ang = b3_madd(ang, axial, ld3(jc, JI(q, JAX)));
        } else {
            ang = ld3(jc, JI(q, JAI));
        }
        if (b3x_f2u(COL(bc, BI(ja, BFLAGS))) & B3_FLAG_DYNAMIC) {
            st3(bc, BI(ja, BV), b3_msub(ld3(bc, BI(ja, BV)), ma, li));
            st3(bc, BI(ja, BW), b3_sub(ld3(bc, BI(ja, BW)), b3_mv(ia, b3_add(b3_cross(ra, li), ang))));
        }
        if (b3x_f2u(COL(bc, BI(jb, BFLAGS))) & B3_FLAG_DYNAMIC) {
            st3(bc, BI(jb, BV), b3_madd(ld3(bc, BI(jb, BV)), mb, li));
            st3(bc, BI(jb, BW), b3_add(ld3(bc, BI(jb, BW)), b3_mv(ib, b3_add(b3_cross(rb, li), ang))));
        }
    }

    // -- substeps (09_step.inl:167-181)
    const float max_lin = hd->max_linear_speed;
    const float max_ang = B3_MAX_ROTATION * inv_dt;
    const float max_lin2 = max_lin * max_lin, max_ang2 = max_ang * max_ang;
    const B3Vec3 gravity = hd->gravity;
    const float restitution_threshold = hd->restitution_threshold;
    for (int s = 0; s < subs; s++) {
        // integrate velocities (09_step.inl:5-18, 41-53)
        for (int k = 0; k < nb; k++) {
            if (ldi(bc, BI(k, BTYPE)) != B3_DYNAMIC) continue;
            const B3Body* b = &bodies[k];
            float inv_mass = COL(bc, BI(k, BMI));
            float ld = 1.0f / (1.0f + h * b->linear_damping);
            float ad = 1.0f / (1.0f + h * b->angular_damping);
            float gs = inv_mass > 0.0f ? b->gravity_scale : 0.0f;
            B3Vec3 dv = b3_add(b3_mul(b->force, h * inv_mass), b3_mul(gravity, h * gs));
            st3(bc, BI(k, BV), b3_madd(dv, ld, ld3(bc, BI(k, BV))));
            B3Vec3 dw = b3_mul(b3_mv(ldm(bc, BI(k, BII)), b->torque), h);
            st3(bc, BI(k, BW), b3_madd(dw, ad, ld3(bc, BI(k, BW))));
        }
        for (int k = 0; k < n; k++) solve_contact(bc, cc, k, inv_h, contact_speed, 1, cs, ss);
        for (int it = 0; it < a.joint_iters; it++)
            for (int q = 0; q < nj; q++)
                if (ldi(jc, JI(q, JOK))) solve_joint(bc, jc, q, h, inv_h, 1);
        // integrate positions (09_step.inl:55-107)
        for (int k = 0; k < nb; k++) {
            if (ldi(bc, BI(k, BTYPE)) == B3_STATIC) continue;
            uint32_t flags = b3x_f2u(COL(bc, BI(k, BFLAGS)));
            B3Vec3 v = ld3(bc, BI(k, BV)), av = ld3(bc, BI(k, BW));
            if (flags & B3_LOCK_LIN_X) v.x = 0.0f;
            if (flags & B3_LOCK_LIN_Y) v.y = 0.0f;
            if (flags & B3_LOCK_LIN_Z) v.z = 0.0f;
            if (flags & B3_LOCK_ANG_X) av.x = 0.0f;
            if (flags & B3_LOCK_ANG_Y) av.y = 0.0f;
            if (flags & B3_LOCK_ANG_Z) av.z = 0.0f;
            float v2 = b3_len2(v);
            if (v2 > max_lin2 && v2 > 0.0f) v = b3_mul(v, max_lin / sqrtf(v2));
            float w2 = b3_len2(av);
            if (w2 > max_ang2 && w2 > 0.0f) av = b3_mul(av, max_ang / sqrtf(w2));
            st3(bc, BI(k, BV), v);
            st3(bc, BI(k, BW), av);
            st3(bc, BI(k, BDP), b3_madd(ld3(bc, BI(k, BDP)), h, v));
            stq(bc, BI(k, BDQ), q_integrate(ldq(bc, BI(k, BDQ)), b3_mul(av, h)));
        }
        for (int k = 0; k < n; k++) solve_contact(bc, cc, k, inv_h, contact_speed, 0, cs, ss);
        for (int it = 0; it < a.relax_iters; it++)
            for (int q = 0; q < nj; q++)
                if (ldi(jc, JI(q, JOK))) solve_joint(bc, jc, q, h, inv_h, 0);
        // restitution (08_contacts.inl:439-480)
        for (int k = 0; k < n; k++) {
            float rest = COL(cc, CI(k, CREST));
            if (rest == 0.0f) continue;
            int ba = ldi(cc, CI(k, CBA)), bb = ldi(cc, CI(k, CBB));
            int cnt = ldi(cc, CI(k, CCNT));
            float ma = COL(bc, BI(ba, BMI)), mb = COL(bc, BI(bb, BMI));
            B3Mat3 ia = ldm(bc, BI(ba, BII)), ib = ldm(bc, BI(bb, BII));
            B3Vec3 va = ld3(bc, BI(ba, BV)), wa = ld3(bc, BI(ba, BW));
            B3Vec3 vb = ld3(bc, BI(bb, BV)), wb = ld3(bc, BI(bb, BW));
            B3Vec3 nrm = ld3(cc, CI(k, CN));
            for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
                if (p >= cnt) break;
                float relv = COL(cc, PI(k, p, PRELV));
                if (relv > -restitution_threshold || COL(cc, PI(k, p, PTOT)) == 0.0f) continue;
                B3Vec3 ra = ld3(cc, PI(k, p, PRA)), rb = ld3(cc, PI(k, p, PRB));
                B3Vec3 vra = b3_add(va, b3_cross(wa, ra)), vrb = b3_add(vb, b3_cross(wb, rb));
                float vn = b3_dot(b3_sub(vrb, vra), nrm);
                float ni = COL(cc, PI(k, p, PNI));
                float imp = -COL(cc, PI(k, p, PNM)) * (vn + rest * relv);
                float nimp = b3_maxf(ni + imp, 0.0f);
                imp = nimp - ni;
                COL(cc, PI(k, p, PNI)) = nimp;
                B3Vec3 P = b3_mul(nrm, imp);
                va = b3_msub(va, ma, P);
                wa = b3_sub(wa, b3_mv(ia, b3_cross(ra, P)));
                vb = b3_madd(vb, mb, P);
                wb = b3_add(wb, b3_mv(ib, b3_cross(rb, P)));
            }
            put_vel(bc, ba, va, wa);
            put_vel(bc, bb, vb, wb);
        }
    }

    // -- finalize transforms (09_step.inl:109-130) and write the body state back
    for (int k = 0; k < nb; k++) {
        B3Body* b = &bodies[k];
        int type = ldi(bc, BI(k, BTYPE));
        uint32_t flags = b3x_f2u(COL(bc, BI(k, BFLAGS)));
        if (type != B3_STATIC || (flags & B3_FLAG_DYNAMIC)) {
            b->lin_vel = ld3(bc, BI(k, BV));
            b->ang_vel = ld3(bc, BI(k, BW));
        }
        if (type == B3_STATIC) continue;
        B3Vec3 center = b3_add(b->center, ld3(bc, BI(k, BDP)));
        B3Quat rot = b3_qnorm(b3_qmul(ldq(bc, BI(k, BDQ)), b->rotation));
        b->center = center;
        b->rotation = rot;
        b->position = b3_sub(center, b3_rotate(rot, b->local_center));
        b->delta_pos = b3_v(0.0f, 0.0f, 0.0f);
        b->delta_rot = b3_q_id();
        b->force = b3_v(0.0f, 0.0f, 0.0f);
        b->torque = b3_v(0.0f, 0.0f, 0.0f);
        if (type == B3_DYNAMIC) b->inv_i_world = b3_world_inv_i(rot, b->inv_inertia);
    }

    // -- solver-owned contact and joint fields, then the header
    for (int k = 0; k < n; k++) {
        B3Contact* oc = &contacts[k];
        int cnt = ldi(cc, CI(k, CCNT));
        for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
            if (p >= cnt) break;
            oc->points[p].normal_impulse = COL(cc, PI(k, p, PNI));
            oc->points[p].total_normal = COL(cc, PI(k, p, PTOT));
        }
        oc->twist_impulse = COL(cc, CI(k, CTWI));
        oc->friction_impulse.x = COL(cc, CI(k, CFI));
        oc->friction_impulse.y = COL(cc, CI(k, CFI + 1));
        oc->rolling_impulse = ld3(cc, CI(k, CRI));
    }
    for (int q = 0; q < nj; q++) {
        if (!ldi(jc, JI(q, JOK))) continue;
        int type = ldi(jc, JI(q, JTYPE));
        B3Joint* jt = &joints[q];
        jt->linear_impulse = ld3(jc, JI(q, JLI));
        if (type == B3_JOINT_WELD) {
            jt->angular_impulse = ld3(jc, JI(q, JAI));
        } else {
            jt->perp_impulse.x = COL(jc, JI(q, JPI));
            jt->perp_impulse.y = COL(jc, JI(q, JPI + 1));
            jt->spring_impulse = COL(jc, JI(q, JSI));
            jt->motor_impulse = COL(jc, JI(q, JMI));
            jt->lower_impulse = COL(jc, JI(q, JLOI));
            jt->upper_impulse = COL(jc, JI(q, JUPI));
            jt->perp_x = ld3(jc, JI(q, JPX));
            jt->perp_y = ld3(jc, JI(q, JPY));
        }
    }
    hd->contact_count = n;
    hd->contact_overflow = overflow;
    hd->contacts_dropped = dropped;
}

}  // namespace b3x
