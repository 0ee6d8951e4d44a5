// b3x_world.cuh -- one warp, 32 worlds, one step: the body of the step kernel
// (b3x_step.cu), over lane-interleaved working columns.
//
// Each lane owns one world.  Phases that only touch the lane's own world
// (loading bodies, shape poses, contact generation, prepares, warm starts,
// integration, restitution, finalize) run independently per lane.  The
// Gauss-Seidel sweeps over contacts and joints are warp-uniform: item k of
// all 32 worlds is one contiguous block of the workspace ([field][lane]),
// and a TMA bulk copy (cp.async.bulk + mbarrier) streams block k+1 into
// shared memory while the lanes solve block k, so the sweeps read their
// operands from shared memory only.  Solver-owned fields go back to the
// workspace with ordinary coalesced stores, made visible to the next pass's
// bulk copies by a proxy fence.
//
// Arithmetic keeps the reference's operation order (file:line cited, paths
// relative to the reference repository root); see b3x_step.cu for the build
// flags that make it bit-exact.  Functions are __host__ __device__ so that
// development tools can also compile the per-world logic for the host
// (there the sweeps read the workspace directly); the library runs them on
// the GPU only.
#pragma once
#include <cstdint>
#include <cstring>

#include "puffysics_b200.h"
#include "b3x_math.cuh"
#include "b3x_narrow.cuh"

namespace b3x {

constexpr int kLanes = 32;

// ---- working-set field indices (32-bit words) --------------------------------
// body columns (shared memory when they fit): velocities, pose deltas,
// type-gated inverse mass / world inverse inertia, flags, type
enum : int { BV = 0, BW = 3, BDP = 6, BDQ = 9, BMI = 13, BII = 14, BFLAGS = 23, BTYPE = 24, NBF = 25 };
// per-body step constants (workspace): velocity / spin increments and damping
// factors of b3_integrate_velocity_state, constant over the substeps
enum : int { KDV = 0, KDW = 3, KLD = 6, KAD = 7, NKF = 8 };
// shape columns (workspace): world pose and padded AABB
enum : int { SPOS = 0, SROT = 3, SLO = 7, SHI = 10, NSF = 13 };
// contact columns (workspace): the first NCG words are what the sweeps read
// and are streamed; point p occupies CP + p * NPF ...
enum : int {
    CBODY = 0, CMETA = 1, CN = 2, CT1 = 5, CT2 = 8, CCA = 11, CCB = 14, CFRIC = 17, CROLL = 18, CTWM = 19,
    CTWI = 20, CFI = 21, CRI = 23, CTM = 26, CP = 30,
    PRA = 0, PRB = 3, PBSEP = 6, PNI = 7, PTOT = 8, PNM = 9, PLEV = 10, NPF = 11,
    NCG = CP + B3_MAX_MANIFOLD * NPF,
    CSA = NCG, CSB = NCG + 1, CREST = NCG + 2, CRELV = NCG + 3, CFEAT = CRELV + B3_MAX_MANIFOLD,
    NCF = CFEAT + B3_MAX_MANIFOLD
};
// joint columns (workspace), all streamed
enum : int {
    JTYPE = 0, JBA = 1, JBB = 2, JFIX = 3, JENS = 4, JENM = 5, JENL = 6, JFPA = 7, JFPB = 10, JFQA = 13,
    JFQB = 17, JDC = 21, JSOFT = 24, JLI = 27, JAI = 30, JAM = 33, JLH = 42, JAH = 43, JLS = 44, JAS = 47,
    JPI = 50, JSI = 52, JMI = 53, JLOI = 54, JUPI = 55, JMMT = 56, JMS = 57, JTA = 58, JLA = 59, JUA = 60,
    JAX = 61, JPX = 64, JPY = 67, JAXM = 70, JSS = 71, JOK = 74, NJF = 75
};
constexpr int kBufWords = ((int)NCG > (int)NJF ? (int)NCG : (int)NJF);     // one streamed item, per lane
constexpr int kStages = 2;                              // streamed items in flight + in use

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

static inline bool layout_from_signature(unsigned long long sig, Layout* L) {
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
    unsigned off_bodies, off_bconst, off_shapes, off_contacts, off_joints;   // word offsets inside a slot
};

// ---- lane-column accessors (c points at an item's column for this lane) -----
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
B3X_HDI B3Soft lds(const float* c, int i) {
    B3Soft s;
    s.bias_rate = COL(c, i); s.mass_scale = COL(c, i + 1); s.impulse_scale = COL(c, i + 2);
    return s;
}
B3X_HDI void sts(float* c, int i, B3Soft s) {
    COL(c, i) = s.bias_rate; COL(c, i + 1) = s.mass_scale; COL(c, i + 2) = s.impulse_scale;
}
B3X_HDI int ldi(const float* c, int i) { return b3x_f2i(COL(c, i)); }
B3X_HDI void sti(float* c, int i, int v) { COL(c, i) = b3x_i2f(v); }
B3X_HDI B3Mat2 ld22(const float* c, int i) {
    B3Mat2 m;
    m.cx.x = COL(c, i); m.cx.y = COL(c, i + 1); m.cy.x = COL(c, i + 2); m.cy.y = COL(c, i + 3);
    return m;
}

// item k of a [item][field][lane] region with nf fields
B3X_HDI float* item(float* base, int k, int nf) { return base + (size_t)k * nf * kLanes; }
B3X_HDI int BI(int k, int f) { return k * NBF + f; }
B3X_HDI int PF(int p, int f) { return CP + p * NPF + f; }

B3X_HDI int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

B3X_HDI bool body_dynamic_flag(const float* bc, int k) {
    return (b3x_f2u(COL(bc, BI(k, BFLAGS))) & B3_FLAG_DYNAMIC) != 0;
}

// Body velocity write-back gated by the dynamic flag (the reference writes a
// solved body only when flags has B3_FLAG_DYNAMIC, 08_contacts.inl:405-412).
B3X_HDI void put_vel(float* bc, int k, B3Vec3 v, B3Vec3 w) {
    if (body_dynamic_flag(bc, k)) {
        st3(bc, BI(k, BV), v);
        st3(bc, BI(k, BW), w);
    }
}

// 08_contacts.inl:184-192
B3X_HDI void apply_impulse(float* bc, int k, float m, const B3Mat3& i, B3Vec3 r, B3Vec3 p, int sign) {
    if (!body_dynamic_flag(bc, k)) return;
    float s = sign > 0 ? 1.0f : -1.0f;
    st3(bc, BI(k, BV), b3_madd(ld3(bc, BI(k, BV)), s * m, p));
    st3(bc, BI(k, BW), b3_add(ld3(bc, BI(k, BW)), b3_mv(i, b3_mul(b3_cross(r, p), s))));
}

// ---- warp collectives and the streaming pipeline ---------------------------------
B3X_HDI int warp_max(int x) {
#if defined(__CUDA_ARCH__)
    return __reduce_max_sync(0xffffffffu, x);
#else
    return x;
#endif
}

struct Pipe {
    float* buf;       // kStages * kBufWords * kLanes floats of shared memory
    uint64_t* bar;    // kStages mbarriers in shared memory
    uint32_t phase;   // wait parity of each stage
    int ok;           // 0 once a wait gave up
};

#if defined(__CUDACC__)
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void pipe_init(Pipe& P) {
    if ((threadIdx.x & 31) == 0) {
        for (int s = 0; s < kStages; s++)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&P.bar[s])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    P.phase = 0;
    P.ok = 1;
}

// One elected lane: expect `bytes` on the stage's barrier and start the copy.
__device__ __forceinline__ void bulk_load(Pipe& P, int s, const float* src, uint32_t bytes) {
    float* dst = P.buf + (size_t)s * kBufWords * kLanes;
    uint32_t bar = smem_addr(&P.bar[s]);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// Bounded wait for a stage: gives up after ~2^31 cycles (about a second).
__device__ __forceinline__ bool stage_wait(Pipe& P, int s) {
    uint32_t bar = smem_addr(&P.bar[s]);
    uint32_t parity = (P.phase >> s) & 1u;
    long long t0 = clock64();
    for (;;) {
        uint32_t done;
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}" : "=r"(done) : "r"(bar), "r"(parity) : "memory");
        if (done) break;
        if (clock64() - t0 > (1ll << 31)) return false;
    }
    P.phase ^= 1u << s;
    return true;
}
#endif

// Run fn(k, col) for k in [0, n), col = item k's column for this lane, items
// read from the workspace `g` (lane-offset, `words` fields per item, the
// first `copy_words` of which fn reads).  n is warp-uniform.  On the GPU
// items arrive in shared memory through the pipeline; elsewhere they are read
// in place.  Returns false if the pipeline failed (the caller abandons the
// step); the verdict is the same on every lane.
template <class F>
B3X_HDI bool stream_items(Pipe& P, const float* g, int words, int copy_words, int n, F&& fn) {
#if defined(__CUDA_ARCH__)
    if (n <= 0) return P.ok;
    const int lane = threadIdx.x & 31;
    const size_t stride = (size_t)words * kLanes;
    const uint32_t bytes = (uint32_t)((size_t)copy_words * kLanes * sizeof(float));
    const float* g0 = g - lane;
    // this lane's earlier workspace stores must be visible to the bulk copies
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncwarp();
    if (lane == 0) bulk_load(P, 0, g0, bytes);
    for (int k = 0; k < n; k++) {
        const int s = k % kStages;
        if (lane == 0 && k + 1 < n) bulk_load(P, (k + 1) % kStages, g0 + (size_t)(k + 1) * stride, bytes);
        if (!__all_sync(0xffffffffu, stage_wait(P, s))) {
            P.ok = 0;
            // drain the copy in flight, again with a bounded wait
            if (k + 1 < n) stage_wait(P, (k + 1) % kStages);
            return false;
        }
        fn(k, (const float*)(P.buf + (size_t)s * kBufWords * kLanes + lane));
        __syncwarp();
    }
    return true;
#else
    (void)P;
    (void)copy_words;
    for (int k = 0; k < n; k++) fn(k, g + (size_t)k * words * kLanes);
    return true;
#endif
}

// ---- contact sweep (08_contacts.inl:315-413, rolling 07_packed.inl:24-45) -------
// Reads contact k from src (shared-memory copy or workspace), writes the
// solver-owned fields to dst (workspace).
B3X_HD void solve_contact(float* bc, const float* src, float* dst, float inv_h, float speed, int use_bias,
        B3Soft cs, B3Soft ss) {
    int bodies = ldi(src, CBODY), meta = ldi(src, CMETA);
    int ba = bodies & 0xffff, bb = (bodies >> 16) & 0xffff;
    int cnt = meta & 0xff;
    B3Soft soft = (meta >> 8) ? ss : cs;
    float ma = COL(bc, BI(ba, BMI)), mb = COL(bc, BI(bb, BMI));
    B3Mat3 ia = ldm(bc, BI(ba, BII)), ib = ldm(bc, BI(bb, BII));
    B3Vec3 va = ld3(bc, BI(ba, BV)), wa = ld3(bc, BI(ba, BW));
    B3Vec3 vb = ld3(bc, BI(bb, BV)), wb = ld3(bc, BI(bb, BW));
    B3Quat dqa = ldq(bc, BI(ba, BDQ)), dqb = ldq(bc, BI(bb, BDQ));
    B3Vec3 dp = b3_sub(ld3(bc, BI(bb, BDP)), ld3(bc, BI(ba, BDP)));
    B3Vec3 n = ld3(src, CN);
    float total_n = 0.0f, twist_lim = 0.0f;
    for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
        if (p >= cnt) break;
        B3Vec3 ra = ld3(src, PF(p, PRA)), rb = ld3(src, PF(p, PRB));
        B3Vec3 ds = b3_add(dp, b3_sub(b3_rotate(dqb, rb), b3_rotate(dqa, ra)));
        float sep = b3_dot(ds, n) + COL(src, PF(p, PBSEP));
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
        float ni = COL(src, PF(p, PNI));
        float dimp = -COL(src, PF(p, PNM)) * (mscale * vn + vbias) - iscale * ni;
        float nimp = b3_maxf(ni + dimp, 0.0f);
        dimp = nimp - ni;
        COL(dst, PF(p, PNI)) = nimp;
        COL(dst, PF(p, PTOT)) = COL(src, PF(p, PTOT)) + nimp;
        total_n += nimp;
        twist_lim += COL(src, PF(p, PLEV)) * nimp;
        B3Vec3 P = b3_mul(n, dimp);
        va = b3_msub(va, ma, P);
        wa = b3_sub(wa, b3_mv(ia, b3_cross(ra, P)));
        vb = b3_madd(vb, mb, P);
        wb = b3_add(wb, b3_mv(ib, b3_cross(rb, P)));
    }
    if (!use_bias) {
        float fric = COL(src, CFRIC);
        float twist_s = b3_dot(n, b3_sub(wb, wa));
        float max_t = fric * twist_lim;
        float dtw = -COL(src, CTWM) * twist_s;
        float old_t = COL(src, CTWI);
        float new_t = b3_clamp(old_t + dtw, -max_t, max_t);
        COL(dst, CTWI) = new_t;
        dtw = new_t - old_t;
        wa = b3_sub(wa, b3_mv(ia, b3_mul(n, dtw)));
        wb = b3_add(wb, b3_mv(ib, b3_mul(n, dtw)));

        B3Vec3 t1 = ld3(src, CT1), t2 = ld3(src, CT2);
        B3Vec3 ra = ld3(src, CCA), rb = ld3(src, CCB);
        B3Vec3 vra = b3_add(va, b3_cross(wa, ra)), vrb = b3_add(vb, b3_cross(wb, rb));
        B3Vec3 vr = b3_sub(vrb, vra);
        B3Vec2 vt;
        vt.x = b3_dot(vr, t1);
        vt.y = b3_dot(vr, t2);
        B3Vec2 tv = m2_mv(ld22(src, CTM), vt);
        B3Vec2 fi;
        fi.x = COL(src, CFI);
        fi.y = COL(src, CFI + 1);
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
        COL(dst, CFI) = ni.x;
        COL(dst, CFI + 1) = ni.y;
        B3Vec3 P = b3_add(b3_mul(t1, df.x), b3_mul(t2, df.y));
        va = b3_msub(va, ma, P);
        wa = b3_sub(wa, b3_mv(ia, b3_cross(ra, P)));
        vb = b3_madd(vb, mb, P);
        wb = b3_add(wb, b3_mv(ib, b3_cross(rb, P)));

        float rolling = COL(src, CROLL);
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
            B3Vec3 imp = ld3(src, CRI);
            B3Vec3 next = b3_sub(imp, b3_add(b3_mul(t1, dd.x), b3_mul(t2, dd.y)));
            float limit = rolling * total_n;
            float l2 = b3_len2(next);
            if (l2 > limit * limit && l2 > 0.0f) next = b3_mul(next, limit / sqrtf(l2));
            B3Vec3 delta = b3_sub(next, imp);
            st3(dst, CRI, next);
            wa = b3_sub(wa, b3_mv(ia, delta));
            wb = b3_add(wb, b3_mv(ib, delta));
        }
    }
    put_vel(bc, ba, va, wa);
    put_vel(bc, bb, vb, wb);
}

// ---- joints (06_joints.inl:241-642) -----------------------------------------
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
B3X_HDI void solve_point(float* bc, const float* src, float* dst, int ja, int jb, float ma, float mb,
        const B3Mat3& ia, const B3Mat3& ib, B3Vec3& va, B3Vec3& wa, B3Vec3& vb, B3Vec3& wb, B3Soft soft,
        int use_bias) {
    B3Vec3 ra = b3_rotate(ldq(bc, BI(ja, BDQ)), ld3(src, JFPA));
    B3Vec3 rb = b3_rotate(ldq(bc, BI(jb, BDQ)), ld3(src, JFPB));
    B3Vec3 cdot = b3_sub(b3_add(vb, b3_cross(wb, rb)), b3_add(va, b3_cross(wa, ra)));
    B3Vec3 bias = b3_v(0.0f, 0.0f, 0.0f);
    float mscale = 1.0f, iscale = 0.0f;
    if (use_bias) {
        B3Vec3 sep = b3_add(b3_add(b3_sub(ld3(bc, BI(jb, BDP)), ld3(bc, BI(ja, BDP))), b3_sub(rb, ra)),
            ld3(src, JDC));
        bias = b3_mul(sep, soft.bias_rate);
        mscale = soft.mass_scale;
        iscale = soft.impulse_scale;
    }
    B3Vec3 b = b3_mv(m3_inv(point_k(ma, mb, ia, ib, ra, rb)), b3_add(cdot, bias));
    B3Vec3 li = ld3(src, JLI);
    B3Vec3 impulse = b3_msub(b3_mul(b, -mscale), iscale, li);
    st3(dst, JLI, b3_add(li, impulse));
    va = b3_msub(va, ma, impulse);
    wa = b3_sub(wa, b3_mv(ia, b3_cross(ra, impulse)));
    vb = b3_madd(vb, mb, impulse);
    wb = b3_add(wb, b3_mv(ib, b3_cross(rb, impulse)));
}

// 06_joints.inl:419-434
B3X_HDI float limit_impulse(float c, float cdot, float inv_h, int use_bias, B3Soft soft, float axial_mass,
        float old) {
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

// One joint, either type (dispatch 07_packed.inl:66-79; weld 06_joints.inl:285-332;
// revolute 06_joints.inl:436-642, default uncached path).
B3X_HD void solve_joint(float* bc, const float* src, float* dst, float h, float inv_h, int use_bias) {
    int type = ldi(src, JTYPE);
    int ja = ldi(src, JBA), jb = ldi(src, JBB);
    float ma = COL(bc, BI(ja, BMI)), mb = COL(bc, BI(jb, BMI));
    B3Mat3 ia = ldm(bc, BI(ja, BII)), ib = ldm(bc, BI(jb, BII));
    B3Vec3 va = ld3(bc, BI(ja, BV)), wa = ld3(bc, BI(ja, BW));
    B3Vec3 vb = ld3(bc, BI(jb, BV)), wb = ld3(bc, BI(jb, BW));
    int fixed = ldi(src, JFIX);
    B3Quat qa = b3_qmul(ldq(bc, BI(ja, BDQ)), ldq(src, JFQA));
    B3Quat qb = b3_qmul(ldq(bc, BI(jb, BDQ)), ldq(src, JFQB));
    if (b3_qdot(qa, qb) < 0.0f) qb = b3_qneg(qb);
    B3Quat rel = b3_qinv_mul(qa, qb);
    if (type == B3_JOINT_WELD) {
        float ah = COL(src, JAH);
        if (!fixed) {
            B3Vec3 bias = b3_v(0.0f, 0.0f, 0.0f);
            float mscale = 1.0f, iscale = 0.0f;
            if (use_bias || ah > 0.0f) {
                B3Quat s = rel;
                if (rel.s < 0.0f) s = b3_qneg(rel);
                B3Quat diff = b3_q(-s.v.x, -s.v.y, -s.v.z, 1.0f - s.s);
                B3Vec3 c = b3_neg(b3_rotate(qa, b3_mul(b3_qmul(diff, b3_qconj(s)).v, 2.0f)));
                B3Soft as = lds(src, JAS);
                bias = b3_mul(c, as.bias_rate);
                mscale = as.mass_scale;
                iscale = as.impulse_scale;
            }
            B3Vec3 cdot = b3_sub(wb, wa);
            B3Vec3 ai = ld3(src, JAI);
            B3Vec3 impulse = b3_msub(b3_mul(b3_mv(ldm(src, JAM), b3_add(cdot, bias)), -mscale), iscale, ai);
            st3(dst, JAI, b3_add(ai, impulse));
            wa = b3_sub(wa, b3_mv(ia, impulse));
            wb = b3_add(wb, b3_mv(ib, impulse));
        }
        int lin_bias = use_bias || COL(src, JLH) > 0.0f;
        solve_point(bc, src, dst, ja, jb, ma, mb, ia, ib, va, wa, vb, wb, lds(src, JLS), lin_bias);
        put_vel(bc, ja, va, wa);
        put_vel(bc, jb, vb, wb);
        return;
    }
    B3Vec3 axis = ld3(src, JAX);
    B3Vec3 ia_ax = b3_v(0.0f, 0.0f, 0.0f), ib_ax = b3_v(0.0f, 0.0f, 0.0f);
    float twist = 0.0f;
    int en_spring = ldi(src, JENS), en_motor = ldi(src, JENM), en_limit = ldi(src, JENL);
    int need_twist = (en_spring || en_limit || en_motor) && !fixed;
    if (!fixed) {
        ia_ax = b3_mv(ia, axis);
        ib_ax = b3_mv(ib, axis);
    }
    if (need_twist) twist = b3_twist(rel);
    float axial_mass = COL(src, JAXM);
    float mmt = COL(src, JMMT);
    if (en_spring && !fixed) {
        B3Soft ss = lds(src, JSS);
        float c = twist - COL(src, JTA);
        float bias = ss.bias_rate * c;
        float cdot = b3_dot(b3_sub(wb, wa), axis);
        float old = COL(src, JSI);
        float dimp = -ss.mass_scale * axial_mass * (cdot + bias) - ss.impulse_scale * old;
        float nimp = old + dimp;
        if (mmt > 0.0f) {
            float maxp = mmt * h;
            nimp = b3_clamp(nimp, -maxp, maxp);
        }
        dimp = nimp - old;
        COL(dst, JSI) = nimp;
        wa = b3_msub(wa, dimp, ia_ax);
        wb = b3_madd(wb, dimp, ib_ax);
    }
    if (en_motor && !fixed) {
        float speed = COL(src, JMS);
        int blocked = 0;
        if (en_limit) {
            if (twist >= COL(src, JUA) - 0.01f && speed > 0.0f) blocked = 1;
            if (twist <= COL(src, JLA) + 0.01f && speed < 0.0f) blocked = 1;
        }
        if (blocked) {
            COL(dst, JMI) = 0.0f;
        } else {
            float cdot = b3_dot(b3_sub(wb, wa), axis) - speed;
            float dimp = -axial_mass * cdot;
            float old = COL(src, JMI);
            float nimp = old + dimp;
            float maxp = mmt * h;
            nimp = b3_clamp(nimp, -maxp, maxp);
            dimp = nimp - old;
            COL(dst, JMI) = nimp;
            wa = b3_msub(wa, dimp, ia_ax);
            wb = b3_madd(wb, dimp, ib_ax);
        }
    }
    B3Soft soft = lds(src, JSOFT);
    if (en_limit && !fixed) {
        float old = COL(src, JLOI);
        float lo = limit_impulse(twist - COL(src, JLA), b3_dot(b3_sub(wb, wa), axis), inv_h, use_bias, soft,
            axial_mass, old);
        COL(dst, JLOI) = lo;
        float dimp = lo - old;
        wa = b3_msub(wa, dimp, ia_ax);
        wb = b3_madd(wb, dimp, ib_ax);
        old = COL(src, JUPI);
        float up = limit_impulse(COL(src, JUA) - twist, b3_dot(b3_sub(wa, wb), axis), inv_h, use_bias, soft,
            axial_mass, old);
        COL(dst, JUPI) = up;
        dimp = up - old;
        wa = b3_madd(wa, dimp, ia_ax);
        wb = b3_msub(wb, dimp, ib_ax);
    }
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
        st3(dst, JPX, px);
        st3(dst, JPY, py);
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
        old.x = COL(src, JPI);
        old.y = COL(src, JPI + 1);
        B3Vec2 dimp;
        dimp.x = -mscale * sol.x - iscale * old.x;
        dimp.y = -mscale * sol.y - iscale * old.y;
        COL(dst, JPI) = old.x + dimp.x;
        COL(dst, JPI + 1) = old.y + dimp.y;
        B3Vec3 ang = b3_add(b3_mul(px, dimp.x), b3_mul(py, dimp.y));
        wa = b3_sub(wa, b3_mv(ia, ang));
        wb = b3_add(wb, b3_mv(ib, ang));
    }
    solve_point(bc, src, dst, ja, jb, ma, mb, ia, ib, va, wa, vb, wb, soft, use_bias);
    put_vel(bc, ja, va, wa);
    put_vel(bc, jb, vb, wb);
}

// ---- one warp of worlds, one step ---------------------------------------------
// live: this lane holds a world to step.  bc: body columns, kc: body step
// constants, sc / cc / jc: shape / contact / joint workspace regions (all
// lane-offset).  Returns false when the pipeline failed.
B3X_HD bool world_step(bool live, unsigned char* wp, const StepArgs& a, float* bc, float* kc, float* sc,
        float* cc, float* jc, Pipe& P) {
    const Layout& L = a.L;
    Header* hd = reinterpret_cast<Header*>(wp);
    B3Body* bodies = reinterpret_cast<B3Body*>(wp + B3X_WORLD_HEADER_BYTES);
    B3Shape* shapes = reinterpret_cast<B3Shape*>(wp + L.shape_off);
    B3Contact* contacts = reinterpret_cast<B3Contact*>(wp + L.contact_off);
    B3Joint* joints = reinterpret_cast<B3Joint*>(wp + L.joint_off);

    // Counts beyond the capacities would index past the arrays in the
    // reference; here they are clamped so a corrupt world cannot fault.
    const int nb = live ? clampi(hd->body_count, 0, L.B) : 0;
    const int ns = live ? clampi(hd->shape_count, 0, L.S) : 0;
    const int old_n = live ? clampi(hd->contact_count, 0, L.C) : 0;
    const int nj = live ? clampi(hd->joint_count, 0, L.J) : 0;

    // 09_step.inl:148-157
    const int subs = a.substeps;
    const float dt = a.dt;
    const float h = dt / (float)subs;
    const float inv_dt = 1.0f / dt;
    const float inv_h = (float)subs * inv_dt;
    const float contact_hertz = live ? hd->contact_hertz : 0.0f;
    const float contact_damping = live ? hd->contact_damping : 0.0f;
    const float hertz = b3_minf(contact_hertz, 0.25f * inv_h);
    const B3Soft cs = make_soft(hertz, contact_damping, h);
    const B3Soft ss = make_soft(2.0f * hertz, 0.5f * contact_damping, h);
    const float contact_speed = live ? hd->contact_speed : 0.0f;
    const B3Vec3 gravity = live ? hd->gravity : b3_v(0.0f, 0.0f, 0.0f);

    // -- bodies into working columns (inverse mass / inertia gated by type as
    //    the contact and joint prepares do, 08_contacts.inl:236-239), and the
    //    velocity increments that stay constant over the substeps
    //    (09_step.inl:5-18)
    for (int k = 0; k < nb; k++) {
        const B3Body* b = &bodies[k];
        int type = b->type;
        bool dyn = type == B3_DYNAMIC;
        st3(bc, BI(k, BV), b->lin_vel);
        st3(bc, BI(k, BW), b->ang_vel);
        st3(bc, BI(k, BDP), b->delta_pos);
        stq(bc, BI(k, BDQ), b->delta_rot);
        COL(bc, BI(k, BFLAGS)) = b3x_u2f(b->flags);
        sti(bc, BI(k, BTYPE), type);
        if (dyn) {
            float inv_mass = b->inv_mass;
            B3Mat3 iw = b->inv_i_world;
            COL(bc, BI(k, BMI)) = inv_mass;
            stm(bc, BI(k, BII), iw);
            float* kk = item(kc, k, NKF);
            float gs = inv_mass > 0.0f ? b->gravity_scale : 0.0f;
            st3(kk, KDV, b3_add(b3_mul(b->force, h * inv_mass), b3_mul(gravity, h * gs)));
            st3(kk, KDW, b3_mul(b3_mv(iw, b->torque), h));
            COL(kk, KLD) = 1.0f / (1.0f + h * b->linear_damping);
            COL(kk, KAD) = 1.0f / (1.0f + h * b->angular_damping);
        } else {
            COL(bc, BI(k, BMI)) = 0.0f;
            stm(bc, BI(k, BII), m3_zero());
        }
    }

    // -- shape world poses and padded AABBs (04_world.inl:293-336,
    //    08_contacts.inl:109-114); a shape on an invalid body never overlaps
    for (int s = 0; s < ns; s++) {
        const B3Shape* sh = &shapes[s];
        float* so = item(sc, s, NSF);
        int body = sh->body;
        if (body < 0 || body >= nb) {
            st3(so, SLO, b3_v(INFINITY, INFINITY, INFINITY));
            st3(so, SHI, b3_v(-INFINITY, -INFINITY, -INFINITY));
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
        st3(so, SPOS, p);
        stq(so, SROT, q);
        st3(so, SLO, b3_sub(lo, pad));
        st3(so, SHI, b3_add(hi, pad));
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
    int overflow = live ? hd->contact_overflow : 0, dropped = live ? hd->contacts_dropped : 0;
    for (int i = 0; i < ns; i++) {
        const B3Shape* si = &shapes[i];
        const int body_i = si->body;
        if (body_i < 0 || body_i >= nb) continue;
        const float* soi = item(sc, i, NSF);
        const B3Vec3 lo_i = ld3(soi, SLO), hi_i = ld3(soi, SHI);
        const int btype_i = ldi(bc, BI(body_i, BTYPE));
        for (int j = i + 1; j < ns; j++) {
            const float* soj = item(sc, j, NSF);
            const B3Vec3 lo_j = ld3(soj, SLO), hi_j = ld3(soj, SHI);
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
            ga.p = ld3(soi, SPOS); ga.q = ldq(soi, SROT); ga.type = si->type;
            ga.radius = si->radius; ga.half = si->half;
            gb.p = ld3(soj, SPOS); gb.q = ldq(soj, SROT); gb.type = sj->type;
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
            float* co = item(cc, n, NCF);
            B3Vec3 nrm = m.normal;
            B3Vec3 t1 = b3_perp(nrm);
            B3Vec3 t2 = b3_cross(t1, nrm);
            sti(co, CSA, i);
            sti(co, CSB, j);
            sti(co, CBODY, (body_i & 0xffff) | (body_j << 16));
            sti(co, CMETA, m.count | ((btype_i != B3_DYNAMIC || btype_j != B3_DYNAMIC) ? 0x100 : 0));
            st3(co, CN, nrm);
            st3(co, CT1, t1);
            st3(co, CT2, t2);
            COL(co, CFRIC) = sqrtf(si->friction * sj->friction);
            COL(co, CREST) = si->restitution > sj->restitution ? si->restitution : sj->restitution;
            COL(co, CROLL) = b3_maxf(si->rolling, sj->rolling);
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
                st3(co, PF(p, PRA), ra);
                st3(co, PF(p, PRB), rb);
                COL(co, PF(p, PBSEP)) = m.sep[p] - b3_dot(b3_sub(rb, ra), nrm);
                sti(co, CFEAT + p, (int)m.feat[p]);
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
                if (p < m.count) COL(co, PF(p, PNI)) = ni[p];
            COL(co, CFI) = fi.x;
            COL(co, CFI + 1) = fi.y;
            COL(co, CTWI) = twi;
            st3(co, CRI, ri);
            n++;
        }
    }

    // -- prepare contacts (08_contacts.inl:234-291); the prepared fields are
    //    final for the step, so they go to the world now (the old cache is dead)
    const float inv_tau = 1.0f / B3_SPECULATIVE;
    for (int k = 0; k < n; k++) {
        B3Contact* oc = &contacts[k];
        float* co = item(cc, k, NCF);
        int bodies_k = ldi(co, CBODY), meta = ldi(co, CMETA);
        int ba = bodies_k & 0xffff, bb = (bodies_k >> 16) & 0xffff;
        int cnt = meta & 0xff;
        int stat = meta >> 8;
        float ma = COL(bc, BI(ba, BMI)), mb = COL(bc, BI(bb, BMI));
        B3Mat3 ia = ldm(bc, BI(ba, BII)), ib = ldm(bc, BI(bb, BII));
        B3Vec3 va = ld3(bc, BI(ba, BV)), wa = ld3(bc, BI(ba, BW));
        B3Vec3 vb = ld3(bc, BI(bb, BV)), wb = ld3(bc, BI(bb, BW));
        B3Vec3 nrm = ld3(co, CN);
        B3Vec3 t1 = ld3(co, CT1), t2 = ld3(co, CT2);
        B3Vec3 center_a = b3_v(0.0f, 0.0f, 0.0f), center_b = b3_v(0.0f, 0.0f, 0.0f);
        float wsum = 0.0f;
        for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
            if (p >= cnt) break;
            B3Vec3 ra = ld3(co, PF(p, PRA)), rb = ld3(co, PF(p, PRB));
            B3Vec3 rn_a = b3_cross(ra, nrm), rn_b = b3_cross(rb, nrm);
            float kn = ma + mb + b3_dot(rn_a, b3_mv(ia, rn_a)) + b3_dot(rn_b, b3_mv(ib, rn_b));
            float nm = kn > 0.0f ? 1.0f / kn : 0.0f;
            B3Vec3 vra = b3_add(va, b3_cross(wa, ra)), vrb = b3_add(vb, b3_cross(wb, rb));
            float relv = b3_dot(nrm, b3_sub(vrb, vra));
            float base_sep = COL(co, PF(p, PBSEP));
            float sep = base_sep + b3_dot(b3_sub(rb, ra), nrm);
            float wgt = b3_clamp(2.0f - sep * inv_tau, B3_MIN_FRICTION_W, 1.0f);
            center_a = b3_madd(center_a, wgt, ra);
            center_b = b3_madd(center_b, wgt, rb);
            wsum += wgt;
            COL(co, PF(p, PNM)) = nm;
            COL(co, CRELV + p) = relv;
            COL(co, PF(p, PTOT)) = 0.0f;
            B3Point* op = &oc->points[p];
            op->r_a = ra;
            op->r_b = rb;
            op->base_sep = base_sep;
            op->rel_vel = relv;
            op->normal_mass = nm;
            op->feature = (uint32_t)ldi(co, CFEAT + p);
        }
        float invw = wsum > 0.0f ? 1.0f / wsum : 0.0f;
        B3Vec3 ca = b3_mul(center_a, invw), cb = b3_mul(center_b, invw);
        for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
            if (p >= cnt) break;
            float lev = b3_len(b3_sub(ld3(co, PF(p, PRA)), ca));
            COL(co, PF(p, PLEV)) = lev;
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
        st3(co, CCA, ca);
        st3(co, CCB, cb);
        COL(co, CTM) = tm.cx.x;
        COL(co, CTM + 1) = tm.cx.y;
        COL(co, CTM + 2) = tm.cy.x;
        COL(co, CTM + 3) = tm.cy.y;
        COL(co, CTWM) = twm;
        oc->shape_a = ldi(co, CSA);
        oc->shape_b = ldi(co, CSB);
        oc->body_a = ba;
        oc->body_b = bb;
        oc->point_count = cnt;
        oc->static_contact = stat;
        oc->normal = nrm;
        oc->tangent1 = t1;
        oc->tangent2 = t2;
        oc->center_a = ca;
        oc->center_b = cb;
        oc->friction = COL(co, CFRIC);
        oc->restitution = COL(co, CREST);
        oc->rolling = COL(co, CROLL);
        oc->twist_mass = twm;
        oc->tangent_mass = tm;
        oc->rolling_mass = m3_inv(isum);
        oc->inv_mass_a = ma;
        oc->inv_mass_b = mb;
        oc->inv_i_a = ia;
        oc->inv_i_b = ib;
        oc->softness = stat ? ss : cs;
    }

    // -- prepare joints (06_joints.inl:161-202); invalid body indices make the
    //    joint inert (the reference would index out of bounds)
    for (int q = 0; q < nj; q++) {
        B3Joint* jt = &joints[q];
        float* jo = item(jc, q, NJF);
        int type = jt->type, ja = jt->body_a, jb = jt->body_b;
        if (ja < 0 || ja >= nb || jb < 0 || jb >= nb) {
            sti(jo, JOK, 0);
            continue;
        }
        sti(jo, JOK, 1);
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
        sti(jo, JTYPE, type);
        sti(jo, JBA, ja);
        sti(jo, JBB, jb);
        sti(jo, JFIX, fixed);
        st3(jo, JFPA, fpa);
        st3(jo, JFPB, fpb);
        stq(jo, JFQA, fqa);
        stq(jo, JFQB, fqb);
        st3(jo, JDC, dc);
        sts(jo, JSOFT, soft);
        st3(jo, JLI, jt->linear_impulse);
        if (type == B3_JOINT_WELD) {
            float lh = jt->linear_hertz, ah = jt->angular_hertz;
            B3Mat3 am = m3_inv(isum);
            B3Soft ls = lh == 0.0f ? soft : make_soft(lh, jt->linear_damping, h);
            B3Soft as = ah == 0.0f ? soft : make_soft(ah, jt->angular_damping, h);
            jt->angular_mass = am;
            jt->linear_spring = ls;
            jt->angular_spring = as;
            stm(jo, JAM, am);
            COL(jo, JLH) = lh;
            COL(jo, JAH) = ah;
            sts(jo, JLS, ls);
            sts(jo, JAS, as);
            st3(jo, JAI, jt->angular_impulse);
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
            st3(jo, JAX, axis);
            COL(jo, JAXM) = axm;
            st3(jo, JPX, px);
            st3(jo, JPY, py);
            sts(jo, JSS, sps);
            sti(jo, JENS, jt->enable_spring);
            sti(jo, JENM, jt->enable_motor);
            sti(jo, JENL, jt->enable_limit);
            COL(jo, JPI) = jt->perp_impulse.x;
            COL(jo, JPI + 1) = jt->perp_impulse.y;
            COL(jo, JSI) = jt->spring_impulse;
            COL(jo, JMI) = jt->motor_impulse;
            COL(jo, JLOI) = jt->lower_impulse;
            COL(jo, JUPI) = jt->upper_impulse;
            COL(jo, JMMT) = jt->max_motor_torque;
            COL(jo, JMS) = jt->motor_speed;
            COL(jo, JTA) = jt->target_angle;
            COL(jo, JLA) = jt->lower_angle;
            COL(jo, JUA) = jt->upper_angle;
            if (type != B3_JOINT_REVOLUTE) st3(jo, JAI, jt->angular_impulse);
        }
    }

    // -- warm start contacts (08_contacts.inl:194-232, 293-313)
    for (int k = 0; k < n; k++) {
        const float* co = item(cc, k, NCF);
        int bodies_k = ldi(co, CBODY);
        int ba = bodies_k & 0xffff, bb = (bodies_k >> 16) & 0xffff;
        int cnt = ldi(co, CMETA) & 0xff;
        float ma = COL(bc, BI(ba, BMI)), mb = COL(bc, BI(bb, BMI));
        B3Mat3 ia = ldm(bc, BI(ba, BII)), ib = ldm(bc, BI(bb, BII));
        B3Vec3 nrm = ld3(co, CN);
        for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
            if (p >= cnt) break;
            B3Vec3 P = b3_mul(nrm, COL(co, PF(p, PNI)));
            apply_impulse(bc, ba, ma, ia, ld3(co, PF(p, PRA)), P, -1);
            apply_impulse(bc, bb, mb, ib, ld3(co, PF(p, PRB)), P, 1);
        }
        B3Vec3 f = b3_add(b3_mul(ld3(co, CT1), COL(co, CFI)), b3_mul(ld3(co, CT2), COL(co, CFI + 1)));
        apply_impulse(bc, ba, ma, ia, ld3(co, CCA), f, -1);
        apply_impulse(bc, bb, mb, ib, ld3(co, CCB), f, 1);
        B3Vec3 tr = b3_add(b3_mul(nrm, COL(co, CTWI)), ld3(co, CRI));
        if (body_dynamic_flag(bc, ba)) st3(bc, BI(ba, BW), b3_sub(ld3(bc, BI(ba, BW)), b3_mv(ia, tr)));
        if (body_dynamic_flag(bc, bb)) st3(bc, BI(bb, BW), b3_add(ld3(bc, BI(bb, BW)), b3_mv(ib, tr)));
    }

    // -- warm start joints (06_joints.inl:204-239)
    for (int q = 0; q < nj; q++) {
        const float* jo = item(jc, q, NJF);
        if (!ldi(jo, JOK)) continue;
        int type = ldi(jo, JTYPE);
        int ja = ldi(jo, JBA), jb = ldi(jo, JBB);
        float ma = COL(bc, BI(ja, BMI)), mb = COL(bc, BI(jb, BMI));
        B3Mat3 ia = ldm(bc, BI(ja, BII)), ib = ldm(bc, BI(jb, BII));
        B3Vec3 ra = b3_rotate(ldq(bc, BI(ja, BDQ)), ld3(jo, JFPA));
        B3Vec3 rb = b3_rotate(ldq(bc, BI(jb, BDQ)), ld3(jo, JFPB));
        B3Vec3 li = ld3(jo, JLI);
        B3Vec3 ang;
        if (type == B3_JOINT_REVOLUTE) {
            float axial = COL(jo, JSI) + COL(jo, JMI) + COL(jo, JLOI) - COL(jo, JUPI);
            ang = b3_add(b3_mul(ld3(jo, JPX), COL(jo, JPI)), b3_mul(ld3(jo, JPY), COL(jo, JPI + 1)));
            ang = b3_madd(ang, axial, ld3(jo, JAX));
        } else {
            ang = ld3(jo, JAI);
        }
        if (body_dynamic_flag(bc, ja)) {
            st3(bc, BI(ja, BV), b3_msub(ld3(bc, BI(ja, BV)), ma, li));
            st3(bc, BI(ja, BW), b3_sub(ld3(bc, BI(ja, BW)), b3_mv(ia, b3_add(b3_cross(ra, li), ang))));
        }
        if (body_dynamic_flag(bc, jb)) {
            st3(bc, BI(jb, BV), b3_madd(ld3(bc, BI(jb, BV)), mb, li));
            st3(bc, BI(jb, BW), b3_add(ld3(bc, BI(jb, BW)), b3_mv(ib, b3_add(b3_cross(rb, li), ang))));
        }
    }

    // -- substeps (09_step.inl:167-181).  The sweeps are warp-uniform over the
    //    largest contact / joint count of the warp's worlds.
    const int wn = warp_max(n), wj = warp_max(nj);
    const float max_lin = live ? hd->max_linear_speed : 0.0f;
    const float max_ang = B3_MAX_ROTATION * inv_dt;
    const float max_lin2 = max_lin * max_lin, max_ang2 = max_ang * max_ang;
    const float restitution_threshold = live ? hd->restitution_threshold : 0.0f;
    auto contact_pass = [&](int use_bias) {
        return stream_items(P, cc, NCF, NCG, wn, [&](int k, const float* src) {
            if (k < n) solve_contact(bc, src, item(cc, k, NCF), inv_h, contact_speed, use_bias, cs, ss);
        });
    };
    auto joint_pass = [&](int use_bias) {
        return stream_items(P, jc, NJF, NJF, wj, [&](int q, const float* src) {
            if (q < nj && ldi(src, JOK)) solve_joint(bc, src, item(jc, q, NJF), h, inv_h, use_bias);
        });
    };
    for (int s = 0; s < subs; s++) {
        // integrate velocities (09_step.inl:5-18, 41-53) with the step constants
        for (int k = 0; k < nb; k++) {
            if (ldi(bc, BI(k, BTYPE)) != B3_DYNAMIC) continue;
            const float* kk = item(kc, k, NKF);
            st3(bc, BI(k, BV), b3_madd(ld3(kk, KDV), COL(kk, KLD), ld3(bc, BI(k, BV))));
            st3(bc, BI(k, BW), b3_madd(ld3(kk, KDW), COL(kk, KAD), ld3(bc, BI(k, BW))));
        }
        if (!contact_pass(1)) return false;
        for (int it = 0; it < a.joint_iters; it++)
            if (!joint_pass(1)) return false;
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
        if (!contact_pass(0)) return false;
        for (int it = 0; it < a.relax_iters; it++)
            if (!joint_pass(0)) return false;
        // restitution (08_contacts.inl:439-480)
        for (int k = 0; k < n; k++) {
            float* co = item(cc, k, NCF);
            float rest = COL(co, CREST);
            if (rest == 0.0f) continue;
            int bodies_k = ldi(co, CBODY);
            int ba = bodies_k & 0xffff, bb = (bodies_k >> 16) & 0xffff;
            int cnt = ldi(co, CMETA) & 0xff;
            float ma = COL(bc, BI(ba, BMI)), mb = COL(bc, BI(bb, BMI));
            B3Mat3 ia = ldm(bc, BI(ba, BII)), ib = ldm(bc, BI(bb, BII));
            B3Vec3 va = ld3(bc, BI(ba, BV)), wa = ld3(bc, BI(ba, BW));
            B3Vec3 vb = ld3(bc, BI(bb, BV)), wb = ld3(bc, BI(bb, BW));
            B3Vec3 nrm = ld3(co, CN);
            for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
                if (p >= cnt) break;
                float relv = COL(co, CRELV + p);
                if (relv > -restitution_threshold || COL(co, PF(p, PTOT)) == 0.0f) continue;
                B3Vec3 ra = ld3(co, PF(p, PRA)), rb = ld3(co, PF(p, PRB));
                B3Vec3 vra = b3_add(va, b3_cross(wa, ra)), vrb = b3_add(vb, b3_cross(wb, rb));
                float vn = b3_dot(b3_sub(vrb, vra), nrm);
                float ni = COL(co, PF(p, PNI));
                float imp = -COL(co, PF(p, PNM)) * (vn + rest * relv);
                float nimp = b3_maxf(ni + imp, 0.0f);
                imp = nimp - ni;
                COL(co, PF(p, PNI)) = nimp;
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
        if (type != B3_STATIC || body_dynamic_flag(bc, k)) {
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
        const float* co = item(cc, k, NCF);
        int cnt = ldi(co, CMETA) & 0xff;
        for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
            if (p >= cnt) break;
            oc->points[p].normal_impulse = COL(co, PF(p, PNI));
            oc->points[p].total_normal = COL(co, PF(p, PTOT));
        }
        oc->twist_impulse = COL(co, CTWI);
        oc->friction_impulse.x = COL(co, CFI);
        oc->friction_impulse.y = COL(co, CFI + 1);
        oc->rolling_impulse = ld3(co, CRI);
    }
    for (int q = 0; q < nj; q++) {
        const float* jo = item(jc, q, NJF);
        if (!ldi(jo, JOK)) continue;
        int type = ldi(jo, JTYPE);
        B3Joint* jt = &joints[q];
        jt->linear_impulse = ld3(jo, JLI);
        if (type == B3_JOINT_WELD) {
            jt->angular_impulse = ld3(jo, JAI);
        } else {
            jt->perp_impulse.x = COL(jo, JPI);
            jt->perp_impulse.y = COL(jo, JPI + 1);
            jt->spring_impulse = COL(jo, JSI);
            jt->motor_impulse = COL(jo, JMI);
            jt->lower_impulse = COL(jo, JLOI);
            jt->upper_impulse = COL(jo, JUPI);
            jt->perp_x = ld3(jo, JPX);
            jt->perp_y = ld3(jo, JPY);
        }
    }
    if (live) {
        hd->contact_count = n;
        hd->contact_overflow = overflow;
        hd->contacts_dropped = dropped;
    }
    return true;
}

}  // namespace b3x
