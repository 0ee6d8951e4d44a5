// b3x_solver.cuh -- the per-world solver of the batched step: warm starts,
// the substep loop with its Gauss-Seidel sweeps over contacts and joints,
// restitution, velocity / position integration (run by solve_kernel, one warp
// per tile of 32 worlds, lane = world).
//
// Body state lives in lane-interleaved columns (shared memory when the
// capacities allow it).  The sweeps are warp-uniform: item k of all 32
// worlds is one contiguous block of the workspace ([field][lane]), and a TMA
// bulk copy (cp.async.bulk + mbarrier) streams block k+1 into shared memory
// while the lanes solve block k, so the sweeps read their operands from
// shared memory only.  Solver-owned fields go back to the workspace with
// ordinary coalesced stores, made visible to the next pass's bulk copies by a
// proxy fence.
//
// Arithmetic keeps the reference's operation order (file:line cited, paths
// relative to the reference repository root); see b3x_step.cu for the build
// flags that make it bit-exact.  Functions are __host__ __device__ so that
// development tools can also run the per-world logic on the host (there the
// sweeps read the workspace in place).
#pragma once
#include <cstdint>
#include <type_traits>

#include "b3x_layout.cuh"

namespace b3x {

#ifndef B3X_STAGES
#define B3X_STAGES 2
#endif
constexpr int kStages = B3X_STAGES;   // streamed items in flight + in use

B3X_HDI bool body_dynamic_flag(const float* __restrict__ bk, int k) {
    return (b3x_f2u(COL(bk, BK(k, BFLAGS))) & B3_FLAG_DYNAMIC) != 0;
}

// Body velocity write-back gated by the dynamic flag (the reference writes a
// solved body only when flags has B3_FLAG_DYNAMIC, 08_contacts.inl:405-412).
B3X_HDI void put_vel(float* __restrict__ bc, const float* __restrict__ bk, int k, B3Vec3 v, B3Vec3 w) {
    if (body_dynamic_flag(bk, k)) {
        st3(bc, BI(k, BV), v);
        st3(bc, BI(k, BW), w);
    }
}

// ---- warp collectives and the streaming pipeline ---------------------------------
B3X_HDI int warp_max(int x) {
#if defined(__CUDA_ARCH__)
    return __reduce_max_sync(0xffffffffu, x);
#else
    return x;
#endif
}

B3X_HDI bool warp_any(bool x) {
#if defined(__CUDA_ARCH__)
    return __any_sync(0xffffffffu, x) != 0;
#else
    return x;
#endif
}

struct Pipe {
    float* buf;       // kStages * kStreamWords * kLanes floats of shared memory
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
    float* dst = P.buf + (size_t)s * kStreamWords * kLanes;
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

// Copy one block of `bytes` into stage s and wait for it (same bookkeeping as
// a streamed item).  Returns false if the wait gave up.
__device__ __forceinline__ bool load_block(Pipe& P, int s, const float* src, uint32_t bytes) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) bulk_load(P, s, src, bytes);
    if (!__all_sync(0xffffffffu, stage_wait(P, s))) {
        P.ok = 0;
        return false;
    }
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
        fn(k, (const float*)(P.buf + (size_t)s * kStreamWords * kLanes + lane));
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

// ---- contacts -----------------------------------------------------------------
// Warm start one contact (08_contacts.inl:194-232, 293-313), with the two
// bodies' velocities kept in registers across the contact's impulses (each
// body's updates in the reference's order).
B3X_HDI void warm_contact(float* __restrict__ bc, const float* __restrict__ bk, const float* __restrict__ src) {
    int ba = ldi(src, WBA), bb = ldi(src, WBB);
    int cnt = ldi(src, WCNT);
    float ma = COL(bk, BK(ba, BMI)), mb = COL(bk, BK(bb, BMI));
    B3Mat3 ia = ldm(bk, BK(ba, BII)), ib = ldm(bk, BK(bb, BII));
    const bool da = body_dynamic_flag(bk, ba), db = body_dynamic_flag(bk, bb);
    B3Vec3 va = ld3(bc, BI(ba, BV)), wa = ld3(bc, BI(ba, BW));
    B3Vec3 vb = ld3(bc, BI(bb, BV)), wb = ld3(bc, BI(bb, BW));
    auto impulse = [](B3Vec3& v, B3Vec3& w, float m, const B3Mat3& i, B3Vec3 r, B3Vec3 p, float s) {
        v = b3_madd(v, s * m, p);
        w = b3_add(w, b3_mv(i, b3_mul(b3_cross(r, p), s)));
    };
    B3Vec3 nrm = ld3(src, WN);
    for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
        if (p >= cnt) break;
        B3Vec3 P = b3_mul(nrm, COL(src, PW(p, QNI)));
        if (da) impulse(va, wa, ma, ia, ld3(src, PW(p, QRA)), P, -1.0f);
        if (db) impulse(vb, wb, mb, ib, ld3(src, PW(p, QRB)), P, 1.0f);
    }
    B3Vec3 f = b3_add(b3_mul(ld3(src, WT1), COL(src, WFI)), b3_mul(ld3(src, WT2), COL(src, WFI + 1)));
    if (da) impulse(va, wa, ma, ia, ld3(src, WCA), f, -1.0f);
    if (db) impulse(vb, wb, mb, ib, ld3(src, WCB), f, 1.0f);
    B3Vec3 tr = b3_add(b3_mul(nrm, COL(src, WTWI)), ld3(src, WRI));
    if (da) {
        st3(bc, BI(ba, BV), va);
        st3(bc, BI(ba, BW), b3_sub(wa, b3_mv(ia, tr)));
    }
    if (db) {
        st3(bc, BI(bb, BV), vb);
        st3(bc, BI(bb, BW), b3_add(wb, b3_mv(ib, tr)));
    }
}

// Sweeps over the contacts.  Positions change only between a substep's bias
// and relax sweeps, so a point's separation is computed by the first sweep
// after a position change (kBiasFresh in the first substep, kRelax) and
// stored; the sweeps before the next change read it (kBiasCached, and
// kRelaxCached for the further relax sweeps of the interleaved mode).
enum : int { kBiasFresh = 0, kBiasCached = 1, kRelax = 2, kRelaxCached = 3 };

// One contact of a sweep (08_contacts.inl:315-413, rolling 07_packed.inl:24-45).
// Reads contact k from src (shared-memory copy or workspace), writes the
// solver-owned fields to dst (workspace).
template <int kPass>
B3X_HDI void solve_contact(float* __restrict__ bc, const float* __restrict__ bp, const float* __restrict__ bk,
        const float* __restrict__ src, float* __restrict__ dst, float inv_h, float speed, B3Soft cs, B3Soft ss) {
    constexpr bool use_bias = kPass == kBiasFresh || kPass == kBiasCached;
    constexpr bool cached = kPass == kBiasCached || kPass == kRelaxCached;
    int ba = ldi(src, WBA), bb = ldi(src, WBB);
    int cnt = ldi(src, WCNT);
    B3Soft soft = ldi(src, WSTAT) ? ss : cs;
    float ma = COL(bk, BK(ba, BMI)), mb = COL(bk, BK(bb, BMI));
    B3Mat3 ia = ldm(bk, BK(ba, BII)), ib = ldm(bk, BK(bb, BII));
    B3Vec3 va = ld3(bc, BI(ba, BV)), wa = ld3(bc, BI(ba, BW));
    B3Vec3 vb = ld3(bc, BI(bb, BV)), wb = ld3(bc, BI(bb, BW));
    B3Quat dqa, dqb;
    B3Vec3 dp;
    if (!cached) {
        dqa = ldq(bp, BP(ba, BDQ));
        dqb = ldq(bp, BP(bb, BDQ));
        dp = b3_sub(ld3(bp, BP(bb, BDP)), ld3(bp, BP(ba, BDP)));
    }
    B3Vec3 n = ld3(src, WN);
    float total_n = 0.0f, twist_lim = 0.0f;
    for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
        if (p >= cnt) break;
        B3Vec3 ra = ld3(src, PW(p, QRA)), rb = ld3(src, PW(p, QRB));
        float sep;
        if (cached) {
            sep = COL(src, WSEP + p);
        } else {
            B3Vec3 ds = b3_add(dp, b3_sub(b3_rotate(dqb, rb), b3_rotate(dqa, ra)));
            sep = b3_dot(ds, n) + COL(src, PW(p, QBSEP));
            COL(dst, WSEP + p) = sep;
        }
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
        float ni = COL(src, PW(p, QNI));
        float dimp = -COL(src, PW(p, QNM)) * (mscale * vn + vbias) - iscale * ni;
        float nimp = b3_maxf(ni + dimp, 0.0f);
        dimp = nimp - ni;
        COL(dst, PW(p, QNI)) = nimp;
        COL(dst, PW(p, QTOT)) = COL(src, PW(p, QTOT)) + nimp;
        total_n += nimp;
        twist_lim += COL(src, PW(p, QLEV)) * nimp;
        B3Vec3 P = b3_mul(n, dimp);
        va = b3_msub(va, ma, P);
        wa = b3_sub(wa, b3_mv(ia, b3_cross(ra, P)));
        vb = b3_madd(vb, mb, P);
        wb = b3_add(wb, b3_mv(ib, b3_cross(rb, P)));
    }
    if (!use_bias) {
        float fric = COL(src, WFRIC);
        float twist_s = b3_dot(n, b3_sub(wb, wa));
        float max_t = fric * twist_lim;
        float dtw = -COL(src, WTWM) * twist_s;
        float old_t = COL(src, WTWI);
        float new_t = b3_clamp(old_t + dtw, -max_t, max_t);
        COL(dst, WTWI) = new_t;
        dtw = new_t - old_t;
        wa = b3_sub(wa, b3_mv(ia, b3_mul(n, dtw)));
        wb = b3_add(wb, b3_mv(ib, b3_mul(n, dtw)));

        B3Vec3 t1 = ld3(src, WT1), t2 = ld3(src, WT2);
        B3Vec3 ra = ld3(src, WCA), rb = ld3(src, WCB);
        B3Vec3 vra = b3_add(va, b3_cross(wa, ra)), vrb = b3_add(vb, b3_cross(wb, rb));
        B3Vec3 vr = b3_sub(vrb, vra);
        B3Vec2 vt;
        vt.x = b3_dot(vr, t1);
        vt.y = b3_dot(vr, t2);
        B3Vec2 tv = m2_mv(ld22(src, WTM), vt);
        B3Vec2 fi;
        fi.x = COL(src, WFI);
        fi.y = COL(src, WFI + 1);
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
        COL(dst, WFI) = ni.x;
        COL(dst, WFI + 1) = ni.y;
        B3Vec3 P = b3_add(b3_mul(t1, df.x), b3_mul(t2, df.y));
        va = b3_msub(va, ma, P);
        wa = b3_sub(wa, b3_mv(ia, b3_cross(ra, P)));
        vb = b3_madd(vb, mb, P);
        wb = b3_add(wb, b3_mv(ib, b3_cross(rb, P)));

        float rolling = COL(src, WROLL);
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
            B3Vec3 imp = ld3(src, WRI);
            B3Vec3 next = b3_sub(imp, b3_add(b3_mul(t1, dd.x), b3_mul(t2, dd.y)));
            float limit = rolling * total_n;
            float l2 = b3_len2(next);
            if (l2 > limit * limit && l2 > 0.0f) next = b3_mul(next, limit / sqrtf(l2));
            B3Vec3 delta = b3_sub(next, imp);
            st3(dst, WRI, next);
            wa = b3_sub(wa, b3_mv(ia, delta));
            wb = b3_add(wb, b3_mv(ib, delta));
        }
    }
    put_vel(bc, bk, ba, va, wa);
    put_vel(bc, bk, bb, vb, wb);
}

// Restitution of one contact (08_contacts.inl:439-480).
B3X_HDI void restitute_contact(float* __restrict__ bc, const float* __restrict__ bk, const float* __restrict__ src, float* __restrict__ dst,
        float threshold) {
    float rest = COL(src, WREST);
    if (rest == 0.0f) return;
    int ba = ldi(src, WBA), bb = ldi(src, WBB);
    int cnt = ldi(src, WCNT);
    float ma = COL(bk, BK(ba, BMI)), mb = COL(bk, BK(bb, BMI));
    B3Mat3 ia = ldm(bk, BK(ba, BII)), ib = ldm(bk, BK(bb, BII));
    B3Vec3 va = ld3(bc, BI(ba, BV)), wa = ld3(bc, BI(ba, BW));
    B3Vec3 vb = ld3(bc, BI(bb, BV)), wb = ld3(bc, BI(bb, BW));
    B3Vec3 nrm = ld3(src, WN);
    for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
        if (p >= cnt) break;
        float relv = COL(src, PW(p, QRELV));
        if (relv > -threshold || COL(src, PW(p, QTOT)) == 0.0f) continue;
        B3Vec3 ra = ld3(src, PW(p, QRA)), rb = ld3(src, PW(p, QRB));
        B3Vec3 vra = b3_add(va, b3_cross(wa, ra)), vrb = b3_add(vb, b3_cross(wb, rb));
        float vn = b3_dot(b3_sub(vrb, vra), nrm);
        float ni = COL(src, PW(p, QNI));
        float imp = -COL(src, PW(p, QNM)) * (vn + rest * relv);
        float nimp = b3_maxf(ni + imp, 0.0f);
        imp = nimp - ni;
        COL(dst, PW(p, QNI)) = nimp;
        B3Vec3 P = b3_mul(nrm, imp);
        va = b3_msub(va, ma, P);
        wa = b3_sub(wa, b3_mv(ia, b3_cross(ra, P)));
        vb = b3_madd(vb, mb, P);
        wb = b3_add(wb, b3_mv(ib, b3_cross(rb, P)));
    }
    put_vel(bc, bk, ba, va, wa);
    put_vel(bc, bk, bb, vb, wb);
}

// ---- joints (06_joints.inl:204-642) -------------------------------------------
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

// Warm start one joint (06_joints.inl:204-239).
B3X_HDI void warm_joint(float* __restrict__ bc, const float* __restrict__ bp, const float* __restrict__ bk,
        const float* __restrict__ src) {
    int type = ldi(src, JTYPE);
    int ja = ldi(src, JBA), jb = ldi(src, JBB);
    float ma = COL(bk, BK(ja, BMI)), mb = COL(bk, BK(jb, BMI));
    B3Mat3 ia = ldm(bk, BK(ja, BII)), ib = ldm(bk, BK(jb, BII));
    B3Vec3 ra = b3_rotate(ldq(bp, BP(ja, BDQ)), ld3(src, JFPA));
    B3Vec3 rb = b3_rotate(ldq(bp, BP(jb, BDQ)), ld3(src, JFPB));
    B3Vec3 li = ld3(src, JLI);
    B3Vec3 ang;
    if (type == B3_JOINT_REVOLUTE) {
        float axial = COL(src, JSI) + COL(src, JMI) + COL(src, JLOI) - COL(src, JUPI);
        ang = b3_add(b3_mul(ld3(src, JPX), COL(src, JPI)), b3_mul(ld3(src, JPY), COL(src, JPI + 1)));
        ang = b3_madd(ang, axial, ld3(src, JAX));
    } else {
        ang = ld3(src, JAI);
    }
    if (body_dynamic_flag(bk, ja)) {
        st3(bc, BI(ja, BV), b3_msub(ld3(bc, BI(ja, BV)), ma, li));
        st3(bc, BI(ja, BW), b3_sub(ld3(bc, BI(ja, BW)), b3_mv(ia, b3_add(b3_cross(ra, li), ang))));
    }
    if (body_dynamic_flag(bk, jb)) {
        st3(bc, BI(jb, BV), b3_madd(ld3(bc, BI(jb, BV)), mb, li));
        st3(bc, BI(jb, BW), b3_add(ld3(bc, BI(jb, BW)), b3_mv(ib, b3_add(b3_cross(rb, li), ang))));
    }
}

// 06_joints.inl:257-282
B3X_HDI void solve_point(const float* __restrict__ bp, const float* __restrict__ src, float* __restrict__ dst,
        int ja, int jb, float ma, float mb, const B3Mat3& ia, const B3Mat3& ib, B3Vec3& va, B3Vec3& wa, B3Vec3& vb,
        B3Vec3& wb, B3Soft soft, int use_bias) {
    B3Vec3 ra = b3_rotate(ldq(bp, BP(ja, BDQ)), ld3(src, JFPA));
    B3Vec3 rb = b3_rotate(ldq(bp, BP(jb, BDQ)), ld3(src, JFPB));
    B3Vec3 cdot = b3_sub(b3_add(vb, b3_cross(wb, rb)), b3_add(va, b3_cross(wa, ra)));
    B3Vec3 bias = b3_v(0.0f, 0.0f, 0.0f);
    float mscale = 1.0f, iscale = 0.0f;
    if (use_bias) {
        B3Vec3 sep = b3_add(b3_add(b3_sub(ld3(bp, BP(jb, BDP)), ld3(bp, BP(ja, BDP))), b3_sub(rb, ra)),
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
B3X_HDI void solve_joint(float* __restrict__ bc, const float* __restrict__ bp, const float* __restrict__ bk,
        const float* __restrict__ src, float* __restrict__ dst, float h,
        float inv_h, int use_bias) {
    int type = ldi(src, JTYPE);
    int ja = ldi(src, JBA), jb = ldi(src, JBB);
    float ma = COL(bk, BK(ja, BMI)), mb = COL(bk, BK(jb, BMI));
    B3Mat3 ia = ldm(bk, BK(ja, BII)), ib = ldm(bk, BK(jb, BII));
    B3Vec3 va = ld3(bc, BI(ja, BV)), wa = ld3(bc, BI(ja, BW));
    B3Vec3 vb = ld3(bc, BI(jb, BV)), wb = ld3(bc, BI(jb, BW));
    int fixed = ldi(src, JFIX);
    B3Quat qa = b3_qmul(ldq(bp, BP(ja, BDQ)), ldq(src, JFQA));
    B3Quat qb = b3_qmul(ldq(bp, BP(jb, BDQ)), ldq(src, JFQB));
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
        solve_point(bp, src, dst, ja, jb, ma, mb, ia, ib, va, wa, vb, wb, lds(src, JLS), lin_bias);
        put_vel(bc, bk, ja, va, wa);
        put_vel(bc, bk, jb, vb, wb);
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
    solve_point(bp, src, dst, ja, jb, ma, mb, ia, ib, va, wa, vb, wb, soft, use_bias);
    put_vel(bc, bk, ja, va, wa);
    put_vel(bc, bk, jb, vb, wb);
}

// ---- one warp of worlds, the solver part of one step ------------------------------
// slot: the tile's workspace slot; lane: this world's lane; bc / bp / bk: the
// body velocity, pose-delta and constant columns (lane-offset; shared memory or
// the slot's body / bodyp / bodyk regions).  Returns false when the pipeline failed.  Follows
// 09_step.inl:158-181.
// kInterleave: the B3_INTERLEAVE_CONTACTS mode (a separate instantiation, so
// that the default mode's code is not shaped by the other).
template <bool kInterleave>
B3X_HD bool solve_world(const Args& a, float* slot, int lane, float* __restrict__ bc, float* __restrict__ bp,
        const float* __restrict__ bk, Pipe& P) {
    const float* rec = slot + a.SP.rec + lane;
    const int nb = ldi(rec, RNB);
    const int n = ldi(rec, RN);
    const int nj = ldi(rec, RNJ);
    float* kc = slot + a.SP.konst + lane;
    float* cc = slot + a.SP.cont + lane;
    float* jc = slot + a.SP.joint + lane;

    const int subs = a.substeps;
    const float dt = a.dt;
    const float h = dt / (float)subs;
    const float inv_dt = 1.0f / dt;
    const float inv_h = (float)subs * inv_dt;
    const B3Soft cs = lds(rec, RCS), ss = lds(rec, RSS);
    const float contact_speed = COL(rec, RSPEED);
    const float max_lin = COL(rec, RMAXLIN);
    const float max_ang = B3_MAX_ROTATION * inv_dt;
    const float max_lin2 = max_lin * max_lin, max_ang2 = max_ang * max_ang;
    const float restitution_threshold = COL(rec, RRT);

    const int wn = warp_max(n), wj = warp_max(nj);
    // the tile's step constants of its bodies in use (one contiguous block)
    const uint32_t konst_bytes = (uint32_t)((size_t)warp_max(nb) * NKF * kLanes * sizeof(float));
    constexpr uint32_t kStageBytesEach = (uint32_t)((size_t)kStreamWords * kLanes * sizeof(float));
    (void)konst_bytes;
    (void)kStageBytesEach;
    bool any_rest = false;
    // -- warm start contacts, then joints (09_step.inl:160-163)
    if (!stream_items(P, cc, kCI, kContactStream, wn, [&](int k, const float* src) {
            if (k < n) {
                warm_contact(bc, bk, src);
                any_rest |= COL(src, WREST) != 0.0f;
            }
        }))
        return false;
    any_rest = warp_any(any_rest);
    if (!stream_items(P, jc, NJF, kJointStream, wj, [&](int q, const float* src) {
            if (q < nj && ldi(src, JOK)) warm_joint(bc, bp, bk, src);
        }))
        return false;

    auto contact_pass = [&](auto pass) {
        constexpr int kPass = decltype(pass)::value;
        return stream_items(P, cc, kCI, kContactStream, wn, [&](int k, const float* src) {
            if (k < n) solve_contact<kPass>(bc, bp, bk, src, item(cc, k, kCI), inv_h, contact_speed, cs, ss);
        });
    };
    using Fresh = std::integral_constant<int, kBiasFresh>;
    using Cached = std::integral_constant<int, kBiasCached>;
    using Relax = std::integral_constant<int, kRelax>;
    using RelaxCached = std::integral_constant<int, kRelaxCached>;
    auto joint_pass = [&](int use_bias) {
        return stream_items(P, jc, NJF, kJointStream, wj, [&](int q, const float* src) {
            if (q < nj && ldi(src, JOK)) solve_joint(bc, bp, bk, src, item(jc, q, NJF), h, inv_h, use_bias);
        });
    };
    for (int s = 0; s < subs; s++) {
        // integrate velocities (09_step.inl:5-18, 41-53) with the step
        // constants, copied into a stage with one bulk copy when they fit
        const float* kcs = kc;
#if defined(__CUDA_ARCH__)
        if (konst_bytes <= kStageBytesEach) {
            if (!load_block(P, 0, kc - lane, konst_bytes)) return false;
            kcs = P.buf + lane;
        }
#endif
        for (int k = 0; k < nb; k++) {
            if (ldi(bk, BK(k, BTYPE)) != B3_DYNAMIC) continue;
            const float* kk = item(kcs, k, NKF);
            st3(bc, BI(k, BV), b3_madd(ld3(kk, KDV), COL(kk, KLD), ld3(bc, BI(k, BV))));
            st3(bc, BI(k, BW), b3_madd(ld3(kk, KDW), COL(kk, KAD), ld3(bc, BI(k, BW))));
        }
        // bias phase (09_step.inl:170-172): one contact sweep, then the joint
        // iterations; interleaved, a contact sweep opens every joint iteration
        // (07_packed.inl:61-65)
        if (!kInterleave) {
            if (s == 0 ? !contact_pass(Fresh{}) : !contact_pass(Cached{})) return false;
            for (int it = 0; it < a.joint_iters; it++)
                if (!joint_pass(1)) return false;
        } else {
            for (int it = 0; it < a.joint_iters; it++) {
                if (it == 0 && s == 0 ? !contact_pass(Fresh{}) : !contact_pass(Cached{})) return false;
                if (!joint_pass(1)) return false;
            }
        }
        // integrate positions (09_step.inl:55-107)
        for (int k = 0; k < nb; k++) {
            if (ldi(bk, BK(k, BTYPE)) == B3_STATIC) continue;
            uint32_t flags = b3x_f2u(COL(bk, BK(k, BFLAGS)));
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
            st3(bp, BP(k, BDP), b3_madd(ld3(bp, BP(k, BDP)), h, v));
            stq(bp, BP(k, BDQ), q_integrate(ldq(bp, BP(k, BDQ)), b3_mul(av, h)));
        }
        // relax phase (09_step.inl:173-177), the same way
        if (!kInterleave) {
            if (!contact_pass(Relax{})) return false;
            for (int it = 0; it < a.relax_iters; it++)
                if (!joint_pass(0)) return false;
        } else {
            for (int it = 0; it < a.relax_iters; it++) {
                if (it == 0 ? !contact_pass(Relax{}) : !contact_pass(RelaxCached{})) return false;
                if (!joint_pass(0)) return false;
            }
        }
        // restitution (08_contacts.inl:439-480): skipped when no contact of
        // the warp's worlds has a nonzero coefficient, or in the
        // B3_SKIP_RESTITUTION mode (09_step.inl:178-180)
        if (any_rest && !(a.flags & kStepSkipRestitution)) {
            if (!stream_items(P, cc, kCI, kContactStream, wn, [&](int k, const float* src) {
                    if (k < n) restitute_contact(bc, bk, src, item(cc, k, kCI), restitution_threshold);
                }))
                return false;
        }
    }
    return true;
}

}  // namespace b3x
