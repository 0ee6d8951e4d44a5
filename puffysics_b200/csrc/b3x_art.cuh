// b3x_art.cuh -- articulated contact response (B3_ART_CONTACTS=1) for the
// per-world device step.
//
// With B3_ART_CONTACTS=1 the reference resolves contacts of worlds that have
// joints through the articulation of their revolute joints instead of the
// independent-body masses (reference b3_art.cuh:1-17; selected inside
// b3_warm_start, 08_contacts.inl:194-232, and b3_solve_contacts,
// 08_contacts.inl:424-436).  The revolute joints span a tree of links (a
// breadth-first search from the static roots first, then from dynamic ones;
// edges that close a loop are recorded as cuts); a contact row's response
// is the Delassus operator J M^-1 J^T evaluated matrix-free by one
// articulated-body sweep (Featherstone's ABA with the bias terms off), and a
// row impulse changes every link's velocity by that sweep's acceleration.
// The soft-step joint solver still runs on every joint afterwards.
//
// What is restated here is the part of the reference module the step uses:
// the tree build (b3_art_from_world, b3_art.cuh:340-486), the link refresh
// (:527-570), the linear bias seed (:572-605), the backward and forward
// sweeps (:607-666), the Delassus apply (:723-749), rows, responses and
// impulses (:675-808), the rolling, friction and normal-row solves
// (:810-867, :1034-1121, :1220-1277) and the articulated warm start
// (08_contacts.inl:195-229).  The floating-point operation order is the
// reference's, so results round as its CPU build does (-ffp-contract=off).
// Not needed on this path and not restated: joint coordinates q (whose
// atan2f result nothing here reads), the nonlinear bias, the reduced
// integrator b3_art_step and the loop-cut solves, which only b3_art_step
// calls.
//
// State lives in the thread's local memory (the reference's B3Art), sized by
// the world view's body bound.  Joints naming a body outside the world are
// skipped when the tree is built (the reference would index past its
// arrays), so a corrupt world cannot fault.
#pragma once

#include "puffysics_b200.h"
#include "b3x_math.cuh"

#if defined(__CUDACC__)
namespace b3x {
namespace art {

constexpr int kMaxDeg = 8;        // joints per body in the tree (B3_ART_MAX_DEG)
constexpr int kMaxCuts = 8;       // loop-closing joints (B3_ART_MAX_CUTS)
constexpr float kDMin = 1.0e-8f;  // articulated inertia floor (B3_ART_DMIN)

// Spatial motion (angular, linear at the link's center of mass) and force
// (moment, force), world-aligned axes.
struct Motion {
    B3Vec3 w, v;
};
struct Force {
    B3Vec3 n, f;
};
// 6x6 spatial inertia as four 3x3 blocks [ww wv; vw vv].
struct Inertia {
    B3Mat3 ww, wv, vw, vv;
};
// One constraint row: a unit direction n applied at ra on link_a and rb on
// link_b (or a pure torque about n), links -1 when the body is not in the
// tree.
struct Row {
    int link_a, link_b, torque;
    B3Vec3 ra, rb, n;
};

__device__ __forceinline__ Motion motion0() { return {b3_v(0.0f, 0.0f, 0.0f), b3_v(0.0f, 0.0f, 0.0f)}; }
__device__ __forceinline__ Force force0() { return {b3_v(0.0f, 0.0f, 0.0f), b3_v(0.0f, 0.0f, 0.0f)}; }
__device__ __forceinline__ Inertia inertia0() { return {m3_zero(), m3_zero(), m3_zero(), m3_zero()}; }

__device__ __forceinline__ B3Mat3 m3_sub(B3Mat3 a, B3Mat3 b) {
    B3Mat3 r;
    r.cx = b3_sub(a.cx, b.cx);
    r.cy = b3_sub(a.cy, b.cy);
    r.cz = b3_sub(a.cz, b.cz);
    return r;
}
__device__ __forceinline__ B3Mat3 m3_scale(B3Mat3 a, float s) {
    B3Mat3 r;
    r.cx = b3_mul(a.cx, s);
    r.cy = b3_mul(a.cy, s);
    r.cz = b3_mul(a.cz, s);
    return r;
}
// a b^T (columns a * b.x, a * b.y, a * b.z)
__device__ __forceinline__ B3Mat3 outer(B3Vec3 a, B3Vec3 b) {
    B3Mat3 r;
    r.cx = b3_mul(a, b.x);
    r.cy = b3_mul(a, b.y);
    r.cz = b3_mul(a, b.z);
    return r;
}

// I m (b3_art.cuh:173-178)
__device__ __forceinline__ Force mul(const Inertia& I, const Motion& m) {
    Force f;
    f.n = b3_add(b3_mv(I.ww, m.w), b3_mv(I.wv, m.v));
    f.f = b3_add(b3_mv(I.vw, m.w), b3_mv(I.vv, m.v));
    return f;
}

__device__ __forceinline__ Inertia add(const Inertia& a, const Inertia& b) {
    return {m3_add(a.ww, b.ww), m3_add(a.wv, b.wv), m3_add(a.vw, b.vw), m3_add(a.vv, b.vv)};
}

// Column k of a spatial inertia (0-2 angular, 3-5 linear) set from a force.
__device__ __forceinline__ void set_col(Inertia& I, int k, const Force& f) {
    B3Mat3& ang = k < 3 ? I.ww : I.wv;
    B3Mat3& lin = k < 3 ? I.vw : I.vv;
    const int c = k < 3 ? k : k - 3;
    if (c == 0) {
        ang.cx = f.n;
        lin.cx = f.f;
    } else if (c == 1) {
        ang.cy = f.n;
        lin.cy = f.f;
    } else {
        ang.cz = f.n;
        lin.cz = f.f;
    }
}

// The inertia expressed at a point offset by r, column by column from unit
// motions (b3_art.cuh:189-209).
__device__ inline Inertia shift(const Inertia& I, B3Vec3 r) {
    Inertia O = inertia0();
    for (int k = 0; k < 6; k++) {
        Motion m = motion0();
        if (k < 3) m.w = b3_v(k == 0 ? 1.0f : 0.0f, k == 1 ? 1.0f : 0.0f, k == 2 ? 1.0f : 0.0f);
        else m.v = b3_v(k == 3 ? 1.0f : 0.0f, k == 4 ? 1.0f : 0.0f, k == 5 ? 1.0f : 0.0f);
        m.v = b3_add(m.v, b3_cross(m.w, r));
        const Force f = mul(I, m);
        Force fp;
        fp.n = b3_add(f.n, b3_cross(r, f.f));
        fp.f = f.f;
        set_col(O, k, fp);
    }
    return O;
}

// I - U U^T dinv (b3_art.cuh:211-217)
__device__ __forceinline__ Inertia rank1(Inertia I, const Force& U, float dinv) {
    I.ww = m3_sub(I.ww, m3_scale(outer(U.n, U.n), dinv));
    I.wv = m3_sub(I.wv, m3_scale(outer(U.n, U.f), dinv));
    I.vw = m3_sub(I.vw, m3_scale(outer(U.f, U.n), dinv));
    I.vv = m3_sub(I.vv, m3_scale(outer(U.f, U.f), dinv));
    return I;
}

__device__ __forceinline__ float sdot(const Motion& S, const Force& f) {
    return b3_dot(S.w, f.n) + b3_dot(S.v, f.f);
}
__device__ __forceinline__ Motion smul(const Motion& S, float s) { return {b3_mul(S.w, s), b3_mul(S.v, s)}; }

// Gauss-Jordan elimination with partial pivoting of a 6x6 system; false
// when a pivot falls below 1e-12 (b3_art.cuh:230-277).
__device__ inline bool solve6(const float A[36], const float b[6], float x[6]) {
    float M[6][7];
    for (int r = 0; r < 6; r++) {
        for (int c = 0; c < 6; c++) M[r][c] = A[r * 6 + c];
        M[r][6] = b[r];
    }
    for (int k = 0; k < 6; k++) {
        int piv = k;
        float best = fabsf(M[k][k]);
        for (int r = k + 1; r < 6; r++) {
            const float v = fabsf(M[r][k]);
            if (v > best) {
                best = v;
                piv = r;
            }
        }
        if (best < 1.0e-12f) return false;
        if (piv != k)
            for (int c = k; c < 7; c++) {
                const float t = M[k][c];
                M[k][c] = M[piv][c];
                M[piv][c] = t;
            }
        const float inv = 1.0f / M[k][k];
        for (int c = k; c < 7; c++) M[k][c] *= inv;
        for (int r = 0; r < 6; r++) {
            if (r == k) continue;
            const float s = M[r][k];
            for (int c = k; c < 7; c++) M[r][c] -= s * M[k][c];
        }
    }
    for (int r = 0; r < 6; r++) x[r] = M[r][6];
    return true;
}

// Solve I a = rhs for a floating root (b3_art.cuh:279-318): rows are the
// moment then force components, columns the angular then linear ones.
__device__ inline bool inertia_solve(const Inertia& I, const Force& rhs, Motion* a) {
    float A[36], b[6], x[6];
    const B3Vec3* cols[6] = {&I.ww.cx, &I.ww.cy, &I.ww.cz, &I.wv.cx, &I.wv.cy, &I.wv.cz};
    const B3Vec3* lcols[6] = {&I.vw.cx, &I.vw.cy, &I.vw.cz, &I.vv.cx, &I.vv.cy, &I.vv.cz};
    for (int c = 0; c < 6; c++) {
        A[0 * 6 + c] = cols[c]->x;
        A[1 * 6 + c] = cols[c]->y;
        A[2 * 6 + c] = cols[c]->z;
        A[3 * 6 + c] = lcols[c]->x;
        A[4 * 6 + c] = lcols[c]->y;
        A[5 * 6 + c] = lcols[c]->z;
    }
    b[0] = rhs.n.x;
    b[1] = rhs.n.y;
    b[2] = rhs.n.z;
    b[3] = rhs.f.x;
    b[4] = rhs.f.y;
    b[5] = rhs.f.z;
    if (!solve6(A, b, x)) {
        *a = motion0();
        return false;
    }
    a->w = b3_v(x[0], x[1], x[2]);
    a->v = b3_v(x[3], x[4], x[5]);
    return true;
}

// The articulation of one world (the reference's B3Art, the fields this path
// uses).  ML bounds the links (the world's body capacity).
template <int ML>
struct Tree {
    int n_links, n_cuts;
    int parent[ML], body[ML];
    bool fixed[ML], floating[ML];
    B3Vec3 anchor_a[ML];          // joint anchor on the parent body (local)
    B3Quat rot_a[ML];             // joint frame on the parent body (local)
    B3Vec3 local_center[ML], inertia_local[ML];
    float mass[ML];
    B3Vec3 com[ML], pos[ML], r[ML];
    B3Quat rot[ML];
    Motion S[ML], v[ML], a[ML], c[ML];
    Inertia I[ML], IA[ML];
    Force U[ML], pA[ML];
    float Dinv[ML];
    int cut_joint[kMaxCuts];

    // Link parameters from a body (b3_art.cuh:329-338).
    __device__ void link_from_body(int li, const B3Body& bd) {
        mass[li] = bd.inv_mass > 0.0f ? 1.0f / bd.inv_mass : 0.0f;
        inertia_local[li] = b3_v(bd.inv_inertia.x > 0.0f ? 1.0f / bd.inv_inertia.x : 0.0f,
                                 bd.inv_inertia.y > 0.0f ? 1.0f / bd.inv_inertia.y : 0.0f,
                                 bd.inv_inertia.z > 0.0f ? 1.0f / bd.inv_inertia.z : 0.0f);
        local_center[li] = bd.local_center;
    }

    // The tree of the revolute joints (b3_art.cuh:340-486): false when a
    // joint ties a body to itself, a body has more than kMaxDeg tree joints,
    // more than kMaxCuts loops close, or no dynamic body exists.
    __device__ bool build(const B3Body* bodies, int nb, const B3Joint* joints, int nj) {
        n_links = 0;
        n_cuts = 0;
        int deg[ML], adj_b[ML][kMaxDeg], adj_j[ML][kMaxDeg], body_link[ML], parent_body[ML], parent_joint[ML];
        int queue[ML];
        bool seen[ML];
        for (int i = 0; i < ML; i++) {
            deg[i] = 0;
            body_link[i] = -1;
            seen[i] = false;
            parent_body[i] = -1;
            parent_joint[i] = -1;
        }
        for (int k = 0; k < nj; k++) {
            const B3Joint& j = joints[k];
            if (j.type != B3_JOINT_REVOLUTE) continue;
            const int ja = j.body_a, jb = j.body_b;
            if (ja < 0 || ja >= nb || jb < 0 || jb >= nb) continue;
            if (ja == jb) return false;
            if (deg[ja] >= kMaxDeg || deg[jb] >= kMaxDeg) return false;
            adj_b[ja][deg[ja]] = jb;
            adj_j[ja][deg[ja]] = k;
            deg[ja]++;
            adj_b[jb][deg[jb]] = ja;
            adj_j[jb][deg[jb]] = k;
            deg[jb]++;
        }
        for (int pass = 0; pass < 2; pass++) {
            for (int s = 0; s < nb; s++) {
                const bool is_static = bodies[s].type != B3_DYNAMIC;
                if (deg[s] == 0 || seen[s] || is_static != (pass == 0)) continue;
                int qh = 0, qt = 0;
                queue[qt++] = s;
                seen[s] = true;
                parent_body[s] = -1;
                while (qh < qt) {
                    const int u = queue[qh++];
                    for (int e = 0; e < deg[u]; e++) {
                        const int v2 = adj_b[u][e];
                        if (seen[v2]) {
                            if (parent_body[u] != v2 && parent_body[v2] != u) {
                                const int jk = adj_j[u][e];
                                bool dup = false;
                                for (int c2 = 0; c2 < n_cuts; c2++)
                                    if (cut_joint[c2] == jk) dup = true;
                                if (!dup) {
                                    if (n_cuts >= kMaxCuts) return false;
                                    cut_joint[n_cuts++] = jk;
                                }
                            }
                            continue;
                        }
                        seen[v2] = true;
                        parent_body[v2] = u;
                        parent_joint[v2] = adj_j[u][e];
                        queue[qt++] = v2;
                    }
                }
                for (int t = 0; t < qt; t++) {
                    const int b = queue[t];
                    if (n_links >= ML) return false;
                    const int li = n_links++;
                    body_link[b] = li;
                    body[li] = b;
                    fixed[li] = bodies[b].type != B3_DYNAMIC;
                    floating[li] = parent_body[b] < 0 && !fixed[li];
                    link_from_body(li, bodies[b]);
                    if (parent_body[b] < 0) {
                        parent[li] = -1;
                    } else {
                        parent[li] = body_link[parent_body[b]];
                        const B3Joint& j = joints[parent_joint[b]];
                        if (j.body_b == b) {
                            anchor_a[li] = j.local_anchor_a;
                            rot_a[li] = j.local_rot_a;
                        } else {
                            anchor_a[li] = j.local_anchor_b;
                            rot_a[li] = j.local_rot_b;
                        }
                    }
                }
            }
        }
        for (int s = 0; s < nb; s++) {
            if (seen[s] || bodies[s].type != B3_DYNAMIC) continue;
            if (n_links >= ML) return false;
            const int li = n_links++;
            body_link[s] = li;
            body[li] = s;
            fixed[li] = false;
            floating[li] = true;
            parent[li] = -1;
            link_from_body(li, bodies[s]);
            seen[s] = true;
        }
        return n_links > 0;
    }

    // Link poses from the bodies' current (substep) poses, spatial inertias,
    // joint axes and offsets (b3_art.cuh:492-497, 527-570; velocities and
    // joint coordinates are left out: the Delassus sweep zeroes them).
    __device__ void refresh(const B3Body* bodies) {
        for (int i = 0; i < n_links; i++) {
            const B3Body& b = bodies[body[i]];
            rot[i] = b3_qnorm(b3_qmul(b.delta_rot, b.rotation));
            com[i] = b3_add(b.center, b.delta_pos);
            pos[i] = b3_sub(com[i], b3_rotate(rot[i], local_center[i]));
            if (fixed[i]) {
                I[i] = inertia0();
                mass[i] = 0.0f;
            } else {
                const B3Mat3 iw = b3_world_inv_i(rot[i], inertia_local[i]);
                I[i] = inertia0();
                I[i].ww = iw;
                const float m = mass[i];
                I[i].vv.cx = b3_v(m, 0.0f, 0.0f);
                I[i].vv.cy = b3_v(0.0f, m, 0.0f);
                I[i].vv.cz = b3_v(0.0f, 0.0f, m);
            }
            S[i] = motion0();
            r[i] = b3_v(0.0f, 0.0f, 0.0f);
            c[i] = motion0();
            const int p = parent[i];
            if (p < 0) continue;
            const B3Vec3 anchor = b3_xf_point(pos[p], rot[p], anchor_a[i]);
            const B3Vec3 axis_local = b3_rotate(rot_a[i], b3_v(0.0f, 0.0f, 1.0f));
            const B3Vec3 u = b3_norm(b3_rotate(rot[p], axis_local));
            r[i] = b3_sub(com[i], com[p]);
            S[i].w = u;
            S[i].v = b3_cross(u, b3_sub(com[i], anchor));
        }
    }

    // Backward sweep: articulated inertias and bias forces toward the roots
    // (b3_art.cuh:607-633; joint torques are zero on this path).
    __device__ void backward() {
        for (int i = n_links - 1; i >= 0; i--) {
            const int p = parent[i];
            if (p < 0) continue;
            const Motion Si = S[i];
            U[i] = mul(IA[i], Si);
            float D = sdot(Si, U[i]);
            if (D < kDMin) D = kDMin;
            Dinv[i] = 1.0f / D;
            const float u = 0.0f - sdot(Si, pA[i]);
            const Inertia IAp = rank1(IA[i], U[i], Dinv[i]);
            Force pa = pA[i];
            const Force Ic = mul(IA[i], c[i]);
            pa.n = b3_add(b3_add(pa.n, Ic.n), b3_mul(U[i].n, u * Dinv[i]));
            pa.f = b3_add(b3_add(pa.f, Ic.f), b3_mul(U[i].f, u * Dinv[i]));
            if (!fixed[p]) {
                IA[p] = add(IA[p], shift(IAp, r[i]));
                pA[p].n = b3_add(pA[p].n, b3_add(pa.n, b3_cross(r[i], pa.f)));
                pA[p].f = b3_add(pA[p].f, pa.f);
            }
        }
    }

    // Forward sweep: link accelerations from the roots (b3_art.cuh:635-666).
    __device__ void forward() {
        for (int i = 0; i < n_links; i++) {
            const int p = parent[i];
            if (p < 0) {
                if (fixed[i]) {
                    a[i] = motion0();
                } else if (floating[i]) {
                    Force rhs;
                    rhs.n = b3_neg(pA[i].n);
                    rhs.f = b3_neg(pA[i].f);
                    if (!inertia_solve(IA[i], rhs, &a[i])) a[i] = motion0();
                } else {
                    a[i] = motion0();
                }
                continue;
            }
            Motion ap;
            ap.w = a[p].w;
            ap.v = b3_add(a[p].v, b3_cross(a[p].w, r[i]));
            Motion rhs = ap;
            rhs.w = b3_add(rhs.w, c[i].w);
            rhs.v = b3_add(rhs.v, c[i].v);
            float u = 0.0f - sdot(S[i], pA[i]);
            u -= sdot(S[i], mul(IA[i], rhs));
            const float qdd = Dinv[i] * u;
            const Motion Sq = smul(S[i], qdd);
            a[i].w = b3_add(rhs.w, Sq.w);
            a[i].v = b3_add(rhs.v, Sq.v);
        }
    }

    __device__ int link_of(int b) const {
        for (int i = 0; i < n_links; i++)
            if (body[i] == b) return i;
        return -1;
    }

    // A contact row (b3_art.cuh:769-779): true when either body is a link.
    __device__ bool make_row(int body_a, int body_b, B3Vec3 ra, B3Vec3 rb, B3Vec3 n, Row* row) const {
        row->link_a = body_a >= 0 ? link_of(body_a) : -1;
        row->link_b = body_b >= 0 ? link_of(body_b) : -1;
        row->torque = 0;
        row->ra = ra;
        row->rb = rb;
        row->n = n;
        return row->link_a >= 0 || row->link_b >= 0;
    }

    // Row acceleration from the links' accelerations, with the centripetal
    // term of their (zeroed) velocities (b3_art.cuh:688-721, accel on).
    __device__ float row_eval(const Row& row) const {
        float y = 0.0f;
        if (row.torque == 1) {
            if (row.link_a >= 0) y += b3_dot(a[row.link_a].w, row.n);
            if (row.link_b >= 0) y -= b3_dot(a[row.link_b].w, row.n);
            return y;
        }
        if (row.link_a >= 0) {
            B3Vec3 ac = b3_add(a[row.link_a].v, b3_cross(a[row.link_a].w, row.ra));
            const Motion& va = v[row.link_a];
            ac = b3_add(ac, b3_cross(va.w, b3_cross(va.w, row.ra)));
            y += b3_dot(ac, row.n);
        }
        if (row.link_b >= 0) {
            B3Vec3 ac = b3_add(a[row.link_b].v, b3_cross(a[row.link_b].w, row.rb));
            const Motion& vb = v[row.link_b];
            ac = b3_add(ac, b3_cross(vb.w, b3_cross(vb.w, row.rb)));
            y -= b3_dot(ac, row.n);
        }
        return y;
    }

    // Row impulse x as a spatial force at the link (b3_art.cuh:675-686).
    __device__ static Force wrench(B3Vec3 r0, B3Vec3 n, float x, int torque) {
        Force f;
        if (torque == 1) {
            f.n = b3_mul(n, x);
            f.f = b3_v(0.0f, 0.0f, 0.0f);
        } else {
            f.f = b3_mul(n, x);
            f.n = b3_cross(r0, f.f);
        }
        return f;
    }

    // y = J M^-1 J^T x for n rows (b3_art.cuh:723-749): a refresh, a zero
    // velocity state, the linear bias seed (b3_art.cuh:572-605), the rows'
    // wrenches, the two sweeps, the rows' accelerations.
    __device__ void delassus(const B3Body* bodies, const Row* rows, const float* x, float* y, int n) {
        refresh(bodies);
        for (int i = 0; i < n_links; i++) v[i] = motion0();
        for (int i = 0; i < n_links; i++) {
            IA[i] = I[i];
            pA[i] = force0();
            if (fixed[i]) {
                c[i] = motion0();
                continue;
            }
            const Force ext = force0();
            pA[i].n = b3_sub(pA[i].n, ext.n);
            pA[i].f = b3_sub(pA[i].f, ext.f);
            c[i] = motion0();
        }
        for (int e = 0; e < n; e++) {
            const Row& row = rows[e];
            if (row.link_a >= 0 && !fixed[row.link_a]) {
                const Force f = wrench(row.ra, row.n, x[e], row.torque);
                pA[row.link_a].n = b3_sub(pA[row.link_a].n, f.n);
                pA[row.link_a].f = b3_sub(pA[row.link_a].f, f.f);
            }
            if (row.link_b >= 0 && !fixed[row.link_b]) {
                const Force f = wrench(row.rb, row.n, x[e], row.torque);
                pA[row.link_b].n = b3_add(pA[row.link_b].n, f.n);
                pA[row.link_b].f = b3_add(pA[row.link_b].f, f.f);
            }
        }
        backward();
        forward();
        for (int e = 0; e < n; e++) y[e] = row_eval(rows[e]);
    }

    // n . J M^-1 J^T n of one row (b3_art.cuh:781-787).
    __device__ float response(const B3Body* bodies, const Row& row) {
        const float x = 1.0f;
        float y = 0.0f;
        delassus(bodies, &row, &x, &y, 1);
        return y;
    }

    // A row impulse applied through the articulation (b3_art.cuh:789-808):
    // every non-fixed link's body velocity changes by its acceleration.
    __device__ void apply(B3Body* bodies, const Row& row, float lambda) {
        const float x = -lambda;
        float y = 0.0f;
        delassus(bodies, &row, &x, &y, 1);
        for (int i = 0; i < n_links; i++) {
            if (fixed[i]) continue;
            B3Body& b = bodies[body[i]];
            b.lin_vel = b3_add(b.lin_vel, a[i].v);
            b.ang_vel = b3_add(b.ang_vel, a[i].w);
        }
    }

    // The 2x2 Delassus block of two rows, column by column.
    __device__ B3Mat2 block2(const B3Body* bodies, const Row* rows) {
        const float e0[2] = {1.0f, 0.0f};
        const float e1[2] = {0.0f, 1.0f};
        float col0[2], col1[2];
        delassus(bodies, rows, e0, col0, 2);
        delassus(bodies, rows, e1, col1, 2);
        B3Mat2 K;
        K.cx.x = col0[0];
        K.cx.y = col0[1];
        K.cy.x = col1[0];
        K.cy.y = col1[1];
        return K;
    }

    // Torque-only rolling resistance in the tangent plane
    // (b3_art.cuh:810-867).
    __device__ void solve_rolling(B3Body* bodies, int body_a, int body_b, B3Vec3 t1, B3Vec3 t2, float rolling,
                                  float total_n, B3Vec3* impulse) {
        const float max_r = rolling * total_n;
        if (!(max_r > 0.0f)) return;
        Row rows[2];
        if (!make_row(body_a, body_b, b3_v(0.0f, 0.0f, 0.0f), b3_v(0.0f, 0.0f, 0.0f), t1, &rows[0])) return;
        rows[0].torque = 1;
        make_row(body_a, body_b, b3_v(0.0f, 0.0f, 0.0f), b3_v(0.0f, 0.0f, 0.0f), t2, &rows[1]);
        rows[1].torque = 1;
        const B3Mat2 Minv = m2_inv(block2(bodies, rows));
        const B3Body& ba = bodies[body_a];
        const B3Body& bb = bodies[body_b];
        const B3Vec3 dw = b3_sub(bb.ang_vel, ba.ang_vel);
        B3Vec2 vt;
        vt.x = b3_dot(dw, t1);
        vt.y = b3_dot(dw, t2);
        const B3Vec2 tm = m2_mv(Minv, vt);
        const B3Vec3 old = *impulse;
        B3Vec2 oi, ni;
        oi.x = b3_dot(old, t1);
        oi.y = b3_dot(old, t2);
        ni.x = oi.x - tm.x;
        ni.y = oi.y - tm.y;
        const float fl2 = ni.x * ni.x + ni.y * ni.y;
        if (fl2 > max_r * max_r && fl2 > 0.0f) {
            const float sc = max_r / sqrtf(fl2);
            ni.x *= sc;
            ni.y *= sc;
        }
        B3Vec2 df;
        df.x = ni.x - oi.x;
        df.y = ni.y - oi.y;
        *impulse = b3_add(b3_mul(t1, ni.x), b3_mul(t2, ni.y));
        if (df.x != 0.0f) apply(bodies, rows[0], df.x);
        if (df.y != 0.0f) apply(bodies, rows[1], df.y);
    }

    // Twist, Coulomb-disk friction and rolling of one contact
    // (b3_art.cuh:1034-1121).
    __device__ void solve_friction(B3Body* bodies, B3Contact& c) {
        float total_n = 0.0f, twist_lim = 0.0f;
        for (int p = 0; p < c.point_count; p++) {
            total_n += c.points[p].normal_impulse;
            twist_lim += c.points[p].lever * c.points[p].normal_impulse;
        }
        const float max_t = c.friction * twist_lim;
        if (max_t > 0.0f) {
            Row tw;
            if (make_row(c.body_a, c.body_b, b3_v(0.0f, 0.0f, 0.0f), b3_v(0.0f, 0.0f, 0.0f), c.normal, &tw)) {
                tw.torque = 1;
                const float ww = response(bodies, tw);
                c.twist_mass = ww > 0.0f ? 1.0f / ww : 0.0f;
                const B3Body& ba = bodies[c.body_a];
                const B3Body& bb = bodies[c.body_b];
                const float twist_s = b3_dot(c.normal, b3_sub(bb.ang_vel, ba.ang_vel));
                float dtw = -c.twist_mass * twist_s;
                const float old_t = c.twist_impulse;
                float nt = old_t + dtw;
                if (nt > max_t) nt = max_t;
                else if (nt < -max_t) nt = -max_t;
                dtw = nt - old_t;
                c.twist_impulse = nt;
                if (dtw != 0.0f) apply(bodies, tw, dtw);
            }
        }
        const float max_f = c.friction * total_n;
        if (max_f > 0.0f) {
            Row rows[2];
            if (make_row(c.body_a, c.body_b, c.center_a, c.center_b, c.tangent1, &rows[0])) {
                make_row(c.body_a, c.body_b, c.center_a, c.center_b, c.tangent2, &rows[1]);
                const B3Mat2 Minv = m2_inv(block2(bodies, rows));
                c.tangent_mass = Minv;
                const B3Body& ba = bodies[c.body_a];
                const B3Body& bb = bodies[c.body_b];
                const B3Vec3 vra = b3_add(ba.lin_vel, b3_cross(ba.ang_vel, c.center_a));
                const B3Vec3 vrb = b3_add(bb.lin_vel, b3_cross(bb.ang_vel, c.center_b));
                const B3Vec3 vr = b3_sub(vrb, vra);
                B3Vec2 vt;
                vt.x = b3_dot(vr, c.tangent1);
                vt.y = b3_dot(vr, c.tangent2);
                const B3Vec2 tm = m2_mv(Minv, vt);
                B3Vec2 ni;
                ni.x = c.friction_impulse.x - tm.x;
                ni.y = c.friction_impulse.y - tm.y;
                const float fl2 = ni.x * ni.x + ni.y * ni.y;
                if (fl2 > max_f * max_f && fl2 > 0.0f) {
                    const float sc = max_f / sqrtf(fl2);
                    ni.x *= sc;
                    ni.y *= sc;
                }
                B3Vec2 df;
                df.x = ni.x - c.friction_impulse.x;
                df.y = ni.y - c.friction_impulse.y;
                c.friction_impulse = ni;
                if (df.x != 0.0f) apply(bodies, rows[0], df.x);
                if (df.y != 0.0f) apply(bodies, rows[1], df.y);
            }
        }
        solve_rolling(bodies, c.body_a, c.body_b, c.tangent1, c.tangent2, c.rolling, total_n, &c.rolling_impulse);
    }

    // One sweep over the contacts in index order: normal rows with the
    // articulated normal mass, then (relax sweep) friction
    // (b3_art.cuh:1220-1277, one iteration).
    __device__ void solve_contacts(B3Body* bodies, B3Contact* contacts, int n, float inv_h, float contact_speed,
                                   bool use_bias) {
        for (int i = 0; i < n; i++) {
            B3Contact& c = contacts[i];
            const B3Body& ba = bodies[c.body_a];
            const B3Body& bb = bodies[c.body_b];
            const B3Vec3 nrm = c.normal;
            const B3Vec3 dp = b3_sub(bb.delta_pos, ba.delta_pos);
            const B3Quat dqa = ba.delta_rot, dqb = bb.delta_rot;
            for (int p = 0; p < c.point_count; p++) {
                B3Point& cp = c.points[p];
                Row row;
                if (!make_row(c.body_a, c.body_b, cp.r_a, cp.r_b, nrm, &row)) continue;
                const float ww = response(bodies, row);
                cp.normal_mass = ww > 0.0f ? 1.0f / ww : 0.0f;
                const B3Vec3 ds = b3_add(dp, b3_sub(b3_rotate(dqb, cp.r_b), b3_rotate(dqa, cp.r_a)));
                const float sep = b3_dot(ds, nrm) + cp.base_sep;
                float vbias = 0.0f, mscale = 1.0f, iscale = 0.0f;
                if (sep > 0.0f) {
                    vbias = sep * inv_h;
                } else if (use_bias) {
                    vbias = b3_maxf(c.softness.mass_scale * c.softness.bias_rate * sep, -contact_speed);
                    mscale = c.softness.mass_scale;
                    iscale = c.softness.impulse_scale;
                }
                const B3Vec3 vra = b3_add(bodies[c.body_a].lin_vel, b3_cross(bodies[c.body_a].ang_vel, cp.r_a));
                const B3Vec3 vrb = b3_add(bodies[c.body_b].lin_vel, b3_cross(bodies[c.body_b].ang_vel, cp.r_b));
                const float vn = b3_dot(b3_sub(vrb, vra), nrm);
                float dimp = -cp.normal_mass * (mscale * vn + vbias) - iscale * cp.normal_impulse;
                const float nimp = b3_maxf(cp.normal_impulse + dimp, 0.0f);
                dimp = nimp - cp.normal_impulse;
                cp.normal_impulse = nimp;
                cp.total_normal += dimp;
                if (dimp != 0.0f) apply(bodies, row, dimp);
            }
            if (!use_bias) solve_friction(bodies, c);
        }
    }

    // The articulated warm start (08_contacts.inl:195-229): each contact's
    // cached normal, friction, rolling and twist impulses applied as rows.
    __device__ void warm_start(B3Body* bodies, const B3Contact* contacts, int n) {
        for (int i = 0; i < n; i++) {
            const B3Contact& c = contacts[i];
            Row row;
            for (int p = 0; p < c.point_count; p++) {
                const B3Point& cp = c.points[p];
                if (make_row(c.body_a, c.body_b, cp.r_a, cp.r_b, c.normal, &row))
                    apply(bodies, row, cp.normal_impulse);
            }
            const B3Vec3 t[2] = {c.tangent1, c.tangent2};
            const float f[2] = {c.friction_impulse.x, c.friction_impulse.y};
            for (int k = 0; k < 2; k++) {
                if (make_row(c.body_a, c.body_b, c.center_a, c.center_b, t[k], &row)) apply(bodies, row, f[k]);
                row.torque = 1;
                apply(bodies, row, b3_dot(c.rolling_impulse, t[k]));
            }
            if (make_row(c.body_a, c.body_b, b3_v(0.0f, 0.0f, 0.0f), b3_v(0.0f, 0.0f, 0.0f), c.normal, &row)) {
                row.torque = 1;
                apply(bodies, row, c.twist_impulse);
            }
        }
    }
};

}  // namespace art
}  // namespace b3x
#endif  // __CUDACC__
