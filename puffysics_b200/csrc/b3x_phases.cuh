// b3x_phases.cuh -- the block-cooperative phases of the batched step: contact
// generation and constraint preparation (collide_kernel) and the write-back of
// the stepped worlds (out_kernel), one tile of 32 worlds per 128-thread block.
//
// Every phase is a function of (block state, thread index) and the threads of
// a block meet only between phases (one __syncthreads per phase), so a tile
// driver is a sequence of `x.each(phase)` calls that the GPU runs with one
// thread per index and development tools can run with a loop.
//
// Caller memory is only touched through coalesced transfers: a warp reads or
// writes consecutive words of one world's struct (B3Body, B3Shape, B3Contact,
// B3Joint), and shared memory turns those rows into the per-lane columns of
// the workspace and back.  Work that is independent per item (pairs,
// candidates, contacts) is spread over the block in (item, world) order, so
// consecutive threads touch the same item of consecutive worlds and their
// workspace accesses coalesce as well.
//
// Arithmetic keeps the reference's operation order (file:line cited, paths
// relative to the reference repository root).
#pragma once
#include <cstdint>

#include "b3x_layout.cuh"
#include "b3x_narrow.cuh"

namespace b3x {

constexpr int kCta = 128;            // threads of a collide / write-back block
constexpr int kCtaWarps = kCta / 32;
static_assert(kPairWindow <= kCta && kPairWindow % 32 == 0, "a window's pairs are set up one per thread");
constexpr int kRow = NYW + 1;        // staged struct row (odd: conflict-free columns)
// Collide staging area: rows of caller structs gathered for a group of worlds.
constexpr int kStageFloats = 12 * 1024;

// ---- block state ------------------------------------------------------------------
struct CollideShared {
    int live[kLanes], nb[kLanes], ns[kLanes], oldn[kLanes], nj[kLanes];
    int n[kLanes], ovf[kLanes], drop[kLanes], sorted[kLanes];
    float grav[kLanes][3];
    int maxnb, maxns, maxold, maxnj;
    // pair window: candidate bits per world over the window's pairs, and the
    // (candidate index, world) enumeration that spreads candidates over threads
    int ptab[kPairWindow];                       // i | j << 16 of window pair t, -1 past the end
    uint32_t cmask[kLanes][kPairWindow / 32];    // broadphase survivors of world l
    uint32_t nmask[kLanes][kPairWindow / 32];    // candidates of world l with a manifold
    int ccount[kLanes];
    int icount[kLanes];                          // item counts (sequential executor)
    int nbase[kLanes];                           // contacts of world l before the window
    // (item index, world) enumeration of the window's candidates, then of its
    // new contacts: wmask[r] = worlds with more than r items, off = prefix
    uint32_t wmask[kPairWindow];
    int off[kPairWindow + 1];
    int maxc, total;
    union {
        float hdr[kLanes][NHW];                  // world headers (17: odd)
        float flat[kStageFloats];                // gathered struct rows of a group of worlds
        float clip[48 * kCta];                   // narrowphase clip polygons
    } u;
};

struct OutShared {
    int live[kLanes], nb[kLanes], n[kLanes], nj[kLanes];
    int maxnb, maxn, maxnj;
    float flat[kStageFloats];                    // rows of several items of every world
};

B3X_HDI const float* world_words(const Args& a, int wi) {
    return reinterpret_cast<const float*>(a.data + (size_t)wi * a.stride + a.offset);
}
B3X_HDI float* world_words_w(const Args& a, int wi) {
    return reinterpret_cast<float*>(a.data + (size_t)wi * a.stride + a.offset);
}
B3X_HDI float* slot_of(const Args& a, int bt) { return a.ws + (size_t)bt * a.SP.tile_words; }
// Word w of the B3World of lane l of tile `tile` in the resident world
// columns ([tile][word][lane]: one word of a tile's 32 worlds is one
// contiguous 128-byte line).
B3X_HDI float* res_word(const Args& a, int tile, size_t w, int l) {
    return a.res + ((size_t)tile * a.resW + w) * kLanes + l;
}

// Index of the n-th set bit of a window mask (kPairWindow / 32 words).
B3X_HDI int nth_bit64(const uint32_t* m, int n) {
#pragma unroll
    for (int w = 0; w < kPairWindow / 32 - 1; w++) {
        const int c = popc32(m[w]);
        if (n < c) return 32 * w + nth_bit32(m[w], n);
        n -= c;
    }
    return 32 * (kPairWindow / 32 - 1) + nth_bit32(m[kPairWindow / 32 - 1], n);
}

// ================================ collide ==========================================

// Header of each world (warp w: worlds w, w+4, ...; lane = header word),
// copied asynchronously so all of a thread's loads are in flight at once.
template <bool kRes>
B3X_HD void c_header(const Args& a, int tile, CollideShared& sh, int t) {
    const int w = t >> 5, i = t & 31;
    if (t == 0) sh.maxnb = sh.maxns = sh.maxold = sh.maxnj = 0;
    if constexpr (kRes) {
        // resident columns: consecutive threads read one word of consecutive worlds
        for (int idx = t; idx < NHW * kLanes; idx += kCta) {
            const int l = idx & 31, f = idx >> 5;
            if (tile * kLanes + l < a.count) async_copy4_world(&sh.u.hdr[l][f], res_word(a, tile, f, l));
        }
    } else if (i < NHW) {
        for (int l = w; l < kLanes; l += kCtaWarps) {
            int wi = tile * kLanes + l;
            if (wi < a.count) async_copy4_world(&sh.u.hdr[l][i], world_words(a, wi) + i);
        }
    }
    async_wait();
}

// Clamped counts and the step's per-world constants (09_step.inl:148-157).
// Counts beyond the capacities would index past the arrays in the
// reference; here they are clamped so a corrupt world cannot fault.
B3X_HD void c_record(const Args& a, int tile, float* slot, CollideShared& sh, int l) {
    const Layout& L = a.L;
    const float* hw = sh.u.hdr[l];
    const int wi = tile * kLanes + l;
    const int live = wi < a.count && (!a.active || a.active[wi]);
    sh.live[l] = live;
    const int nb = live ? clampi(b3x_f2i(hw[HNB]), 0, L.B) : 0;
    const int ns = live ? clampi(b3x_f2i(hw[HNS]), 0, L.S) : 0;
    const int oldn = live ? clampi(b3x_f2i(hw[HNC]), 0, L.C) : 0;
    const int nj = live ? clampi(b3x_f2i(hw[HNJ]), 0, L.J) : 0;
    sh.nb[l] = nb;
    sh.ns[l] = ns;
    sh.oldn[l] = oldn;
    sh.nj[l] = nj;
    sh.n[l] = 0;
    sh.sorted[l] = 1;
    sh.ovf[l] = live ? b3x_f2i(hw[HOVC]) : 0;
    sh.drop[l] = live ? b3x_f2i(hw[HDROP]) : 0;
    for (int c = 0; c < 3; c++) sh.grav[l][c] = live ? hw[HGRAV + c] : 0.0f;
    shared_max(&sh.maxnb, nb);
    shared_max(&sh.maxns, ns);
    shared_max(&sh.maxold, oldn);
    shared_max(&sh.maxnj, nj);

    const int subs = a.substeps;
    const float h = a.dt / (float)subs;
    const float inv_h = (float)subs * (1.0f / a.dt);
    const float contact_hertz = live ? hw[HHZ] : 0.0f;
    const float contact_damping = live ? hw[HDAMP] : 0.0f;
    const float hertz = b3_minf(contact_hertz, 0.25f * inv_h);
    float* rec = slot + a.SP.rec + l;
    sti(rec, RLIVE, live);
    sti(rec, RNB, nb);
    sti(rec, RNS, ns);
    sti(rec, ROLDN, oldn);
    sti(rec, RNJ, nj);
    COL(rec, RSPEED) = live ? hw[HSPEED] : 0.0f;
    COL(rec, RRT) = live ? hw[HRT] : 0.0f;
    COL(rec, RMAXLIN) = live ? hw[HMAXLIN] : 0.0f;
    sts(rec, RCS, make_soft(hertz, contact_damping, h));
    sts(rec, RSS, make_soft(2.0f * hertz, 0.5f * contact_damping, h));
}

// ---- grouped gathers -------------------------------------------------------------
// A group is worlds [l0, l0 + G) of the tile.  Item k of group world g lands in
// the staging row (g * M + k) of stride RS (M * RS odd, so lanes reading one
// field of consecutive worlds hit distinct banks).  Warps take whole worlds:
// the items of a world are one contiguous region of the caller's struct
// array, copied with consecutive words on consecutive lanes.
template <int PER, bool kRes>
B3X_HD void c_gather_group(const Args& a, int tile, CollideShared& sh, const int* count, int l0, int G, int M,
        int RS, unsigned base, int dst, int t) {
    const int w = t >> 5, i = t & 31;
    if constexpr (kRes) {
        // resident columns: consecutive threads take one word of consecutive worlds
        for (int idx = t; idx < M * PER * G; idx += kCta) {
            const int g = idx % G, r = idx / G, k = r / PER, c = r - k * PER;
            const int l = l0 + g;
            if (k < count[l])
                async_copy4_world(sh.u.flat + dst + (g * M + k) * RS + c,
                                  res_word(a, tile, base / 4 + (size_t)k * PER + c, l));
        }
    } else {
        for (int g = w; g < G; g += kCtaWarps) {
            const int l = l0 + g;
            const int words = count[l] * PER;
            const float* src = world_words(a, tile * kLanes + l) + base / 4;
            float* row0 = sh.u.flat + dst + g * M * RS;
            for (int idx = i; idx < words; idx += 32) {
                const int k = idx / PER, c = idx - k * PER;
                async_copy4_world(row0 + k * RS + c, src + idx);
            }
        }
    }
}

// Words of a previous-step contact that the warm-start cache keeps
// (08_contacts.inl:68-87), in OLD field order.
B3X_HDI int old_word(int i) {
    return i == OSA ? WSA : i == OSB ? WSB : i == OCNT ? WCNT : i < OTWI ? WFI + (i - OFI)
        : i == OTWI ? WTWI : i < OFEAT ? WRI + (i - ORI) : i < ONI ? PW(i - OFEAT, QFEAT) : PW(i - ONI, QNI);
}

// The N words of a struct row of one world in the resident columns into y.
template <int N>
B3X_HDI void load_row(const float* col, float (&y)[N]) {
#pragma unroll
    for (int f = 0; f < N; f++) y[f] = col[(size_t)f * kLanes];
}

// A struct row of one world in the resident columns: word f at p[f * 32].
struct ColRow {
    float* p;
    B3X_HDI float& operator[](int f) const { return p[(size_t)f * kLanes]; }
};

template <bool kRes>
B3X_HD void c_gather_old(const Args& a, int tile, CollideShared& sh, int l0, int G, int M, int dst, int t) {
    const int w = t >> 5, i = t & 31;
    if constexpr (kRes) {
        for (int idx = t; idx < M * NOF * G; idx += kCta) {
            const int g = idx % G, r = idx / G, k = r / NOF, f = r - k * NOF;
            const int l = l0 + g;
            if (k < sh.oldn[l])
                async_copy4_world(sh.u.flat + dst + (g * M + k) * NOF + f,
                                  res_word(a, tile, a.L.contact_off / 4 + (size_t)k * NCW + old_word(f), l));
        }
    } else {
        if (i >= NOF) return;
        const int word = old_word(i);
        for (int g = w; g < G; g += kCtaWarps) {
            const int l = l0 + g;
            const float* src = world_words(a, tile * kLanes + l) + a.L.contact_off / 4 + word;
            float* row0 = sh.u.flat + dst + g * M * NOF;
            for (int k = 0; k < sh.oldn[l]; k++) async_copy4_world(row0 + k * NOF + i, src + k * (B3X_CONTACT_BYTES / 4));
        }
    }
}

// Thread t's staged items of a group: j -> (item k = j / G, group world g =
// j % G), so consecutive threads take one item of consecutive worlds and
// their workspace column stores coalesce.
#define FOR_GROUP_ITEMS(t, G, M, k, g) \
    for (int j_ = (t), k = j_ / (G), g = j_ - k * (G); j_ < (G) * (M); \
         j_ += kCta, k = j_ / (G), g = j_ - k * (G))

// Body k of world l (row y): solver columns, step constants and pose
// (inverse mass / inertia gated by type as the contact and joint prepares do,
// 08_contacts.inl:236-239; velocity increments of 09_step.inl:5-18).
template <class Y>
B3X_HD void c_body(const Args& a, float* slot, const CollideShared& sh, int k, int l, const Y& y) {
    const float h = a.dt / (float)a.substeps;
    float* bc = item(slot + a.SP.body, k, NBF) + l;
    float* kb = item(slot + a.SP.bodyk, k, NBC) + l;
    float* pb = item(slot + a.SP.bodyp, k, NBP) + l;
    float* pc = item(slot + a.SP.pose, k, NPF) + l;
    const int type = b3x_f2i(y[YTYPE]);
    auto v3 = [&](int f) { return b3_v(y[f], y[f + 1], y[f + 2]); };
    st3(bc, BV, v3(YLV));
    st3(bc, BW, v3(YAV));
    st3(pb, BDP, v3(YDP));
    stq(pb, BDQ, b3_q(y[YDQ], y[YDQ + 1], y[YDQ + 2], y[YDQ + 3]));
    COL(kb, BFLAGS) = y[YFLAGS];
    COL(kb, BTYPE) = y[YTYPE];
    if (type == B3_DYNAMIC) {
        const float inv_mass = y[YIM];
        B3Mat3 iw;
        iw.cx = v3(YIW);
        iw.cy = v3(YIW + 3);
        iw.cz = v3(YIW + 6);
        COL(kb, BMI) = inv_mass;
        stm(kb, BII, iw);
        float* kc = item(slot + a.SP.konst, k, NKF) + l;
        const B3Vec3 gravity = b3_v(sh.grav[l][0], sh.grav[l][1], sh.grav[l][2]);
        const float gs = inv_mass > 0.0f ? y[YGS] : 0.0f;
        st3(kc, KDV, b3_add(b3_mul(v3(YF), h * inv_mass), b3_mul(gravity, h * gs)));
        st3(kc, KDW, b3_mul(b3_mv(iw, v3(YT)), h));
        COL(kc, KLD) = 1.0f / (1.0f + h * y[YLD]);
        COL(kc, KAD) = 1.0f / (1.0f + h * y[YAD]);
    } else {
        COL(kb, BMI) = 0.0f;
        stm(kb, BII, m3_zero());
    }
    for (int f = 0; f < NPF; f++) COL(pc, f) = y[f];
}

// Shape s of world l (row y): world pose and padded AABB (04_world.inl:293-336,
// 08_contacts.inl:109-114); a shape on an invalid body never overlaps.
template <class Y>
B3X_HD void c_shape(const Args& a, float* slot, const CollideShared& sh, int s, int l, const Y& y) {
    float* so = item(slot + a.SP.shape, s, NSF) + l;
    const int body = b3x_f2i(y[XBODY]);
    const int type = b3x_f2i(y[XTYPE]);
    const float radius = y[XRAD];
    const B3Vec3 half = b3_v(y[XHALF], y[XHALF + 1], y[XHALF + 2]);
    COL(so, STYPE) = y[XTYPE];
    COL(so, SBODY) = y[XBODY];
    COL(so, SRAD) = radius;
    st3(so, SHALF, half);
    COL(so, SCAT) = y[XCAT];
    COL(so, SCAT + 1) = y[XCAT + 1];
    COL(so, SMASK) = y[XMASK];
    COL(so, SMASK + 1) = y[XMASK + 1];
    COL(so, SFRIC) = y[XFRIC];
    COL(so, SREST) = y[XREST];
    COL(so, SROLL) = y[XROLL];
    if (body < 0 || body >= sh.nb[l]) {
        st3(so, SLO, b3_v(INFINITY, INFINITY, INFINITY));
        st3(so, SHI, b3_v(-INFINITY, -INFINITY, -INFINITY));
        return;
    }
    const float* pc = item(slot + a.SP.pose, body, NPF) + l;
    const B3Vec3 bp = ld3(pc, PPOS);
    const B3Quat bq = ldq(pc, PROT);
    const B3Vec3 p = b3_xf_point(bp, bq, b3_v(y[XLPOS], y[XLPOS + 1], y[XLPOS + 2]));
    const B3Quat q = b3_qmul(bq, b3_q(y[XLROT], y[XLROT + 1], y[XLROT + 2], y[XLROT + 3]));
    B3Vec3 lo, hi;
    if (type == B3_SPHERE) {
        B3Vec3 e = b3_v(radius, radius, radius);
        lo = b3_sub(p, e);
        hi = b3_add(p, e);
    } else if (type == B3_CAPSULE) {
        B3Vec3 yv = b3_rotate(q, b3_v(0.0f, half.y, 0.0f));
        B3Vec3 c1 = b3_sub(p, yv), c2 = b3_add(p, yv);
        B3Vec3 e = b3_v(radius, radius, radius);
        lo = b3_sub(b3_v(b3_minf(c1.x, c2.x), b3_minf(c1.y, c2.y), b3_minf(c1.z, c2.z)), e);
        hi = b3_add(b3_v(b3_maxf(c1.x, c2.x), b3_maxf(c1.y, c2.y), b3_maxf(c1.z, c2.z)), e);
    } else {
        B3Vec3 ax, ay, az;
        b3_axes(q, &ax, &ay, &az);
        B3Vec3 e = b3_v(fabsf(ax.x) * half.x + fabsf(ay.x) * half.y + fabsf(az.x) * half.z,
            fabsf(ax.y) * half.x + fabsf(ay.y) * half.y + fabsf(az.y) * half.z,
            fabsf(ax.z) * half.x + fabsf(ay.z) * half.y + fabsf(az.z) * half.z);
        lo = b3_sub(p, e);
        hi = b3_add(p, e);
    }
    const B3Vec3 pad = b3_v(B3_SPECULATIVE, B3_SPECULATIVE, B3_SPECULATIVE);
    st3(so, SPOS, p);
    stq(so, SROT, q);
    st3(so, SLO, b3_sub(lo, pad));
    st3(so, SHI, b3_add(hi, pad));
}

// Rounds of a group plan: G worlds per round, balanced over the tile.
B3X_HDI int group_size(int per_world_floats, int budget) {
    int g = per_world_floats > 0 ? budget / per_world_floats : kLanes;
    if (g >= kLanes) return kLanes;
    if (g < 1) g = 1;
    const int rounds = (kLanes + g - 1) / g;
    return (kLanes + rounds - 1) / rounds;
}

// Old contact k of world l from its staged row y: the warm-start cache
// columns, and whether the cache's (shape_a, shape_b) keys strictly increase
// (then the reference matches with a merge cursor, else with a full scan;
// both pick the same entry), 08_contacts.inl:70-79.  `prev` is the staged
// row of contact k - 1.
template <class Y>
B3X_HD void c_old_row(const Args& a, float* slot, CollideShared& sh, int k, int l, const Y& y, const Y& prev) {
    float* oc = item(slot + a.SP.old, k, NOF) + l;
    for (int f = 0; f < NOF; f++) COL(oc, f) = y[f];
    if (k > 0) {
        const int pa = b3x_f2i(prev[OSA]), pb = b3x_f2i(prev[OSB]);
        const int sa = b3x_f2i(y[OSA]), sb = b3x_f2i(y[OSB]);
        if (pa > sa || (pa == sa && pb >= sb)) sh.sorted[l] = 0;
    }
}

// Joints per collide round: as many B3Joint rows of every world as the
// staging area holds.
constexpr int kJointRound = kStageFloats / (kLanes * NVW);
static_assert(kJointRound >= 1, "one joint of every world must fit the staging area");

// Staged row of joint q0 + qq of world l (odd stride NVW: conflict-free
// columns).
B3X_HDI float* joint_row(CollideShared& sh, int qq, int l) { return sh.u.flat + (qq * kLanes + l) * NVW; }

// Joints [q0, q0 + Q) of every world, each world's run of rows in one
// contiguous copy (warp w: worlds w, w+4, ...).
template <bool kRes>
B3X_HD void c_joint_gather(const Args& a, int tile, CollideShared& sh, int q0, int Q, int t) {
    const int w = t >> 5, i = t & 31;
    if constexpr (kRes) {
        for (int idx = t; idx < Q * NVW * kLanes; idx += kCta) {
            const int l = idx & 31, r = idx >> 5, qq = r / NVW, c = r - qq * NVW;
            if (q0 + qq < sh.nj[l])
                async_copy4_world(joint_row(sh, qq, l) + c,
                                  res_word(a, tile, a.L.joint_off / 4 + (size_t)(q0 + qq) * NVW + c, l));
        }
        async_wait();
    } else {
        for (int l = w; l < kLanes; l += kCtaWarps) {
            const int n = (sh.nj[l] < q0 + Q ? sh.nj[l] : q0 + Q) - q0;
            if (n <= 0) continue;
            const float* src = world_words(a, tile * kLanes + l) + (a.L.joint_off + (size_t)B3X_JOINT_BYTES * q0) / 4;
            for (int idx = i; idx < n * NVW; idx += 32) {
                const int qq = idx / NVW, c = idx - qq * NVW;
                async_copy4_world(joint_row(sh, qq, l) + c, src + idx);
            }
        }
        async_wait();
    }
}

// Prepare joint q of world l (06_joints.inl:161-202): the solver columns, and
// the B3Joint row with the prepared fields in place (jimg) for the write-back.
// Invalid body indices make the joint inert (the reference would index out
// of bounds).
B3X_HD void c_joint(const Args& a, float* slot, CollideShared& sh, int q, int l, float* y) {
    if (q >= sh.nj[l]) return;
    auto v3 = [&](int f) { return b3_v(y[f], y[f + 1], y[f + 2]); };
    auto v4 = [&](int f) { return b3_q(y[f], y[f + 1], y[f + 2], y[f + 3]); };
    auto put3 = [&](int f, B3Vec3 v) { y[f] = v.x; y[f + 1] = v.y; y[f + 2] = v.z; };
    auto put4 = [&](int f, B3Quat v) { y[f] = v.v.x; y[f + 1] = v.v.y; y[f + 2] = v.v.z; y[f + 3] = v.s; };
    auto putm = [&](int f, const B3Mat3& m) { put3(f, m.cx); put3(f + 3, m.cy); put3(f + 6, m.cz); };
    auto puts = [&](int f, B3Soft v) { y[f] = v.bias_rate; y[f + 1] = v.mass_scale; y[f + 2] = v.impulse_scale; };
    const float h = a.dt / (float)a.substeps;
    float* jo = item(slot + a.SP.joint, q, NJF) + l;
    float* ji = item(slot + a.SP.jimg, q, NVW) + l;
    const int type = b3x_f2i(y[VTYPE]), ja = b3x_f2i(y[VBA]), jb = b3x_f2i(y[VBB]);
    const int nb = sh.nb[l];
    sti(jo, JTYPE, type);
    sti(jo, JBA, ja);
    sti(jo, JBB, jb);
    COL(jo, JCC) = y[VCC];
    if (ja < 0 || ja >= nb || jb < 0 || jb >= nb) {
        sti(jo, JOK, 0);
        return;
    }
    sti(jo, JOK, 1);
    const float* bca = item(slot + a.SP.bodyk, ja, NBC) + l;
    const float* bcb = item(slot + a.SP.bodyk, jb, NBC) + l;
    const float* ia_img = item(slot + a.SP.pose, ja, NPF) + l;
    const float* ib_img = item(slot + a.SP.pose, jb, NPF) + l;
    const float ma = COL(bca, BMI), mb = COL(bcb, BMI);
    const B3Mat3 ia = ldm(bca, BII), ib = ldm(bcb, BII);
    const B3Mat3 isum = m3_add(ia, ib);
    const int fixed = b3_dot(isum.cx, b3_cross(isum.cy, isum.cz)) < 1.0e-20f;
    const B3Soft soft = make_soft(y[VCHZ], y[VCDMP], h);
    const B3Quat rot_a = ldq(ia_img, YROT), rot_b = ldq(ib_img, YROT);
    const B3Quat fqa = b3_qmul(rot_a, v4(VLRA)), fqb = b3_qmul(rot_b, v4(VLRB));
    const B3Vec3 fpa = b3_rotate(rot_a, b3_sub(v3(VLAA), ld3(ia_img, YLC)));
    const B3Vec3 fpb = b3_rotate(rot_b, b3_sub(v3(VLAB), ld3(ib_img, YLC)));
    const B3Vec3 dc = b3_sub(ld3(ib_img, YCEN), ld3(ia_img, YCEN));
    sti(jo, JFIX, fixed);
    sts(jo, JSOFT, soft);
    stq(jo, JFQA, fqa);
    stq(jo, JFQB, fqb);
    st3(jo, JFPA, fpa);
    st3(jo, JFPB, fpb);
    st3(jo, JDC, dc);
    st3(jo, JLI, v3(VLI));
    y[VIMA] = ma;
    y[VIMB] = mb;
    putm(VIIA, ia);
    putm(VIIB, ib);
    y[VFIX] = b3x_i2f(fixed);
    puts(VSOFT, soft);
    put4(VFQA, fqa);
    put4(VFQB, fqb);
    put3(VFPA, fpa);
    put3(VFPB, fpb);
    put3(VDC, dc);
    if (type == B3_JOINT_WELD) {
        const float lh = y[VLHZ], ah = y[VAHZ];
        const B3Soft ls = lh == 0.0f ? soft : make_soft(lh, y[VLDMP], h);
        const B3Soft as = ah == 0.0f ? soft : make_soft(ah, y[VADMP], h);
        const B3Mat3 am = m3_inv(isum);
        stm(jo, JAM, am);
        COL(jo, JLH) = lh;
        COL(jo, JAH) = ah;
        sts(jo, JLS, ls);
        sts(jo, JAS, as);
        st3(jo, JAI, v3(VAI));
        putm(VAM, am);
        puts(VLS, ls);
        puts(VAS, as);
    } else {
        const B3Vec3 axis = b3_rotate(fqa, b3_v(0.0f, 0.0f, 1.0f));
        const float kx = b3_dot(axis, b3_mv(isum, axis));
        const float axm = kx > 0.0f ? 1.0f / kx : 0.0f;
        const B3Quat rel = b3_qinv_mul(fqa, fqb);
        B3Vec3 px, py;
        hinge_perps(fqa, rel, &px, &py);
        const B3Soft sps = make_soft(y[VHZ], y[VDR], h);
        st3(jo, JAX, axis);
        COL(jo, JAXM) = axm;
        st3(jo, JPX, px);
        st3(jo, JPY, py);
        sts(jo, JSS, sps);
        COL(jo, JENS) = y[VENS];
        COL(jo, JENM) = y[VENM];
        COL(jo, JENL) = y[VENL];
        COL(jo, JPI) = y[VPI];
        COL(jo, JPI + 1) = y[VPI + 1];
        COL(jo, JSI) = y[VSI];
        COL(jo, JMI) = y[VMI];
        COL(jo, JLOI) = y[VLOI];
        COL(jo, JUPI) = y[VUPI];
        COL(jo, JMMT) = y[VMMT];
        COL(jo, JMS) = y[VMS];
        COL(jo, JTA) = y[VTA];
        COL(jo, JLA) = y[VLA];
        COL(jo, JUA) = y[VUA];
        if (type != B3_JOINT_REVOLUTE) st3(jo, JAI, v3(VAI));
        put3(VAX, axis);
        y[VAXM] = axm;
        put3(VPX, px);
        put3(VPY, py);
        puts(VSS, sps);
    }
    for (int f = 0; f < NVW; f++) COL(ji, f) = y[f];
}

// -- pair windows -----------------------------------------------------------------
// Pair p of the lexicographic (i < j < ns) order -> (i, j).
B3X_HDI int pair_of(int p, int ns) {
    int i = 0;
    while (i < ns - 1 && p >= ns - 1 - i) {
        p -= ns - 1 - i;
        i++;
    }
    if (i >= ns - 1) return -1;
    return i | ((i + 1 + p) << 16);
}

B3X_HD void c_window_setup(CollideShared& sh, int p0, int npairs, int t) {
    if (t < kPairWindow) {
        sh.ptab[t] = p0 + t < npairs ? pair_of(p0 + t, sh.maxns) : -1;
    }
    if (t < kLanes) {
        for (int c = 0; c < kPairWindow / 32; c++) {
            sh.cmask[t][c] = 0;
            sh.nmask[t][c] = 0;
        }
    }
}

// Broadphase of window pair pp for world l: the reference's predicate
// (08_contacts.inl:44-58; AABB overlap first, the side-effect-free tests in
// a cheaper order) with its joint-connection filter (08_contacts.inl:94-104).
B3X_HD void c_broadphase(const Args& a, float* slot, CollideShared& sh, int npw, int t) {
    const float* sc = slot + a.SP.shape;
    for (int idx = t; idx < npw * kLanes; idx += kCta) {
        const int pp = idx >> 5, l = idx & 31;
        const int pr = sh.ptab[pp];
        if (pr < 0) continue;
        const int i = pr & 0xffff, j = pr >> 16;
        if (j >= sh.ns[l]) continue;
        const float* si = item(sc, i, NSF) + l;
        const float* sj = item(sc, j, NSF) + l;
        const B3Vec3 lo_i = ld3(si, SLO), hi_i = ld3(si, SHI), lo_j = ld3(sj, SLO), hi_j = ld3(sj, SHI);
        if (!(lo_i.x <= hi_j.x && hi_i.x >= lo_j.x && lo_i.y <= hi_j.y && hi_i.y >= lo_j.y && lo_i.z <= hi_j.z
                && hi_i.z >= lo_j.z))
            continue;
        const int bi = ldi(si, SBODY), bj = ldi(sj, SBODY);
        if (bi == bj) continue;
        const float* kb = slot + a.SP.bodyk + l;
        if (ldi(item(kb, bi, NBC), BTYPE) == B3_STATIC && ldi(item(kb, bj, NBC), BTYPE) == B3_STATIC) continue;
        const uint64_t cat_i = (uint64_t)b3x_f2u(COL(si, SCAT)) | ((uint64_t)b3x_f2u(COL(si, SCAT + 1)) << 32);
        const uint64_t msk_i = (uint64_t)b3x_f2u(COL(si, SMASK)) | ((uint64_t)b3x_f2u(COL(si, SMASK + 1)) << 32);
        const uint64_t cat_j = (uint64_t)b3x_f2u(COL(sj, SCAT)) | ((uint64_t)b3x_f2u(COL(sj, SCAT + 1)) << 32);
        const uint64_t msk_j = (uint64_t)b3x_f2u(COL(sj, SMASK)) | ((uint64_t)b3x_f2u(COL(sj, SMASK + 1)) << 32);
        if ((cat_i & msk_j) == 0 || (cat_j & msk_i) == 0) continue;
        bool connected = false;
        const float* jc = slot + a.SP.joint + l;
        for (int q = 0; q < sh.nj[l]; q++) {
            const float* jo = item(jc, q, NJF);
            const int ja = ldi(jo, JBA), jb = ldi(jo, JBB);
            if (!ldi(jo, JCC) && ((ja == bi && jb == bj) || (ja == bj && jb == bi))) connected = true;
        }
        if (connected) continue;
        shared_or(&sh.cmask[l][pp >> 5], 1u << (pp & 31));
    }
}

// Per-world item counts -> the (item, world) enumeration (wmask, off, maxc,
// total).  Run by the 32 threads of warp 0, lane = world.
B3X_HD void enumerate(CollideShared& sh, int c, int l) {
#if defined(__CUDA_ARCH__)
    const int maxc = __reduce_max_sync(0xffffffffu, c);
    int off = 0;
    for (int ci = 0; ci < maxc; ci++) {
        const uint32_t b = __ballot_sync(0xffffffffu, c > ci);
        if (l == 0) {
            sh.wmask[ci] = b;
            sh.off[ci] = off;
        }
        off += __popc(b);
    }
    if (l == 0) {
        sh.off[maxc] = off;
        sh.maxc = maxc;
        sh.total = off;
    }
#else
    // sequential executor: the last world's call sees every count
    sh.icount[l] = c;
    if (l != kLanes - 1) return;
    int maxc = 0, off = 0;
    for (int w = 0; w < kLanes; w++) maxc = sh.icount[w] > maxc ? sh.icount[w] : maxc;
    for (int ci = 0; ci < maxc; ci++) {
        uint32_t b = 0;
        for (int w = 0; w < kLanes; w++)
            if (sh.icount[w] > ci) b |= 1u << w;
        sh.wmask[ci] = b;
        sh.off[ci] = off;
        off += popc32(b);
    }
    sh.off[maxc] = off;
    sh.maxc = maxc;
    sh.total = off;
#endif
}

// Candidates of world l (warp 0, lane = world).
B3X_HD void c_count(CollideShared& sh, int l) {
    int c = 0;
    for (int w = 0; w < kPairWindow / 32; w++) c += popc32(sh.cmask[l][w]);
    sh.ccount[l] = c;
    enumerate(sh, c, l);
}

// Enumeration index -> (candidate index ci, world l).
B3X_HDI void decode(const CollideShared& sh, int idx, int& ci, int& l) {
    int lo = 0, hi = sh.maxc - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (sh.off[mid] <= idx) lo = mid;
        else hi = mid - 1;
    }
    ci = lo;
    l = nth_bit32(sh.wmask[ci], idx - sh.off[ci]);
}

// Contact slots of world l's manifolds in this window (08_contacts.inl:120-134):
// in candidate order, slots are handed out while the capacity lasts, then
// overflow is counted -- so the r-th manifold of the window takes slot
// nbase + r.  Then the (contact, world) enumeration of the contact build.
// Warp 0, lane = world.
B3X_HD void c_plan(const Args& a, CollideShared& sh, int l) {
    int m = 0;
    for (int w = 0; w < kPairWindow / 32; w++) m += popc32(sh.nmask[l][w]);
    const int base = sh.n[l];
    const int room = a.L.C - base > 0 ? a.L.C - base : 0;
    const int kept = m < room ? m : room;
    if (m > kept) {
        sh.ovf[l] = 1;
        sh.drop[l] += m - kept;
    }
    sh.nbase[l] = base;
    sh.n[l] = base + kept;
    enumerate(sh, kept, l);
}

// Warm-cache entries to match for the key (i, j) (08_contacts.inl:136-153):
// with strictly increasing old keys the reference's merge cursor stands, for
// each contact it keeps, on the first old entry not below the contact's key
// (keys of kept contacts increase, so the cursor is that lower bound whatever
// the candidates before); it matches [cursor, cursor + 1).  Otherwise every
// entry is scanned.
B3X_HDI void warm_range(const float* oc, int on, int sorted, int i, int j, int guess, int& first, int& end) {
    if (!sorted) {
        first = 0;
        end = on;
        return;
    }
    // a cache that this step's contacts will mostly reproduce: try the
    // entry at the contact's own slot first (keys are unique when sorted)
    if (guess < on) {
        const float* o = item(oc, guess, NOF);
        if (ldi(o, OSA) == i && ldi(o, OSB) == j) {
            first = guess;
            end = guess + 1;
            return;
        }
    }
    int lo = 0, hi = on;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        const float* o = item(oc, mid, NOF);
        const int sa = ldi(o, OSA), sb = ldi(o, OSB);
        if (sa < i || (sa == i && sb < j)) lo = mid + 1;
        else hi = mid;
    }
    first = lo;
    end = lo < on ? lo + 1 : on;
}

// Every candidate of the window (spread over (candidate, world)): the
// narrowphase (05_collision.inl); a manifold is parked in region mani at the
// candidate's index and marked in nmask.
B3X_HD void c_narrow(const Args& a, float* slot, CollideShared& sh, int t) {
    const float* sc = slot + a.SP.shape;
    Poly P;
    P.base = sh.u.clip + t;
    P.stride = kCta;
    for (int idx = t; idx < sh.total; idx += kCta) {
        int ci, l;
        decode(sh, idx, ci, l);
        const int pr = sh.ptab[nth_bit64(sh.cmask[l], ci)];
        const int i = pr & 0xffff, j = pr >> 16;
        const float* si = item(sc, i, NSF) + l;
        const float* sj = item(sc, j, NSF) + l;
        Geo ga, gb;
        ga.p = ld3(si, SPOS); ga.q = ldq(si, SROT); ga.type = ldi(si, STYPE);
        ga.radius = COL(si, SRAD); ga.half = ld3(si, SHALF);
        gb.p = ld3(sj, SPOS); gb.q = ldq(sj, SROT); gb.type = ldi(sj, STYPE);
        gb.radius = COL(sj, SRAD); gb.half = ld3(sj, SHALF);
        Mani m;
        collide(m, ga, gb, P);
        if (m.count == 0) continue;
        shared_or(&sh.nmask[l][ci >> 5], 1u << (ci & 31));
        float* mo = item(slot + a.SP.mani, ci, NMW) + l;
        sti(mo, MCNT, m.count);
        st3(mo, MN, m.normal);
#pragma unroll
        for (int q = 0; q < B3_MAX_MANIFOLD; q++) {
            if (q >= m.count) continue;
            st3(mo, MPA + 3 * q, m.pa[q]);
            st3(mo, MPB + 3 * q, m.pb[q]);
            COL(mo, MSEP + q) = m.sep[q];
            sti(mo, MFEAT + q, (int)m.feat[q]);
        }
    }
}

// Every new contact of the window that fits the capacity (spread over
// (contact, world)): the r-th manifold of world l becomes contact slot
// nbase + r -- b3_contact_from_mani (08_contacts.inl:5-39), the warm-start
// carry (08_contacts.inl:136-171) and b3_prepare_one_contact
// (08_contacts.inl:234-291); words [0, kCW), point slots past the point
// count are not written.
// The tile's warm-start cache into the staging area (same [item][field][lane]
// layout), so that the contact build's cache lookups read shared memory.
B3X_HD void c_stage_old(const Args& a, float* slot, CollideShared& sh, int t) {
    const float* src = slot + a.SP.old;
    const int n = sh.maxold * NOF * kLanes;
    for (int idx = t; idx < n; idx += kCta) async_copy4(sh.u.flat + idx, src + idx);
    async_wait();
}

B3X_HD void c_build(const Args& a, float* slot, CollideShared& sh, int t, const float* old_base) {
    const float* sc = slot + a.SP.shape;
    for (int idx = t; idx < sh.total; idx += kCta) {
        int r, l;
        decode(sh, idx, r, l);
        const int ci = nth_bit64(sh.nmask[l], r);
        const int pr = sh.ptab[nth_bit64(sh.cmask[l], ci)];
        const int i = pr & 0xffff, j = pr >> 16;
        const float* si = item(sc, i, NSF) + l;
        const float* sj = item(sc, j, NSF) + l;
        const float* mo = item(slot + a.SP.mani, ci, NMW) + l;
        // every point slot is read (those past the count hold stale
        // values that nothing below uses), so the loads need not wait for
        // the count
        Mani m;
        m.count = clampi(ldi(mo, MCNT), 0, B3_MAX_MANIFOLD);
        m.normal = ld3(mo, MN);
#pragma unroll
        for (int q = 0; q < B3_MAX_MANIFOLD; q++) {
            m.pa[q] = ld3(mo, MPA + 3 * q);
            m.pb[q] = ld3(mo, MPB + 3 * q);
            m.sep[q] = COL(mo, MSEP + q);
            m.feat[q] = (uint32_t)ldi(mo, MFEAT + q);
        }

        const int bi = ldi(si, SBODY), bj = ldi(sj, SBODY);
        const float* ba = item(slot + a.SP.body, bi, NBF) + l;
        const float* bb = item(slot + a.SP.body, bj, NBF) + l;
        const float* kba = item(slot + a.SP.bodyk, bi, NBC) + l;
        const float* kbb = item(slot + a.SP.bodyk, bj, NBC) + l;
        const B3Vec3 ca = ld3(item(slot + a.SP.pose, bi, NPF) + l, PCEN);
        const B3Vec3 cb = ld3(item(slot + a.SP.pose, bj, NPF) + l, PCEN);
        const int cnt = m.count;
        const int p = sh.nbase[l] + r;
        const B3Vec3 nrm = m.normal;
        const B3Vec3 t1 = b3_perp(nrm);
        const B3Vec3 t2 = b3_cross(t1, nrm);
        const float rest_i = COL(si, SREST), rest_j = COL(sj, SREST);
        const int stat = ldi(kba, BTYPE) != B3_DYNAMIC || ldi(kbb, BTYPE) != B3_DYNAMIC;

        // warm-start carry by (shape_a, shape_b) and feature id
        float ni[B3_MAX_MANIFOLD];
#pragma unroll
        for (int q = 0; q < B3_MAX_MANIFOLD; q++) ni[q] = 0.0f;
        B3Vec2 fi;
        fi.x = 0.0f;
        fi.y = 0.0f;
        float twi = 0.0f;
        B3Vec3 ri = b3_v(0.0f, 0.0f, 0.0f);
        const float* oc = old_base + l;
        int first, end;
        warm_range(oc, sh.oldn[l], sh.sorted[l], i, j, p, first, end);
        for (int kk = first; kk < end; kk++) {
            const float* o = item(oc, kk, NOF);
            if (ldi(o, OSA) != i || ldi(o, OSB) != j) continue;
            const int ocnt = clampi(ldi(o, OCNT), 0, B3_MAX_MANIFOLD);
#pragma unroll
            for (int q = 0; q < B3_MAX_MANIFOLD; q++) {
                if (q >= cnt) continue;
#pragma unroll
                for (int r = 0; r < B3_MAX_MANIFOLD; r++)
                    if (r < ocnt && m.feat[q] == b3x_f2u(COL(o, OFEAT + r))) ni[q] = COL(o, ONI + r);
            }
            fi.x = COL(o, OFI);
            fi.y = COL(o, OFI + 1);
            twi = COL(o, OTWI);
            ri = ld3(o, ORI);
        }

        // prepare
        const float ma = COL(kba, BMI), mb = COL(kbb, BMI);
        const B3Mat3 ia = ldm(kba, BII), ib = ldm(kbb, BII);
        const B3Vec3 va = ld3(ba, BV), wa = ld3(ba, BW), vb = ld3(bb, BV), wb = ld3(bb, BW);
        float* co = item(slot + a.SP.cont, p, kCI) + l;
        const float inv_tau = 1.0f / B3_SPECULATIVE;
        B3Vec3 center_a = b3_v(0.0f, 0.0f, 0.0f), center_b = b3_v(0.0f, 0.0f, 0.0f);
        float wsum = 0.0f;
        B3Vec3 ras[B3_MAX_MANIFOLD];
#pragma unroll
        for (int q = 0; q < B3_MAX_MANIFOLD; q++) {
            if (q >= cnt) continue;
            const B3Vec3 ra = b3_sub(m.pa[q], ca), rb = b3_sub(m.pb[q], cb);
            const float base_sep = m.sep[q] - b3_dot(b3_sub(rb, ra), nrm);
            ras[q] = ra;
            const B3Vec3 rn_a = b3_cross(ra, nrm), rn_b = b3_cross(rb, nrm);
            const float kn = ma + mb + b3_dot(rn_a, b3_mv(ia, rn_a)) + b3_dot(rn_b, b3_mv(ib, rn_b));
            const float nm = kn > 0.0f ? 1.0f / kn : 0.0f;
            const B3Vec3 vra = b3_add(va, b3_cross(wa, ra)), vrb = b3_add(vb, b3_cross(wb, rb));
            const float relv = b3_dot(nrm, b3_sub(vrb, vra));
            const float sep = base_sep + b3_dot(b3_sub(rb, ra), nrm);
            const float wgt = b3_clamp(2.0f - sep * inv_tau, B3_MIN_FRICTION_W, 1.0f);
            center_a = b3_madd(center_a, wgt, ra);
            center_b = b3_madd(center_b, wgt, rb);
            wsum += wgt;
            st3(co, PW(q, QRA), ra);
            st3(co, PW(q, QRB), rb);
            COL(co, PW(q, QBSEP)) = base_sep;
            COL(co, PW(q, QRELV)) = relv;
            COL(co, PW(q, QNI)) = ni[q];
            COL(co, PW(q, QTOT)) = 0.0f;
            COL(co, PW(q, QNM)) = nm;
            sti(co, PW(q, QFEAT), (int)m.feat[q]);
        }
        const float invw = wsum > 0.0f ? 1.0f / wsum : 0.0f;
        const B3Vec3 cA = b3_mul(center_a, invw), cB = b3_mul(center_b, invw);
#pragma unroll
        for (int q = 0; q < B3_MAX_MANIFOLD; q++)
            if (q < cnt) COL(co, PW(q, QLEV)) = b3_len(b3_sub(ras[q], cA));
        const B3Vec3 rta1 = b3_cross(cA, t1), rta2 = b3_cross(cA, t2);
        const B3Vec3 rtb1 = b3_cross(cB, t1), rtb2 = b3_cross(cB, t2);
        B3Mat2 kt2;
        kt2.cx.x = ma + mb + b3_dot(rta1, b3_mv(ia, rta1)) + b3_dot(rtb1, b3_mv(ib, rtb1));
        kt2.cy.y = ma + mb + b3_dot(rta2, b3_mv(ia, rta2)) + b3_dot(rtb2, b3_mv(ib, rtb2));
        kt2.cx.y = kt2.cy.x = b3_dot(rta1, b3_mv(ia, rta2)) + b3_dot(rtb1, b3_mv(ib, rtb2));
        const float ktw = b3_dot(nrm, b3_mv(m3_add(ia, ib), nrm));
        sti(co, WSA, i);
        sti(co, WSB, j);
        sti(co, WBA, bi);
        sti(co, WBB, bj);
        sti(co, WCNT, cnt);
        sti(co, WSTAT, stat);
        st3(co, WN, nrm);
        st3(co, WT1, t1);
        st3(co, WT2, t2);
        st3(co, WCA, cA);
        st3(co, WCB, cB);
        COL(co, WFRIC) = sqrtf(COL(si, SFRIC) * COL(sj, SFRIC));
        COL(co, WREST) = rest_i > rest_j ? rest_i : rest_j;
        COL(co, WROLL) = b3_maxf(COL(si, SROLL), COL(sj, SROLL));
        COL(co, WTWM) = ktw > 0.0f ? 1.0f / ktw : 0.0f;
        COL(co, WTWI) = twi;
        COL(co, WFI) = fi.x;
        COL(co, WFI + 1) = fi.y;
        st3(co, WRI, ri);
        st22(co, WTM, m2_inv(kt2));
    }
}

B3X_HD void c_finish(const Args& a, float* slot, CollideShared& sh, int l) {
    float* rec = slot + a.SP.rec + l;
    sti(rec, RN, sh.n[l]);
    sti(rec, ROVF, sh.ovf[l]);
    sti(rec, RDROP, sh.drop[l]);
}

// The collide phases of tile `bt` of the launch.
template <bool kRes, class X>
B3X_HD void collide_tile(X& x, const Args& a, int bt, CollideShared& sh) {
    float* slot = slot_of(a, bt);
    const int tile = a.tile0 + bt;
    x.each([&](int t) { c_header<kRes>(a, tile, sh, t); });
    x.each([&](int t) { if (t < kLanes) c_record(a, tile, slot, sh, t); });
    if constexpr (kRes) {
        // resident columns: each (item, world) reads its row straight from
        // the columns, consecutive threads one word of consecutive worlds
        const size_t bw = B3X_WORLD_HEADER_BYTES / 4, sw = a.L.shape_off / 4, cw = a.L.contact_off / 4;
        // (each row is loaded whole into registers first, so that its loads
        // are in flight together)
        x.each([&](int t) {
            for (int j = t; j < sh.maxnb * kLanes; j += kCta) {
                const int k = j >> 5, l = j & 31;
                if (k >= sh.nb[l]) continue;
                float y[NYW];
                load_row(res_word(a, tile, bw + (size_t)k * NYW, l), y);
                c_body(a, slot, sh, k, l, (const float*)y);
            }
        });
        x.each([&](int t) {
            for (int j = t; j < sh.maxns * kLanes; j += kCta) {
                const int k = j >> 5, l = j & 31;
                if (k >= sh.ns[l]) continue;
                float y[NXW];
                load_row(res_word(a, tile, sw + (size_t)k * NXW, l), y);
                c_shape(a, slot, sh, k, l, (const float*)y);
            }
            for (int j = t; j < sh.maxold * kLanes; j += kCta) {
                const int k = j >> 5, l = j & 31;
                if (k >= sh.oldn[l]) continue;
                const float* row = res_word(a, tile, cw + (size_t)k * NCW, l);
                float y[NOF];
#pragma unroll
                for (int f = 0; f < NOF; f++) y[f] = row[(size_t)old_word(f) * kLanes];
                const float* prow = k > 0 ? row - (size_t)NCW * kLanes : row;
                float prev[OSB + 1];
                prev[OSA] = prow[(size_t)WSA * kLanes];
                prev[OSB] = prow[(size_t)WSB * kLanes];
                c_old_row(a, slot, sh, k, l, (const float*)y, (const float*)prev);
            }
        });
    } else {
        {
            // bodies: whole body arrays of G worlds per round
            const int M = sh.maxnb | 1, RS = kRow;
            const int G = group_size(M * RS, kStageFloats);
            for (int l0 = 0; l0 < kLanes; l0 += G) {
                const int Gr = kLanes - l0 < G ? kLanes - l0 : G;
                x.each([&](int t) {
                    c_gather_group<NYW, kRes>(a, tile, sh, sh.nb, l0, Gr, M, RS, B3X_WORLD_HEADER_BYTES, 0, t);
                    async_wait();
                });
                x.each([&](int t) {
                    FOR_GROUP_ITEMS(t, Gr, M, k, g) {
                        if (k < sh.nb[l0 + g]) c_body(a, slot, sh, k, l0 + g, sh.u.flat + (g * M + k) * RS);
                    }
                });
            }
        }
        {
            // shapes and the old contacts' warm-cache words, together when both fit
            const int Ms = sh.maxns | 1, Mo = sh.maxold | 1;
            const int per_s = Ms * (NXW + 1), per_o = Mo * NOF;
            const bool joint_round = kLanes * (per_s + per_o) <= kStageFloats;
            const int Gs = joint_round ? kLanes : group_size(per_s, kStageFloats);
            for (int l0 = 0; l0 < kLanes; l0 += Gs) {
                const int Gr = kLanes - l0 < Gs ? kLanes - l0 : Gs;
                const int odst = Gr * per_s;
                x.each([&](int t) {
                    c_gather_group<NXW, kRes>(a, tile, sh, sh.ns, l0, Gr, Ms, NXW + 1, a.L.shape_off, 0, t);
                    if (joint_round) c_gather_old<kRes>(a, tile, sh, l0, Gr, Mo, odst, t);
                    async_wait();
                });
                x.each([&](int t) {
                    FOR_GROUP_ITEMS(t, Gr, Ms, k, g) {
                        if (k < sh.ns[l0 + g]) c_shape(a, slot, sh, k, l0 + g, sh.u.flat + (g * Ms + k) * (NXW + 1));
                    }
                    if (joint_round) {
                        FOR_GROUP_ITEMS(t, Gr, Mo, k, g) {
                            if (k < sh.oldn[l0 + g]) {
                                const float* y = sh.u.flat + odst + (g * Mo + k) * NOF;
                                c_old_row(a, slot, sh, k, l0 + g, y, y - NOF);
                            }
                        }
                    }
                });
            }
            if (!joint_round) {
                const int Go = group_size(per_o, kStageFloats);
                for (int l0 = 0; l0 < kLanes; l0 += Go) {
                    const int Gr = kLanes - l0 < Go ? kLanes - l0 : Go;
                    x.each([&](int t) {
                        c_gather_old<kRes>(a, tile, sh, l0, Gr, Mo, 0, t);
                        async_wait();
                    });
                    x.each([&](int t) {
                        FOR_GROUP_ITEMS(t, Gr, Mo, k, g) {
                            if (k < sh.oldn[l0 + g]) {
                                const float* y = sh.u.flat + (g * Mo + k) * NOF;
                                c_old_row(a, slot, sh, k, l0 + g, y, y - NOF);
                            }
                        }
                    });
                }
            }
        }
    }
    for (int q0 = 0; q0 < sh.maxnj; q0 += kJointRound) {
        const int Q = sh.maxnj - q0 < kJointRound ? sh.maxnj - q0 : kJointRound;
        x.each([&](int t) { c_joint_gather<kRes>(a, tile, sh, q0, Q, t); });
        x.each([&](int t) {
            for (int j = t; j < Q * kLanes; j += kCta) c_joint(a, slot, sh, q0 + (j >> 5), j & 31, joint_row(sh, j >> 5, j & 31));
        });
    }
    const int maxns = sh.maxns;
    const int npairs = maxns * (maxns - 1) / 2;
    for (int p0 = 0; p0 < npairs; p0 += kPairWindow) {
        x.each([&](int t) { c_window_setup(sh, p0, npairs, t); });
        const int npw = npairs - p0 < kPairWindow ? npairs - p0 : kPairWindow;
        x.each([&](int t) { c_broadphase(a, slot, sh, npw, t); });
        x.each([&](int t) { if (t < kLanes) c_count(sh, t); });
        if (sh.total == 0) continue;
        x.each([&](int t) { c_narrow(a, slot, sh, t); });
        x.each([&](int t) { if (t < kLanes) c_plan(a, sh, t); });
        if (sh.total == 0) continue;
        // the staging area is free between the narrowphase and the next window
        const bool stage_old = sh.maxold > 0 && sh.maxold * NOF * kLanes <= kStageFloats;
        if (stage_old) x.each([&](int t) { c_stage_old(a, slot, sh, t); });
        x.each([&](int t) { c_build(a, slot, sh, t, stage_old ? sh.u.flat : slot + a.SP.old); });
    }
    x.each([&](int t) { if (t < kLanes) c_finish(a, slot, sh, t); });
}

// ================================ write-back =======================================

B3X_HD void o_record(const Args& a, float* slot, OutShared& sh, int l) {
    const float* rec = slot + a.SP.rec + l;
    sh.live[l] = ldi(rec, RLIVE);
    sh.nb[l] = ldi(rec, RNB);
    sh.n[l] = ldi(rec, RN);
    sh.nj[l] = ldi(rec, RNJ);
}

B3X_HD void o_maxima(OutShared& sh) {
    int mb = 0, mn = 0, mj = 0;
    for (int l = 0; l < kLanes; l++) {
        mb = sh.nb[l] > mb ? sh.nb[l] : mb;
        mn = sh.n[l] > mn ? sh.n[l] : mn;
        mj = sh.nj[l] > mj ? sh.nj[l] : mj;
    }
    sh.maxnb = mb;
    sh.maxn = mn;
    sh.maxnj = mj;
}

// Items [k0, k0 + K) of every world are staged as rows ((k - k0) * 32 + l) of
// odd stride RS; the write-back stores each world's run of items as one
// contiguous region with consecutive words on consecutive lanes.
B3X_HDI float* out_row(OutShared& sh, int l, int kk, int K, int RS) {
    (void)K;
    return sh.flat + (kk * kLanes + l) * RS;
}

// Bodies [k0, k0 + K) of every world: each world's run of B3Body rows,
// gathered from the caller's array (rows stay untouched until written back).
B3X_HD void o_body_gather(const Args& a, int tile, OutShared& sh, int k0, int K, int t) {
    const int w = t >> 5, i = t & 31;
    for (int l = w; l < kLanes; l += kCtaWarps) {
        const int n = (sh.nb[l] < k0 + K ? sh.nb[l] : k0 + K) - k0;
        if (n <= 0) continue;
        const float* src = world_words(a, tile * kLanes + l) + (B3X_WORLD_HEADER_BYTES + (size_t)B3X_BODY_BYTES * k0) / 4;
        for (int idx = i; idx < n * NYW; idx += 32) {
            const int kk = idx / NYW, c = idx - kk * NYW;
            async_copy4_world(out_row(sh, l, kk, K, kRow) + c, src + idx);
        }
    }
    async_wait();
}


// Finalize body k of world l (09_step.inl:109-130) in its B3Body row y: the
// fields the reference's step writes are replaced, the others keep their
// bytes, so the write-back stores whole rows.
template <class Y>
B3X_HD void o_body(const Args& a, float* slot, int k, int l, const Y& y) {
    const float* bc = item(slot + a.SP.body, k, NBF) + l;
    const float* kb = item(slot + a.SP.bodyk, k, NBC) + l;
    const float* pb = item(slot + a.SP.bodyp, k, NBP) + l;
    auto get3 = [&](int f) { return b3_v(y[f], y[f + 1], y[f + 2]); };
    auto put3 = [&](int f, B3Vec3 v) { y[f] = v.x; y[f + 1] = v.y; y[f + 2] = v.z; };
    auto put4 = [&](int f, B3Quat q) { y[f] = q.v.x; y[f + 1] = q.v.y; y[f + 2] = q.v.z; y[f + 3] = q.s; };
    const int type = ldi(kb, BTYPE);
    const bool dyn_flag = (b3x_f2u(COL(kb, BFLAGS)) & B3_FLAG_DYNAMIC) != 0;
    if (type != B3_STATIC || dyn_flag) {
        put3(YLV, ld3(bc, BV));
        put3(YAV, ld3(bc, BW));
    }
    if (type != B3_STATIC) {
        const B3Vec3 center = b3_add(get3(YCEN), ld3(pb, BDP));
        const B3Quat rot = b3_qnorm(b3_qmul(ldq(pb, BDQ), b3_q(y[YROT], y[YROT + 1], y[YROT + 2], y[YROT + 3])));
        put3(YCEN, center);
        put4(YROT, rot);
        put3(YPOS, b3_sub(center, b3_rotate(rot, get3(YLC))));
        put3(YDP, b3_v(0.0f, 0.0f, 0.0f));
        put4(YDQ, b3_q_id());
        put3(YF, b3_v(0.0f, 0.0f, 0.0f));
        put3(YT, b3_v(0.0f, 0.0f, 0.0f));
        if (type == B3_DYNAMIC) {
            const B3Mat3 iw = b3_world_inv_i(rot, get3(YII));
            put3(YIW, iw.cx);
            put3(YIW + 3, iw.cy);
            put3(YIW + 6, iw.cz);
        }
    }
}

B3X_HD void o_bodies(const Args& a, float* slot, OutShared& sh, int k0, int K, int t) {
    for (int j = t; j < K * kLanes; j += kCta) {
        const int kk = j >> 5, l = j & 31;
        if (k0 + kk < sh.nb[l]) o_body(a, slot, k0 + kk, l, out_row(sh, l, kk, K, kRow));
    }
}

B3X_HD void o_body_write(const Args& a, int tile, OutShared& sh, int k0, int K, int t) {
    const int w = t >> 5, i = t & 31;
    for (int l = w; l < kLanes; l += kCtaWarps) {
        const int n = (sh.nb[l] < k0 + K ? sh.nb[l] : k0 + K) - k0;
        if (n <= 0) continue;
        float* dst = world_words_w(a, tile * kLanes + l) + (B3X_WORLD_HEADER_BYTES + (size_t)B3X_BODY_BYTES * k0) / 4;
        for (int idx = i; idx < n * NYW; idx += 32) {
            const int kk = idx / NYW, c = idx - kk * NYW;
            store_world(dst + idx, out_row(sh, l, kk, K, kRow)[c]);
        }
    }
}


// Items [k0, k0 + K) of a [item][word][lane] region -> rows, copied
// asynchronously (`words` words per item, row stride RS >= words).
B3X_HD void o_stage(const float* src, OutShared& sh, int K, int words, int RS, int t) {
    for (int idx = t; idx < K * words * kLanes; idx += kCta) {
        const int l = idx & 31, r = idx >> 5, kk = r / words, c = r - kk * words;
        async_copy4(out_row(sh, l, kk, K, RS) + c, src + idx);
    }
    async_wait();
}

// The words of contact k of world l the workspace does not keep, from the
// body columns and the step softness, as b3_prepare_one_contact
// (08_contacts.inl:234-245) computes them.
template <class Y>
B3X_HD void o_contact_fill(const Args& a, float* slot, int l, const Y& row) {
    const int ba = b3x_f2i(row[WBA]), bb = b3x_f2i(row[WBB]);
    const float* ca = item(slot + a.SP.bodyk, ba, NBC) + l;
    const float* cb = item(slot + a.SP.bodyk, bb, NBC) + l;
    const B3Mat3 ia = ldm(ca, BII), ib = ldm(cb, BII);
    const B3Mat3 rm = m3_inv(m3_add(ia, ib));
    auto put3 = [&](int f, B3Vec3 v) { row[f] = v.x; row[f + 1] = v.y; row[f + 2] = v.z; };
    auto putm = [&](int f, const B3Mat3& m) { put3(f, m.cx); put3(f + 3, m.cy); put3(f + 6, m.cz); };
    putm(WRM, rm);
    row[WMA] = COL(ca, BMI);
    row[WMB] = COL(cb, BMI);
    putm(WIA, ia);
    putm(WIB, ib);
    const float* rec = slot + a.SP.rec + l;
    const B3Soft soft = lds(rec, b3x_f2i(row[WSTAT]) ? RSS : RCS);
    row[WSOFT] = soft.bias_rate;
    row[WSOFT + 1] = soft.mass_scale;
    row[WSOFT + 2] = soft.impulse_scale;
}

B3X_HD void o_contacts(const Args& a, float* slot, OutShared& sh, int k0, int K, int t) {
    for (int j = t; j < K * kLanes; j += kCta) {
        const int kk = j >> 5, l = j & 31;
        if (k0 + kk < sh.n[l]) o_contact_fill(a, slot, l, out_row(sh, l, kk, K, NCW));
    }
}

// Contacts [k0, k0 + K) of every world.  Point slots past a contact's point
// count keep their previous bytes, as in the reference (b3_contact_from_mani
// writes only the manifold's points).
B3X_HD void o_contact_write(const Args& a, int tile, OutShared& sh, int k0, int K, int t) {
    const int w = t >> 5, i = t & 31;
    for (int l = w; l < kLanes; l += kCtaWarps) {
        const int n = (sh.n[l] < k0 + K ? sh.n[l] : k0 + K) - k0;
        if (n <= 0) continue;
        float* dst = world_words_w(a, tile * kLanes + l) + (a.L.contact_off + (size_t)B3X_CONTACT_BYTES * k0) / 4;
        for (int kk = 0; kk < n; kk++) {    // row by row: each row's point count is read once
            const float* row = out_row(sh, l, kk, K, NCW);
            const int hi = WP + clampi(b3x_f2i(row[WCNT]), 0, B3_MAX_MANIFOLD) * NQW;
            for (int c = i; c < NCW; c += 32)
                if (c < hi || c >= WCA) store_world(dst + kk * NCW + c, row[c]);
        }
    }
}


// The solver's results into the prepared B3Joint row of joint q of world l:
// linear impulse; angular impulse (weld); axial and hinge impulses and the
// hinge rows (revolute) -- 06_joints.inl finalize.
B3X_HD void o_joint_patch(const Args& a, float* slot, int q, int l, float* y) {
    const float* jo = item(slot + a.SP.joint, q, NJF) + l;
    if (!ldi(jo, JOK)) return;
    auto put3 = [&](int f, B3Vec3 v) { y[f] = v.x; y[f + 1] = v.y; y[f + 2] = v.z; };
    put3(VLI, ld3(jo, JLI));
    if (ldi(jo, JTYPE) == B3_JOINT_WELD) {
        put3(VAI, ld3(jo, JAI));
    } else {
        y[VPI] = COL(jo, JPI);
        y[VPI + 1] = COL(jo, JPI + 1);
        y[VSI] = COL(jo, JSI);
        y[VMI] = COL(jo, JMI);
        y[VLOI] = COL(jo, JLOI);
        y[VUPI] = COL(jo, JUPI);
        put3(VPX, ld3(jo, JPX));
        put3(VPY, ld3(jo, JPY));
    }
}

B3X_HD void o_joints(const Args& a, float* slot, OutShared& sh, int q0, int K, int t) {
    for (int j = t; j < K * kLanes; j += kCta) {
        const int kk = j >> 5, l = j & 31;
        if (q0 + kk < sh.nj[l]) o_joint_patch(a, slot, q0 + kk, l, out_row(sh, l, kk, K, NVW));
    }
}

// Joints [q0, q0 + K) of every world (the caller's AoS worlds); invalid
// joints (body index out of range) are left as they were.
B3X_HD void o_joint_write(const Args& a, int tile, float* slot, OutShared& sh, int q0, int K, int t) {
    const int w = t >> 5, i = t & 31;
    for (int l = w; l < kLanes; l += kCtaWarps) {
        const int n = (sh.nj[l] < q0 + K ? sh.nj[l] : q0 + K) - q0;
        if (n <= 0) continue;
        float* dst = world_words_w(a, tile * kLanes + l) + (a.L.joint_off + (size_t)B3X_JOINT_BYTES * q0) / 4;
        for (int kk = 0; kk < n; kk++) {
            if (!ldi(item(slot + a.SP.joint, q0 + kk, NJF) + l, JOK)) continue;
            const float* row = out_row(sh, l, kk, K, NVW);
            for (int c = i; c < NVW; c += 32) store_world(dst + kk * NVW + c, row[c]);
        }
    }
}

// The state-only write-back of the resident columns (kStepStateOnly): of a
// contact only the words a later step reads -- its warm-start cache (pair,
// point count, features, impulses; point words up to the point count, as the
// full write-back) -- straight from the workspace columns; of a joint only
// its impulses.  The words steps merely output (prepared solver terms) keep
// the bytes of the last full write-back.
B3X_HD void o_contact_state(const Args& a, int tile, float* slot, OutShared& sh, int t) {
    for (int j = t; j < sh.maxn * kLanes; j += kCta) {
        const int k = j >> 5, l = j & 31;
        if (k >= sh.n[l]) continue;
        const float* co = item(slot + a.SP.cont, k, kCI) + l;
        const int cnt = clampi(ldi(co, WCNT), 0, B3_MAX_MANIFOLD);
        const size_t base = a.L.contact_off / 4 + (size_t)k * NCW;
        for (int f = 0; f < NOF; f++) {
            const int p = f < OFEAT ? -1 : (f < ONI ? f - OFEAT : f - ONI);
            if (p >= cnt) continue;
            const int w = old_word(f);
            store_world(res_word(a, tile, base + w, l), COL(co, w));
        }
    }
}

B3X_HD void o_joint_state(const Args& a, int tile, float* slot, OutShared& sh, int t) {
    for (int j = t; j < sh.maxnj * kLanes; j += kCta) {
        const int q = j >> 5, l = j & 31;
        if (q >= sh.nj[l]) continue;
        const float* jo = item(slot + a.SP.joint, q, NJF) + l;
        if (!ldi(jo, JOK)) continue;
        const size_t base = a.L.joint_off / 4 + (size_t)q * NVW;
        auto put = [&](int v, int c) { store_world(res_word(a, tile, base + v, l), COL(jo, c)); };
        for (int c = 0; c < 3; c++) put(VLI + c, JLI + c);
        if (ldi(jo, JTYPE) == B3_JOINT_WELD) {
            for (int c = 0; c < 3; c++) put(VAI + c, JAI + c);
        } else {
            put(VPI, JPI);
            put(VPI + 1, JPI + 1);
            put(VSI, JSI);
            put(VMI, JMI);
            put(VLOI, JLOI);
            put(VUPI, JUPI);
        }
    }
}

// ---- contact and joint rows of the resident columns --------------------------------
// A contact's words [0, kCW) are the workspace item's (the same
// [item][word][lane] order: one line per word), copied straight across (point
// words up to the point count); the words the workspace does not keep are
// derived in place.  All but the solver's impulses are final once the
// collide phase has built the contact, so warps 1-3 write them while warp 0
// solves the tile (o_rows_early, 96 threads), and the write-back then
// stores the impulses (o_contact_impulses).  Prepared joint rows go the same
// way: all words but the impulses and hinge axes the solve finalizes during
// the solve, those after it (o_joint_impulses).

// The contact words the solve writes: per point its normal and accumulated
// impulses, then twist, friction and rolling impulses (08_contacts.inl:315-413).
B3X_HDI bool solver_word(int c) {
    if (c >= WP && c < WCA) {
        const int f = (c - WP) % NQW;
        return f == QNI || f == QTOT;
    }
    return c == WTWI || c == WFI || c == WFI + 1 || (c >= WRI && c < WRI + 3);
}

// The words of a prepared B3Joint row that the solve finalizes (put in by
// o_joint_patch): the linear impulse, then the angular impulse of a weld or
// the hinge impulses and perpendicular axes of a revolute joint.
B3X_HDI bool joint_solver_word(int v, bool weld) {
    if (v >= VLI && v < VLI + 3) return true;
    if (weld) return v >= VAI && v < VAI + 3;
    return v == VPI || v == VPI + 1 || v == VSI || v == VMI || v == VLOI || v == VUPI || (v >= VPX && v < VPX + 3)
        || (v >= VPY && v < VPY + 3);
}

// Run by the 96 threads of warps 1-3 (e = threadIdx.x - 32) during the
// solve: the other contact words of every contact, the derived words, then
// the joint rows but for the words the solve finalizes.  Reads only what the
// solve leaves unchanged (the contacts' other words, the prepared joint rows,
// the body constants, the record), writes only the columns' contact and
// joint rows.
B3X_HD void o_rows_early(const Args& a, int tile, float* slot, int e) {
    constexpr int kThreads = kCta - kLanes, kWarps = kThreads / kLanes;
    constexpr int kRun = (kCW + kWarps - 1) / kWarps;
    const size_t cw = a.L.contact_off / 4;
    const int l = e & 31, w0 = e >> 5;
    const int n = ldi(slot + a.SP.rec + l, RN);
    for (int k = 0; k < n; k++) {
        const float* co = item(slot + a.SP.cont, k, kCI) + l;
        const int hi = WP + clampi(ldi(co, WCNT), 0, B3_MAX_MANIFOLD) * NQW;
        float* dst = res_word(a, tile, cw + (size_t)k * NCW, l);
        float v[kRun];
#pragma unroll
        for (int i = 0; i < kRun; i++) {
            const int c = w0 + i * kWarps;
            v[i] = c < kCW && !solver_word(c) ? COL(co, c) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < kRun; i++) {
            const int c = w0 + i * kWarps;
            if (c < kCW && (c < hi || c >= WCA) && !solver_word(c)) store_world(dst + (size_t)c * kLanes, v[i]);
        }
    }
    // the derived words, read back from the rows the threads above wrote
#if defined(__CUDA_ARCH__)
    asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory");
#endif
    for (int k = w0; k < n; k += kWarps)
        o_contact_fill(a, slot, l, ColRow{res_word(a, tile, cw + (size_t)k * NCW, l)});
    // the prepared joint rows (collide phase), but for the words the solve
    // finalizes; invalid joints are left as they were
    const size_t jw = a.L.joint_off / 4;
    const int nj = ldi(slot + a.SP.rec + l, RNJ);
    for (int q = 0; q < nj; q++) {
        const float* jo = item(slot + a.SP.joint, q, NJF) + l;
        if (!ldi(jo, JOK)) continue;
        const bool weld = ldi(jo, JTYPE) == B3_JOINT_WELD;
        const float* ji = item(slot + a.SP.jimg, q, NVW) + l;
        float* dst = res_word(a, tile, jw + (size_t)q * NVW, l);
        for (int c = w0; c < NVW; c += kWarps)
            if (!joint_solver_word(c, weld)) store_world(dst + (size_t)c * kLanes, COL(ji, c));
    }
}

// After the solve: each valid joint's finalized words (o_joint_patch's).
B3X_HD void o_joint_impulses(const Args& a, int tile, float* slot, OutShared& sh, int t) {
    for (int j = t; j < sh.maxnj * kLanes; j += kCta) {
        const int q = j >> 5, l = j & 31;
        if (q >= sh.nj[l]) continue;
        const float* jo = item(slot + a.SP.joint, q, NJF) + l;
        if (!ldi(jo, JOK)) continue;
        const size_t base = a.L.joint_off / 4 + (size_t)q * NVW;
        auto put = [&](int v, int c) { store_world(res_word(a, tile, base + v, l), COL(jo, c)); };
        for (int c = 0; c < 3; c++) put(VLI + c, JLI + c);
        if (ldi(jo, JTYPE) == B3_JOINT_WELD) {
            for (int c = 0; c < 3; c++) put(VAI + c, JAI + c);
        } else {
            put(VPI, JPI);
            put(VPI + 1, JPI + 1);
            put(VSI, JSI);
            put(VMI, JMI);
            put(VLOI, JLOI);
            put(VUPI, JUPI);
            for (int c = 0; c < 3; c++) put(VPX + c, JPX + c);
            for (int c = 0; c < 3; c++) put(VPY + c, JPY + c);
        }
    }
}

// After the solve: each contact's impulses (point words up to its count).
B3X_HD void o_contact_impulses(const Args& a, int tile, const float* slot, OutShared& sh, int t) {
    const size_t cw = a.L.contact_off / 4;
    const int l = t & 31;
    for (int k = t >> 5; k < sh.n[l]; k += kCtaWarps) {
        const float* co = item(slot + a.SP.cont, k, kCI) + l;
        const int cnt = clampi(ldi(co, WCNT), 0, B3_MAX_MANIFOLD);
        float* dst = res_word(a, tile, cw + (size_t)k * NCW, l);
        float v[2 * B3_MAX_MANIFOLD + 6];
#pragma unroll
        for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
            v[2 * p] = COL(co, PW(p, QNI));
            v[2 * p + 1] = COL(co, PW(p, QTOT));
        }
        const int q = 2 * B3_MAX_MANIFOLD;
        v[q] = COL(co, WTWI);
        v[q + 1] = COL(co, WFI);
        v[q + 2] = COL(co, WFI + 1);
        v[q + 3] = COL(co, WRI);
        v[q + 4] = COL(co, WRI + 1);
        v[q + 5] = COL(co, WRI + 2);
#pragma unroll
        for (int p = 0; p < B3_MAX_MANIFOLD; p++) {
            if (p >= cnt) continue;
            store_world(dst + (size_t)PW(p, QNI) * kLanes, v[2 * p]);
            store_world(dst + (size_t)PW(p, QTOT) * kLanes, v[2 * p + 1]);
        }
        store_world(dst + (size_t)WTWI * kLanes, v[q]);
        store_world(dst + (size_t)WFI * kLanes, v[q + 1]);
        store_world(dst + (size_t)(WFI + 1) * kLanes, v[q + 2]);
        store_world(dst + (size_t)WRI * kLanes, v[q + 3]);
        store_world(dst + (size_t)(WRI + 1) * kLanes, v[q + 4]);
        store_world(dst + (size_t)(WRI + 2) * kLanes, v[q + 5]);
    }
}

// Items per write-back round: as many as the staging area holds, balanced.
B3X_HDI int out_items(int count, int row_floats) {
    int k = kStageFloats / (kLanes * row_floats);
    if (k < 1) k = 1;
    if (count <= 0) return 1;
    const int rounds = (count + k - 1) / k;
    return (count + rounds - 1) / rounds;
}

template <bool kRes>
B3X_HD void o_header(const Args& a, int tile, float* slot, OutShared& sh, int l) {
    if (!sh.live[l]) return;
    const float* rec = slot + a.SP.rec + l;
    if constexpr (kRes) {
        *res_word(a, tile, HNC, l) = COL(rec, RN);
        *res_word(a, tile, HOVC, l) = COL(rec, ROVF);
        *res_word(a, tile, HDROP, l) = COL(rec, RDROP);
    } else {
        float* hw = world_words_w(a, tile * kLanes + l);
        hw[HNC] = COL(rec, RN);
        hw[HOVC] = COL(rec, ROVF);
        hw[HDROP] = COL(rec, RDROP);
    }
}

template <bool kRes, class X>
B3X_HD void out_tile(X& x, const Args& a, int bt, OutShared& sh) {
    float* slot = slot_of(a, bt);
    const int tile = a.tile0 + bt;
    x.each([&](int t) { if (t < kLanes) o_record(a, slot, sh, t); });
    x.each([&](int t) { if (t == 0) o_maxima(sh); });
    if constexpr (kRes) {
        // resident columns: each (body, world) is finalized in place, one
        // word of consecutive worlds per warp access
        const size_t bw = B3X_WORLD_HEADER_BYTES / 4;
        x.each([&](int t) {
            for (int j = t; j < sh.maxnb * kLanes; j += kCta) {
                const int k = j >> 5, l = j & 31;
                if (k >= sh.nb[l]) continue;
                // the row in registers (loads in flight together), finalized,
                // then the words a finalize can write stored back (the
                // others keep their bytes; rewriting an unchanged word
                // stores the same bits)
                float* col = res_word(a, tile, bw + (size_t)k * NYW, l);
                float y[NYW];
                load_row(col, y);
                o_body(a, slot, k, l, (float*)y);
#pragma unroll
                for (int f = YPOS; f < YIM; f++) col[(size_t)f * kLanes] = y[f];
#pragma unroll
                for (int f = YIW; f < YIW + 9; f++) col[(size_t)f * kLanes] = y[f];
            }
        });
    } else {
        const int K = out_items(sh.maxnb, kRow);
        for (int k0 = 0; k0 < sh.maxnb; k0 += K) {
            x.each([&](int t) { o_body_gather(a, tile, sh, k0, K, t); });
            x.each([&](int t) { o_bodies(a, slot, sh, k0, K, t); });
            x.each([&](int t) { o_body_write(a, tile, sh, k0, K, t); });
        }
    }
    const bool state_only = kRes && (a.flags & kStepStateOnly) != 0;
    if (state_only) {
        x.each([&](int t) { o_contact_state(a, tile, slot, sh, t); });
        x.each([&](int t) { o_joint_state(a, tile, slot, sh, t); });
    }
    if constexpr (kRes) {
        // resident columns: every other contact word went to the columns
        // while the tile was solved (o_rows_early); the solver's impulses
        // follow now
        if (!state_only) x.each([&](int t) { o_contact_impulses(a, tile, slot, sh, t); });
    } else {
        const int K = out_items(sh.maxn, NCW);
        for (int k0 = 0; k0 < sh.maxn; k0 += K) {
            const int Kr = sh.maxn - k0 < K ? sh.maxn - k0 : K;
            // whole items: their separation words land on row words the
            // fill below overwrites
            x.each([&](int t) { o_stage(item(slot + a.SP.cont, k0, kCI), sh, Kr, kCI, NCW, t); });
            x.each([&](int t) { o_contacts(a, slot, sh, k0, Kr, t); });
            x.each([&](int t) { o_contact_write(a, tile, sh, k0, Kr, t); });
        }
    }
    if (!state_only) {
        if constexpr (kRes) {
            // the joint rows went to the columns during the solve too
            x.each([&](int t) { o_joint_impulses(a, tile, slot, sh, t); });
        } else {
            const int K = out_items(sh.maxnj, NVW);
            for (int q0 = 0; q0 < sh.maxnj; q0 += K) {
                const int Kr = sh.maxnj - q0 < K ? sh.maxnj - q0 : K;
                x.each([&](int t) { o_stage(item(slot + a.SP.jimg, q0, NVW), sh, Kr, NVW, NVW, t); });
                x.each([&](int t) { o_joints(a, slot, sh, q0, Kr, t); });
                x.each([&](int t) { o_joint_write(a, tile, slot, sh, q0, Kr, t); });
            }
        }
    }
    x.each([&](int t) { if (t < kLanes) o_header<kRes>(a, tile, slot, sh, t); });
}

}  // namespace b3x
