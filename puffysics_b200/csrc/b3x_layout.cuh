// b3x_layout.cuh -- world layout, workspace layout and column accessors of the
// batched step (kernels in b3x_step.cu, phases in b3x_phases.cuh).
//
// Tiles.  A tile is 32 consecutive worlds; world `l` of a tile is its lane.
// Every per-world working value lives in a per-tile workspace slot in global
// memory as lane-interleaved columns, region[item][field][lane]: the 32 values
// of one field of item k of the tile's worlds are one contiguous 128-byte
// line, so a warp whose lanes are the tile's worlds reads or writes a field
// with one coalesced access, and one item of all 32 worlds is one contiguous
// block (the unit the solver streams into shared memory with bulk copies).
//
// Contacts keep the word order of the reference's B3Contact
// (src/puffysics/02_types.inl) as their column order, so the kernel that
// writes the world back turns a contact column block into 32 B3Contact images
// without a lookup table; joints use a solver-first column order and a table.
#pragma once
#include <cstdint>
#include <cstring>

#include "puffysics_b200.h"
#include "b3x_math.cuh"

namespace b3x {

constexpr int kLanes = 32;

// ---- AoS word offsets of the reference structs (02_types.inl) ----------------
// B3World header: gravity, contact parameters, counts (02_types.inl:306-327).
enum : int {
    HGRAV = 0, HHZ = 3, HDAMP = 4, HSPEED = 5, HRT = 6, HMAXLIN = 7, HNB = 8, HNS = 9, HNC = 10, HNJ = 11,
    HOVB = 12, HOVS = 13, HOVJ = 14, HOVC = 15, HDROP = 16, NHW = 17
};
// B3Body (50 words)
enum : int {
    YPOS = 0, YROT = 3, YCEN = 7, YLC = 10, YLV = 13, YAV = 16, YF = 19, YT = 22, YDP = 25, YDQ = 28, YIM = 32,
    YII = 33, YIW = 36, YLD = 45, YAD = 46, YGS = 47, YTYPE = 48, YFLAGS = 49, NYW = 50
};
// B3Shape (22 words; words 18-19 / 20-21 hold the 64-bit category / mask)
enum : int {
    XBODY = 0, XTYPE = 1, XLPOS = 2, XLROT = 5, XRAD = 9, XHALF = 10, XFRIC = 13, XREST = 14, XROLL = 15,
    XCAT = 18, XMASK = 20, NXW = 22
};
// B3Contact (119 words), also the contact column order.  Point p occupies
// WP + p * NQW ...
enum : int {
    WSA = 0, WSB = 1, WBA = 2, WBB = 3, WCNT = 4, WSTAT = 5, WN = 6, WT1 = 9, WT2 = 12, WP = 15,
    QRA = 0, QRB = 3, QBSEP = 6, QRELV = 7, QNI = 8, QTOT = 9, QNM = 10, QLEV = 11, QFEAT = 12, NQW = 13,
    WCA = WP + B3_MAX_MANIFOLD * NQW, WCB = WCA + 3, WFRIC = WCB + 3, WREST = WFRIC + 1, WROLL = WREST + 1,
    WTWM = WROLL + 1, WTWI = WTWM + 1, WFI = WTWI + 1, WRI = WFI + 2, WTM = WRI + 3, WRM = WTM + 4,
    WMA = WRM + 9, WMB = WMA + 1, WIA = WMB + 1, WIB = WIA + 9, WSOFT = WIB + 9, NCW = WSOFT + 3
};
static_assert(NCW * 4 == B3X_CONTACT_BYTES, "contact word layout");
// The workspace keeps contact words [0, kCW): everything the solver reads or
// writes; the write-back derives the rest (masses, inertias, rolling mass,
// softness) from the body columns.
constexpr int kCW = WTM + 4;
// A workspace contact item is those words, then the separation of each point
// as the last relax sweep computed it (WSEP + p): positions do not move
// between a substep's relax sweep and the next substep's bias sweep, so that
// sweep reads the separations instead of recomputing them.
constexpr int WSEP = kCW;
constexpr int kCI = kCW + B3_MAX_MANIFOLD;
constexpr int kContactStream = kCI;
// B3Joint (115 words)
enum : int {
    VTYPE = 0, VBA = 1, VBB = 2, VCC = 3, VFIX = 4, VLAA = 5, VLAB = 8, VLRA = 11, VLRB = 15, VCHZ = 19,
    VCDMP = 20, VSOFT = 21, VIMA = 24, VIMB = 25, VIIA = 26, VIIB = 35, VFPA = 44, VFPB = 47, VFQA = 50,
    VFQB = 54, VDC = 58, VLI = 61, VAI = 64, VAM = 67, VLHZ = 76, VLDMP = 77, VAHZ = 78, VADMP = 79, VLS = 80,
    VAS = 83, VPI = 86, VSI = 88, VMI = 89, VLOI = 90, VUPI = 91, VHZ = 92, VDR = 93, VMMT = 94, VMS = 95,
    VTA = 96, VLA = 97, VUA = 98, VENS = 99, VENM = 100, VENL = 101, VAX = 102, VPX = 105, VPY = 108,
    VAXM = 111, VSS = 112, NVW = 115
};
static_assert(NVW * 4 == B3X_JOINT_BYTES, "joint word layout");

// ---- workspace column fields ---------------------------------------------------
// per-world record
// (live flag, clamped counts, new contact count and overflow accounting,
// header parameters, contact / static-contact softness of the step)
enum : int {
    RLIVE = 0, RNB = 1, RNS = 2, ROLDN = 3, RNJ = 4, RN = 5, ROVF = 6, RDROP = 7, RSPEED = 8, RRT = 9,
    RMAXLIN = 10, RCS = 11, RSS = 14, NRF = 17
};
// body velocities (region body): the fields every contact and joint row
// updates
enum : int { BV = 0, BW = 3, NBF = 6 };
// body pose deltas (region bodyp), advanced once per substep
enum : int { BDP = 0, BDQ = 3, NBP = 7 };
// body constants of the step (region bodyk): inverse mass and world inverse
// inertia gated by type, flags, type
enum : int { BMI = 0, BII = 1, BFLAGS = 10, BTYPE = 11, NBC = 12 };
// per-body step constants: velocity / spin increments and damping factors
// of b3_integrate_velocity_state, constant over the substeps
enum : int { KDV = 0, KDW = 3, KLD = 6, KAD = 7, NKF = 8 };
// shape: world pose, padded AABB, geometry, filter, material
enum : int {
    SPOS = 0, SROT = 3, SLO = 7, SHI = 10, STYPE = 13, SBODY = 14, SRAD = 15, SHALF = 16, SCAT = 19, SMASK = 21,
    SFRIC = 23, SREST = 24, SROLL = 25, NSF = 26
};
// warm-start cache of the previous step's contacts
enum : int { OSA = 0, OSB = 1, OCNT = 2, OFI = 3, OTWI = 5, ORI = 6, OFEAT = 9, ONI = 13, NOF = 17 };
// body pose: the first 13 words of B3Body (position, rotation, center,
// local center)
enum : int { PPOS = YPOS, PROT = YROT, PCEN = YCEN, PLC = YLC, NPF = YLC + 3 };
// joints: the solver's columns [0, kJointStream), then the collide filter's
// collide_connected flag
enum : int {
    JTYPE = 0, JBA = 1, JBB = 2, JFIX = 3, JENS = 4, JENM = 5, JENL = 6, JFPA = 7, JFPB = 10, JFQA = 13,
    JFQB = 17, JDC = 21, JSOFT = 24, JLI = 27, JAI = 30, JAM = 33, JLH = 42, JAH = 43, JLS = 44, JAS = 47,
    JPI = 50, JSI = 52, JMI = 53, JLOI = 54, JUPI = 55, JMMT = 56, JMS = 57, JTA = 58, JLA = 59, JUA = 60,
    JAX = 61, JPX = 64, JPY = 67, JAXM = 70, JSS = 71, JOK = 74, JCC = 75, NJF = 76
};
constexpr int kJointStream = JOK + 1;
constexpr int kStreamWords = kContactStream > kJointStream ? kContactStream : kJointStream;

// Candidate pairs are tested in windows of kPairWindow consecutive pair
// indices (lexicographic (i, j) order, the reference's loop order).
constexpr int kPairWindow = 128;
// A manifold of the narrowphase, parked between the narrowphase and the
// contact build of a window (region mani, one item per window candidate):
// point count, normal, then per point p_a, p_b, separation, feature id.
enum : int { MCNT = 0, MN = 1, MPA = 4, MPB = 16, MSEP = 28, MFEAT = 32, NMW = 36 };

// World header (the first 68 bytes of B3World).
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

// Word offsets of the regions of one tile's workspace slot.
// Besides the solver columns, the prepared B3Joint rows (jimg) travel from the
// collide phase to the write-back, which then writes whole rows.  The
// manifolds of a pair window wait in region mani until their contact slots
// are known.
struct Space {
    unsigned long long rec, body, bodyp, bodyk, konst, pose, shape, old, cont, mani, joint, jimg, tile_words;
};

static inline Space space_from_layout(const Layout& L) {
    Space s;
    unsigned long long w = 0;
    auto take = [&](unsigned long long items, int fields) {
        unsigned long long at = w;
        w += items * (unsigned long long)fields * kLanes;
        return at;
    };
    s.rec = take(1, NRF);
    s.body = take(L.B, NBF);
    s.bodyp = take(L.B, NBP);
    s.bodyk = take(L.B, NBC);
    s.konst = take(L.B, NKF);
    s.pose = take(L.B, NPF);
    s.shape = take(L.S, NSF);
    s.old = take(L.C, NOF);
    s.cont = take(L.C, kCI);
    s.mani = take(kPairWindow, NMW);
    s.joint = take(L.J, NJF);
    s.jimg = take(L.J, NVW);
    s.tile_words = (w + 63) & ~63ull;   // 256-byte aligned slots
    return s;
}

// Launch arguments shared by the step kernels.
struct Args {
    unsigned char* data;
    unsigned long long stride, offset;
    int count;
    const unsigned char* active;
    float dt;
    int substeps, joint_iters, relax_iters;
    int flags;     // kStepInterleaveContacts | kStepSkipRestitution
    Layout L;
    Space SP;
    float* ws;     // workspace slot of the launch's first tile
    int tile0;     // first tile of this launch
    // Resident world columns (the b3x_engine_* entry points): word w of the
    // B3World of tile-lane l of tile t at res[(t * resW + w) * 32 + l]; null
    // when the step reads and writes the caller's AoS worlds.
    float* res;
    unsigned long long resW;   // words of one B3World
};

// ---- column accessors (c points at an item's column of one lane) -----------
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
B3X_HDI void st22(float* c, int i, B3Mat2 m) {
    COL(c, i) = m.cx.x; COL(c, i + 1) = m.cx.y; COL(c, i + 2) = m.cy.x; COL(c, i + 3) = m.cy.y;
}

// item k of a [item][field][lane] region with nf fields
B3X_HDI float* item(float* base, int k, int nf) { return base + (size_t)k * nf * kLanes; }
B3X_HDI const float* item(const float* base, int k, int nf) { return base + (size_t)k * nf * kLanes; }
// word of contact point p
B3X_HDI int PW(int p, int f) { return WP + p * NQW + f; }
// body column field of body k (body columns are [body][field][lane])
B3X_HDI int BI(int k, int f) { return k * NBF + f; }
// pose-delta field f of body k (bodyp columns are [body][field][lane])
B3X_HDI int BP(int k, int f) { return k * NBP + f; }
// constant field f of body k (bodyk columns are [body][field][lane])
B3X_HDI int BK(int k, int f) { return k * NBC + f; }

B3X_HDI int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Read-only global load (the caller's worlds are not written while read).
B3X_HDI float ldg(const float* p) {
#if defined(__CUDA_ARCH__)
    return __ldg(p);
#else
    return *p;
#endif
}

// ---- bit helpers (device intrinsics or portable equivalents) --------------------
B3X_HDI int popc32(uint32_t x) {
#if defined(__CUDA_ARCH__)
    return __popc(x);
#else
    return __builtin_popcount(x);
#endif
}
// index of the n-th (0-based) set bit of x; x has more than n set bits
B3X_HDI int nth_bit32(uint32_t x, int n) {
#if defined(__CUDA_ARCH__)
    return (int)__fns(x, 0, n + 1);
#else
    for (int b = 0; b < 32; b++)
        if ((x >> b) & 1u) {
            if (n == 0) return b;
            n--;
        }
    return -1;
#endif
}
B3X_HDI int ctz32(uint32_t x) {
#if defined(__CUDA_ARCH__)
    return __ffs((int)x) - 1;
#else
    return __builtin_ctz(x);
#endif
}
B3X_HDI void shared_max(int* p, int v) {
#if defined(__CUDA_ARCH__)
    atomicMax(p, v);
#else
    if (v > *p) *p = v;
#endif
}
// 4-byte asynchronous copy global -> shared (cp.async); the copies of a
// thread complete at async_wait(), and a block barrier then publishes them.
B3X_HDI void async_copy4(float* dst_shared, const float* src_global) {
#if defined(__CUDA_ARCH__)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst_shared)),
                 "l"(__cvta_generic_to_global(src_global)) : "memory");
#else
    *dst_shared = *src_global;
#endif
}
// The same for the caller's world array, which a step reads once and writes
// once: its lines are marked first for eviction from L2, so the workspace,
// which the step re-reads many times, stays resident.
B3X_HDI void async_copy4_world(float* dst_shared, const float* src_global) {
#if defined(__CUDA_ARCH__)
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 4, %2;"
                 ::"r"((uint32_t)__cvta_generic_to_shared(dst_shared)),
                 "l"(__cvta_generic_to_global(src_global)), "l"(pol) : "memory");
#else
    *dst_shared = *src_global;
#endif
}
B3X_HDI void store_world(float* p, float v) {
#if defined(__CUDA_ARCH__)
    __stcs(p, v);
#else
    *p = v;
#endif
}
B3X_HDI void async_wait() {
#if defined(__CUDA_ARCH__)
    asm volatile("cp.async.wait_all;" ::: "memory");
#endif
}
B3X_HDI void shared_or(uint32_t* p, uint32_t v) {
#if defined(__CUDA_ARCH__)
    atomicOr(p, v);
#else
    *p |= v;
#endif
}

}  // namespace b3x
