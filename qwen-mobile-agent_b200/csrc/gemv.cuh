// gemv.cuh -- super-block dot "units" for Q4_K / Q6_K / Q8_0 weights against
// Q8_K activations, and the warp-cooperative GEMV built on them.
//
// A unit is the slice of one weight row a lane owns: 64 weights of a Q4_K
// super-block (one (scale, min) pair of 32-lane sub-blocks), 128 weights
// (one half) of a Q6_K super-block, or 64 weights (two blocks) of Q8_0.
// Consecutive lanes own consecutive units, so a warp streams contiguous row
// bytes with 16-byte loads; the activation slice of a unit stays in
// registers and is reused for every row the warp visits.
//
// Integer work is exact (__dp4a): per-sub-block int32 sums equal the
// reference's SDOT partials (q8k.c:89-262).  Only the fp32 combination of
// those integers with the fp16 scales is ordered differently.
#pragma once
#include "common.cuh"

namespace qma {


// ------------------------------------------------------------------ Q4_K --
struct FmtQ4K {
    static constexpr int UNIT = 64;
    static constexpr int XW = 16;           // activation words per unit
    using Ptr = const uint8_t *;
    struct Act { int x[16]; float xd; int xs01, xs23; };
    struct Wt { uint4 h, q0, q1; };

    __device__ static void load_act(Act &a, const int8_t *xq, const float *xd,
                                    const int16_t *xsum, int u) {
        const int sb = u >> 2, g = u & 3;
        const int4 *p = reinterpret_cast<const int4 *>(xq + sb * 256 + g * 64);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int4 v = p[k];
            a.x[4 * k] = v.x; a.x[4 * k + 1] = v.y; a.x[4 * k + 2] = v.z; a.x[4 * k + 3] = v.w;
        }
        a.xd = xd[sb];
        const int16_t *s = xsum + sb * 16 + g * 4;
        a.xs01 = int(s[0]) + int(s[1]);
        a.xs23 = int(s[2]) + int(s[3]);
    }
    __device__ static void prefetch_rows(Ptr W, int r0, int nrows, int n_in) {
        prefetch_l2_range(W + size_t(r0) * (n_in / 256) * 144, size_t(nrows) * (n_in / 256) * 144);
    }
    __device__ static void load_w(Wt &w, Ptr W, int row, int n_in, int u) {
        const uint8_t *b = W + size_t(row) * (n_in / 256) * 144 + (u >> 2) * 144;
        w.h = ld_stream16(b);
        w.q0 = ld_stream16(b + 16 + (u & 3) * 32);
        w.q1 = ld_stream16(b + 32 + (u & 3) * 32);
    }
    // the same unit from a copy of the rows in shared memory
    __device__ static void load_w_smem(Wt &w, Ptr W, int row, int n_in, int u) {
        const uint8_t *b = W + size_t(row) * (n_in / 256) * 144 + (u >> 2) * 144;
        w.h = *reinterpret_cast<const uint4 *>(b);
        w.q0 = *reinterpret_cast<const uint4 *>(b + 16 + (u & 3) * 32);
        w.q1 = *reinterpret_cast<const uint4 *>(b + 32 + (u & 3) * 32);
    }
    // exact integer sub-block sums (low nibbles -> sub-block 2g, high -> 2g+1)
    __device__ static void isums(const Wt &w, const Act &a, int &lo, int &hi) {
        const uint32_t q[8] = {w.q0.x, w.q0.y, w.q0.z, w.q0.w, w.q1.x, w.q1.y, w.q1.z, w.q1.w};
        int s0 = 0, s1 = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            s0 = __dp4a(int(q[k] & 0x0F0F0F0Fu), a.x[k], s0);
            s1 = __dp4a(int((q[k] >> 4) & 0x0F0F0F0Fu), a.x[8 + k], s1);
        }
        lo = s0;
        hi = s1;
    }
    __device__ static float dot(const Wt &w, const Act &a, int u) {
        int lo, hi;
        isums(w, a, lo, hi);
        // get_scale_min_k4 (quants.c:18-26) for sub-blocks 2g and 2g+1, both
        // at once on byte pairs and without branching on the lane's g:
        //   j < 4 : sc = s[j] & 63, m = s[j+4] & 63
        //   j >= 4: sc = (s[j+4] & 15) | (s[j-4] >> 6) << 4,
        //           m  = (s[j+4] >> 4) | (s[j] >> 6) << 4
        const int g = u & 3;
        const uint32_t sh = 16u * uint32_t(g & 1);
        const uint32_t A = (w.h.y >> sh) & 0xffffu;        // s[2g'], s[2g'+1]
        const uint32_t B = (w.h.z >> sh) & 0xffffu;        // s[4+2g'], s[5+2g']
        const uint32_t Cc = (w.h.w >> sh) & 0xffffu;       // s[8+2g'], s[9+2g']
        const uint32_t scp = g < 2 ? (A & 0x3f3fu) : ((Cc & 0x0f0fu) | ((A & 0xc0c0u) >> 2));
        const uint32_t mp = g < 2 ? (B & 0x3f3fu) : (((Cc >> 4) & 0x0f0fu) | ((B & 0xc0c0u) >> 2));
        const int sc0 = int(scp & 0xffu), sc1 = int(scp >> 8), m0 = int(mp & 0xffu), m1 = int(mp >> 8);
        const int I1 = sc0 * lo + sc1 * hi;
        const int I2 = m0 * a.xs01 + m1 * a.xs23;
        const float d = h2f(uint16_t(w.h.x & 0xffff));
        const float dmin = h2f(uint16_t(w.h.x >> 16));
        return a.xd * (d * float(I1) - dmin * float(I2));
    }
};

// ------------------------------------------------------------------ Q6_K --
struct FmtQ6K {
    static constexpr int UNIT = 128;
    static constexpr int XW = 32;
    using Ptr = Q6Planes;
    struct Act { int x[32]; float xd; };
    struct Wt { uint4 l0, l1, l2, l3, h0, h1; uint2 sc; uint16_t d; };

    __device__ static void load_act(Act &a, const int8_t *xq, const float *xd,
                                    const int16_t *, int u) {
        const int4 *p = reinterpret_cast<const int4 *>(xq + u * 128);
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int4 v = p[k];
            a.x[4 * k] = v.x; a.x[4 * k + 1] = v.y; a.x[4 * k + 2] = v.z; a.x[4 * k + 3] = v.w;
        }
        a.xd = xd[u >> 1];
    }
    __device__ static void prefetch_rows(const Ptr &P, int r0, int nrows, int n_in) {
        prefetch_l2_range(P.ql + size_t(r0) * (n_in / 2), size_t(nrows) * (n_in / 2));
        prefetch_l2_range(P.qh + size_t(r0) * (n_in / 4), size_t(nrows) * (n_in / 4));
        prefetch_l2_range(P.sc + size_t(r0) * (n_in / 16), size_t(nrows) * (n_in / 16));
        prefetch_l2_range(P.d + size_t(r0) * (n_in / 256), size_t(nrows) * (n_in / 256) * 2);
    }
    // unit u = (sb, half j) of a row: ql chunks 4j..4j+3 and qh chunks 2j, 2j+1
    // of segment s = row * (n_in/256) + sb, at their swizzled places
    __device__ static void load_w(Wt &w, const Ptr &P, int row, int n_in, int u) {
        const int sb = u >> 1, j = u & 1, s = row * (n_in / 256) + sb;
        const uint8_t *ql = P.ql + size_t(row) * (n_in / 2) + sb * 128;
        const uint8_t *qh = P.qh + size_t(row) * (n_in / 4) + sb * 64;
        w.l0 = ld_stream16(ql + 16 * q6_ql_chunk(4 * j, s));
        w.l1 = ld_stream16(ql + 16 * q6_ql_chunk(4 * j + 1, s));
        w.l2 = ld_stream16(ql + 16 * q6_ql_chunk(4 * j + 2, s));
        w.l3 = ld_stream16(ql + 16 * q6_ql_chunk(4 * j + 3, s));
        w.h0 = ld_stream16(qh + 16 * q6_qh_chunk(2 * j, s));
        w.h1 = ld_stream16(qh + 16 * q6_qh_chunk(2 * j + 1, s));
        w.sc = ld_stream8(P.sc + size_t(row) * (n_in / 16) + sb * 16 + j * 8);
        w.d = ld_stream2(P.d + size_t(row) * (n_in / 256) + sb);
    }
    __device__ static void load_w_smem(Wt &w, const Ptr &P, int row, int n_in, int u) {
        const int sb = u >> 1, j = u & 1, s = row * (n_in / 256) + sb;
        const uint8_t *ql = P.ql + size_t(row) * (n_in / 2) + sb * 128;
        const uint8_t *qh = P.qh + size_t(row) * (n_in / 4) + sb * 64;
        w.l0 = *reinterpret_cast<const uint4 *>(ql + 16 * q6_ql_chunk(4 * j, s));
        w.l1 = *reinterpret_cast<const uint4 *>(ql + 16 * q6_ql_chunk(4 * j + 1, s));
        w.l2 = *reinterpret_cast<const uint4 *>(ql + 16 * q6_ql_chunk(4 * j + 2, s));
        w.l3 = *reinterpret_cast<const uint4 *>(ql + 16 * q6_ql_chunk(4 * j + 3, s));
        w.h0 = *reinterpret_cast<const uint4 *>(qh + 16 * q6_qh_chunk(2 * j, s));
        w.h1 = *reinterpret_cast<const uint4 *>(qh + 16 * q6_qh_chunk(2 * j + 1, s));
        w.sc = *reinterpret_cast<const uint2 *>(P.sc + size_t(row) * (n_in / 16) + sb * 16 + j * 8);
        w.d = *reinterpret_cast<const uint16_t *>(P.d + size_t(row) * (n_in / 256) + sb);
    }
    // exact sum over the 8 sixteen-lane groups of scale_g * sum((q-32)*xq)
    __device__ static int isum(const Wt &w, const Act &a) {
        const uint32_t QL[16] = {w.l0.x, w.l0.y, w.l0.z, w.l0.w, w.l1.x, w.l1.y, w.l1.z, w.l1.w,
                                 w.l2.x, w.l2.y, w.l2.z, w.l2.w, w.l3.x, w.l3.y, w.l3.z, w.l3.w};
        const uint32_t QH[8] = {w.h0.x, w.h0.y, w.h0.z, w.h0.w, w.h1.x, w.h1.y, w.h1.z, w.h1.w};
        int I = 0;
#pragma unroll
        for (int g = 0; g < 8; g++) {
            int p = 0;
#pragma unroll
            for (int i4 = 0; i4 < 4; i4++) {
                const int i = 4 * g + i4;              // quad of lanes 4i..4i+3
                const int hi = i >> 4;
                const int shift = 2 * (((i >> 3) & 1) + 2 * hi);
                const uint32_t lo4 = (QL[i & 15] >> (4 * hi)) & 0x0F0F0F0Fu;
                const uint32_t h2 = ((QH[i & 7] >> shift) & 0x03030303u) << 4;
                const int v = int(__vsub4(lo4 | h2, 0x20202020u));
                p = __dp4a(v, a.x[i], p);
            }
            const uint32_t sw = g < 4 ? w.sc.x : w.sc.y;
            const int sc = int(int8_t((sw >> ((g & 3) * 8)) & 0xff));
            I += sc * p;
        }
        return I;
    }
    __device__ static float dot(const Wt &w, const Act &a, int) {
        const int I = isum(w, a);
        return h2f(w.d) * a.xd * float(I);
    }
};

// ------------------------------------------------------------------ Q8_0 --
struct FmtQ80 {
    static constexpr int UNIT = 64;
    static constexpr int XW = 16;
    using Ptr = Q8Planes;
    struct Act { int x[16]; float xd; };
    struct Wt { uint4 q0, q1, q2, q3; uint32_t d2; };

    __device__ static void load_act(Act &a, const int8_t *xq, const float *xd,
                                    const int16_t *, int u) {
        const int4 *p = reinterpret_cast<const int4 *>(xq + u * 64);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int4 v = p[k];
            a.x[4 * k] = v.x; a.x[4 * k + 1] = v.y; a.x[4 * k + 2] = v.z; a.x[4 * k + 3] = v.w;
        }
        a.xd = xd[u >> 2];
    }
    __device__ static void prefetch_rows(const Ptr &P, int r0, int nrows, int n_in) {
        prefetch_l2_range(P.q + size_t(r0) * n_in, size_t(nrows) * n_in);
        prefetch_l2_range(P.d + size_t(r0) * (n_in / 32), size_t(nrows) * (n_in / 32) * 2);
    }
    __device__ static void load_w(Wt &w, const Ptr &P, int row, int n_in, int u) {
        const int8_t *q = P.q + size_t(row) * n_in + u * 64;
        w.q0 = ld_stream16(q);
        w.q1 = ld_stream16(q + 16);
        w.q2 = ld_stream16(q + 32);
        w.q3 = ld_stream16(q + 48);
        w.d2 = ld_stream4(P.d + size_t(row) * (n_in / 32) + u * 2);
    }
    __device__ static void load_w_smem(Wt &w, const Ptr &P, int row, int n_in, int u) {
        const uint4 *q = reinterpret_cast<const uint4 *>(P.q + size_t(row) * n_in + u * 64);
        w.q0 = q[0]; w.q1 = q[1]; w.q2 = q[2]; w.q3 = q[3];
        w.d2 = *reinterpret_cast<const uint32_t *>(P.d + size_t(row) * (n_in / 32) + u * 2);
    }
    __device__ static void isums(const Wt &w, const Act &a, int &i0, int &i1) {
        const uint32_t q[16] = {w.q0.x, w.q0.y, w.q0.z, w.q0.w, w.q1.x, w.q1.y, w.q1.z, w.q1.w,
                                w.q2.x, w.q2.y, w.q2.z, w.q2.w, w.q3.x, w.q3.y, w.q3.z, w.q3.w};
        int s0 = 0, s1 = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            s0 = __dp4a(int(q[k]), a.x[k], s0);
            s1 = __dp4a(int(q[8 + k]), a.x[8 + k], s1);
        }
        i0 = s0;
        i1 = s1;
    }
    __device__ static float dot(const Wt &w, const Act &a, int) {
        int i0, i1;
        isums(w, a, i0, i1);
        const float d0 = h2f(uint16_t(w.d2 & 0xffff)), d1 = h2f(uint16_t(w.d2 >> 16));
        return (float(i0) * d0 + float(i1) * d1) * a.xd;
    }
};

// Staging of rows [r0, r0 + nr) of a matrix into shared memory by the TMA
// engine (one bulk copy per plane), and the view of that copy as a matrix
// of nr rows.  Plane copies start 16-byte aligned (r0 a multiple of 8) and
// are rounded up to 16 bytes, which stays inside the packed matrix (every
// plane is padded to 16 bytes).
__host__ __device__ constexpr uint32_t up16(uint32_t x) { return (x + 15u) & ~15u; }
template <class F> struct Stage;
template <> struct Stage<FmtQ4K> {
    __host__ __device__ static uint32_t bytes(int nr, int n) { return up16(uint32_t(nr) * (n / 256) * 144); }
    __device__ static void issue(const uint8_t *W, int r0, int nr, int n, uint8_t *dst, uint64_t *bar, int lane) {
        const uint32_t b = bytes(nr, n);
        if (lane == 0) mbar_expect_tx(bar, b);
        __syncwarp();
        bulk_g2s_warp(dst, W + size_t(r0) * (n / 256) * 144, b, bar, lane);
    }
    __device__ static const uint8_t *view(const uint8_t *dst, int, int) { return dst; }
};
template <> struct Stage<FmtQ6K> {
    __host__ __device__ static uint32_t ql(int nr, int n) { return up16(uint32_t(nr) * (n / 2)); }
    __host__ __device__ static uint32_t qh(int nr, int n) { return up16(uint32_t(nr) * (n / 4)); }
    __host__ __device__ static uint32_t sc(int nr, int n) { return up16(uint32_t(nr) * (n / 16)); }
    __host__ __device__ static uint32_t d(int nr, int n) { return up16(uint32_t(nr) * (n / 256) * 2); }
    __host__ __device__ static uint32_t bytes(int nr, int n) { return ql(nr, n) + qh(nr, n) + sc(nr, n) + d(nr, n); }
    __device__ static void issue(const Q6Planes &P, int r0, int nr, int n, uint8_t *dst, uint64_t *bar, int lane) {
        if (lane == 0) mbar_expect_tx(bar, bytes(nr, n));
        __syncwarp();
        bulk_g2s_warp(dst, P.ql + size_t(r0) * (n / 2), ql(nr, n), bar, lane);
        dst += ql(nr, n);
        bulk_g2s_warp(dst, P.qh + size_t(r0) * (n / 4), qh(nr, n), bar, lane);
        dst += qh(nr, n);
        bulk_g2s_warp(dst, P.sc + size_t(r0) * (n / 16), sc(nr, n), bar, lane);
        dst += sc(nr, n);
        bulk_g2s_warp(dst, P.d + size_t(r0) * (n / 256), d(nr, n), bar, lane);
    }
    __device__ static Q6Planes view(const uint8_t *dst, int nr, int n) {
        Q6Planes P;
        P.ql = dst;
        P.qh = dst + ql(nr, n);
        P.sc = reinterpret_cast<const int8_t *>(P.qh + qh(nr, n));
        P.d = reinterpret_cast<const __half *>(reinterpret_cast<const uint8_t *>(P.sc) + sc(nr, n));
        return P;
    }
};
template <> struct Stage<FmtQ80> {
    __host__ __device__ static uint32_t q(int nr, int n) { return up16(uint32_t(nr) * n); }
    __host__ __device__ static uint32_t d(int nr, int n) { return up16(uint32_t(nr) * (n / 32) * 2); }
    __host__ __device__ static uint32_t bytes(int nr, int n) { return q(nr, n) + d(nr, n); }
    __device__ static void issue(const Q8Planes &P, int r0, int nr, int n, uint8_t *dst, uint64_t *bar, int lane) {
        if (lane == 0) mbar_expect_tx(bar, bytes(nr, n));
        __syncwarp();
        bulk_g2s_warp(dst, P.q + size_t(r0) * n, q(nr, n), bar, lane);
        bulk_g2s_warp(dst + q(nr, n), P.d + size_t(r0) * (n / 32), d(nr, n), bar, lane);
    }
    __device__ static Q8Planes view(const uint8_t *dst, int nr, int n) {
        Q8Planes P;
        P.q = reinterpret_cast<const int8_t *>(dst);
        P.d = reinterpret_cast<const __half *>(dst + q(nr, n));
        return P;
    }
};

// A format whose weights are read from a copy in shared memory.
template <class F> struct SmemRows : F {
    __device__ static void load_w(typename F::Wt &w, const typename F::Ptr &W, int row, int n_in, int u) {
        F::load_w_smem(w, W, row, n_in, u);
    }
};

// ---------------------------------------------------------------- GEMV ----
// LPR lanes cooperate on one row (LPR = units per row when a row has fewer
// than 32 units, else 32); each lane owns UPL units of the row; T tokens
// are processed per pass with their activation slices in registers.  A warp
// issues the loads of RU row groups before computing any of them, so every
// lane keeps RU*UPL units of weights in flight.  With PRE, the first sweep's
// weights are loaded before pdl_wait(): a launch sized so that one sweep
// covers the matrix has all its weights in registers by the time the
// upstream kernel's activations are ready.
template <class F, int T, int LPR, int UPL, int RU, bool PRE = false>
__device__ __forceinline__ void gemv_warp_rows(const typename F::Ptr &W, int n_in, int n_out,
                                               const int8_t *xq, const float *xd,
                                               const int16_t *xsum, float *out, int out_ld,
                                               int warp, int nwarps, int lane,
                                               const float *resid = nullptr) {
    constexpr int RPW = 32 / LPR;
    const int lir = lane % LPR, slot = lane / LPR;
    typename F::Wt w[RU][UPL];
    auto load_rows = [&](int rb) {
#pragma unroll
        for (int ru = 0; ru < RU; ru++) {
            const int r = rb + ru * RPW + slot;
            if (r < n_out) {
#pragma unroll
                for (int k = 0; k < UPL; k++) F::load_w(w[ru][k], W, r, n_in, lir + k * LPR);
            }
        }
    };
    const int rb0 = warp * RPW * RU;
    if (PRE) {
        load_rows(rb0);
        pdl_wait();
    }
    typename F::Act act[UPL][T];
#pragma unroll
    for (int k = 0; k < UPL; k++)
#pragma unroll
        for (int t = 0; t < T; t++)
            F::load_act(act[k][t], xq + size_t(t) * n_in, xd + size_t(t) * (n_in / 256),
                        xsum + size_t(t) * (n_in / 16), lir + k * LPR);
    for (int rb = rb0; rb < n_out; rb += nwarps * RPW * RU) {
        if (!PRE || rb != rb0) load_rows(rb);
#pragma unroll
        for (int ru = 0; ru < RU; ru++) {
            const int r = rb + ru * RPW + slot;
            float acc[T];
#pragma unroll
            for (int t = 0; t < T; t++) acc[t] = 0.0f;
            if (r < n_out) {
#pragma unroll
                for (int k = 0; k < UPL; k++)
#pragma unroll
                    for (int t = 0; t < T; t++) acc[t] += F::dot(w[ru][k], act[k][t], lir + k * LPR);
            }
#pragma unroll
            for (int t = 0; t < T; t++) acc[t] = group_sum(acc[t], LPR);
            if (lir == 0 && r < n_out) {
                // optional residual: out = dot + resid (add_m, nn.c:375)
#pragma unroll
                for (int t = 0; t < T; t++)
                    out[size_t(t) * out_ld + r] =
                        resid ? __fadd_rn(acc[t], resid[size_t(t) * out_ld + r]) : acc[t];
            }
        }
    }
}

// int8 tensor-core MMA (mma.sync m16n8k32 / m16n8k16, s8 x s8 -> s32,
// accumulate into d) and the 8 scale/min pairs of a Q4_K super-block.
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// get_scale_min_k4 (quants.c:18-26) of all 8 sub-blocks of a super-block
__device__ __forceinline__ void q4k_scales8(const uint8_t *hdr, int (&sc)[8], int (&mn)[8]) {
    const uint32_t w0 = *reinterpret_cast<const uint32_t *>(hdr + 4);
    const uint32_t w1 = *reinterpret_cast<const uint32_t *>(hdr + 8);
    const uint32_t w2 = *reinterpret_cast<const uint32_t *>(hdr + 12);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t a = (w0 >> (8 * j)) & 0xffu, b = (w1 >> (8 * j)) & 0xffu, c = (w2 >> (8 * j)) & 0xffu;
        sc[j] = int(a & 63u);
        mn[j] = int(b & 63u);
        sc[j + 4] = int((c & 15u) | ((a >> 6) << 4));
        mn[j + 4] = int((c >> 4) | ((b >> 6) << 4));
    }
}

__device__ __forceinline__ void mma_s8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

// A 32-column tile of int8 activations for one 256-element super-block,
// staged in shared memory for the MMA kernels' B fragments.  Column c is
// activation row rows[c] (-1: zeros).  Rows are padded to 272 bytes so the
// fragment reads (8 columns x 4 words) fall in 32 different banks.
constexpr int BT_COLS = 32, BT_STRIDE = 272;
__device__ __forceinline__ void stage_btile(int8_t (*bs)[BT_STRIDE], const int *rows, const int8_t *x, size_t ld,
                                            int k0) {
    for (int i = threadIdx.x; i < BT_COLS * 16; i += blockDim.x) {
        const int c = i >> 4, q = i & 15;
        int4 v = make_int4(0, 0, 0, 0);
        if (rows[c] >= 0) v = *reinterpret_cast<const int4 *>(x + size_t(rows[c]) * ld + k0 + 16 * q);
        *reinterpret_cast<int4 *>(&bs[c][16 * q]) = v;
    }
}

// The same tile staged with cp.async (16-byte global -> shared copies that
// bypass the registers; a column without a row is zero-filled: source size
// 0), committed as one group: the caller waits with cp_async_wait<n>() and a
// barrier, so the next super-block's tile can be in flight while this one's
// MMAs run.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(smem)), "l"(gmem),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void stage_btile_async(int8_t (*bs)[BT_STRIDE], const int *rows, const int8_t *x,
                                                  size_t ld, int k0) {
    for (int i = threadIdx.x; i < BT_COLS * 16; i += blockDim.x) {
        const int c = i >> 4, q = i & 15, r = rows[c];
        cp_async16(&bs[c][16 * q], r >= 0 ? x + size_t(r) * ld + k0 + 16 * q : x, r >= 0);
    }
    cp_async_commit();
}

// Optional epilogue of a single-token GEMV over the gated delta net's input
// projection: rows r < n are also the causal conv's channels (conv1d_layer
// + SiLU, nn.c:717-741 / nn.c:2196), applied in the row's own thread with
// the same operation order as the conv kernel.
struct ConvEpi {
    const float *w = nullptr;     // [n][4] taps
    float *state = nullptr;       // [n][3] last three inputs
    float *out = nullptr;         // [n] silu(conv)
    int n = 0;
};

// Host launcher (gemv.cu): out[t][r] = <W[r], x_t> (+ resid[t][r]).  W is
// the packed matrix; T tokens are processed in passes of 4/2/1.
int matvec(int wtype, const void *W, int n_in, int n_out, int T, const int8_t *xq,
           const float *xd, const int16_t *xsum, float *out, cudaStream_t st,
           const float *resid = nullptr, const ConvEpi *conv = nullptr);
int num_sms();
// Bounded waits of the staged GEMV that ran out since the last call.
int gemv_wait_timeouts();

}  // namespace qma
