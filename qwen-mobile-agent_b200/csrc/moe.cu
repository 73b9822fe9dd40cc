// moe.cu -- the qwen35moe MoE FFN block on B200: router + top-8, fused
// gate/up + SwiGLU, down projection + weighted combine + residual.
//
// Reference: moe_ffn (nn.c:509-649), moe_expert_one_q8k (nn.c:412-439),
// moe_shared_q8k (nn.c:446-473), the residual in qma_eval (nn.c:2246-2252).
//
// Two kernels per call (T tokens, grid.y = token), both thread-block
// clusters of 16 CTAs exchanging data through distributed shared memory:
//   1. router : per token, 16 CTAs x 16 experts.  Every CTA forms
//               xn = rms_norm(x2) * post_norm, each warp computes two router
//               logits exactly in fp64 with a proven bound on the
//               reference's sequential fp32 sum and stores them in the
//               leader CTA; the leader selects the top 8 (falling back to
//               the reference's own summation order for any rank the bound
//               cannot settle) and renormalises the weights.  CTAs 0..7 also
//               quantize xn to Q8_K and form the shared-expert gate.
//   2. experts: per (slot, token), 9 slots (8 routed + shared) x 16 CTAs:
//               gate/up + SwiGLU rows, the hidden vector gathered across the
//               cluster, Q8_K, down rows; the last of the 9 slot CTAs of a
//               128-row chunk combines the slots in the reference's order
//               and adds the residual.
#include <math.h>

#include <type_traits>

#include "common.cuh"
#include "gemv.cuh"
#include "moe.cuh"
#include "quant.cuh"

namespace qma {

// ----------------------------------------------------------------- scratch --
static inline size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

size_t moe_scratch_bytes(int T) {
    size_t b = 0;
    b += al256(sizeof(unsigned) * T * MOE_DOWN_CHUNKS);   // dcount
    b += al256(sizeof(double) * T * MOE_NEXP) * 2;        // S, B
    b += al256(sizeof(int) * T);                          // fallback
    b += al256(sizeof(int) * T * MOE_TOPK);               // sel
    b += al256(sizeof(float) * T * MOE_TOPK);             // w
    b += al256(size_t(T) * MOE_EMBD);                     // xq
    b += al256(sizeof(float) * T * (MOE_EMBD / 256));     // xd
    b += al256(sizeof(int16_t) * T * (MOE_EMBD / 16));    // xs
    b += al256(sizeof(float) * T);                        // gs
    b += al256(sizeof(float) * T * MOE_NSLOT * MOE_EMBD); // part
    if (T >= MOE_GROUPED_MIN_T && T <= MOE_GROUPED_MAX_T) {
        const size_t q = size_t(T) * MOE_NSLOT;
        b += al256(sizeof(int) * 2 * (MOE_NEXP + 1));     // goff, active-expert list
        b += al256(sizeof(int) * T * MOE_TOPK);           // plist
        b += al256(sizeof(float) * q * 2 * MOE_FF);       // hg
        b += al256(q * MOE_FF);                           // hq
        b += al256(sizeof(float) * q * (MOE_FF / 256));   // hd
        b += al256(sizeof(int16_t) * q * (MOE_FF / 16));  // hs
    }
    return b;
}

MoeScratch moe_scratch_layout(void *base, int T) {
    uint8_t *p = static_cast<uint8_t *>(base);
    MoeScratch s;
    auto take = [&](size_t n) { uint8_t *q = p; p += al256(n); return q; };
    s.dcount = reinterpret_cast<unsigned *>(take(sizeof(unsigned) * T * MOE_DOWN_CHUNKS));
    s.S = reinterpret_cast<double *>(take(sizeof(double) * T * MOE_NEXP));
    s.B = reinterpret_cast<double *>(take(sizeof(double) * T * MOE_NEXP));
    s.fallback = reinterpret_cast<int *>(take(sizeof(int) * T));
    s.sel = reinterpret_cast<int *>(take(sizeof(int) * T * MOE_TOPK));
    s.w = reinterpret_cast<float *>(take(sizeof(float) * T * MOE_TOPK));
    s.xq = reinterpret_cast<int8_t *>(take(size_t(T) * MOE_EMBD));
    s.xd = reinterpret_cast<float *>(take(sizeof(float) * T * (MOE_EMBD / 256)));
    s.xs = reinterpret_cast<int16_t *>(take(sizeof(int16_t) * T * (MOE_EMBD / 16)));
    s.gs = reinterpret_cast<float *>(take(sizeof(float) * T));
    s.part = reinterpret_cast<float *>(take(sizeof(float) * T * MOE_NSLOT * MOE_EMBD));
    s.goff = nullptr; s.plist = nullptr; s.hg = nullptr; s.hq = nullptr; s.hd = nullptr; s.hs = nullptr;
    if (T >= MOE_GROUPED_MIN_T && T <= MOE_GROUPED_MAX_T) {
        const size_t q = size_t(T) * MOE_NSLOT;
        s.goff = reinterpret_cast<int *>(take(sizeof(int) * 2 * (MOE_NEXP + 1)));
        s.plist = reinterpret_cast<int *>(take(sizeof(int) * T * MOE_TOPK));
        s.hg = reinterpret_cast<float *>(take(sizeof(float) * q * 2 * MOE_FF));
        s.hq = reinterpret_cast<int8_t *>(take(q * MOE_FF));
        s.hd = reinterpret_cast<float *>(take(sizeof(float) * q * (MOE_FF / 256)));
        s.hs = reinterpret_cast<int16_t *>(take(sizeof(int16_t) * q * (MOE_FF / 16)));
    }
    return s;
}

// Bounded waits of the MoE kernels that ran out (read and reset by the host).
__device__ unsigned g_moe_timeouts;

// --------------------------------------------------------------- helpers --
__device__ __forceinline__ double warp_max_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// xn lives in shared memory in natural order (lanes read 16-byte words at
// consecutive addresses).
__device__ __forceinline__ int xn_idx(int i) { return i; }

// The reference ranks experts by probability p = expf(l - max) / sum and
// breaks ties to the lower expert id (repeated argmax with '>', nn.c:528-533).
// p is non-decreasing in the logit l, so ranking by l is the same except
// where p ties for different l.  Besides exact logit ties that happens when
// expf underflows: for l - max < -104.5, expf and hence p are exactly 0 and
// all such experts tie, ordered by id.  Between -104.5 and -81, p may be
// subnormal and coarsely rounded; those experts are ranked by logit.  So the
// rank key is (class, logit, id) with class 2 = normal p, 1 = subnormal p,
// 0 = p exactly zero (ranked by id alone).
constexpr double P_ZERO_BELOW = -104.5, P_NORMAL_ABOVE = -81.0;

__device__ __forceinline__ int p_class(double l, double mx) {
    const double d = l - mx;
    return d < P_ZERO_BELOW ? 0 : (d < P_NORMAL_ABOVE ? 1 : 2);
}

// Strict "a ranks above b" under the key (class, logit, id).
__device__ __forceinline__ bool ranks_above_c(int ca, double va, int ea, int cb, double vb, int eb) {
    if (ca != cb) return ca > cb;
    if (ca == 0) return ea < eb;
    return va > vb || (va == vb && ea < eb);
}
__device__ __forceinline__ bool ranks_above(double va, int ea, double vb, int eb) {
    return va > vb || (va == vb && ea < eb);
}

// -------------------------------------------------------------- router ----
// Top-8 selection over the (class, logit, id) key of 256 experts whose
// logits are S +- B, done by one warp; returns whether every comparison that
// decides the set and its order is settled by the intervals.
__device__ bool select_top8(const double *sS, const double *sB, const int *cls, int lane, int *top) {
    unsigned picked = 0;
    for (int k = 0; k < MOE_TOPK; k++) {
        int bc = -1, be = 0x7fffffff;
        double bv = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int e = lane + 32 * j;
            if (!((picked >> j) & 1u) && ranks_above_c(cls[e], sS[e], e, bc, bv, be)) {
                bc = cls[e]; bv = sS[e]; be = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const int oc = __shfl_xor_sync(0xffffffffu, bc, o);
            const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (ranks_above_c(oc, ov, oe, bc, bv, be)) { bc = oc; bv = ov; be = oe; }
        }
        top[k] = be;
        if ((be & 31) == lane) picked |= 1u << (be >> 5);
    }
    // upper bound of the best unselected expert in the 8th's class
    const int c8 = cls[top[MOE_TOPK - 1]];
    double ub = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int e = lane + 32 * j;
        if (!((picked >> j) & 1u) && cls[e] == c8) ub = fmax(ub, sS[e] + sB[e]);
    }
    ub = warp_max_d(ub);
    bool ok = true;
    for (int k = 0; k < MOE_TOPK; k++) {
        const int a = top[k];
        if (cls[a] == 0) continue;                      // ties at p = 0: ranked by id
        double hi;
        if (k + 1 < MOE_TOPK) {
            const int b = top[k + 1];
            if (cls[b] != cls[a]) continue;             // different class: settled
            hi = sS[b] + sB[b];
        } else {
            hi = ub;                                    // -inf if no rival in class
        }
        // separated intervals, with a margin that keeps the probabilities'
        // order strict after expf and division rounding
        if (!(sS[a] - sB[a] - hi > 1e-6 * (1.0 + fabs(sS[a])))) ok = false;
    }
    return ok;
}

// Exact logit S (fp64 sum of the fp32 products) and a bound B on the
// reference's sequential fp32 sum, for one router row in shared memory (a
// warp per row; lane l takes elements 128 k + 4 l .. +3 of chunk k, so the
// 16-byte reads are consecutive).  The reference sums s += g_i * x_i in fp32
// (nn.c:519-521).  With a_i = fl(g_i * x_i) (the same products) and S_i the
// exact prefix sums, recursive summation satisfies |s_fp32 - S_n| <= u'
// sum_i |S_i| with u' = 2^-24 (1 + n u) for n = 2048.  S_n is summed in fp64
// (error ~1e-13 relative).  sum_i |S_i| is bounded group by group: a lane's
// four elements start at prefix Q (a warp scan per 128-element chunk) and
//   sum_{i<4} |Q + a_0 + .. + a_i| <= 4|Q| + 4|a_0| + 3|a_1| + 2|a_2| + |a_3|.
// The fp32 prefixes come from sums at most ~30 additions deep (error
// <= 2e-6 sum|a|, under 0.1% of the bound, which is >= 4 sum|a|); the 1.01
// factor covers that and the (1 + n u) term.
__device__ __forceinline__ void router_logit(const float *row, const float *xn, int lane, double &S,
                                             double &B) {
    double t4[4] = {0.0, 0.0, 0.0, 0.0};
    float P = 0.0f, el = 0.0f;        // P: prefix of the previous chunks
#pragma unroll
    for (int h = 0; h < 2; h++) {     // chunks 8 h .. 8 h + 7
        float c[8], wa[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int o = 128 * (8 * h + k) + 4 * lane;
            const float4 g = *reinterpret_cast<const float4 *>(row + o);
            const float4 x = *reinterpret_cast<const float4 *>(xn + o);
            const float a0 = __fmul_rn(g.x, x.x), a1 = __fmul_rn(g.y, x.y);
            const float a2 = __fmul_rn(g.z, x.z), a3 = __fmul_rn(g.w, x.w);
            t4[0] += double(a0);
            t4[1] += double(a1);
            t4[2] += double(a2);
            t4[3] += double(a3);
            c[k] = (a0 + a1) + (a2 + a3);
            wa[k] = (4.0f * fabsf(a0) + 3.0f * fabsf(a1)) + (2.0f * fabsf(a2) + fabsf(a3));
        }
        // inclusive scan of the lane sums within each chunk (8 independent scans)
        float incl[8];
#pragma unroll
        for (int k = 0; k < 8; k++) incl[k] = c[k];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1)
#pragma unroll
            for (int k = 0; k < 8; k++) {
                const float v = __shfl_up_sync(0xffffffffu, incl[k], o);
                if (lane >= o) incl[k] += v;
            }
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const float q = P + (incl[k] - c[k]);       // prefix before this lane's group
            el += 4.0f * fabsf(q) + wa[k];
            P += __shfl_sync(0xffffffffu, incl[k], 31);
        }
    }
    S = warp_sum_d((t4[0] + t4[1]) + (t4[2] + t4[3]));
    const float E = warp_sum(el);
    B = double(E) * 0x1.0p-24 * 1.01 + 1e-30;
}

// Leader-side fast selection by one warp (lane l holds experts l + 32 j):
// top9[r] = the expert of rank r < 9 by S rounded to fp32 (nine rounds of a
// warp max over sortable 32-bit keys; equal keys go to the lowest lane,
// then the lowest j).  Returns whether that ranking settles the reference's
// selection: the 8th expert's probability is a normal float (then no lower
// class can compete) and the intervals S +- B of consecutive selected
// experts, and of the 8th against every unselected one, are separated with
// a margin that keeps the probabilities' order strict after expf and
// division rounding.  Two logits that fp32 rounding could tie or misorder
// are within one fp32 ulp of each other, far inside that margin, so a
// ranking they could spoil is never accepted; the exact path runs instead.
__device__ __forceinline__ uint32_t sort_key(double S) {
    const uint32_t u = __float_as_uint(float(S));
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);   // > 0 for every non-NaN
}
__device__ bool select_fast(const double *sS, const double *sB, int lane, int *top9) {
    uint32_t key[8];
#pragma unroll
    for (int j = 0; j < 8; j++) key[j] = sort_key(sS[lane + 32 * j]);
    unsigned taken = 0;                                  // bit j: taken in rounds 0..7
    int mine = -1;                                       // lane k's expert of rank k
    int e8 = 0;
#pragma unroll 1
    for (int r = 0; r <= MOE_TOPK; r++) {
        uint32_t m = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) m = max(m, key[j]);
        const uint32_t M = __reduce_max_sync(0xffffffffu, m);
        const int owner = __ffs(__ballot_sync(0xffffffffu, m == M)) - 1;
        int e = 0;
        if (lane == owner) {
            int jj = 0;
#pragma unroll
            for (int j = 7; j >= 0; j--) if (key[j] == M) jj = j;
#pragma unroll
            for (int j = 0; j < 8; j++)
                if (j == jj) {
                    key[j] = 0;
                    if (r < MOE_TOPK) taken |= 1u << j;
                }
            e = lane + 32 * jj;
        }
        e = __shfl_sync(0xffffffffu, e, owner);
        if (lane == r) mine = e;
        if (r == MOE_TOPK) e8 = e;
    }
    if (lane <= MOE_TOPK) top9[lane] = lane == MOE_TOPK ? e8 : mine;
    // largest S + B among the unselected (everything but ranks 0..7)
    double ub = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; j++)
        if (!((taken >> j) & 1u)) ub = fmax(ub, sS[lane + 32 * j] + sB[lane + 32 * j]);
    ub = warp_max_d(ub);
    // lane k < 8 checks the gap below rank k
    const int nxt = __shfl_down_sync(0xffffffffu, mine, 1);
    const int top0 = __shfl_sync(0xffffffffu, mine, 0);
    bool ok = true;
    if (lane < MOE_TOPK) {
        const double hi = lane + 1 < MOE_TOPK ? sS[nxt] + sB[nxt] : ub;
        ok = sS[mine] - sB[mine] - hi > 1e-6 * (1.0 + fabs(sS[mine]));
        if (lane == MOE_TOPK - 1) ok = ok && p_class(sS[mine], sS[top0]) == 2;
    }
    return __all_sync(0xffffffffu, ok);
}

// Router: one cluster of RCL CTAs per token (grid (RCL, T)), 16 warps per
// CTA, one expert per warp.  Every CTA forms xn = rms_norm(x2) * post_norm
// (rms_norm_m, nn.c:348-357) in shared memory; each warp computes its exact
// logit and bound and stores them into the leader CTA's shared memory; CTAs
// 0..7 also quantize 256-block `rank` of xn to Q8_K (shared by every expert)
// and send the leader their part of the shared-expert gate input
// sum_i g_i * xq_i * xd (nn.c:453).  After the cluster barrier the leader
// selects the top 8 (falling back to the reference's own summation order for
// any rank the bounds cannot settle) and writes the renormalised weights
// (nn.c:524-547) and the shared-expert gate sigmoid.
constexpr int RCL = 16;                       // CTAs per router cluster
constexpr int RTHREADS = 512;                 // one warp per expert row
constexpr int RROWS = MOE_NEXP / RCL;         // router rows per CTA
constexpr uint32_t ROW_BYTES = MOE_EMBD * 4;
constexpr uint32_t ROUTER_SMEM = uint32_t(RROWS) * ROW_BYTES;   // 16 fp32 rows
static_assert(RROWS == RTHREADS / 32, "one router row per warp");
constexpr int XCL = 16;                       // CTAs per expert cluster (two CTAs per SM)
constexpr int XTHREADS = 512;                 // threads per expert CTA
constexpr int XGU = MOE_FF / XCL;             // gate/up rows per expert CTA
constexpr int XDN = MOE_EMBD / XCL;           // down rows per expert CTA
static_assert(XDN == MOE_DOWN_CHUNK && XCL == MOE_DOWN_CHUNKS, "combine chunks = expert CTAs");

// The reference's own summation order for one logit, s = fl(s + fl(g_i x_i))
// for i = 0..2047 (nn.c:519-521), from a row and xn in shared memory.
__device__ __forceinline__ float router_logit_seq(const float *row, const float *xn) {
    float acc = 0.0f;
#pragma unroll 4
    for (int i = 0; i < MOE_EMBD; i += 4) {
        const float4 g = *reinterpret_cast<const float4 *>(row + i);
        const float4 x = *reinterpret_cast<const float4 *>(xn + i);
        acc = __fadd_rn(acc, __fmul_rn(g.x, x.x));
        acc = __fadd_rn(acc, __fmul_rn(g.y, x.y));
        acc = __fadd_rn(acc, __fmul_rn(g.z, x.z));
        acc = __fadd_rn(acc, __fmul_rn(g.w, x.w));
    }
    return acc;
}

// With a router bias the logit is fl(s + b_e): its interval S + b +- B'
// with B' = B + 2^-24 (|S + b| + B) (1 + 2^-20) covers the extra rounding
// (and the fp64 sum S + b), and the exact path adds b_e to the recomputed
// fp32 sum in fp32, as the biased reference does.
__device__ __forceinline__ void bias_interval(double &S, double &B, float b) {
    const double Sb = S + double(b);
    B = B + 0x1.0p-24 * (fabs(Sb) + B) * (1.0 + 0x1.0p-20) + 1e-30;
    S = Sb;
}

__global__ void __launch_bounds__(RTHREADS, 1) moe_router_kernel(const float *__restrict__ x2,
                                                               const float *__restrict__ post_norm,
                                                               const float *__restrict__ Wr,
                                                               const float *__restrict__ gis,
                                                               MoeScratch s, int *sel_out,
                                                               float *w_out, const float *__restrict__ bias) {
    QMA_TRACE_SCOPE(TK_ROUTER);
    extern __shared__ __align__(128) float rrows[];        // this CTA's 16 router rows
    const unsigned rank = cluster_rank();
    // every CTA of the cluster must have started before its shared memory is
    // written remotely: arrive now, wait just before the first remote store
    cluster_arrive();
    const int t = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = RTHREADS / 32;
    __shared__ __align__(8) uint64_t rbar;
    __shared__ __align__(16) float xn[MOE_EMBD];
    __shared__ double dred[NW];
    __shared__ double sS[MOE_NEXP], sB[MOE_NEXP];
    __shared__ float gpart[MOE_EMBD / 256];
    __shared__ int need_exact, ncand;
    __shared__ int cls[MOE_NEXP];
    __shared__ int top9[MOE_TOPK + 1];
    __shared__ int cand[MOE_NEXP];

    // this CTA's router rows: independent of the upstream kernel, copied
    // into shared memory by the TMA engine before waiting on it
    const int e0 = int(rank) * RROWS + warp;
    if (warp == 0) {
        if (lane == 0) {
            mbar_init(&rbar, 1);
            mbar_fence_init();
            mbar_expect_tx(&rbar, ROUTER_SMEM);
        }
        __syncwarp();
        bulk_g2s_warp(rrows, Wr + size_t(rank) * RROWS * MOE_EMBD, ROUTER_SMEM, &rbar, lane);
    }
    // this CTA's slice of the shared-expert gate row (CTAs 0..7, warp 0)
    float gisv[8] = {};
    if (rank < MOE_EMBD / 256 && warp == 0) {
        const float4 g0 = __ldg(reinterpret_cast<const float4 *>(gis + rank * 256 + lane * 8));
        const float4 g1 = __ldg(reinterpret_cast<const float4 *>(gis + rank * 256 + lane * 8 + 4));
        gisv[0] = g0.x; gisv[1] = g0.y; gisv[2] = g0.z; gisv[3] = g0.w;
        gisv[4] = g1.x; gisv[5] = g1.y; gisv[6] = g1.z; gisv[7] = g1.w;
    }
    // the norm weights and this warp's router bias: constants, read before
    // the wait too
    constexpr int XPT = MOE_EMBD / RTHREADS;
    float pn[XPT];
#pragma unroll
    for (int k = 0; k < XPT; k++) pn[k] = __ldg(post_norm + tid + RTHREADS * k);
    const float bias_e = bias ? __ldg(bias + e0) : 0.0f;
    QMA_TRACE_MARK(TK_ROUTER, 1);
    pdl_trigger();
    pdl_wait();
    QMA_TRACE_MARK(TK_ROUTER, 2);
    // ---- xn = rms_norm(x2) * post_norm ------------------------------------
    const float *x = x2 + size_t(t) * MOE_EMBD;
    float xv[XPT];
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < XPT; k++) {
        xv[k] = x[tid + RTHREADS * k];
        ss += double(xv[k]) * double(xv[k]);
    }
    ss = warp_sum_d(ss);
    if (lane == 0) dred[warp] = ss;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < NW; w++) tot += dred[w];
    const float r = 1.0f / sqrtf(float(tot / MOE_EMBD) + 1e-6f);
#pragma unroll
    for (int k = 0; k < XPT; k++) {
        const int i = tid + RTHREADS * k;
        xn[xn_idx(i)] = __fmul_rn(__fmul_rn(xv[k], r), pn[k]);
    }
    __syncthreads();
    QMA_TRACE_MARK(TK_ROUTER, 3);
    // ---- one exact logit per warp, sent to the leader -----------------------
    bool rows_ok = mbar_wait(&rbar, 0);
    if (!rows_ok) {
        if (lane == 0) atomicAdd(&g_moe_timeouts, 1u);
        mbar_wait(&rbar, 0);
    }
    cluster_wait();
    {
        double S0, B0;
        router_logit(rrows + size_t(warp) * MOE_EMBD, xn, lane, S0, B0);
        if (bias) bias_interval(S0, B0, bias_e);
        if (lane == 0) {
            st_cluster_f64(cluster_map(&sS[e0], 0), S0);
            st_cluster_f64(cluster_map(&sB[e0], 0), B0);
        }
    }
    // ---- Q8_K block `rank` of xn and its part of the shared-expert gate ----
    if (rank < MOE_EMBD / 256 && warp == 0) {
        const int blk = int(rank), i0 = blk * 256 + lane * 8;
        const float4 a0 = *reinterpret_cast<const float4 *>(xn + xn_idx(i0));
        const float4 a1 = *reinterpret_cast<const float4 *>(xn + xn_idx(i0 + 4));
        const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        int q[8];
        float sc;
        q8k_block_warp_q(v, lane, s.xq + size_t(t) * MOE_EMBD + blk * 256,
                         s.xd + size_t(t) * (MOE_EMBD / 256) + blk,
                         s.xs + size_t(t) * (MOE_EMBD / 16) + blk * 16, q, sc);
        float gp = 0.0f;
#pragma unroll
        for (int c = 0; c < 8; c++) gp += __fmul_rn(__fmul_rn(gisv[c], float(q[c])), sc);
        gp = warp_sum(gp);
        if (lane == 0) st_cluster_f32(cluster_map(&gpart[blk], 0), gp);
    }
    QMA_TRACE_MARK(TK_ROUTER, 4);
    cluster_sync();
    QMA_TRACE_MARK(TK_ROUTER, 5);
    if (rank != 0) return;

    // ---- leader: top 8 ------------------------------------------------------
    // Expert e ranks by (S descending, id ascending), counting the experts
    // above it.  That is the reference's order (probability, then lowest id)
    // whenever the 8th expert's probability is a normal float (class 2: the
    // classes below only ever hold lower logits) and every decision is
    // settled by the bounds; otherwise the exact path below runs.
    if (warp == 0) {
        const bool ok = select_fast(sS, sB, lane, top9);
        if (lane == 0) {
            need_exact = !ok;
            ncand = 0;
        }
    }
    __syncthreads();
    if (need_exact) {
        // Every expert whose rank the bounds leave open gets its logit
        // recomputed in the reference's exact order; its interval then
        // collapses to the exact value.  The candidates' rows are copied, 16
        // at a time, into the row buffer (its own rows are consumed).
        const double mx = sS[top9[0]];
        // an expert whose upper bound is below every selected expert's lower
        // bound (with margin) is out of the top 8 whatever the exact values
        const int e8 = top9[MOE_TOPK - 1];
        double thresh = INFINITY;
#pragma unroll
        for (int k = 0; k < MOE_TOPK; k++) thresh = fmin(thresh, sS[top9[k]] - sB[top9[k]]);
        if (tid < MOE_NEXP) {
            cls[tid] = p_class(sS[tid], mx);
            if (cls[tid] > 0 && sS[tid] + sB[tid] >= thresh - 1e-6 * (1.0 + fabs(sS[e8])))
                cand[atomicAdd(&ncand, 1)] = tid;
        }
        __syncthreads();
        for (int base = 0, phase = 1; base < ncand; base += RROWS, phase ^= 1) {
            const int nb = min(RROWS, ncand - base);
            if (warp == 0) {
                fence_proxy_async_smem();              // generic reads of the buffer are done
                if (lane == 0) mbar_expect_tx(&rbar, uint32_t(nb) * ROW_BYTES);
                __syncwarp();
                for (int c = 0; c < nb; c++)
                    bulk_g2s_warp(rrows + size_t(c) * MOE_EMBD, Wr + size_t(cand[base + c]) * MOE_EMBD,
                                  ROW_BYTES, &rbar, lane);
            }
            if (!mbar_wait(&rbar, uint32_t(phase))) {
                if (tid == 0) atomicAdd(&g_moe_timeouts, 1u);
                mbar_wait(&rbar, uint32_t(phase));
            }
            if (tid < nb) {
                const int e = cand[base + tid];
                const float l = router_logit_seq(rrows + size_t(tid) * MOE_EMBD, xn);
                sS[e] = double(bias ? __fadd_rn(l, bias[e]) : l);
                sB[e] = 0.0;
            }
            __syncthreads();
        }
        if (warp == 0) {
            double m2 = -INFINITY;
            for (int j = 0; j < 8; j++) m2 = fmax(m2, sS[lane + 32 * j]);
            m2 = warp_max_d(m2);
            for (int j = 0; j < 8; j++) cls[lane + 32 * j] = p_class(sS[lane + 32 * j], m2);
            __syncwarp();
            select_top8(sS, sB, cls, lane, top9);   // settled by exact values
        }
        __syncthreads();
    }
    QMA_TRACE_MARK(TK_ROUTER, 6);
    if (warp == 0) {
        // renormalised softmax weights of the selected experts (nn.c:524-547)
        const float l0 = float(sS[top9[0]]);
        const float ev = lane < MOE_TOPK ? expf(float(sS[top9[lane]]) - l0) : 0.0f;
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < MOE_TOPK; k++) sum += __shfl_sync(0xffffffffu, ev, k);
        if (lane < MOE_TOPK) {
            const float wk = ev / sum;
            const int e = top9[lane];
            s.sel[t * MOE_TOPK + lane] = e;
            s.w[t * MOE_TOPK + lane] = wk;
            if (sel_out) sel_out[t * MOE_TOPK + lane] = e;
            if (w_out) w_out[t * MOE_TOPK + lane] = wk;
        } else if (lane == MOE_TOPK) {
            float g = 0.0f;
            for (int b = 0; b < MOE_EMBD / 256; b++) g += gpart[b];
            s.gs[t] = 1.0f / (1.0f + expf(-g));
            s.fallback[t] = need_exact;
        }
    }
}

// Router of several tokens (prefill chunks, expert-parallel steps): the
// single-token kernel's arithmetic, with each cluster taking RTPC tokens so
// that its 2 MB of router rows are staged into shared memory once per RTPC
// tokens instead of once per token.  Every warp computes its row's logits
// for the cluster's tokens in turn; the leader's warps 0..RTPC-1 select the
// tokens' top 8 side by side, then any token the bounds leave open takes
// the exact path in turn (the whole CTA, the candidate rows staged through
// the consumed row buffer as above).
constexpr int RTPC = 4;                       // tokens per router cluster
struct RouterMultiSmem {
    float rows[RROWS][MOE_EMBD];              // this CTA's router rows (128 KB)
    float xn[RTPC][MOE_EMBD];
    double S[RTPC][MOE_NEXP], B[RTPC][MOE_NEXP];
};
constexpr size_t ROUTER_MULTI_SMEM = sizeof(RouterMultiSmem);

__global__ void __launch_bounds__(RTHREADS, 1) moe_router_multi_kernel(const float *__restrict__ x2, int T,
                                                                     const float *__restrict__ post_norm,
                                                                     const float *__restrict__ Wr,
                                                                     const float *__restrict__ gis,
                                                                     MoeScratch s, int *sel_out, float *w_out,
                                                                     const float *__restrict__ bias) {
    QMA_TRACE_SCOPE(TK_ROUTER);
    extern __shared__ __align__(128) uint8_t rmsm_raw[];
    RouterMultiSmem &R = *reinterpret_cast<RouterMultiSmem *>(rmsm_raw);
    const unsigned rank = cluster_rank();
    cluster_arrive();
    const int t0 = blockIdx.y * RTPC, nt = min(RTPC, T - t0);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = RTHREADS / 32;
    __shared__ __align__(8) uint64_t rbar;
    __shared__ double dred[RTPC][NW];
    __shared__ float gpart[RTPC][MOE_EMBD / 256];
    __shared__ int need_exact[RTPC], ncand;
    __shared__ int cls[MOE_NEXP];
    __shared__ int top9[RTPC][MOE_TOPK + 1];
    __shared__ int cand[MOE_NEXP];
    const int e0 = int(rank) * RROWS + warp;
    if (warp == 0) {
        if (lane == 0) {
            mbar_init(&rbar, 1);
            mbar_fence_init();
            mbar_expect_tx(&rbar, ROUTER_SMEM);
        }
        __syncwarp();
        bulk_g2s_warp(&R.rows[0][0], Wr + size_t(rank) * RROWS * MOE_EMBD, ROUTER_SMEM, &rbar, lane);
    }
    float gisv[8] = {};
    if (rank < MOE_EMBD / 256 && warp == 0) {
        const float4 g0 = __ldg(reinterpret_cast<const float4 *>(gis + rank * 256 + lane * 8));
        const float4 g1 = __ldg(reinterpret_cast<const float4 *>(gis + rank * 256 + lane * 8 + 4));
        gisv[0] = g0.x; gisv[1] = g0.y; gisv[2] = g0.z; gisv[3] = g0.w;
        gisv[4] = g1.x; gisv[5] = g1.y; gisv[6] = g1.z; gisv[7] = g1.w;
    }
    // the norm weights and this warp's router bias: constants, read before
    // the wait too
    constexpr int XPT = MOE_EMBD / RTHREADS;
    float pn[XPT];
#pragma unroll
    for (int k = 0; k < XPT; k++) pn[k] = __ldg(post_norm + tid + RTHREADS * k);
    const float bias_e = bias ? __ldg(bias + e0) : 0.0f;
    pdl_trigger();
    pdl_wait();
    // ---- xn of each token (rms_norm_m, nn.c:348-357) ---------------------------
    float xv[RTPC][XPT];
#pragma unroll
    for (int u = 0; u < RTPC; u++) {
        double ss = 0.0;
#pragma unroll
        for (int k = 0; k < XPT; k++) {
            xv[u][k] = u < nt ? x2[size_t(t0 + u) * MOE_EMBD + tid + RTHREADS * k] : 0.0f;
            ss += double(xv[u][k]) * double(xv[u][k]);
        }
        ss = warp_sum_d(ss);
        if (lane == 0) dred[u][warp] = ss;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < RTPC; u++) {
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < NW; w++) tot += dred[u][w];
        const float r = 1.0f / sqrtf(float(tot / MOE_EMBD) + 1e-6f);
#pragma unroll
        for (int k = 0; k < XPT; k++) {
            const int i = tid + RTHREADS * k;
            R.xn[u][i] = __fmul_rn(__fmul_rn(xv[u][k], r), pn[k]);
        }
    }
    __syncthreads();
    // ---- the tokens' exact logits of this warp's row ------------------------------
    if (!mbar_wait(&rbar, 0)) {
        if (lane == 0) atomicAdd(&g_moe_timeouts, 1u);
        mbar_wait(&rbar, 0);
    }
    cluster_wait();
    for (int u = 0; u < nt; u++) {
        double S0, B0;
        router_logit(&R.rows[warp][0], R.xn[u], lane, S0, B0);
        if (bias) bias_interval(S0, B0, bias_e);
        if (lane == 0) {
            st_cluster_f64(cluster_map(&R.S[u][e0], 0), S0);
            st_cluster_f64(cluster_map(&R.B[u][e0], 0), B0);
        }
    }
    // ---- Q8_K block `rank` of each token's xn, its shared-expert gate part ---
    if (rank < MOE_EMBD / 256 && warp == 0) {
        const int blk = int(rank), i0 = blk * 256 + lane * 8;
        for (int u = 0; u < nt; u++) {
            const int t = t0 + u;
            const float4 a0 = *reinterpret_cast<const float4 *>(&R.xn[u][i0]);
            const float4 a1 = *reinterpret_cast<const float4 *>(&R.xn[u][i0 + 4]);
            const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            int q[8];
            float sc;
            q8k_block_warp_q(v, lane, s.xq + size_t(t) * MOE_EMBD + blk * 256,
                             s.xd + size_t(t) * (MOE_EMBD / 256) + blk,
                             s.xs + size_t(t) * (MOE_EMBD / 16) + blk * 16, q, sc);
            float gp = 0.0f;
#pragma unroll
            for (int c = 0; c < 8; c++) gp += __fmul_rn(__fmul_rn(gisv[c], float(q[c])), sc);
            gp = warp_sum(gp);
            if (lane == 0) st_cluster_f32(cluster_map(&gpart[u][blk], 0), gp);
        }
    }
    cluster_sync();
    if (rank != 0) return;

    // ---- leader: each token's top 8 -----------------------------------------------
    if (warp < nt) {
        const bool ok = select_fast(R.S[warp], R.B[warp], lane, top9[warp]);
        if (lane == 0) need_exact[warp] = !ok;
    }
    __syncthreads();
    uint32_t phase = 1;
    for (int u = 0; u < nt; u++) {
        if (!need_exact[u]) continue;                  // CTA-uniform
        double *sS = R.S[u], *sB = R.B[u];
        const int *tp = top9[u];
        if (tid == 0) ncand = 0;
        __syncthreads();
        const double mx = sS[tp[0]];
        const int e8 = tp[MOE_TOPK - 1];
        double thresh = INFINITY;
#pragma unroll
        for (int k = 0; k < MOE_TOPK; k++) thresh = fmin(thresh, sS[tp[k]] - sB[tp[k]]);
        if (tid < MOE_NEXP) {
            cls[tid] = p_class(sS[tid], mx);
            if (cls[tid] > 0 && sS[tid] + sB[tid] >= thresh - 1e-6 * (1.0 + fabs(sS[e8])))
                cand[atomicAdd(&ncand, 1)] = tid;
        }
        __syncthreads();
        for (int base = 0; base < ncand; base += RROWS, phase ^= 1) {
            const int nb = min(RROWS, ncand - base);
            if (warp == 0) {
                fence_proxy_async_smem();
                if (lane == 0) mbar_expect_tx(&rbar, uint32_t(nb) * ROW_BYTES);
                __syncwarp();
                for (int c = 0; c < nb; c++)
                    bulk_g2s_warp(&R.rows[c][0], Wr + size_t(cand[base + c]) * MOE_EMBD, ROW_BYTES, &rbar, lane);
            }
            if (!mbar_wait(&rbar, phase)) {
                if (tid == 0) atomicAdd(&g_moe_timeouts, 1u);
                mbar_wait(&rbar, phase);
            }
            if (tid < nb) {
                const int e = cand[base + tid];
                const float l = router_logit_seq(&R.rows[tid][0], R.xn[u]);
                sS[e] = double(bias ? __fadd_rn(l, bias[e]) : l);
                sB[e] = 0.0;
            }
            __syncthreads();
        }
        if (warp == 0) {
            double m2 = -INFINITY;
            for (int j = 0; j < 8; j++) m2 = fmax(m2, sS[lane + 32 * j]);
            m2 = warp_max_d(m2);
            for (int j = 0; j < 8; j++) cls[lane + 32 * j] = p_class(sS[lane + 32 * j], m2);
            __syncwarp();
            select_top8(sS, sB, cls, lane, top9[u]);
        }
        __syncthreads();
    }
    if (warp < nt) {
        const int u = warp, t = t0 + u;
        const double *sS = R.S[u];
        const float l0 = float(sS[top9[u][0]]);
        const float ev = lane < MOE_TOPK ? expf(float(sS[top9[u][lane]]) - l0) : 0.0f;
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < MOE_TOPK; k++) sum += __shfl_sync(0xffffffffu, ev, k);
        if (lane < MOE_TOPK) {
            const float wk = ev / sum;
            const int e = top9[u][lane];
            s.sel[t * MOE_TOPK + lane] = e;
            s.w[t * MOE_TOPK + lane] = wk;
            if (sel_out) sel_out[t * MOE_TOPK + lane] = e;
            if (w_out) w_out[t * MOE_TOPK + lane] = wk;
        } else if (lane == MOE_TOPK) {
            float g = 0.0f;
            for (int b = 0; b < MOE_EMBD / 256; b++) g += gpart[u][b];
            s.gs[t] = 1.0f / (1.0f + expf(-g));
            s.fallback[t] = need_exact[u];
        }
    }
}

// ---------------------------------------------------------------- experts --
__device__ __forceinline__ Q6Planes shift_rows(Q6Planes P, int r0, int n) {
    P.ql += size_t(r0) * (n / 2);
    P.qh += size_t(r0) * (n / 4);
    P.sc += size_t(r0) * (n / 16);
    P.d += size_t(r0) * (n / 256);
    return P;
}
__device__ __forceinline__ const uint8_t *shift_rows(const uint8_t *P, int r0, int n) {
    return P + size_t(r0) * (n / 256) * Q4K_BYTES;
}
__device__ __forceinline__ void prefetch_rows(const Q6Planes &P, int rows, int n) {
    prefetch_l2(P.ql, uint32_t(rows) * (n / 2));
    prefetch_l2(P.qh, uint32_t(rows) * (n / 4));
    prefetch_l2(P.sc, uint32_t(rows) * (n / 16));
    prefetch_l2(P.d, uint32_t(rows) * (n / 256) * 2);
}
__device__ __forceinline__ void prefetch_rows(const uint8_t *P, int rows, int n) {
    prefetch_l2(P, uint32_t(rows) * (n / 256) * Q4K_BYTES);
}

template <class F> struct DownPtr;
template <> struct DownPtr<FmtQ6K> {
    __device__ static Q6Planes at(const uint8_t *base) {
        Q6Planes P;
        P.ql = base;
        P.qh = base + q6_plane_ql(MOE_EMBD, MOE_FF);
        P.sc = reinterpret_cast<const int8_t *>(P.qh + q6_plane_qh(MOE_EMBD, MOE_FF));
        P.d = reinterpret_cast<const __half *>(reinterpret_cast<const uint8_t *>(P.sc) +
                                               q6_plane_sc(MOE_EMBD, MOE_FF));
        return P;
    }
};
template <> struct DownPtr<FmtQ4K> {
    __device__ static const uint8_t *at(const uint8_t *base) { return base; }
};

// One cluster of XCL CTAs per (slot, token): grid (9 x XCL, T); slots 0..7
// are the routed experts in selection order, slot 8 the shared expert
// (moe_expert_one_q8k nn.c:412-439, moe_shared_q8k nn.c:446-473).  144 CTAs
// of 512 threads, sized (registers <= 64, 74 KB of shared memory) so that
// two fit on an SM: the 9 clusters of 16 are co-resident beside the router's
// cluster and the next kernels' early CTAs.  CTA `rank` owns gate/up rows
// rank*XGU.. and down rows rank*XDN..:
//   1. its 32 gate and 32 up rows (74 KB) are copied into shared memory by
//      the TMA engine as soon as the expert is known (the shared expert's
//      before the router has finished), its down rows prefetched into L2;
//   2. one warp per 2 row pairs computes silu(gate) * up;
//   3. every CTA pushes its 32 hidden values into all 16 CTAs' shared
//      memory (one cluster barrier) while the down rows are copied into the
//      freed buffer;
//   4. every CTA quantizes the hidden vector to Q8_K and computes its 128
//      down rows; the last of the 9 slot CTAs of a row chunk combines the
//      slots in the reference's order and adds the residual (nn.c:615-629,
//      nn.c:2246-2252).
// Every wait on a copy is bounded; a copy that never lands is counted in
// g_moe_timeouts (the host fails the call) and the CTA still takes part in
// the cluster barriers so that no peer waits forever.
// The down rows' format, read from shared memory.  For Q6_K the hidden
// vector's Q8_K bytes are read from a unit-interleaved copy (16-byte chunk k
// of 128-byte unit u at chunk 4k + u): the four lanes of a row, which take
// units 0..3, then hit four different bank groups instead of one.
template <class F> struct DownRows : SmemRows<F> {};
template <> struct DownRows<FmtQ6K> : SmemRows<FmtQ6K> {
    __device__ static void load_act(Act &a, const int8_t *xq, const float *xd, const int16_t *, int u) {
        const int4 *p = reinterpret_cast<const int4 *>(xq);
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int4 v = p[4 * k + u];
            a.x[4 * k] = v.x; a.x[4 * k + 1] = v.y; a.x[4 * k + 2] = v.z; a.x[4 * k + 3] = v.w;
        }
        a.xd = xd[u >> 1];
    }
};
static_assert(MOE_FF / FmtQ6K::UNIT == 4, "interleave stride = units per down row");

template <class F> struct DownBytes;
template <> struct DownBytes<FmtQ6K> {
    static constexpr uint32_t QL = XDN * (MOE_FF / 2), QH = XDN * (MOE_FF / 4), SC = XDN * (MOE_FF / 16),
                              D = XDN * (MOE_FF / 256) * 2, ALL = QL + QH + SC + D;
    __device__ static void issue(uint8_t *dst, const uint8_t *expert, int d0, uint64_t *bar, int lane) {
        const Q6Planes P = shift_rows(DownPtr<FmtQ6K>::at(expert), d0, MOE_FF);
        if (lane == 0) mbar_expect_tx(bar, ALL);
        __syncwarp();
        bulk_g2s_warp(dst, P.ql, QL, bar, lane);
        bulk_g2s_warp(dst + QL, P.qh, QH, bar, lane);
        bulk_g2s_warp(dst + QL + QH, P.sc, SC, bar, lane);
        bulk_g2s_warp(dst + QL + QH + SC, P.d, D, bar, lane);
    }
    __device__ static Q6Planes at(const uint8_t *dst) {
        Q6Planes P;
        P.ql = dst;
        P.qh = dst + QL;
        P.sc = reinterpret_cast<const int8_t *>(dst + QL + QH);
        P.d = reinterpret_cast<const __half *>(dst + QL + QH + SC);
        return P;
    }
};
template <> struct DownBytes<FmtQ4K> {
    static constexpr uint32_t ALL = XDN * (MOE_FF / 256) * Q4K_BYTES;
    __device__ static void issue(uint8_t *dst, const uint8_t *expert, int d0, uint64_t *bar, int lane) {
        if (lane == 0) mbar_expect_tx(bar, ALL);
        __syncwarp();
        bulk_g2s_warp(dst, shift_rows(expert, d0, MOE_FF), ALL, bar, lane);
    }
    __device__ static const uint8_t *at(const uint8_t *dst) { return dst; }
};
constexpr uint32_t XROW = uint32_t(MOE_EMBD / 256) * Q4K_BYTES;     // one gate/up row
constexpr uint32_t XGU_BYTES = XGU * XROW;                          // 32 rows
constexpr size_t EXPERT_SMEM = 2 * size_t(XGU_BYTES);
static_assert(DownBytes<FmtQ6K>::ALL <= EXPERT_SMEM && DownBytes<FmtQ4K>::ALL <= EXPERT_SMEM,
              "down rows reuse the gate/up buffer");

template <class F>
__global__ void __launch_bounds__(XTHREADS, 2) moe_expert_kernel(const uint8_t *__restrict__ gate_exps,
                                                         const uint8_t *__restrict__ up_exps,
                                                         const uint8_t *__restrict__ gate_sh,
                                                         const uint8_t *__restrict__ up_sh,
                                                         const uint8_t *__restrict__ down_exps,
                                                         size_t down_bytes,
                                                         const uint8_t *__restrict__ down_sh,
                                                         const float *x2, float *x_out,
                                                         MoeScratch s, int combine, Prefetch pf) {
    QMA_TRACE_SCOPE(TK_EXPERT);
    extern __shared__ __align__(128) uint8_t xbuf[];       // gate rows | up rows, then down rows
    const unsigned rank = cluster_rank();
    cluster_arrive();                   // paired with the wait before the first remote store
    const int slot = blockIdx.x / XCL, t = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr size_t GU_BYTES = size_t(MOE_FF) * XROW;
    constexpr int LPR = MOE_FF / F::UNIT;
    __shared__ __align__(8) uint64_t bar[2];
    __shared__ float hpart[XGU];
    __shared__ __align__(16) float hfull[MOE_FF];
    __shared__ __align__(16) int8_t hq[MOE_FF];
    __shared__ __align__(16) int8_t hqi[MOE_FF];           // unit-interleaved copy (Q6_K down rows)
    __shared__ float hd[MOE_FF / 256];
    __shared__ int16_t hs[MOE_FF / 16];
    __shared__ int is_last;
    const int g0 = int(rank) * XGU, d0 = int(rank) * XDN;
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        mbar_fence_init();
    }
    __syncthreads();
    // the next layer's L2 plan (output projection, router rows, shared
    // expert), each range split evenly over the grid's CTAs: a CTA does not
    // retire until its bulk prefetches are issued in full, so no CTA takes
    // more than a small slice
    if (warp == 1 && lane < Prefetch::N && pf.p[lane]) {
        const size_t per = ((pf.bytes[lane] + gridDim.x - 1) / gridDim.x + 15) & ~size_t(15);
        const size_t lo = per * blockIdx.x;
        if (lo < pf.bytes[lane]) {
            const size_t n = pf.bytes[lane] - lo < per ? pf.bytes[lane] - lo : per;
            prefetch_l2_range(static_cast<const uint8_t *>(pf.p[lane]) + lo, n);
        }
    }
    const uint8_t *Db = down_sh;
    if (slot == MOE_TOPK && warp == 0) {
        if (lane == 0) mbar_expect_tx(&bar[0], 2 * XGU_BYTES);
        __syncwarp();
        bulk_g2s_warp(xbuf, gate_sh + g0 * XROW, XGU_BYTES, &bar[0], lane);
        bulk_g2s_warp(xbuf + XGU_BYTES, up_sh + g0 * XROW, XGU_BYTES, &bar[0], lane);
        if (lane == 0) prefetch_rows(shift_rows(DownPtr<F>::at(Db), d0, MOE_FF), XDN, MOE_FF);
    }
    pdl_wait();
    if (slot < MOE_TOPK) {
        const int e = __ldcg(&s.sel[t * MOE_TOPK + slot]);
        Db = down_exps + size_t(e) * down_bytes;
        if (warp == 0) {
            if (lane == 0) mbar_expect_tx(&bar[0], 2 * XGU_BYTES);
            __syncwarp();
            bulk_g2s_warp(xbuf, gate_exps + size_t(e) * GU_BYTES + g0 * XROW, XGU_BYTES, &bar[0], lane);
            bulk_g2s_warp(xbuf + XGU_BYTES, up_exps + size_t(e) * GU_BYTES + g0 * XROW, XGU_BYTES, &bar[0], lane);
            if (lane == 0) prefetch_rows(shift_rows(DownPtr<F>::at(Db), d0, MOE_FF), XDN, MOE_FF);
        }
    }
    // ---- gate / up rows g0 + 4 warp .. + 3 from shared memory ---------------
    FmtQ4K::Act act;
    FmtQ4K::load_act(act, s.xq + size_t(t) * MOE_EMBD, s.xd + size_t(t) * 8, s.xs + size_t(t) * 128,
                     lane);
    QMA_TRACE_MARK(TK_EXPERT, 1);
    const bool gu_ok = mbar_wait(&bar[0], 0);
    QMA_TRACE_MARK(TK_EXPERT, 2);
    {
        constexpr int RPWARP = XGU / (XTHREADS / 32);
        static_assert(RPWARP == 2, "4 dots (2 gate + 2 up rows) per warp");
        float dv[4];
#pragma unroll
        for (int k = 0; k < RPWARP; k++) {
            FmtQ4K::Wt wg, wu;
            FmtQ4K::load_w_smem(wg, xbuf, warp * RPWARP + k, MOE_EMBD, lane);
            FmtQ4K::load_w_smem(wu, xbuf + XGU_BYTES, warp * RPWARP + k, MOE_EMBD, lane);
            dv[k] = FmtQ4K::dot(wg, act, lane);
            dv[2 + k] = FmtQ4K::dot(wu, act, lane);
        }
        const float tot = warp_sum4(dv, lane);          // lane: row (index & 1), gate/up (index & 2)
        const float u = __shfl_xor_sync(0xffffffffu, tot, 16);
        if ((lane & 23) == 0) {                          // gate lanes 0 and 8, one per row
            const float g = tot;
            hpart[warp * RPWARP + (warp_sum4_index(lane) & 1)] = gu_ok ? (g / (1.0f + expf(-g))) * u : 0.0f;
        }
    }
    __syncthreads();                    // gate/up rows consumed: reuse the buffer
    if (warp == 0) {
        if (lane == 0 && !gu_ok) atomicAdd(&g_moe_timeouts, 1u);
        fence_proxy_async_smem();
        DownBytes<F>::issue(xbuf, Db, d0, &bar[1], lane);
    }
    // ---- the cluster's 512 hidden values: every CTA pushes its 32 ----------
    cluster_wait();                     // every CTA of the cluster has started
    for (int i = tid; i < XGU * XCL; i += XTHREADS)
        st_cluster_f32(cluster_map(&hfull[g0 + i % XGU], unsigned(i / XGU)), hpart[i % XGU]);
    QMA_TRACE_MARK(TK_EXPERT, 3);
    cluster_sync();                     // all pushes landed; no remote access after this
    QMA_TRACE_MARK(TK_EXPERT, 4);
    if (warp < MOE_FF / 256) {
        const float4 a0 = *reinterpret_cast<const float4 *>(hfull + warp * 256 + lane * 8);
        const float4 a1 = *reinterpret_cast<const float4 *>(hfull + warp * 256 + lane * 8 + 4);
        const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        q8k_block_warp(v, lane, hq + warp * 256, hd + warp, hs + warp * 16);
    }
    __syncthreads();
    if constexpr (std::is_same<F, FmtQ6K>::value) {
        if (tid < MOE_FF / 16) {
            const int u = tid >> 3, k = tid & 7;          // chunk k of 128-byte unit u
            reinterpret_cast<int4 *>(hqi)[4 * k + u] = reinterpret_cast<const int4 *>(hq)[tid];
        }
        __syncthreads();
    }
    // ---- down rows d0 .. d0 + XDN from shared memory --------------------------
    QMA_TRACE_MARK(TK_EXPERT, 5);
    const bool dn_ok = mbar_wait(&bar[1], 0);
    QMA_TRACE_MARK(TK_EXPERT, 6);
    float *part = s.part + (size_t(t) * MOE_NSLOT + slot) * MOE_EMBD + d0;
    if (dn_ok) {
        gemv_warp_rows<DownRows<F>, 1, LPR, 1, 1>(DownBytes<F>::at(xbuf), MOE_FF, XDN,
                                                  std::is_same<F, FmtQ6K>::value ? hqi : hq, hd, hs, part, 0,
                                                  warp, XTHREADS / 32, lane);
    } else {
        if (tid == 0) atomicAdd(&g_moe_timeouts, 1u);
        if (tid < XDN) part[tid] = 0.0f;
        mbar_wait(&bar[1], 0);          // let a late copy land before the CTA exits
    }

    QMA_TRACE_MARK(TK_EXPERT, 7);
    // the next layer's kernels may launch now: this kernel's weight traffic
    // is done, only the combine remains
    pdl_trigger();
    if (!combine) return;               // moe_combine_norm_kernel combines
    // ---- the last of the 9 slot CTAs of this row chunk combines --------------
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned ticket = atomicAdd(&s.dcount[t * MOE_DOWN_CHUNKS + rank], 1u);
        is_last = ticket == MOE_NSLOT - 1;
    }
    __syncthreads();
    if (is_last) {
        __threadfence();
        if (tid < XDN) {
            const int r = d0 + tid;
            float acc = 0.0f;
#pragma unroll
            for (int k = 0; k < MOE_TOPK; k++) {
                const float p = __ldcg(&s.part[(size_t(t) * MOE_NSLOT + k) * MOE_EMBD + r]);
                acc = __fadd_rn(acc, __fmul_rn(__ldcg(&s.w[t * MOE_TOPK + k]), p));
            }
            const float psh = __ldcg(&s.part[(size_t(t) * MOE_NSLOT + MOE_TOPK) * MOE_EMBD + r]);
            acc = __fadd_rn(acc, __fmul_rn(__ldcg(&s.gs[t]), psh));
            x_out[size_t(t) * MOE_EMBD + r] = __fadd_rn(acc, x2[size_t(t) * MOE_EMBD + r]);
        }
        if (tid == 0) s.dcount[t * MOE_DOWN_CHUNKS + rank] = 0;
    }
}

// Combine + residual + next RMSNorm + Q8_K, one CTA of 256 threads per
// token, 8 rows per thread: the slots are combined in the reference's order
// exactly as the expert kernel's combine does (nn.c:615-629, residual
// nn.c:2246-2252), then rms_norm_m (nn.c:348-357) and the Q8_K quantization
// of the next matmul (nn.c:318-324) with the arithmetic of
// rmsnorm_quant_kernel.
__global__ void __launch_bounds__(256) moe_combine_norm_kernel(MoeScratch s, const float *x2, float *x_out,
                                                               const float *__restrict__ w, int norm_from,
                                                               int8_t *xq, float *xd, int16_t *xs,
                                                               Prefetch pf) {
    QMA_TRACE_SCOPE(TK_MOE_NORM);
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ double red[8];
    pdl_trigger();
    if (t == 0) {
#pragma unroll
        for (int i = 0; i < Prefetch::N; i++)
            if (tid == i && pf.p[i]) prefetch_l2_range(pf.p[i], pf.bytes[i]);
    }
    const bool norm = w != nullptr && t >= norm_from;
    float wv[8] = {};
    if (norm) {
        const float4 wa = __ldg(reinterpret_cast<const float4 *>(w + tid * 8));
        const float4 wb = __ldg(reinterpret_cast<const float4 *>(w + tid * 8 + 4));
        wv[0] = wa.x; wv[1] = wa.y; wv[2] = wa.z; wv[3] = wa.w;
        wv[4] = wb.x; wv[5] = wb.y; wv[6] = wb.z; wv[7] = wb.w;
    }
    pdl_wait();
    const size_t r0 = size_t(t) * MOE_EMBD + tid * 8;
    float acc[8] = {};
#pragma unroll
    for (int k = 0; k <= MOE_TOPK; k++) {
        const float4 *pp = reinterpret_cast<const float4 *>(s.part + (size_t(t) * MOE_NSLOT + k) * MOE_EMBD + tid * 8);
        const float4 a = __ldcg(pp), b = __ldcg(pp + 1);
        const float p[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        const float wk = k < MOE_TOPK ? __ldcg(&s.w[t * MOE_TOPK + k]) : __ldcg(&s.gs[t]);
#pragma unroll
        for (int j = 0; j < 8; j++) acc[j] = __fadd_rn(acc[j], __fmul_rn(wk, p[j]));
    }
    const float4 xa = __ldcg(reinterpret_cast<const float4 *>(x2 + r0));
    const float4 xb = __ldcg(reinterpret_cast<const float4 *>(x2 + r0 + 4));
    const float xr[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = __fadd_rn(acc[j], xr[j]);
    reinterpret_cast<float4 *>(x_out + r0)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4 *>(x_out + r0)[1] = make_float4(v[4], v[5], v[6], v[7]);
    if (!norm) return;                  // block-uniform
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < 8; k++) ss += double(v[k]) * double(v[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    const double tot = ((red[0] + red[1]) + (red[2] + red[3])) + ((red[4] + red[5]) + (red[6] + red[7]));
    const float r = 1.0f / sqrtf(float(tot / MOE_EMBD) + 1e-6f);
#pragma unroll
    for (int k = 0; k < 8; k++) v[k] = __fmul_rn(__fmul_rn(v[k], r), wv[k]);
    const int row = t - norm_from;
    q8k_block_warp(v, lane, xq + size_t(row) * MOE_EMBD + warp * 256, xd + size_t(row) * 8 + warp,
                   xs + size_t(row) * 128 + warp * 16);
}

int moe_wait_timeouts() {
    unsigned n = 0;
    if (cudaMemcpyFromSymbol(&n, g_moe_timeouts, sizeof(n)) != cudaSuccess) return -1;
    if (n) {
        const unsigned zero = 0;
        cudaMemcpyToSymbol(g_moe_timeouts, &zero, sizeof(zero));
    }
    return int(n);
}

static PerDevice g_moe_attrs;

static int moe_attrs() {
    if (g_moe_attrs.done()) return QMA_CUDA_OK;
    QMA_CHECK_CUDA(cudaFuncSetAttribute(moe_router_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    QMA_CHECK_CUDA(cudaFuncSetAttribute(moe_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(ROUTER_SMEM)));
    QMA_CHECK_CUDA(cudaFuncSetAttribute(moe_router_multi_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    QMA_CHECK_CUDA(cudaFuncSetAttribute(moe_router_multi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(ROUTER_MULTI_SMEM)));
    QMA_CHECK_CUDA(cudaFuncSetAttribute(moe_expert_kernel<FmtQ6K>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    QMA_CHECK_CUDA(cudaFuncSetAttribute(moe_expert_kernel<FmtQ4K>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    QMA_CHECK_CUDA(cudaFuncSetAttribute(moe_expert_kernel<FmtQ6K>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(EXPERT_SMEM)));
    QMA_CHECK_CUDA(cudaFuncSetAttribute(moe_expert_kernel<FmtQ4K>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(EXPERT_SMEM)));
    // the 9 expert clusters must be co-resident beside other kernels' CTAs:
    // prefer the largest shared-memory carveout (two CTAs per SM)
    QMA_CHECK_CUDA(cudaFuncSetAttribute(moe_expert_kernel<FmtQ6K>, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    QMA_CHECK_CUDA(cudaFuncSetAttribute(moe_expert_kernel<FmtQ4K>, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    g_moe_attrs.mark();
    return QMA_CUDA_OK;
}

// The router for T tokens: the single-token kernel per token below 8 tokens
// (decode), the multi-token kernel (RTPC tokens per cluster) from 8 on.
static cudaError_t launch_router(const qma_cuda_moe_weights &w, const float *x2, int T, const MoeScratch &s, int *sel,
                                 float *wts, cudaStream_t st, bool pdl) {
    if (T >= 8)
        return launch_ex(moe_router_multi_kernel, dim3(RCL, (T + RTPC - 1) / RTPC), dim3(RTHREADS), ROUTER_MULTI_SMEM,
                         st, RCL, pdl, x2, T, w.post_norm, w.gate_inp, w.gate_inp_shexp, s, sel, wts, w.router_bias);
    return launch_ex(moe_router_kernel, dim3(RCL, T), dim3(RTHREADS), ROUTER_SMEM, st, RCL, pdl, x2, w.post_norm,
                     w.gate_inp, w.gate_inp_shexp, s, sel, wts, w.router_bias);
}

int moe_route(const qma_cuda_moe_weights &w, const float *x2, int T, const MoeScratch &s, int *sel, float *wts,
              cudaStream_t st) {
    int rc = moe_attrs();
    if (rc) return rc;
    QMA_CHECK_CUDA(launch_router(w, x2, T, s, sel, wts, st, false));
    return QMA_CUDA_OK;
}

int moe_combine(const MoeScratch &s, const float *x2, float *x_out, int T, cudaStream_t st) {
    const MoeNormTail none;
    QMA_CHECK_CUDA(launch_ex(moe_combine_norm_kernel, dim3(T), dim3(256), 0, st, 1, pdl_enabled(), s, x2, x_out,
                             none.w, none.norm_from, none.xq, none.xd, none.xs, none.pf));
    return QMA_CUDA_OK;
}

int moe_layer(const qma_cuda_moe_weights &w, const float *x2, int T, float *x_out, int *sel,
              float *wts, void *scratch, cudaStream_t st, bool clear_counters, const MoeNormTail *tail) {
    MoeScratch s = moe_scratch_layout(scratch, T);
    int rc0 = moe_attrs();
    if (rc0) return rc0;
    if (clear_counters) {
        QMA_CHECK_CUDA(cudaMemsetAsync(s.dcount, 0, sizeof(unsigned) * T * MOE_DOWN_CHUNKS, st));
    }
    const bool pdl = pdl_enabled() && !clear_counters;
    QMA_CHECK_CUDA(launch_router(w, x2, T, s, sel, wts, st, pdl));
    if (s.goff && w.down_type == QMA_TYPE_Q6_K) {
        // a chunk of tokens: experts grouped, tensor-core MMAs, then the combine
        // (and the next norm when asked) in one kernel
        int rc = moe_grouped(w, T, s, st);
        if (rc) return rc;
        const MoeNormTail none;
        const MoeNormTail &tl = tail ? *tail : none;
        QMA_CHECK_CUDA(launch_ex(moe_combine_norm_kernel, dim3(T), dim3(256), 0, st, 1, pdl_enabled(), s, x2, x_out,
                                 tl.w, tl.norm_from, tl.xq, tl.xd, tl.xs, tl.pf));
        return QMA_CUDA_OK;
    }
    const size_t eb = packed_bytes(w.down_type, MOE_EMBD, MOE_FF);
    const dim3 grid(MOE_NSLOT * XCL, T);
    const uint8_t *ge = static_cast<const uint8_t *>(w.gate_exps), *ue = static_cast<const uint8_t *>(w.up_exps);
    const uint8_t *gsh = static_cast<const uint8_t *>(w.gate_shexp), *ush = static_cast<const uint8_t *>(w.up_shexp);
    const uint8_t *de = static_cast<const uint8_t *>(w.down_exps), *dsh = static_cast<const uint8_t *>(w.down_shexp);
    // the next layer's L2 plan goes with the expert kernel's many CTAs, not
    // with the single-CTA combine
    const Prefetch plan = tail ? tail->pf : Prefetch();
    if (w.down_type == QMA_TYPE_Q6_K)
        QMA_CHECK_CUDA(launch_ex(moe_expert_kernel<FmtQ6K>, grid, dim3(XTHREADS), EXPERT_SMEM, st, XCL, pdl_enabled(), ge, ue,
                                 gsh, ush, de, eb, dsh, x2, x_out, s, tail ? 0 : 1, plan));
    else
        QMA_CHECK_CUDA(launch_ex(moe_expert_kernel<FmtQ4K>, grid, dim3(XTHREADS), EXPERT_SMEM, st, XCL, pdl_enabled(), ge, ue,
                                 gsh, ush, de, eb, dsh, x2, x_out, s, tail ? 0 : 1, plan));
    if (tail)
        QMA_CHECK_CUDA(launch_ex(moe_combine_norm_kernel, dim3(T), dim3(256), 0, st, 1, pdl_enabled(), s, x2, x_out,
                                 tail->w, tail->norm_from, tail->xq, tail->xd, tail->xs, Prefetch()));
    return QMA_CUDA_OK;
}

}  // namespace qma

extern "C" {

size_t qma_cuda_moe_scratch_bytes(int T) { return T > 0 ? qma::moe_scratch_bytes(T) : 0; }

int qma_cuda_moe_layer(const qma_cuda_moe_weights *w, const float *x2, int T, float *x_out,
                       int32_t *sel, float *wts, void *scratch, size_t scratch_bytes,
                       void *stream) {
    qma::clear_error();
    QMA_REQUIRE(w && x2 && x_out && scratch && T > 0 && T <= 65535,
                "qma_cuda_moe_layer: bad arguments (T %d)", T);
    QMA_REQUIRE(qma::aligned_to(x2, 16) && qma::aligned_to(x_out, 16) && qma::aligned_to(scratch, 256),
                "qma_cuda_moe_layer: x2 / x_out must be 16-byte and scratch 256-byte aligned");
    QMA_REQUIRE(w->post_norm && w->gate_inp && w->gate_exps && w->up_exps && w->down_exps &&
                    w->gate_inp_shexp && w->gate_shexp && w->up_shexp && w->down_shexp,
                "qma_cuda_moe_layer: missing weight pointer");
    QMA_REQUIRE(w->down_type == QMA_TYPE_Q6_K || w->down_type == QMA_TYPE_Q4_K,
                "qma_cuda_moe_layer: down_type %d must be Q6_K or Q4_K", w->down_type);
    QMA_REQUIRE(w->down_shexp_type == w->down_type,
                "qma_cuda_moe_layer: shared and routed down projections must share a type");
    QMA_REQUIRE(scratch_bytes >= qma::moe_scratch_bytes(T),
                "qma_cuda_moe_layer: scratch %zu bytes < %zu needed", scratch_bytes,
                qma::moe_scratch_bytes(T));
    return qma::moe_layer(*w, x2, T, x_out, sel, wts, scratch, qma::as_stream(stream), true);
}

int qma_cuda_moe_exact_fallbacks(const void *scratch, int T, int *count) {
    qma::clear_error();
    QMA_REQUIRE(scratch && count && T > 0, "qma_cuda_moe_exact_fallbacks: bad arguments");
    qma::MoeScratch s = qma::moe_scratch_layout(const_cast<void *>(scratch), T);
    int *h = new int[T];
    cudaError_t e = cudaMemcpy(h, s.fallback, sizeof(int) * T, cudaMemcpyDeviceToHost);
    int c = 0;
    for (int i = 0; i < T; i++) c += h[i] != 0;
    delete[] h;
    if (e != cudaSuccess) {
        qma::set_error("qma_cuda_moe_exact_fallbacks: %s", cudaGetErrorString(e));
        return QMA_CUDA_ERR_CUDA;
    }
    *count = c;
    return QMA_CUDA_OK;
}

}  // extern "C"
