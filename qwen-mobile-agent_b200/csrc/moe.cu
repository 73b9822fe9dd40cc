// moe.cu -- the qwen35moe MoE FFN block on B200: router + top-8, fused
// gate/up + SwiGLU, down projection + weighted combine + residual.
//
// Reference: moe_ffn (nn.c:509-649), moe_expert_one_q8k (nn.c:412-439),
// moe_shared_q8k (nn.c:446-473), the residual in qma_eval (nn.c:2246-2252).
//
// Three kernels per call (T tokens, grid.y = token):
//   1. router   : 64 CTAs x 4 warps, one warp per expert.  Every CTA forms
//                 xn = rms_norm(x2) * post_norm in shared memory, each warp
//                 computes one router logit exactly in fp64 together with a
//                 proven bound on the reference's sequential fp32 sum; the
//                 last CTA to finish selects the top 8 (falling back to the
//                 reference's own summation order for any rank the bound
//                 cannot settle), renormalises the weights, quantizes xn to
//                 Q8_K and computes the shared-expert gate.
//   2. gate/up  : 9 slots (8 routed + shared) x 16 chunks of 32 rows; one
//                 warp streams a gate row and an up row (Q4_K), SwiGLU.
//   3. down     : 9 slots x 16 chunks of 128 output rows; each CTA
//                 quantizes its slot's hidden vector to Q8_K in shared memory
//                 and runs the Q6_K (or Q4_K) GEMV; the last of the 9 CTAs of
//                 a chunk combines the slots in the reference's order and
//                 adds the residual.
#include <math.h>

#include "common.cuh"
#include "gemv.cuh"
#include "moe.cuh"
#include "quant.cuh"

namespace qma {

// ----------------------------------------------------------------- scratch --
static inline size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

size_t moe_scratch_bytes(int T) {
    size_t b = 0;
    b += al256(sizeof(unsigned) * T);                     // rcount
    b += al256(sizeof(unsigned) * T * MOE_DOWN_CHUNKS);   // dcount
    b += al256(sizeof(double) * T * MOE_NEXP) * 2;        // S, B
    b += al256(sizeof(int) * T);                          // fallback
    b += al256(sizeof(int) * T * MOE_TOPK);               // sel
    b += al256(sizeof(float) * T * MOE_TOPK);             // w
    b += al256(size_t(T) * MOE_EMBD);                     // xq
    b += al256(sizeof(float) * T * (MOE_EMBD / 256));     // xd
    b += al256(sizeof(int16_t) * T * (MOE_EMBD / 16));    // xs
    b += al256(sizeof(float) * T);                        // gs
    b += al256(sizeof(float) * T * MOE_NSLOT * MOE_FF);   // h
    b += al256(sizeof(float) * T * MOE_NSLOT * MOE_EMBD); // part
    return b;
}

MoeScratch moe_scratch_layout(void *base, int T) {
    uint8_t *p = static_cast<uint8_t *>(base);
    MoeScratch s;
    auto take = [&](size_t n) { uint8_t *q = p; p += al256(n); return q; };
    s.rcount = reinterpret_cast<unsigned *>(take(sizeof(unsigned) * T));
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
    s.h = reinterpret_cast<float *>(take(sizeof(float) * T * MOE_NSLOT * MOE_FF));
    s.part = reinterpret_cast<float *>(take(sizeof(float) * T * MOE_NSLOT * MOE_EMBD));
    return s;
}

// --------------------------------------------------------------- helpers --
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_max_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// xn lives in shared memory in chunks of 64 floats padded to 68, so a lane
// reading its own contiguous 64 elements with 16-byte loads is bank-conflict
// free.
__device__ __forceinline__ int xn_idx(int i) { return (i >> 6) * 68 + (i & 63); }

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

__global__ void __launch_bounds__(128) moe_router_kernel(const float *__restrict__ x2,
                                                         const float *__restrict__ post_norm,
                                                         const float *__restrict__ Wr,
                                                         const float *__restrict__ gis,
                                                         MoeScratch s, int *sel_out,
                                                         float *w_out) {
    const int t = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int e_mine = blockIdx.x * 4 + warp;
    __shared__ __align__(16) float xn[MOE_EMBD / 64 * 68];
    __shared__ double dred[4];
    __shared__ float fred[4];
    __shared__ int is_last, need_exact, ncand;
    __shared__ double sS[MOE_NEXP], sB[MOE_NEXP];
    __shared__ int cls[MOE_NEXP];
    __shared__ int top[MOE_TOPK];
    __shared__ float topL[MOE_TOPK];
    __shared__ int cand[MOE_NEXP];

    // router row of this warp's expert: independent of the upstream kernel,
    // so it is requested before waiting on it
    float4 wv[16];
    {
        const float4 *wr = reinterpret_cast<const float4 *>(Wr + size_t(e_mine) * MOE_EMBD + lane * 64);
#pragma unroll
        for (int k = 0; k < 16; k++) wv[k] = __ldg(wr + k);
    }
    pdl_wait();
    // ---- xn = rms_norm(x2) * post_norm (rms_norm_m, nn.c:348-357) -------
    const float *x = x2 + size_t(t) * MOE_EMBD;
    float xv[16];
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < 16; k++) {
        xv[k] = x[tid + 128 * k];
        ss += double(xv[k]) * double(xv[k]);
    }
    ss = warp_sum_d(ss);
    if (lane == 0) dred[warp] = ss;
    __syncthreads();
    const double tot = (dred[0] + dred[1]) + (dred[2] + dred[3]);
    const float r = 1.0f / sqrtf(float(tot / MOE_EMBD) + 1e-6f);
#pragma unroll
    for (int k = 0; k < 16; k++) {
        const int i = tid + 128 * k;
        xn[xn_idx(i)] = __fmul_rn(__fmul_rn(xv[k], r), post_norm[i]);
    }
    __syncthreads();

    // ---- one router logit per warp: exact value + bound -----------------
    // The reference sums s += g_i * x_i sequentially in fp32 (nn.c:519-521).
    // With a_i = fl(g_i * x_i) (the same products) and S_i the exact prefix
    // sums, recursive summation satisfies |s_fp32 - S_n| <= u' sum_i |S_i|
    // with u' = 2^-24 (1 + n u) for n = 2048.  S_n is summed in fp64
    // (error ~1e-13 relative); sum_i |S_i| in fp32 prefix sums, whose own
    // error (< 1e-3 relative) the 1.01 factor covers.
    {
        const float4 *xr = reinterpret_cast<const float4 *>(xn + lane * 68);
        float a[64];
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const float4 xw = xr[k];
            a[4 * k + 0] = __fmul_rn(wv[k].x, xw.x);
            a[4 * k + 1] = __fmul_rn(wv[k].y, xw.y);
            a[4 * k + 2] = __fmul_rn(wv[k].z, xw.z);
            a[4 * k + 3] = __fmul_rn(wv[k].w, xw.w);
        }
        double t4[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
        for (int j = 0; j < 64; j++) t4[j & 3] += double(a[j]);
        const double tl = (t4[0] + t4[1]) + (t4[2] + t4[3]);
        double incl = tl;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        float p = float(incl - tl), el = 0.0f;
#pragma unroll
        for (int j = 0; j < 64; j++) {
            p += a[j];
            el += fabsf(p);
        }
        const float E = warp_sum(el);
        const double S = __shfl_sync(0xffffffffu, incl, 31);
        if (lane == 0) {
            s.S[size_t(t) * MOE_NEXP + e_mine] = S;
            s.B[size_t(t) * MOE_NEXP + e_mine] = double(E) * 0x1.0p-24 * 1.01 + 1e-30;
        }
    }

    // ---- the last CTA of this token selects ------------------------------
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned ticket = atomicAdd(&s.rcount[t], 1u);
        is_last = ticket == gridDim.x - 1;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (int i = tid; i < MOE_NEXP; i += 128) {
        sS[i] = __ldcg(&s.S[size_t(t) * MOE_NEXP + i]);
        sB[i] = __ldcg(&s.B[size_t(t) * MOE_NEXP + i]);
    }
    __syncthreads();
    if (warp == 0) {
        double mx = -INFINITY;
        for (int j = 0; j < 8; j++) mx = fmax(mx, sS[lane + 32 * j]);
        mx = warp_max_d(mx);
        for (int j = 0; j < 8; j++) cls[lane + 32 * j] = p_class(sS[lane + 32 * j], mx);
        __syncwarp();
        const bool ok = select_top8(sS, sB, cls, lane, top);
        if (lane == 0) {
            need_exact = !ok;
            ncand = 0;
        }
    }
    __syncthreads();
    if (need_exact) {
        // Every expert whose rank the bounds leave open gets its logit
        // recomputed in the reference's exact order, s = fl(s + fl(g_i x_i)),
        // i = 0..2047; their intervals then collapse to the exact value.
        const int e8 = top[MOE_TOPK - 1];
        const double thresh = sS[e8] - sB[e8];
        for (int e = tid; e < MOE_NEXP; e += 128)
            if (cls[e] > 0 && sS[e] + sB[e] >= thresh - 1e-6 * (1.0 + fabs(sS[e8]))) cand[atomicAdd(&ncand, 1)] = e;
        __syncthreads();
        for (int c = tid; c < ncand; c += 128) {
            const int e = cand[c];
            const float *wr = Wr + size_t(e) * MOE_EMBD;
            float acc = 0.0f;
            for (int i = 0; i < MOE_EMBD; i++) acc = __fadd_rn(acc, __fmul_rn(__ldg(wr + i), xn[xn_idx(i)]));
            sS[e] = double(acc);
            sB[e] = 0.0;
        }
        __syncthreads();
        if (warp == 0) {
            double mx = -INFINITY;
            for (int j = 0; j < 8; j++) mx = fmax(mx, sS[lane + 32 * j]);
            mx = warp_max_d(mx);
            for (int j = 0; j < 8; j++) cls[lane + 32 * j] = p_class(sS[lane + 32 * j], mx);
            __syncwarp();
            select_top8(sS, sB, cls, lane, top);   // now settled by exact values
        }
    }
    __syncthreads();
    if (tid < MOE_TOPK) topL[tid] = float(sS[top[tid]]);
    __syncthreads();
    if (tid == 0) {
        // renormalised softmax weights of the selected experts (nn.c:524-547)
        float ev[MOE_TOPK], sum = 0.0f;
        for (int k = 0; k < MOE_TOPK; k++) { ev[k] = expf(topL[k] - topL[0]); sum += ev[k]; }
        for (int k = 0; k < MOE_TOPK; k++) {
            const float wk = ev[k] / sum;
            s.sel[t * MOE_TOPK + k] = top[k];
            s.w[t * MOE_TOPK + k] = wk;
            if (sel_out) sel_out[t * MOE_TOPK + k] = top[k];
            if (w_out) w_out[t * MOE_TOPK + k] = wk;
        }
        s.fallback[t] = need_exact;
    }
    // ---- Q8_K of xn (shared by every expert) and the shared-expert gate --
    float gpart = 0.0f;
    for (int blk = warp; blk < MOE_EMBD / 256; blk += 4) {
        const int i0 = blk * 256 + lane * 8;
        const float4 a0 = *reinterpret_cast<const float4 *>(xn + xn_idx(i0));
        const float4 a1 = *reinterpret_cast<const float4 *>(xn + xn_idx(i0 + 4));
        const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        int q[8];
        float sc;
        q8k_block_warp_q(v, lane, s.xq + size_t(t) * MOE_EMBD + blk * 256,
                         s.xd + size_t(t) * (MOE_EMBD / 256) + blk,
                         s.xs + size_t(t) * (MOE_EMBD / 16) + blk * 16, q, sc);
        // shared-expert gate input: sum_i g_i * xq_i * xd (nn.c:453)
#pragma unroll
        for (int c = 0; c < 8; c++) gpart += __fmul_rn(__fmul_rn(gis[i0 + c], float(q[c])), sc);
    }
    gpart = warp_sum(gpart);
    if (lane == 0) fred[warp] = gpart;
    __syncthreads();
    if (tid == 0) {
        const float g = (fred[0] + fred[1]) + (fred[2] + fred[3]);
        s.gs[t] = 1.0f / (1.0f + expf(-g));
        s.rcount[t] = 0;   // ready for the next call
    }
}

// ------------------------------------------------------------ gate / up ---
__global__ void __launch_bounds__(256) moe_gateup_kernel(const uint8_t *__restrict__ gate_exps,
                                                         const uint8_t *__restrict__ up_exps,
                                                         const uint8_t *__restrict__ gate_sh,
                                                         const uint8_t *__restrict__ up_sh,
                                                         MoeScratch s) {
    const int t = blockIdx.y;
    const int slot = blockIdx.x / MOE_GU_CHUNKS, chunk = blockIdx.x % MOE_GU_CHUNKS;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr size_t EXP_BYTES = size_t(MOE_FF) * (MOE_EMBD / 256) * Q4K_BYTES;
    pdl_wait();
    const uint8_t *G, *U;
    if (slot < MOE_TOPK) {
        const int e = __ldcg(&s.sel[t * MOE_TOPK + slot]);
        G = gate_exps + size_t(e) * EXP_BYTES;
        U = up_exps + size_t(e) * EXP_BYTES;
    } else {
        G = gate_sh;
        U = up_sh;
    }
    FmtQ4K::Act act;
    FmtQ4K::load_act(act, s.xq + size_t(t) * MOE_EMBD, s.xd + size_t(t) * 8,
                     s.xs + size_t(t) * 128, lane);
    constexpr int RPWARP = MOE_GU_ROWS / 8;       // row pairs per warp
    const int r0 = chunk * MOE_GU_ROWS + warp * RPWARP;
    FmtQ4K::Wt wg[RPWARP], wu[RPWARP];
#pragma unroll
    for (int k = 0; k < RPWARP; k++) {
        FmtQ4K::load_w(wg[k], G, r0 + k, MOE_EMBD, lane);
        FmtQ4K::load_w(wu[k], U, r0 + k, MOE_EMBD, lane);
    }
#pragma unroll
    for (int k = 0; k < RPWARP; k++) {
        const float g = warp_sum(FmtQ4K::dot(wg[k], act, lane));
        const float u = warp_sum(FmtQ4K::dot(wu[k], act, lane));
        if (lane == 0)
            s.h[(size_t(t) * MOE_NSLOT + slot) * MOE_FF + r0 + k] = (g / (1.0f + expf(-g))) * u;
    }
}

// ---------------------------------------------------------- down + combine -
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

template <class F>
__global__ void __launch_bounds__(256) moe_down_kernel(const uint8_t *__restrict__ down_exps,
                                                       size_t expert_bytes,
                                                       const uint8_t *__restrict__ down_sh,
                                                       const float *x2, float *x_out,
                                                       MoeScratch s) {
    const int t = blockIdx.y;
    const int slot = blockIdx.x / MOE_DOWN_CHUNKS, chunk = blockIdx.x % MOE_DOWN_CHUNKS;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ __align__(16) int8_t hq[MOE_FF];
    __shared__ float hd[MOE_FF / 256];
    __shared__ int16_t hs[MOE_FF / 16];
    __shared__ int is_last;
    pdl_wait();
    // Q8_K of this slot's gated hidden vector (nn.c:434 / :467)
    if (warp < MOE_FF / 256) {
        const float *h = s.h + (size_t(t) * MOE_NSLOT + slot) * MOE_FF + warp * 256 + lane * 8;
        const float4 a0 = __ldcg(reinterpret_cast<const float4 *>(h));
        const float4 a1 = __ldcg(reinterpret_cast<const float4 *>(h + 4));
        const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        q8k_block_warp(v, lane, hq + warp * 256, hd + warp, hs + warp * 16);
    }
    __syncthreads();
    const uint8_t *base;
    if (slot < MOE_TOPK) base = down_exps + size_t(__ldcg(&s.sel[t * MOE_TOPK + slot])) * expert_bytes;
    else base = down_sh;
    const auto P = shift_rows(DownPtr<F>::at(base), chunk * MOE_DOWN_CHUNK, MOE_FF);
    constexpr int LPR = MOE_FF / F::UNIT;
    float *part = s.part + (size_t(t) * MOE_NSLOT + slot) * MOE_EMBD + chunk * MOE_DOWN_CHUNK;
    gemv_warp_rows<F, 1, LPR, 1, 1>(P, MOE_FF, MOE_DOWN_CHUNK, hq, hd, hs, part, 0, warp, 8, lane);

    // the last of the 9 slot CTAs of this chunk combines (nn.c:615-629)
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned ticket = atomicAdd(&s.dcount[t * MOE_DOWN_CHUNKS + chunk], 1u);
        is_last = ticket == MOE_NSLOT - 1;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    if (tid < MOE_DOWN_CHUNK) {
        const int r = chunk * MOE_DOWN_CHUNK + tid;
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
    if (tid == 0) s.dcount[t * MOE_DOWN_CHUNKS + chunk] = 0;
}

int moe_layer(const qma_cuda_moe_weights &w, const float *x2, int T, float *x_out, int *sel,
              float *wts, void *scratch, cudaStream_t st) {
    MoeScratch s = moe_scratch_layout(scratch, T);
    QMA_CHECK_CUDA(cudaMemsetAsync(s.rcount, 0, sizeof(unsigned) * T, st));
    QMA_CHECK_CUDA(cudaMemsetAsync(s.dcount, 0, sizeof(unsigned) * T * MOE_DOWN_CHUNKS, st));
    moe_router_kernel<<<dim3(MOE_NEXP / 4, T), 128, 0, st>>>(x2, w.post_norm, w.gate_inp,
                                                            w.gate_inp_shexp, s, sel, wts);
    QMA_CHECK_LAUNCH();
    moe_gateup_kernel<<<dim3(MOE_NSLOT * MOE_GU_CHUNKS, T), 256, 0, st>>>(
        static_cast<const uint8_t *>(w.gate_exps), static_cast<const uint8_t *>(w.up_exps),
        static_cast<const uint8_t *>(w.gate_shexp), static_cast<const uint8_t *>(w.up_shexp), s);
    QMA_CHECK_LAUNCH();
    const size_t eb = packed_bytes(w.down_type, MOE_EMBD, MOE_FF);
    const dim3 dg(MOE_NSLOT * MOE_DOWN_CHUNKS, T);
    if (w.down_type == QMA_TYPE_Q6_K)
        moe_down_kernel<FmtQ6K><<<dg, 256, 0, st>>>(static_cast<const uint8_t *>(w.down_exps), eb,
                                                   static_cast<const uint8_t *>(w.down_shexp), x2,
                                                   x_out, s);
    else
        moe_down_kernel<FmtQ4K><<<dg, 256, 0, st>>>(static_cast<const uint8_t *>(w.down_exps), eb,
                                                    static_cast<const uint8_t *>(w.down_shexp), x2,
                                                    x_out, s);
    QMA_CHECK_LAUNCH();
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
    return qma::moe_layer(*w, x2, T, x_out, sel, wts, scratch, qma::as_stream(stream));
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
