// attn.cu -- gated full attention over the 4-bit / 2-bit quantized KV ring
// with HCM tiers (sink + hot + heavy-hitter arena + q2 gist), T queries.
//
// Reference: the attention branch of qma_eval (nn.c:2110-2163), kv_append
// (nn.c:1455-1509), attn_worker (nn.c:1215-1446), the kvq record kernels
// (kvq.c:25-241) and the heavy-hitter arena copy of hcm_rebuild
// (nn.c:1092-1104).
//
// KV layout per attention layer (as the reference's KV slab, nn.c:1887):
//   [K head 0][K head 1][V head 0][V head 1], each n_ctx slots of 240 B:
//   q4 record (8 x {fp16 d, fp16 m, 16 B nibbles}) at 0, q2 record
//   (4 x {d, m, 16 B of 2-bit}) at 160.  Arena: [4 heads][2048][240].
// Attention positions of query t are, in order: the live index
// live[0 .. n_live) (ring q4 | arena q4 | ring q2 segments) and then the tail
// of positions rebuilt_at .. n_pos + t read from the ring at q4; with no live
// index, positions 0 .. n_pos + t.
#include <math.h>

#include "attn.cuh"
#include "common.cuh"
#include "layers.cuh"
#include "quant.cuh"

namespace qma {

__device__ __forceinline__ uint16_t f2h(float x) { return __half_as_ushort(__float2half_rn(x)); }

__device__ __forceinline__ int nk_of(const StepParams &sp, int t) {
    return sp.n_live > 0 ? sp.n_live + (sp.n_pos + t - sp.rebuilt_at + 1) : sp.n_pos + t + 1;
}

// Record of attention position jj for the given KV head: returns the record
// pointer and whether it is a q2 record.
__device__ __forceinline__ const uint8_t *rec_of(const StepParams &sp, const int *live,
                                                 const uint8_t *ring, const uint8_t *arena,
                                                 int jj, bool &q2) {
    q2 = false;
    if (sp.n_live > 0 && jj < sp.n_live) {
        const int e = live[jj];
        if (jj < sp.n_ring_q4) return ring + size_t(e) * KVQ_SLOT;
        if (jj < sp.n4) return arena + size_t(e - HCM_ARENA_BASE) * KVQ_SLOT;
        q2 = true;
        return ring + size_t(e) * KVQ_SLOT + KVQ2_OFF;
    }
    const int p = sp.n_live > 0 ? sp.rebuilt_at + (jj - sp.n_live) : jj;
    return ring + size_t(hcm_slot(p, sp.n_ctx)) * KVQ_SLOT;
}

// ------------------------------------------------------ q/k prep + append --
// One CTA (256 threads) per token: q_norm / k_norm (nn.c:2116-2137, v *=
// r * w with a double accumulator), IMROPE on dims (j, j+32), j < 32
// (rope_imrope, nn.c:841-861; cos/sin come from a host-built table so they
// equal the reference's libm values), the gate copy to z, and the append of
// K and V as q4 + q2 records into the ring slot (kv_append): the Q-Hitter
// score of the slot's previous contents first (kvq4_qf, kvq.c:84-100), then
// the new records (kvq4_quant / kvq2_quant, kvq.c:25-70), then the slot's
// salience in every layer reset to 0.
__global__ void __launch_bounds__(256) qk_prep_append_kernel(
    const float *__restrict__ proj, int proj_ld, const float *__restrict__ qn,
    const float *__restrict__ kn, const float *__restrict__ rope, const StepParams *spp,
    float *qr, float *z, uint8_t *kv, float *qf, float *sal) {
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ __align__(16) float hv[NHEAD + 2 * NHEAD_KV][HEAD_DIM];   // q heads, k heads, v heads
    __shared__ float qfv[4];
    pdl_wait();
    const StepParams sp = *spp;
    const int pos = sp.n_pos + t;
    const int slot = hcm_slot(pos, sp.n_ctx);
    const float *row = proj + size_t(t) * proj_ld;
    // norms: warp w handles vectors w, w + 8, w + 16 (16 q heads, 2 k heads)
    for (int v = warp; v < NHEAD + NHEAD_KV; v += 8) {
        const bool isq = v < NHEAD;
        const float *src = isq ? row + v * (2 * HEAD_DIM) : row + WQ_DIM + (v - NHEAD) * HEAD_DIM;
        const float *w = isq ? qn : kn;
        float x[8];
        double ss = 0.0;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            x[k] = src[lane * 8 + k];
            ss += double(x[k]) * double(x[k]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float r = 1.0f / sqrtf(float(ss / HEAD_DIM) + 1e-6f);
#pragma unroll
        for (int k = 0; k < 8; k++) hv[v][lane * 8 + k] = __fmul_rn(x[k], __fmul_rn(r, w[lane * 8 + k]));
        if (isq) {
#pragma unroll
            for (int k = 0; k < 8; k++)
                z[size_t(t) * WO_DIM + v * HEAD_DIM + lane * 8 + k] = row[v * (2 * HEAD_DIM) + HEAD_DIM + lane * 8 + k];
        }
    }
    // V heads (raw)
    for (int i = tid; i < NHEAD_KV * HEAD_DIM; i += 256)
        hv[NHEAD + NHEAD_KV + i / HEAD_DIM][i % HEAD_DIM] = row[WQ_DIM + WKV_DIM + i];
    __syncthreads();
    // IMROPE: 18 rotated vectors x 32 pairs
    const float *cs = rope + size_t(pos) * NROT;     // [32 cos][32 sin]
    for (int i = tid; i < (NHEAD + NHEAD_KV) * (NROT / 2); i += 256) {
        const int v = i / (NROT / 2), j = i % (NROT / 2);
        const float c = cs[j], s = cs[NROT / 2 + j];
        const float x0 = hv[v][j], x1 = hv[v][j + NROT / 2];
        hv[v][j] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        hv[v][j + NROT / 2] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    __syncthreads();
    for (int i = tid; i < NHEAD * HEAD_DIM; i += 256)
        qr[size_t(t) * NHEAD * HEAD_DIM + i] = hv[i / HEAD_DIM][i % HEAD_DIM];
    // Q-Hitter score of the slot's current q4 records vs the new K/V
    // (warps 0..3: K head 0, K head 1, V head 0, V head 1)
    if (warp < 4) {
        const int kh = warp & 1;
        const uint8_t *rec = kv + (size_t(warp >> 1) * NHEAD_KV + kh) * sp.n_ctx * KVQ_SLOT + size_t(slot) * KVQ_SLOT;
        const float *x = hv[NHEAD + warp];   // K0, K1, V0, V1 in that order
        double se = 0.0, sx = 0.0;
        for (int i = lane; i < HEAD_DIM; i += 32) {
            const int sb = i / 32, l = i % 32;
            const float d = h2f(uint16_t(rec[sb * 20] | (rec[sb * 20 + 1] << 8)));
            const float m = h2f(uint16_t(rec[sb * 20 + 2] | (rec[sb * 20 + 3] << 8)));
            const uint8_t b = rec[sb * 20 + 4 + l / 2];
            const int q = (l & 1) ? (b >> 4) : (b & 0xF);
            const float v = __fadd_rn(__fmul_rn(float(q), d), m);
            const float e = __fsub_rn(v, x[i]);
            se += double(e) * double(e);
            sx += double(x[i]) * double(x[i]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            se += __shfl_xor_sync(0xffffffffu, se, o);
            sx += __shfl_xor_sync(0xffffffffu, sx, o);
        }
        if (lane == 0) qfv[warp] = sx <= 0 ? 0.0f : float(sqrt(se / sx));
    }
    __syncthreads();
    if (tid == 0) {
        const float qk = __fadd_rn(qfv[0], qfv[1]), qv = __fadd_rn(qfv[2], qfv[3]);
        qf[slot] = __fadd_rn(qk, qv) / (2.0f * NHEAD_KV);
    }
    // new records: warp w < 4 writes record w (K0, K1, V0, V1).  Every
    // 20-byte sub-block is {fp16 d, fp16 m, 16 payload bytes}: the header and
    // the payload are packed in registers and stored as aligned 32-bit words
    // (slot, record and sub-block offsets are multiples of 4 bytes).
    if (warp < 4) {
        const int kh = warp & 1;
        uint8_t *rec = kv + (size_t(warp >> 1) * NHEAD_KV + kh) * sp.n_ctx * KVQ_SLOT + size_t(slot) * KVQ_SLOT;
        const float *x = hv[NHEAD + warp];
        // q4: 8 sub-blocks of 32 lanes, q = rint((x - mn) / d) in [0, 15];
        // value i is nibble (i & 1) of payload byte i / 2 (kvq.c:25-46)
        for (int sb = 0; sb < 8; sb++) {
            const float v = x[sb * 32 + lane];
            float mn = v, mx = v;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            }
            float d = __fsub_rn(mx, mn) / 15.0f;
            if (!(d > 0)) d = 1.0f;
            int q = __float2int_rn(__fsub_rn(v, mn) / d);
            q = q < 0 ? 0 : (q > 15 ? 15 : q);
            // payload word k holds values 8k .. 8k+7
            uint32_t w = uint32_t(q) << (4 * (lane & 7));
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) w |= __shfl_xor_sync(0xffffffffu, w, o);
            uint32_t *blk = reinterpret_cast<uint32_t *>(rec + sb * 20);
            if ((lane & 7) == 0) blk[1 + lane / 8] = w;
            if (lane == 0) blk[0] = uint32_t(f2h(d)) | (uint32_t(f2h(mn)) << 16);
        }
        // q2: 4 sub-blocks of 64, value i at bits 2 (i & 3) of payload byte
        // i / 4, OR-ed into the existing payload (kvq.c:50-70)
        for (int sb = 0; sb < 4; sb++) {
            const float v0 = x[sb * 64 + lane], v1 = x[sb * 64 + 32 + lane];
            float mn = fminf(v0, v1), mx = fmaxf(v0, v1);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            }
            float d = __fsub_rn(mx, mn) / 3.0f;
            if (!(d > 0)) d = 1.0f;
            int q0 = __float2int_rn(__fsub_rn(v0, mn) / d), q1 = __float2int_rn(__fsub_rn(v1, mn) / d);
            q0 = q0 < 0 ? 0 : (q0 > 3 ? 3 : q0);
            q1 = q1 < 0 ? 0 : (q1 > 3 ? 3 : q1);
            // payload word k holds values 16k .. 16k+15: v0 -> words 0, 1; v1 -> 2, 3
            uint32_t w0 = uint32_t(q0) << (2 * (lane & 15)), w1 = uint32_t(q1) << (2 * (lane & 15));
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) {
                w0 |= __shfl_xor_sync(0xffffffffu, w0, o);
                w1 |= __shfl_xor_sync(0xffffffffu, w1, o);
            }
            uint32_t *blk = reinterpret_cast<uint32_t *>(rec + KVQ2_OFF + sb * 20);
            if ((lane & 15) == 0) {
                blk[1 + lane / 16] |= w0;
                blk[3 + lane / 16] |= w1;
            }
            if (lane == 0) blk[0] = uint32_t(f2h(d)) | (uint32_t(f2h(mn)) << 16);
        }
    }
    if (tid < NATTN) sal[size_t(tid) * sp.n_ctx + slot] = 0.0f;
}

// --------------------------------------------------------------- scores --
// Q.K of every attended position for the 8 query heads of one KV head
// (GQA: kv head = q head / 8): one thread per (position, pair of heads),
// the record dequantized on the fly (kvq4_dot / kvq2_dot, kvq.c:183-213,
// keeping their 4-lane partial sums and pairwise reduction).
constexpr int SC_POS = 64;          // positions per scores CTA

__device__ __forceinline__ float rec_dot(const uint8_t *rec, bool q2, const float *q) {
    float acc = 0.0f;
    if (!q2) {
        for (int sb = 0; sb < 8; sb++) {
            const uint8_t *b = rec + sb * 20;
            const float d = h2f(uint16_t(b[0] | (b[1] << 8))), m = h2f(uint16_t(b[2] | (b[3] << 8)));
            float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int k = 0; k < 8; k++)
#pragma unroll
                for (int l = 0; l < 4; l++) {
                    const int i = 4 * k + l;
                    const uint8_t byte = b[4 + i / 2];
                    const int qv = (i & 1) ? (byte >> 4) : (byte & 0xF);
                    const float e = __fadd_rn(m, __fmul_rn(float(qv), d));
                    a[l] = __fadd_rn(a[l], __fmul_rn(e, q[sb * 32 + i]));
                }
            acc = __fadd_rn(acc, __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])));
        }
    } else {
        for (int sb = 0; sb < 4; sb++) {
            const uint8_t *b = rec + sb * 20;
            const float d = h2f(uint16_t(b[0] | (b[1] << 8))), m = h2f(uint16_t(b[2] | (b[3] << 8)));
            float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int k = 0; k < 16; k++)
#pragma unroll
                for (int l = 0; l < 4; l++) {
                    const int i = 4 * k + l;
                    const int qv = (b[4 + i / 4] >> (2 * (i & 3))) & 3;
                    const float e = __fadd_rn(m, __fmul_rn(float(qv), d));
                    a[l] = __fadd_rn(a[l], __fmul_rn(e, q[sb * 64 + i]));
                }
            acc = __fadd_rn(acc, __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])));
        }
    }
    return acc;
}

__global__ void __launch_bounds__(256) attn_scores_kernel(const float *__restrict__ qr,
                                                          const uint8_t *__restrict__ kv,
                                                          const uint8_t *__restrict__ arena,
                                                          const int *__restrict__ live,
                                                          const StepParams *spp, float *scores,
                                                          int nk_max, float *cmax, int nchunk) {
    const int chunk = blockIdx.x, kh = blockIdx.y, t = blockIdx.z;
    const int tid = threadIdx.x, pi = tid >> 2, hp = tid & 3;
    __shared__ __align__(16) float qs[8][HEAD_DIM];
    __shared__ float mred[SC_POS][8];
    pdl_wait();
    const StepParams sp = *spp;
    for (int i = tid; i < 8 * HEAD_DIM; i += 256)
        qs[i / HEAD_DIM][i % HEAD_DIM] = qr[(size_t(t) * NHEAD + kh * 8) * HEAD_DIM + i];
    __syncthreads();
    const int nk = nk_of(sp, t);
    const int jj = chunk * SC_POS + pi;
    float s0 = -INFINITY, s1 = -INFINITY;
    if (jj < nk) {
        bool q2;
        const uint8_t *rec = rec_of(sp, live, kv + size_t(kh) * sp.n_ctx * KVQ_SLOT,
                                    arena + size_t(kh) * HCM_H_PIN * KVQ_SLOT, jj, q2);
        const float scale = 1.0f / sqrtf(float(HEAD_DIM));
        s0 = __fmul_rn(rec_dot(rec, q2, qs[2 * hp]), scale);
        s1 = __fmul_rn(rec_dot(rec, q2, qs[2 * hp + 1]), scale);
        float *srow = scores + (size_t(t) * NHEAD + kh * 8 + 2 * hp) * nk_max;
        srow[jj] = s0;
        srow[nk_max + jj] = s1;
    }
    mred[pi][2 * hp] = s0;
    mred[pi][2 * hp + 1] = s1;
    __syncthreads();
    if (tid < 8) {
        float m = -INFINITY;
        for (int p = 0; p < SC_POS; p++) m = fmaxf(m, mred[p][tid]);
        cmax[(size_t(t) * NHEAD + kh * 8 + tid) * nchunk + chunk] = m;
    }
}

// -------------------------------------------------------- softmax . V -----
// Per (position chunk, KV head, query): p = expf(s - max) with the global
// max of the head, the chunk's sum of p, and the chunk's sum of p * V
// (kvq4_vacc / kvq2_vacc, kvq.c:215-241) for its 8 heads; one thread per
// output dimension.
__global__ void __launch_bounds__(256) attn_pv_kernel(const float *__restrict__ scores,
                                                      int nk_max, const float *__restrict__ cmax,
                                                      int nchunk_sc, const uint8_t *__restrict__ kv,
                                                      const uint8_t *__restrict__ arena,
                                                      const int *__restrict__ live,
                                                      const StepParams *spp, int chunk_pos,
                                                      float *opart, float *lpart, int nchunk) {
    const int chunk = blockIdx.x, kh = blockIdx.y, t = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ float M[8], pj[8][64];
    pdl_wait();
    const StepParams sp = *spp;
    const int nk = nk_of(sp, t);
    {   // warp h: global max of head kh*8 + h
        const float *cm = cmax + (size_t(t) * NHEAD + kh * 8 + warp) * nchunk_sc;
        float m = -INFINITY;
        for (int c = lane; c < nchunk_sc; c += 32) m = fmaxf(m, cm[c]);
        m = warp_max(m);
        if (lane == 0) M[warp] = m;
    }
    __syncthreads();
    const int j0 = chunk * chunk_pos, j1 = min(nk, j0 + chunk_pos);
    float acc[8], lsum = 0.0f;
#pragma unroll
    for (int h = 0; h < 8; h++) acc[h] = 0.0f;
    const uint8_t *ring = kv + size_t(NHEAD_KV + kh) * sp.n_ctx * KVQ_SLOT;
    const uint8_t *ar = arena + size_t(NHEAD_KV + kh) * HCM_H_PIN * KVQ_SLOT;
    const int d = tid;
    for (int b0 = j0; b0 < j1; b0 += 64) {
        const int bn = min(64, j1 - b0);
        __syncthreads();
        for (int i = tid; i < 8 * 64; i += 256) {
            const int h = i / 64, jj = i % 64;
            pj[h][jj] = jj < bn ? expf(scores[(size_t(t) * NHEAD + kh * 8 + h) * nk_max + b0 + jj] - M[h]) : 0.0f;
        }
        __syncthreads();
        if (warp == 0) {
            // sum of p over this block, per head (lane h)
            for (int h = 0; h < 8; h++) {
                float s = pj[h][lane] + pj[h][lane + 32];
                s = warp_sum(s);
                if (lane == h) lsum += s;
            }
        }
        for (int jj = 0; jj < bn; jj++) {
            bool q2;
            const uint8_t *rec = rec_of(sp, live, ring, ar, b0 + jj, q2);
            float v;
            if (!q2) {
                const uint8_t *b = rec + (d / 32) * 20;
                const float dd = h2f(uint16_t(b[0] | (b[1] << 8))), m = h2f(uint16_t(b[2] | (b[3] << 8)));
                const uint8_t byte = b[4 + (d % 32) / 2];
                const int qv = (d & 1) ? (byte >> 4) : (byte & 0xF);
                v = __fadd_rn(m, __fmul_rn(float(qv), dd));
            } else {
                const uint8_t *b = rec + (d / 64) * 20;
                const float dd = h2f(uint16_t(b[0] | (b[1] << 8))), m = h2f(uint16_t(b[2] | (b[3] << 8)));
                const int qv = (b[4 + (d % 64) / 4] >> (2 * (d & 3))) & 3;
                v = __fadd_rn(m, __fmul_rn(float(qv), dd));
            }
#pragma unroll
            for (int h = 0; h < 8; h++) acc[h] = __fadd_rn(acc[h], __fmul_rn(pj[h][jj], v));
        }
    }
#pragma unroll
    for (int h = 0; h < 8; h++)
        opart[((size_t(t) * NHEAD + kh * 8 + h) * nchunk + chunk) * HEAD_DIM + d] = acc[h];
    if (warp == 0 && lane < 8) lpart[(size_t(t) * NHEAD + kh * 8 + lane) * nchunk + chunk] = lsum;
}

// -------------------------------------- combine + sigmoid gate + Q8_K ----
// o = (sum of chunk partials) * (1 / sum of p) (nn.c:1410-1412), aout = o *
// sigmoid(gate) (nn.c:2157-2159), quantized for attn_output; also keeps the
// per-head max and sum of p for the salience update.
__global__ void __launch_bounds__(1024) attn_combine_kernel(const float *__restrict__ opart,
                                                            const float *__restrict__ lpart,
                                                            const float *__restrict__ cmax,
                                                            int nchunk_sc, int nchunk,
                                                            const float *__restrict__ z,
                                                            float *ml, int8_t *xq, float *xd,
                                                            int16_t *xs) {
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ float inv[NHEAD];
    __shared__ __align__(16) float y[WO_DIM];
    pdl_wait();
    if (warp < NHEAD) {
        const float *cm = cmax + (size_t(t) * NHEAD + warp) * nchunk_sc;
        const float *lp = lpart + (size_t(t) * NHEAD + warp) * nchunk;
        float m = -INFINITY, l = 0.0f;
        for (int c = lane; c < nchunk_sc; c += 32) m = fmaxf(m, cm[c]);
        for (int c = lane; c < nchunk; c += 32) l += lp[c];
        m = warp_max(m);
        l = warp_sum(l);
        if (lane == 0) {
            inv[warp] = 1.0f / l;
            ml[(size_t(t) * NHEAD + warp) * 2] = m;
            ml[(size_t(t) * NHEAD + warp) * 2 + 1] = l;
        }
    }
    __syncthreads();
    for (int i = tid; i < WO_DIM; i += 1024) {
        const int h = i / HEAD_DIM, d = i % HEAD_DIM;
        const float *op = opart + (size_t(t) * NHEAD + h) * nchunk * HEAD_DIM + d;
        float o = 0.0f;
        for (int c = 0; c < nchunk; c++) o += op[size_t(c) * HEAD_DIM];
        o = __fmul_rn(o, inv[h]);
        const float g = z[size_t(t) * WO_DIM + i];
        y[i] = __fmul_rn(o, 1.0f / (1.0f + expf(-g)));
    }
    __syncthreads();
    if (warp < WO_DIM / 256) {
        const float4 a = *reinterpret_cast<const float4 *>(y + warp * 256 + lane * 8);
        const float4 b = *reinterpret_cast<const float4 *>(y + warp * 256 + lane * 8 + 4);
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        q8k_block_warp(v, lane, xq + size_t(t) * WO_DIM + warp * 256, xd + size_t(t) * 16 + warp,
                       xs + size_t(t) * 256 + warp * 16);
    }
}

// -------------------------------------------------------------- salience --
// The salience EMA of attn_worker (nn.c:1414-1443): every attended position
// of the live index and tail gets sal = (1 - a) sal + a * p, heads in order
// 0..15 and within a head tokens in order, exactly as the single-threaded
// reference applies them.  Ring positions update sal[layer][slot]; arena
// entries update the arena's own salience.
__global__ void __launch_bounds__(256) attn_salience_kernel(const float *__restrict__ scores,
                                                            int nk_max, const float *__restrict__ ml,
                                                            const int *__restrict__ live,
                                                            const StepParams *spp, float *sal,
                                                            float *pin_sal) {
    const int jj = blockIdx.x * blockDim.x + threadIdx.x;
    pdl_wait();
    const StepParams sp = *spp;
    if (sp.n_live <= 0) return;
    const int nkmax = nk_of(sp, sp.T - 1);
    if (jj >= nkmax) return;
    float *dst;
    if (jj < sp.n_live) {
        const int e = live[jj];
        dst = (jj >= sp.n_ring_q4 && jj < sp.n4) ? pin_sal + (e - HCM_ARENA_BASE) : sal + e;
    } else {
        dst = sal + hcm_slot(sp.rebuilt_at + (jj - sp.n_live), sp.n_ctx);
    }
    const float keep = 1.0f - 0.05f, take = 0.05f;
    float s = *dst;
    for (int h = 0; h < NHEAD; h++)
        for (int t = 0; t < sp.T; t++) {
            if (jj >= nk_of(sp, t)) continue;
            const float m = ml[(size_t(t) * NHEAD + h) * 2], l = ml[(size_t(t) * NHEAD + h) * 2 + 1];
            const float p = expf(scores[(size_t(t) * NHEAD + h) * nk_max + jj] - m) / l;
            s = __fadd_rn(__fmul_rn(keep, s), __fmul_rn(take, p));
        }
    *dst = s;
}

// ------------------------------------------------------------ arena copy --
// hcm_rebuild's promotion of ring slots into the heavy-hitter arena
// (nn.c:1092-1104): per pair (src ring slot, dst arena index), the 240-byte
// slots of all 4 KV heads of every attention layer, and the ring salience.
__global__ void arena_copy_kernel(const int2 *pairs, int n, uint8_t *const *kv, uint8_t *const *arena,
                                  const float *sal, float *pin_sal, int n_ctx) {
    const int i = blockIdx.x;
    if (i >= n) return;
    const int src = pairs[i].x, dst = pairs[i].y;
    for (int k = threadIdx.x; k < NATTN * 2 * NHEAD_KV * (KVQ_SLOT / 16); k += blockDim.x) {
        const int l = k / (2 * NHEAD_KV * (KVQ_SLOT / 16));
        const int r = k % (2 * NHEAD_KV * (KVQ_SLOT / 16));
        const int kh = r / (KVQ_SLOT / 16), c = r % (KVQ_SLOT / 16);
        const uint4 *s = reinterpret_cast<const uint4 *>(kv[l] + (size_t(kh) * n_ctx + src) * KVQ_SLOT) + c;
        uint4 *d = reinterpret_cast<uint4 *>(arena[l] + (size_t(kh) * HCM_H_PIN + dst) * KVQ_SLOT) + c;
        *d = *s;
    }
    if (threadIdx.x < NATTN)
        pin_sal[threadIdx.x * HCM_H_PIN + dst] = sal[size_t(threadIdx.x) * n_ctx + src];
}

// -------------------------------------------------------------- launchers --
int launch_qk_prep_append(const float *proj, int proj_ld, const float *qn, const float *kn,
                          const float *rope, const StepParams *sp, int T, float *qr, float *z,
                          uint8_t *kv, float *qf, float *sal, cudaStream_t st) {
    qk_prep_append_kernel<<<T, 256, 0, st>>>(proj, proj_ld, qn, kn, rope, sp, qr, z, kv, qf, sal);
    QMA_CHECK_LAUNCH();
    return QMA_CUDA_OK;
}

int launch_attention(const AttnArgs &a, cudaStream_t st) {
    const int nchunk_sc = (a.nk_max + SC_POS - 1) / SC_POS;
    attn_scores_kernel<<<dim3(nchunk_sc, NHEAD_KV, a.T), 256, 0, st>>>(
        a.qr, a.kv, a.arena, a.live, a.sp, a.scores, a.nk_max, a.cmax, nchunk_sc);
    QMA_CHECK_LAUNCH();
    const int nchunk = (a.nk_max + a.pv_chunk - 1) / a.pv_chunk;
    attn_pv_kernel<<<dim3(nchunk, NHEAD_KV, a.T), 256, 0, st>>>(
        a.scores, a.nk_max, a.cmax, nchunk_sc, a.kv, a.arena, a.live, a.sp, a.pv_chunk, a.opart,
        a.lpart, nchunk);
    QMA_CHECK_LAUNCH();
    attn_combine_kernel<<<a.T, 1024, 0, st>>>(a.opart, a.lpart, a.cmax, nchunk_sc, nchunk, a.z,
                                              a.ml, a.xq, a.xd, a.xs);
    QMA_CHECK_LAUNCH();
    attn_salience_kernel<<<(a.nk_max + 255) / 256, 256, 0, st>>>(a.scores, a.nk_max, a.ml, a.live,
                                                                 a.sp, a.sal, a.pin_sal);
    QMA_CHECK_LAUNCH();
    return QMA_CUDA_OK;
}

int launch_arena_copy(const int2 *pairs, int n, uint8_t *const *kv, uint8_t *const *arena,
                      const float *sal, float *pin_sal, int n_ctx, cudaStream_t st) {
    if (n <= 0) return QMA_CUDA_OK;
    arena_copy_kernel<<<n, 256, 0, st>>>(pairs, n, kv, arena, sal, pin_sal, n_ctx);
    QMA_CHECK_LAUNCH();
    return QMA_CUDA_OK;
}

}  // namespace qma
