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
// Grid (T, 5), 128 threads; each warp owns one 256-wide head vector, lane l
// holding elements 8l .. 8l+7.  CTAs y = 0..3 handle query heads 4y .. 4y+3:
// q_norm (v *= r * w, r from a double sum of squares, nn.c:2116-2137), the
// IMROPE rotation of dims (j, j+32), j < 32 (rope_imrope, nn.c:841-861; the
// cos/sin table is built on the host with the reference's libm calls), and
// the copy of the head's gate half to z.  CTA y = 4 appends the token to the
// KV ring (kv_append, nn.c:1455-1509): warps 0, 1 normalise and rotate K
// heads 0, 1, warps 2, 3 take V heads 0, 1 raw; each warp scores its slot's
// old q4 record against the new vector (kvq4_qf, kvq.c:84-100), then writes
// the q4 and q2 records (kvq4_quant / kvq2_quant, kvq.c:25-70), and the
// slot's salience in every layer is reset to 0.
__device__ __forceinline__ void head_norm(float (&x)[8], const float (&wv)[8]) {
    double ss = 0.0;
#pragma unroll
    for (int k = 0; k < 8; k++) ss += double(x[k]) * double(x[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = 1.0f / sqrtf(float(ss / HEAD_DIM) + 1e-6f);
#pragma unroll
    for (int k = 0; k < 8; k++) x[k] = __fmul_rn(x[k], __fmul_rn(r, wv[k]));
}

// rotate pairs (j, j+32), j < 32: lanes 0..3 hold j, lanes 4..7 hold j+32;
// c / sn: the cos / sin of the lane's 8 pairs (lanes < 8)
__device__ __forceinline__ void head_rope(float (&x)[8], const float (&c)[8], const float (&sn)[8], int lane) {
    float y[8];
#pragma unroll
    for (int k = 0; k < 8; k++) y[k] = __shfl_xor_sync(0xffffffffu, x[k], 4);
    if (lane < 8) {
#pragma unroll
        for (int k = 0; k < 8; k++) {
            if (lane < 4) x[k] = __fsub_rn(__fmul_rn(x[k], c[k]), __fmul_rn(y[k], sn[k]));
            else x[k] = __fadd_rn(__fmul_rn(y[k], sn[k]), __fmul_rn(x[k], c[k]));
        }
    }
}

__device__ __forceinline__ void ld8(float (&x)[8], const float *p) {
    const float4 a = *reinterpret_cast<const float4 *>(p), b = *reinterpret_cast<const float4 *>(p + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
__device__ __forceinline__ void st8(float *p, const float (&x)[8]) {
    *reinterpret_cast<float4 *>(p) = make_float4(x[0], x[1], x[2], x[3]);
    *reinterpret_cast<float4 *>(p + 4) = make_float4(x[4], x[5], x[6], x[7]);
}

__global__ void __launch_bounds__(128) qk_prep_append_kernel(
    const float *__restrict__ proj, int proj_ld, const float *__restrict__ qn,
    const float *__restrict__ kn, const float *__restrict__ rope, const StepParams *spp,
    float *qr, float *z, uint8_t *kv, float *qf, float *sal, const AttnRow *rows) {
    QMA_TRACE_SCOPE(TK_QK_PREP);
    const int t = blockIdx.x, part = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (rows) {                 // one token of sequence row blockIdx.z
        const AttnRow &r = rows[blockIdx.z];
        proj = r.proj; rope = r.rope; spp = r.sp; qr = r.qr; z = r.z; kv = r.kv; qf = r.qf; sal = r.sal_all;
    }
    __shared__ float qfv[4];
    // Everything but the projection row was written before this step began
    // (step parameters, rope table, norm weights, the slot's old record):
    // read it before waiting on the input projection.
    const StepParams sp = *spp;
    const int pos = sp.n_pos + t;
    const int slot = hcm_slot(pos, sp.n_ctx);
    const float *cs = rope + size_t(pos) * NROT;     // [32 cos][32 sin]
    float wv[8], c[8], sn[8];
    if (part < 4 || warp < 2) {
        ld8(wv, (part < 4 ? qn : kn) + lane * 8);
        if (lane < 8) {
            ld8(c, cs + (lane & 3) * 8);
            ld8(sn, cs + NROT / 2 + (lane & 3) * 8);
        }
    }
    const int kh = warp & 1;
    uint8_t *rec = kv + (size_t(warp >> 1) * NHEAD_KV + kh) * sp.n_ctx * KVQ_SLOT + size_t(slot) * KVQ_SLOT;
    uint32_t old_hdr = 0, old_nw = 0;
    if (part == 4) {
        const uint32_t *sbw = reinterpret_cast<const uint32_t *>(rec + (lane >> 2) * 20);
        old_hdr = sbw[0];
        old_nw = sbw[1 + (lane & 3)];
    }
    pdl_trigger();
    pdl_wait();
    const float *row = proj + size_t(t) * proj_ld;
    float x[8];
    if (part < 4) {
        const int h = part * 4 + warp;
        ld8(x, row + h * (2 * HEAD_DIM) + lane * 8);
        head_norm(x, wv);
        head_rope(x, c, sn, lane);
        st8(qr + (size_t(t) * NHEAD + h) * HEAD_DIM + lane * 8, x);
        float g[8];
        ld8(g, row + h * (2 * HEAD_DIM) + HEAD_DIM + lane * 8);
        st8(z + size_t(t) * WO_DIM + h * HEAD_DIM + lane * 8, g);
        return;
    }
    // warp w: record w = K0, K1, V0, V1
    if (warp < 2) {
        ld8(x, row + WQ_DIM + kh * HEAD_DIM + lane * 8);
        head_norm(x, wv);
        head_rope(x, c, sn, lane);
    } else {
        ld8(x, row + WQ_DIM + WKV_DIM + kh * HEAD_DIM + lane * 8);
    }
    {   // Q-Hitter score of the slot's current q4 record against x (lane:
        // elements 8l .. 8l+7, sub-block l / 4)
        const uint32_t hdr = old_hdr, nw = old_nw;
        const float d = h2f(uint16_t(hdr & 0xffff)), m = h2f(uint16_t(hdr >> 16));
        double se = 0.0, sx = 0.0;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int q = (nw >> (4 * k)) & 0xF;
            const float v = __fadd_rn(__fmul_rn(float(q), d), m);
            const float e = __fsub_rn(v, x[k]);
            se += double(e) * double(e);
            sx += double(x[k]) * double(x[k]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            se += __shfl_xor_sync(0xffffffffu, se, o);
            sx += __shfl_xor_sync(0xffffffffu, sx, o);
        }
        if (lane == 0) qfv[warp] = sx <= 0 ? 0.0f : float(sqrt(se / sx));
    }
    // Every 20-byte sub-block is {fp16 d, fp16 m, 16 payload bytes}, packed
    // in registers and stored as aligned 32-bit words.
    // q4: 8 sub-blocks of 32; value i is nibble (i & 1) of payload byte i / 2.
    // Lane l holds values 8l .. 8l+7 = sub-block l / 4, payload word l % 4.
    {
        float mn = x[0], mx = x[0];
#pragma unroll
        for (int k = 1; k < 8; k++) { mn = fminf(mn, x[k]); mx = fmaxf(mx, x[k]); }
#pragma unroll
        for (int o = 1; o < 4; o <<= 1) {
            mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        float d = __fsub_rn(mx, mn) / 15.0f;
        if (!(d > 0)) d = 1.0f;
        uint32_t w = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            int q = __float2int_rn(__fsub_rn(x[k], mn) / d);
            q = q < 0 ? 0 : (q > 15 ? 15 : q);
            w |= uint32_t(q) << (4 * k);
        }
        uint32_t *blk = reinterpret_cast<uint32_t *>(rec + (lane >> 2) * 20);
        blk[1 + (lane & 3)] = w;
        if ((lane & 3) == 0) blk[0] = uint32_t(f2h(d)) | (uint32_t(f2h(mn)) << 16);
    }
    // q2: 4 sub-blocks of 64; value i at bits 2 (i & 3) of payload byte i / 4;
    // each payload word is assembled from a lane pair and stored whole.  Lane l: sub-block l / 8, values
    // 8 (l % 8) .. +7 = payload bytes 2 (l % 8), 2 (l % 8) + 1 = the half
    // (l % 2) of payload word (l % 8) / 2.
    {
        float mn = x[0], mx = x[0];
#pragma unroll
        for (int k = 1; k < 8; k++) { mn = fminf(mn, x[k]); mx = fmaxf(mx, x[k]); }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        float d = __fsub_rn(mx, mn) / 3.0f;
        if (!(d > 0)) d = 1.0f;
        uint32_t w = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            int q = __float2int_rn(__fsub_rn(x[k], mn) / d);
            q = q < 0 ? 0 : (q > 3 ? 3 : q);
            w |= uint32_t(q) << (2 * k);
        }
        w <<= 16 * (lane & 1);
        w |= __shfl_xor_sync(0xffffffffu, w, 1);
        uint32_t *blk = reinterpret_cast<uint32_t *>(rec + KVQ2_OFF + (lane >> 3) * 20);
        if ((lane & 1) == 0) blk[1 + ((lane & 7) >> 1)] = w;   // both halves: the whole word
        if ((lane & 7) == 0) blk[0] = uint32_t(f2h(d)) | (uint32_t(f2h(mn)) << 16);
    }
    __syncthreads();
    if (tid == 0) {
        const float qk = __fadd_rn(qfv[0], qfv[1]), qv = __fadd_rn(qfv[2], qfv[3]);
        qf[slot] = __fadd_rn(qk, qv) / (2.0f * NHEAD_KV);
    }
    if (tid < NATTN) sal[size_t(tid) * sp.n_ctx + slot] = 0.0f;
}

// ---------------------------------------------------- chunked attention ----
// Grid (ceil(nk_max / span), KV head, query t), 256 threads.  A CTA covers
// `span` attended positions of one KV head for its 8 query heads (GQA: KV
// head = query head / 8), in sub-chunks of up to SUB positions whose K and V
// records (q4: 160 B, q2: 80 B) are staged in shared memory with 16-byte
// loads.  The record arithmetic of kvq.c:183-241 is folded: a sub-block
// with scale d and offset m contributes d * sum(q_i x_i) + m * sum(x_i) to a
// score, and p * d * q + p * m to an output, so the quantized values enter
// as small integers (converted through the float exponent field) in fused
// multiply-adds.  This reassociates the reference's fp32 sums; the
// attention output agrees within fp32 rounding, not bit for bit.
//   scores : thread (position i, head quad hq) -> 4 heads;
//   softmax: warp h keeps the running max and sum of p = expf(s - max);
//   p . V  : thread = output dim, 8 heads; p * d per (position, head,
//            sub-block) precomputed in shared memory, sum p * m per
//            (head, sub-block) accumulated separately.
// Outputs: the raw scores (for the salience update) and per-CTA (max, sum,
// partial output).
constexpr int SUB = 128;

__device__ __forceinline__ float small2f(uint32_t v) {      // exact float of v < 2^23
    return __int_as_float(0x4B000000u | v) - 8388608.0f;
}

struct ChunkSmem {
    float qT[HEAD_DIM][8];          // query, element-major (8 heads contiguous)
    float X4[8][8], X2[8][4];       // query sums over 32- / 64-element sub-blocks
    uint4 kst[SUB][10], vst[SUB][10];
    const uint8_t *kp[SUB], *vp[SUB];
    int isq2[SUB];
    float ps[8][SUB];               // scores, then p
    float W[SUB][8][8];             // p * d of V record i, sub-block sb, head h: [i][sb][h]
    float U4[8][8], U2[8][4];       // sum p * m per head and q4 / q2 sub-block
    float scl[8];
};

__global__ void __launch_bounds__(256) attn_chunk_kernel(const float *__restrict__ qr,
                                                         const uint8_t *__restrict__ kv,
                                                         const uint8_t *__restrict__ arena,
                                                         const int *__restrict__ live,
                                                         const StepParams *spp, int nk_max,
                                                         int span, int nchunk, float *scores,
                                                         float *mpart, float *lpart, float *opart) {
    QMA_TRACE_SCOPE(TK_ATTN_CHUNK);
    extern __shared__ __align__(16) uint8_t chunk_raw[];
    ChunkSmem &S = *reinterpret_cast<ChunkSmem *>(chunk_raw);
    const int chunk = blockIdx.x, kh = blockIdx.y, t = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_trigger();
    pdl_wait();
    const StepParams sp = *spp;
    const int nk = nk_of(sp, t);
    const int j0 = chunk * span;
    if (j0 >= nk) return;
    const int j1 = min(nk, j0 + span);
    for (int i = tid; i < 8 * HEAD_DIM; i += 256) {
        const int h = i / HEAD_DIM, e = i % HEAD_DIM;
        S.qT[e][h] = qr[(size_t(t) * NHEAD + kh * 8) * HEAD_DIM + i];
    }
    {   // warp h: sub-block sums of query head h
        const float *q = qr + (size_t(t) * NHEAD + kh * 8 + warp) * HEAD_DIM;
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = q[lane + 32 * k];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const float x4 = warp_sum(v[k]);          // elements 32 k .. 32 k + 31
            if (lane == 0) S.X4[warp][k] = x4;
        }
        if (lane < 4) S.X2[warp][lane] = 0.0f;
        __syncwarp();
        if (lane == 0)
            for (int k = 0; k < 4; k++) S.X2[warp][k] = S.X4[warp][2 * k] + S.X4[warp][2 * k + 1];
        if (lane < 8) {
            S.U4[warp][lane] = 0.0f;
            if (lane < 4) S.U2[warp][lane] = 0.0f;
        }
    }
    const uint8_t *kring = kv + size_t(kh) * sp.n_ctx * KVQ_SLOT;
    const uint8_t *vring = kv + size_t(NHEAD_KV + kh) * sp.n_ctx * KVQ_SLOT;
    const uint8_t *kar = arena + size_t(kh) * HCM_H_PIN * KVQ_SLOT;
    const uint8_t *var = arena + size_t(NHEAD_KV + kh) * HCM_H_PIN * KVQ_SLOT;
    float m_run = -INFINITY, l_run = 0.0f;     // warp h: head h (lane-uniform)
    float acc[8];
#pragma unroll
    for (int h = 0; h < 8; h++) acc[h] = 0.0f;
    const int d = tid;
    for (int b0 = j0; b0 < j1; b0 += SUB) {
        const int bn = min(SUB, j1 - b0);
        __syncthreads();     // previous sub-chunk fully consumed; query sums ready
        if (tid < bn) {
            bool q2;
            S.kp[tid] = rec_of(sp, live, kring, kar, b0 + tid, q2);
            bool q2v;
            S.vp[tid] = rec_of(sp, live, vring, var, b0 + tid, q2v);
            S.isq2[tid] = q2;
        }
        __syncthreads();
        for (int idx = tid; idx < bn * 10; idx += 256) {
            const int i = idx / 10, wq = idx % 10;
            if (wq < (S.isq2[i] ? 5 : 10)) {
                S.kst[i][wq] = __ldg(reinterpret_cast<const uint4 *>(S.kp[i]) + wq);
                S.vst[i][wq] = __ldg(reinterpret_cast<const uint4 *>(S.vp[i]) + wq);
            }
        }
        __syncthreads();
        {   // scores: thread (position i, heads 4 hq .. 4 hq + 3)
            const int i = tid & (SUB - 1), hq = tid >> 7;
            float sc[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            if (i < bn) {
                const uint32_t *w = reinterpret_cast<const uint32_t *>(S.kst[i]);
                float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (!S.isq2[i]) {
#pragma unroll 2
                    for (int sb = 0; sb < 8; sb++) {
                        const uint32_t hdr = w[5 * sb];
                        const float dd = h2f(uint16_t(hdr & 0xffff)), mm = h2f(uint16_t(hdr >> 16));
                        float a4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                        for (int wi = 0; wi < 4; wi++) {
                            const uint32_t nw = w[5 * sb + 1 + wi];
#pragma unroll
                            for (int k = 0; k < 8; k++) {
                                const float qf = small2f((nw >> (4 * k)) & 0xFu);
                                const float4 x = *reinterpret_cast<const float4 *>(&S.qT[sb * 32 + wi * 8 + k][4 * hq]);
                                a4[0] = fmaf(qf, x.x, a4[0]);
                                a4[1] = fmaf(qf, x.y, a4[1]);
                                a4[2] = fmaf(qf, x.z, a4[2]);
                                a4[3] = fmaf(qf, x.w, a4[3]);
                            }
                        }
#pragma unroll
                        for (int h = 0; h < 4; h++) s4[h] = fmaf(mm, S.X4[4 * hq + h][sb], fmaf(dd, a4[h], s4[h]));
                    }
                } else {
#pragma unroll 1
                    for (int sb = 0; sb < 4; sb++) {
                        const uint32_t hdr = w[5 * sb];
                        const float dd = h2f(uint16_t(hdr & 0xffff)), mm = h2f(uint16_t(hdr >> 16));
                        float a4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                        for (int wi = 0; wi < 4; wi++) {
                            const uint32_t pw = w[5 * sb + 1 + wi];
#pragma unroll
                            for (int k = 0; k < 16; k++) {
                                const float qf = small2f((pw >> (2 * k)) & 3u);
                                const float4 x = *reinterpret_cast<const float4 *>(&S.qT[sb * 64 + wi * 16 + k][4 * hq]);
                                a4[0] = fmaf(qf, x.x, a4[0]);
                                a4[1] = fmaf(qf, x.y, a4[1]);
                                a4[2] = fmaf(qf, x.z, a4[2]);
                                a4[3] = fmaf(qf, x.w, a4[3]);
                            }
                        }
#pragma unroll
                        for (int h = 0; h < 4; h++) s4[h] = fmaf(mm, S.X2[4 * hq + h][sb], fmaf(dd, a4[h], s4[h]));
                    }
                }
#pragma unroll
                for (int h = 0; h < 4; h++) {
                    sc[h] = __fmul_rn(s4[h], 0.0625f);    // 1 / sqrtf(256)
                    scores[(size_t(t) * NHEAD + kh * 8 + 4 * hq + h) * nk_max + b0 + i] = sc[h];
                }
            }
#pragma unroll
            for (int h = 0; h < 4; h++) S.ps[4 * hq + h][i] = sc[h];
        }
        __syncthreads();
        {   // warp h: running max / sum of head h, p of this sub-chunk
            const int h = warp;
            float sv[SUB / 32];
            float mloc = -INFINITY;
#pragma unroll
            for (int k = 0; k < SUB / 32; k++) {
                sv[k] = S.ps[h][lane + 32 * k];
                mloc = fmaxf(mloc, sv[k]);
            }
            mloc = warp_max(mloc);
            const float m_new = fmaxf(m_run, mloc);
            float lsum = 0.0f;
#pragma unroll
            for (int k = 0; k < SUB / 32; k++) {
                const float p = lane + 32 * k < bn ? expf(sv[k] - m_new) : 0.0f;
                S.ps[h][lane + 32 * k] = p;
                lsum += p;
            }
            const float c = m_run == -INFINITY ? 0.0f : expf(m_run - m_new);
            l_run = __fadd_rn(__fmul_rn(l_run, c), warp_sum(lsum));
            m_run = m_new;
            if (lane == 0) S.scl[h] = c;
        }
        __syncthreads();
        // p * d per (position, sub-block, head); sum p * m per (head, sub-block)
        for (int e = tid; e < bn * 64; e += 256) {
            const int i = e >> 6, sb = (e >> 3) & 7, h = e & 7;
            float wv = 0.0f;
            if (!S.isq2[i] || sb < 4) {
                const uint32_t hdr = reinterpret_cast<const uint32_t *>(S.vst[i])[5 * sb];
                wv = __fmul_rn(S.ps[h][i], h2f(uint16_t(hdr & 0xffff)));
            }
            S.W[i][sb][h] = wv;
        }
        {   // thread (h, sb, quarter): a quarter of the positions, then a 4-lane sum
            const int h = tid >> 5, sb = (tid >> 2) & 7, qtr = tid & 3;
            float u4 = 0.0f, u2 = 0.0f;
            for (int i = qtr; i < bn; i += 4) {
                const uint32_t *w = reinterpret_cast<const uint32_t *>(S.vst[i]);
                if (!S.isq2[i]) u4 = fmaf(S.ps[h][i], h2f(uint16_t(w[5 * sb] >> 16)), u4);
                else if (sb < 4) u2 = fmaf(S.ps[h][i], h2f(uint16_t(w[5 * sb] >> 16)), u2);
            }
            u4 += __shfl_xor_sync(0xffffffffu, u4, 1);
            u4 += __shfl_xor_sync(0xffffffffu, u4, 2);
            u2 += __shfl_xor_sync(0xffffffffu, u2, 1);
            u2 += __shfl_xor_sync(0xffffffffu, u2, 2);
            if (qtr == 0) {
                S.U4[h][sb] = fmaf(S.U4[h][sb], S.scl[h], u4);
                if (sb < 4) S.U2[h][sb] = fmaf(S.U2[h][sb], S.scl[h], u2);
            }
        }
        __syncthreads();
        // p . V for output dim d (the q * (p d) part)
#pragma unroll
        for (int h = 0; h < 8; h++) acc[h] = __fmul_rn(acc[h], S.scl[h]);
        for (int i = 0; i < bn; i++) {
            const uint32_t *w = reinterpret_cast<const uint32_t *>(S.vst[i]);
            float qf;
            int sb;
            if (!S.isq2[i]) {
                sb = d >> 5;
                qf = small2f((w[5 * sb + 1 + ((d & 31) >> 3)] >> (4 * (d & 7))) & 0xFu);
            } else {
                sb = d >> 6;
                qf = small2f((w[5 * sb + 1 + ((d & 63) >> 4)] >> (2 * (d & 15))) & 3u);
            }
            const float4 wa = *reinterpret_cast<const float4 *>(&S.W[i][sb][0]);
            const float4 wb = *reinterpret_cast<const float4 *>(&S.W[i][sb][4]);
            acc[0] = fmaf(wa.x, qf, acc[0]);
            acc[1] = fmaf(wa.y, qf, acc[1]);
            acc[2] = fmaf(wa.z, qf, acc[2]);
            acc[3] = fmaf(wa.w, qf, acc[3]);
            acc[4] = fmaf(wb.x, qf, acc[4]);
            acc[5] = fmaf(wb.y, qf, acc[5]);
            acc[6] = fmaf(wb.z, qf, acc[6]);
            acc[7] = fmaf(wb.w, qf, acc[7]);
        }
    }
    __syncthreads();
    const size_t base = (size_t(t) * NHEAD + kh * 8) * nchunk + chunk;
#pragma unroll
    for (int h = 0; h < 8; h++)
        opart[(base + size_t(h) * nchunk) * HEAD_DIM + d] = acc[h] + S.U4[h][d >> 5] + S.U2[h][d >> 6];
    if (lane == 0) {
        mpart[base + size_t(warp) * nchunk] = m_run;
        lpart[base + size_t(warp) * nchunk] = l_run;
    }
}

// ------------------------------------------ single-token chunk attention --
// The decode form of attn_chunk_kernel (one query token, span <= 64), same
// outputs and the same folded record arithmetic, arranged for latency:
//   * the records of every position but the newest (the one this step's
//     qk_prep appends) are copied into shared memory before waiting on the
//     upstream kernel: the live index and the older records were written
//     before this step's first kernel started;
//   * scores: thread (position i = tid / 4, dim quarter tid % 4) takes 64
//     dims of all 8 query heads, then a 4-lane butterfly; the query rows are
//     stored at row e ^ ((e >> 6) & 3) so the four quarters read different
//     banks.
constexpr int DSPAN = 64;

struct DecSmem {
    float qT[HEAD_DIM][8];
    float X4[8][8], X2[8][4];
    uint4 kst[DSPAN][10], vst[DSPAN][10];
    int isq2[DSPAN];
    float ps[8][DSPAN];
    float W[DSPAN][8][8];
    float U4[8][8], U2[8][4];
};

__device__ __forceinline__ int qrow(int e) { return e ^ ((e >> 6) & 3); }

__global__ void __launch_bounds__(256) attn_decode_kernel(const float *__restrict__ qr,
                                                          const uint8_t *__restrict__ kv,
                                                          const uint8_t *__restrict__ arena,
                                                          const int *__restrict__ live,
                                                          const StepParams *spp, int nk_max,
                                                          int span, int nchunk, float *scores,
                                                          float *mpart, float *lpart, float *opart,
                                                          const AttnRow *rows) {
    QMA_TRACE_SCOPE(TK_ATTN_CHUNK);
    extern __shared__ __align__(16) uint8_t dec_raw[];
    DecSmem &S = *reinterpret_cast<DecSmem *>(dec_raw);
    const int chunk = blockIdx.x, kh = blockIdx.y;
    if (rows) {                 // sequence row blockIdx.z
        const AttnRow &r = rows[blockIdx.z];
        qr = r.qr; kv = r.kv; arena = r.arena; live = r.live; spp = r.sp; nk_max = r.nk_max; span = r.span;
        nchunk = r.nchunk; scores = r.scores; mpart = r.cmax; lpart = r.lpart; opart = r.opart;
    }
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const StepParams sp = *spp;                  // written before this step began
    const int nk = nk_of(sp, 0);
    const int j0 = chunk * span;
    if (j0 >= nk) {
        pdl_trigger();
        return;
    }
    const int bn = min(nk, j0 + span) - j0;
    const uint8_t *kring = kv + size_t(kh) * sp.n_ctx * KVQ_SLOT;
    const uint8_t *vring = kv + size_t(NHEAD_KV + kh) * sp.n_ctx * KVQ_SLOT;
    const uint8_t *kar = arena + size_t(kh) * HCM_H_PIN * KVQ_SLOT;
    const uint8_t *var = arena + size_t(NHEAD_KV + kh) * HCM_H_PIN * KVQ_SLOT;
    // the ring slot qk_prep rewrites in this step: a record in it is read
    // after the wait (the newest position, or an older one it overwrites)
    const uint8_t *knew = kring + size_t(hcm_slot(sp.n_pos, sp.n_ctx)) * KVQ_SLOT;
    // record words: thread (position i, word wq)
    for (int idx = tid; idx < bn * 10; idx += 256) {
        const int i = idx / 10, wq = idx % 10;
        bool q2, q2v;
        const uint8_t *kp = rec_of(sp, live, kring, kar, j0 + i, q2);
        const uint8_t *vp = rec_of(sp, live, vring, var, j0 + i, q2v);
        const bool late = kp == knew || kp == knew + KVQ2_OFF;
        if (wq == 0) S.isq2[i] = int(q2) | (late ? 2 : 0);
        if (!late && wq < (q2 ? 5 : 10)) {
            S.kst[i][wq] = __ldg(reinterpret_cast<const uint4 *>(kp) + wq);
            S.vst[i][wq] = __ldg(reinterpret_cast<const uint4 *>(vp) + wq);
        }
    }
    pdl_trigger();
    pdl_wait();
    // the query heads of this KV head (the upstream output), issued before
    // the late records so that both are in flight together: qt = dim tid of
    // head k, qv = dims lane + 32 k of head `warp`
    float qt[8], qv[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        qt[k] = qr[(size_t(kh) * 8) * HEAD_DIM + tid + HEAD_DIM * k];
        qv[k] = qr[(size_t(kh) * 8 + warp) * HEAD_DIM + lane + 32 * k];
    }
    __syncthreads();
    for (int idx = tid; idx < bn * 10; idx += 256) {
        const int i = idx / 10, wq = idx % 10;
        if (!(S.isq2[i] & 2)) continue;
        bool q2, q2v;
        const uint8_t *kp = rec_of(sp, live, kring, kar, j0 + i, q2);
        const uint8_t *vp = rec_of(sp, live, vring, var, j0 + i, q2v);
        if (wq < (q2 ? 5 : 10)) {
            S.kst[i][wq] = __ldcg(reinterpret_cast<const uint4 *>(kp) + wq);
            S.vst[i][wq] = __ldcg(reinterpret_cast<const uint4 *>(vp) + wq);
        }
    }
    __syncthreads();
    if (tid < bn) S.isq2[tid] &= 1;
#pragma unroll
    for (int k = 0; k < 8; k++) S.qT[qrow(tid)][k] = qt[k];
    {   // warp h: sub-block sums of query head h
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const float x4 = warp_sum(qv[k]);
            if (lane == 0) S.X4[warp][k] = x4;
        }
        __syncwarp();
        if (lane < 4) S.X2[warp][lane] = S.X4[warp][2 * lane] + S.X4[warp][2 * lane + 1];
    }
    __syncthreads();
    {   // scores: thread (position i, quarter qd) over dims 64 qd .. 64 qd + 63
        const int i = tid >> 2, qd = tid & 3;
        float s8[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        const bool live_i = i < bn;
        if (live_i) {
            const uint32_t *w = reinterpret_cast<const uint32_t *>(S.kst[i]);
            if (!S.isq2[i]) {
#pragma unroll
                for (int half = 0; half < 2; half++) {
                    const int sb = 2 * qd + half;
                    const uint32_t hdr = w[5 * sb];
                    const float dd = h2f(uint16_t(hdr & 0xffff)), mm = h2f(uint16_t(hdr >> 16));
                    float a8[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                    for (int wi = 0; wi < 4; wi++) {
                        const uint32_t nw = w[5 * sb + 1 + wi];
#pragma unroll
                        for (int k = 0; k < 8; k++) {
                            const float qf = small2f((nw >> (4 * k)) & 0xFu);
                            const float *x = S.qT[qrow(sb * 32 + wi * 8 + k)];
                            const float4 xa = *reinterpret_cast<const float4 *>(x);
                            const float4 xb = *reinterpret_cast<const float4 *>(x + 4);
                            a8[0] = fmaf(qf, xa.x, a8[0]); a8[1] = fmaf(qf, xa.y, a8[1]);
                            a8[2] = fmaf(qf, xa.z, a8[2]); a8[3] = fmaf(qf, xa.w, a8[3]);
                            a8[4] = fmaf(qf, xb.x, a8[4]); a8[5] = fmaf(qf, xb.y, a8[5]);
                            a8[6] = fmaf(qf, xb.z, a8[6]); a8[7] = fmaf(qf, xb.w, a8[7]);
                        }
                    }
#pragma unroll
                    for (int h = 0; h < 8; h++) s8[h] = fmaf(mm, S.X4[h][sb], fmaf(dd, a8[h], s8[h]));
                }
            } else {
                const int sb = qd;
                const uint32_t hdr = w[5 * sb];
                const float dd = h2f(uint16_t(hdr & 0xffff)), mm = h2f(uint16_t(hdr >> 16));
                float a8[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int wi = 0; wi < 4; wi++) {
                    const uint32_t pw = w[5 * sb + 1 + wi];
#pragma unroll
                    for (int k = 0; k < 16; k++) {
                        const float qf = small2f((pw >> (2 * k)) & 3u);
                        const float *x = S.qT[qrow(sb * 64 + wi * 16 + k)];
                        const float4 xa = *reinterpret_cast<const float4 *>(x);
                        const float4 xb = *reinterpret_cast<const float4 *>(x + 4);
                        a8[0] = fmaf(qf, xa.x, a8[0]); a8[1] = fmaf(qf, xa.y, a8[1]);
                        a8[2] = fmaf(qf, xa.z, a8[2]); a8[3] = fmaf(qf, xa.w, a8[3]);
                        a8[4] = fmaf(qf, xb.x, a8[4]); a8[5] = fmaf(qf, xb.y, a8[5]);
                        a8[6] = fmaf(qf, xb.z, a8[6]); a8[7] = fmaf(qf, xb.w, a8[7]);
                    }
                }
#pragma unroll
                for (int h = 0; h < 8; h++) s8[h] = fmaf(mm, S.X2[h][sb], fmaf(dd, a8[h], s8[h]));
            }
        }
#pragma unroll
        for (int h = 0; h < 8; h++) {
            s8[h] += __shfl_xor_sync(0xffffffffu, s8[h], 1);
            s8[h] += __shfl_xor_sync(0xffffffffu, s8[h], 2);
        }
#pragma unroll
        for (int h = 0; h < 8; h++) {
            if ((h >> 1) != qd) continue;               // lane qd keeps heads 2 qd, 2 qd + 1
            const float sc = live_i ? __fmul_rn(s8[h], 0.0625f) : -INFINITY;    // 1 / sqrtf(256)
            if (live_i) scores[(size_t(kh) * 8 + h) * nk_max + j0 + i] = sc;
            S.ps[h][i] = sc;
        }
    }
    __syncthreads();
    float m_h = -INFINITY, l_h = 0.0f;
    {   // warp h: max and sum of p = expf(s - max) of head h over the chunk
        const int h = warp;
        const float s0 = S.ps[h][lane], s1 = S.ps[h][lane + 32];
        m_h = warp_max(fmaxf(s0, s1));
        const float p0 = lane < bn ? expf(s0 - m_h) : 0.0f;
        const float p1 = lane + 32 < bn ? expf(s1 - m_h) : 0.0f;
        S.ps[h][lane] = p0;
        S.ps[h][lane + 32] = p1;
        l_h = warp_sum(p0 + p1);
    }
    __syncthreads();
    // p * d per (position, sub-block, head); sum p * m per (head, sub-block)
    for (int e = tid; e < bn * 64; e += 256) {
        const int i = e >> 6, sb = (e >> 3) & 7, h = e & 7;
        float wv = 0.0f;
        if (!S.isq2[i] || sb < 4) {
            const uint32_t hdr = reinterpret_cast<const uint32_t *>(S.vst[i])[5 * sb];
            wv = __fmul_rn(S.ps[h][i], h2f(uint16_t(hdr & 0xffff)));
        }
        S.W[i][sb][h] = wv;
    }
    {   // thread (h, sb, quarter): a quarter of the positions, then a 4-lane sum
        const int h = tid >> 5, sb = (tid >> 2) & 7, qtr = tid & 3;
        float u4 = 0.0f, u2 = 0.0f;
        for (int i = qtr; i < bn; i += 4) {
            const uint32_t *w = reinterpret_cast<const uint32_t *>(S.vst[i]);
            if (!S.isq2[i]) u4 = fmaf(S.ps[h][i], h2f(uint16_t(w[5 * sb] >> 16)), u4);
            else if (sb < 4) u2 = fmaf(S.ps[h][i], h2f(uint16_t(w[5 * sb] >> 16)), u2);
        }
        u4 += __shfl_xor_sync(0xffffffffu, u4, 1);
        u4 += __shfl_xor_sync(0xffffffffu, u4, 2);
        u2 += __shfl_xor_sync(0xffffffffu, u2, 1);
        u2 += __shfl_xor_sync(0xffffffffu, u2, 2);
        if (qtr == 0) {
            S.U4[h][sb] = u4;
            if (sb < 4) S.U2[h][sb] = u2;
        }
    }
    __syncthreads();
    // p . V for output dim d (the q * (p d) part)
    const int d = tid;
    float acc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    for (int i = 0; i < bn; i++) {
        const uint32_t *w = reinterpret_cast<const uint32_t *>(S.vst[i]);
        float qf;
        int sb;
        if (!S.isq2[i]) {
            sb = d >> 5;
            qf = small2f((w[5 * sb + 1 + ((d & 31) >> 3)] >> (4 * (d & 7))) & 0xFu);
        } else {
            sb = d >> 6;
            qf = small2f((w[5 * sb + 1 + ((d & 63) >> 4)] >> (2 * (d & 15))) & 3u);
        }
        const float4 wa = *reinterpret_cast<const float4 *>(&S.W[i][sb][0]);
        const float4 wb = *reinterpret_cast<const float4 *>(&S.W[i][sb][4]);
        acc[0] = fmaf(wa.x, qf, acc[0]);
        acc[1] = fmaf(wa.y, qf, acc[1]);
        acc[2] = fmaf(wa.z, qf, acc[2]);
        acc[3] = fmaf(wa.w, qf, acc[3]);
        acc[4] = fmaf(wb.x, qf, acc[4]);
        acc[5] = fmaf(wb.y, qf, acc[5]);
        acc[6] = fmaf(wb.z, qf, acc[6]);
        acc[7] = fmaf(wb.w, qf, acc[7]);
    }
    const size_t base = (size_t(kh) * 8) * nchunk + chunk;
#pragma unroll
    for (int h = 0; h < 8; h++)
        opart[(base + size_t(h) * nchunk) * HEAD_DIM + d] = acc[h] + S.U4[h][d >> 5] + S.U2[h][d >> 6];
    if (lane == 0) {
        mpart[base + size_t(warp) * nchunk] = m_h;
        lpart[base + size_t(warp) * nchunk] = l_h;
    }
}

// -------------------------------------- combine + sigmoid gate + Q8_K ----
// One CTA per (query head h, query t), thread = output dim: M = max of the
// chunk maxima, f_c = expf(m_c - M), L = sum f_c l_c, o = (sum_c f_c o_c) *
// (1 / L) (the softmax of attn_worker, nn.c:1340-1412), aout = o *
// sigmoid(gate) (nn.c:2157-2159) and its Q8_K block (the head's 256 dims
// are one block); (M, L) are kept for the salience update.
__global__ void __launch_bounds__(256) attn_combine_kernel(const float *__restrict__ opart,
                                                           const float *__restrict__ mpart,
                                                           const float *__restrict__ lpart,
                                                           const StepParams *spp, int span,
                                                           int nchunk, const float *__restrict__ z,
                                                           float *ml, int8_t *xq, float *xd,
                                                           int16_t *xs, const AttnRow *rows) {
    QMA_TRACE_SCOPE(TK_ATTN_COMBINE);
    extern __shared__ float fsh[];              // [nchunk] chunk factors of this head
    const int h = blockIdx.x, t = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (rows) {                 // sequence row blockIdx.z
        const AttnRow &r = rows[blockIdx.z];
        opart = r.opart; mpart = r.cmax; lpart = r.lpart; spp = r.sp; span = r.span; nchunk = r.nchunk; z = r.z;
        ml = r.ml; xq = r.xq; xd = r.xd; xs = r.xs;
    }
    __shared__ float wred[8], wsum[8];
    __shared__ __align__(16) float y[HEAD_DIM];
    const StepParams sp = *spp;                  // written before this step began
    const int nc = (nk_of(sp, t) + span - 1) / span;
    const size_t base = (size_t(t) * NHEAD + h) * nchunk;
    pdl_trigger();
    pdl_wait();
    // one round trip for the gate lane and the first chunk's maximum and sum
    // of this thread (chunks past 256 are read in the loops)
    const float g = z[size_t(t) * WO_DIM + h * HEAD_DIM + tid];
    const float m0 = tid < nc ? mpart[base + tid] : -INFINITY;
    const float l0 = tid < nc ? lpart[base + tid] : 0.0f;
    float m = m0;
    for (int c = tid + 256; c < nc; c += 256) m = fmaxf(m, mpart[base + c]);
    m = warp_max(m);
    if (lane == 0) wred[warp] = m;
    __syncthreads();
    m = wred[0];
#pragma unroll
    for (int w = 1; w < 8; w++) m = fmaxf(m, wred[w]);
    float l = 0.0f;
    for (int c = tid; c < nc; c += 256) {
        const float f = expf((c == tid ? m0 : mpart[base + c]) - m);
        fsh[c] = f;
        l = __fadd_rn(l, __fmul_rn(f, c == tid ? l0 : lpart[base + c]));
    }
    l = warp_sum(l);
    if (lane == 0) wsum[warp] = l;
    __syncthreads();
    l = ((wsum[0] + wsum[1]) + (wsum[2] + wsum[3])) + ((wsum[4] + wsum[5]) + (wsum[6] + wsum[7]));
    if (tid == 0) {
        ml[(size_t(t) * NHEAD + h) * 2] = m;
        ml[(size_t(t) * NHEAD + h) * 2 + 1] = l;
    }
    const float *op = opart + base * HEAD_DIM + tid;
    float o = 0.0f;
    for (int c = 0; c < nc; c++) o = __fadd_rn(o, __fmul_rn(fsh[c], op[size_t(c) * HEAD_DIM]));
    o = __fmul_rn(o, 1.0f / l);
    y[tid] = __fmul_rn(o, 1.0f / (1.0f + expf(-g)));
    __syncthreads();
    if (warp == 0) {
        const float4 a = *reinterpret_cast<const float4 *>(y + lane * 8);
        const float4 b = *reinterpret_cast<const float4 *>(y + lane * 8 + 4);
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        q8k_block_warp(v, lane, xq + size_t(t) * WO_DIM + h * 256, xd + size_t(t) * 16 + h,
                       xs + size_t(t) * 256 + h * 16);
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
                                                            float *pin_sal, const AttnRow *rows) {
    QMA_TRACE_SCOPE(TK_SALIENCE);
    const int jj = blockIdx.x * blockDim.x + threadIdx.x;
    if (rows) {                 // sequence row blockIdx.z
        const AttnRow &r = rows[blockIdx.z];
        scores = r.scores; nk_max = r.nk_max; ml = r.ml; live = r.live; spp = r.sp; sal = r.sal;
        pin_sal = r.pin_sal;
    }
    pdl_trigger();
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

// The same EMA for a chunk of T > 1 queries.  Per position the 16 * T
// updates are sequential (head-major, then query: the order above), but
// their probabilities are not: a CTA takes 32 positions, its warps 1..7
// compute the probabilities of the next (head, 64 queries) tile into shared
// memory while warp 0 (lane = position) runs the EMA over the current one.
constexpr int SAL_POS = 32, SAL_TQ = 64;

__global__ void __launch_bounds__(256) attn_salience_chunk_kernel(const float *__restrict__ scores, int nk_max,
                                                                  const float *__restrict__ ml,
                                                                  const int *__restrict__ live,
                                                                  const StepParams *spp, float *sal,
                                                                  float *pin_sal) {
    QMA_TRACE_SCOPE(TK_SALIENCE);
    __shared__ float P[2][SAL_TQ][SAL_POS];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int jj0 = blockIdx.x * SAL_POS;
    pdl_trigger();
    pdl_wait();
    const StepParams sp = *spp;
    if (sp.n_live <= 0) return;
    const int nk0 = nk_of(sp, 0), nkmax = nk_of(sp, sp.T - 1);
    if (jj0 >= nkmax) return;                      // CTA-uniform
    const int T = sp.T, ntq = (T + SAL_TQ - 1) / SAL_TQ, ntile = NHEAD * ntq;
    // tile i = (head i / ntq, queries 64 (i % ntq) ..): probabilities of the
    // 32 positions, computed by `nthr` threads starting at thread `first`
    auto fill = [&](int i, int first, int nthr) {
        const int h = i / ntq, t0 = (i % ntq) * SAL_TQ;
        float(*dst)[SAL_POS] = P[i & 1];
        for (int k = tid - first; k < SAL_TQ * SAL_POS; k += nthr) {
            const int tq = k / SAL_POS, pos = k % SAL_POS, t = t0 + tq, jj = jj0 + pos;
            float p = 0.0f;
            if (t < T && jj < nk_of(sp, t)) {
                const float m = ml[(size_t(t) * NHEAD + h) * 2], l = ml[(size_t(t) * NHEAD + h) * 2 + 1];
                p = expf(scores[(size_t(t) * NHEAD + h) * nk_max + jj] - m) / l;
            }
            dst[tq][pos] = p;
        }
    };
    fill(0, 0, 256);
    __syncthreads();
    const int jj = jj0 + lane;
    float *dst = nullptr;
    float s = 0.0f;
    if (warp == 0 && jj < nkmax) {
        if (jj < sp.n_live) {
            const int e = live[jj];
            dst = (jj >= sp.n_ring_q4 && jj < sp.n4) ? pin_sal + (e - HCM_ARENA_BASE) : sal + e;
        } else {
            dst = sal + hcm_slot(sp.rebuilt_at + (jj - sp.n_live), sp.n_ctx);
        }
        s = *dst;
    }
    // first query that attends position jj (positions of this chunk's own
    // tokens are attended from their token on)
    const int tmin = jj < nk0 ? 0 : jj - nk0 + 1;
    const float keep = 1.0f - 0.05f, take = 0.05f;
    for (int i = 0; i < ntile; i++) {
        if (warp == 0) {
            if (dst) {
                const int t0 = (i % ntq) * SAL_TQ, nq = min(SAL_TQ, T - t0);
                const float(*src)[SAL_POS] = P[i & 1];
                for (int tq = 0; tq < nq; tq++)
                    if (t0 + tq >= tmin) s = __fadd_rn(__fmul_rn(keep, s), __fmul_rn(take, src[tq][lane]));
            }
        } else if (i + 1 < ntile) {
            fill(i + 1, 32, 224);
        }
        __syncthreads();
    }
    if (dst) *dst = s;
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
    QMA_CHECK_CUDA(launch_ex(qk_prep_append_kernel, dim3(T, 5), dim3(128), 0, st, 1, pdl_enabled(), proj, proj_ld, qn, kn,
                             rope, sp, qr, z, kv, qf, sal, static_cast<const AttnRow *>(nullptr)));
    QMA_CHECK_LAUNCH();
    return QMA_CUDA_OK;
}

int launch_attention(const AttnArgs &a, cudaStream_t st) {
    const int nchunk = (a.nk_max + a.pv_chunk - 1) / a.pv_chunk;
    static PerDevice attr;
    if (!attr.done()) {
        QMA_CHECK_CUDA(cudaFuncSetAttribute(attn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            int(sizeof(ChunkSmem))));
        QMA_CHECK_CUDA(cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            int(sizeof(DecSmem))));
        attr.mark();
    }
    // QMA_CUDA_ATTN_GENERAL=1: single tokens through the multi-query kernel
    // (a cross-check of the decode kernel; same results up to fp32 rounding)
    static_assert(DSPAN <= 256, "decode spans fit the multi-query kernel's chunk");
    const char *gen = getenv("QMA_CUDA_ATTN_GENERAL");
    if (a.T == 1 && a.pv_chunk <= DSPAN && !(gen && atoi(gen) != 0))
        QMA_CHECK_CUDA(launch_ex(attn_decode_kernel, dim3(nchunk, NHEAD_KV), dim3(256), sizeof(DecSmem), st, 1,
                                 pdl_enabled(), a.qr, a.kv, a.arena, a.live, a.sp, a.nk_max, a.pv_chunk, nchunk,
                                 a.scores, a.cmax, a.lpart, a.opart, static_cast<const AttnRow *>(nullptr)));
    else
        QMA_CHECK_CUDA(launch_ex(attn_chunk_kernel, dim3(nchunk, NHEAD_KV, a.T), dim3(256), sizeof(ChunkSmem), st, 1,
                                 pdl_enabled(), a.qr, a.kv, a.arena, a.live, a.sp, a.nk_max, a.pv_chunk, nchunk,
                                 a.scores, a.cmax, a.lpart, a.opart));
    QMA_CHECK_LAUNCH();
    const size_t fsh = sizeof(float) * size_t(nchunk);
    if (fsh > 48 * 1024) {
        set_error("attention: %d position chunks exceed the combine kernel's shared memory", nchunk);
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
    QMA_CHECK_CUDA(launch_ex(attn_combine_kernel, dim3(NHEAD, a.T), dim3(256), fsh, st, 1, pdl_enabled(), a.opart,
                             a.cmax, a.lpart, a.sp, a.pv_chunk, nchunk, a.z, a.ml, a.xq, a.xd, a.xs,
                             static_cast<const AttnRow *>(nullptr)));
    return QMA_CUDA_OK;
}

int launch_salience(const AttnArgs &a, cudaStream_t st) {
    if (a.T > 1)
        QMA_CHECK_CUDA(launch_ex(attn_salience_chunk_kernel, dim3((a.nk_max + SAL_POS - 1) / SAL_POS), dim3(256), 0,
                                 st, 1, false, a.scores, a.nk_max, a.ml, a.live, a.sp, a.sal, a.pin_sal));
    else
        QMA_CHECK_CUDA(launch_ex(attn_salience_kernel, dim3((a.nk_max + 255) / 256), dim3(256), 0, st, 1, false,
                                 a.scores, a.nk_max, a.ml, a.live, a.sp, a.sal, a.pin_sal,
                                 static_cast<const AttnRow *>(nullptr)));
    return QMA_CUDA_OK;
}

int launch_attention_rows(const AttnRow *rows, int n, int proj_ld, const float *qn, const float *kn, int max_nchunk,
                          int max_nk, cudaStream_t st) {
    static PerDevice attr;
    if (!attr.done()) {
        QMA_CHECK_CUDA(cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            int(sizeof(DecSmem))));
        attr.mark();
    }
    const size_t fsh = sizeof(float) * size_t(max_nchunk);
    if (fsh > 48 * 1024) {
        set_error("attention: %d position chunks exceed the combine kernel's shared memory", max_nchunk);
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
    const StepParams *nsp = nullptr;
    const float *nf = nullptr;
    float *nw = nullptr;
    QMA_CHECK_CUDA(launch_ex(qk_prep_append_kernel, dim3(1, 5, n), dim3(128), 0, st, 1, pdl_enabled(), nf, proj_ld,
                             qn, kn, nf, nsp, nw, nw, static_cast<uint8_t *>(nullptr), nw, nw, rows));
    QMA_CHECK_CUDA(launch_ex(attn_decode_kernel, dim3(max_nchunk, NHEAD_KV, n), dim3(256), sizeof(DecSmem), st, 1,
                             pdl_enabled(), nf, static_cast<const uint8_t *>(nullptr),
                             static_cast<const uint8_t *>(nullptr), static_cast<const int *>(nullptr), nsp, 0, 1, 1,
                             nw, nw, nw, nw, rows));
    QMA_CHECK_CUDA(launch_ex(attn_combine_kernel, dim3(NHEAD, 1, n), dim3(256), fsh, st, 1, pdl_enabled(), nf, nf, nf,
                             nsp, 1, 1, nf, nw, static_cast<int8_t *>(nullptr), nw, static_cast<int16_t *>(nullptr),
                             rows));
    QMA_CHECK_CUDA(launch_ex(attn_salience_kernel, dim3((max_nk + 255) / 256, 1, n), dim3(256), 0, st, 1, false, nf,
                             0, nf, static_cast<const int *>(nullptr), nsp, nw, nw, rows));
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
