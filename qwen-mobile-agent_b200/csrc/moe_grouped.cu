// moe_grouped.cu -- the MoE FFN block for a chunk of tokens (prefill), with
// the (token, expert) pairs grouped by expert so that each expert's weights
// are read once per chunk and its tokens share int8 tensor-core MMAs.
//
// Same arithmetic as the per-token expert kernel (moe_expert_one_q8k
// nn.c:412-439, moe_shared_q8k nn.c:446-473): the integer sub-block partials
// sum(q * xq) are exact (mma.sync s8 x s8 -> s32), folded with the
// sub-block scales in integer registers; each super-block adds
// xd * (d * I1 - dmin * I2) (Q4_K) or d * xd * I (Q6_K) in fp32.  After the
// router (moe_router_kernel), per chunk:
//   1. moe_lists_kernel   : pair ids t * 8 + k grouped by expert, in token order;
//   2. moe_gateup_kernel  : gate and up rows of every expert for its tokens
//                           (the shared expert takes every token);
//   3. moe_swiglu_kernel  : silu(gate) * up and its Q8_K per pair;
//   4. moe_down_kernel    : down rows per expert, into the per-slot partials;
//   5. moe_combine_norm_kernel (moe.cu) combines the slots.
#include <algorithm>

#include "common.cuh"
#include "gemv.cuh"
#include "moe.cuh"
#include "quant.cuh"
#include "tc.cuh"

namespace qma {

constexpr int GT = BT_COLS;     // tokens (pairs) per CTA tile: 4 MMA column tiles of 8
constexpr int GR = 64;          // rows per CTA: 4 warps x 16
constexpr int NSHARED = MOE_NEXP;   // group index of the shared expert

// 1. ---------------------------------------------------------------- lists --
// One CTA over the chunk's T x 8 (token, expert) pairs, one pair per thread
// at a time: shared-memory atomics count each expert's pairs, an exclusive
// scan (thread e = expert e) gives the offsets, then the pairs are placed in
// rounds of 256 in token order -- a pair's rank among the earlier pairs of
// its expert is the expert's count in earlier rounds, plus its count in the
// lower warps of this round, plus the pair's rank among the matching lanes
// of its own warp (__match_any_sync).  The experts that have pairs are also
// listed compactly (goff[257] = their number, then their ids ascending) so
// that the expert kernels launch no CTA for the others.  A pair with no
// expert (-1: the padding of an expert-parallel exchange) is not listed.
__global__ void __launch_bounds__(256) moe_lists_kernel(const int *__restrict__ sel, int T, int *goff,
                                                        int *plist) {
    __shared__ int ssel[MOE_GROUPED_MAX_T * MOE_TOPK];
    __shared__ int cnt[MOE_NEXP], run[MOE_NEXP];
    __shared__ int wc[8][MOE_NEXP];     // this round's count of expert e in warp w
    __shared__ int wsum[8], wact[8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    cnt[tid] = 0;
    run[tid] = 0;
#pragma unroll
    for (int w = 0; w < 8; w++) wc[w][tid] = 0;
    pdl_trigger();
    pdl_wait();
    const int np = T * MOE_TOPK;
    __syncthreads();
    for (int p = tid; p < np; p += 256) ssel[p] = sel[p];   // loads all in flight
    __syncthreads();
    for (int p = tid; p < np; p += 256) {
        const int e = ssel[p];
        if (e >= 0) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    const int c = cnt[tid];
    // exclusive scan of the 256 counts
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    const unsigned am = __ballot_sync(0xffffffffu, c > 0);
    if (lane == 0) wact[warp] = __popc(am);
    __syncthreads();
    int base = 0, abase = 0;
    for (int w = 0; w < warp; w++) {
        base += wsum[w];
        abase += wact[w];
    }
    const int off = base + incl - c;
    goff[tid] = off;
    if (tid == 255) goff[256] = off + c;
    // the active experts, ascending: the rank of e among them
    int *act = goff + MOE_NEXP + 1;
    if (c > 0) act[1 + abase + __popc(am & ((1u << lane) - 1u))] = tid;
    if (tid == 255) act[0] = abase + __popc(am);
    cnt[tid] = off;                     // from here on: the offsets
    __syncthreads();
    for (int p0 = 0; p0 < np; p0 += 256) {
        const int p = p0 + tid;
        const int e = p < np ? ssel[p] : -1;
        // lanes without an expert match nothing (a key of their own)
        const unsigned m = __match_any_sync(0xffffffffu, e >= 0 ? e : -1 - lane);
        const int lr = __popc(m & ((1u << lane) - 1u));
        if (e >= 0 && lr == 0) wc[warp][e] = __popc(m);
        __syncthreads();
        if (e >= 0) {
            int pre = run[e];
            for (int w = 0; w < warp; w++) pre += wc[w][e];
            plist[cnt[e] + pre + lr] = p;
        }
        __syncthreads();
        int add = 0;
#pragma unroll
        for (int w = 0; w < 8; w++) {
            add += wc[w][tid];
            wc[w][tid] = 0;
        }
        run[tid] += add;
        __syncthreads();
    }
}

// The group of grid row y of an expert kernel: rows below nyr take the
// active routed experts in order (-1 past the last), the row after them the
// shared expert.
__device__ __forceinline__ int group_of_row(int y, int nyr, const int *goff) {
    if (y >= nyr) return NSHARED;
    const int *act = goff + MOE_NEXP + 1;
    return y < act[0] ? act[1 + y] : -1;
}

// The pair slot of tile column tk of group e: routed pairs t * 8 + k, the
// shared expert's T * 8 + t.
__device__ __forceinline__ int pair_of(int e, int tk, int T, const int *goff, const int *plist) {
    return e < NSHARED ? plist[goff[e] + tk] : T * MOE_TOPK + tk;
}
__device__ __forceinline__ int group_size(int e, int T, const int *goff) {
    return e < NSHARED ? goff[e + 1] - goff[e] : T;
}

// One lane's share of super-block sb of two Q4_K rows (rows gid and gid + 8
// of a warp's 16): each row's 16-byte header and the quant words
// 16 + 32 g + 4 tig and 32 + 32 g + 4 tig (g = 0..3), the A fragments of
// the 8 sub-blocks.
struct Q4Words {
    uint4 h0, h1;
    uint32_t q0[8], q1[8];
    __device__ __forceinline__ void load(const uint8_t *w0, const uint8_t *w1, int sb, int tig) {
        const uint8_t *b0 = w0 + size_t(sb) * Q4K_BYTES, *b1 = w1 + size_t(sb) * Q4K_BYTES;
        h0 = __ldg(reinterpret_cast<const uint4 *>(b0));
        h1 = __ldg(reinterpret_cast<const uint4 *>(b1));
#pragma unroll
        for (int g = 0; g < 4; g++) {
            q0[2 * g] = __ldg(reinterpret_cast<const uint32_t *>(b0 + 16 + 32 * g + 4 * tig));
            q0[2 * g + 1] = __ldg(reinterpret_cast<const uint32_t *>(b0 + 32 + 32 * g + 4 * tig));
            q1[2 * g] = __ldg(reinterpret_cast<const uint32_t *>(b1 + 16 + 32 * g + 4 * tig));
            q1[2 * g + 1] = __ldg(reinterpret_cast<const uint32_t *>(b1 + 32 + 32 * g + 4 * tig));
        }
    }
};

// q4k_scales8 on the header's scale words (bytes 4..15 of the block)
__device__ __forceinline__ void q4k_scales8_words(uint32_t w0, uint32_t w1, uint32_t w2, int (&sc)[8],
                                                  int (&mn)[8]) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t a = (w0 >> (8 * j)) & 0xffu, b = (w1 >> (8 * j)) & 0xffu, c = (w2 >> (8 * j)) & 0xffu;
        sc[j] = int(a & 63u);
        mn[j] = int(b & 63u);
        sc[j + 4] = int((c & 15u) | ((a >> 6) << 4));
        mn[j + 4] = int((c >> 4) | ((b >> 6) << 4));
    }
}

// 2. ---------------------------------------------------------- gate / up --
// Grid (1024 / GR rows of [gate | up], 257 groups, ceil(T / GT) tiles); warp
// w: 16 rows, 4 column tiles of 8 pairs.  Output hg[pair][1024].
__global__ void __launch_bounds__(128, 4) moe_gateup_kernel(const uint8_t *__restrict__ gate_exps,
                                                         const uint8_t *__restrict__ up_exps,
                                                         const uint8_t *__restrict__ gate_sh,
                                                         const uint8_t *__restrict__ up_sh, int T,
                                                         MoeScratch s, int nyr) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, tig = lane & 3;
    const int tok0 = blockIdx.z * GT;
    __shared__ __align__(16) int8_t bt[2][BT_COLS][BT_STRIDE];
    __shared__ int brow[BT_COLS];
    pdl_trigger();
    pdl_wait();
    const int e = group_of_row(int(blockIdx.y), nyr, s.goff);
    if (e < 0) return;                                   // CTA-uniform: no more active experts
    const int ne = group_size(e, T, s.goff);
    if (tok0 >= ne) return;                              // CTA-uniform
    if (threadIdx.x < BT_COLS) {
        const int tk = tok0 + int(threadIdx.x);
        brow[threadIdx.x] = tk < ne ? (e < NSHARED ? pair_of(e, tk, T, s.goff, s.plist) / MOE_TOPK : tk) : -1;
    }
    const int r = blockIdx.x * GR + warp * 16;          // row of [gate | up]
    constexpr size_t RB = size_t(MOE_EMBD / 256) * Q4K_BYTES;
    const uint8_t *W = r < MOE_FF ? (e < NSHARED ? gate_exps + size_t(e) * MOE_FF * RB : gate_sh)
                                  : (e < NSHARED ? up_exps + size_t(e) * MOE_FF * RB : up_sh);
    const int wr = r < MOE_FF ? r : r - MOE_FF;
    const uint8_t *w0 = W + size_t(wr + gid) * RB, *w1 = w0 + 8 * RB;
    // pair of accumulator columns 2 tig, 2 tig + 1 of each tile
    int pc[4][2];
#pragma unroll
    for (int n = 0; n < 4; n++) {
#pragma unroll
        for (int c = 0; c < 2; c++) {
            const int tc = tok0 + 8 * n + 2 * tig + c;
            pc[n][c] = tc < ne ? pair_of(e, tc, T, s.goff, s.plist) : -1;
        }
    }
    float acc[4][4];
#pragma unroll
    for (int n = 0; n < 4; n++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[n][i] = 0.0f;
    // the two rows' words of super-block sb: the 16-byte header (d, dmin,
    // 12 scale bytes) and this lane's 8 quant words; the next super-block's
    // are loaded before this one's activation tile is staged, so their HBM
    // latency overlaps the staging and the MMAs
    Q4Words cur, nxt;
    cur.load(w0, w1, 0, tig);
    // activation tiles double-buffered: tile sb + 1 is copied while sb's MMAs run
    __syncthreads();                                     // brow
    stage_btile_async(bt[0], brow, s.xq, MOE_EMBD, 0);
    for (int sb = 0; sb < MOE_EMBD / 256; sb++) {
        if (sb + 1 < MOE_EMBD / 256) nxt.load(w0, w1, sb + 1, tig);
        __syncthreads();                                 // the tile of sb - 1 is consumed
        if (sb + 1 < MOE_EMBD / 256) {
            stage_btile_async(bt[(sb + 1) & 1], brow, s.xq, MOE_EMBD, (sb + 1) * 256);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();                                 // tile sb is in shared memory
        const int8_t(*bt_)[BT_STRIDE] = bt[sb & 1];
        int sc0[8], mn0[8], sc1[8], mn1[8];
        q4k_scales8_words(cur.h0.y, cur.h0.z, cur.h0.w, sc0, mn0);
        q4k_scales8_words(cur.h1.y, cur.h1.z, cur.h1.w, sc1, mn1);
        const float d0 = h2f(uint16_t(cur.h0.x & 0xffffu)), dm0 = h2f(uint16_t(cur.h0.x >> 16));
        const float d1 = h2f(uint16_t(cur.h1.x & 0xffffu)), dm1 = h2f(uint16_t(cur.h1.x >> 16));
        int I1[4][4];
#pragma unroll
        for (int n = 0; n < 4; n++)
#pragma unroll
            for (int i = 0; i < 4; i++) I1[n][i] = 0;
#pragma unroll
        for (int g = 0; g < 4; g++) {
            const uint32_t r0a = cur.q0[2 * g], r0b = cur.q0[2 * g + 1];
            const uint32_t r1a = cur.q1[2 * g], r1b = cur.q1[2 * g + 1];
#pragma unroll
            for (int half = 0; half < 2; half++) {
                const int j = 2 * g + half, sh = 4 * half;
                const uint32_t a[4] = {(r0a >> sh) & 0x0f0f0f0fu, (r1a >> sh) & 0x0f0f0f0fu,
                                       (r0b >> sh) & 0x0f0f0f0fu, (r1b >> sh) & 0x0f0f0f0fu};
#pragma unroll
                for (int n = 0; n < 4; n++) {
                    const int8_t *bp = &bt_[8 * n + gid][32 * j + 4 * tig];
                    const uint32_t b0 = *reinterpret_cast<const uint32_t *>(bp);
                    const uint32_t b1 = *reinterpret_cast<const uint32_t *>(bp + 16);
                    int p[4] = {0, 0, 0, 0};
                    mma_s8(p, a, b0, b1);
                    I1[n][0] += sc0[j] * p[0];
                    I1[n][1] += sc0[j] * p[1];
                    I1[n][2] += sc1[j] * p[2];
                    I1[n][3] += sc1[j] * p[3];
                }
            }
        }
        int md0[4], md1[4];
        q4k_mins_dup(mn0, md0);
        q4k_mins_dup(mn1, md1);
#pragma unroll
        for (int n = 0; n < 4; n++)
#pragma unroll
            for (int c = 0; c < 2; c++) {
                if (pc[n][c] < 0) continue;
                const int t = pc[n][c] < T * MOE_TOPK ? pc[n][c] / MOE_TOPK : pc[n][c] - T * MOE_TOPK;
                const int16_t *bs = s.xs + size_t(t) * (MOE_EMBD / 16) + sb * 16;
                const int I2a = q4k_i2(bs, md0), I2b = q4k_i2(bs, md1);
                const float x = s.xd[size_t(t) * (MOE_EMBD / 256) + sb];
                acc[n][c] = q4k_fold(acc[n][c], x, d0, dm0, I1[n][c], I2a);
                acc[n][2 + c] = q4k_fold(acc[n][2 + c], x, d1, dm1, I1[n][2 + c], I2b);
            }
        cur = nxt;
    }
#pragma unroll
    for (int n = 0; n < 4; n++)
#pragma unroll
        for (int c = 0; c < 2; c++) {
            if (pc[n][c] < 0) continue;
            float *o = s.hg + size_t(pc[n][c]) * (2 * MOE_FF) + r + gid;
            o[0] = acc[n][c];
            o[8] = acc[n][2 + c];
        }
}

// 3. -------------------------------------------------------- SwiGLU + Q8_K --
// One CTA per pair slot, warp b: hidden block b of silu(gate) * up.
__global__ void __launch_bounds__(64) moe_swiglu_kernel(MoeScratch s, int q0) {
    const int q = q0 + int(blockIdx.x), lane = threadIdx.x & 31, b = threadIdx.x >> 5;
    pdl_trigger();
    pdl_wait();
    const float *h = s.hg + size_t(q) * (2 * MOE_FF);
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int i = b * 256 + lane * 8 + k;
        const float g = h[i], u = h[MOE_FF + i];
        v[k] = (g / (1.0f + expf(-g))) * u;
    }
    q8k_block_warp(v, lane, s.hq + size_t(q) * MOE_FF + b * 256, s.hd + size_t(q) * 2 + b,
                   s.hs + size_t(q) * (MOE_FF / 16) + b * 16);
}

// 4. ---------------------------------------------------------------- down --
// Q6_K down rows (2048 x 512, planes with swizzled ql / qh chunks) of every
// group for its pairs: m16n8k16 MMAs, one per 16-element sub-block with its
// int8 scale.  Grid (2048 / GR, 257, tiles); output part[t][slot][row].
__global__ void __launch_bounds__(128) moe_down_kernel(const uint8_t *__restrict__ down_exps, size_t down_bytes,
                                                       const uint8_t *__restrict__ down_sh, int T,
                                                       MoeScratch s, int nyr) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, tig = lane & 3;
    const int tok0 = blockIdx.z * GT;
    __shared__ __align__(16) int8_t bt[2][BT_COLS][BT_STRIDE];
    __shared__ int brow[BT_COLS];
    pdl_trigger();
    pdl_wait();
    const int e = group_of_row(int(blockIdx.y), nyr, s.goff);
    if (e < 0) return;                                   // CTA-uniform: no more active experts
    const int ne = group_size(e, T, s.goff);
    if (tok0 >= ne) return;                              // CTA-uniform
    if (threadIdx.x < BT_COLS) {
        const int tk = tok0 + int(threadIdx.x);
        brow[threadIdx.x] = tk < ne ? pair_of(e, tk, T, s.goff, s.plist) : -1;
    }
    constexpr int N = MOE_FF, NSB = N / 256;
    const int r0 = blockIdx.x * GR + warp * 16 + gid;   // rows r0 and r0 + 8
    const Q6Planes P = q6_planes(e < NSHARED ? down_exps + size_t(e) * down_bytes : down_sh, MOE_EMBD, N);
    int pc[4][2];
#pragma unroll
    for (int n = 0; n < 4; n++) {
#pragma unroll
        for (int c = 0; c < 2; c++) {
            const int tc = tok0 + 8 * n + 2 * tig + c;
            pc[n][c] = tc < ne ? pair_of(e, tc, T, s.goff, s.plist) : -1;
        }
    }
    float acc[4][4];
#pragma unroll
    for (int n = 0; n < 4; n++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[n][i] = 0.0f;
    __syncthreads();                                     // brow
    stage_btile_async(bt[0], brow, s.hq, N, 0);
    for (int sb = 0; sb < NSB; sb++) {
        __syncthreads();                                 // the tile of sb - 1 is consumed
        if (sb + 1 < NSB) {
            stage_btile_async(bt[(sb + 1) & 1], brow, s.hq, N, (sb + 1) * 256);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();                                 // tile sb is in shared memory
        const int8_t(*bt_)[BT_STRIDE] = bt[sb & 1];
        int I[4][4];
#pragma unroll
        for (int n = 0; n < 4; n++)
#pragma unroll
            for (int i = 0; i < 4; i++) I[n][i] = 0;
#pragma unroll 4
        for (int g = 0; g < 16; g++) {
            // elements 16 g + 4 tig .. + 3 of super-block sb: quad i of unit j
            const int j = g >> 3, i = 4 * (g & 7) + tig;
            const int hi = i >> 4, shift = 2 * (((i >> 3) & 1) + 2 * hi);
            const int qi = i & 15, hq = i & 7;
            uint32_t a[2];
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const int row = r0 + 8 * rr;
                const int seg = row * NSB + sb;
                const int cl = 4 * j + (qi >> 2), ch = 2 * j + (hq >> 2);
                const uint32_t lw = *reinterpret_cast<const uint32_t *>(
                    P.ql + size_t(row) * (N / 2) + sb * 128 + (q6_ql_chunk(cl, seg) << 4) + 4 * (qi & 3));
                const uint32_t hw = *reinterpret_cast<const uint32_t *>(
                    P.qh + size_t(row) * (N / 4) + sb * 64 + (q6_qh_chunk(ch, seg) << 4) + 4 * (hq & 3));
                const uint32_t v = ((lw >> (4 * hi)) & 0x0f0f0f0fu) | (((hw >> shift) & 0x03030303u) << 4);
                a[rr] = __vsub4(v, 0x20202020u);
            }
            const int sc0 = P.sc[size_t(r0) * (N / 16) + sb * 16 + g];
            const int sc1 = P.sc[size_t(r0 + 8) * (N / 16) + sb * 16 + g];
#pragma unroll
            for (int n = 0; n < 4; n++) {
                const uint32_t b0 = *reinterpret_cast<const uint32_t *>(&bt_[8 * n + gid][16 * g + 4 * tig]);
                int p[4] = {0, 0, 0, 0};
                mma_s8_k16(p, a[0], a[1], b0);
                I[n][0] += sc0 * p[0];
                I[n][1] += sc0 * p[1];
                I[n][2] += sc1 * p[2];
                I[n][3] += sc1 * p[3];
            }
        }
        const float d0 = __half2float(P.d[size_t(r0) * NSB + sb]), d1 = __half2float(P.d[size_t(r0 + 8) * NSB + sb]);
#pragma unroll
        for (int n = 0; n < 4; n++)
#pragma unroll
            for (int c = 0; c < 2; c++) {
                if (pc[n][c] < 0) continue;
                const float x = s.hd[size_t(pc[n][c]) * NSB + sb];
                acc[n][c] = q6k_fold(acc[n][c], x, d0, I[n][c]);
                acc[n][2 + c] = q6k_fold(acc[n][2 + c], x, d1, I[n][2 + c]);
            }
    }
#pragma unroll
    for (int n = 0; n < 4; n++)
#pragma unroll
        for (int c = 0; c < 2; c++) {
            const int q = pc[n][c];
            if (q < 0) continue;
            const int t = q < T * MOE_TOPK ? q / MOE_TOPK : q - T * MOE_TOPK;
            const int slot = q < T * MOE_TOPK ? q % MOE_TOPK : MOE_TOPK;
            float *o = s.part + (size_t(t) * MOE_NSLOT + slot) * MOE_EMBD + r0;
            o[0] = acc[n][c];
            o[8] = acc[n][2 + c];
        }
}

int moe_grouped_range(const qma_cuda_moe_weights &w, int T, const MoeScratch &s, cudaStream_t st, int g0, int ng,
                      bool lists, int q0, int nq) {
    const bool pdl = pdl_enabled();
    const int tiles = (T + GT - 1) / GT;
    if (lists)
        QMA_CHECK_CUDA(launch_ex(moe_lists_kernel, dim3(1), dim3(256), 0, st, 1, pdl, s.sel, T, s.goff, s.plist));
    // grid rows: the routed groups of [g0, g0 + ng) through the active-expert
    // list (at most one per pair), then the shared expert if in range
    const int nr = g0 < NSHARED ? std::min(g0 + ng, NSHARED) - g0 : 0;
    const int nyr = std::min(nr, T * MOE_TOPK);
    const int ny = nyr + (g0 + ng > NSHARED ? 1 : 0);
    if (nr > 0 && g0 != 0) {
        set_error("grouped experts: routed groups must start at expert 0 (got %d)", g0);
        return QMA_CUDA_ERR_INVALID;
    }
    if (!tc_grouped()) {
        QMA_CHECK_CUDA(launch_ex(moe_gateup_kernel, dim3(2 * MOE_FF / GR, ny, tiles), dim3(128), 0, st, 1, pdl,
                                 static_cast<const uint8_t *>(w.gate_exps), static_cast<const uint8_t *>(w.up_exps),
                                 static_cast<const uint8_t *>(w.gate_shexp), static_cast<const uint8_t *>(w.up_shexp),
                                 T, s, nyr));
    } else {
        const int rc = launch_gateup_tc(w, T, s, st, g0, ng);
        if (rc) return rc;
    }
    QMA_CHECK_CUDA(launch_ex(moe_swiglu_kernel, dim3(nq), dim3(64), 0, st, 1, pdl, s, q0));
    QMA_CHECK_CUDA(launch_ex(moe_down_kernel, dim3(MOE_EMBD / GR, ny, tiles), dim3(128), 0, st, 1, pdl,
                             static_cast<const uint8_t *>(w.down_exps), packed_bytes(w.down_type, MOE_EMBD, MOE_FF),
                             static_cast<const uint8_t *>(w.down_shexp), T, s, nyr));
    return QMA_CUDA_OK;
}

int moe_grouped(const qma_cuda_moe_weights &w, int T, const MoeScratch &s, cudaStream_t st) {
    return moe_grouped_range(w, T, s, st, 0, NSHARED + 1, true, 0, T * MOE_NSLOT);
}

}  // namespace qma
