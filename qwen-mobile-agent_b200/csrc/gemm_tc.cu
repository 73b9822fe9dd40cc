// gemm_tc.cu -- several tokens against Q4_K rows (prefill chunks of the
// dense projections) on the 5th-generation tensor cores: tcgen05 int8 MMAs
// accumulating in tensor memory (TMEM).
//
// Same result as gemm_q4k_mma_kernel (gemv.cu), bit for bit: out[t][r] =
// sum over super-blocks of xd * (d * I1 - dmin * I2) folded by q4k_fold in
// super-block order, with the exact integer sums I1 = sum_j sc_j sum_{k in j}
// q_k x_k and I2 = sum_j m_j bsum_j of dot_q4_K_q8k (q8k.c:89-131).  The
// tensor core forms I1 with the sub-block scale folded into the weight,
// a_k = q_k * sc_j = 32 hi_k + lo_k (both digits int8): one
// tcgen05.mma.kind::i8 of M = 128 rows x N = 128 tokens x K = 32 per
// (sub-block, digit), accumulating H = sum hi x and L = sum lo x over the
// super-block in int32 (exact), I1 = 32 H + L.
//
// CTA (416 threads) = 128 rows x tn tokens, tn = 128, 64 or 32 chosen per
// launch (the narrowest that keeps the grid within one wave of CTAs, so a
// projection with few row tiles still spreads over the SMs; N = 32 / 64
// MMAs when the tile holds at most that many tokens), the super-blocks in
// order as a three-stage pipeline over two buffers of every operand:
//   warps 0-3 (producers, thread = row): the tokens' Q8_K slice (B, by
//     16-byte asynchronous copies, in flight while the rest is formed),
//     their 32-lane sums and scales, and the super-block's Q4_K block ->
//     nibbles x scale -> two digit tiles (canonical K-major A);
//   warp 4, one lane: the 16 MMAs of the super-block into one of two TMEM
//     buffers (2 x 256 columns), then a commit;
//   warps 5-12 (epilogue, thread = row of its TMEM lane quarter, half of
//     the tile's tokens): the super-block's H and L from TMEM, the mins and
//     the fp32 fold into up to 64 register accumulators.
// The producer of super-block sb + 1 overlaps the MMAs of sb and the
// epilogue of sb - 1; it reuses the buffers of sb - 1 once the MMAs and the
// epilogue of sb - 1 are done with them.  Every wait is a bounded mbarrier
// wait.
#include "common.cuh"
#include "gemv.cuh"
#include "tc.cuh"

namespace qma {

constexpr int GTM = 128, GTN = 128;            // rows x tokens per CTA
constexpr uint32_t GT_TILE_A = GTM * 32, GT_TILE_B = GTN * 32;
constexpr uint32_t GT_TMEM_COLS = 512;         // two buffers of 2 digits x 128 tokens
constexpr int GT_THREADS = 416;               // 4 producer warps, 1 MMA warp, 8 epilogue warps
constexpr int GT_EPI = 256;                   // epilogue threads

struct GemmTcSmem {
    uint8_t a[2][2][8][GT_TILE_A];             // [buffer][digit][sub-block]           (128 KB)
    uint8_t b[2][8][GT_TILE_B];                // [buffer][sub-block]                  (64 KB)
    int16_t bsum[2][GTN][8];                   // [buffer][token][sub-block]: 32-lane sums (|s| <= 4064)
    float xd[2][GTN];
};
constexpr size_t GEMM_TC_SMEM = sizeof(GemmTcSmem);

// Bounded waits of this kernel that ran out (read and reset by the host).
__device__ unsigned g_gemm_tc_timeouts;

__device__ __forceinline__ bool gt_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_wait(bar, parity)) return true;
    if ((threadIdx.x & 31) == 0) atomicAdd(&g_gemm_tc_timeouts, 1u);
    return false;
}

// nibbles (one per byte, 0..15) x scale -> the digits hi = v >> 5, lo = v & 31
__device__ __forceinline__ void gt_digits(uint32_t n, uint32_t sc, uint32_t &hi, uint32_t &lo) {
    const uint32_t pe = (n & 0x00FF00FFu) * sc, po = ((n >> 8) & 0x00FF00FFu) * sc;
    hi = ((pe >> 5) & 0x001F001Fu) | (((po >> 5) & 0x001F001Fu) << 8);
    lo = (pe & 0x001F001Fu) | ((po & 0x001F001Fu) << 8);
}

__device__ __forceinline__ void gt_scales(uint32_t w0, uint32_t w1, uint32_t w2, int (&sc)[8], int (&mn)[8]) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t a = (w0 >> (8 * j)) & 0xffu, b = (w1 >> (8 * j)) & 0xffu, c = (w2 >> (8 * j)) & 0xffu;
        sc[j] = int(a & 63u);
        mn[j] = int(b & 63u);
        sc[j + 4] = int((c & 15u) | ((a >> 6) << 4));
        mn[j + 4] = int((c >> 4) | ((b >> 6) << 4));
    }
}

// Grid (ceil(n_out / 128), ceil(T / tn)), tn in {32, 64, 128}.  One CTA per
// SM, 128 registers a thread (13 warps, allocated as 16, fill the register
// file).
__global__ void __launch_bounds__(GT_THREADS, 1) gemm_q4k_tc_kernel(const uint8_t *__restrict__ W, int n_in,
                                                                   int n_out, int T, int tn,
                                                                   const int8_t *__restrict__ xq,
                                                                   const float *__restrict__ xd,
                                                                   const int16_t *__restrict__ xsum, float *out,
                                                                   const float *resid) {
    QMA_TRACE_SCOPE(TK_GEMV);
    extern __shared__ __align__(128) uint8_t gtsm_raw[];
    GemmTcSmem &S = *reinterpret_cast<GemmTcSmem *>(gtsm_raw);
    __shared__ __align__(8) uint64_t bar_a[2], bar_mma[2], bar_epi[2];
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r0 = blockIdx.x * GTM, t0 = blockIdx.y * tn;
    const int nsb = n_in / 256;
    const size_t RB = size_t(nsb) * Q4K_BYTES;
    pdl_trigger();
    pdl_wait();
    if (warp == 0) tmem_alloc(&tmem_base, GT_TMEM_COLS);
    if (tid == 0) {
        mbar_init(&bar_a[0], 128);
        mbar_init(&bar_a[1], 128);
        mbar_init(&bar_mma[0], 1);
        mbar_init(&bar_mma[1], 1);
        mbar_init(&bar_epi[0], GT_EPI);
        mbar_init(&bar_epi[1], GT_EPI);
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    if (warp < 4) {
        // ---- producers ------------------------------------------------------------
        const int m = tid, r = r0 + m;
        const bool live = r < n_out;
        const uint4 *row = reinterpret_cast<const uint4 *>(W + size_t(live ? r : 0) * RB);
        uint4 cur[9], nxt[9];
#pragma unroll
        for (int k = 0; k < 9; k++) cur[k] = live ? __ldg(row + k) : make_uint4(0, 0, 0, 0);
        for (int sb = 0; sb < nsb; sb++) {
            const int buf = sb & 1;
            if (sb + 1 < nsb) {
#pragma unroll
                for (int k = 0; k < 9; k++) nxt[k] = live ? __ldg(row + 9 * (sb + 1) + k) : make_uint4(0, 0, 0, 0);
            }
            // buffer `buf` (A, B) is free once the MMAs of sb - 2 completed, its
            // sums and scales once the epilogue of sb - 2 is done with them
            if (sb >= 2) {
                gt_wait(&bar_mma[buf], uint32_t(((sb - 2) >> 1) & 1));
                gt_wait(&bar_epi[buf], uint32_t(((sb - 2) >> 1) & 1));
            }
            // B: token m of the tile (the first tn producers take one token
            // each): its 256 Q8_K values by asynchronous copies straight into
            // the canonical layout (zeros past T), its sums and scale into
            // registers, all in flight while the weight digits are formed
            const int t = t0 + m;
            const bool tb = m < tn, tv = tb && t < T;
            int4 bu = make_int4(0, 0, 0, 0), bw = make_int4(0, 0, 0, 0);
            float xs = 0.0f;
            if (tb) {
                const int8_t *src = xq + size_t(tv ? t : 0) * n_in + sb * 256;
#pragma unroll
                for (int c = 0; c < 16; c++)
                    cp_async16(&S.b[buf][c >> 1][tc_off(m, 16 * (c & 1))], src + 16 * c, tv);
                if (tv) {
                    const int4 *bs = reinterpret_cast<const int4 *>(xsum + size_t(t) * (n_in / 16) + sb * 16);
                    bu = __ldg(bs);
                    bw = __ldg(bs + 1);
                    xs = xd[size_t(t) * nsb + sb];
                }
            }
            cp_async_commit();
            int sc[8], mn[8];
            gt_scales(cur[0].y, cur[0].z, cur[0].w, sc, mn);
#pragma unroll
            for (int g = 0; g < 4; g++) {
#pragma unroll
                for (int kc = 0; kc < 2; kc++) {
                    const uint4 q = cur[1 + 2 * g + kc];
                    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int half = 0; half < 2; half++) {
                        const int j = 2 * g + half;
                        uint32_t hi[4], lo[4];
#pragma unroll
                        for (int c = 0; c < 4; c++)
                            gt_digits((w[c] >> (4 * half)) & 0x0F0F0F0Fu, uint32_t(sc[j]), hi[c], lo[c]);
                        *reinterpret_cast<uint4 *>(&S.a[buf][0][j][tc_off(m, 16 * kc)]) =
                            make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        *reinterpret_cast<uint4 *>(&S.a[buf][1][j][tc_off(m, 16 * kc)]) =
                            make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    }
                }
            }
            if (tb) {
                // the token's sixteen 16-lane sums -> eight 32-lane sums, one store
                const int w[8] = {bu.x, bu.y, bu.z, bu.w, bw.x, bw.y, bw.z, bw.w};
                uint32_t pk[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int s0 = int(int16_t(w[2 * i] & 0xffff)) + (w[2 * i] >> 16);
                    const int s1 = int(int16_t(w[2 * i + 1] & 0xffff)) + (w[2 * i + 1] >> 16);
                    pk[i] = (uint32_t(s0) & 0xffffu) | (uint32_t(s1) << 16);
                }
                *reinterpret_cast<int4 *>(&S.bsum[buf][m][0]) =
                    make_int4(int(pk[0]), int(pk[1]), int(pk[2]), int(pk[3]));
                S.xd[buf][m] = xs;
            }
            cp_async_wait<0>();
            fence_async_smem();
            mbar_arrive(&bar_a[buf]);
            if (sb + 1 < nsb) {
#pragma unroll
                for (int k = 0; k < 9; k++) cur[k] = nxt[k];
            }
        }
    } else if (warp == 4) {
        // ---- MMA issue --------------------------------------------------------------
        if (lane == 0) {
            // N = the narrowest of 32 / 64 / 128 that covers the tile's tokens
            // (B rows past N are not read)
            const int nt = min(T - t0, tn);
            const uint32_t idesc = tc_idesc_s8(GTM, nt <= 32 ? 32 : nt <= 64 ? 64 : GTN);
            for (int sb = 0; sb < nsb; sb++) {
                const int buf = sb & 1;
                gt_wait(&bar_a[buf], uint32_t((sb >> 1) & 1));
                if (sb >= 2) gt_wait(&bar_epi[buf], uint32_t(((sb - 2) >> 1) & 1));   // TMEM buffer free
                tc_fence_after();
                const uint32_t d0 = tmem + uint32_t(buf * 2 * GTN);
#pragma unroll 1
                for (int j = 0; j < 8; j++) {
                    const uint64_t bd = tc_desc(S.b[buf][j]);
                    tc_mma_s8(d0, tc_desc(S.a[buf][0][j]), bd, idesc, j > 0);
                    tc_mma_s8(d0 + GTN, tc_desc(S.a[buf][1][j]), bd, idesc, j > 0);
                }
                tc_commit(&bar_mma[buf]);
            }
        }
        __syncwarp();
    } else {
        // ---- epilogue: warps 5..12, row m = 32 (warp % 4) + lane, tokens of half
        // (warp - 5) / 4 of the tile ------------------------------------------------
        // the tile's tokens split evenly over the two halves of the epilogue
        // warps, in multiples of 16 (a tile of 64 tokens: 32 each)
        constexpr int NH = GTN / 2;
        const int ntile = min(T - t0, tn), half = ((ntile + 31) / 32) * 16;
        const int n0 = ((warp - 5) >> 2) * half, cnt = max(0, min(half, ntile - n0));
        const int q4 = warp & 3, m = 32 * q4 + lane, r = r0 + m;
        const bool live = r < n_out;
        const uint8_t *hrow = W + size_t(live ? r : 0) * RB;
        const uint32_t lane_addr = tmem + (uint32_t(32 * q4) << 16);
        float acc[NH];
#pragma unroll
        for (int n = 0; n < NH; n++) acc[n] = 0.0f;
        for (int sb = 0; sb < nsb; sb++) {
            const int buf = sb & 1;
            const uint4 h = __ldg(reinterpret_cast<const uint4 *>(hrow + size_t(sb) * Q4K_BYTES));
            int sc[8], mn[8];
            gt_scales(h.y, h.z, h.w, sc, mn);
            // the eight 6-bit mins as packed bytes for the 16 x 8-bit dot products
            const int mlo = mn[0] | (mn[1] << 8) | (mn[2] << 16) | (mn[3] << 24);
            const int mhi = mn[4] | (mn[5] << 8) | (mn[6] << 16) | (mn[7] << 24);
            const float d = h2f(uint16_t(h.x & 0xffffu)), dm = h2f(uint16_t(h.x >> 16));
            gt_wait(&bar_mma[buf], uint32_t((sb >> 1) & 1));
            tc_fence_after();
#pragma unroll
            for (int c0 = 0; c0 < NH; c0 += 16) {
                if (c0 >= cnt) break;                // warp-uniform: past this half's tokens
                int H[16], L[16];
                tmem_ld16(lane_addr + uint32_t(buf * 2 * GTN + n0 + c0), H);
                tmem_ld16(lane_addr + uint32_t(buf * 2 * GTN + GTN + n0 + c0), L);
                tmem_wait_ld();
#pragma unroll
                for (int n = 0; n < 16; n++) {
                    // I2 = sum_j m_j bsum_j: four 2-way 16 x 8-bit integer dot products
                    const int4 b = *reinterpret_cast<const int4 *>(&S.bsum[buf][n0 + c0 + n][0]);
                    int I2 = __dp2a_lo(b.x, mlo, 0);
                    I2 = __dp2a_hi(b.y, mlo, I2);
                    I2 = __dp2a_lo(b.z, mhi, I2);
                    I2 = __dp2a_hi(b.w, mhi, I2);
                    acc[c0 + n] = q4k_fold(acc[c0 + n], S.xd[buf][n0 + c0 + n], d, dm, 32 * H[n] + L[n], I2);
                }
            }
            tc_fence_before();
            mbar_arrive(&bar_epi[buf]);
        }
        if (live) {
#pragma unroll
            for (int n = 0; n < NH; n++) {
                const int t = t0 + n0 + n;
                if (n < cnt && t < T) {
                    const size_t o = size_t(t) * n_out + r;
                    out[o] = resid ? __fadd_rn(acc[n], resid[o]) : acc[n];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, GT_TMEM_COLS);
    }
}

int launch_gemm_q4k_tc(const uint8_t *W, int n_in, int n_out, int T, const int8_t *xq, const float *xd,
                       const int16_t *xsum, float *out, const float *resid, cudaStream_t st) {
    static PerDevice attr;
    if (!attr.done()) {
        QMA_CHECK_CUDA(cudaFuncSetAttribute(gemm_q4k_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            int(GEMM_TC_SMEM)));
        attr.mark();
    }
    // token tile: the narrowest of 32 / 64 whose grid still fits one wave
    // (one CTA per SM), else 128
    const int rt = (n_out + GTM - 1) / GTM;
    int tn = GTN;
    for (const int c : {32, 64})
        if (rt * ((T + c - 1) / c) <= num_sms()) {
            tn = c;
            break;
        }
    const dim3 grid(unsigned(rt), unsigned((T + tn - 1) / tn));
    QMA_CHECK_CUDA(launch_ex(gemm_q4k_tc_kernel, grid, dim3(GT_THREADS), GEMM_TC_SMEM, st, 1, pdl_enabled(), W, n_in,
                             n_out, T, tn, xq, xd, xsum, out, resid));
    return QMA_CUDA_OK;
}

int gemm_tc_wait_timeouts() {
    unsigned n = 0;
    if (cudaMemcpyFromSymbol(&n, g_gemm_tc_timeouts, sizeof(n)) != cudaSuccess) return -1;
    if (n) {
        const unsigned zero = 0;
        cudaMemcpyToSymbol(g_gemm_tc_timeouts, &zero, sizeof(zero));
    }
    return int(n);
}

}  // namespace qma
