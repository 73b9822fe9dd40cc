// moe_tc.cu -- the grouped expert gate/up GEMM of the MoE block on the
// 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
//
// Same result as moe_gateup_kernel (moe_grouped.cu), bit for bit: the
// integer super-block sums are exact and the fp32 fold is the shared
// q4k_fold.  What changes is how the integer sums are formed.  A Q4_K
// super-block row contributes I1 = sum_j sc_j * sum_{k in j} q_k * x_k over
// its eight 32-element sub-blocks j (dot_q4_K_q8k, q8k.c:89-131).  With the
// scale folded into the weight, a_k = q_k * sc_j (0..945, ten bits), I1 =
// sum_k a_k x_k over the whole super-block -- but a_k does not fit int8, so
// it is split into two digits, a_k = 32 hi_k + lo_k (hi 0..29, lo 0..31),
// and the tensor core accumulates H = sum hi x and L = sum lo x in int32
// (|H|, |L| <= 256 * 31 * 127, exact); I1 = 32 H + L.  One tcgen05.mma of
// M = 128 rows x N = 16 pairs x K = 32 per (sub-block, digit), 16 per
// super-block, all eight super-blocks' accumulators resident in TMEM
// (8 x 2 x 16 = 256 columns).  The mins term I2 = sum_j m_j * bsum_j and
// the fp32 fold run in the epilogue, one thread per row.
//
// CTA: 256 threads, ~100 KB of shared memory and 256 TMEM columns, so two
// CTAs share an SM.  Warps 0-3 are the producers (thread = row of the
// 128-row tile: read the Q4_K block, unpack nibbles, multiply by the
// sub-block scale, split into digits, write the canonical K-major A tiles
// of both digits for one super-block at a time, the next super-block's
// bytes already in registers) and then the epilogue (TMEM lane quarter =
// warp); lane 0 of warp 4 issues the MMAs.  All threads stage the pairs'
// Q8_K activation tiles (B) once.
#include "common.cuh"
#include "moe.cuh"
#include "tc.cuh"

namespace qma {

constexpr int TCM = 128;                       // rows per CTA (TMEM lanes)
constexpr int TCN = 16;                        // pairs per CTA (MMA N)
constexpr int TC_NSB = MOE_EMBD / 256;         // super-blocks of a gate/up row
constexpr uint32_t TC_TILE_A = TCM * 32;       // one 128 x 32 int8 tile
constexpr uint32_t TC_TILE_B = TCN * 32;       // one 16 x 32 int8 tile
constexpr uint32_t TC_TMEM_COLS = 256;
static_assert(TC_NSB * 2 * TCN == int(TC_TMEM_COLS), "all super-blocks' accumulators in TMEM");

struct GateupTcSmem {
    uint8_t a[2][8][TC_TILE_A];                // [digit hi|lo][sub-block], one super-block
    uint8_t b[TC_NSB][8][TC_TILE_B];           // [super-block][sub-block]
    int bsum[TCN][TC_NSB * 8];                 // per pair: Q8_K 32-lane sums
    float xd[TCN][TC_NSB];
};
constexpr size_t GATEUP_TC_SMEM = sizeof(GateupTcSmem);

__device__ unsigned g_tc_timeouts;

// q4k_scales8 on the header words 1..3 of a Q4_K block (get_scale_min_k4,
// quants.c:18-26, for all eight sub-blocks)
__device__ __forceinline__ void tc_q4k_scales(uint32_t w0, uint32_t w1, uint32_t w2, int (&sc)[8], int (&mn)[8]) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t a = (w0 >> (8 * j)) & 0xffu, b = (w1 >> (8 * j)) & 0xffu, c = (w2 >> (8 * j)) & 0xffu;
        sc[j] = int(a & 63u);
        mn[j] = int(b & 63u);
        sc[j + 4] = int((c & 15u) | ((a >> 6) << 4));
        mn[j + 4] = int((c >> 4) | ((b >> 6) << 4));
    }
}

// Four nibble values (one per byte of n, each 0..15) times the scale sc,
// split into the digits hi = (v >> 5) and lo = (v & 31), one per byte.
__device__ __forceinline__ void tc_digits(uint32_t n, uint32_t sc, uint32_t &hi, uint32_t &lo) {
    const uint32_t pe = (n & 0x00FF00FFu) * sc, po = ((n >> 8) & 0x00FF00FFu) * sc;   // 16-bit lanes, < 1024
    hi = ((pe >> 5) & 0x001F001Fu) | (((po >> 5) & 0x001F001Fu) << 8);
    lo = (pe & 0x001F001Fu) | ((po & 0x001F001Fu) << 8);
}

__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity) {
    if (mbar_wait(bar, parity)) return true;
    if ((threadIdx.x & 31) == 0) atomicAdd(&g_tc_timeouts, 1u);
    return false;
}

// Grid (1024 / 128 row tiles of [gate | up], ng groups, ceil(T / 16) pair
// tiles); output hg[pair][1024] as moe_gateup_kernel.
__global__ void __launch_bounds__(256, 2) moe_gateup_tc_kernel(const uint8_t *__restrict__ gate_exps,
                                                               const uint8_t *__restrict__ up_exps,
                                                               const uint8_t *__restrict__ gate_sh,
                                                               const uint8_t *__restrict__ up_sh, int T,
                                                               MoeScratch s, int e0) {
    extern __shared__ __align__(128) uint8_t tcsm_raw[];
    GateupTcSmem &S = *reinterpret_cast<GateupTcSmem *>(tcsm_raw);
    __shared__ __align__(8) uint64_t bar_a, bar_m, bar_done;
    __shared__ uint32_t tmem_base;
    __shared__ int prow[TCN], ptok[TCN];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tile = blockIdx.x, e = e0 + int(blockIdx.y), tok0 = blockIdx.z * TCN;
    pdl_trigger();
    pdl_wait();
    const int ne = e < MOE_NEXP ? s.goff[e + 1] - s.goff[e] : T;
    if (tok0 >= ne) return;                               // CTA-uniform, before any TMEM is held
    if (warp == 0) tmem_alloc(&tmem_base, TC_TMEM_COLS);
    if (tid == 0) {
        mbar_init(&bar_a, 128);
        mbar_init(&bar_m, 1);
        mbar_init(&bar_done, 1);
        mbar_fence_init();
    }
    if (tid < TCN) {
        const int tk = tok0 + tid;
        int pair = -1, t = -1;
        if (tk < ne) {
            pair = e < MOE_NEXP ? s.plist[s.goff[e] + tk] : T * MOE_TOPK + tk;
            t = pair < T * MOE_TOPK ? pair / MOE_TOPK : pair - T * MOE_TOPK;
        }
        prow[tid] = pair;
        ptok[tid] = t;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    // ---- B: the pairs' Q8_K rows as canonical 16 x 32 tiles, sums, scales --
    for (int i = tid; i < TCN * TC_NSB * 8 * 2; i += 256) {
        const int kc = i & 1, j = (i >> 1) & 7, sb = (i >> 4) & 7, n = i >> 7;   // n < TCN
        const int t = ptok[n];
        int4 v = make_int4(0, 0, 0, 0);
        if (t >= 0) v = *reinterpret_cast<const int4 *>(s.xq + size_t(t) * MOE_EMBD + sb * 256 + j * 32 + kc * 16);
        *reinterpret_cast<int4 *>(&S.b[sb][j][tc_off(n, kc * 16)]) = v;
    }
    for (int i = tid; i < TCN * TC_NSB * 8; i += 256) {
        const int n = i >> 6, q = i & 63;
        const int t = ptok[n];
        S.bsum[n][q] = t >= 0 ? int(s.xs[size_t(t) * (MOE_EMBD / 16) + 2 * q]) +
                                    int(s.xs[size_t(t) * (MOE_EMBD / 16) + 2 * q + 1])
                              : 0;
    }
    if (tid < TCN * TC_NSB) {
        const int n = tid >> 3, sb = tid & 7;
        S.xd[n][sb] = ptok[n] >= 0 ? s.xd[size_t(ptok[n]) * TC_NSB + sb] : 0.0f;
    }
    fence_async_smem();
    __syncthreads();

    if (warp < 4) {
        // ---- producers: row m of the tile ---------------------------------------
        const int m = tid;
        constexpr size_t RB = size_t(TC_NSB) * Q4K_BYTES;
        const int r = (tile & 3) * TCM + m;                 // row of the gate or up matrix
        const uint8_t *W = tile < 4 ? (e < MOE_NEXP ? gate_exps + size_t(e) * MOE_FF * RB : gate_sh)
                                    : (e < MOE_NEXP ? up_exps + size_t(e) * MOE_FF * RB : up_sh);
        const uint4 *row = reinterpret_cast<const uint4 *>(W + size_t(r) * RB);
        uint4 cur[9], nxt[9];
#pragma unroll
        for (int k = 0; k < 9; k++) cur[k] = __ldg(row + k);
        for (int sb = 0; sb < TC_NSB; sb++) {
            if (sb + 1 < TC_NSB) {
#pragma unroll
                for (int k = 0; k < 9; k++) nxt[k] = __ldg(row + 9 * (sb + 1) + k);
            }
            if (sb >= 1) tc_wait(&bar_m, uint32_t((sb - 1) & 1));      // the MMAs of sb - 1 read the tiles
            int sc[8], mn[8];
            tc_q4k_scales(cur[0].y, cur[0].z, cur[0].w, sc, mn);
#pragma unroll
            for (int g = 0; g < 4; g++) {
#pragma unroll
                for (int kc = 0; kc < 2; kc++) {
                    const uint4 q = cur[1 + 2 * g + kc];          // bytes 32 g + 16 kc .. + 15
                    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int half = 0; half < 2; half++) {        // low nibbles: sub-block 2g, high: 2g + 1
                        const int j = 2 * g + half;
                        uint32_t hi[4], lo[4];
#pragma unroll
                        for (int c = 0; c < 4; c++)
                            tc_digits((w[c] >> (4 * half)) & 0x0F0F0F0Fu, uint32_t(sc[j]), hi[c], lo[c]);
                        *reinterpret_cast<uint4 *>(&S.a[0][j][tc_off(m, 16 * kc)]) =
                            make_uint4(hi[0], hi[1], hi[2], hi[3]);
                        *reinterpret_cast<uint4 *>(&S.a[1][j][tc_off(m, 16 * kc)]) =
                            make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    }
                }
            }
            fence_async_smem();
            mbar_arrive(&bar_a);
            if (sb + 1 < TC_NSB) {
#pragma unroll
                for (int k = 0; k < 9; k++) cur[k] = nxt[k];
            }
        }
    } else if (warp == 4 && lane == 0) {
        // ---- MMA issue ------------------------------------------------------------
        constexpr uint32_t idesc = tc_idesc_s8(TCM, TCN);
        for (int sb = 0; sb < TC_NSB; sb++) {
            tc_wait(&bar_a, uint32_t(sb & 1));
            tc_fence_after();
#pragma unroll 1
            for (int j = 0; j < 8; j++) {
                const uint64_t bd = tc_desc(S.b[sb][j]);
#pragma unroll
                for (int dg = 0; dg < 2; dg++)
                    tc_mma_s8(tmem + uint32_t(sb * 2 * TCN + dg * TCN), tc_desc(S.a[dg][j]), bd, idesc, j > 0);
            }
            tc_commit(&bar_m);
        }
        tc_commit(&bar_done);
    }
    // ---- epilogue: warps 0-3, thread = row ------------------------------------------
    if (warp < 4) {
        const int m = tid;
        // the row's super-block headers (d, dmin, scales), read again from
        // global memory (L2) instead of being kept in shared memory
        constexpr size_t RB = size_t(TC_NSB) * Q4K_BYTES;
        const int r = (tile & 3) * TCM + m;
        const uint8_t *W = tile < 4 ? (e < MOE_NEXP ? gate_exps + size_t(e) * MOE_FF * RB : gate_sh)
                                    : (e < MOE_NEXP ? up_exps + size_t(e) * MOE_FF * RB : up_sh);
        uint4 hdr[TC_NSB];
#pragma unroll
        for (int sb = 0; sb < TC_NSB; sb++) hdr[sb] = __ldg(reinterpret_cast<const uint4 *>(W + size_t(r) * RB + sb * Q4K_BYTES));
        tc_wait(&bar_done, 0);
        tc_fence_after();
        float acc[TCN];
#pragma unroll
        for (int n = 0; n < TCN; n++) acc[n] = 0.0f;
        const uint32_t lane_addr = tmem + (uint32_t(warp * 32) << 16);
#pragma unroll 1
        for (int sb = 0; sb < TC_NSB; sb++) {
            int H[TCN], Lo[TCN];
            tmem_ld16(lane_addr + uint32_t(sb * 2 * TCN), H);
            tmem_ld16(lane_addr + uint32_t(sb * 2 * TCN + TCN), Lo);
            tmem_wait_ld();
            int sc[8], mn[8];
            tc_q4k_scales(hdr[sb].y, hdr[sb].z, hdr[sb].w, sc, mn);
            const float d = h2f(uint16_t(hdr[sb].x & 0xffffu)), dm = h2f(uint16_t(hdr[sb].x >> 16));
#pragma unroll
            for (int n = 0; n < TCN; n++) {
                const int4 b0 = *reinterpret_cast<const int4 *>(&S.bsum[n][sb * 8]);
                const int4 b1 = *reinterpret_cast<const int4 *>(&S.bsum[n][sb * 8 + 4]);
                const int I2 = mn[0] * b0.x + mn[1] * b0.y + mn[2] * b0.z + mn[3] * b0.w + mn[4] * b1.x +
                               mn[5] * b1.y + mn[6] * b1.z + mn[7] * b1.w;
                const int I1 = 32 * H[n] + Lo[n];
                acc[n] = q4k_fold(acc[n], S.xd[n][sb], d, dm, I1, I2);
            }
        }
        const int rr = tile * TCM + m;                       // row of [gate | up]
#pragma unroll
        for (int n = 0; n < TCN; n++)
            if (prow[n] >= 0) s.hg[size_t(prow[n]) * (2 * MOE_FF) + rr] = acc[n];
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TC_TMEM_COLS);
    }
}

bool tc_disabled() {
    const char *v = getenv("QMA_CUDA_MMA_SYNC");
    return v && atoi(v) != 0;
}

// The grouped gate/up GEMM takes this kernel only with QMA_CUDA_TC_GROUPED=1
// in the environment: at the few pairs per expert of prefill chunks and
// expert-parallel steps (N = 16 tiles, mostly empty) the warp-level MMA
// kernel is faster, since the digit split doubles the unpacked weight bytes
// the producers write for every 128 x 16 tile.  The same bits either way.
bool tc_grouped() {
    const char *v = getenv("QMA_CUDA_TC_GROUPED");
    return v && atoi(v) != 0 && !tc_disabled();
}

int launch_gateup_tc(const qma_cuda_moe_weights &w, int T, const MoeScratch &s, cudaStream_t st, int g0, int ng) {
    static PerDevice attr;
    if (!attr.done()) {
        QMA_CHECK_CUDA(cudaFuncSetAttribute(moe_gateup_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            int(GATEUP_TC_SMEM)));
        attr.mark();
    }
    const int tiles = (T + TCN - 1) / TCN;
    QMA_CHECK_CUDA(launch_ex(moe_gateup_tc_kernel, dim3(2 * MOE_FF / TCM, ng, tiles), dim3(256), GATEUP_TC_SMEM, st, 1,
                             pdl_enabled(), static_cast<const uint8_t *>(w.gate_exps),
                             static_cast<const uint8_t *>(w.up_exps), static_cast<const uint8_t *>(w.gate_shexp),
                             static_cast<const uint8_t *>(w.up_shexp), T, s, g0));
    return QMA_CUDA_OK;
}

int tc_wait_timeouts() {
    unsigned n = 0;
    if (cudaMemcpyFromSymbol(&n, g_tc_timeouts, sizeof(n)) != cudaSuccess) return -1;
    if (n) {
        const unsigned zero = 0;
        cudaMemcpyToSymbol(g_tc_timeouts, &zero, sizeof(zero));
    }
    return int(n);
}

}  // namespace qma
