// gemv.cu -- standalone Q8_K quantization and quantized GEMV entry points
// (qma_cuda_q8k_quant, qma_cuda_matvec, qma_cuda_dot_partials).
#include <cstdlib>
#include <type_traits>

#include "common.cuh"
#include "gemv.cuh"
#include "tc.cuh"
#include "quant.cuh"

namespace qma {

// ------------------------------------------------------------------ Q8_K --
__global__ void __launch_bounds__(256) q8k_quant_kernel(const float *__restrict__ x, int rows,
                                                        int n, int8_t *xq, float *xd,
                                                        int16_t *xsum) {
    const int lane = threadIdx.x & 31;
    const long warp = (long(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const long nwarps = (long(gridDim.x) * blockDim.x) >> 5;
    const int nb = n / 256;
    for (long b = warp; b < long(rows) * nb; b += nwarps) {
        const long r = b / nb, j = b % nb;
        const float4 *p = reinterpret_cast<const float4 *>(x + r * n + j * 256 + lane * 8);
        const float4 a = p[0], c = p[1];
        const float v[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
        q8k_block_warp(v, lane, xq + r * n + j * 256, xd + r * nb + j, xsum + r * (n / 16) + j * 16);
    }
}

// ---------------------------------------------------------------- GEMV ----
// Single-token Q4_K projections: 3 CTAs per SM, so that one sweep of the
// one-wave grid (4 rows per warp) covers the decode in-projections.
template <class F, int T, int UPL>
constexpr int gemv_min_blocks() { return std::is_same<F, FmtQ4K>::value && T == 1 && UPL == 1 ? 3 : 1; }

template <class F, int T, int LPR, int UPL, int RU>
__global__ void __launch_bounds__(256, gemv_min_blocks<F, T, UPL>()) gemv_kernel(typename F::Ptr W, int n_in, int n_out,
                                                   const int8_t *xq, const float *xd,
                                                   const int16_t *xsum, float *out, int out_ld,
                                                   const float *resid) {
    QMA_TRACE_SCOPE(TK_GEMV);
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    pdl_trigger();
    if (threadIdx.x == 0) {
        // this CTA's rows after the first sweep (8 consecutive warp row
        // groups per sweep; the first sweep is loaded into registers before
        // the wait): into L2 while the upstream kernel finishes
        constexpr int RG = (32 / LPR) * RU;
        for (int r0 = blockIdx.x * 8 * RG + nwarps * RG; r0 < n_out; r0 += nwarps * RG)
            F::prefetch_rows(W, r0, min(8 * RG, n_out - r0), n_in);
    }
    gemv_warp_rows<F, T, LPR, UPL, RU, true>(W, n_in, n_out, xq, xd, xsum, out, out_ld, warp, nwarps,
                                             lane, resid);
}

// Single-token GEMV over a row block per CTA staged whole in shared memory:
// the bulk copy is issued at launch, before waiting on the upstream kernel
// (whose output is the activation), so the weight transfer overlaps it;
// after the wait only the activation load and the dot products remain.
__device__ unsigned g_gemv_timeouts;

// Rows of a 32-lanes-per-row matrix (n_in >= 2048): each warp takes an
// equal share of the CTA's rows, in batches of up to 8 independent dot
// products followed by one 8-way warp reduction.
template <class F, int UPL>
__device__ __forceinline__ void staged_rows32(const typename F::Ptr &P, int n_in, int nr,
                                              const typename F::Act (&act)[UPL], float *out,
                                              const float *resid, int warp, int nwarps, int lane,
                                              int row0, const ConvEpi &conv, const float4 *cw,
                                              const float *cs) {
    const int idx = warp_sum8_index(lane);
    // the CTA's rows spread evenly over its warps, in batches of up to 8
    const int rpw = (nr + nwarps - 1) / nwarps;
    const int r_end = min(nr, (warp + 1) * rpw);
    for (int rb = warp * rpw; rb < r_end; rb += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            v[j] = 0.0f;
            if (rb + j < r_end) {
#pragma unroll
                for (int k = 0; k < UPL; k++) {
                    typename F::Wt w;
                    F::load_w_smem(w, P, rb + j, n_in, lane + 32 * k);
                    v[j] += F::dot(w, act[k], lane + 32 * k);
                }
            }
        }
        const float tot = warp_sum8(v, lane);
        const int r = rb + idx;
        if ((lane & 3) == 0 && r < r_end) {
            out[r] = resid ? __fadd_rn(tot, resid[r]) : tot;
            if (r + row0 < conv.n) {
                // taps and state of the row were read into shared memory
                // before the upstream wait
                const int c = r + row0;
                const float4 wc = cw[r];
                float *stc = conv.state + size_t(c) * 3;
                const float s0 = cs[3 * r], s1 = cs[3 * r + 1], s2 = cs[3 * r + 2];
                float sum = __fmul_rn(s0, wc.x);
                sum = __fadd_rn(sum, __fmul_rn(s1, wc.y));
                sum = __fadd_rn(sum, __fmul_rn(s2, wc.z));
                sum = __fadd_rn(sum, __fmul_rn(tot, wc.w));
                conv.out[c] = sum / (1.0f + expf(-sum));
                stc[0] = s1;
                stc[1] = s2;
                stc[2] = tot;
            }
        }
    }
}

template <class F, int LPR, int UPL, int RU>
__global__ void __launch_bounds__(512) gemv_staged_kernel(typename F::Ptr W, int n_in, int n_out,
                                                          int rows_cta, const int8_t *xq,
                                                          const float *xd, const int16_t *xsum,
                                                          float *out, const float *resid, ConvEpi conv) {
    QMA_TRACE_SCOPE(TK_GEMV);
    extern __shared__ __align__(128) uint8_t wbuf[];
    __shared__ __align__(8) uint64_t bar;
    const int r0 = blockIdx.x * rows_cta;
    const int nr = min(rows_cta, n_out - r0);
    if (threadIdx.x < 32 && nr > 0) {
        if (threadIdx.x == 0) {
            mbar_init(&bar, 1);
            mbar_fence_init();
        }
        __syncwarp();
        Stage<F>::issue(W, r0, nr, n_in, wbuf, &bar, threadIdx.x);
    }
    // the conv epilogue's taps and state for this CTA's rows: written by
    // earlier steps only, so read before the upstream wait
    constexpr int CONV_ROWS = 160;
    __shared__ float4 cw[CONV_ROWS];
    __shared__ float cs[3 * CONV_ROWS];
    if (conv.n && nr <= CONV_ROWS) {
        for (int r = threadIdx.x; r < nr; r += blockDim.x) {
            const int c = r0 + r;
            if (c < conv.n) {
                cw[r] = *reinterpret_cast<const float4 *>(conv.w + size_t(c) * 4);
                cs[3 * r] = conv.state[size_t(c) * 3];
                cs[3 * r + 1] = conv.state[size_t(c) * 3 + 1];
                cs[3 * r + 2] = conv.state[size_t(c) * 3 + 2];
            }
        }
    }
    __syncthreads();
    pdl_trigger();
    pdl_wait();
    QMA_TRACE_MARK(TK_GEMV, 1);
    if (nr <= 0) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    // the activation slices load while the last weight bytes land
    typename F::Act act[LPR == 32 ? UPL : 1];
    if constexpr (LPR == 32) {
#pragma unroll
        for (int k = 0; k < UPL; k++) F::load_act(act[k], xq, xd, xsum, lane + 32 * k);
    }
    if (!mbar_wait(&bar, 0)) {
        if (threadIdx.x == 0) atomicAdd(&g_gemv_timeouts, 1u);
        mbar_wait(&bar, 0);     // let a late copy land before the CTA exits
        return;
    }
    QMA_TRACE_MARK(TK_GEMV, 2);
    const auto P = Stage<F>::view(wbuf, nr, n_in);
    if constexpr (LPR == 32)
        staged_rows32<F, UPL>(P, n_in, nr, act, out + r0, resid ? resid + r0 : nullptr, warp, nwarps, lane, r0,
                              conv, cw, cs);
    else
        gemv_warp_rows<SmemRows<F>, 1, LPR, UPL, RU>(P, n_in, nr, xq, xd, xsum, out + r0, 0, warp, nwarps,
                                                     lane, resid ? resid + r0 : nullptr);
    QMA_TRACE_MARK(TK_GEMV, 3);
}

// Single-token GEMV over a matrix too large for one staged block per SM (the
// LM head): one persistent CTA per SM streams its contiguous row range
// through a ring of STREAM_NST shared-memory stages, each a bulk copy of
// `rows_blk` rows.  The copies of the next stages are in flight while the
// current one is computed, so every SM keeps ~STREAM_NST stages of weights
// outstanding; the first stages are issued before waiting on the upstream
// kernel.  Warp w computes rows w, w + 16, ... of a stage; the last warp to
// finish a stage issues its next copy (no CTA-wide barrier per stage).
constexpr int STREAM_NST = 4;
constexpr uint32_t STREAM_STAGE = 36 * 1024;    // target bytes per stage

template <class F, int UPL>
__global__ void __launch_bounds__(512, 1) gemv_stream_kernel(typename F::Ptr W, int n_in, int n_out,
                                                           int rows_cta, int rows_blk, uint32_t stage_bytes,
                                                           const int8_t *xq, const float *xd,
                                                           const int16_t *xsum, float *out,
                                                           const float *resid) {
    QMA_TRACE_SCOPE(TK_GEMV);
    extern __shared__ __align__(128) uint8_t sbuf[];
    __shared__ __align__(8) uint64_t bar[STREAM_NST];
    __shared__ unsigned done[STREAM_NST];          // warps finished with the stage's current block
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    const int c0 = blockIdx.x * rows_cta;
    const int c1 = min(n_out, c0 + rows_cta);
    const int nblk = c1 > c0 ? (c1 - c0 + rows_blk - 1) / rows_blk : 0;
    if (tid == 0) {
        for (int i = 0; i < STREAM_NST; i++) {
            mbar_init(&bar[i], 1);
            done[i] = 0;
        }
        mbar_fence_init();
    }
    __syncthreads();
    auto issue = [&](int b) {
        const int r0 = c0 + b * rows_blk, nr = min(rows_blk, c1 - r0);
        Stage<F>::issue(W, r0, nr, n_in, sbuf + size_t(b % STREAM_NST) * stage_bytes, &bar[b % STREAM_NST], lane);
    };
    if (warp == 0)
        for (int b = 0; b < min(STREAM_NST, nblk); b++) issue(b);
    pdl_trigger();
    pdl_wait();
    typename F::Act act[UPL];
#pragma unroll
    for (int k = 0; k < UPL; k++) F::load_act(act[k], xq, xd, xsum, lane + 32 * k);
    bool ok = true;
    for (int b = 0; b < nblk; b++) {
        const int st = b % STREAM_NST;
        const uint32_t par = uint32_t(b / STREAM_NST) & 1u;
        if (!mbar_wait(&bar[st], par)) {
            ok = false;
            mbar_wait(&bar[st], par);            // let a late copy land before reuse or exit
        }
        const int r0 = c0 + b * rows_blk, nr = min(rows_blk, c1 - r0);
        const auto P = Stage<F>::view(sbuf + size_t(st) * stage_bytes, nr, n_in);
        for (int r = warp; r < nr; r += nwarps) {
            float v = 0.0f;
#pragma unroll
            for (int k = 0; k < UPL; k++) {
                typename F::Wt w;
                F::load_w_smem(w, P, r, n_in, lane + 32 * k);
                v += F::dot(w, act[k], lane + 32 * k);
            }
            v = warp_sum(v);
            if (lane == 0) out[r0 + r] = resid ? __fadd_rn(v, resid[r0 + r]) : v;
        }
        // the last warp done with this block refills the stage; the others
        // go on to the next block without waiting
        __syncwarp();
        unsigned last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&done[st], 1u) == unsigned(nwarps - 1);
        }
        if (__shfl_sync(0xffffffffu, last, 0)) {
            if (lane == 0) done[st] = 0;
            if (b + STREAM_NST < nblk) {
                fence_proxy_async_smem();
                issue(b + STREAM_NST);
            }
        }
    }
    if (!ok && lane == 0) atomicAdd(&g_gemv_timeouts, 1u);
}

template <class F, int UPL>
static int launch_stream(const typename F::Ptr &W, int n_in, int n_out, const int8_t *xq, const float *xd,
                         const int16_t *xsum, float *out, const float *resid, cudaStream_t st) {
    const int row_bytes = int(Stage<F>::bytes(8, n_in) / 8);
    int rows_blk = (int(STREAM_STAGE) / row_bytes) & ~7;
    if (rows_blk < 8) rows_blk = 8;
    const uint32_t stage_bytes = Stage<F>::bytes(rows_blk, n_in);
    const size_t smem = size_t(stage_bytes) * STREAM_NST;
    static PerDevice attr;
    if (!attr.done()) {
        QMA_CHECK_CUDA(cudaFuncSetAttribute(gemv_stream_kernel<F, UPL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            int(STREAM_NST * (STREAM_STAGE + 8 * 1024))));
        attr.mark();
    }
    const int grid = num_sms();
    int rows_cta = (n_out + grid - 1) / grid;
    rows_cta = (rows_cta + 7) & ~7;
    QMA_CHECK_CUDA(launch_ex(gemv_stream_kernel<F, UPL>, dim3(unsigned(grid)), dim3(512), smem, st, 1, pdl_enabled(),
                             W, n_in, n_out, rows_cta, rows_blk, stage_bytes, xq, xd, xsum, out, resid));
    return QMA_CUDA_OK;
}

int gemv_wait_timeouts() {
    unsigned n = 0;
    if (cudaMemcpyFromSymbol(&n, g_gemv_timeouts, sizeof(n)) != cudaSuccess) return -1;
    if (n) {
        const unsigned zero = 0;
        cudaMemcpyToSymbol(g_gemv_timeouts, &zero, sizeof(zero));
    }
    return int(n);
}

constexpr uint32_t STAGED_MAX = 160 * 1024;    // shared memory per CTA for a staged GEMV

template <class F, int LPR, int UPL, int RU>
static int launch_staged(const typename F::Ptr &W, int n_in, int n_out, const int8_t *xq,
                         const float *xd, const int16_t *xsum, float *out, const float *resid,
                         int rows_cta, uint32_t smem, cudaStream_t st, const ConvEpi &conv) {
    static PerDevice attr;
    if (!attr.done()) {
        QMA_CHECK_CUDA(cudaFuncSetAttribute(gemv_staged_kernel<F, LPR, UPL, RU>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, int(STAGED_MAX)));
        QMA_CHECK_CUDA(cudaFuncSetAttribute(gemv_staged_kernel<F, LPR, UPL, RU>,
                                            cudaFuncAttributePreferredSharedMemoryCarveout, 100));
        attr.mark();
    }
    const int grid = (n_out + rows_cta - 1) / rows_cta;
    const unsigned threads = 512;
    QMA_CHECK_CUDA(launch_ex(gemv_staged_kernel<F, LPR, UPL, RU>, dim3(unsigned(grid)), dim3(threads), smem, st, 1,
                             pdl_enabled(), W, n_in, n_out, rows_cta, xq, xd, xsum, out, resid, conv));
    return QMA_CUDA_OK;
}

// SM count of the current device (looked up once per device)
static std::atomic<int> g_num_sms[64];
int num_sms() {
    int dev = PerDevice::current();
    if (dev < 0 || dev >= 64) dev = 0;
    int n = g_num_sms[dev].load(std::memory_order_relaxed);
    if (n <= 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_num_sms[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

// One full wave: as many 256-thread CTAs as fit on every SM at once (from
// the kernel's own register use), capped by the rows there are to do.
template <class F, int T, int LPR, int UPL, int RU>
static int launch_gemv(const typename F::Ptr &W, int n_in, int n_out, const int8_t *xq,
                       const float *xd, const int16_t *xsum, float *out, int out_ld,
                       const float *resid, cudaStream_t st) {
    constexpr int RPW = 32 / LPR;
    static int per_sm = 0;
    if (!per_sm) {
        QMA_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &per_sm, gemv_kernel<F, T, LPR, UPL, RU>, 256, 0));
        if (per_sm < 1) per_sm = 1;
    }
    const long warps_needed = (n_out + RPW * RU - 1) / (RPW * RU);
    long blocks = (warps_needed + 7) / 8;
    const long wave = long(num_sms()) * per_sm;
    if (blocks > wave) blocks = wave;
    QMA_CHECK_CUDA(launch_ex(gemv_kernel<F, T, LPR, UPL, RU>, dim3(unsigned(blocks)), dim3(256), 0, st, 1,
                             pdl_enabled(), W, n_in, n_out, xq, xd, xsum, out, out_ld, resid));
    return QMA_CUDA_OK;
}

// Shape dispatch: units per row U = n_in / F::UNIT.  Single-token passes
// keep four row groups of loads in flight per warp (so that one sweep of a
// one-wave grid covers the decode projections).
template <class F, int T, int RU = (T == 1 ? 4 : 1)>
static int dispatch_shape(const typename F::Ptr &W, int n_in, int n_out, const int8_t *xq,
                          const float *xd, const int16_t *xsum, float *out, int out_ld,
                          const float *resid, cudaStream_t st) {
    const int U = n_in / F::UNIT;
    switch (U) {
    case 2: return launch_gemv<F, T, 2, 1, RU>(W, n_in, n_out, xq, xd, xsum, out, out_ld, resid, st);
    case 4: return launch_gemv<F, T, 4, 1, RU>(W, n_in, n_out, xq, xd, xsum, out, out_ld, resid, st);
    case 8: return launch_gemv<F, T, 8, 1, RU>(W, n_in, n_out, xq, xd, xsum, out, out_ld, resid, st);
    case 16: return launch_gemv<F, T, 16, 1, RU>(W, n_in, n_out, xq, xd, xsum, out, out_ld, resid, st);
    case 32: return launch_gemv<F, T, 32, 1, RU>(W, n_in, n_out, xq, xd, xsum, out, out_ld, resid, st);
    case 64: return launch_gemv<F, T, 32, 2, (RU > 1 ? RU / 2 : 1)>(W, n_in, n_out, xq, xd, xsum, out, out_ld, resid, st);
    default:
        set_error("matvec: n_in %d unsupported for this weight type", n_in);
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
}

// Single-token launch with each CTA's rows staged in shared memory when the
// matrix spread over one CTA per SM fits (the decode projections); false
// when it does not (the LM head streams through the register GEMV).
template <class F>
static bool try_staged(const typename F::Ptr &W, int n_in, int n_out, const int8_t *xq, const float *xd,
                       const int16_t *xsum, float *out, const float *resid, cudaStream_t st, int &rc,
                       const ConvEpi &conv) {
    int rows_cta = (n_out + num_sms() - 1) / num_sms();
    rows_cta = (rows_cta + 7) & ~7;
    const uint32_t smem = Stage<F>::bytes(rows_cta, n_in);
    if (smem > STAGED_MAX || (conv.n && rows_cta > 160)) return false;
    const int U = n_in / F::UNIT;
    switch (U) {
    case 4: if (conv.n) return false;
        rc = launch_staged<F, 4, 1, 2>(W, n_in, n_out, xq, xd, xsum, out, resid, rows_cta, smem, st, conv); return true;
    case 8: if (conv.n) return false;
        rc = launch_staged<F, 8, 1, 2>(W, n_in, n_out, xq, xd, xsum, out, resid, rows_cta, smem, st, conv); return true;
    case 16: if (conv.n) return false;
        rc = launch_staged<F, 16, 1, 2>(W, n_in, n_out, xq, xd, xsum, out, resid, rows_cta, smem, st, conv); return true;
    case 32: rc = launch_staged<F, 32, 1, 2>(W, n_in, n_out, xq, xd, xsum, out, resid, rows_cta, smem, st, conv); return true;
    case 64: rc = launch_staged<F, 32, 2, 1>(W, n_in, n_out, xq, xd, xsum, out, resid, rows_cta, smem, st, conv); return true;
    default: return false;
    }
}

// ------------------------------------------------ Q4_K GEMM on tensor cores --
// Several tokens against Q4_K rows (prefill chunks): int8 tensor-core MMAs
// (mma.sync m16n8k32 s8 x s8 -> s32) compute each 32-element sub-block's
// exact integer partial sum(q * xq) for 16 rows x 8 tokens at once; the
// partials are folded with the sub-block scales in integer registers
// (I1 = sum_j sc_j * P_j, exact), the mins through the Q8_K block sums
// (I2 = sum_j m_j * bsum_j), and each super-block contributes
// xd * (d * I1 - dmin * I2) in fp32 -- the GEMV's arithmetic per super-block
// (dot_q4_K_q8k, q8k.c:89-131) with the integer part on the tensor cores.
// A Q4_K sub-block pair (2g, 2g+1) is the low and high nibbles of the same
// 32 bytes, so one 32-bit weight load per fragment register serves both.
// Warp: 16 rows x (8 * GNT) tokens; CTA: 4 warps = 64 rows.
constexpr int GNT = 4;

__global__ void __launch_bounds__(128) gemm_q4k_mma_kernel(const uint8_t *__restrict__ W, int n_in, int n_out,
                                                           int T, const int8_t *__restrict__ xq,
                                                           const float *__restrict__ xd,
                                                           const int16_t *__restrict__ xsum, float *out,
                                                           const float *resid) {
    QMA_TRACE_SCOPE(TK_GEMV);
    static_assert(8 * GNT == BT_COLS, "one staged activation tile per CTA");
    __shared__ __align__(16) int8_t bt[2][BT_COLS][BT_STRIDE];
    __shared__ int brow[BT_COLS];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    const int row0 = (blockIdx.x * 4 + warp) * 16;
    const int tok0 = blockIdx.y * (8 * GNT);
    const bool active = row0 < n_out;            // warp-uniform; every warp stages and syncs
    if (threadIdx.x < BT_COLS) brow[threadIdx.x] = tok0 + int(threadIdx.x) < T ? tok0 + int(threadIdx.x) : -1;
    pdl_trigger();
    pdl_wait();
    const int nsb = n_in / 256;
    const size_t rb = size_t(nsb) * 144;
    const uint8_t *wr0 = W + size_t(active ? row0 + gid : 0) * rb, *wr1 = wr0 + 8 * rb;
    float acc[GNT][4];
#pragma unroll
    for (int n = 0; n < GNT; n++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[n][i] = 0.0f;
    // the two token columns this lane's accumulators hold, per token tile
    int tc[GNT][2];
    bool tv[GNT][2];
#pragma unroll
    for (int n = 0; n < GNT; n++)
#pragma unroll
        for (int c = 0; c < 2; c++) {
            tc[n][c] = tok0 + 8 * n + 2 * tig + c;
            tv[n][c] = tc[n][c] < T;
        }
    // activation tiles double-buffered: tile sb + 1 is copied while sb's MMAs run
    __syncthreads();                              // brow
    stage_btile_async(bt[0], brow, xq, size_t(n_in), 0);
    for (int sb = 0; sb < nsb; sb++) {
        __syncthreads();                          // the tile of sb - 1 is consumed
        if (sb + 1 < nsb) {
            stage_btile_async(bt[(sb + 1) & 1], brow, xq, size_t(n_in), (sb + 1) * 256);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();                          // tile sb is in shared memory
        if (!active) continue;
        const int8_t(*bt_)[BT_STRIDE] = bt[sb & 1];
        const uint8_t *h0 = wr0 + size_t(sb) * 144, *h1 = wr1 + size_t(sb) * 144;
        int sc0[8], mn0[8], sc1[8], mn1[8];
        q4k_scales8(h0, sc0, mn0);
        q4k_scales8(h1, sc1, mn1);
        const float d0 = h2f(*reinterpret_cast<const uint16_t *>(h0)), dm0 = h2f(*reinterpret_cast<const uint16_t *>(h0 + 2));
        const float d1 = h2f(*reinterpret_cast<const uint16_t *>(h1)), dm1 = h2f(*reinterpret_cast<const uint16_t *>(h1 + 2));
        int I1[GNT][4];
#pragma unroll
        for (int n = 0; n < GNT; n++)
#pragma unroll
            for (int i = 0; i < 4; i++) I1[n][i] = 0;
#pragma unroll
        for (int g = 0; g < 4; g++) {
            // rows gid / gid + 8, bytes 32 g + 4 tig (k 0..15) and + 16 (k 16..31)
            const uint32_t r0a = *reinterpret_cast<const uint32_t *>(h0 + 16 + 32 * g + 4 * tig);
            const uint32_t r0b = *reinterpret_cast<const uint32_t *>(h0 + 16 + 32 * g + 16 + 4 * tig);
            const uint32_t r1a = *reinterpret_cast<const uint32_t *>(h1 + 16 + 32 * g + 4 * tig);
            const uint32_t r1b = *reinterpret_cast<const uint32_t *>(h1 + 16 + 32 * g + 16 + 4 * tig);
#pragma unroll
            for (int half = 0; half < 2; half++) {
                const int j = 2 * g + half;
                const int sh = 4 * half;
                const uint32_t a[4] = {(r0a >> sh) & 0x0f0f0f0fu, (r1a >> sh) & 0x0f0f0f0fu,
                                       (r0b >> sh) & 0x0f0f0f0fu, (r1b >> sh) & 0x0f0f0f0fu};
#pragma unroll
                for (int n = 0; n < GNT; n++) {
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
        // mins through the block sums of each token column, then the fp32 fold
        int md0[4], md1[4];
        q4k_mins_dup(mn0, md0);
        q4k_mins_dup(mn1, md1);
#pragma unroll
        for (int n = 0; n < GNT; n++)
#pragma unroll
            for (int c = 0; c < 2; c++) {
                if (!tv[n][c]) continue;
                const int16_t *bs = xsum + size_t(tc[n][c]) * (n_in / 16) + sb * 16;
                const int I2a = q4k_i2(bs, md0), I2b = q4k_i2(bs, md1);
                const float x = xd[size_t(tc[n][c]) * nsb + sb];
                acc[n][c] = q4k_fold(acc[n][c], x, d0, dm0, I1[n][c], I2a);
                acc[n][2 + c] = q4k_fold(acc[n][2 + c], x, d1, dm1, I1[n][2 + c], I2b);
            }
    }
    if (!active) return;
#pragma unroll
    for (int n = 0; n < GNT; n++)
#pragma unroll
        for (int c = 0; c < 2; c++) {
            if (!tv[n][c]) continue;
            const size_t o0 = size_t(tc[n][c]) * n_out + row0 + gid, o1 = o0 + 8;
            out[o0] = resid ? __fadd_rn(acc[n][c], resid[o0]) : acc[n][c];
            out[o1] = resid ? __fadd_rn(acc[n][2 + c], resid[o1]) : acc[n][2 + c];
        }
}

// ------------------------------------------------ Q8_0 GEMM on tensor cores --
// Several tokens against Q8_0 rows (the LM head of a batched step, the
// logits of a prefill chunk): one mma.sync m16n8k32 (s8 x s8 -> s32) per
// 32-element block gives its exact integer dot for 16 rows x 8 tokens; a
// 64-element unit contributes (i0 d0 + i1 d1) xd in fp32 as in FmtQ80::dot,
// the units summed in order.  Warp: 16 rows x 32 tokens; CTA: 4 warps = 64
// rows.  Grid (token tiles, row blocks): the token tiles of one row block
// run next to each other, so the weight rows are read from HBM once.
__global__ void __launch_bounds__(128) gemm_q80_mma_kernel(Q8Planes P, int n_in, int n_out, int T,
                                                           const int8_t *__restrict__ xq,
                                                           const float *__restrict__ xd, float *out,
                                                           const float *resid) {
    QMA_TRACE_SCOPE(TK_GEMV);
    __shared__ __align__(16) int8_t bt[2][BT_COLS][BT_STRIDE];
    __shared__ int brow[BT_COLS];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    const int row0 = (blockIdx.y * 4 + warp) * 16;
    const int tok0 = blockIdx.x * (8 * GNT);
    const bool active = row0 < n_out;            // warp-uniform; every warp stages and syncs
    if (threadIdx.x < BT_COLS) brow[threadIdx.x] = tok0 + int(threadIdx.x) < T ? tok0 + int(threadIdx.x) : -1;
    pdl_trigger();
    pdl_wait();
    const int nsb = n_in / 256, nb = n_in / 32;
    const int8_t *q0 = P.q + size_t(active ? row0 + gid : 0) * n_in, *q1 = q0 + size_t(8) * n_in;
    const __half *dr0 = P.d + size_t(active ? row0 + gid : 0) * nb, *dr1 = dr0 + size_t(8) * nb;
    float acc[GNT][4];
#pragma unroll
    for (int n = 0; n < GNT; n++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[n][i] = 0.0f;
    int tc[GNT][2];
    bool tv[GNT][2];
#pragma unroll
    for (int n = 0; n < GNT; n++)
#pragma unroll
        for (int c = 0; c < 2; c++) {
            tc[n][c] = tok0 + 8 * n + 2 * tig + c;
            tv[n][c] = tc[n][c] < T;
        }
    __syncthreads();                              // brow
    stage_btile_async(bt[0], brow, xq, size_t(n_in), 0);
    for (int sb = 0; sb < nsb; sb++) {
        __syncthreads();                          // the tile of sb - 1 is consumed
        if (sb + 1 < nsb) {
            stage_btile_async(bt[(sb + 1) & 1], brow, xq, size_t(n_in), (sb + 1) * 256);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();                          // tile sb is in shared memory
        if (!active) continue;
        const int8_t(*bt_)[BT_STRIDE] = bt[sb & 1];
        float x[GNT][2];
#pragma unroll
        for (int n = 0; n < GNT; n++)
#pragma unroll
            for (int c = 0; c < 2; c++) x[n][c] = tv[n][c] ? xd[size_t(tc[n][c]) * nsb + sb] : 0.0f;
#pragma unroll
        for (int u = 0; u < 4; u++) {             // units of 64: blocks 2u, 2u + 1
            int p[2][GNT][4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int k = sb * 256 + 32 * (2 * u + h) + 4 * tig;
                const uint32_t a[4] = {*reinterpret_cast<const uint32_t *>(q0 + k),
                                       *reinterpret_cast<const uint32_t *>(q1 + k),
                                       *reinterpret_cast<const uint32_t *>(q0 + k + 16),
                                       *reinterpret_cast<const uint32_t *>(q1 + k + 16)};
#pragma unroll
                for (int n = 0; n < GNT; n++) {
                    const int8_t *bp = &bt_[8 * n + gid][32 * (2 * u + h) + 4 * tig];
#pragma unroll
                    for (int i = 0; i < 4; i++) p[h][n][i] = 0;
                    mma_s8(p[h][n], a, *reinterpret_cast<const uint32_t *>(bp),
                           *reinterpret_cast<const uint32_t *>(bp + 16));
                }
            }
            const int b = sb * 8 + 2 * u;
            const float d00 = __half2float(dr0[b]), d01 = __half2float(dr0[b + 1]);
            const float d10 = __half2float(dr1[b]), d11 = __half2float(dr1[b + 1]);
#pragma unroll
            for (int n = 0; n < GNT; n++)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const float t0 = __fmul_rn(__fadd_rn(__fmul_rn(float(p[0][n][c]), d00),
                                                         __fmul_rn(float(p[1][n][c]), d01)), x[n][c]);
                    const float t1 = __fmul_rn(__fadd_rn(__fmul_rn(float(p[0][n][2 + c]), d10),
                                                         __fmul_rn(float(p[1][n][2 + c]), d11)), x[n][c]);
                    acc[n][c] = __fadd_rn(acc[n][c], t0);
                    acc[n][2 + c] = __fadd_rn(acc[n][2 + c], t1);
                }
        }
    }
    if (!active) return;
#pragma unroll
    for (int n = 0; n < GNT; n++)
#pragma unroll
        for (int c = 0; c < 2; c++) {
            if (!tv[n][c]) continue;
            const size_t o0 = size_t(tc[n][c]) * n_out + row0 + gid, o1 = o0 + 8;
            out[o0] = resid ? __fadd_rn(acc[n][c], resid[o0]) : acc[n][c];
            out[o1] = resid ? __fadd_rn(acc[n][2 + c], resid[o1]) : acc[n][2 + c];
        }
}

static int launch_gemm_q80(const Q8Planes &P, int n_in, int n_out, int T, const int8_t *xq, const float *xd,
                           float *out, const float *resid, cudaStream_t st) {
    const dim3 grid(unsigned((T + 8 * GNT - 1) / (8 * GNT)), unsigned((n_out + 63) / 64));
    QMA_CHECK_CUDA(launch_ex(gemm_q80_mma_kernel, grid, dim3(128), 0, st, 1, pdl_enabled(), P, n_in, n_out, T, xq,
                             xd, out, resid));
    return QMA_CUDA_OK;
}

// gemm_tc.cu
int launch_gemm_q4k_tc(const uint8_t *W, int n_in, int n_out, int T, const int8_t *xq, const float *xd,
                       const int16_t *xsum, float *out, const float *resid, cudaStream_t st);

static int launch_gemm_q4k(const uint8_t *W, int n_in, int n_out, int T, const int8_t *xq, const float *xd,
                           const int16_t *xsum, float *out, const float *resid, cudaStream_t st) {
    const dim3 grid(unsigned((n_out + 63) / 64), unsigned((T + 8 * GNT - 1) / (8 * GNT)));
    QMA_CHECK_CUDA(launch_ex(gemm_q4k_mma_kernel, grid, dim3(128), 0, st, 1, pdl_enabled(), W, n_in, n_out, T, xq,
                             xd, xsum, out, resid));
    return QMA_CUDA_OK;
}

template <class F, int TMAX>
static int gemv_tokens(const typename F::Ptr &W, int n_in, int n_out, int T, const int8_t *xq,
                       const float *xd, const int16_t *xsum, float *out, const float *resid,
                       cudaStream_t st, const ConvEpi &conv) {
    int rc;
    if (T == 1 && pdl_enabled() && try_staged<F>(W, n_in, n_out, xq, xd, xsum, out, resid, st, rc, conv)) return rc;
    // a single token over a larger matrix (the LM head): streamed per SM
    if (T == 1 && !conv.n && n_in == 32 * F::UNIT)
        return launch_stream<F, 1>(W, n_in, n_out, xq, xd, xsum, out, resid, st);
    if (T == 1 && !conv.n && n_in == 64 * F::UNIT)
        return launch_stream<F, 2>(W, n_in, n_out, xq, xd, xsum, out, resid, st);
    if (conv.n) {
        set_error("matvec: the conv epilogue needs the single-token staged path");
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
    // several tokens over Q4_K rows: the tensor-core GEMM (tcgen05 from 64
    // tokens on, the warp-level MMA kernel below that or when asked)
    if constexpr (std::is_same<F, FmtQ4K>::value) {
        if (T >= 64 && !tc_disabled())
            return launch_gemm_q4k_tc(W, n_in, n_out, T, xq, xd, xsum, out, resid, st);
        if (T >= 8 && n_out % 16 == 0)
            return launch_gemm_q4k(W, n_in, n_out, T, xq, xd, xsum, out, resid, st);
    }
    // several tokens over Q8_0 rows (batched LM head, prefill logits): the
    // MMA kernel reads the rows once for every 32 tokens instead of once per
    // pass of 4
    if constexpr (std::is_same<F, FmtQ80>::value) {
        if (T >= 8 && n_out % 16 == 0) return launch_gemm_q80(W, n_in, n_out, T, xq, xd, out, resid, st);
    }
    int t0 = 0;
    while (t0 < T) {
        const int rem = T - t0;
        const int8_t *q = xq + size_t(t0) * n_in;
        const float *d = xd + size_t(t0) * (n_in / 256);
        const int16_t *s = xsum + size_t(t0) * (n_in / 16);
        float *o = out + size_t(t0) * n_out;
        const float *rs = resid ? resid + size_t(t0) * n_out : nullptr;
        int rc, tn;
        if constexpr (TMAX >= 4) {
            if (rem >= 4) {
                rc = dispatch_shape<F, 4>(W, n_in, n_out, q, d, s, o, n_out, rs, st);
                tn = 4;
                if (rc) return rc;
                t0 += tn;
                continue;
            }
        }
        if (rem >= 2) {
            rc = dispatch_shape<F, 2>(W, n_in, n_out, q, d, s, o, n_out, rs, st);
            tn = 2;
        } else {
            rc = dispatch_shape<F, 1>(W, n_in, n_out, q, d, s, o, n_out, rs, st);
            tn = 1;
        }
        if (rc) return rc;
        t0 += tn;
    }
    return QMA_CUDA_OK;
}

int matvec(int wtype, const void *W, int n_in, int n_out, int T, const int8_t *xq,
           const float *xd, const int16_t *xsum, float *out, cudaStream_t st,
           const float *resid, const ConvEpi *conv) {
    const ConvEpi ce = conv ? *conv : ConvEpi();
    switch (wtype) {
    case QMA_TYPE_Q4_K:
        return gemv_tokens<FmtQ4K, 4>(static_cast<const uint8_t *>(W), n_in, n_out, T, xq, xd,
                                      xsum, out, resid, st, ce);
    case QMA_TYPE_Q6_K:
        return gemv_tokens<FmtQ6K, 2>(q6_planes(W, n_out, n_in), n_in, n_out, T, xq, xd, xsum,
                                      out, resid, st, ce);
    case QMA_TYPE_Q8_0:
        return gemv_tokens<FmtQ80, 4>(q8_planes(W, n_out, n_in), n_in, n_out, T, xq, xd, xsum,
                                      out, resid, st, ce);
    default:
        set_error("matvec: unsupported weight type %d", wtype);
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
}

// --------------------------------------------------------- int partials ---
// One thread per (row, unit), with the GEMV's own unit arithmetic.
template <class F>
__global__ void partials_kernel_safe(typename F::Ptr W, int n_in, int n_out, const int8_t *xq,
                                     const float *xd, const int16_t *xsum, int32_t *isum) {
    const int U = n_in / F::UNIT;
    const long total = long(n_out) * U;
    for (long i = blockIdx.x * long(blockDim.x) + threadIdx.x; i < total;
         i += long(gridDim.x) * blockDim.x) {
        const int r = int(i / U), u = int(i % U);
        typename F::Act a;
        F::load_act(a, xq, xd, xsum, u);
        typename F::Wt w;
        F::load_w(w, W, r, n_in, u);
        if constexpr (F::UNIT == 128) {
            atomicAdd(isum + size_t(r) * (n_in / 256) + (u >> 1), F::isum(w, a));
        } else {
            int p0, p1;
            F::isums(w, a, p0, p1);
            isum[size_t(r) * (n_in / 32) + 2 * u] = p0;
            isum[size_t(r) * (n_in / 32) + 2 * u + 1] = p1;
        }
    }
}
}  // namespace qma

extern "C" {

int qma_cuda_q8k_quant(const float *x, int rows, int n, int8_t *xq, float *xd, int16_t *xsum,
                       void *stream) {
    qma::clear_error();
    QMA_REQUIRE(x && xq && xd && xsum && rows > 0 && n > 0 && n % 256 == 0,
                "qma_cuda_q8k_quant: bad arguments (rows %d, n %d)", rows, n);
    const long warps = long(rows) * (n / 256);
    long blocks = (warps + 7) / 8;
    if (blocks > 4096) blocks = 4096;
    qma::q8k_quant_kernel<<<int(blocks), 256, 0, qma::as_stream(stream)>>>(x, rows, n, xq, xd, xsum);
    QMA_CHECK_LAUNCH();
    return QMA_CUDA_OK;
}

int qma_cuda_matvec(int wtype, const void *W, int n_in, int n_out, int T, const int8_t *xq,
                    const float *xd, const int16_t *xsum, float *out, void *stream) {
    qma::clear_error();
    QMA_REQUIRE(W && xq && xd && xsum && out && n_in > 0 && n_in % 256 == 0 && n_out > 0 && T > 0,
                "qma_cuda_matvec: bad arguments (n_in %d, n_out %d, T %d)", n_in, n_out, T);
    QMA_REQUIRE(qma::aligned_to(W, 16) && qma::aligned_to(xq, 16) && qma::aligned_to(xd, 16) &&
                    qma::aligned_to(xsum, 16) && qma::aligned_to(out, 16),
                "qma_cuda_matvec: device buffers must be 16-byte aligned");
    return qma::matvec(wtype, W, n_in, n_out, T, xq, xd, xsum, out, qma::as_stream(stream));
}

int qma_cuda_dot_partials(int wtype, const void *W, int n_in, int n_out, const int8_t *xq,
                          int32_t *isum, void *stream) {
    qma::clear_error();
    QMA_REQUIRE(W && xq && isum && n_in > 0 && n_in % 256 == 0 && n_out > 0,
                "qma_cuda_dot_partials: bad arguments");
    cudaStream_t st = qma::as_stream(stream);
    // xd / xsum do not enter the integer partials; give the loaders a
    // harmless zero buffer of the right size.
    static float *dummy_xd = nullptr;
    static int16_t *dummy_xs = nullptr;
    static int dummy_n = 0;
    if (dummy_n < n_in) {
        cudaFree(dummy_xd);
        cudaFree(dummy_xs);
        QMA_CHECK_CUDA(cudaMalloc(&dummy_xd, sizeof(float) * (n_in / 256)));
        QMA_CHECK_CUDA(cudaMalloc(&dummy_xs, sizeof(int16_t) * (n_in / 16)));
        QMA_CHECK_CUDA(cudaMemset(dummy_xd, 0, sizeof(float) * (n_in / 256)));
        QMA_CHECK_CUDA(cudaMemset(dummy_xs, 0, sizeof(int16_t) * (n_in / 16)));
        dummy_n = n_in;
    }
    const int grid = 1024;
    switch (wtype) {
    case QMA_TYPE_Q4_K:
        qma::partials_kernel_safe<qma::FmtQ4K><<<grid, 256, 0, st>>>(
            static_cast<const uint8_t *>(W), n_in, n_out, xq, dummy_xd, dummy_xs, isum);
        break;
    case QMA_TYPE_Q6_K:
        QMA_CHECK_CUDA(cudaMemsetAsync(isum, 0, sizeof(int32_t) * size_t(n_out) * (n_in / 256), st));
        qma::partials_kernel_safe<qma::FmtQ6K><<<grid, 256, 0, st>>>(
            qma::q6_planes(W, n_out, n_in), n_in, n_out, xq, dummy_xd, dummy_xs, isum);
        break;
    case QMA_TYPE_Q8_0:
        qma::partials_kernel_safe<qma::FmtQ80><<<grid, 256, 0, st>>>(
            qma::q8_planes(W, n_out, n_in), n_in, n_out, xq, dummy_xd, dummy_xs, isum);
        break;
    default:
        qma::set_error("qma_cuda_dot_partials: unsupported weight type %d", wtype);
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
    QMA_CHECK_LAUNCH();
    return QMA_CUDA_OK;
}

}  // extern "C"
