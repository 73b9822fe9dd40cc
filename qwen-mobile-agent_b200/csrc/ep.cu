// ep.cu -- the MoE FFN block with expert parallelism: the 256 experts of a
// layer are sharded 256 / N per rank (rank r owns experts r * 256/N ..), the
// router, the shared expert and the combine stay on the rank that owns the
// token, and the (token, expert) work crosses NVLink twice per layer through
// NCCL point-to-point transfers:
//
//   1. moe_route          : RMSNorm, Q8_K of the normed input, exact top-8
//                           (the reference's moe_ffn router, nn.c:513-551);
//   2. ep_plan_kernel     : per destination rank, the tokens that have at
//                           least one expert there (token order) and the
//                           return row of every (token, k) pair;
//   3. ep_pack_kernel     : one Q8_K row (2048 + 32 + 256 bytes) per
//                           (token, destination), deduplicated over the k,
//                           with the token's 8 shard-local expert ids
//                           (-1 where another rank owns the expert);
//   4. the dispatch: grouped ncclSend / ncclRecv of fixed blocks of t_max
//      rows per destination (padding rows carry no expert), rows landing in
//      the receiver's scratch in source rank order (or, with the counted
//      exchange, an all-gather of the [N][2] counts read on the host and
//      exact-size transfers);
//   5. the grouped expert pipeline (moe_grouped.cu) on the received rows,
//      groups = the shard's experts (counted exchange: ep_recv_plan_kernel /
//      ep_gather_kernel pack each owned pair's down projection in (row, k)
//      order, the source's pair order);
//   6. the return transfer (the blocks' slot partials whole, or the packed
//      pairs), ep_unpack_fixed_kernel / ep_unpack_kernel into the source's
//      slot partials, the shared expert on the source's own tokens, and the
//      combine in the reference's order (moe_xpar_worker + combine,
//      nn.c:604-629, 652-707; residual nn.c:2246-2252).
//
// Every pair is computed by the same kernels, on the same bytes, as on one
// GPU, and the combine reads the slots in the same order: the result equals
// qma_cuda_moe_layer's grouped path bit for bit.
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "moe.cuh"

namespace qma {

constexpr int EP_MAX_RANKS = 8;
constexpr int EP_MAX_T = 256;                  // tokens per rank and call
constexpr int EP_ROW_META = MOE_TOPK;          // shard-local expert ids per row

// 2. --------------------------------------------------------------- plan --
// One CTA, thread t = token.  tokidx[t][d]: the token's row in the send
// buffer of rank d (-1: nothing to send there); srcrow[t * 8 + k]: the row
// of the return buffer that will hold pair (t, k); cnt[d] = {rows, pairs}
// sent to rank d.  The return buffer holds rank 0's pairs first, each
// rank's in (token, k) order.
__global__ void __launch_bounds__(EP_MAX_T) ep_plan_kernel(const int *__restrict__ sel, int T, int n, int n_local,
                                                          int *tokidx, int *srcrow, int *cnt) {
    __shared__ unsigned char smask[EP_MAX_T];
    __shared__ unsigned char spc[EP_MAX_T][EP_MAX_RANKS];
    __shared__ int tbase[EP_MAX_T][EP_MAX_RANKS], pbase[EP_MAX_T][EP_MAX_RANKS];
    __shared__ int dpairs[EP_MAX_RANKS], dpoff[EP_MAX_RANKS];
    const int t = threadIdx.x;
    int owner[MOE_TOPK];
    if (t < T) {
        unsigned m = 0;
        unsigned char pc[EP_MAX_RANKS] = {};
#pragma unroll
        for (int k = 0; k < MOE_TOPK; k++) {
            owner[k] = sel[t * MOE_TOPK + k] / n_local;
            m |= 1u << owner[k];
            pc[owner[k]]++;
        }
        smask[t] = static_cast<unsigned char>(m);
#pragma unroll
        for (int d = 0; d < EP_MAX_RANKS; d++) spc[t][d] = pc[d];
    }
    __syncthreads();
    if (t < n) {
        const int d = t;
        int nt = 0, np = 0;
        for (int u = 0; u < T; u++) {
            const int bit = (smask[u] >> d) & 1;
            tbase[u][d] = bit ? nt : -1;
            nt += bit;
            pbase[u][d] = np;
            np += spc[u][d];
        }
        cnt[2 * d] = nt;
        cnt[2 * d + 1] = np;
        dpairs[d] = np;
    }
    __syncthreads();
    if (t == 0) {
        int o = 0;
        for (int d = 0; d < n; d++) {
            dpoff[d] = o;
            o += dpairs[d];
        }
    }
    __syncthreads();
    if (t < T) {
        for (int d = 0; d < n; d++) tokidx[t * EP_MAX_RANKS + d] = tbase[t][d];
        int seen[EP_MAX_RANKS] = {};
#pragma unroll
        for (int k = 0; k < MOE_TOPK; k++) {
            const int d = owner[k];
            int idx = 0;
#pragma unroll
            for (int j = 0; j < EP_MAX_RANKS; j++)
                if (j == d) idx = seen[j]++;
            srcrow[t * MOE_TOPK + k] = dpoff[d] + pbase[t][d] + idx;
        }
    }
}

// Send buffers, one region of t_max rows per destination rank.
struct EpSend {
    int8_t *xq;      // [N][t_max][2048]
    float *xd;       // [N][t_max][8]
    int16_t *xs;     // [N][t_max][128]
    int *meta;       // [N][t_max][8] shard-local expert id or -1
};

// 3. --------------------------------------------------------------- pack --
// Grid (T, N), 128 threads: the Q8_K row of token t for rank d.
__global__ void __launch_bounds__(128) ep_pack_kernel(MoeScratch s, const int *__restrict__ tokidx, int t_max,
                                                      int n_local, EpSend b) {
    const int t = blockIdx.x, d = blockIdx.y, tid = threadIdx.x;
    const int j = tokidx[t * EP_MAX_RANKS + d];
    if (j < 0) return;
    const size_t row = size_t(d) * t_max + j;
    reinterpret_cast<int4 *>(b.xq + row * MOE_EMBD)[tid] =
        reinterpret_cast<const int4 *>(s.xq + size_t(t) * MOE_EMBD)[tid];
    if (tid < MOE_EMBD / 16 / 8)      // 128 int16 = 16 int4
        reinterpret_cast<int4 *>(b.xs + row * (MOE_EMBD / 16))[tid] =
            reinterpret_cast<const int4 *>(s.xs + size_t(t) * (MOE_EMBD / 16))[tid];
    if (tid < MOE_EMBD / 256) b.xd[row * (MOE_EMBD / 256) + tid] = s.xd[size_t(t) * (MOE_EMBD / 256) + tid];
    if (tid < MOE_TOPK) {
        const int e = s.sel[t * MOE_TOPK + tid];
        b.meta[row * EP_ROW_META + tid] = e / n_local == d ? e - d * n_local : -1;
    }
}

// 5. ------------------------------------------------ receiver's pair rows --
// One CTA over the R x 8 (row, k) entries, 16 per thread: prow = the pair's
// row in the return buffer ((row, k) order over owned pairs), or -1.
__global__ void __launch_bounds__(256) ep_recv_plan_kernel(const int *__restrict__ meta, int R, int *prow) {
    __shared__ int wsum[8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n = R * MOE_TOPK, per = 16, i0 = tid * per;
    int c = 0;
    for (int i = i0; i < i0 + per && i < n; i++) c += meta[i] >= 0;
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    int base = incl - c;
    for (int w = 0; w < warp; w++) base += wsum[w];
    for (int i = i0; i < i0 + per && i < n; i++) prow[i] = meta[i] >= 0 ? base++ : -1;
}

// Grid (R * 8), 256 threads: pair q's down projection into its return row.
__global__ void __launch_bounds__(256) ep_gather_kernel(const float *__restrict__ part, const int *__restrict__ prow,
                                                        float *ret) {
    const int q = blockIdx.x, r = prow[q];
    if (r < 0) return;
    const int i = q / MOE_TOPK, k = q % MOE_TOPK;
    const float4 *src = reinterpret_cast<const float4 *>(part + (size_t(i) * MOE_NSLOT + k) * MOE_EMBD);
    float4 *dst = reinterpret_cast<float4 *>(ret + size_t(r) * MOE_EMBD);
    dst[threadIdx.x] = src[threadIdx.x];
    dst[threadIdx.x + 256] = src[threadIdx.x + 256];
}

// 6. ------------------------------------------------------------- unpack --
// Grid (T * 8), 256 threads: slot k of token t from its return row.
__global__ void __launch_bounds__(256) ep_unpack_kernel(const float *__restrict__ ret, const int *__restrict__ srcrow,
                                                        float *part) {
    const int q = blockIdx.x, t = q / MOE_TOPK, k = q % MOE_TOPK;
    const float4 *src = reinterpret_cast<const float4 *>(ret + size_t(srcrow[q]) * MOE_EMBD);
    float4 *dst = reinterpret_cast<float4 *>(part + (size_t(t) * MOE_NSLOT + k) * MOE_EMBD);
    dst[threadIdx.x] = src[threadIdx.x];
    dst[threadIdx.x + 256] = src[threadIdx.x + 256];
}

// 6'. ----------------------------------------------- unpack, fixed blocks --
// The fixed-capacity exchange returns, from each rank d, the slot partials
// of the whole block of rows this rank sent it: row j of block d holds
// token t's pairs at its slots k (those whose expert d owns).  Grid (T * 8),
// 256 threads: slot k of token t from its owner's block.
__global__ void __launch_bounds__(256) ep_unpack_fixed_kernel(const float *__restrict__ ret,
                                                              const int *__restrict__ sel,
                                                              const int *__restrict__ tokidx, int n_local, int t_max,
                                                              float *part) {
    const int q = blockIdx.x, t = q / MOE_TOPK, k = q % MOE_TOPK;
    const int d = sel[q] / n_local, j = tokidx[t * EP_MAX_RANKS + d];
    const float4 *src =
        reinterpret_cast<const float4 *>(ret + ((size_t(d) * t_max + j) * MOE_NSLOT + k) * MOE_EMBD);
    float4 *dst = reinterpret_cast<float4 *>(part + (size_t(t) * MOE_NSLOT + k) * MOE_EMBD);
    dst[threadIdx.x] = src[threadIdx.x];
    dst[threadIdx.x + 256] = src[threadIdx.x + 256];
}

}  // namespace qma

struct qma_cuda_ep {
    int device = 0, rank = 0, n = 1, t_max = 0, n_local = 0, r_max = 0;
    ncclComm_t comm = nullptr;
    std::vector<void *> allocs;
    qma::MoeScratch sl{}, sr{};       // own tokens; received rows
    qma::EpSend snd{};
    float *ret_send = nullptr, *ret_recv = nullptr;
    float *ret_fixed = nullptr;       // [N][t_max][9][2048]: the blocks' slot partials, returned
    int *tokidx = nullptr, *srcrow = nullptr, *cnt = nullptr, *allcnt = nullptr, *prow = nullptr;
    int *h_allcnt = nullptr;          // pinned [N][N][2]
    uint64_t sent = 0, recvd = 0;     // bytes of the last call
    int rows_in = 0;
    int timeout_ms = 0;               // wall-clock limit of every host-side wait
    bool aborted = false;             // the communicator was aborted after a failure
};

namespace {

using Clock = std::chrono::steady_clock;

int ms_since(Clock::time_point t0) {
    return int(std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count());
}

// Ends the communicator after a failure or a timeout: its peers' pending
// operations fail instead of waiting for this rank forever.
void ep_abort(qma_cuda_ep *ep) {
    if (ep->comm && !ep->aborted) ncclCommAbort(ep->comm);
    ep->comm = nullptr;
    ep->aborted = true;
}

// The communicator is non-blocking: a call may return ncclInProgress while
// it connects to its peers (the first transfer to a peer sets up that
// connection).  Poll its state until it settles, for at most the handle's
// wall-clock limit; a peer that never answers aborts the communicator and
// fails the call with QMA_CUDA_ERR_TIMEOUT.
int ep_settle(qma_cuda_ep *ep, ncclResult_t r, const char *what) {
    const Clock::time_point t0 = Clock::now();
    while (r == ncclInProgress) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t q = ncclCommGetAsyncError(ep->comm, &st);
        r = q != ncclSuccess ? q : st;
        if (r != ncclInProgress) break;
        const int el = ms_since(t0);
        if (el > ep->timeout_ms) {
            ep_abort(ep);
            qma::set_error("%s: no answer from the other ranks within %d ms (communicator aborted)", what,
                           ep->timeout_ms);
            return QMA_CUDA_ERR_TIMEOUT;
        }
        // a transfer enqueue settles within microseconds: poll without
        // sleeping at first, then back off (connection set-up, a slow peer)
        if (el < 20) std::this_thread::yield();
        else std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
    if (r == ncclSuccess) return QMA_CUDA_OK;
    qma::set_error("%s: %s", what, ncclGetErrorString(r));
    ep_abort(ep);
    return QMA_CUDA_ERR_CUDA;
}
#define EP_NCCL(call)                                        \
    do {                                                     \
        int rc_ = ep_settle(ep, (call), #call);              \
        if (rc_) return rc_;                                 \
    } while (0)

// The stream's work (including transfers that wait on other ranks) done,
// for at most the wall-clock limit; an asynchronous communicator error or
// the limit aborts the communicator.
int ep_sync(qma_cuda_ep *ep, cudaStream_t st) {
    const Clock::time_point t0 = Clock::now();
    for (;;) {
        const cudaError_t e = cudaStreamQuery(st);
        if (e == cudaSuccess) return QMA_CUDA_OK;
        if (e != cudaErrorNotReady) {
            qma::set_error("qma_cuda_ep_moe_layer: %s", cudaGetErrorString(e));
            return QMA_CUDA_ERR_CUDA;
        }
        ncclResult_t as = ncclSuccess;
        if (ncclCommGetAsyncError(ep->comm, &as) != ncclSuccess || (as != ncclSuccess && as != ncclInProgress)) {
            qma::set_error("qma_cuda_ep_moe_layer: communicator error: %s", ncclGetErrorString(as));
            ep_abort(ep);
            return QMA_CUDA_ERR_CUDA;
        }
        const int el = ms_since(t0);
        if (el > ep->timeout_ms) {
            ep_abort(ep);
            qma::set_error("qma_cuda_ep_moe_layer: the exchange did not finish within %d ms (communicator aborted)",
                           ep->timeout_ms);
            return QMA_CUDA_ERR_TIMEOUT;
        }
        if (el < 20) std::this_thread::yield();
        else std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

int ep_alloc(qma_cuda_ep *ep, size_t bytes, void **out) {
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        qma::set_error("qma_cuda_ep_init: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
        return QMA_CUDA_ERR_NOMEM;
    }
    ep->allocs.push_back(p);
    *out = p;
    return QMA_CUDA_OK;
}

void ep_release(qma_cuda_ep *ep) {
    if (ep->comm) {
        // a communicator whose peers may be gone cannot be finalized
        // collectively: abort it instead of waiting for them
        if (ep->aborted) ncclCommAbort(ep->comm);
        else ncclCommDestroy(ep->comm);
    }
    for (void *p : ep->allocs) cudaFree(p);
    if (ep->h_allcnt) cudaFreeHost(ep->h_allcnt);
    delete ep;
}

}  // namespace

// QMA_CUDA_EP_COUNTED=1 in the environment: the counted exchange (the
// [N][2] counts all-gathered and read on the host, exact-size transfers,
// one host synchronisation per layer) instead of the fixed-capacity one;
// the same results, fewer bytes on NVLink.
static bool ep_counted() {
    const char *v = getenv("QMA_CUDA_EP_COUNTED");
    return v && atoi(v) != 0;
}

// The fixed-capacity exchange: every rank sends every rank (itself
// included) its whole block of t_max rows, padding rows carrying no
// shard-local expert (ids -1), so no count has to reach the host; the
// receiver runs the grouped experts over all N * t_max rows (the expert
// lists skip the padding) and returns each block's slot partials whole.
// Nothing in a call waits on the host: a step of layers is queued back to
// back (and can be captured in a CUDA graph); qma_cuda_ep_sync is the
// bounded wait for its end.
static int ep_moe_fixed(qma_cuda_ep *ep, const qma_cuda_moe_weights *w, const float *x2, int T, float *x_out, int32_t *sel,
                 float *wts, cudaStream_t st) {
    using namespace qma;
    const int n = ep->n, tm = ep->t_max, R = n * tm;
    int rc;
    QMA_CHECK_CUDA(cudaMemsetAsync(ep->snd.meta, 0xff, sizeof(int) * size_t(R) * EP_ROW_META, st));
    if (T > 0) {
        if ((rc = moe_route(*w, x2, T, ep->sl, sel, wts, st))) return rc;
        ep_plan_kernel<<<1, EP_MAX_T, 0, st>>>(ep->sl.sel, T, n, ep->n_local, ep->tokidx, ep->srcrow, ep->cnt);
        QMA_CHECK_LAUNCH();
        ep_pack_kernel<<<dim3(T, n), 128, 0, st>>>(ep->sl, ep->tokidx, tm, ep->n_local, ep->snd);
        QMA_CHECK_LAUNCH();
    }
    const size_t row_bytes = MOE_EMBD + 4 * (MOE_EMBD / 256) + 2 * (MOE_EMBD / 16) + 4 * EP_ROW_META;
    EP_NCCL(ncclGroupStart());
    for (int d = 0; d < n; d++) {
        const size_t row = size_t(d) * tm, c = size_t(tm);
        EP_NCCL(ncclSend(ep->snd.xq + row * MOE_EMBD, c * MOE_EMBD, ncclInt8, d, ep->comm, st));
        EP_NCCL(ncclSend(ep->snd.xd + row * (MOE_EMBD / 256), c * (MOE_EMBD / 256), ncclFloat32, d, ep->comm, st));
        EP_NCCL(ncclSend(ep->snd.xs + row * (MOE_EMBD / 16), c * (MOE_EMBD / 16) * 2, ncclInt8, d, ep->comm, st));
        EP_NCCL(ncclSend(ep->snd.meta + row * EP_ROW_META, c * EP_ROW_META, ncclInt32, d, ep->comm, st));
    }
    for (int s = 0; s < n; s++) {
        const size_t row = size_t(s) * tm, c = size_t(tm);
        EP_NCCL(ncclRecv(ep->sr.xq + row * MOE_EMBD, c * MOE_EMBD, ncclInt8, s, ep->comm, st));
        EP_NCCL(ncclRecv(ep->sr.xd + row * (MOE_EMBD / 256), c * (MOE_EMBD / 256), ncclFloat32, s, ep->comm, st));
        EP_NCCL(ncclRecv(ep->sr.xs + row * (MOE_EMBD / 16), c * (MOE_EMBD / 16) * 2, ncclInt8, s, ep->comm, st));
        EP_NCCL(ncclRecv(ep->sr.sel + row * EP_ROW_META, c * EP_ROW_META, ncclInt32, s, ep->comm, st));
    }
    EP_NCCL(ncclGroupEnd());
    if ((rc = moe_grouped_range(*w, R, ep->sr, st, 0, ep->n_local, true, 0, R * MOE_TOPK))) return rc;
    // the shared expert of the own tokens needs no exchange
    if (T > 0 && (rc = moe_grouped_range(*w, T, ep->sl, st, MOE_NEXP, 1, false, T * MOE_TOPK, T))) return rc;
    const size_t blk = size_t(tm) * MOE_NSLOT * MOE_EMBD;
    EP_NCCL(ncclGroupStart());
    for (int s = 0; s < n; s++) EP_NCCL(ncclSend(ep->sr.part + s * blk, blk, ncclFloat32, s, ep->comm, st));
    for (int d = 0; d < n; d++) EP_NCCL(ncclRecv(ep->ret_fixed + d * blk, blk, ncclFloat32, d, ep->comm, st));
    EP_NCCL(ncclGroupEnd());
    if (T > 0) {
        ep_unpack_fixed_kernel<<<T * MOE_TOPK, 256, 0, st>>>(ep->ret_fixed, ep->sl.sel, ep->tokidx, ep->n_local, tm,
                                                             ep->sl.part);
        QMA_CHECK_LAUNCH();
        if ((rc = moe_combine(ep->sl, x2, x_out, T, st))) return rc;
    }
    ep->sent = ep->recvd = uint64_t(n) * (tm * row_bytes + blk * 4);
    ep->rows_in = -1;
    return QMA_CUDA_OK;
}

extern "C" {

int qma_cuda_ep_sync(qma_cuda_ep *ep, void *stream) {
    qma::clear_error();
    QMA_REQUIRE(ep, "qma_cuda_ep_sync: null handle");
    QMA_REQUIRE(!ep->aborted && ep->comm, "qma_cuda_ep_sync: the communicator was aborted after a failure");
    return ep_sync(ep, qma::as_stream(stream));
}

int qma_cuda_ep_unique_id(uint8_t *uid) {
    qma::clear_error();
    QMA_REQUIRE(uid, "qma_cuda_ep_unique_id: null output");
    ncclUniqueId id;
    const ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) {
        qma::set_error("qma_cuda_ep_unique_id: %s", ncclGetErrorString(r));
        return QMA_CUDA_ERR_CUDA;
    }
    static_assert(sizeof(id) == QMA_CUDA_EP_UID_BYTES, "NCCL unique id size");
    memcpy(uid, &id, sizeof(id));
    return QMA_CUDA_OK;
}

int qma_cuda_ep_init_timeout(int device, const uint8_t *uid, int rank, int n_ranks, int t_max, int timeout_ms,
                             qma_cuda_ep **out);

int qma_cuda_ep_init(int device, const uint8_t *uid, int rank, int n_ranks, int t_max, qma_cuda_ep **out) {
    const char *env = getenv("QMA_CUDA_EP_TIMEOUT_MS");
    const int ms = env && atoi(env) > 0 ? atoi(env) : 300000;
    return qma_cuda_ep_init_timeout(device, uid, rank, n_ranks, t_max, ms, out);
}

int qma_cuda_ep_init_timeout(int device, const uint8_t *uid, int rank, int n_ranks, int t_max, int timeout_ms,
                             qma_cuda_ep **out) {
    qma::clear_error();
    QMA_REQUIRE(timeout_ms > 0, "qma_cuda_ep_init: timeout %d ms must be positive", timeout_ms);
    QMA_REQUIRE(uid && out, "qma_cuda_ep_init: null argument");
    QMA_REQUIRE(n_ranks >= 1 && n_ranks <= qma::EP_MAX_RANKS && qma::MOE_NEXP % n_ranks == 0,
                "qma_cuda_ep_init: %d ranks (1..8, dividing 256)", n_ranks);
    QMA_REQUIRE(rank >= 0 && rank < n_ranks, "qma_cuda_ep_init: rank %d of %d", rank, n_ranks);
    QMA_REQUIRE(t_max >= 1 && t_max <= qma::EP_MAX_T && t_max * n_ranks <= qma::MOE_GROUPED_MAX_T,
                "qma_cuda_ep_init: t_max %d (1..256, t_max x ranks <= 512)", t_max);
    *out = nullptr;
    QMA_CHECK_CUDA(cudaSetDevice(device));
    qma_cuda_ep *ep = new qma_cuda_ep;
    ep->device = device;
    ep->rank = rank;
    ep->n = n_ranks;
    ep->t_max = t_max;
    ep->n_local = qma::MOE_NEXP / n_ranks;
    ep->r_max = t_max * n_ranks;
    ep->timeout_ms = timeout_ms;
    using namespace qma;
    // both scratch views carry the grouped buffers (16 rows at least)
    const int tl = t_max < MOE_GROUPED_MIN_T ? MOE_GROUPED_MIN_T : t_max;
    const int tr = ep->r_max < MOE_GROUPED_MIN_T ? MOE_GROUPED_MIN_T : ep->r_max;
    const size_t rows = size_t(n_ranks) * t_max;
    void *p[13];
    int rc = 0;
    const size_t sizes[13] = {
        moe_scratch_bytes(tl), moe_scratch_bytes(tr),
        rows * MOE_EMBD, rows * sizeof(float) * (MOE_EMBD / 256), rows * sizeof(int16_t) * (MOE_EMBD / 16),
        rows * sizeof(int) * EP_ROW_META,
        size_t(ep->r_max) * MOE_TOPK * MOE_EMBD * sizeof(float), size_t(t_max) * MOE_TOPK * MOE_EMBD * sizeof(float),
        size_t(t_max) * EP_MAX_RANKS * sizeof(int), size_t(t_max) * MOE_TOPK * sizeof(int),
        sizeof(int) * (2 * n_ranks + 2 * n_ranks * n_ranks), size_t(ep->r_max) * MOE_TOPK * sizeof(int),
        size_t(ep->r_max) * MOE_NSLOT * MOE_EMBD * sizeof(float)};
    for (int i = 0; i < 13 && !rc; i++) {
        rc = ep_alloc(ep, sizes[i], &p[i]);
        // zeroed: the MoE scratch's tickets must start at zero (every call
        // leaves them zero again)
        if (!rc && cudaMemset(p[i], 0, sizes[i]) != cudaSuccess) {
            set_error("qma_cuda_ep_init: cudaMemset: %s", cudaGetErrorString(cudaGetLastError()));
            rc = QMA_CUDA_ERR_CUDA;
        }
    }
    if (!rc && cudaMallocHost(&ep->h_allcnt, sizeof(int) * 2 * n_ranks * n_ranks) != cudaSuccess) {
        ep->h_allcnt = nullptr;
        set_error("qma_cuda_ep_init: pinned host buffer");
        rc = QMA_CUDA_ERR_NOMEM;
    }
    if (rc) {
        ep_release(ep);
        return rc;
    }
    ep->sl = moe_scratch_layout(p[0], tl);
    ep->sr = moe_scratch_layout(p[1], tr);
    ep->snd = EpSend{static_cast<int8_t *>(p[2]), static_cast<float *>(p[3]), static_cast<int16_t *>(p[4]),
                     static_cast<int *>(p[5])};
    ep->ret_send = static_cast<float *>(p[6]);
    ep->ret_recv = static_cast<float *>(p[7]);
    ep->tokidx = static_cast<int *>(p[8]);
    ep->srcrow = static_cast<int *>(p[9]);
    ep->cnt = static_cast<int *>(p[10]);
    ep->allcnt = ep->cnt + 2 * n_ranks;
    ep->prow = static_cast<int *>(p[11]);
    ep->ret_fixed = static_cast<float *>(p[12]);
    ncclUniqueId id;
    memcpy(&id, uid, sizeof(id));
    // non-blocking initialisation, polled against the wall-clock limit: a
    // rank that never joins fails the others' init instead of hanging it
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&ep->comm, n_ranks, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        ep->comm = nullptr;
        ep_release(ep);
        set_error("qma_cuda_ep_init: ncclCommInitRankConfig: %s", ncclGetErrorString(r));
        return QMA_CUDA_ERR_CUDA;
    }
    if ((rc = ep_settle(ep, r, "qma_cuda_ep_init"))) {
        const std::string msg = qma_cuda_last_error();
        ep_release(ep);
        set_error("%s", msg.c_str());
        return rc;
    }
    *out = ep;
    return QMA_CUDA_OK;
}

int qma_cuda_ep_free(qma_cuda_ep *ep) {
    qma::clear_error();
    if (!ep) return QMA_CUDA_OK;
    cudaSetDevice(ep->device);
    ep_release(ep);
    return QMA_CUDA_OK;
}

int qma_cuda_ep_moe_layer(qma_cuda_ep *ep, const qma_cuda_moe_weights *w, const float *x2, int T, float *x_out,
                          int32_t *sel, float *wts, void *stream) {
    using namespace qma;
    clear_error();
    QMA_REQUIRE(ep && w && x2 && x_out, "qma_cuda_ep_moe_layer: null argument");
    QMA_REQUIRE(aligned_to(x2, 16) && aligned_to(x_out, 16), "qma_cuda_ep_moe_layer: x2 / x_out must be 16-byte aligned");
    QMA_REQUIRE(T >= 0 && T <= ep->t_max, "qma_cuda_ep_moe_layer: T %d (0..%d)", T, ep->t_max);
    QMA_REQUIRE(w->post_norm && w->gate_inp && w->gate_exps && w->up_exps && w->down_exps && w->gate_inp_shexp &&
                    w->gate_shexp && w->up_shexp && w->down_shexp,
                "qma_cuda_ep_moe_layer: missing weight pointer");
    QMA_REQUIRE(w->down_type == QMA_TYPE_Q6_K && w->down_shexp_type == QMA_TYPE_Q6_K,
                "qma_cuda_ep_moe_layer: down projections must be Q6_K");
    QMA_REQUIRE(!ep->aborted && ep->comm, "qma_cuda_ep_moe_layer: the communicator was aborted after a failure");
    cudaStream_t st = as_stream(stream);
    if (!ep_counted()) return ep_moe_fixed(ep, w, x2, T, x_out, sel, wts, st);
    const int n = ep->n, me = ep->rank;
    int rc;
    // 1-3: route, plan, pack (T == 0: this rank only serves others)
    if (T > 0) {
        if ((rc = moe_route(*w, x2, T, ep->sl, sel, wts, st))) return rc;
        ep_plan_kernel<<<1, EP_MAX_T, 0, st>>>(ep->sl.sel, T, n, ep->n_local, ep->tokidx, ep->srcrow, ep->cnt);
        QMA_CHECK_LAUNCH();
        ep_pack_kernel<<<dim3(T, n), 128, 0, st>>>(ep->sl, ep->tokidx, ep->t_max, ep->n_local, ep->snd);
        QMA_CHECK_LAUNCH();
    } else {
        QMA_CHECK_CUDA(cudaMemsetAsync(ep->cnt, 0, sizeof(int) * 2 * n, st));
    }
    // 4: counts, then the dispatch
    EP_NCCL(ncclAllGather(ep->cnt, ep->allcnt, 2 * n, ncclInt32, ep->comm, st));
    QMA_CHECK_CUDA(cudaMemcpyAsync(ep->h_allcnt, ep->allcnt, sizeof(int) * 2 * n * n, cudaMemcpyDeviceToHost, st));
    if ((rc = ep_sync(ep, st))) return rc;
    const int *ac = ep->h_allcnt;      // ac[(src * n + dst) * 2 + {0 rows, 1 pairs}]
    auto rows_to = [&](int s, int d) { return ac[(s * n + d) * 2]; };
    auto pairs_to = [&](int s, int d) { return ac[(s * n + d) * 2 + 1]; };
    int R = 0;
    for (int s = 0; s < n; s++) R += rows_to(s, me);
    uint64_t sent = 0, recvd = 0;
    EP_NCCL(ncclGroupStart());
    for (int d = 0; d < n; d++) {
        const size_t c = size_t(rows_to(me, d)), row = size_t(d) * ep->t_max;
        if (!c) continue;
        EP_NCCL(ncclSend(ep->snd.xq + row * MOE_EMBD, c * MOE_EMBD, ncclInt8, d, ep->comm, st));
        EP_NCCL(ncclSend(ep->snd.xd + row * (MOE_EMBD / 256), c * (MOE_EMBD / 256), ncclFloat32, d, ep->comm, st));
        EP_NCCL(ncclSend(ep->snd.xs + row * (MOE_EMBD / 16), c * (MOE_EMBD / 16) * 2, ncclInt8, d, ep->comm, st));
        EP_NCCL(ncclSend(ep->snd.meta + row * EP_ROW_META, c * EP_ROW_META, ncclInt32, d, ep->comm, st));
        sent += c * (MOE_EMBD + 4 * (MOE_EMBD / 256) + 2 * (MOE_EMBD / 16) + 4 * EP_ROW_META);
    }
    for (int s = 0, off = 0; s < n; off += rows_to(s, me), s++) {
        const size_t c = size_t(rows_to(s, me));
        if (!c) continue;
        EP_NCCL(ncclRecv(ep->sr.xq + size_t(off) * MOE_EMBD, c * MOE_EMBD, ncclInt8, s, ep->comm, st));
        EP_NCCL(ncclRecv(ep->sr.xd + size_t(off) * (MOE_EMBD / 256), c * (MOE_EMBD / 256), ncclFloat32, s, ep->comm, st));
        EP_NCCL(ncclRecv(ep->sr.xs + size_t(off) * (MOE_EMBD / 16), c * (MOE_EMBD / 16) * 2, ncclInt8, s, ep->comm, st));
        EP_NCCL(ncclRecv(ep->sr.sel + size_t(off) * EP_ROW_META, c * EP_ROW_META, ncclInt32, s, ep->comm, st));
        recvd += c * (MOE_EMBD + 4 * (MOE_EMBD / 256) + 2 * (MOE_EMBD / 16) + 4 * EP_ROW_META);
    }
    EP_NCCL(ncclGroupEnd());
    // 5: the shard's experts over the received rows, packed for the return
    if (R > 0) {
        if ((rc = moe_grouped_range(*w, R, ep->sr, st, 0, ep->n_local, true, 0, R * MOE_TOPK))) return rc;
        ep_recv_plan_kernel<<<1, 256, 0, st>>>(ep->sr.sel, R, ep->prow);
        QMA_CHECK_LAUNCH();
        ep_gather_kernel<<<R * MOE_TOPK, 256, 0, st>>>(ep->sr.part, ep->prow, ep->ret_send);
        QMA_CHECK_LAUNCH();
    }
    // the shared expert of the own tokens meanwhile needs no exchange
    if (T > 0 && (rc = moe_grouped_range(*w, T, ep->sl, st, MOE_NEXP, 1, false, T * MOE_TOPK, T)))
        return rc;
    // 6: the return
    EP_NCCL(ncclGroupStart());
    for (int s = 0, off = 0; s < n; off += pairs_to(s, me), s++) {
        const size_t c = size_t(pairs_to(s, me));
        if (!c) continue;
        EP_NCCL(ncclSend(ep->ret_send + size_t(off) * MOE_EMBD, c * MOE_EMBD, ncclFloat32, s, ep->comm, st));
        sent += c * MOE_EMBD * 4;
    }
    for (int d = 0, off = 0; d < n; off += pairs_to(me, d), d++) {
        const size_t c = size_t(pairs_to(me, d));
        if (!c) continue;
        EP_NCCL(ncclRecv(ep->ret_recv + size_t(off) * MOE_EMBD, c * MOE_EMBD, ncclFloat32, d, ep->comm, st));
        recvd += c * MOE_EMBD * 4;
    }
    EP_NCCL(ncclGroupEnd());
    if (T > 0) {
        ep_unpack_kernel<<<T * MOE_TOPK, 256, 0, st>>>(ep->ret_recv, ep->srcrow, ep->sl.part);
        QMA_CHECK_LAUNCH();
        if ((rc = moe_combine(ep->sl, x2, x_out, T, st))) return rc;
    }
    ep->sent = sent;
    ep->recvd = recvd;
    ep->rows_in = R;
    return QMA_CUDA_OK;
}

int qma_cuda_ep_stats(const qma_cuda_ep *ep, uint64_t *sent_bytes, uint64_t *recv_bytes, int *rows_in) {
    qma::clear_error();
    QMA_REQUIRE(ep, "qma_cuda_ep_stats: null handle");
    if (sent_bytes) *sent_bytes = ep->sent;
    if (recv_bytes) *recv_bytes = ep->recvd;
    if (rows_in) *rows_in = ep->rows_in;
    return QMA_CUDA_OK;
}

}  // extern "C"
