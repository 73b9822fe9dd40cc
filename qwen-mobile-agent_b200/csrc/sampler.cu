// sampler.cu -- the first phase of qma's sampler on the GPU: repeat
// penalty, temperature and the top-k candidate list (sampler_candidates,
// sampler.c:36-95), computed from device logits so that only the k
// candidates (not the 151936 logits) cross to the host, where the grammar
// mask and sampler_pick (sampler.c:100-134) run as before.
//
// One CTA of 1024 threads: a 4-pass radix select (8 bits per pass) over the
// order-preserving integer keys of the scaled logits finds the k-th largest
// value exactly, a block scan collects the candidates, and one thread sorts
// them.  The scaled logit of every token is recomputed in each pass from the
// input (no scratch copy): l = logits[i], the penalty applied once per
// occurrence of i among the last tokens in their order, then l / temp --
// the reference's operations in its order, so the values are bit-identical.
#include "common.cuh"

namespace qma {

constexpr int SMP_THREADS = 1024;
constexpr int SMP_MAX_K = 64;        // QMA_CUDA_SAMPLE_MAX_K
constexpr int SMP_MAX_LAST = 64;     // sampler_t::last_tokens (qma.h:285)
constexpr int SMP_MAX_VOCAB = 1 << 18;

struct SmpArgs {
    int last[SMP_MAX_LAST];
    int n_last;
    float penalty, temp;
    int k;
};

__device__ int g_smp_ids[SMP_MAX_K];
__device__ float g_smp_lgs[SMP_MAX_K];

// float -> unsigned key with the same order (larger float, larger key);
// -0.0f maps to the key of +0.0f, since the reference's float comparisons
// treat the two as equal
__device__ __forceinline__ unsigned order_key(float f) {
    const unsigned b = __float_as_uint(f == 0.0f ? 0.0f : f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void __launch_bounds__(SMP_THREADS, 1) sample_topk_kernel(const float *__restrict__ logits, int n,
                                                                   SmpArgs a) {
    __shared__ unsigned pen_bits[SMP_MAX_VOCAB / 32];   // tokens among the last ones
    __shared__ int pen_id[SMP_MAX_LAST];
    __shared__ float pen_val[SMP_MAX_LAST];
    __shared__ int n_pen;
    __shared__ unsigned hist[256];
    __shared__ unsigned s_prefix;
    __shared__ int s_remaining;
    __shared__ int wsum[2][SMP_THREADS / 32];
    __shared__ int c_id[SMP_MAX_K];
    __shared__ float c_val[SMP_MAX_K];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool use_pen = a.penalty != 1.0f;
    for (int i = tid; i < (n + 31) / 32; i += SMP_THREADS) pen_bits[i] = 0u;
    __syncthreads();
    if (tid == 0) {
        // the penalised logit of each distinct last token, occurrences in order
        int m = 0;
        if (use_pen)
            for (int j = 0; j < a.n_last; j++) {
                const int id = a.last[j];
                if (id < 0 || id >= n) continue;
                int slot = -1;
                for (int u = 0; u < m; u++)
                    if (pen_id[u] == id) slot = u;
                if (slot < 0) {
                    slot = m++;
                    pen_id[slot] = id;
                    pen_val[slot] = logits[id];
                    pen_bits[id >> 5] |= 1u << (id & 31);
                }
                float l = pen_val[slot];
                l = l < 0.0f ? l * a.penalty : l / a.penalty;
                pen_val[slot] = l;
            }
        n_pen = m;
        s_prefix = 0u;
        s_remaining = a.k;
    }
    __syncthreads();
    auto value = [&](int i) {
        float l = __ldg(logits + i);
        if ((pen_bits[i >> 5] >> (i & 31)) & 1u)
            for (int u = 0; u < n_pen; u++)
                if (pen_id[u] == i) l = pen_val[u];
        if (a.temp > 0.0f) l = l / a.temp;
        return l;
    };
    // ---- radix select of the k-th largest key, 8 bits at a time ------------
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = tid; b < 256; b += SMP_THREADS) hist[b] = 0u;
        __syncthreads();
        const unsigned prefix = s_prefix;
        const unsigned hi_mask = shift == 24 ? 0u : ~0u << (shift + 8);
        for (int i = tid; i < n; i += SMP_THREADS) {
            const unsigned key = order_key(value(i));
            if ((key & hi_mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            int rem = s_remaining;
            int b = 255;
            for (; b > 0; b--) {
                if (int(hist[b]) >= rem) break;
                rem -= int(hist[b]);
            }
            s_prefix = prefix | (unsigned(b) << shift);
            s_remaining = rem;
        }
        __syncthreads();
    }
    const unsigned thr = s_prefix;        // key of the k-th largest value
    const int ties_wanted = s_remaining;   // how many values equal to it are kept
    // ---- collect: contiguous id ranges, scanned in id order -----------------
    const int per = (n + SMP_THREADS - 1) / SMP_THREADS, i0 = tid * per, i1 = min(n, i0 + per);
    int ngt = 0, neq = 0;
    for (int i = i0; i < i1; i++) {
        const unsigned key = order_key(value(i));
        ngt += key > thr;
        neq += key == thr;
    }
    int gt_in = ngt, eq_in = neq;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int g = __shfl_up_sync(0xffffffffu, gt_in, o), e = __shfl_up_sync(0xffffffffu, eq_in, o);
        if (lane >= o) {
            gt_in += g;
            eq_in += e;
        }
    }
    if (lane == 31) {
        wsum[0][warp] = gt_in;
        wsum[1][warp] = eq_in;
    }
    __syncthreads();
    int gt_base = gt_in - ngt, eq_base = eq_in - neq, gt_total = 0;
    for (int w = 0; w < SMP_THREADS / 32; w++) {
        if (w < warp) {
            gt_base += wsum[0][w];
            eq_base += wsum[1][w];
        }
        gt_total += wsum[0][w];
    }
    if (ngt || (neq && eq_base < ties_wanted)) {
        for (int i = i0; i < i1; i++) {
            const float v = value(i);
            const unsigned key = order_key(v);
            if (key > thr) {
                c_id[gt_base] = i;
                c_val[gt_base++] = v;
            } else if (key == thr && eq_base < ties_wanted) {
                c_id[gt_total + eq_base] = i;
                c_val[gt_total + eq_base++] = v;
            }
        }
    }
    __syncthreads();
    // ---- sort: value descending, equal values by id -------------------------
    if (tid == 0) {
        for (int i = 1; i < a.k; i++) {
            const int id = c_id[i];
            const float v = c_val[i];
            int j = i - 1;
            while (j >= 0 && (c_val[j] < v || (c_val[j] == v && c_id[j] > id))) {
                c_id[j + 1] = c_id[j];
                c_val[j + 1] = c_val[j];
                j--;
            }
            c_id[j + 1] = id;
            c_val[j + 1] = v;
        }
    }
    __syncthreads();
    if (tid < a.k) {
        g_smp_ids[tid] = c_id[tid];
        g_smp_lgs[tid] = c_val[tid];
    }
}

}  // namespace qma

extern "C" {

int qma_cuda_sample_candidates(const float *logits, int n_vocab, const int32_t *last_tokens, int n_last,
                               float repeat_penalty, float temp, int top_k, int max_k, int32_t *ids,
                               float *lgs, int *n_out, void *stream) {
    using namespace qma;
    clear_error();
    QMA_REQUIRE(logits && ids && lgs && n_out && n_vocab > 0 && n_vocab <= SMP_MAX_VOCAB,
                "qma_cuda_sample_candidates: bad arguments (n_vocab %d)", n_vocab);
    QMA_REQUIRE(n_last >= 0 && n_last <= SMP_MAX_LAST && (n_last == 0 || last_tokens),
                "qma_cuda_sample_candidates: %d last tokens (0..64)", n_last);
    QMA_REQUIRE(max_k >= 1 && max_k <= SMP_MAX_K, "qma_cuda_sample_candidates: max_k %d (1..64)", max_k);
    SmpArgs a{};
    for (int i = 0; i < n_last; i++) a.last[i] = last_tokens[i];
    a.n_last = n_last;
    a.penalty = repeat_penalty;
    a.temp = temp;
    int k = top_k < 1 ? 1 : top_k;       // sampler.c:58-61
    if (k > n_vocab) k = n_vocab;
    if (k > max_k) k = max_k;
    a.k = k;
    cudaStream_t st = as_stream(stream);
    sample_topk_kernel<<<1, SMP_THREADS, 0, st>>>(logits, n_vocab, a);
    QMA_CHECK_LAUNCH();
    QMA_CHECK_CUDA(cudaMemcpyFromSymbolAsync(ids, g_smp_ids, sizeof(int32_t) * k, 0, cudaMemcpyDeviceToHost, st));
    QMA_CHECK_CUDA(cudaMemcpyFromSymbolAsync(lgs, g_smp_lgs, sizeof(float) * k, 0, cudaMemcpyDeviceToHost, st));
    QMA_CHECK_CUDA(cudaStreamSynchronize(st));
    *n_out = k;
    return QMA_CUDA_OK;
}

}  // extern "C"
