// attn.cuh -- launch interface of the quantized-KV attention kernels (attn.cu).
#pragma once
#include "common.cuh"
#include "layers.cuh"

namespace qma {

struct AttnArgs {
    const float *qr;          // [T][16][256] normed, rotated queries
    const uint8_t *kv;        // layer KV slab [4 heads][n_ctx][240]
    const uint8_t *arena;     // layer heavy-hitter arena [4 heads][2048][240]
    const int *live;          // live index (device)
    const StepParams *sp;
    int T;
    int nk_max;               // attended positions of the last query
    int pv_chunk;             // positions per softmax.V CTA
    float *scores;            // [T][16][nk_max]
    float *cmax;              // [T][16][ceil(nk_max/64)]
    float *opart;             // [T][16][nchunk][256]
    float *lpart;             // [T][16][nchunk]
    float *ml;                // [T][16][2] max, sum of p
    const float *z;           // [T][4096] gate
    int8_t *xq;               // [T][4096] Q8_K of the gated output
    float *xd;
    int16_t *xs;
    float *sal;               // this layer's ring salience [n_ctx]
    float *pin_sal;           // this layer's arena salience [2048]
};

// One sequence's arguments of the single-token attention kernels for one
// attention layer, in a device table indexed by blockIdx.z: the kernels of a
// batched step serve every sequence of the step in one launch each.
struct AttnRow {
    const StepParams *sp;
    const float *proj;        // the row's input projection (q | gate | k | v)
    const float *rope;
    float *qr, *z;            // the sequence's query / gate scratch
    uint8_t *kv;              // this layer's KV slab of the sequence
    const uint8_t *arena;
    const int *live;
    float *qf, *sal_all;      // QF scores [n_ctx]; salience of all layers [10][n_ctx]
    float *scores, *cmax, *lpart, *opart, *ml;
    int8_t *xq;               // the row's Q8_K output
    float *xd;
    int16_t *xs;
    float *sal, *pin_sal;     // this layer's
    int nk_max, span, nchunk;
};

int launch_qk_prep_append(const float *proj, int proj_ld, const float *qn, const float *kn,
                          const float *rope, const StepParams *sp, int T, float *qr, float *z,
                          uint8_t *kv, float *qf, float *sal, cudaStream_t st);
// chunked attention + combine (the token's output, Q8_K for attn_output)
int launch_attention(const AttnArgs &a, cudaStream_t st);
// the salience EMA of the attended positions (needs the combine's max/sum)
int launch_salience(const AttnArgs &a, cudaStream_t st);
// The attention of one token for each of n sequences (rows: device
// [n]): qk prep + append, the decode kernel, the combine and the salience
// update, four launches.  max_nchunk / max_nk: the largest of the rows'.
// Every row's span must be at most 64 positions (attn_span of one query
// over at most 16384 positions).
int launch_attention_rows(const AttnRow *rows, int n, int proj_ld, const float *qn, const float *kn, int max_nchunk,
                          int max_nk, cudaStream_t st);
constexpr int ATTN_ROWS_MAX_SPAN = 64;
// positions per chunk CTA for T queries over at most nk positions
__host__ __device__ inline int attn_span(int T, int nk) {
    return T > 1 ? 256 : (nk <= 1024 ? 16 : (nk <= 4096 ? 32 : (nk <= 16384 ? 64 : 128)));
}
int launch_arena_copy(const int2 *pairs, int n, uint8_t *const *kv, uint8_t *const *arena,
                      const float *sal, float *pin_sal, int n_ctx, cudaStream_t st);

}  // namespace qma
