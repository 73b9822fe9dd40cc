// moe.cuh -- constants and scratch layout of the MoE FFN block (moe.cu).
#pragma once
#include "common.cuh"

namespace qma {

constexpr int MOE_EMBD = 2048;        // N_EMBD (qma.h:28)
constexpr int MOE_NEXP = 256;         // N_EXPERT (qma.h:57)
constexpr int MOE_TOPK = 8;           // N_EXPERT_USED (qma.h:58)
constexpr int MOE_FF = 512;           // N_FF_EXP / N_FF_SHEXP (qma.h:59-60)
constexpr int MOE_NSLOT = MOE_TOPK + 1;   // routed experts + the shared expert
constexpr int MOE_DOWN_CHUNK = 128;   // down-projection output rows per CTA
// Chunks of MOE_GROUPED_MIN_T .. MOE_GROUPED_MAX_T tokens take the grouped
// path (moe_grouped.cu): pairs grouped by expert, tensor-core MMAs.
constexpr int MOE_GROUPED_MIN_T = 16;
constexpr int MOE_GROUPED_MAX_T = 512;
constexpr int MOE_DOWN_CHUNKS = MOE_EMBD / MOE_DOWN_CHUNK;

// Per-call device scratch of the MoE block for T tokens (moe_scratch_layout
// carves one caller-provided buffer).  The combine tickets (dcount) must be
// zero when a call starts; every call leaves them zero again.
struct MoeScratch {
    unsigned *dcount;      // [T][16] slot CTAs finished per 128-row output chunk
    double *S, *B;         // [T][256] exact logit, bound on the fp32 logit
    int *fallback;         // [T] 1 if the exact sequential recompute ran
    int *sel;              // [T][8] selected experts, selection order
    float *w;              // [T][8] renormalised weights
    int8_t *xq;            // [T][2048] Q8_K of the normed FFN input
    float *xd;             // [T][8]
    int16_t *xs;           // [T][128]
    float *gs;             // [T] shared-expert gate sigmoid
    float *part;           // [T][9][2048] down projections per slot
    // grouped path only (null below MOE_GROUPED_MIN_T tokens):
    int *goff;             // [257] first pair of each expert in plist, then [1 + 256]: the
                           // number of experts with pairs and their ids, ascending
    int *plist;            // [T * 8] pair ids t * 8 + k grouped by expert
    float *hg;             // [T * 9][1024] gate | up per pair slot
    int8_t *hq;            // [T * 9][512] Q8_K of silu(gate) * up
    float *hd;             // [T * 9][2]
    int16_t *hs;           // [T * 9][32]
};
int moe_grouped(const qma_cuda_moe_weights &w, int T, const MoeScratch &s, cudaStream_t st);
// The grouped pipeline on part of the work: groups g0 .. g0 + ng - 1 of the
// 257 (256 = the shared expert; routed group e reads expert e of the tables
// w points at), the pair lists built first when `lists`, the SwiGLU on pair
// slots q0 .. q0 + nq - 1.  The expert-parallel layer runs the routed groups
// of its shard over received rows and the shared group over its own tokens.
int moe_grouped_range(const qma_cuda_moe_weights &w, int T, const MoeScratch &s, cudaStream_t st, int g0, int ng,
                      bool lists, int q0, int nq);
// The grouped gate/up GEMM on the 5th-generation tensor cores (moe_tc.cu),
// in place of moe_gateup_kernel when tc_grouped() (QMA_CUDA_TC_GROUPED=1).
int launch_gateup_tc(const qma_cuda_moe_weights &w, int T, const MoeScratch &s, cudaStream_t st, int g0, int ng);
bool tc_grouped();
// Bounded waits of the tensor-core kernels that ran out (reset by reading).
int tc_wait_timeouts();
// The router alone (RMSNorm, Q8_K of the normed input, exact top-8, the
// shared-expert gate) into s, and the slot combine + residual alone.
int moe_route(const qma_cuda_moe_weights &w, const float *x2, int T, const MoeScratch &s, int *sel, float *wts,
              cudaStream_t st);
int moe_combine(const MoeScratch &s, const float *x2, float *x_out, int T, cudaStream_t st);

size_t moe_scratch_bytes(int T);
MoeScratch moe_scratch_layout(void *base, int T);
// clear_counters: zero the combine tickets first (a caller's fresh scratch);
// the engine's own scratch starts zeroed and every call leaves it zeroed, so
// it skips the memset and launches the router with programmatic dependent
// launch.
// Optional tail of the MoE block (the engine's decode path): instead of the
// expert CTAs' ticketed combine, one kernel after the experts combines the
// slots, adds the residual and, when w is set, applies the next RMSNorm
// (the next layer's attn_norm or the output norm) and its Q8_K
// quantization to tokens norm_from.. (row t - norm_from of xq), issuing the
// next layer's L2 prefetch plan pf.
struct MoeNormTail {
    const float *w = nullptr;
    int norm_from = 0;
    int8_t *xq = nullptr;
    float *xd = nullptr;
    int16_t *xs = nullptr;
    Prefetch pf;
};
int moe_layer(const qma_cuda_moe_weights &w, const float *x2, int T, float *x_out, int *sel,
              float *wts, void *scratch, cudaStream_t st, bool clear_counters,
              const MoeNormTail *tail = nullptr);
// Bounded waits of the expert kernel that ran out since the last call (reset
// by reading); -1 if the counter cannot be read.
int moe_wait_timeouts();

}  // namespace qma
