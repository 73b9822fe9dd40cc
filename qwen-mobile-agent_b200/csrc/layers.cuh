// layers.cuh -- per-layer kernels of the qwen35moe forward (norms,
// embedding, gated delta net, quantized-KV attention) and the device-side
// step parameters they read.
#pragma once
#include "common.cuh"

namespace qma {

constexpr int EMBD = 2048;          // N_EMBD (qma.h:28)
constexpr int NLAYER = 40;          // N_LAYER
constexpr int NHEAD = 16;           // N_HEAD
constexpr int NHEAD_KV = 2;         // N_HEAD_KV
constexpr int HEAD_DIM = 256;       // N_EMBD_HEAD
constexpr int NROT = 64;            // N_ROT
constexpr int CONV_DIM = 8192;      // CONV_DIM (qma.h:48)
constexpr int KEY_DIM = 2048;
constexpr int VAL_DIM = 4096;
constexpr int SSTATE = 128;         // S_D_STATE
constexpr int VHEADS = 32;          // S_DT_RANK
constexpr int KHEADS = 16;          // S_N_GROUP
constexpr int WQ_DIM = 8192;        // 16 heads x (256 Q + 256 gate)
constexpr int WKV_DIM = 512;
constexpr int WO_DIM = 4096;
constexpr int NATTN = 10;
constexpr int KVQ_SLOT = 240;       // kvq.h:22
constexpr int KVQ2_OFF = 160;       // kvq.h:29
constexpr int HCM_SINK = 4;         // nn.c:897
constexpr int HCM_H_PIN = 2048;     // nn.c:895
constexpr int HCM_ARENA_BASE = 1 << 24;   // nn.c:937
constexpr int LIVE_Q2_FLAG = 1 << 30;     // engine's tag for q2-segment entries
constexpr int MAX_CHUNK = 512;      // nn.c:1799

__host__ __device__ inline bool is_attn(int il) { return ((il + 1) % 4) == 0; }
__host__ __device__ inline int hcm_slot(int p, int n_ctx) {
    return p < HCM_SINK ? p : HCM_SINK + (p - HCM_SINK) % (n_ctx - HCM_SINK);
}

// Parameters of the current forward step, kept in device memory so a
// captured decode graph replays without host edits between tokens.
struct StepParams {
    int n_pos;        // absolute position of the first token of the step
    int T;            // tokens in the step
    int n_live;       // live-index entries (0: dense attention over 0..abs)
    int n_ring_q4;    // live[0, n_ring_q4) ring q4 slots
    int n4;           // live[n_ring_q4, n4) arena q4 entries, [n4, n_live) q2
    int rebuilt_at;   // positions >= rebuilt_at are attended directly (tail)
    int n_ctx;
    int token;        // decode: the step's input token (written by argmax)
};

// ---- launchers (layers.cu) -------------------------------------------------
// tokens: device [T] ids, or null to read StepParams::token (T = 1)
int launch_embed(const void *embd, int type, int n_vocab, const int *tokens,
                 const StepParams *sp, int T, float *x, cudaStream_t st);
int launch_rmsnorm_quant(const float *x, const float *w, int T, int n, int8_t *xq, float *xd,
                         int16_t *xs, cudaStream_t st, const Prefetch &pf = Prefetch());
int launch_conv1d(const float *qkv, int ld, const float *w, float *state, int T, float *out,
                  cudaStream_t st);
// Per-token recurrent state of a batch of sequences: token t of a step
// belongs to sequence seq[t] (device [n], distinct), whose state for the
// layer is state[seq[t]] (device table of pointers).
struct SeqTable {
    float *const *state = nullptr;
    const int *seq = nullptr;
};
// conv1d + SiLU of one token per sequence (row t of qkv, its own state)
int launch_conv1d_seqs(const float *qkv, int ld, const float *w, const SeqTable &sq, int n, float *out,
                       cudaStream_t st);
// Optional tail of a single-token gated delta net: the gated RMSNorm and the
// Q8_K for ssm_out written to xq / xd / xs (cnt: 16 zeroed tickets).
struct GdnNormArgs {
    const float *z;
    const float *w;
    int8_t *xq;
    float *xd;
    int16_t *xs;
    unsigned *cnt;
};
int launch_gdn(const float *conv_out, const float *proj, int proj_ld, int beta_off, int alpha_off,
               const float *dt, const float *a, float *ssm, int T, float *o, cudaStream_t st,
               const GdnNormArgs *norm = nullptr, float *kq_scratch = nullptr, float *chunk_scratch = nullptr);
// (T > 1 with kq_scratch [T][16]: q and k are L2-normed in place in conv_out
// first; then, with chunk_scratch (gdn_chunk_scratch_bytes(), T <= 512), the
// chunked gated-delta form, else the token-sequential recurrence.)
size_t gdn_chunk_scratch_bytes();
// The single-token recurrence for one token of each of n sequences (row t
// of conv_out / proj / o, state sq.state[sq.seq[t]]), without the norm tail.
int launch_gdn_seqs(const float *conv_out, const float *proj, int proj_ld, int beta_off, int alpha_off,
                    const float *dt, const float *a, const SeqTable &sq, int n, float *o, cudaStream_t st);
int launch_gated_norm_quant(const float *o, const float *z, int z_ld, const float *w, int T,
                            int8_t *xq, float *xd, int16_t *xs, cudaStream_t st);

}  // namespace qma
