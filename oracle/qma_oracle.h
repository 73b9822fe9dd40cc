/*
 * qma_oracle.h -- CPU restatement of the qma qwen35moe engine hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA engine: it is loaded by tests/, by __graft_entry__.smoke() and by the
 * cpu_baseline leg of bench.py, never by the engine itself.  Every function
 * restates one reference function (file:line in the qma sources cited per
 * declaration) in plain C with the same operation order, so that it can be
 * pinned bit-for-bit against the reference compiled from its own sources
 * (oracle/_ref, built by oracle/Makefile).
 *
 * Build flags (oracle/Makefile): -O2 -fno-fast-math -ffp-contract=off, so
 * every fp32 operation rounds exactly where the C source says it does.
 */
#ifndef QMA_ORACLE_H
#define QMA_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- model constants (qma.h:28-64) -------------------------------------- */
#define QO_EMBD        2048
#define QO_LAYER       40
#define QO_HEAD        16
#define QO_HEAD_KV     2
#define QO_HEAD_DIM    256
#define QO_ROT         64
#define QO_CONV        4
#define QO_INNER       4096
#define QO_STATE       128
#define QO_VHEADS      32
#define QO_KHEADS      16
#define QO_CONV_DIM    8192
#define QO_KEY_DIM     2048
#define QO_VAL_DIM     4096
#define QO_WQ_DIM      8192
#define QO_WKV_DIM     512
#define QO_WO_DIM      4096
#define QO_EXPERT      256
#define QO_EXPERT_USED 8
#define QO_FF          512
#define QO_ATTN_LAYERS 10
#define QO_IS_ATTN(il) ((((il) + 1) % 4) == 0)
#define QO_RMS_EPS     1e-6f
#define QO_FREQ_BASE   10000000.0f

/* GGML type ids (qma.h:67-69); Q8_0 = 8 is ggml's id for block_q8_0 */
#define QO_F32  0
#define QO_Q8_0 8
#define QO_Q4_K 12
#define QO_Q6_K 14

#define QO_QK_K 256
#define QO_Q4K_BYTES 144   /* block_q4_K, qma.h:77-82 */
#define QO_Q6K_BYTES 210   /* block_q6_K, qma.h:85-90 */
#define QO_Q80_BYTES 34    /* block_q8_0, qma.h:92-94 */

/* KV record layout (kvq.h:22-29) */
#define QO_KVQ_SLOT 240
#define QO_KVQ2_OFF 160

/* HCM constants (nn.c:894-901) */
#define QO_HCM_W_HOT   4096
#define QO_HCM_H_PIN   2048
#define QO_HCM_W_GIST  32768
#define QO_HCM_SINK    4
#define QO_HCM_ALPHA   0.05f
#define QO_HCM_QF_BIAS 2.0f
#define QO_HCM_REBUILD 128
#define QO_HCM_ARENA_BASE (1 << 24)
#define QO_MAX_CHUNK   512

/* ---- threading of independent loops (results are thread-count independent) */
void qo_set_threads(int n);
void qo_pfor(int n, void (*fn)(void *ctx, int i0, int i1), void *ctx);

/* ---- fp16 (qma.h:101-152, AArch64 FCVT semantics: round-to-nearest-even) */
float    qo_half_to_float(uint16_t h);
uint16_t qo_float_to_half(float x);

/* ---- weight bytes per row ----------------------------------------------- */
size_t qo_row_bytes(int wtype, int n_in);

/* ---- Q8_K activation quantization (q8k.c:34-85) ------------------------- */
void qo_q8k_quant(const float *x, int n, int8_t *xq, float *xd, int16_t *xsum);

/* ---- super-block dots against Q8_K activations -------------------------- */
/* dot_q4_K_q8k (q8k.c:89-131).  isum (optional, n/32 int32) receives the
 * exact integer dot of every 32-lane sub-block: sum(nibble * xq). */
float qo_dot_q4k(const uint8_t *row, const int8_t *xq, const float *xd,
                 const int16_t *xsum, int n, int32_t *isum);
/* dot_q4_K_gateup_q8k (q8k.c:140-207) */
void  qo_gateup_q4k(const uint8_t *g, const uint8_t *u, const int8_t *xq,
                    const float *xd, const int16_t *xsum, int n,
                    float *gate, float *up);
/* dot_q6_K_q8k (q8k.c:210-262).  isum (optional, n/256 int32) receives the
 * exact per-super-block sum over g of scale_g * sum16((q-32) * xq). */
float qo_dot_q6k(const uint8_t *row, const int8_t *xq, const float *xd, int n,
                 int32_t *isum);
/* Q8_0 weights x Q8_K activations.  No reference kernel exists (the
 * reference rejects Q8_0 weights, gguf.c:272-287); this is the engine's own
 * definition: per 32-lane block b, isum_b = sum(q * xq) (exact int32); per
 * 256-lane super-block acc = sum_b isum_b * d_b in block order; total +=
 * acc * xd.  isum (optional, n/32 int32) receives the per-block sums. */
float qo_dot_q80(const uint8_t *row, const int8_t *xq, const float *xd, int n,
                 int32_t *isum);
/* qma_q8k_dot dispatch (q8k.c:305-316) plus Q8_0 */
float qo_dot(const uint8_t *row, int wtype, const int8_t *xq, const float *xd,
             const int16_t *xsum, int n);

/* ---- dequantization (quants.c:29-75) + Q8_0 ----------------------------- */
void qo_dequant_row(const uint8_t *row, int wtype, float *y, int n);

/* ---- matmul: quantize each token row once, then row dots (nn.c:261-345) */
void qo_matmul(const float *x, const uint8_t *W, int n_in, int n_out, int T,
               int wtype, float *out);

/* ---- weight quantizers (the engine's own; the reference ships none) ----- */
void qo_quantize_q4k(const float *x, uint8_t *blk);   /* 256 values -> 144 B */
void qo_quantize_q6k(const float *x, uint8_t *blk);   /* 256 values -> 210 B */
void qo_quantize_q80(const float *x, uint8_t *blk);   /* 32 values  ->  34 B */

/* ---- synthetic model ------------------------------------------------------
 * A GGUF-style tensor table over one contiguous data blob.  Names follow the
 * reference's GGUF names (gguf.c:308-345). */
typedef struct {
    char     name[64];
    uint32_t type;
    int64_t  ne[3];
    uint64_t off;
    uint64_t nbytes;
} qo_tensor;

typedef struct {
    int n_vocab;
    int embd_type;    /* token_embd.weight: Q8_0 / Q4_K / Q6_K */
    int out_type;     /* output.weight */
    int down_type;    /* ffn_down_exps / ffn_down_shexp: Q6_K or Q4_K */
    int proj_type;    /* every other projection: Q4_K */
} qo_synth_cfg;

/* Fills `t` (capacity cap) and returns the tensor count; *blob_bytes gets
 * the data-section size.  Every tensor offset is 256-byte aligned. */
int  qo_synth_layout(const qo_synth_cfg *cfg, qo_tensor *t, int cap,
                     uint64_t *blob_bytes);
/* Generates tensor `t` into blob + t->off.  Values are a seeded function of
 * (seed, tensor name, element index): an Irwin-Hall(4) normal scaled per
 * tensor kind, then quantized per the tensor type.  Multi-threaded over
 * n_threads. */
void qo_synth_tensor(const qo_tensor *t, uint8_t *blob, uint64_t seed,
                     int n_threads);
/* First-element-of-block generator, exposed for tests: value of element
 * `idx` of the tensor with name-hash `key` before quantization. */
float qo_synth_value(uint64_t key, uint64_t idx, float mu, float sigma);
uint64_t qo_name_key(const char *name, uint64_t seed);

/* ---- model view over a blob ---------------------------------------------- */
typedef struct qo_model qo_model;
qo_model *qo_model_new(const qo_tensor *t, int n, const uint8_t *blob, int n_vocab);
void      qo_model_free(qo_model *m);

/* ---- MoE FFN for T tokens (nn.c:509-649, q8k path) ------------------------
 * x [T][2048] post-norm input -> out [T][2048] (no residual).  sel/w (T*8,
 * optional) receive the routing in selection order. */
void qo_moe_ffn(const qo_model *m, int il, const float *x, int T, float *out,
                int *sel, float *w);
/* FFN half of a layer (nn.c:2246-2252): out = x2 + moe_ffn(rms_norm(x2) *
 * post_attention_norm). */
void qo_moe_block(const qo_model *m, int il, const float *x2, int T, float *out,
                  int *sel, float *w);
/* the same with an additive per-expert router bias (256 floats, or NULL):
 * each fp32 logit gets one fp32 addition before the softmax (configs[4]'s
 * serving prior; the reference has none) */
void qo_moe_block_biased(const qo_model *m, int il, const float *x2, int T, const float *bias, float *out,
                         int *sel, float *w);
/* router only: logits (256) of one token in the reference's sequential
 * fp32 order (nn.c:513-523) */
void qo_router_logits(const float *gate_inp, const float *x, float *logits);
/* routing of T normed tokens (nn.c:513-551): sel/wt [T][8] in selection
 * order; bias (256, optional) is added to each fp32 logit before the
 * softmax (the configs[4] router prior; the reference has none) */
void qo_route(const float *gate_inp, const float *bias, const float *x, int T, int *sel, float *wt);
/* the same from the residual input x2: rms_norm_m * post_norm first */
void qo_moe_route(const float *post_norm, const float *gate_inp, const float *bias, const float *x2, int T,
                  int *sel, float *wt);

/* ---- sequence state + full forward ---------------------------------------- */
typedef struct qo_state qo_state;
qo_state *qo_state_new(int n_ctx);
void      qo_state_free(qo_state *s);
int       qo_state_n_pos(const qo_state *s);
/* a qma session resumed in a fresh process from the KV slab and salience
 * files (hcm_load semantics, nn.c:1173-1209); 0 or -1 */
int       qo_state_resume(qo_state *s, const char *kv_path, const char *sal_path, int n_pos);
/* live index segments after the last rebuild: ring q4, + arena q4, + ring q2 */
void      qo_state_live_segments(const qo_state *s, int *n_ring_q4, int *n4, int *live_n);
/* 240-byte KV slot of attention layer lay, head (0,1 K; 2,3 V), ring slot */
const uint8_t *qo_state_kv_slot(const qo_state *s, int lay, int head, int slot);
/* qma_eval (nn.c:2056-2308), single-threaded, q8k path, quantized KV + HCM.
 * Writes the last token's logits (n_vocab) or all (T*n_vocab). */
int qo_eval(const qo_model *m, qo_state *s, const int *tokens, int n_tokens,
            float *logits, int logits_all);

/* qo_eval through the first n_layers layers; hidden [n_tokens][2048] gets
 * the residual stream after them (parity aid). */
int qo_eval_hidden(const qo_model *m, qo_state *s, const int *tokens, int n_tokens,
                   int n_layers, float *hidden);

/* One full layer (mixer + residual + MoE block + residual, nn.c:2105-2252)
 * from x_in [T][2048] to x_out, tokens at positions n_pos.. (parity aid). */
void qo_layer_forward(const qo_model *m, qo_state *s, int il, const float *x_in, int T,
                      int n_pos, float *x_out);
/* Layer il's mixer + residual over n_tokens caller-given inputs, chunked
 * and HCM-rebuilt as qma_eval does (nn.c:2081-2245); advances the state's
 * position (parity aid for long contexts). */
void qo_mixer_forward(const qo_model *m, qo_state *s, int il, const float *x_in, int n_tokens,
                      float *x_out);

/* ---- per-layer pieces, for layer-level parity ------------------------------ */
/* GDN (recurrent) layer core from the post-norm input xn [T][2048] to the
 * ssm_out projection input z [T][4096] (nn.c:2164-2242), updating the conv
 * and ssm state of layer il held in s. */
void qo_gdn_layer(const qo_model *m, qo_state *s, int il, const float *xn,
                  int T, float *out /* [T][2048] after ssm_out */);
/* Direct access to the recurrent state of layer il (conv [8192*3], ssm
 * [32*128*128]) for state comparisons. */
float *qo_state_conv(qo_state *s, int il);
float *qo_state_ssm(qo_state *s, int il);

/* ---- quantized KV records (kvq.c) ----------------------------------------- */
void  qo_kvq4_quant(const float *x, uint8_t *slot);          /* kvq.c:25-46 */
void  qo_kvq2_quant(const float *x, uint8_t *slot);          /* kvq.c:50-70 */
float qo_kvq4_dot(const uint8_t *rec, const float *x);       /* kvq.c:183-197 */
float qo_kvq2_dot(const uint8_t *rec, const float *x);       /* kvq.c:199-213 */
void  qo_kvq4_vacc(const uint8_t *rec, float w, float *o);   /* kvq.c:215-227 */
void  qo_kvq2_vacc(const uint8_t *rec, float w, float *o);   /* kvq.c:229-241 */
float qo_kvq4_qf(const uint8_t *slot, const float *x);       /* kvq.c:84-100 */

#ifdef __cplusplus
}
#endif
#endif /* QMA_ORACLE_H */
