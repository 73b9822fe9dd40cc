/*
 * ref_glue.c -- drives the qma reference engine, compiled from its own
 * sources in place, as a CPU oracle (TEST INFRASTRUCTURE; built into
 * oracle/_ref/libqmaref.so by oracle/Makefile, never linked by the engine).
 *
 * nn.c is compiled inside this translation unit so that its static layer
 * functions (moe_ffn, conv1d_layer, gdn_worker, ...) can be called one at a
 * time; the same trick the reference's own tests/test_intern.c uses for
 * intern.c.  Nothing of the reference is copied here.
 *
 * Build-recipe change to the reference's behaviour, and why:
 *   moe_ffn mallocs the per-(token, expert) accumulator (nn.c:604) and the
 *   expert kernels accumulate into it with += (nn.c:436), so the reference
 *   reads uninitialised heap memory (at decode usually the previous layer's
 *   partial sums).  malloc is redirected to calloc for nn.c so the oracle
 *   is reproducible; zero is the evident intent of the code.
 */
#include <stdlib.h>
#include <stdint.h>
#include <string.h>

#define malloc(n) calloc(1, (n))
#include "nn.c"
#undef malloc

/* tensor table entry: same layout as qo_tensor in qma_oracle.h */
typedef struct {
    char     name[64];
    uint32_t type;
    int64_t  ne[3];
    uint64_t off;
    uint64_t nbytes;
} qr_tensor;

static const qr_tensor *qr_find(const qr_tensor *t, int n, const char *name)
{
    for (int i = 0; i < n; i++)
        if (strcmp(t[i].name, name) == 0) return &t[i];
    return NULL;
}

void qr_init(int n_threads) { pool_init(n_threads); }

int qr_n_vocab(void) { return N_VOCAB; }

/* Build a qma_t over an in-memory data section (the layout qma_load
 * produces from a GGUF, gguf.c:302-345), experts read zero-copy through
 * m->map (mmap_exps = 1, nn.c:668-674). */
qma_t *qr_model_new(const qr_tensor *t, int n, uint8_t *blob, uint64_t blob_size)
{
    qma_t *m = calloc(1, sizeof(qma_t));
    if (!m) return NULL;
    m->fd = -1;
    m->dio_fd = -1;
    m->map = blob;
    m->map_size = (size_t)blob_size;
    m->data = blob;
    m->data_section_abs = 0;
    m->mmap_exps = 1;
    m->n_vocab = N_VOCAB;
    const qr_tensor *x;
    char nm[96];
#define GETT(dst, tt, name) do { x = qr_find(t, n, name); if (!x) { free(m); return NULL; } \
        dst = blob + x->off; tt = x->type; } while (0)
#define GETO(dst, tt, offp, name) do { GETT(dst, tt, name); offp = (size_t)x->off; } while (0)
    uint32_t dummy;
    GETT(m->token_embd, m->t_token_embd, "token_embd.weight");
    GETT(m->output_norm, dummy, "output_norm.weight");
    GETT(m->output, m->t_output, "output.weight");
    for (int il = 0; il < N_LAYER; il++) {
#define L(suffix) (snprintf(nm, sizeof(nm), "blk.%d.%s", il, suffix), nm)
        GETT(m->layers[il].attn_norm, dummy, L("attn_norm.weight"));
        GETT(m->layers[il].attn_post_norm, dummy, L("post_attention_norm.weight"));
        GETT(m->layers[il].ffn_gate_inp, dummy, L("ffn_gate_inp.weight"));
        GETO(m->layers[il].ffn_gate_exps, m->layers[il].t_gate_exps, m->layers[il].off_gate_exps, L("ffn_gate_exps.weight"));
        GETO(m->layers[il].ffn_up_exps, m->layers[il].t_up_exps, m->layers[il].off_up_exps, L("ffn_up_exps.weight"));
        GETO(m->layers[il].ffn_down_exps, m->layers[il].t_down_exps, m->layers[il].off_down_exps, L("ffn_down_exps.weight"));
        GETT(m->layers[il].ffn_gate_inp_shexp, dummy, L("ffn_gate_inp_shexp.weight"));
        GETO(m->layers[il].ffn_gate_shexp, m->layers[il].t_gate_shexp, m->layers[il].off_gate_shexp, L("ffn_gate_shexp.weight"));
        GETO(m->layers[il].ffn_up_shexp, m->layers[il].t_up_shexp, m->layers[il].off_up_shexp, L("ffn_up_shexp.weight"));
        GETO(m->layers[il].ffn_down_shexp, m->layers[il].t_down_shexp, m->layers[il].off_down_shexp, L("ffn_down_shexp.weight"));
        if (IS_ATTN(il)) {
            GETT(m->layers[il].wq, m->layers[il].t_wq, L("attn_q.weight"));
            GETT(m->layers[il].wk, m->layers[il].t_wk, L("attn_k.weight"));
            GETT(m->layers[il].wv, m->layers[il].t_wv, L("attn_v.weight"));
            GETT(m->layers[il].wo, m->layers[il].t_wo, L("attn_output.weight"));
            GETT(m->layers[il].q_norm, dummy, L("attn_q_norm.weight"));
            GETT(m->layers[il].k_norm, dummy, L("attn_k_norm.weight"));
        } else {
            GETT(m->layers[il].wqkv, m->layers[il].t_wqkv, L("attn_qkv.weight"));
            GETT(m->layers[il].attn_gate, m->layers[il].t_gate, L("attn_gate.weight"));
            GETT(m->layers[il].ssm_conv1d, dummy, L("ssm_conv1d.weight"));
            GETT(m->layers[il].ssm_dt, dummy, L("ssm_dt.bias"));
            GETT(m->layers[il].ssm_a, dummy, L("ssm_a"));
            GETT(m->layers[il].ssm_beta, m->layers[il].t_beta, L("ssm_beta.weight"));
            GETT(m->layers[il].ssm_alpha, m->layers[il].t_alpha, L("ssm_alpha.weight"));
            GETT(m->layers[il].ssm_norm, dummy, L("ssm_norm.weight"));
            GETT(m->layers[il].ssm_out, m->layers[il].t_out, L("ssm_out.weight"));
        }
#undef L
    }
#undef GETT
#undef GETO
    (void)dummy;
    return m;
}

void qr_model_free(qma_t *m) { free(m); }

runstate_t *qr_state_new(int n_ctx)
{
    runstate_t *rs = calloc(1, sizeof(runstate_t));
    if (!rs) return NULL;
    if (runstate_init_kv(rs, n_ctx, NULL, 0) != 0) { free(rs); return NULL; }
    return rs;
}

void qr_state_free(runstate_t *rs) { if (rs) { runstate_free(rs); free(rs); } }

int qr_eval(qma_t *m, runstate_t *rs, const int *tokens, int n, float *logits,
            int n_threads, int logits_all)
{
    return qma_eval(m, rs, tokens, n, logits, n_threads, 0, logits_all);
}

/* the reference's quantized matmul (nn.c:307-345) on n_threads pool workers */
void qr_matmul(const float *x, const uint8_t *W, int n_in, int n_out, int T, int wtype,
               float *out, int n_threads)
{
    pool_init(n_threads);
    matmul(x, W, n_in, n_out, T, wtype, out);
}

/* one MoE FFN (nn.c:509-649); sel8 (optional) gets the last token's
   routing from the history the reference keeps (nn.c:549-550) */
void qr_moe_ffn(qma_t *m, int il, const float *x, int T, float *out, int *sel8)
{
    pool_init(1);
    moe_ffn(m, il, x, NULL, out, T);
    if (sel8) for (int k = 0; k < N_EXPERT_USED; k++) sel8[k] = g_hist_ids[il][k];
}

/* recurrent (GDN) layer from the post-norm input to the ssm_out output,
   calling the reference's own kernels in qma_eval's order (nn.c:2164-2244) */
void qr_gdn_layer(qma_t *m, runstate_t *rs, int il, const float *xn, int T, float *ra)
{
    pool_init(1);
    float *qkv = calloc((size_t)T * QKV_DIM, sizeof(float));
    float *z = calloc((size_t)T * VAL_DIM, sizeof(float));
    float *beta = calloc((size_t)T * S_DT_RANK, sizeof(float));
    float *gt = calloc((size_t)T * S_DT_RANK, sizeof(float));
    float *cout = calloc((size_t)T * CONV_DIM, sizeof(float));
    float *gkv = calloc((size_t)T * S_D_STATE * S_DT_RANK * 3, sizeof(float));
    float *gdout = calloc((size_t)T * VAL_DIM, sizeof(float));
    matmul(xn, m->layers[il].wqkv, N_EMBD, QKV_DIM, T, m->layers[il].t_wqkv, qkv);
    matmul(xn, m->layers[il].attn_gate, N_EMBD, VAL_DIM, T, m->layers[il].t_gate, z);
    matmul(xn, m->layers[il].ssm_beta, N_EMBD, S_DT_RANK, T, m->layers[il].t_beta, beta);
    for (size_t i = 0; i < (size_t)S_DT_RANK * T; i++) beta[i] = 1.0f / (1.0f + expf(-beta[i]));
    matmul(xn, m->layers[il].ssm_alpha, N_EMBD, S_DT_RANK, T, m->layers[il].t_alpha, gt);
    {
        const float *dt = (const float *)m->layers[il].ssm_dt;
        const float *sa = (const float *)m->layers[il].ssm_a;
        for (int t = 0; t < T; t++)
            for (int h = 0; h < S_DT_RANK; h++) {
                float a = gt[(size_t)t * S_DT_RANK + h] + dt[h];
                float sp = a > 20.0f ? a : log1pf(expf(a));
                gt[(size_t)t * S_DT_RANK + h] = sp * sa[h];
            }
    }
    conv1d_layer(rs->conv_state[il], qkv, (const float *)m->layers[il].ssm_conv1d, cout, T);
    silu_m(cout, CONV_DIM, T);
    {
        const int S_v = S_D_STATE;
        for (int t = 0; t < T; t++)
            for (int h = 0; h < S_DT_RANK; h++) {
                const int qh = h % S_N_GROUP;
                float *o = gkv + (size_t)t * S_v * S_DT_RANK * 3 + (size_t)h * S_v;
                for (int i = 0; i < S_v; i++) {
                    o[i] = cout[(size_t)(qh * S_v + i) * T + t];
                    o[S_v * S_DT_RANK + i] = cout[(size_t)(KEY_DIM + qh * S_v + i) * T + t];
                    o[2 * S_v * S_DT_RANK + i] = cout[(size_t)(KEY_DIM * 2 + h * S_v + i) * T + t];
                }
            }
        l2norm_skv(gkv, S_DT_RANK, T);
        l2norm_skv(gkv + (size_t)VAL_DIM, S_DT_RANK, T);
    }
    {
        const int ts = S_D_STATE * S_DT_RANK * 3;
        gdn_ctx gc = { rs->ssm_state[il], gkv, gkv + (size_t)VAL_DIM, gkv + (size_t)(VAL_DIM * 2),
                       gt, beta, gdout, T, ts };
        gdn_worker(&gc, 0, S_DT_RANK);
    }
    rms_norm_head(gdout, (const float *)m->layers[il].ssm_norm, S_DT_RANK, T);
    for (size_t i = 0; i < (size_t)VAL_DIM * T; i++) z[i] = gdout[i] * (z[i] / (1.0f + expf(-z[i])));
    matmul(z, m->layers[il].ssm_out, VAL_DIM, N_EMBD, T, m->layers[il].t_out, ra);
    free(qkv); free(z); free(beta); free(gt); free(cout); free(gkv); free(gdout);
}

float *qr_state_conv(runstate_t *rs, int il) { return rs->conv_state[il]; }
float *qr_state_ssm(runstate_t *rs, int il) { return rs->ssm_state[il]; }
int qr_state_n_pos(runstate_t *rs) { return rs->n_pos; }

/* the reference's fp16 helpers (qma.h:101-152) as built here */
float qr_half_to_float(uint16_t h) { return half_to_float(h); }
uint16_t qr_float_to_half(float f) { return float_to_half(f); }

/* qma_load (gguf.c:104-513) on a GGUF file: its tensor table (up to cap
 * entries), the count, the data section's offset in the file and the
 * vocabulary size; or -1 with qma_load's message in err. */
int qr_gguf_load(const char *path, qr_tensor *out, int cap, int *n, uint64_t *data_off, int *n_vocab,
                 char *err, int errlen)
{
    qma_t *m = calloc(1, sizeof(qma_t));
    if (!m) return -1;
    err[0] = 0;
    int rc = qma_load(m, path, err, (size_t)errlen);
    if (rc == 0) {
        *n = (int)m->n_tensors;
        for (int i = 0; i < cap && i < (int)m->n_tensors; i++) {
            memcpy(out[i].name, m->tensors[i].name, sizeof out[i].name);
            out[i].type = m->tensors[i].type;
            for (int d = 0; d < 3; d++) out[i].ne[d] = m->tensors[i].ne[d];
            out[i].off = m->tensors[i].off;
            out[i].nbytes = m->tensors[i].nbytes;
        }
        *data_off = (uint64_t)(m->data - m->map);
        *n_vocab = m->n_vocab;
    }
    if (m->fd >= 0 || m->tensors) qma_free(m);
    free(m);
    return rc;
}

/* sampler_candidates (sampler.c:36-95) with a sampler set up by
 * sampler_init and holding the given last tokens (oldest first). */
int qr_sampler_candidates(int n_vocab, const float *logits, const int *last, int n_last, float penalty,
                          float temp, int top_k, int *ids, float *lgs, int max_k)
{
    sampler_t s;
    sampler_init(&s, 1, temp, top_k, 0.95f, penalty);
    for (int i = 0; i < n_last && i < 64; i++) s.last_tokens[i] = last[i];
    s.n_last = n_last < 64 ? n_last : 64;
    return sampler_candidates(n_vocab, logits, &s, ids, lgs, max_k);
}

/* runstate_load (nn.c:2027-2042) into a state made by qr_state_new. */
int qr_runstate_load(runstate_t *rs, const char *path) { return runstate_load(rs, path); }
