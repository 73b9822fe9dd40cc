/*
 * qo_model.c -- CPU restatement of qma's qwen35moe forward pass (TEST
 * INFRASTRUCTURE: the parity checker for the CUDA engine; see qma_oracle.h).
 *
 * Restated reference functions (qma sources):
 *   rms_norm_m / rms_norm_head        nn.c:348-372
 *   moe_ffn, moe_expert_one_q8k,
 *   moe_shared_q8k (q8k path)         nn.c:412-473, 509-649
 *   conv1d_layer, l2norm_skv,
 *   gdn_worker + GDN glue             nn.c:717-833, 2164-2244
 *   rope_imrope                        nn.c:841-861
 *   kvq4/kvq2 quant, dot, vacc, qf    kvq.c:25-241
 *   hcm_slot, hcm_rebuild             nn.c:908-1150
 *   attn_worker, kv_append            nn.c:1215-1509
 *   embed_row, qma_eval               nn.c:2044-2308
 * with the reference's single-thread operation order (n_threads = 1; the
 * reference's salience EMA races between heads when threaded, nn.c:1416).
 * Independent loops (matmul rows, expert tasks, recurrent heads) run on
 * pthreads (qo_pfor); every output element is still produced by one thread in the
 * reference's order, so results do not depend on the thread count.
 *
 * One deliberate difference from the reference binary: the per-task expert
 * accumulator is zero-initialised.  The reference mallocs it (nn.c:604) and
 * accumulates into it with += (nn.c:436), reading uninitialised heap memory;
 * zero is the evident intent and the only reproducible choice.
 */
#include "qma_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <stdio.h>

/* ------------------------------------------------------------ model view */
typedef struct {
    const float *attn_norm, *post_norm;
    const uint8_t *wqkv, *attn_gate, *ssm_beta, *ssm_alpha, *ssm_out;
    const float *conv1d, *ssm_dt, *ssm_a, *ssm_norm;
    const uint8_t *wq, *wk, *wv, *wo;
    const float *q_norm, *k_norm;
    const float *gate_inp, *gate_inp_sh;
    const uint8_t *gate_exps, *up_exps, *down_exps, *gate_sh, *up_sh, *down_sh;
    int t_wqkv, t_gate, t_beta, t_alpha, t_out, t_wq, t_wk, t_wv, t_wo;
    int t_down, t_down_sh;
} qo_layer;

struct qo_model {
    const uint8_t *embd, *output;
    const float *output_norm;
    int t_embd, t_output;
    int n_vocab;
    qo_layer L[QO_LAYER];
};

static const qo_tensor *find_t(const qo_tensor *t, int n, const char *name)
{
    for (int i = 0; i < n; i++)
        if (strcmp(t[i].name, name) == 0) return &t[i];
    return NULL;
}

qo_model *qo_model_new(const qo_tensor *t, int n, const uint8_t *blob, int n_vocab)
{
    qo_model *m = calloc(1, sizeof(*m));
    if (!m) return NULL;
    m->n_vocab = n_vocab;
    char nm[96];
    const qo_tensor *x;
#define GET(dst, type_dst, name)                                \
    do {                                                        \
        x = find_t(t, n, name);                                 \
        if (!x) { free(m); return NULL; }                       \
        dst = (const void *)(blob + x->off);                    \
        type_dst = (int)x->type;                                \
    } while (0)
    int dummy;
    GET(m->embd, m->t_embd, "token_embd.weight");
    GET(m->output_norm, dummy, "output_norm.weight");
    GET(m->output, m->t_output, "output.weight");
    for (int il = 0; il < QO_LAYER; il++) {
        qo_layer *L = &m->L[il];
#define GL(dst, tdst, suffix) do { snprintf(nm, sizeof(nm), "blk.%d.%s", il, suffix); GET(dst, tdst, nm); } while (0)
        GL(L->attn_norm, dummy, "attn_norm.weight");
        GL(L->post_norm, dummy, "post_attention_norm.weight");
        GL(L->gate_inp, dummy, "ffn_gate_inp.weight");
        GL(L->gate_exps, dummy, "ffn_gate_exps.weight");
        GL(L->up_exps, dummy, "ffn_up_exps.weight");
        GL(L->down_exps, L->t_down, "ffn_down_exps.weight");
        GL(L->gate_inp_sh, dummy, "ffn_gate_inp_shexp.weight");
        GL(L->gate_sh, dummy, "ffn_gate_shexp.weight");
        GL(L->up_sh, dummy, "ffn_up_shexp.weight");
        GL(L->down_sh, L->t_down_sh, "ffn_down_shexp.weight");
        if (QO_IS_ATTN(il)) {
            GL(L->wq, L->t_wq, "attn_q.weight");
            GL(L->wk, L->t_wk, "attn_k.weight");
            GL(L->wv, L->t_wv, "attn_v.weight");
            GL(L->wo, L->t_wo, "attn_output.weight");
            GL(L->q_norm, dummy, "attn_q_norm.weight");
            GL(L->k_norm, dummy, "attn_k_norm.weight");
        } else {
            GL(L->wqkv, L->t_wqkv, "attn_qkv.weight");
            GL(L->attn_gate, L->t_gate, "attn_gate.weight");
            GL(L->conv1d, dummy, "ssm_conv1d.weight");
            GL(L->ssm_dt, dummy, "ssm_dt.bias");
            GL(L->ssm_a, dummy, "ssm_a");
            GL(L->ssm_beta, L->t_beta, "ssm_beta.weight");
            GL(L->ssm_alpha, L->t_alpha, "ssm_alpha.weight");
            GL(L->ssm_norm, dummy, "ssm_norm.weight");
            GL(L->ssm_out, L->t_out, "ssm_out.weight");
        }
#undef GL
    }
#undef GET
    (void)dummy;
    return m;
}

void qo_model_free(qo_model *m) { free(m); }

/* ------------------------------------------------------------ elementwise */
static void rms_norm_m(float *out, const float *x, const float *w, int n, int T)
{
    for (int t = 0; t < T; t++) {
        const float *xp = x + (size_t)t * n;
        float *op = out + (size_t)t * n;
        double sum = 0.0;
        for (int i = 0; i < n; i++) sum += (double)xp[i] * xp[i];
        const float r = 1.0f / sqrtf((float)(sum / n) + QO_RMS_EPS);
        for (int i = 0; i < n; i++) op[i] = xp[i] * r * w[i];
    }
}

/* in-place per-head RMS norm with the (r * w) association of nn.c:360-371 */
static void rms_norm_inplace_rw(float *v, const float *w, int n)
{
    double sum = 0.0;
    for (int i = 0; i < n; i++) sum += (double)v[i] * v[i];
    const float r = 1.0f / sqrtf((float)(sum / n) + QO_RMS_EPS);
    for (int i = 0; i < n; i++) v[i] *= r * w[i];
}

static inline float silu(float x) { return x / (1.0f + expf(-x)); }

/* ------------------------------------------------------------------ MoE -- */
void qo_router_logits(const float *gate_inp, const float *x, float *logits)
{
    for (int e = 0; e < QO_EXPERT; e++) {
        const float *gi = gate_inp + (size_t)e * QO_EMBD;
        float s = 0;
        for (int i = 0; i < QO_EMBD; i++) s += gi[i] * x[i];
        logits[e] = s;
    }
}

static void expert_one(const uint8_t *ge, const uint8_t *ue, const uint8_t *de,
                       int de_type, const int8_t *xq, const float *xd,
                       const int16_t *xsum, float we, float *acc)
{
    const size_t gu_row = qo_row_bytes(QO_Q4_K, QO_EMBD);
    const size_t dn_row = qo_row_bytes(de_type, QO_FF);
    float gate[QO_FF];
    for (int i = 0; i < QO_FF; i++) {
        float g, u;
        qo_gateup_q4k(ge + (size_t)i * gu_row, ue + (size_t)i * gu_row, xq, xd, xsum,
                      QO_EMBD, &g, &u);
        gate[i] = (g / (1.0f + expf(-g))) * u;
    }
    int8_t gq[QO_FF];
    float gd[QO_FF / QO_QK_K];
    int16_t gs[QO_FF / 16];
    qo_q8k_quant(gate, QO_FF, gq, gd, gs);
    for (int i = 0; i < QO_EMBD; i++)
        acc[i] += we * qo_dot(de + (size_t)i * dn_row, de_type, gq, gd, gs, QO_FF);
}

static void shared_expert(const qo_layer *L, const int8_t *xq, const float *xd,
                          const int16_t *xsum, float *acc)
{
    float gs = 0;
    for (int i = 0; i < QO_EMBD; i++) gs += L->gate_inp_sh[i] * xq[i] * xd[i / QO_QK_K];
    gs = 1.0f / (1.0f + expf(-gs));
    const size_t gu_row = qo_row_bytes(QO_Q4_K, QO_EMBD);
    float gate[QO_FF];
    for (int i = 0; i < QO_FF; i++) {
        float g, u;
        qo_gateup_q4k(L->gate_sh + (size_t)i * gu_row, L->up_sh + (size_t)i * gu_row,
                      xq, xd, xsum, QO_EMBD, &g, &u);
        gate[i] = (g / (1.0f + expf(-g))) * u;
    }
    int8_t gq[QO_FF];
    float gd[QO_FF / QO_QK_K];
    int16_t g2[QO_FF / 16];
    qo_q8k_quant(gate, QO_FF, gq, gd, g2);
    const size_t dn_row = qo_row_bytes(L->t_down_sh, QO_FF);
    for (int i = 0; i < QO_EMBD; i++)
        acc[i] += gs * qo_dot(L->down_sh + (size_t)i * dn_row, L->t_down_sh, gq, gd, g2, QO_FF);
}

typedef struct {
    const qo_layer *L;
    const int *sel;
    const float *wt;
    const int8_t *xq;
    const float *xd;
    const int16_t *xs;
    float *pacc;
    size_t ge_bytes, dn_bytes;
} moe_task_ctx;

/* moe_xpar_worker (nn.c:652-707): one (token, expert) pair per task */
static void moe_tasks(void *arg, int i0, int i1)
{
    const moe_task_ctx *c = arg;
    const qo_layer *L = c->L;
    for (int id = i0; id < i1; id++) {
        const int t = id / QO_EXPERT_USED;
        const int ex = c->sel[id];
        expert_one(L->gate_exps + (size_t)ex * c->ge_bytes, L->up_exps + (size_t)ex * c->ge_bytes,
                   L->down_exps + (size_t)ex * c->dn_bytes, L->t_down,
                   c->xq + (size_t)t * QO_EMBD, c->xd + (size_t)t * 8, c->xs + (size_t)t * 128,
                   c->wt[id], c->pacc + (size_t)id * QO_EMBD);
    }
}

/* Router of moe_ffn (nn.c:513-551) for T normed tokens: the sequential fp32
 * logits, then (the engine's configs[4] extension, absent in the reference)
 * one fp32 addition of bias[e] per logit when bias is given, softmax (expf
 * of l - max, divided by the sum), eight rounds of argmax with '>' (ties to
 * the lower id) and the renormalised weights. */
void qo_route(const float *gate_inp, const float *bias, const float *x, int T, int *sel, float *wt)
{
    for (int t = 0; t < T; t++) {
        const float *xp = x + (size_t)t * QO_EMBD;
        float logits[QO_EXPERT];
        qo_router_logits(gate_inp, xp, logits);
        if (bias)
            for (int e = 0; e < QO_EXPERT; e++) logits[e] = logits[e] + bias[e];
        float mx = -1e30f;
        for (int e = 0; e < QO_EXPERT; e++) if (logits[e] > mx) mx = logits[e];
        float sum = 0;
        for (int e = 0; e < QO_EXPERT; e++) { logits[e] = expf(logits[e] - mx); sum += logits[e]; }
        for (int e = 0; e < QO_EXPERT; e++) logits[e] /= sum;
        for (int k = 0; k < QO_EXPERT_USED; k++) {
            int best = 0;
            float bv = -1e30f;
            for (int e = 0; e < QO_EXPERT; e++) if (logits[e] > bv) { bv = logits[e]; best = e; }
            sel[t * 8 + k] = best;
            wt[t * 8 + k] = bv;
            logits[best] = -1e30f;
        }
        float ws = 0;
        for (int k = 0; k < QO_EXPERT_USED; k++) ws += wt[t * 8 + k];
        for (int k = 0; k < QO_EXPERT_USED; k++) wt[t * 8 + k] /= ws;
    }
}

/* rms_norm_m (nn.c:348-357) with post_attention_norm, then qo_route: the
 * routing of the FFN half of a layer from its residual input x2. */
void qo_moe_route(const float *post_norm, const float *gate_inp, const float *bias, const float *x2, int T,
                  int *sel, float *wt)
{
    float *xn = malloc(sizeof(float) * (size_t)T * QO_EMBD);
    rms_norm_m(xn, x2, post_norm, QO_EMBD, T);
    qo_route(gate_inp, bias, xn, T, sel, wt);
    free(xn);
}

static void moe_ffn_impl(const qo_model *m, int il, const float *x, int T, const float *bias, float *out,
                         int *sel_out, float *w_out);

void qo_moe_ffn(const qo_model *m, int il, const float *x, int T, float *out,
                int *sel_out, float *w_out)
{
    moe_ffn_impl(m, il, x, T, NULL, out, sel_out, w_out);
}

static void moe_ffn_impl(const qo_model *m, int il, const float *x, int T, const float *bias, float *out,
                         int *sel_out, float *w_out)
{
    const qo_layer *L = &m->L[il];
    int *sel = malloc(sizeof(int) * (size_t)T * QO_EXPERT_USED);
    float *wt = malloc(sizeof(float) * (size_t)T * QO_EXPERT_USED);
    qo_route(L->gate_inp, bias, x, T, sel, wt);
    int8_t *xq = malloc((size_t)T * QO_EMBD);
    float *xd = malloc(sizeof(float) * (size_t)T * (QO_EMBD / QO_QK_K));
    int16_t *xs = malloc(sizeof(int16_t) * (size_t)T * (QO_EMBD / 16));
    for (int t = 0; t < T; t++)
        qo_q8k_quant(x + (size_t)t * QO_EMBD, QO_EMBD, xq + (size_t)t * QO_EMBD,
                     xd + (size_t)t * 8, xs + (size_t)t * 128);
    float *pacc = calloc((size_t)T * QO_EXPERT_USED * QO_EMBD, sizeof(float));
    const size_t ge_bytes = qo_row_bytes(QO_Q4_K, QO_EMBD) * QO_FF;
    const size_t dn_bytes = qo_row_bytes(L->t_down, QO_FF) * QO_EMBD;
    moe_task_ctx mc = { L, sel, wt, xq, xd, xs, pacc, ge_bytes, dn_bytes };
    qo_pfor(T * QO_EXPERT_USED, moe_tasks, &mc);
    memset(out, 0, sizeof(float) * (size_t)T * QO_EMBD);
    for (int t = 0; t < T; t++) {
        float *acc = out + (size_t)t * QO_EMBD;
        for (int k = 0; k < QO_EXPERT_USED; k++) {
            const float *part = pacc + ((size_t)t * QO_EXPERT_USED + k) * QO_EMBD;
            for (int i = 0; i < QO_EMBD; i++) acc[i] += part[i];
        }
        shared_expert(L, xq + (size_t)t * QO_EMBD, xd + (size_t)t * 8, xs + (size_t)t * 128, acc);
    }
    if (sel_out) memcpy(sel_out, sel, sizeof(int) * (size_t)T * 8);
    if (w_out) memcpy(w_out, wt, sizeof(float) * (size_t)T * 8);
    free(pacc);
    free(xq);
    free(xd);
    free(xs);
    free(sel);
    free(wt);
}

typedef struct {
    const uint8_t *W;
    size_t rb;
    int wtype, n_in, n_out, T;
    const int8_t *xq;
    const float *xd;
    const int16_t *xs;
    float *out;
} mm_ctx;

/* mm_worker (nn.c:276-289), q8k path */
static void mm_rows(void *arg, int r0, int r1)
{
    const mm_ctx *c = arg;
    for (int r = r0; r < r1; r++) {
        const uint8_t *wr = c->W + (size_t)r * c->rb;
        for (int t = 0; t < c->T; t++)
            c->out[(size_t)t * c->n_out + r] =
                qo_dot(wr, c->wtype, c->xq + (size_t)t * c->n_in,
                       c->xd + (size_t)t * (c->n_in / QO_QK_K),
                       c->xs + (size_t)t * (c->n_in / 16), c->n_in);
    }
}

/* The FFN half of a layer in qma_eval (nn.c:2246-2252):
 * xn = rms_norm(x2) * post_norm; out = moe_ffn(xn) + x2. */
void qo_moe_block(const qo_model *m, int il, const float *x2, int T, float *out,
                  int *sel, float *w)
{
    qo_moe_block_biased(m, il, x2, T, NULL, out, sel, w);
}

void qo_moe_block_biased(const qo_model *m, int il, const float *x2, int T, const float *bias, float *out,
                         int *sel, float *w)
{
    float *xn = malloc(sizeof(float) * (size_t)T * QO_EMBD);
    float *ra = malloc(sizeof(float) * (size_t)T * QO_EMBD);
    rms_norm_m(xn, x2, m->L[il].post_norm, QO_EMBD, T);
    moe_ffn_impl(m, il, xn, T, bias, ra, sel, w);
    for (size_t i = 0; i < (size_t)QO_EMBD * T; i++) out[i] = ra[i] + x2[i];
    free(xn);
    free(ra);
}

/* parallel matmul (rows independent; same per-element arithmetic) */
static void matmul_p(const float *x, const uint8_t *W, int n_in, int n_out, int T,
                     int wtype, float *out)
{
    int8_t *xq = malloc((size_t)T * n_in);
    float *xd = malloc((size_t)T * (n_in / QO_QK_K) * sizeof(float));
    int16_t *xs = malloc((size_t)T * (n_in / 16) * sizeof(int16_t));
    for (int t = 0; t < T; t++)
        qo_q8k_quant(x + (size_t)t * n_in, n_in, xq + (size_t)t * n_in,
                     xd + (size_t)t * (n_in / QO_QK_K), xs + (size_t)t * (n_in / 16));
    mm_ctx c = { W, qo_row_bytes(wtype, n_in), wtype, n_in, n_out, T, xq, xd, xs, out };
    qo_pfor(n_out, mm_rows, &c);
    free(xq);
    free(xd);
    free(xs);
}

/* ------------------------------------------------------ sequence state -- */
struct qo_state {
    int n_ctx, n_pos;
    float *conv[QO_LAYER];
    float *ssm[QO_LAYER];
    uint8_t *kv[QO_ATTN_LAYERS];      /* [2*HEAD_KV][n_ctx][240] K heads, then V */
    /* hierarchical context memory (nn.c:912-937, per process there) */
    float *sal[QO_ATTN_LAYERS];
    float *qf;
    int *live;
    uint8_t *tier;
    int live_n, n4, n_ring_q4, rebuilt_at, next_rebuild;
    uint8_t *pin_kv[QO_ATTN_LAYERS];  /* [2*HEAD_KV][H_PIN][240] */
    int32_t pin_pos[QO_HCM_H_PIN];
    float pin_sal[QO_ATTN_LAYERS][QO_HCM_H_PIN];
    int pin_n;
};

qo_state *qo_state_new(int n_ctx)
{
    qo_state *s = calloc(1, sizeof(*s));
    if (!s) return NULL;
    s->n_ctx = n_ctx;
    for (int il = 0; il < QO_LAYER; il++) {
        if (QO_IS_ATTN(il)) {
            s->kv[il / 4] = calloc((size_t)2 * QO_HEAD_KV * n_ctx, QO_KVQ_SLOT);
            s->sal[il / 4] = calloc((size_t)n_ctx, sizeof(float));
            s->pin_kv[il / 4] = calloc((size_t)2 * QO_HEAD_KV * QO_HCM_H_PIN, QO_KVQ_SLOT);
        } else {
            s->conv[il] = calloc((size_t)QO_CONV_DIM * 3, sizeof(float));
            s->ssm[il] = calloc((size_t)QO_VHEADS * QO_STATE * QO_STATE, sizeof(float));
        }
    }
    s->qf = calloc((size_t)n_ctx, sizeof(float));
    s->live = calloc((size_t)n_ctx, sizeof(int));
    s->tier = calloc((size_t)n_ctx, 1);
    memset(s->pin_pos, -1, sizeof(s->pin_pos));
    s->next_rebuild = QO_HCM_REBUILD;
    return s;
}

void qo_state_free(qo_state *s)
{
    if (!s) return;
    for (int i = 0; i < QO_LAYER; i++) { free(s->conv[i]); free(s->ssm[i]); }
    for (int i = 0; i < QO_ATTN_LAYERS; i++) { free(s->kv[i]); free(s->sal[i]); free(s->pin_kv[i]); }
    free(s->qf);
    free(s->live);
    free(s->tier);
    free(s);
}

int qo_state_n_pos(const qo_state *s) { return s->n_pos; }

/* A qma session resumed in a fresh process (agent.c:765-816): the KV slab
 * file (runstate_init_kv's layout, nn.c:1878-1935) and the salience file
 * read as hcm_load reads it (nn.c:1173-1209) into hcm_init's fresh
 * bookkeeping (nn.c:947-970: tiers, live index and quantisation scores
 * cleared, next rebuild at 128), the position count as runstate_load sets
 * it.  The recurrent state is not read (callers drive single layers).
 * Returns 0, or -1 when a file is missing, short or for another n_ctx. */
int qo_state_resume(qo_state *s, const char *kv_path, const char *sal_path, int n_pos)
{
    const size_t per = (size_t)2 * QO_HEAD_KV * s->n_ctx * QO_KVQ_SLOT;
    FILE *f = fopen(kv_path, "rb");
    if (!f) return -1;
    for (int l = 0; l < QO_ATTN_LAYERS; l++)
        if (fread(s->kv[l], 1, per, f) != per) { fclose(f); return -1; }
    fclose(f);
    memset(s->tier, 0, (size_t)s->n_ctx);
    memset(s->qf, 0, sizeof(float) * (size_t)s->n_ctx);
    memset(s->live, 0, sizeof(int) * (size_t)s->n_ctx);
    s->live_n = s->n4 = s->n_ring_q4 = s->rebuilt_at = 0;
    s->next_rebuild = QO_HCM_REBUILD;
    memset(s->pin_pos, -1, sizeof(s->pin_pos));
    memset(s->pin_sal, 0, sizeof(s->pin_sal));
    s->pin_n = 0;
    f = fopen(sal_path, "rb");
    if (!f) return -1;
    uint32_t nc = 0;
    if (fread(&nc, 4, 1, f) != 1 || (int)nc != s->n_ctx) { fclose(f); return -1; }
    for (int l = 0; l < QO_ATTN_LAYERS; l++)
        if (fread(s->sal[l], sizeof(float), (size_t)s->n_ctx, f) != (size_t)s->n_ctx) { fclose(f); return -1; }
    s->n_pos = n_pos;
    int ok = fread(s->pin_pos, sizeof(int32_t), QO_HCM_H_PIN, f) == (size_t)QO_HCM_H_PIN;
    for (int l = 0; l < QO_ATTN_LAYERS && ok; l++)
        ok = fread(s->pin_sal[l], sizeof(float), QO_HCM_H_PIN, f) == (size_t)QO_HCM_H_PIN;
    for (int l = 0; l < QO_ATTN_LAYERS && ok; l++)
        ok = fread(s->pin_kv[l], (size_t)2 * QO_HEAD_KV * QO_HCM_H_PIN, QO_KVQ_SLOT, f) == (size_t)QO_KVQ_SLOT;
    fclose(f);
    if (!ok) { memset(s->pin_pos, -1, sizeof(s->pin_pos)); return 0; }   /* optional arena */
    for (int a = 0; a < QO_HCM_H_PIN; a++) s->pin_n += s->pin_pos[a] >= 0;
    return 0;
}

/* The live index's segments after the last rebuild: [0, n_ring_q4) ring q4,
 * [n_ring_q4, n4) arena q4, [n4, live_n) ring q2 (parity aid). */
void qo_state_live_segments(const qo_state *s, int *n_ring_q4, int *n4, int *live_n)
{
    *n_ring_q4 = s->n_ring_q4;
    *n4 = s->n4;
    *live_n = s->live_n;
}
const uint8_t *qo_state_kv_slot(const qo_state *s, int lay, int head, int slot)
{
    return s->kv[lay] + ((size_t)head * s->n_ctx + slot) * QO_KVQ_SLOT;
}
float *qo_state_conv(qo_state *s, int il) { return s->conv[il]; }
float *qo_state_ssm(qo_state *s, int il) { return s->ssm[il]; }

/* ---------------------------------------------------------------- GDN -- */
static void conv1d_layer(float *state, const float *x, const float *w, float *out, int T)
{
    for (int ch = 0; ch < QO_CONV_DIM; ch++) {
        float *st = state + (size_t)ch * 3;
        const float *wc = w + (size_t)ch * QO_CONV;
        float *oc = out + (size_t)ch * T;
        for (int t = 0; t < T; t++) {
            float sum = 0.0f;
            for (int k = 0; k < QO_CONV; k++) {
                const float v = (t + k < 3) ? st[t + k] : x[(size_t)(t + k - 3) * QO_CONV_DIM + ch];
                sum += v * wc[k];
            }
            oc[t] = sum;
        }
        float nst[3];
        for (int j = 0; j < 3; j++)
            nst[j] = (T + j < 3) ? st[T + j] : x[(size_t)(T + j - 3) * QO_CONV_DIM + ch];
        for (int j = 0; j < 3; j++) st[j] = nst[j];
    }
}

static void l2norm_heads(float *x, int T)
{
    const size_t TS = (size_t)QO_STATE * QO_VHEADS * 3;
    for (int t = 0; t < T; t++) {
        float *base = x + (size_t)t * TS;
        for (int h = 0; h < QO_VHEADS; h++) {
            float *v = base + (size_t)h * QO_STATE;
            double sum = 0.0;
            for (int i = 0; i < QO_STATE; i++) sum += (double)v[i] * v[i];
            const float r = 1.0f / fmaxf(sqrtf((float)sum), 1e-6f);
            for (int i = 0; i < QO_STATE; i++) v[i] *= r;
        }
    }
}

static void gdn_head(float *M, const float *q0, const float *k0, const float *v0,
                     const float *gate, const float *beta, float *out, int h, int T)
{
    const int S = QO_STATE, H = QO_VHEADS;
    const size_t ts = (size_t)S * H * 3;
    const float scale = 1.0f / sqrtf((float)S);
    const int qh = h % QO_KHEADS;
    for (int t = 0; t < T; t++) {
        const float *qp = q0 + (size_t)t * ts + (size_t)qh * S;
        const float *kp = k0 + (size_t)t * ts + (size_t)qh * S;
        const float *vp = v0 + (size_t)t * ts + (size_t)h * S;
        float *op = out + (size_t)t * H * S + (size_t)h * S;
        const float g = gate[(size_t)t * H + h];
        const float b = beta[(size_t)t * H + h];
        const float expg = expf(g);
        float dq[QO_STATE], dk[QO_STATE];
        for (int j = 0; j < S; j++) {
            const float *Mj = M + (size_t)j * S;
            float s1 = 0.0f, s2 = 0.0f;
            for (int i = 0; i < S; i++) { s1 += Mj[i] * qp[i]; s2 += Mj[i] * kp[i]; }
            dq[j] = s1;
            dk[j] = s2;
        }
        float kq = 0.0f;
        for (int i = 0; i < S; i++) kq += kp[i] * qp[i];
        for (int j = 0; j < S; j++) {
            const float delta = (vp[j] - expg * dk[j]) * b;
            float *Mj = M + (size_t)j * S;
            for (int i = 0; i < S; i++) Mj[i] = expg * Mj[i] + kp[i] * delta;
            op[j] = (expg * dq[j] + delta * kq) * scale;
        }
    }
}

typedef struct {
    float *ssm;
    const float *gkv, *gt, *beta;
    float *gdout;
    int T;
} gdn_ctx;

static void gdn_heads(void *arg, int h0, int h1)
{
    const gdn_ctx *c = arg;
    for (int h = h0; h < h1; h++)
        gdn_head(c->ssm + (size_t)h * QO_STATE * QO_STATE, c->gkv, c->gkv + QO_VAL_DIM,
                 c->gkv + 2 * QO_VAL_DIM, c->gt, c->beta, c->gdout, h, c->T);
}

void qo_gdn_layer(const qo_model *m, qo_state *s, int il, const float *xn, int T, float *ra)
{
    const qo_layer *L = &m->L[il];
    float *qkv = malloc(sizeof(float) * (size_t)T * QO_CONV_DIM);
    float *z = malloc(sizeof(float) * (size_t)T * QO_VAL_DIM);
    float *beta = malloc(sizeof(float) * (size_t)T * QO_VHEADS);
    float *gt = malloc(sizeof(float) * (size_t)T * QO_VHEADS);
    float *cout = malloc(sizeof(float) * (size_t)T * QO_CONV_DIM);
    float *gkv = malloc(sizeof(float) * (size_t)T * QO_STATE * QO_VHEADS * 3);
    float *gdout = malloc(sizeof(float) * (size_t)T * QO_VAL_DIM);
    matmul_p(xn, L->wqkv, QO_EMBD, QO_CONV_DIM, T, L->t_wqkv, qkv);
    matmul_p(xn, L->attn_gate, QO_EMBD, QO_VAL_DIM, T, L->t_gate, z);
    matmul_p(xn, L->ssm_beta, QO_EMBD, QO_VHEADS, T, L->t_beta, beta);
    for (size_t i = 0; i < (size_t)QO_VHEADS * T; i++) beta[i] = 1.0f / (1.0f + expf(-beta[i]));
    matmul_p(xn, L->ssm_alpha, QO_EMBD, QO_VHEADS, T, L->t_alpha, gt);
    for (int t = 0; t < T; t++)
        for (int h = 0; h < QO_VHEADS; h++) {
            const float a = gt[(size_t)t * QO_VHEADS + h] + L->ssm_dt[h];
            const float sp = a > 20.0f ? a : log1pf(expf(a));
            gt[(size_t)t * QO_VHEADS + h] = sp * L->ssm_a[h];
        }
    conv1d_layer(s->conv[il], qkv, L->conv1d, cout, T);
    for (size_t i = 0; i < (size_t)QO_CONV_DIM * T; i++) cout[i] = silu(cout[i]);
    const int S = QO_STATE;
    for (int t = 0; t < T; t++)
        for (int h = 0; h < QO_VHEADS; h++) {
            const int qh = h % QO_KHEADS;
            float *o = gkv + (size_t)t * S * QO_VHEADS * 3 + (size_t)h * S;
            for (int i = 0; i < S; i++) {
                o[i] = cout[(size_t)(qh * S + i) * T + t];
                o[S * QO_VHEADS + i] = cout[(size_t)(QO_KEY_DIM + qh * S + i) * T + t];
                o[2 * S * QO_VHEADS + i] = cout[(size_t)(QO_KEY_DIM * 2 + h * S + i) * T + t];
            }
        }
    l2norm_heads(gkv, T);
    l2norm_heads(gkv + QO_VAL_DIM, T);
    gdn_ctx gc = { s->ssm[il], gkv, gt, beta, gdout, T };
    qo_pfor(QO_VHEADS, gdn_heads, &gc);
    for (int t = 0; t < T; t++)
        for (int h = 0; h < QO_VHEADS; h++)
            rms_norm_inplace_rw(gdout + (size_t)t * QO_VAL_DIM + (size_t)h * S, L->ssm_norm, S);
    for (size_t i = 0; i < (size_t)QO_VAL_DIM * T; i++) z[i] = gdout[i] * silu(z[i]);
    matmul_p(z, L->ssm_out, QO_VAL_DIM, QO_EMBD, T, L->t_out, ra);
    free(qkv); free(z); free(beta); free(gt); free(cout); free(gkv); free(gdout);
}

/* ----------------------------------------------------------------- kvq -- */
static inline int clamp_q(int v, int hi) { return v < 0 ? 0 : (v > hi ? hi : v); }

void qo_kvq4_quant(const float *x, uint8_t *slot)
{
    for (int sb = 0; sb < 8; sb++) {
        const float *xp = x + sb * 32;
        uint8_t *q = slot + sb * 20;
        float mn = xp[0], mx = xp[0];
        for (int i = 1; i < 32; i++) {
            if (xp[i] < mn) mn = xp[i];
            if (xp[i] > mx) mx = xp[i];
        }
        float d = (mx - mn) / 15.0f;
        if (!(d > 0)) d = 1.0f;
        const uint16_t dh = qo_float_to_half(d), mh = qo_float_to_half(mn);
        memcpy(q, &dh, 2);
        memcpy(q + 2, &mh, 2);
        for (int i = 0; i < 32; i++) {
            const int qi = clamp_q((int)lrintf((xp[i] - mn) / d), 15);
            if (i & 1) q[4 + i / 2] = (uint8_t)((q[4 + i / 2] & 0x0F) | (qi << 4));
            else       q[4 + i / 2] = (uint8_t)((q[4 + i / 2] & 0xF0) | qi);
        }
    }
}

void qo_kvq2_quant(const float *x, uint8_t *slot)
{
    for (int sb = 0; sb < 4; sb++) {
        const float *xp = x + sb * 64;
        uint8_t *q = slot + QO_KVQ2_OFF + sb * 20;
        float mn = xp[0], mx = xp[0];
        for (int i = 1; i < 64; i++) {
            if (xp[i] < mn) mn = xp[i];
            if (xp[i] > mx) mx = xp[i];
        }
        float d = (mx - mn) / 3.0f;
        if (!(d > 0)) d = 1.0f;
        const uint16_t dh = qo_float_to_half(d), mh = qo_float_to_half(mn);
        memcpy(q, &dh, 2);
        memcpy(q + 2, &mh, 2);
        /* the reference ORs into the record without clearing it first
           (kvq.c:67); records are only ever written once per slot in the
           configurations here (the ring never wraps) */
        for (int i = 0; i < 64; i++) {
            const int qi = clamp_q((int)lrintf((xp[i] - mn) / d), 3);
            q[4 + i / 4] |= (uint8_t)(qi << (2 * (i & 3)));
        }
    }
}

static inline void sub_meta(const uint8_t *rec, int sb, float *d, float *m)
{
    uint16_t dh, mh;
    memcpy(&dh, rec + sb * 20, 2);
    memcpy(&mh, rec + sb * 20 + 2, 2);
    *d = qo_half_to_float(dh);
    *m = qo_half_to_float(mh);
}

float qo_kvq4_qf(const uint8_t *slot, const float *x)
{
    double se = 0, sx = 0;
    for (int sb = 0; sb < 8; sb++) {
        float d, m;
        sub_meta(slot, sb, &d, &m);
        const uint8_t *q = slot + sb * 20 + 4;
        for (int i = 0; i < 32; i++) {
            const int qi = (i & 1) ? (q[i / 2] >> 4) : (q[i / 2] & 0x0F);
            const float v = qi * d + m;
            const float e = v - x[sb * 32 + i];
            se += (double)e * e;
            sx += (double)x[sb * 32 + i] * x[sb * 32 + i];
        }
    }
    if (sx <= 0) return 0.0f;
    return (float)sqrt(se / sx);
}

/* element value of a q4 / q2 record: m + q*d, unfused (vmlaq_f32) */
static inline float q4_elem(const uint8_t *rec, int i, float d, float m)
{
    const uint8_t b = rec[(i / 32) * 20 + 4 + (i % 32) / 2];
    const int q = (i & 1) ? (b >> 4) : (b & 0xF);
    const float p = (float)q * d;
    return m + p;
}
static inline float q2_elem(const uint8_t *rec, int i, float d, float m)
{
    const uint8_t b = rec[(i / 64) * 20 + 4 + (i % 64) / 4];
    const int q = (b >> (2 * (i & 3))) & 3;
    const float p = (float)q * d;
    return m + p;
}

float qo_kvq4_dot(const uint8_t *rec, const float *x)
{
    float acc = 0.0f;
    for (int sb = 0; sb < 8; sb++) {
        float d, m;
        sub_meta(rec, sb, &d, &m);
        float a[4] = {0, 0, 0, 0};
        for (int k = 0; k < 8; k++)
            for (int l = 0; l < 4; l++) {
                const int i = sb * 32 + 4 * k + l;
                const float p = q4_elem(rec, i, d, m) * x[i];
                a[l] = a[l] + p;
            }
        const float s01 = a[0] + a[1], s23 = a[2] + a[3];
        acc += s01 + s23;
    }
    return acc;
}

float qo_kvq2_dot(const uint8_t *rec, const float *x)
{
    float acc = 0.0f;
    for (int sb = 0; sb < 4; sb++) {
        float d, m;
        sub_meta(rec, sb, &d, &m);
        float a[4] = {0, 0, 0, 0};
        for (int k = 0; k < 16; k++)
            for (int l = 0; l < 4; l++) {
                const int i = sb * 64 + 4 * k + l;
                const float p = q2_elem(rec, i, d, m) * x[i];
                a[l] = a[l] + p;
            }
        const float s01 = a[0] + a[1], s23 = a[2] + a[3];
        acc += s01 + s23;
    }
    return acc;
}

void qo_kvq4_vacc(const uint8_t *rec, float w, float *o)
{
    for (int sb = 0; sb < 8; sb++) {
        float d, m;
        sub_meta(rec, sb, &d, &m);
        for (int i = sb * 32; i < sb * 32 + 32; i++) {
            const float p = w * q4_elem(rec, i, d, m);
            o[i] = o[i] + p;
        }
    }
}

void qo_kvq2_vacc(const uint8_t *rec, float w, float *o)
{
    for (int sb = 0; sb < 4; sb++) {
        float d, m;
        sub_meta(rec, sb, &d, &m);
        for (int i = sb * 64; i < sb * 64 + 64; i++) {
            const float p = w * q2_elem(rec, i, d, m);
            o[i] = o[i] + p;
        }
    }
}

/* ----------------------------------------------------------------- HCM -- */
static inline int hcm_slot(int p, int n_ctx)
{
    if (p < QO_HCM_SINK) return p;
    return QO_HCM_SINK + (p - QO_HCM_SINK) % (n_ctx - QO_HCM_SINK);
}

typedef struct { float sc; int pos; int is_arena; } hcm_ent;

static void heap_push(hcm_ent *heap, int *hn, float sc, int pos, int is_a)
{
    if (*hn < QO_HCM_H_PIN) {
        int i = (*hn)++;
        heap[i].sc = sc; heap[i].pos = pos; heap[i].is_arena = is_a;
        while (i > 0) {
            const int par = (i - 1) / 2;
            if (heap[par].sc <= heap[i].sc) break;
            hcm_ent t = heap[par]; heap[par] = heap[i]; heap[i] = t;
            i = par;
        }
    } else if (sc > heap[0].sc) {
        heap[0].sc = sc; heap[0].pos = pos; heap[0].is_arena = is_a;
        int i = 0;
        for (;;) {
            const int lc = 2 * i + 1, rc = 2 * i + 2;
            int sm = i;
            if (lc < *hn && heap[lc].sc < heap[sm].sc) sm = lc;
            if (rc < *hn && heap[rc].sc < heap[sm].sc) sm = rc;
            if (sm == i) break;
            hcm_ent t = heap[sm]; heap[sm] = heap[i]; heap[i] = t;
            i = sm;
        }
    }
}

static void hcm_rebuild(qo_state *s, int n_pos)
{
    const int cap = s->n_ctx;
    const int ring = cap - QO_HCM_SINK;
    const int oldest = n_pos - ring;
    if (n_pos <= QO_HCM_SINK + QO_HCM_W_HOT) {
        for (int p = 0; p < n_pos; p++) {
            s->live[p] = hcm_slot(p, cap);
            s->tier[hcm_slot(p, cap)] = 2;
        }
        s->live_n = s->n4 = s->n_ring_q4 = n_pos;
        return;
    }
    int n = 0;
    int hot_lo = n_pos - QO_HCM_W_HOT;
    if (hot_lo < oldest) hot_lo = oldest;
    for (int p = 0; p < QO_HCM_SINK && p < hot_lo; p++) {
        s->live[n++] = hcm_slot(p, cap);
        s->tier[hcm_slot(p, cap)] = 2;
    }
    for (int p = hot_lo; p < n_pos; p++) {
        s->live[n++] = hcm_slot(p, cap);
        s->tier[hcm_slot(p, cap)] = 2;
    }
    int cand_lo = QO_HCM_SINK;
    if (oldest > cand_lo) cand_lo = oldest;
    hcm_ent *heap = malloc(sizeof(hcm_ent) * QO_HCM_H_PIN);
    int hn = 0;
    for (int p = cand_lo; p < hot_lo; p++) {
        const int sl = hcm_slot(p, cap);
        float sc = 0.0f;
        for (int l = 0; l < QO_ATTN_LAYERS; l++) sc += s->sal[l][sl];
        const float qf = s->qf[sl] > 0 ? s->qf[sl] : 0.05f;
        sc = sc * (1.0f - QO_HCM_QF_BIAS * qf);
        heap_push(heap, &hn, sc, p, 0);
    }
    for (int a = 0; a < QO_HCM_H_PIN; a++) {
        if (s->pin_pos[a] < 0) continue;
        float sc = 0.0f;
        for (int l = 0; l < QO_ATTN_LAYERS; l++) sc += s->pin_sal[l][a];
        heap_push(heap, &hn, sc, a, 1);
    }
    int *new_arena = malloc(sizeof(int) * QO_HCM_H_PIN);
    for (int i = 0; i < hn; i++) new_arena[i] = heap[i].is_arena ? heap[i].pos : -1;
    for (int i = 0; i < hn; i++) {
        if (heap[i].is_arena) continue;
        const int src = hcm_slot(heap[i].pos, cap);
        int slot = -1;
        for (int a = 0; a < QO_HCM_H_PIN; a++) if (s->pin_pos[a] < 0) { slot = a; break; }
        if (slot < 0) {
            float worst = 1e30f;
            int wi = -1;
            for (int a = 0; a < QO_HCM_H_PIN; a++) {
                if (s->pin_pos[a] < 0) continue;
                int kept = 0;
                for (int k = 0; k < hn; k++) if (new_arena[k] == a) { kept = 1; break; }
                if (kept) continue;
                float sc = 0.0f;
                for (int l = 0; l < QO_ATTN_LAYERS; l++) sc += s->pin_sal[l][a];
                if (sc < worst) { worst = sc; wi = a; }
            }
            slot = wi;
        }
        if (slot < 0) continue;
        new_arena[i] = slot;
        for (int l = 0; l < QO_ATTN_LAYERS; l++) {
            for (int kh = 0; kh < 2 * QO_HEAD_KV; kh++)
                memcpy(s->pin_kv[l] + ((size_t)kh * QO_HCM_H_PIN + slot) * QO_KVQ_SLOT,
                       s->kv[l] + ((size_t)kh * cap + src) * QO_KVQ_SLOT, QO_KVQ_SLOT);
            s->pin_sal[l][slot] = s->sal[l][src];
        }
        s->pin_pos[slot] = heap[i].pos;
    }
    s->pin_n = 0;
    for (int i = 0; i < hn; i++) if (new_arena[i] >= 0) s->pin_n++;
    const int n_ring_q4 = n;
    for (int i = 0; i < hn; i++) {
        if (new_arena[i] < 0) continue;
        s->live[n++] = QO_HCM_ARENA_BASE + new_arena[i];
    }
    int gist_lo = hot_lo - QO_HCM_W_GIST;
    if (gist_lo < cand_lo) gist_lo = cand_lo;
    for (int p = gist_lo; p < hot_lo; p++) {
        const int sl = hcm_slot(p, cap);
        if (s->tier[sl] == 2) continue;
        s->live[n++] = sl;
        s->tier[sl] = 1;
    }
    for (int p = cand_lo; p < gist_lo; p++) {
        const int sl = hcm_slot(p, cap);
        if (s->tier[sl] != 2) s->tier[sl] = 0;
    }
    s->live_n = n;
    s->n4 = n_ring_q4 + hn;
    s->n_ring_q4 = n_ring_q4;
    free(heap);
    free(new_arena);
}

/* --------------------------------------------------------- attention -- */
static void rope_imrope(float *x, int n_head, int hstride, int T, const int *pos)
{
    const float theta_scale = powf(QO_FREQ_BASE, -2.0f / QO_ROT);
    for (int t = 0; t < T; t++) {
        float cosv[QO_ROT / 2], sinv[QO_ROT / 2];
        float theta = (float)pos[t];
        for (int j = 0; j < QO_ROT / 2; j++) {
            cosv[j] = cosf(theta);
            sinv[j] = sinf(theta);
            theta *= theta_scale;
        }
        for (int h = 0; h < n_head; h++) {
            float *v = x + (size_t)t * n_head * hstride + (size_t)h * hstride;
            for (int j = 0; j < QO_ROT / 2; j++) {
                const float x0 = v[j], x1 = v[j + QO_ROT / 2];
                v[j] = x0 * cosv[j] - x1 * sinv[j];
                v[j + QO_ROT / 2] = x0 * sinv[j] + x1 * cosv[j];
            }
        }
    }
}

static void kv_append(qo_state *s, int lay, const float *K, const float *V, int T, int n_pos)
{
    uint8_t *cb = s->kv[lay];
    const int cap = s->n_ctx;
    for (int t = 0; t < T; t++) {
        const int slot = hcm_slot(n_pos + t, cap);
        float qf_k = 0, qf_v = 0;
        for (int kh = 0; kh < QO_HEAD_KV; kh++) {
            const uint8_t *Ks = cb + ((size_t)kh * cap + slot) * QO_KVQ_SLOT;
            const uint8_t *Vs = cb + ((size_t)(QO_HEAD_KV + kh) * cap + slot) * QO_KVQ_SLOT;
            qf_k += qo_kvq4_qf(Ks, K + (size_t)t * QO_WKV_DIM + (size_t)kh * QO_HEAD_DIM);
            qf_v += qo_kvq4_qf(Vs, V + (size_t)t * QO_WKV_DIM + (size_t)kh * QO_HEAD_DIM);
        }
        s->qf[slot] = (qf_k + qf_v) / (2.0f * QO_HEAD_KV);
        for (int kh = 0; kh < QO_HEAD_KV; kh++) {
            uint8_t *Ks = cb + ((size_t)kh * cap + slot) * QO_KVQ_SLOT;
            uint8_t *Vs = cb + ((size_t)(QO_HEAD_KV + kh) * cap + slot) * QO_KVQ_SLOT;
            const float *kv = K + (size_t)t * QO_WKV_DIM + (size_t)kh * QO_HEAD_DIM;
            const float *vv = V + (size_t)t * QO_WKV_DIM + (size_t)kh * QO_HEAD_DIM;
            qo_kvq4_quant(kv, Ks);
            qo_kvq2_quant(kv, Ks);
            qo_kvq4_quant(vv, Vs);
            qo_kvq2_quant(vv, Vs);
        }
        s->tier[slot] = 2;
        for (int l = 0; l < QO_ATTN_LAYERS; l++) s->sal[l][slot] = 0.0f;
    }
}

typedef struct {
    const int *live;
    int n_rq, n4;
    const uint8_t *Ks, *ApK;
    const float *q;
    float scale;
    float *scores;
} score_ctx;

/* Q.K scores over the three live segments [ring q4 | arena q4 | ring q2] */
static void score_live(void *arg, int j0, int j1)
{
    const score_ctx *c = arg;
    for (int j = j0; j < j1; j++) {
        const int e = c->live[j];
        float v;
        if (j < c->n_rq) v = qo_kvq4_dot(c->Ks + (size_t)e * QO_KVQ_SLOT, c->q) * c->scale;
        else if (j < c->n4) v = qo_kvq4_dot(c->ApK + (size_t)(e - QO_HCM_ARENA_BASE) * QO_KVQ_SLOT, c->q) * c->scale;
        else v = qo_kvq2_dot(c->Ks + (size_t)e * QO_KVQ_SLOT + QO_KVQ2_OFF, c->q) * c->scale;
        c->scores[j] = v;
    }
}

/* One head's queries t0..t1-1: scores, softmax and P.V over the live
 * entries plus the dense tail since the last rebuild.  Leaves each query's
 * exp-scores in scores + t * nmax and its denominator in sums[t] for the
 * salience update, which runs afterwards in the reference's order. */
typedef struct {
    const qo_state *s;
    const uint8_t *Ks, *Vs, *ApK, *ApV;
    const float *Q;
    float *out, *scores, *sums;
    int h, n_pos, nmax;
    float scale;
} head_ctx;

static void head_queries(void *arg, int t0, int t1)
{
    const head_ctx *c = arg;
    const qo_state *s = c->s;
    const int cap = s->n_ctx;
    const int use_live = s->live_n > 0;
    const int nl_all = s->live_n, n4 = s->n4, n_rq = s->n_ring_q4, batch_lo = s->rebuilt_at;
    for (int t = t0; t < t1; t++) {
        const int abs = c->n_pos + t;
        const float *q = c->Q + (size_t)t * QO_WQ_DIM + (size_t)c->h * (QO_HEAD_DIM * 2);
        float *scores = c->scores + (size_t)t * c->nmax;
        const int nl = use_live ? nl_all : abs + 1;
        float maxs = -1e30f;
        int nk;
        if (use_live) {
            score_ctx sc = { s->live, n_rq, n4, c->Ks, c->ApK, q, c->scale, scores };
            score_live(&sc, 0, nl);
            for (int p = batch_lo; p <= abs; p++)
                scores[nl + (p - batch_lo)] =
                    qo_kvq4_dot(c->Ks + (size_t)hcm_slot(p, cap) * QO_KVQ_SLOT, q) * c->scale;
            nk = nl + (abs - batch_lo + 1);
        } else {
            for (int p = 0; p <= abs; p++)
                scores[p] = qo_kvq4_dot(c->Ks + (size_t)hcm_slot(p, cap) * QO_KVQ_SLOT, q) * c->scale;
            nk = abs + 1;
        }
        for (int j = 0; j < nk; j++) if (scores[j] > maxs) maxs = scores[j];
        float sum = 0.0f;
        for (int j = 0; j < nk; j++) { scores[j] = expf(scores[j] - maxs); sum += scores[j]; }
        float oacc[QO_HEAD_DIM];
        memset(oacc, 0, sizeof(oacc));
        if (use_live) {
            for (int j = 0; j < nl; j++) {
                const int e = s->live[j];
                if (j < n_rq) qo_kvq4_vacc(c->Vs + (size_t)e * QO_KVQ_SLOT, scores[j], oacc);
                else if (j < n4) qo_kvq4_vacc(c->ApV + (size_t)(e - QO_HCM_ARENA_BASE) * QO_KVQ_SLOT, scores[j], oacc);
                else qo_kvq2_vacc(c->Vs + (size_t)e * QO_KVQ_SLOT + QO_KVQ2_OFF, scores[j], oacc);
            }
            for (int p = batch_lo; p <= abs; p++)
                qo_kvq4_vacc(c->Vs + (size_t)hcm_slot(p, cap) * QO_KVQ_SLOT, scores[nl + (p - batch_lo)], oacc);
        } else {
            for (int p = 0; p <= abs; p++)
                qo_kvq4_vacc(c->Vs + (size_t)hcm_slot(p, cap) * QO_KVQ_SLOT, scores[p], oacc);
        }
        const float inv = 1.0f / sum;
        float *o = c->out + (size_t)t * QO_WO_DIM + (size_t)c->h * QO_HEAD_DIM;
        for (int d = 0; d < QO_HEAD_DIM; d++) o[d] = oacc[d] * inv;
        c->sums[t] = sum;
    }
}

/* attn_worker (nn.c:1215-1446) for all 16 heads, heads in order 0..15.
 * A head's queries are independent of one another (split over threads);
 * the salience EMA then folds them in head-major, query-minor order. */
static void attn_heads(qo_state *s, int lay, const float *Q, float *out, int T, int n_pos)
{
    const int cap = s->n_ctx;
    const uint8_t *cb = s->kv[lay];
    const int use_live = s->live_n > 0;
    const int nmax = (use_live ? s->live_n + (n_pos + T - s->rebuilt_at) : n_pos + T) + 1;
    float *scores = malloc(sizeof(float) * (size_t)nmax * T);
    float *sums = malloc(sizeof(float) * (size_t)T);
    const int nl_all = s->live_n, n4 = s->n4, n_rq = s->n_ring_q4, batch_lo = s->rebuilt_at;
    for (int h = 0; h < QO_HEAD; h++) {
        const int kh = h / (QO_HEAD / QO_HEAD_KV);
        head_ctx hc = {
            s, cb + (size_t)kh * cap * QO_KVQ_SLOT, cb + (size_t)(QO_HEAD_KV + kh) * cap * QO_KVQ_SLOT,
            s->pin_kv[lay] + (size_t)kh * QO_HCM_H_PIN * QO_KVQ_SLOT,
            s->pin_kv[lay] + (size_t)(QO_HEAD_KV + kh) * QO_HCM_H_PIN * QO_KVQ_SLOT,
            Q, out, scores, sums, h, n_pos, nmax, 1.0f / sqrtf((float)QO_HEAD_DIM)
        };
        qo_pfor(T, head_queries, &hc);
        if (!use_live) continue;
        float *sal = s->sal[lay];
        for (int t = 0; t < T; t++) {
            const int abs = n_pos + t;
            const int nl = nl_all;
            const float *sc = scores + (size_t)t * nmax;
            const float sum = sums[t];
            for (int j = 0; j < n_rq && j < nl; j++) {
                const int sl = s->live[j];
                sal[sl] = (1 - QO_HCM_ALPHA) * sal[sl] + QO_HCM_ALPHA * (sc[j] / sum);
            }
            for (int j = n_rq; j < n4 && j < nl; j++) {
                const int a = s->live[j] - QO_HCM_ARENA_BASE;
                float *psal = s->pin_sal[lay];
                psal[a] = (1 - QO_HCM_ALPHA) * psal[a] + QO_HCM_ALPHA * (sc[j] / sum);
            }
            for (int j = n4; j < nl; j++) {
                const int sl = s->live[j];
                sal[sl] = (1 - QO_HCM_ALPHA) * sal[sl] + QO_HCM_ALPHA * (sc[j] / sum);
            }
            for (int p = batch_lo; p <= abs; p++) {
                const int sl = hcm_slot(p, cap);
                sal[sl] = (1 - QO_HCM_ALPHA) * sal[sl] +
                          QO_HCM_ALPHA * (sc[nl + (p - batch_lo)] / sum);
            }
        }
    }
    free(scores);
    free(sums);
}

static void attn_layer(const qo_model *m, qo_state *s, int il, const float *xn, int T,
                       int n_pos, float *ra)
{
    const qo_layer *L = &m->L[il];
    float *qfull = malloc(sizeof(float) * (size_t)T * QO_WQ_DIM);
    float *K = malloc(sizeof(float) * (size_t)T * QO_WKV_DIM);
    float *V = malloc(sizeof(float) * (size_t)T * QO_WKV_DIM);
    float *z = malloc(sizeof(float) * (size_t)T * QO_WO_DIM);
    float *aout = malloc(sizeof(float) * (size_t)T * QO_WO_DIM);
    int *pos = malloc(sizeof(int) * (size_t)T);
    matmul_p(xn, L->wq, QO_EMBD, QO_WQ_DIM, T, L->t_wq, qfull);
    matmul_p(xn, L->wk, QO_EMBD, QO_WKV_DIM, T, L->t_wk, K);
    matmul_p(xn, L->wv, QO_EMBD, QO_WKV_DIM, T, L->t_wv, V);
    for (int t = 0; t < T; t++)
        for (int h = 0; h < QO_HEAD; h++) {
            float *v = qfull + (size_t)t * QO_WQ_DIM + (size_t)h * (QO_HEAD_DIM * 2);
            rms_norm_inplace_rw(v, L->q_norm, QO_HEAD_DIM);
            memcpy(z + (size_t)t * QO_WO_DIM + (size_t)h * QO_HEAD_DIM, v + QO_HEAD_DIM,
                   QO_HEAD_DIM * sizeof(float));
        }
    for (int t = 0; t < T; t++)
        for (int h = 0; h < QO_HEAD_KV; h++)
            rms_norm_inplace_rw(K + (size_t)t * QO_WKV_DIM + (size_t)h * QO_HEAD_DIM, L->k_norm, QO_HEAD_DIM);
    for (int t = 0; t < T; t++) pos[t] = n_pos + t;
    rope_imrope(qfull, QO_HEAD, QO_HEAD_DIM * 2, T, pos);
    rope_imrope(K, QO_HEAD_KV, QO_HEAD_DIM, T, pos);
    kv_append(s, il / 4, K, V, T, n_pos);
    attn_heads(s, il / 4, qfull, aout, T, n_pos);
    for (size_t i = 0; i < (size_t)QO_WO_DIM * T; i++) aout[i] *= 1.0f / (1.0f + expf(-z[i]));
    matmul_p(aout, L->wo, QO_WO_DIM, QO_EMBD, T, L->t_wo, ra);
    free(qfull); free(K); free(V); free(z); free(aout); free(pos);
}

/* ------------------------------------------------------------ qma_eval -- */
static int eval_impl(const qo_model *m, qo_state *s, const int *tokens, int n_tokens,
                     float *logits, int logits_all, int n_layers, float *hidden);

/* One layer of qma_eval's loop body (nn.c:2105-2252) on T tokens at
 * positions n_pos.., from the residual x_in to the residual x_out, using
 * and updating that layer's state in s (no HCM rebuild: call with a state
 * whose live index is current).  Parity aid: lets a caller feed each layer
 * the engine's own input so differences cannot compound across layers. */
void qo_layer_forward(const qo_model *m, qo_state *s, int il, const float *x_in, int T,
                      int n_pos, float *x_out)
{
    const qo_layer *L = &m->L[il];
    float *xn = malloc(sizeof(float) * (size_t)T * QO_EMBD);
    float *ra = malloc(sizeof(float) * (size_t)T * QO_EMBD);
    float *x2 = malloc(sizeof(float) * (size_t)T * QO_EMBD);
    rms_norm_m(xn, x_in, L->attn_norm, QO_EMBD, T);
    if (QO_IS_ATTN(il)) attn_layer(m, s, il, xn, T, n_pos, ra);
    else qo_gdn_layer(m, s, il, xn, T, ra);
    for (size_t i = 0; i < (size_t)QO_EMBD * T; i++) x2[i] = ra[i] + x_in[i];
    qo_moe_block(m, il, x2, T, x_out, NULL, NULL);
    free(xn);
    free(ra);
    free(x2);
}

int qo_eval(const qo_model *m, qo_state *s, const int *tokens, int n_tokens,
            float *logits, int logits_all)
{
    return eval_impl(m, s, tokens, n_tokens, logits, logits_all, QO_LAYER, NULL);
}

/* qo_eval through the first n_layers layers only; the hidden state after
 * them goes to hidden [n_tokens][2048] (parity aid, no logits). */
int qo_eval_hidden(const qo_model *m, qo_state *s, const int *tokens, int n_tokens,
                   int n_layers, float *hidden)
{
    return eval_impl(m, s, tokens, n_tokens, NULL, 0, n_layers, hidden);
}

/* Layer il's mixer and its residual (nn.c:2105-2245) over n_tokens inputs
 * x_in [n_tokens][2048] taken from the caller instead of the layers below,
 * in qma_eval's chunks of 512 with the HCM rebuild at each chunk start
 * (nn.c:2081-2087), writing x_out = x_in + mixer(rms_norm(x_in)).  The
 * state's position advances by n_tokens.  Parity aid for long contexts: the
 * attention layer's heavy-hitter arena and salience are driven by the
 * caller's inputs alone. */
void qo_mixer_forward(const qo_model *m, qo_state *s, int il, const float *x_in, int n_tokens,
                      float *x_out)
{
    const qo_layer *L = &m->L[il];
    float *xn = malloc(sizeof(float) * (size_t)QO_MAX_CHUNK * QO_EMBD);
    float *ra = malloc(sizeof(float) * (size_t)QO_MAX_CHUNK * QO_EMBD);
    for (int done = 0; done < n_tokens;) {
        const int T = (n_tokens - done < QO_MAX_CHUNK) ? n_tokens - done : QO_MAX_CHUNK;
        const int pos_now = s->n_pos + done;
        if (pos_now >= s->next_rebuild) {
            hcm_rebuild(s, pos_now);
            s->rebuilt_at = pos_now;
            s->next_rebuild = pos_now + QO_HCM_REBUILD;
        }
        const float *x = x_in + (size_t)done * QO_EMBD;
        rms_norm_m(xn, x, L->attn_norm, QO_EMBD, T);
        if (QO_IS_ATTN(il)) attn_layer(m, s, il, xn, T, pos_now, ra);
        else qo_gdn_layer(m, s, il, xn, T, ra);
        for (size_t i = 0; i < (size_t)QO_EMBD * T; i++)
            x_out[(size_t)done * QO_EMBD + i] = ra[i] + x[i];
        done += T;
    }
    s->n_pos += n_tokens;
    free(xn);
    free(ra);
}

static int eval_impl(const qo_model *m, qo_state *s, const int *tokens, int n_tokens,
                     float *logits, int logits_all, int n_layers, float *hidden)
{
    const int TM = QO_MAX_CHUNK;
    float *x = malloc(sizeof(float) * (size_t)TM * QO_EMBD);
    float *xn = malloc(sizeof(float) * (size_t)TM * QO_EMBD);
    float *x2 = malloc(sizeof(float) * (size_t)TM * QO_EMBD);
    float *ra = malloc(sizeof(float) * (size_t)TM * QO_EMBD);
    const size_t erow = qo_row_bytes(m->t_embd, QO_EMBD);
    int done = 0;
    while (done < n_tokens) {
        const int T = (n_tokens - done < TM) ? n_tokens - done : TM;
        for (int t = 0; t < T; t++)
            qo_dequant_row(m->embd + (size_t)tokens[done + t] * erow, m->t_embd,
                           x + (size_t)t * QO_EMBD, QO_EMBD);
        const int pos_now = s->n_pos + done;
        if (pos_now >= s->next_rebuild) {
            hcm_rebuild(s, pos_now);
            s->rebuilt_at = pos_now;
            s->next_rebuild = pos_now + QO_HCM_REBUILD;
        }
        const int nl = n_layers < 0 ? -n_layers : n_layers;
        for (int il = 0; il < nl; il++) {
            const qo_layer *L = &m->L[il];
            rms_norm_m(xn, x, L->attn_norm, QO_EMBD, T);
            if (QO_IS_ATTN(il)) attn_layer(m, s, il, xn, T, pos_now, ra);
            else qo_gdn_layer(m, s, il, xn, T, ra);
            for (size_t i = 0; i < (size_t)QO_EMBD * T; i++) x2[i] = ra[i] + x[i];
            if (n_layers < 0 && il == nl - 1) {   /* stop after this layer's mixer */
                memcpy(x, x2, sizeof(float) * (size_t)QO_EMBD * T);
                break;
            }
            rms_norm_m(xn, x2, L->post_norm, QO_EMBD, T);
            qo_moe_ffn(m, il, xn, T, ra, NULL, NULL);
            for (size_t i = 0; i < (size_t)QO_EMBD * T; i++) x[i] = ra[i] + x2[i];
        }
        if (hidden) memcpy(hidden + (size_t)done * QO_EMBD, x, sizeof(float) * (size_t)QO_EMBD * T);
        if (n_layers < QO_LAYER) { done += T; continue; }
        rms_norm_m(xn, x, m->output_norm, QO_EMBD, T);
        if (logits_all) {
            if (logits)
                matmul_p(xn, m->output, QO_EMBD, m->n_vocab, T, m->t_output,
                         logits + (size_t)done * m->n_vocab);
        } else if (logits && done + T == n_tokens) {
            matmul_p(xn + (size_t)(T - 1) * QO_EMBD, m->output, QO_EMBD, m->n_vocab, 1,
                     m->t_output, logits);
        }
        done += T;
    }
    s->n_pos += n_tokens;
    free(x); free(xn); free(x2); free(ra);
    return 0;
}
