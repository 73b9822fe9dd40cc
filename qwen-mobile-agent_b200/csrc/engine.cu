// engine.cu -- the qma_eval replacement: device-resident qwen35moe weights,
// per-sequence state (KV ring, recurrent state, HCM tiers) and the forward
// loop, for prefill chunks and CUDA-graph decode steps.
//
// Reference: qma_eval (nn.c:2056-2308), runstate_init_kv (nn.c:1878-1979),
// hcm_rebuild (nn.c:981-1150), embed_row (nn.c:2044-2054), qma_load's tensor
// resolution (gguf.c:302-345), session files (runstate_save/load
// nn.c:2011-2042, hcm_save/load nn.c:1156-1209).
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "attn.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "layers.cuh"
#include "moe.cuh"
#include "synth.cuh"
#include "tc.cuh"

namespace qma {

constexpr int HCM_W_HOT = 4096, HCM_W_GIST = 32768, HCM_REBUILD = 128;   // nn.c:894-901
constexpr float HCM_QF_BIAS = 2.0f;

struct LayerW {
    const float *attn_norm = nullptr, *post_norm = nullptr;
    void *in_proj = nullptr;       // GDN: qkv | gate | beta | alpha ; attn: q | k | v
    int in_type = 0, in_rows = 0;
    void *out_proj = nullptr;      // ssm_out / attn_output, 4096 -> 2048
    int out_type = 0;
    const float *conv1d = nullptr, *dt = nullptr, *a = nullptr, *ssm_norm = nullptr;
    const float *q_norm = nullptr, *k_norm = nullptr;
    qma_cuda_moe_weights moe{};
};

}  // namespace qma

struct qma_cuda_model {
    int device = 0;
    int n_vocab = 0;
    std::vector<void *> allocs;
    void *embd = nullptr;
    int embd_type = 0;
    void *out = nullptr;
    int out_type = 0;
    const float *out_norm = nullptr;
    qma::LayerW L[qma::NLAYER];
    size_t weight_bytes = 0;
    // expert-cache holds (qma_ecache_hold / _release, ecache.c:500-520):
    // bookkeeping only, every record stays resident for the model's life
    std::mutex ec_mu;
    int ec_held = 0;
};

constexpr int ARG_CTAS = 64;      // CTAs of the greedy argmax

struct qma_cuda_state {
    qma_cuda_model *m = nullptr;
    int n_ctx = 0, n_pos = 0;
    cudaStream_t st = nullptr;
    std::vector<void *> allocs;
    // device state
    float *conv[qma::NLAYER] = {};
    float *ssm[qma::NLAYER] = {};
    uint8_t *kv[qma::NATTN] = {};
    uint8_t *arena[qma::NATTN] = {};
    uint8_t **kv_dev = nullptr, **arena_dev = nullptr;
    float *sal = nullptr;       // [10][n_ctx]
    float *pin_sal = nullptr;   // [10][2048]
    float *qf = nullptr;        // [n_ctx]
    int *live_dev = nullptr;    // [n_ctx]
    float *rope = nullptr;      // [n_ctx][32 cos | 32 sin]
    qma::StepParams *sp_dev = nullptr, *sp_host = nullptr;
    // activations, sized for MAX_CHUNK tokens
    int *tokens_dev = nullptr;
    float *x = nullptr, *x2 = nullptr, *proj = nullptr, *conv_out = nullptr, *gdo = nullptr;
    float *qr = nullptr, *z = nullptr;
    int8_t *xq = nullptr;
    float *xd = nullptr;
    int16_t *xs = nullptr;
    void *moe_scratch = nullptr;
    size_t moe_scratch_bytes = 0;
    float *logits = nullptr;    // [MAX_CHUNK][n_vocab] (logits_all) or [1][n_vocab]
    int logits_rows = 0;
    int *argmax_dev = nullptr;
    float *argmax_pv = nullptr;         // per-CTA partial maxima
    int *argmax_pi = nullptr;
    unsigned *argmax_cnt = nullptr;     // ticket, zero between steps
    unsigned *gdn_cnt = nullptr;        // [16] gated-norm tickets, zero between layers
    float *gdn_kq = nullptr;            // [MAX_CHUNK][16] k . q of a prefill chunk
    float *gdn_chunk = nullptr;         // chunked gated-delta scratch (W, U, P, G of a prefill chunk)
    // attention scratch, grown on demand
    float *scores = nullptr, *cmax = nullptr, *opart = nullptr, *lpart = nullptr, *ml = nullptr;
    size_t scores_cap = 0, cmax_cap = 0, opart_cap = 0, lpart_cap = 0;
    int2 *pairs_dev = nullptr;
    // host mirror of the HCM bookkeeping (nn.c:912-937)
    std::vector<int> live;
    std::vector<uint8_t> tier;
    std::vector<int> pin_pos;
    int live_n = 0, n4 = 0, n_ring_q4 = 0, rebuilt_at = 0, next_rebuild = HCM_REBUILD_INIT;
    float *h_sal = nullptr, *h_qf = nullptr, *h_pin_sal = nullptr;   // pinned, the rebuild's reads
    int *h_tok = nullptr;               // pinned, a greedy decode's tokens (h_tok_cap of them)
    int h_tok_cap = 0;
    // decode graph
    cudaGraphExec_t graph = nullptr;
    int graph_nk = -1;
    int graph_kernels = 0;
    size_t state_bytes = 0;
    bool stop_before_moe = false;   // qma_cuda_eval_hidden with n_layers < 0
    // the salience update of an attention layer runs on a side stream,
    // joined before the next attention layer (or the end of the step)
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    bool shared_stream = false;     // st / side belong to a batch
    static constexpr int HCM_REBUILD_INIT = 128;
};

namespace qma {

// ------------------------------------------------------------------ model --
static const qma_cuda_tensor *find_tensor(const qma_cuda_tensor *t, uint32_t n, const char *name) {
    for (uint32_t i = 0; i < n; i++)
        if (strncmp(t[i].name, name, sizeof(t[i].name)) == 0) return &t[i];
    return nullptr;
}

static size_t gguf_row_bytes(int type, int64_t n) {
    switch (type) {
    case QMA_TYPE_Q4_K: return size_t(n / 256) * Q4K_BYTES;
    case QMA_TYPE_Q6_K: return size_t(n / 256) * Q6K_BYTES;
    case QMA_TYPE_Q8_0: return size_t(n / 32) * Q80_BYTES;
    case QMA_TYPE_F32: return size_t(n) * 4;
    default: return 0;
    }
}

struct Loader {
    qma_cuda_model *m;
    const qma_cuda_tensor *t;
    uint32_t n;
    const uint8_t *host;
    uint64_t host_size;
    bool synth;
    uint64_t seed;
    cudaStream_t st;
    // dry: check names, shapes, types and data ranges only (host, no device
    // memory or stream touched; the pointers handed out are placeholders)
    bool dry = false;
    uint8_t *tmp = nullptr;
    size_t tmp_cap = 0;

    int dalloc(void **p, size_t bytes) {
        if (dry) {
            *p = reinterpret_cast<void *>(uintptr_t(256));
            return QMA_CUDA_OK;
        }
        QMA_CHECK_CUDA(cudaMalloc(p, bytes ? bytes : 16));
        m->allocs.push_back(*p);
        m->weight_bytes += bytes;
        return QMA_CUDA_OK;
    }
    // GGUF bytes of a tensor into device memory at dst (H2D or generated)
    int fetch(const qma_cuda_tensor *x, void *dst) {
        const uint64_t nel = uint64_t(x->ne[0]) * uint64_t(x->ne[1] ? x->ne[1] : 1) *
                             uint64_t(x->ne[2] ? x->ne[2] : 1);
        const size_t bytes = gguf_row_bytes(x->type, x->ne[0]) * (nel / uint64_t(x->ne[0]));
        if (synth) return dry ? QMA_CUDA_OK : synth_tensor_gguf(x->name, int(x->type), nel, seed, dst, st);
        if (x->off > host_size || bytes > host_size - x->off) {
            set_error("model_load: tensor %s out of the data section", x->name);
            return QMA_CUDA_ERR_INVALID;
        }
        if (dry) return QMA_CUDA_OK;
        QMA_CHECK_CUDA(cudaMemcpyAsync(dst, host + x->off, bytes, cudaMemcpyHostToDevice, st));
        return QMA_CUDA_OK;
    }
    // The tensor `name` with the shape the kernels are written for: every
    // device buffer is sized from ne[], so a shape the kernels do not expect
    // (another expert count, a short norm vector) is refused here instead of
    // letting a kernel read past an allocation.  ne[1] / ne[2] of 0 read as 1.
    const qma_cuda_tensor *need(const char *name, int *rc, int64_t e0, int64_t e1, int64_t e2 = 1) {
        const qma_cuda_tensor *x = find_tensor(t, n, name);
        if (!x) {
            set_error("model_load: missing tensor %s", name);
            *rc = QMA_CUDA_ERR_INVALID;
            return nullptr;
        }
        const int64_t n1 = x->ne[1] ? x->ne[1] : 1, n2 = x->ne[2] ? x->ne[2] : 1;
        if (x->ne[0] != e0 || n1 != e1 || n2 != e2) {
            set_error("model_load: %s has shape [%lld, %lld, %lld], expected [%lld, %lld, %lld]", name,
                      (long long)x->ne[0], (long long)n1, (long long)n2, (long long)e0, (long long)e1,
                      (long long)e2);
            *rc = QMA_CUDA_ERR_INVALID;
            return nullptr;
        }
        return x;
    }
    int ensure_tmp(size_t bytes) {
        if (dry || bytes <= tmp_cap) return QMA_CUDA_OK;
        if (tmp) {
            QMA_CHECK_CUDA(cudaStreamSynchronize(st));
            cudaFree(tmp);
        }
        QMA_CHECK_CUDA(cudaMalloc(&tmp, bytes));
        tmp_cap = bytes;
        return QMA_CUDA_OK;
    }
    // F32 vector / matrix, kept as is
    int f32(const char *name, const float **out, int64_t e0, int64_t e1 = 1) {
        int rc = 0;
        const qma_cuda_tensor *x = need(name, &rc, e0, e1);
        if (rc) return rc;
        if (x->type != QMA_TYPE_F32) {
            set_error("model_load: %s must be F32", name);
            return QMA_CUDA_ERR_UNSUPPORTED;
        }
        void *d;
        const size_t bytes = size_t(x->ne[0]) * (x->ne[1] ? x->ne[1] : 1) * 4;
        if ((rc = dalloc(&d, bytes))) return rc;
        if ((rc = fetch(x, d))) return rc;
        *out = static_cast<const float *>(d);
        return QMA_CUDA_OK;
    }
    // quantized matrices stacked along rows (all of one type), packed
    // names[i] must be [ncols, rows[i]]
    int stacked(const std::vector<std::string> &names, const std::vector<int64_t> &nrows, int64_t width,
                void **out, int *type, int *rows_out) {
        int rc = 0;
        std::vector<const qma_cuda_tensor *> xs;
        int64_t rows = 0, ncols = -1;
        int ty = -1;
        for (size_t i = 0; i < names.size(); i++) {
            const std::string &nm = names[i];
            const qma_cuda_tensor *x = need(nm.c_str(), &rc, width, nrows[i]);
            if (rc) return rc;
            if (ty < 0) { ty = int(x->type); ncols = x->ne[0]; }
            if (int(x->type) != ty || x->ne[0] != ncols) {
                set_error("model_load: %s differs in type/width from %s", nm.c_str(), names[0].c_str());
                return QMA_CUDA_ERR_UNSUPPORTED;
            }
            rows += x->ne[1];
            xs.push_back(x);
        }
        if (ty != QMA_TYPE_Q4_K && ty != QMA_TYPE_Q6_K && ty != QMA_TYPE_Q8_0) {
            set_error("model_load: %s must be Q4_K, Q6_K or Q8_0 (type %d)", names[0].c_str(), ty);
            return QMA_CUDA_ERR_UNSUPPORTED;
        }
        const size_t rb = gguf_row_bytes(ty, ncols);
        if ((rc = ensure_tmp(rb * size_t(rows)))) return rc;
        size_t o = 0;
        for (auto *x : xs) {
            if ((rc = fetch(x, tmp + o))) return rc;
            o += rb * size_t(x->ne[1]);
        }
        void *d;
        if ((rc = dalloc(&d, packed_bytes(ty, int(rows), int(ncols))))) return rc;
        if (!dry && (rc = repack(ty, tmp, int(rows), int(ncols), d, st))) return rc;
        *out = d;
        *type = ty;
        if (rows_out) *rows_out = int(rows);
        return QMA_CUDA_OK;
    }
    // 3-D expert tensor [ne2 experts][ne1 rows][ne0]: one packed matrix each
    int experts(const char *name, void **out, int *type, int64_t e0, int64_t e1) {
        int rc = 0;
        const qma_cuda_tensor *x = need(name, &rc, e0, e1, MOE_NEXP);
        if (rc) return rc;
        if (x->type != QMA_TYPE_Q4_K && x->type != QMA_TYPE_Q6_K) {
            set_error("model_load: %s must be Q4_K or Q6_K (type %u)", name, x->type);
            return QMA_CUDA_ERR_UNSUPPORTED;
        }
        const int rows = int(x->ne[1]), cols = int(x->ne[0]), ne = int(x->ne[2]);
        const size_t gb = gguf_row_bytes(int(x->type), cols) * rows;
        const size_t pb = packed_bytes(int(x->type), rows, cols);
        if ((rc = ensure_tmp(gb * ne))) return rc;
        if ((rc = fetch(x, tmp))) return rc;
        void *d;
        if ((rc = dalloc(&d, pb * ne))) return rc;
        for (int e = 0; e < ne && !dry; e++)
            if ((rc = repack(int(x->type), tmp + gb * e, rows, cols, static_cast<uint8_t *>(d) + pb * e, st)))
                return rc;
        *out = d;
        *type = int(x->type);
        return QMA_CUDA_OK;
    }
};

// dry: the host-only check of the table (names, shapes, types, data
// ranges) that runs before anything is allocated; *out is left untouched.
static int build_model(int device, const qma_cuda_tensor *t, uint32_t n, const void *host,
                       uint64_t host_size, bool synth, uint64_t seed, qma_cuda_model **out,
                       bool dry = false) {
    QMA_REQUIRE(t && n > 0 && (out || dry) && (synth || host || dry), "model: bad arguments");
    if (!dry) {
        int rc0 = build_model(device, t, n, host, host_size, synth || !host, seed, nullptr, true);
        if (rc0) return rc0;
        QMA_CHECK_CUDA(cudaSetDevice(device));
    }
    qma_cuda_model *m = new qma_cuda_model();
    m->device = device;
    cudaStream_t st = nullptr;
    if (!dry) QMA_CHECK_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    Loader ld{m, t, n, static_cast<const uint8_t *>(host), host_size, synth, seed, st};
    ld.dry = dry;
    int rc = 0;
    char nm[96];
    auto fail = [&](int code) {
        if (!dry) {
            cudaStreamSynchronize(st);
            if (ld.tmp) cudaFree(ld.tmp);
            cudaStreamDestroy(st);
            for (void *p : m->allocs) cudaFree(p);
        }
        delete m;
        return code;
    };
    const qma_cuda_tensor *te = find_tensor(t, n, "token_embd.weight");
    if (!te || te->ne[0] != EMBD || te->ne[1] < 1 || te->ne[1] > (int64_t(1) << 22) ||
        (te->ne[2] != 0 && te->ne[2] != 1)) {
        set_error("model: token_embd.weight missing or not [%d, 1..%d]", EMBD, 1 << 22);
        return fail(QMA_CUDA_ERR_INVALID);
    }
    m->n_vocab = int(te->ne[1]);
    const int64_t V = m->n_vocab;
    int rows;
    if ((rc = ld.stacked({"token_embd.weight"}, {V}, EMBD, &m->embd, &m->embd_type, &rows))) return fail(rc);
    if ((rc = ld.stacked({"output.weight"}, {V}, EMBD, &m->out, &m->out_type, &rows))) return fail(rc);
    if ((rc = ld.f32("output_norm.weight", &m->out_norm, EMBD))) return fail(rc);
    for (int il = 0; il < NLAYER; il++) {
        LayerW &L = m->L[il];
        auto N = [&](const char *s) { snprintf(nm, sizeof(nm), "blk.%d.%s", il, s); return std::string(nm); };
        if ((rc = ld.f32(N("attn_norm.weight").c_str(), &L.attn_norm, EMBD))) return fail(rc);
        if ((rc = ld.f32(N("post_attention_norm.weight").c_str(), &L.post_norm, EMBD))) return fail(rc);
        if (is_attn(il)) {
            if ((rc = ld.stacked({N("attn_q.weight"), N("attn_k.weight"), N("attn_v.weight")},
                                 {WQ_DIM, WKV_DIM, WKV_DIM}, EMBD, &L.in_proj, &L.in_type, &L.in_rows)))
                return fail(rc);
            if ((rc = ld.stacked({N("attn_output.weight")}, {EMBD}, WO_DIM, &L.out_proj, &L.out_type, &rows)))
                return fail(rc);
            if ((rc = ld.f32(N("attn_q_norm.weight").c_str(), &L.q_norm, HEAD_DIM))) return fail(rc);
            if ((rc = ld.f32(N("attn_k_norm.weight").c_str(), &L.k_norm, HEAD_DIM))) return fail(rc);
        } else {
            if ((rc = ld.stacked({N("attn_qkv.weight"), N("attn_gate.weight"), N("ssm_beta.weight"),
                                  N("ssm_alpha.weight")}, {CONV_DIM, VAL_DIM, VHEADS, VHEADS}, EMBD, &L.in_proj,
                                 &L.in_type, &L.in_rows))) return fail(rc);
            if ((rc = ld.stacked({N("ssm_out.weight")}, {EMBD}, VAL_DIM, &L.out_proj, &L.out_type, &rows)))
                return fail(rc);
            if ((rc = ld.f32(N("ssm_conv1d.weight").c_str(), &L.conv1d, 4, CONV_DIM))) return fail(rc);
            if ((rc = ld.f32(N("ssm_dt.bias").c_str(), &L.dt, VHEADS))) return fail(rc);
            if ((rc = ld.f32(N("ssm_a").c_str(), &L.a, VHEADS))) return fail(rc);
            if ((rc = ld.f32(N("ssm_norm.weight").c_str(), &L.ssm_norm, SSTATE))) return fail(rc);
        }
        qma_cuda_moe_weights &w = L.moe;
        w.post_norm = L.post_norm;
        if ((rc = ld.f32(N("ffn_gate_inp.weight").c_str(), &w.gate_inp, EMBD, MOE_NEXP))) return fail(rc);
        if ((rc = ld.f32(N("ffn_gate_inp_shexp.weight").c_str(), &w.gate_inp_shexp, EMBD))) return fail(rc);
        int ty;
        void *p;
        if ((rc = ld.experts(N("ffn_gate_exps.weight").c_str(), &p, &ty, EMBD, MOE_FF))) return fail(rc);
        w.gate_exps = p;
        if (ty != QMA_TYPE_Q4_K) { set_error("model: expert gate/up must be Q4_K"); return fail(QMA_CUDA_ERR_UNSUPPORTED); }
        if ((rc = ld.experts(N("ffn_up_exps.weight").c_str(), &p, &ty, EMBD, MOE_FF))) return fail(rc);
        w.up_exps = p;
        if (ty != QMA_TYPE_Q4_K) { set_error("model: expert gate/up must be Q4_K"); return fail(QMA_CUDA_ERR_UNSUPPORTED); }
        if ((rc = ld.experts(N("ffn_down_exps.weight").c_str(), &p, &w.down_type, MOE_FF, EMBD))) return fail(rc);
        w.down_exps = p;
        if ((rc = ld.stacked({N("ffn_gate_shexp.weight")}, {MOE_FF}, EMBD, &p, &ty, &rows))) return fail(rc);
        w.gate_shexp = p;
        if (ty != QMA_TYPE_Q4_K) { set_error("model: shared expert gate/up must be Q4_K"); return fail(QMA_CUDA_ERR_UNSUPPORTED); }
        if ((rc = ld.stacked({N("ffn_up_shexp.weight")}, {MOE_FF}, EMBD, &p, &ty, &rows))) return fail(rc);
        w.up_shexp = p;
        if (ty != QMA_TYPE_Q4_K) { set_error("model: shared expert gate/up must be Q4_K"); return fail(QMA_CUDA_ERR_UNSUPPORTED); }
        if ((rc = ld.stacked({N("ffn_down_shexp.weight")}, {EMBD}, MOE_FF, &p, &w.down_shexp_type, &rows)))
            return fail(rc);
        w.down_shexp = p;
        if ((w.down_type != QMA_TYPE_Q6_K && w.down_type != QMA_TYPE_Q4_K) || w.down_shexp_type != w.down_type) {
            set_error("model: expert down projections must be Q6_K or Q4_K, routed and shared alike");
            return fail(QMA_CUDA_ERR_UNSUPPORTED);
        }
    }
    if (dry) {
        delete m;
        return QMA_CUDA_OK;
    }
    QMA_CHECK_CUDA(cudaStreamSynchronize(st));
    if (ld.tmp) cudaFree(ld.tmp);
    cudaStreamDestroy(st);
    *out = m;
    return QMA_CUDA_OK;
}

// ------------------------------------------------------------------ state --
static int salloc(qma_cuda_state *s, void **p, size_t bytes, cudaStream_t st) {
    QMA_CHECK_CUDA(cudaMalloc(p, bytes ? bytes : 16));
    s->allocs.push_back(*p);
    s->state_bytes += bytes;
    QMA_CHECK_CUDA(cudaMemsetAsync(*p, 0, bytes ? bytes : 16, st));
    return QMA_CUDA_OK;
}

template <class T>
static int salloc_t(qma_cuda_state *s, T **p, size_t count, cudaStream_t st) {
    void *v;
    const int rc = salloc(s, &v, sizeof(T) * count, st);
    *p = static_cast<T *>(v);
    return rc;
}

// Attention scratch that grows with the attended context: stream-ordered
// allocations on the state's stream (no device synchronisation, no host
// wait: a prefill grows these buffers at almost every chunk, and a
// synchronous cudaFree / cudaMalloc pair there stalled chunks by up to a
// second), at least 1.5x the old size so that growth is rare; the device's
// default pool keeps freed blocks for reuse.
static int grow(float **p, size_t *cap, cudaStream_t st, size_t need) {
    if (need <= *cap) return QMA_CUDA_OK;
    static PerDevice pool_set;
    if (!pool_set.done()) {
        int dev = 0;
        cudaMemPool_t pool;
        QMA_CHECK_CUDA(cudaGetDevice(&dev));
        QMA_CHECK_CUDA(cudaDeviceGetDefaultMemPool(&pool, dev));
        uint64_t keep = UINT64_MAX;
        QMA_CHECK_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
        pool_set.mark();
    }
    const size_t n = std::max(need, *cap + *cap / 2);
    if (*p) QMA_CHECK_CUDA(cudaFreeAsync(*p, st));
    *p = nullptr;
    QMA_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void **>(p), n * sizeof(float), st));
    *cap = n;
    return QMA_CUDA_OK;
}

// shared: a stream the state runs on (its salience updates included)
// instead of streams of its own, for the sequences of a batch.
static int create_state(qma_cuda_model *m, int n_ctx, qma_cuda_state **out, cudaStream_t shared = nullptr) {
    QMA_REQUIRE(m && out && n_ctx > HCM_SINK + 1, "state: bad arguments (n_ctx %d)", n_ctx);
    QMA_CHECK_CUDA(cudaSetDevice(m->device));
    qma_cuda_state *s = new qma_cuda_state();
    s->m = m;
    s->n_ctx = n_ctx;
    if (shared) {
        s->st = s->side = shared;
        s->shared_stream = true;
    } else {
        QMA_CHECK_CUDA(cudaStreamCreateWithFlags(&s->st, cudaStreamNonBlocking));
        QMA_CHECK_CUDA(cudaStreamCreateWithFlags(&s->side, cudaStreamNonBlocking));
    }
    QMA_CHECK_CUDA(cudaEventCreateWithFlags(&s->ev_fork, cudaEventDisableTiming));
    QMA_CHECK_CUDA(cudaEventCreateWithFlags(&s->ev_join, cudaEventDisableTiming));
    cudaStream_t st = s->st;
    int rc = 0;
#define TRY(x) do { if ((rc = (x))) return rc; } while (0)
    for (int il = 0; il < NLAYER; il++) {
        if (is_attn(il)) {
            TRY(salloc_t(s, &s->kv[il / 4], size_t(2) * NHEAD_KV * n_ctx * KVQ_SLOT, st));
            TRY(salloc_t(s, &s->arena[il / 4], size_t(2) * NHEAD_KV * HCM_H_PIN * KVQ_SLOT, st));
        } else {
            TRY(salloc_t(s, &s->conv[il], size_t(CONV_DIM) * 3, st));
            TRY(salloc_t(s, &s->ssm[il], size_t(VHEADS) * SSTATE * SSTATE, st));
        }
    }
    TRY(salloc_t(s, &s->kv_dev, NATTN, st));
    TRY(salloc_t(s, &s->arena_dev, NATTN, st));
    QMA_CHECK_CUDA(cudaMemcpyAsync(s->kv_dev, s->kv, sizeof(s->kv), cudaMemcpyHostToDevice, st));
    QMA_CHECK_CUDA(cudaMemcpyAsync(s->arena_dev, s->arena, sizeof(s->arena), cudaMemcpyHostToDevice, st));
    TRY(salloc_t(s, &s->sal, size_t(NATTN) * n_ctx, st));
    TRY(salloc_t(s, &s->pin_sal, size_t(NATTN) * HCM_H_PIN, st));
    TRY(salloc_t(s, &s->qf, size_t(n_ctx), st));
    TRY(salloc_t(s, &s->live_dev, size_t(n_ctx), st));
    TRY(salloc_t(s, &s->pairs_dev, size_t(HCM_H_PIN), st));
    // IMROPE table (rope_imrope, nn.c:841-861), computed with the host libm
    // exactly as the reference does: theta_0 = p, theta_{j+1} = theta_j * s
    {
        std::vector<float> tab(size_t(n_ctx) * NROT);
        const float theta_scale = powf(10000000.0f, -2.0f / NROT);
        for (int p = 0; p < n_ctx; p++) {
            float theta = float(p);
            for (int j = 0; j < NROT / 2; j++) {
                tab[size_t(p) * NROT + j] = cosf(theta);
                tab[size_t(p) * NROT + NROT / 2 + j] = sinf(theta);
                theta *= theta_scale;
            }
        }
        TRY(salloc_t(s, &s->rope, tab.size(), st));
        QMA_CHECK_CUDA(cudaMemcpyAsync(s->rope, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, st));
        QMA_CHECK_CUDA(cudaStreamSynchronize(st));
    }
    TRY(salloc_t(s, &s->sp_dev, 1, st));
    QMA_CHECK_CUDA(cudaMallocHost(&s->sp_host, sizeof(StepParams)));
    const int TM = MAX_CHUNK;
    TRY(salloc_t(s, &s->tokens_dev, TM, st));
    TRY(salloc_t(s, &s->x, size_t(TM) * EMBD, st));
    TRY(salloc_t(s, &s->x2, size_t(TM) * EMBD, st));
    TRY(salloc_t(s, &s->proj, size_t(TM) * (CONV_DIM + VAL_DIM + 2 * VHEADS), st));
    TRY(salloc_t(s, &s->conv_out, size_t(TM) * CONV_DIM, st));
    TRY(salloc_t(s, &s->gdo, size_t(TM) * VAL_DIM, st));
    TRY(salloc_t(s, &s->qr, size_t(TM) * NHEAD * HEAD_DIM, st));
    TRY(salloc_t(s, &s->z, size_t(TM) * WO_DIM, st));
    TRY(salloc_t(s, &s->xq, size_t(TM) * VAL_DIM, st));
    TRY(salloc_t(s, &s->xd, size_t(TM) * VAL_DIM / 256, st));
    TRY(salloc_t(s, &s->xs, size_t(TM) * VAL_DIM / 16, st));
    s->moe_scratch_bytes = moe_scratch_bytes(TM);
    TRY(salloc(s, &s->moe_scratch, s->moe_scratch_bytes, st));
    TRY(salloc_t(s, &s->ml, size_t(TM) * NHEAD * 2, st));
    TRY(salloc_t(s, &s->argmax_dev, 4, st));
    TRY(salloc_t(s, &s->argmax_pv, ARG_CTAS, st));
    TRY(salloc_t(s, &s->argmax_pi, ARG_CTAS, st));
    TRY(salloc_t(s, &s->argmax_cnt, 1, st));
    TRY(salloc_t(s, &s->gdn_cnt, VHEADS / 2, st));
    TRY(salloc_t(s, &s->gdn_kq, size_t(MAX_CHUNK) * KHEADS, st));
    TRY(salloc_t(s, &s->gdn_chunk, gdn_chunk_scratch_bytes() / sizeof(float), st));
    s->logits_rows = 1;
    TRY(salloc_t(s, &s->logits, size_t(m->n_vocab), st));
#undef TRY
    s->live.assign(n_ctx, 0);
    s->tier.assign(n_ctx, 0);
    s->pin_pos.assign(HCM_H_PIN, -1);
    s->next_rebuild = qma_cuda_state::HCM_REBUILD_INIT;
    QMA_CHECK_CUDA(cudaStreamSynchronize(st));
    *out = s;
    return QMA_CUDA_OK;
}

// ------------------------------------------------------------ HCM rebuild --
// hcm_rebuild (nn.c:981-1150), host side, in the reference's exact order:
// the live index is [sink + hot ring q4 | arena q4 | gist ring q2]; the
// heavy-hitter heap keeps the top HCM_H_PIN of (ring middle positions scored
// sum_l sal * (1 - 2 qf), existing arena occupants scored sum_l pin_sal);
// fresh winners are copied ring -> arena on the device.
struct HEnt { float sc; int pos; int is_arena; };

static void heap_push(std::vector<HEnt> &heap, int &hn, float sc, int pos, int is_a) {
    if (hn < HCM_H_PIN) {
        int i = hn++;
        heap[i] = {sc, pos, is_a};
        while (i > 0) {
            const int par = (i - 1) / 2;
            if (heap[par].sc <= heap[i].sc) break;
            std::swap(heap[par], heap[i]);
            i = par;
        }
    } else if (sc > heap[0].sc) {
        heap[0] = {sc, pos, is_a};
        int i = 0;
        for (;;) {
            const int lc = 2 * i + 1, rc = 2 * i + 2;
            int sm = i;
            if (lc < hn && heap[lc].sc < heap[sm].sc) sm = lc;
            if (rc < hn && heap[rc].sc < heap[sm].sc) sm = rc;
            if (sm == i) break;
            std::swap(heap[sm], heap[i]);
            i = sm;
        }
    }
}

static int hcm_rebuild(qma_cuda_state *s, int n_pos) {
    const int cap = s->n_ctx, ring = cap - HCM_SINK, oldest = n_pos - ring;
    cudaStream_t st = s->st;
    if (n_pos <= HCM_SINK + HCM_W_HOT) {
        for (int p = 0; p < n_pos; p++) {
            s->live[p] = hcm_slot(p, cap);
            s->tier[hcm_slot(p, cap)] = 2;
        }
        s->live_n = s->n4 = s->n_ring_q4 = n_pos;
    } else {
        if (!s->h_sal) {
            QMA_CHECK_CUDA(cudaMallocHost(&s->h_sal, sizeof(float) * NATTN * size_t(cap)));
            QMA_CHECK_CUDA(cudaMallocHost(&s->h_qf, sizeof(float) * size_t(cap)));
            QMA_CHECK_CUDA(cudaMallocHost(&s->h_pin_sal, sizeof(float) * NATTN * size_t(HCM_H_PIN)));
        }
        QMA_CHECK_CUDA(cudaMemcpyAsync(s->h_sal, s->sal, sizeof(float) * NATTN * size_t(cap), cudaMemcpyDeviceToHost,
                                       st));
        QMA_CHECK_CUDA(cudaMemcpyAsync(s->h_qf, s->qf, sizeof(float) * size_t(cap), cudaMemcpyDeviceToHost, st));
        QMA_CHECK_CUDA(cudaMemcpyAsync(s->h_pin_sal, s->pin_sal, sizeof(float) * NATTN * size_t(HCM_H_PIN),
                                       cudaMemcpyDeviceToHost, st));
        QMA_CHECK_CUDA(cudaStreamSynchronize(st));
        int n = 0;
        int hot_lo = n_pos - HCM_W_HOT;
        if (hot_lo < oldest) hot_lo = oldest;
        for (int p = 0; p < HCM_SINK && p < hot_lo; p++) {
            s->live[n++] = hcm_slot(p, cap);
            s->tier[hcm_slot(p, cap)] = 2;
        }
        for (int p = hot_lo; p < n_pos; p++) {
            s->live[n++] = hcm_slot(p, cap);
            s->tier[hcm_slot(p, cap)] = 2;
        }
        int cand_lo = HCM_SINK;
        if (oldest > cand_lo) cand_lo = oldest;
        std::vector<HEnt> heap(HCM_H_PIN);
        int hn = 0;
        for (int p = cand_lo; p < hot_lo; p++) {
            const int sl = hcm_slot(p, cap);
            float sc = 0.0f;
            for (int l = 0; l < NATTN; l++) sc += s->h_sal[size_t(l) * cap + sl];
            const float qf = s->h_qf[sl] > 0 ? s->h_qf[sl] : 0.05f;
            sc = sc * (1.0f - HCM_QF_BIAS * qf);
            heap_push(heap, hn, sc, p, 0);
        }
        for (int a = 0; a < HCM_H_PIN; a++) {
            if (s->pin_pos[a] < 0) continue;
            float sc = 0.0f;
            for (int l = 0; l < NATTN; l++) sc += s->h_pin_sal[size_t(l) * HCM_H_PIN + a];
            heap_push(heap, hn, sc, a, 1);
        }
        // Each winner not yet in the arena takes the first free slot, else
        // evicts the lowest-scoring occupied slot that no winner keeps
        // (lowest index on equal scores), as the reference's scans do
        // (nn.c:1092-1127).  Without rescanning every slot per winner: a
        // slot's score changes only when a winner takes it, and then it is
        // kept, so one list of the occupied, unkept slots sorted by (score,
        // index) serves every eviction; free slots only fill, so the first
        // free one is found by a forward pointer.
        std::vector<int> new_arena(HCM_H_PIN, -1);
        std::vector<uint8_t> kept(HCM_H_PIN, 0);
        for (int i = 0; i < hn; i++) {
            new_arena[i] = heap[i].is_arena ? heap[i].pos : -1;
            if (new_arena[i] >= 0) kept[new_arena[i]] = 1;
        }
        std::vector<std::pair<float, int>> evict;
        for (int a = 0; a < HCM_H_PIN; a++) {
            if (s->pin_pos[a] < 0 || kept[a]) continue;
            float sc = 0.0f;
            for (int l = 0; l < NATTN; l++) sc += s->h_pin_sal[size_t(l) * HCM_H_PIN + a];
            if (sc < 1e30f) evict.push_back(std::make_pair(sc, a));   // the scans' bound (never NaN)
        }
        std::sort(evict.begin(), evict.end());
        size_t ev = 0;
        int next_free = 0;
        std::vector<int2> pairs;
        for (int i = 0; i < hn; i++) {
            if (heap[i].is_arena) continue;
            const int src = hcm_slot(heap[i].pos, cap);
            int slot = -1;
            while (next_free < HCM_H_PIN && s->pin_pos[next_free] >= 0) next_free++;
            if (next_free < HCM_H_PIN) {
                slot = next_free;
            } else {
                while (ev < evict.size() && kept[evict[ev].second]) ev++;
                if (ev < evict.size()) slot = evict[ev].second;
            }
            if (slot < 0) continue;
            new_arena[i] = slot;
            kept[slot] = 1;
            pairs.push_back(make_int2(src, slot));
            for (int l = 0; l < NATTN; l++)
                s->h_pin_sal[size_t(l) * HCM_H_PIN + slot] = s->h_sal[size_t(l) * cap + src];
            s->pin_pos[slot] = heap[i].pos;
        }
        const int n_ring_q4 = n;
        for (int i = 0; i < hn; i++)
            if (new_arena[i] >= 0) s->live[n++] = HCM_ARENA_BASE + new_arena[i];
        int gist_lo = hot_lo - HCM_W_GIST;
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
        if (!pairs.empty()) {
            QMA_CHECK_CUDA(cudaMemcpyAsync(s->pairs_dev, pairs.data(), pairs.size() * sizeof(int2),
                                           cudaMemcpyHostToDevice, st));
            int rc = launch_arena_copy(s->pairs_dev, int(pairs.size()), s->kv_dev, s->arena_dev, s->sal,
                                       s->pin_sal, cap, st);
            if (rc) return rc;
            QMA_CHECK_CUDA(cudaStreamSynchronize(st));
        }
    }
    if (s->live_n > 0)
        QMA_CHECK_CUDA(cudaMemcpyAsync(s->live_dev, s->live.data(), size_t(s->live_n) * 4,
                                       cudaMemcpyHostToDevice, st));
    QMA_CHECK_CUDA(cudaStreamSynchronize(st));
    return QMA_CUDA_OK;
}

// ---------------------------------------------------------------- forward --
static int nk_upper(const qma_cuda_state *s, int pos_now, int T, bool graph) {
    if (graph) {
        // a decode graph serves positions [pos_now, next_rebuild)
        const int last = s->next_rebuild - 1;
        return s->live_n > 0 ? s->live_n + (last - s->rebuilt_at + 1) : last + 1;
    }
    return s->live_n > 0 ? s->live_n + (pos_now + T - 1 - s->rebuilt_at + 1) : pos_now + T;
}

static int ensure_attn_scratch(qma_cuda_state *s, int T, int nk, int pv_chunk) {
    // cmax holds the per-chunk maxima of the chunked attention
    const size_t npv = size_t((nk + pv_chunk - 1) / pv_chunk), nsc = npv;
    const bool moves = size_t(T) * NHEAD * nk > s->scores_cap || size_t(T) * NHEAD * nsc > s->cmax_cap ||
                       size_t(T) * NHEAD * npv * HEAD_DIM > s->opart_cap ||
                       size_t(T) * NHEAD * npv > s->lpart_cap;
    if (moves && s->graph) {
        // a captured decode graph holds the old buffers
        QMA_CHECK_CUDA(cudaStreamSynchronize(s->st));
        cudaGraphExecDestroy(s->graph);
        s->graph = nullptr;
    }
    int rc;
    if ((rc = grow(&s->scores, &s->scores_cap, s->st, size_t(T) * NHEAD * nk))) return rc;
    if ((rc = grow(&s->cmax, &s->cmax_cap, s->st, size_t(T) * NHEAD * nsc))) return rc;
    if ((rc = grow(&s->opart, &s->opart_cap, s->st, size_t(T) * NHEAD * npv * HEAD_DIM))) return rc;
    if ((rc = grow(&s->lpart, &s->lpart_cap, s->st, size_t(T) * NHEAD * npv))) return rc;
    return QMA_CUDA_OK;
}

// Greedy token of the last logits row: ARG_CTAS CTAs each reduce a slice to
// (max, first index); the last CTA to finish (atomic ticket, reset for the
// next step) reduces the slices.  Ties keep the lowest index.

__device__ __forceinline__ void argmax_merge(float &v, int &idx, float ov, int oi) {
    if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
}

__global__ void __launch_bounds__(512) argmax_kernel(const float *__restrict__ logits, int n,
                                                     StepParams *sp, int *out, float *pv, int *pi,
                                                     unsigned *cnt) {
    QMA_TRACE_SCOPE(TK_ARGMAX);
    __shared__ float bv[16];
    __shared__ int bi[16];
    __shared__ int last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_trigger();
    pdl_wait();
    const int per = (n + gridDim.x - 1) / gridDim.x;
    const int i0 = blockIdx.x * per, i1 = min(n, i0 + per);
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = i0 + tid; i < i1; i += blockDim.x) {
        const float x = logits[i];
        if (x > v) { v = x; idx = i; }     // ascending i: keeps the first maximum
    }
    for (int o = 16; o > 0; o >>= 1)
        argmax_merge(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
    if (lane == 0) { bv[warp] = v; bi[warp] = idx; }
    __syncthreads();
    if (warp == 0) {
        v = lane < 16 ? bv[lane] : -INFINITY;
        idx = lane < 16 ? bi[lane] : 0x7fffffff;
        for (int o = 16; o > 0; o >>= 1)
            argmax_merge(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
        if (lane == 0) {
            pv[blockIdx.x] = v;
            pi[blockIdx.x] = idx;
            __threadfence();
            last = atomicAdd(cnt, 1u) == gridDim.x - 1;
        }
    }
    __syncthreads();
    if (!last || warp != 0) return;
    __threadfence();
    v = -INFINITY;
    idx = 0x7fffffff;
    for (int c = lane; c < int(gridDim.x); c += 32) argmax_merge(v, idx, __ldcg(pv + c), __ldcg(pi + c));
    for (int o = 16; o > 0; o >>= 1)
        argmax_merge(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
    if (lane == 0) {
        *out = idx;
        *cnt = 0;
        if (sp) {            // next decode step: this token at the next position
            sp->token = idx;
            sp->n_pos += 1;
        }
    }
}

// The mixer half of layer il (gated delta net or gated attention) on the
// T tokens whose normed Q8_K input is in s->xq / xd / xs and residual in
// s->x; writes the residual after it to s->x2 (nn.c:2107-2246).
// side_pending: a salience update of an earlier attention layer is still
// running on s->side (joined here before the next one starts).
static int mixer(qma_cuda_state *s, int il, int T, int nk_cap, int pv_chunk, bool &side_pending) {
    qma_cuda_model *m = s->m;
    cudaStream_t st = s->st;
    const LayerW &L = m->L[il];
    int rc;
#define TRY(x) do { if ((rc = (x))) return rc; } while (0)
    // a single token's gated-delta-net conv runs in the input projection's epilogue
    ConvEpi ce;
    const bool conv_fused = !is_attn(il) && T == 1 && pdl_enabled();
    if (conv_fused) {
        ce.w = L.conv1d;
        ce.state = s->conv[il];
        ce.out = s->conv_out;
        ce.n = CONV_DIM;
    }
    TRY(matvec(L.in_type, L.in_proj, EMBD, L.in_rows, T, s->xq, s->xd, s->xs, s->proj, st, nullptr,
               conv_fused ? &ce : nullptr));
    if (is_attn(il)) {
        const int lay = il / 4;
        if (side_pending) {
            // the previous layer's salience reads `scores` and writes
            // the slot this append resets
            QMA_CHECK_CUDA(cudaStreamWaitEvent(st, s->ev_join, 0));
            side_pending = false;
        }
        TRY(launch_qk_prep_append(s->proj, L.in_rows, L.q_norm, L.k_norm, s->rope, s->sp_dev, T,
                                  s->qr, s->z, s->kv[lay], s->qf, s->sal, st));
        AttnArgs a;
        a.qr = s->qr; a.kv = s->kv[lay]; a.arena = s->arena[lay]; a.live = s->live_dev;
        a.sp = s->sp_dev; a.T = T; a.nk_max = nk_cap; a.pv_chunk = pv_chunk;
        a.scores = s->scores; a.cmax = s->cmax; a.opart = s->opart; a.lpart = s->lpart;
        a.ml = s->ml; a.z = s->z; a.xq = s->xq; a.xd = s->xd; a.xs = s->xs;
        a.sal = s->sal + size_t(lay) * s->n_ctx;
        a.pin_sal = s->pin_sal + size_t(lay) * HCM_H_PIN;
        TRY(launch_attention(a, st));
        QMA_CHECK_CUDA(cudaEventRecord(s->ev_fork, st));
        QMA_CHECK_CUDA(cudaStreamWaitEvent(s->side, s->ev_fork, 0));
        TRY(launch_salience(a, s->side));
        QMA_CHECK_CUDA(cudaEventRecord(s->ev_join, s->side));
        side_pending = true;
        TRY(matvec(L.out_type, L.out_proj, WO_DIM, EMBD, T, s->xq, s->xd, s->xs, s->x2, st, s->x));
    } else {
        const int ld = L.in_rows;     // qkv 8192 | gate 4096 | beta 32 | alpha 32
        if (!conv_fused) TRY(launch_conv1d(s->proj, ld, L.conv1d, s->conv[il], T, s->conv_out, st));
        if (T == 1) {
            // one token: the gated norm + Q8_K run in the recurrence kernel's tail
            const GdnNormArgs gna = {s->proj + CONV_DIM, L.ssm_norm, s->xq, s->xd, s->xs, s->gdn_cnt};
            TRY(launch_gdn(s->conv_out, s->proj, ld, CONV_DIM + VAL_DIM, CONV_DIM + VAL_DIM + VHEADS,
                           L.dt, L.a, s->ssm[il], T, s->gdo, st, &gna));
        } else {
            TRY(launch_gdn(s->conv_out, s->proj, ld, CONV_DIM + VAL_DIM, CONV_DIM + VAL_DIM + VHEADS,
                           L.dt, L.a, s->ssm[il], T, s->gdo, st, nullptr, s->gdn_kq, s->gdn_chunk));
            TRY(launch_gated_norm_quant(s->gdo, s->proj + CONV_DIM, ld, L.ssm_norm, T, s->xq, s->xd,
                                        s->xs, st));
        }
        TRY(matvec(L.out_type, L.out_proj, VAL_DIM, EMBD, T, s->xq, s->xd, s->xs, s->x2, st, s->x));
    }
#undef TRY
    return QMA_CUDA_OK;
}

// A layer's output projection, router and shared expert go into L2 while
// its input projection and mixer run.
static Prefetch layer_plan(const qma_cuda_model *m, int il) {
    const LayerW &L = m->L[il];
    Prefetch pf;
    pf.p[0] = L.out_proj;
    pf.bytes[0] = packed_bytes(L.out_type, EMBD, is_attn(il) ? WO_DIM : VAL_DIM);
    pf.p[1] = L.moe.gate_inp;
    pf.bytes[1] = sizeof(float) * size_t(EMBD) * 256;
    pf.p[2] = L.moe.gate_shexp;
    pf.bytes[2] = packed_bytes(QMA_TYPE_Q4_K, 512, EMBD);
    pf.p[3] = L.moe.up_shexp;
    pf.bytes[3] = packed_bytes(QMA_TYPE_Q4_K, 512, EMBD);
    pf.p[4] = L.moe.down_shexp;
    pf.bytes[4] = packed_bytes(L.moe.down_shexp_type, EMBD, 512);
    return pf;
}

// The forward of T tokens at the positions in *sp_dev (host copy hs):
// embedding -> 40 layers -> (optionally) final norm + LM head.
static int forward(qma_cuda_state *s, const StepParams &hs, const int *tokens_dev, int nk_cap,
                   int logits_mode /*0 none, 1 last, 2 all*/, int n_layers = NLAYER) {
    qma_cuda_model *m = s->m;
    cudaStream_t st = s->st;
    const int T = hs.T;
    int rc;
#define TRY(x) do { if ((rc = (x))) return rc; } while (0)
    TRY(launch_embed(m->embd, m->embd_type, m->n_vocab, tokens_dev, s->sp_dev, T, s->x, st));
    const int pv_chunk = attn_span(T, nk_cap);
    bool side_pending = false;     // a salience update is running on s->side
    auto plan = [&](int il) { return layer_plan(m, il); };
    bool normed = false;           // s->xq already holds the next norm's output
    for (int il = 0; il < n_layers; il++) {
        const LayerW &L = m->L[il];
        if (!normed) TRY(launch_rmsnorm_quant(s->x, L.attn_norm, T, EMBD, s->xq, s->xd, s->xs, st, plan(il)));
        normed = false;
        TRY(mixer(s, il, T, nk_cap, pv_chunk, side_pending));
        if (il == n_layers - 1 && s->stop_before_moe) {
            // parity aid: return the residual after the mixer of this layer
            QMA_CHECK_CUDA(cudaMemcpyAsync(s->x, s->x2, sizeof(float) * size_t(T) * EMBD,
                                           cudaMemcpyDeviceToDevice, st));
            break;
        }
        // x = x2 + moe(rms_norm(x2) * post_norm); the block's last kernel also
        // forms the next RMSNorm's Q8_K input (the next layer's, or the
        // output norm's for the rows the LM head reads)
        MoeNormTail tail;
        tail.xq = s->xq;
        tail.xd = s->xd;
        tail.xs = s->xs;
        if (il + 1 < n_layers) {
            tail.w = m->L[il + 1].attn_norm;
            tail.pf = plan(il + 1);
        } else if (logits_mode) {
            tail.w = m->out_norm;
            tail.norm_from = logits_mode == 2 ? 0 : T - 1;
        }
        TRY(moe_layer(L.moe, s->x2, T, s->x, nullptr, nullptr, s->moe_scratch, st, false, &tail));
        normed = tail.w != nullptr;
    }
    if (side_pending) QMA_CHECK_CUDA(cudaStreamWaitEvent(st, s->ev_join, 0));
    if (logits_mode) {
        const int rows = logits_mode == 2 ? T : 1;
        const float *xin = logits_mode == 2 ? s->x : s->x + size_t(T - 1) * EMBD;
        if (!normed) TRY(launch_rmsnorm_quant(xin, m->out_norm, rows, EMBD, s->xq, s->xd, s->xs, st));
        TRY(matvec(m->out_type, m->out, EMBD, m->n_vocab, rows, s->xq, s->xd, s->xs, s->logits, st));
    }
#undef TRY
    return QMA_CUDA_OK;
}

// A bounded wait inside a kernel that gave up (a copy that never landed)
// fails the call instead of returning silently wrong results.
static int check_wait_timeouts() {
    const int a = moe_wait_timeouts(), b = gemv_wait_timeouts(), c = tc_wait_timeouts(),
              d = gemm_tc_wait_timeouts();
    const int n = a < 0 || b < 0 || c < 0 || d < 0 ? -1 : a + b + c + d;
    if (n == 0) return QMA_CUDA_OK;
    set_error("%d bounded waits for weight copies ran out (or the counter could not be read)", n);
    return QMA_CUDA_ERR_TIMEOUT;
}

static void fill_params(qma_cuda_state *s, StepParams &p, int pos_now, int T, int token) {
    p.n_pos = pos_now;
    p.T = T;
    p.n_live = s->live_n;
    p.n_ring_q4 = s->n_ring_q4;
    p.n4 = s->n4;
    p.rebuilt_at = s->rebuilt_at;
    p.n_ctx = s->n_ctx;
    p.token = token;
}

static int maybe_rebuild(qma_cuda_state *s, int pos_now) {
    if (pos_now >= s->next_rebuild) {
        const int rc = hcm_rebuild(s, pos_now);
        if (rc) return rc;
        s->rebuilt_at = pos_now;
        s->next_rebuild = pos_now + HCM_REBUILD;
        if (s->graph) {
            cudaGraphExecDestroy(s->graph);
            s->graph = nullptr;
        }
    }
    return QMA_CUDA_OK;
}

static int capture_decode(qma_cuda_state *s);

// One token with its logits to the host: a replay of the captured decode
// step (the same kernels eager launches would run, without ~300 host-side
// launches per token).  The step's argmax also runs; eval ignores it.
static int eval_one_graph(qma_cuda_state *s, int token, float *logits) {
    cudaStream_t st = s->st;
    int rc;
    const int pos = s->n_pos;
    QMA_CHECK_CUDA(cudaStreamSynchronize(st));
    if ((rc = maybe_rebuild(s, pos))) return rc;
    fill_params(s, *s->sp_host, pos, 1, token);
    QMA_CHECK_CUDA(cudaMemcpyAsync(s->sp_dev, s->sp_host, sizeof(StepParams), cudaMemcpyHostToDevice, st));
    if (!s->graph && (rc = capture_decode(s))) return rc;
    s->tier[hcm_slot(pos, s->n_ctx)] = 2;
    QMA_CHECK_CUDA(cudaGraphLaunch(s->graph, st));
    if (logits)
        QMA_CHECK_CUDA(cudaMemcpyAsync(logits, s->logits, sizeof(float) * s->m->n_vocab, cudaMemcpyDeviceToHost,
                                       st));
    QMA_CHECK_CUDA(cudaStreamSynchronize(st));
    s->n_pos += 1;
    return check_wait_timeouts();
}

// QMA_CUDA_EAGER=1 in the environment: qma_cuda_eval launches every kernel
// itself, also for single tokens (no graph replay), for debugging.
static bool eager_only() {
    const char *v = getenv("QMA_CUDA_EAGER");
    return v && atoi(v) != 0;
}

static int eval(qma_cuda_state *s, const int *tokens, int n_tokens, float *logits, int logits_all,
                int n_layers = NLAYER, float *hidden = nullptr) {
    qma_cuda_model *m = s->m;
    cudaStream_t st = s->st;
    QMA_CHECK_CUDA(cudaSetDevice(m->device));
    if (s->n_pos + n_tokens > s->n_ctx - HCM_SINK) {
        set_error("eval: %d + %d positions exceed this state's ring of %d (no wrap-around)", s->n_pos,
                  n_tokens, s->n_ctx);
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
    if (n_tokens == 1 && !logits_all && n_layers == NLAYER && !hidden && pdl_enabled() && !eager_only())
        return eval_one_graph(s, tokens[0], logits);
    if (logits_all && MAX_CHUNK > s->logits_rows) {
        void *p;
        QMA_CHECK_CUDA(cudaMalloc(&p, sizeof(float) * size_t(MAX_CHUNK) * m->n_vocab));
        s->allocs.push_back(p);
        s->logits = static_cast<float *>(p);
        s->logits_rows = MAX_CHUNK;
        if (s->graph) {
            // a captured decode step writes the old logits buffer
            QMA_CHECK_CUDA(cudaStreamSynchronize(st));
            cudaGraphExecDestroy(s->graph);
            s->graph = nullptr;
        }
    }
    int done = 0, rc;
    while (done < n_tokens) {
        const int T = n_tokens - done < MAX_CHUNK ? n_tokens - done : MAX_CHUNK;
        const int pos_now = s->n_pos + done;
        QMA_CHECK_CUDA(cudaMemcpyAsync(s->tokens_dev, tokens + done, sizeof(int) * T,
                                       cudaMemcpyHostToDevice, st));
        if ((rc = maybe_rebuild(s, pos_now))) return rc;
        for (int t = 0; t < T; t++) s->tier[hcm_slot(pos_now + t, s->n_ctx)] = 2;   // kv_append
        fill_params(s, *s->sp_host, pos_now, T, tokens[done + T - 1]);
        QMA_CHECK_CUDA(cudaMemcpyAsync(s->sp_dev, s->sp_host, sizeof(StepParams),
                                       cudaMemcpyHostToDevice, st));
        const int nk = nk_upper(s, pos_now, T, false);
        if ((rc = ensure_attn_scratch(s, T, nk, attn_span(T, nk)))) return rc;
        const bool last = done + T == n_tokens;
        const int mode = n_layers < NLAYER ? 0 : (logits_all ? 2 : (last && logits ? 1 : 0));
        if ((rc = forward(s, *s->sp_host, s->tokens_dev, nk, mode, n_layers))) return rc;
        if (hidden)
            QMA_CHECK_CUDA(cudaMemcpyAsync(hidden + size_t(done) * EMBD, s->x, sizeof(float) * size_t(T) * EMBD,
                                           cudaMemcpyDeviceToHost, st));
        if (mode == 2 && logits)
            QMA_CHECK_CUDA(cudaMemcpyAsync(logits + size_t(done) * m->n_vocab, s->logits,
                                           sizeof(float) * size_t(T) * m->n_vocab,
                                           cudaMemcpyDeviceToHost, st));
        else if (mode == 1)
            QMA_CHECK_CUDA(cudaMemcpyAsync(logits, s->logits, sizeof(float) * m->n_vocab,
                                           cudaMemcpyDeviceToHost, st));
        // sp_host is reused by the next chunk: let this chunk consume it
        QMA_CHECK_CUDA(cudaStreamSynchronize(st));
        done += T;
    }
    s->n_pos += n_tokens;
    return check_wait_timeouts();
}

// One layer's mixer on caller activations (the layer-level parity points):
// x [T][2048] device residual input at the state's positions n_pos ..
// n_pos + T - 1; out [T][2048] device residual after the mixer.  With
// advance, the live index is rebuilt first when due (as qma_eval does at a
// chunk start, nn.c:2074-2088) and n_pos moves on by T afterwards.
static int mixer_call(qma_cuda_state *s, int il, const float *x, int T, float *out, bool advance) {
    qma_cuda_model *m = s->m;
    cudaStream_t st = s->st;
    QMA_CHECK_CUDA(cudaSetDevice(m->device));
    if (s->n_pos + T > s->n_ctx - HCM_SINK) {
        set_error("mixer: %d + %d positions exceed this state's ring of %d (no wrap-around)", s->n_pos, T,
                  s->n_ctx);
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
    int rc;
    const int pos_now = s->n_pos;
    if (advance && (rc = maybe_rebuild(s, pos_now))) return rc;
    if (is_attn(il))
        for (int t = 0; t < T; t++) s->tier[hcm_slot(pos_now + t, s->n_ctx)] = 2;   // kv_append
    fill_params(s, *s->sp_host, pos_now, T, 0);
    QMA_CHECK_CUDA(cudaMemcpyAsync(s->sp_dev, s->sp_host, sizeof(StepParams), cudaMemcpyHostToDevice, st));
    const int nk = nk_upper(s, pos_now, T, false);
    if ((rc = ensure_attn_scratch(s, T, nk, attn_span(T, nk)))) return rc;
    QMA_CHECK_CUDA(cudaMemcpyAsync(s->x, x, sizeof(float) * size_t(T) * EMBD, cudaMemcpyDeviceToDevice, st));
    if ((rc = launch_rmsnorm_quant(s->x, m->L[il].attn_norm, T, EMBD, s->xq, s->xd, s->xs, st))) return rc;
    bool side_pending = false;
    if ((rc = mixer(s, il, T, nk, attn_span(T, nk), side_pending))) return rc;
    if (side_pending) QMA_CHECK_CUDA(cudaStreamWaitEvent(st, s->ev_join, 0));
    QMA_CHECK_CUDA(cudaMemcpyAsync(out, s->x2, sizeof(float) * size_t(T) * EMBD, cudaMemcpyDeviceToDevice, st));
    QMA_CHECK_CUDA(cudaStreamSynchronize(st));
    if (advance) s->n_pos += T;
    if (s->graph) {          // the decode graph's step parameters are stale now
        cudaGraphExecDestroy(s->graph);
        s->graph = nullptr;
    }
    return check_wait_timeouts();
}

// n_tokens single-token steps of gated-delta-net layer il back to back (the
// decode kernels, one token at a time, no host synchronisation between
// them): the recurrence of a GDN layer reads no step parameters, so the
// tokens only need to run in order.
static int gdn_decode_call(qma_cuda_state *s, int il, const float *x, int n_tokens, float *out) {
    qma_cuda_model *m = s->m;
    cudaStream_t st = s->st;
    QMA_CHECK_CUDA(cudaSetDevice(m->device));
    if (s->n_pos + n_tokens > s->n_ctx - HCM_SINK) {
        set_error("gdn_decode: %d + %d positions exceed this state's ring of %d", s->n_pos, n_tokens, s->n_ctx);
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
    int rc;
    bool side_pending = false;
    for (int t = 0; t < n_tokens; t++) {
        // the copies also order the steps: the gated-delta kernel and the
        // in-projection's conv epilogue read the layer's recurrent and conv
        // state before their upstream wait, which is safe only once the
        // previous step's writers have finished; a copy in the stream ends
        // the chain of early-launched kernels between two steps
        QMA_CHECK_CUDA(cudaMemcpyAsync(s->x, x + size_t(t) * EMBD, sizeof(float) * EMBD, cudaMemcpyDeviceToDevice,
                                       st));
        if ((rc = launch_rmsnorm_quant(s->x, m->L[il].attn_norm, 1, EMBD, s->xq, s->xd, s->xs, st))) return rc;
        if ((rc = mixer(s, il, 1, 1, attn_span(1, 1), side_pending))) return rc;
        QMA_CHECK_CUDA(cudaMemcpyAsync(out + size_t(t) * EMBD, s->x2, sizeof(float) * EMBD,
                                       cudaMemcpyDeviceToDevice, st));
    }
    QMA_CHECK_CUDA(cudaStreamSynchronize(st));
    s->n_pos += n_tokens;
    if (s->graph) {
        cudaGraphExecDestroy(s->graph);
        s->graph = nullptr;
    }
    return check_wait_timeouts();
}

// Capture one decode step (T = 1, token and position read from sp_dev,
// argmax writes the next token and advances the position) as a graph.
static int capture_decode(qma_cuda_state *s) {
    cudaStream_t st = s->st;
    const int nk = nk_upper(s, s->n_pos, 1, true);
    int rc = ensure_attn_scratch(s, 1, nk, attn_span(1, nk));
    if (rc) return rc;
    QMA_CHECK_CUDA(cudaStreamSynchronize(st));
    cudaGraph_t g;
    QMA_CHECK_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    StepParams hs;
    fill_params(s, hs, s->n_pos, 1, 0);
    rc = forward(s, hs, nullptr, nk, 1);
    if (!rc) {
        if (launch_ex(argmax_kernel, dim3(ARG_CTAS), dim3(512), 0, st, 1, pdl_enabled(), s->logits,
                      s->m->n_vocab, s->sp_dev, s->argmax_dev, s->argmax_pv, s->argmax_pi,
                      s->argmax_cnt) != cudaSuccess)
            rc = QMA_CUDA_ERR_CUDA;
    }
    const cudaError_t e = cudaStreamEndCapture(st, &g);
    if (rc) return rc;
    if (e != cudaSuccess) {
        set_error("decode capture: %s", cudaGetErrorString(e));
        return QMA_CUDA_ERR_CUDA;
    }
    size_t nn = 0;
    cudaGraphGetNodes(g, nullptr, &nn);
    std::vector<cudaGraphNode_t> nodes(nn);
    if (nn) cudaGraphGetNodes(g, nodes.data(), &nn);
    int kernels = 0;
    for (size_t i = 0; i < nn; i++) {
        cudaGraphNodeType ty;
        if (cudaGraphNodeGetType(nodes[i], &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) kernels++;
    }
    s->graph_kernels = kernels;
    const cudaError_t e2 = cudaGraphInstantiate(&s->graph, g, 0);
    cudaGraphDestroy(g);
    if (e2 != cudaSuccess) {
        set_error("decode instantiate: %s", cudaGetErrorString(e2));
        return QMA_CUDA_ERR_CUDA;
    }
    s->graph_nk = nk;
    return QMA_CUDA_OK;
}

static int decode_greedy(qma_cuda_state *s, int token, int n_steps, int *tokens_out, float *logits) {
    qma_cuda_model *m = s->m;
    cudaStream_t st = s->st;
    QMA_CHECK_CUDA(cudaSetDevice(m->device));
    if (s->n_pos + n_steps > s->n_ctx - HCM_SINK) {
        set_error("decode: %d + %d positions exceed this state's ring of %d", s->n_pos, n_steps, s->n_ctx);
        return QMA_CUDA_ERR_UNSUPPORTED;
    }
    // the tokens land in pinned memory (an asynchronous copy per step, so the
    // host runs ahead of the device instead of waiting on every step) and
    // reach tokens_out after the last step
    if (tokens_out && n_steps > s->h_tok_cap) {
        const int cap = std::max(n_steps, std::max(1024, 2 * s->h_tok_cap));
        QMA_CHECK_CUDA(cudaStreamSynchronize(st));
        if (s->h_tok) QMA_CHECK_CUDA(cudaFreeHost(s->h_tok));
        s->h_tok = nullptr;
        s->h_tok_cap = 0;
        QMA_CHECK_CUDA(cudaMallocHost(&s->h_tok, sizeof(int) * size_t(cap)));
        s->h_tok_cap = cap;
    }
    int rc;
    int cur = token;
    for (int i = 0; i < n_steps; i++) {
        const int pos = s->n_pos;
        const bool rebuild = pos >= s->next_rebuild;
        if (rebuild || !s->graph || i == 0) {
            // host state is current only after the device caught up
            QMA_CHECK_CUDA(cudaStreamSynchronize(st));
            if (i > 0) {
                int dev_tok;
                QMA_CHECK_CUDA(cudaMemcpy(&dev_tok, s->argmax_dev, sizeof(int), cudaMemcpyDeviceToHost));
                cur = dev_tok;
            }
            if ((rc = maybe_rebuild(s, pos))) return rc;
            fill_params(s, *s->sp_host, pos, 1, cur);
            QMA_CHECK_CUDA(cudaMemcpyAsync(s->sp_dev, s->sp_host, sizeof(StepParams),
                                           cudaMemcpyHostToDevice, st));
            if (!s->graph && (rc = capture_decode(s))) return rc;
        }
        s->tier[hcm_slot(pos, s->n_ctx)] = 2;
        QMA_CHECK_CUDA(cudaGraphLaunch(s->graph, st));
        if (tokens_out) {
            if (i == 0) s->h_tok[0] = cur;
            if (i + 1 < n_steps)
                QMA_CHECK_CUDA(cudaMemcpyAsync(s->h_tok + i + 1, s->argmax_dev, sizeof(int),
                                               cudaMemcpyDeviceToHost, st));
        }
        s->n_pos += 1;
    }
    if (logits)
        QMA_CHECK_CUDA(cudaMemcpyAsync(logits, s->logits, sizeof(float) * m->n_vocab,
                                       cudaMemcpyDeviceToHost, st));
    QMA_CHECK_CUDA(cudaStreamSynchronize(st));
    if (tokens_out) memcpy(tokens_out, s->h_tok, sizeof(int) * size_t(n_steps));
    return check_wait_timeouts();
}

}  // namespace qma

// ------------------------------------------------------------------- C ABI --
extern "C" {

int qma_cuda_model_load(int device, const qma_cuda_tensor *tensors, uint32_t n,
                        const void *host_data, uint64_t data_size, qma_cuda_model **out) {
    qma::clear_error();
    return qma::build_model(device, tensors, n, host_data, data_size, false, 0, out);
}

int qma_cuda_model_synth(int device, const qma_cuda_tensor *tensors, uint32_t n, uint64_t seed,
                         qma_cuda_model **out) {
    qma::clear_error();
    return qma::build_model(device, tensors, n, nullptr, 0, true, seed, out);
}

int qma_cuda_model_check(const qma_cuda_tensor *tensors, uint32_t n, uint64_t data_size) {
    qma::clear_error();
    return qma::build_model(0, tensors, n, nullptr, data_size, data_size == 0, 0, nullptr, true);
}

int qma_cuda_model_free(qma_cuda_model *m) {
    qma::clear_error();
    if (!m) return QMA_CUDA_OK;
    cudaSetDevice(m->device);
    for (void *p : m->allocs) cudaFree(p);
    delete m;
    return QMA_CUDA_OK;
}

int qma_cuda_model_n_vocab(const qma_cuda_model *m) { return m ? m->n_vocab : 0; }

const float *qma_cuda_state_logits(const qma_cuda_state *s) { return s ? s->logits : nullptr; }

int qma_cuda_ecache_get(const qma_cuda_model *m, int layer, int expert, const void **gate,
                        const void **up, const void **down) {
    qma::clear_error();
    QMA_REQUIRE(m && layer >= 0 && layer < qma::NLAYER && expert >= 0 && expert < qma::MOE_NEXP,
                "qma_cuda_ecache_get: bad (layer %d, expert %d)", layer, expert);
    const qma_cuda_moe_weights &w = m->L[layer].moe;
    const size_t gu = size_t(qma::MOE_FF) * (qma::MOE_EMBD / 256) * qma::Q4K_BYTES;
    const size_t dn = qma::packed_bytes(w.down_type, qma::MOE_EMBD, qma::MOE_FF);
    if (gate) *gate = static_cast<const uint8_t *>(w.gate_exps) + gu * expert;
    if (up) *up = static_cast<const uint8_t *>(w.up_exps) + gu * expert;
    if (down) *down = static_cast<const uint8_t *>(w.down_exps) + dn * expert;
    return QMA_CUDA_OK;
}

namespace qma {

constexpr int EC_PF_MAX = 64;      // ecache.h:52

// One CTA: thread i asks L2 for record i / 3 of the list (its gate, up or
// down matrix), as a speculative fill with no completion to wait for.
struct EcRange {
    const void *p[3 * EC_PF_MAX];
    uint32_t bytes[3 * EC_PF_MAX];
};
__global__ void ecache_l2_fill_kernel(EcRange r, int n) {
    const int i = threadIdx.x;
    if (i < n) prefetch_l2_range(r.p[i], r.bytes[i]);
}

static int ecache_fill(const qma_cuda_model *m, int layer, const int *ids, int n, void *stream, const char *fn) {
    QMA_REQUIRE(m && layer >= 0 && layer < NLAYER && n >= 0 && (ids || n == 0), "%s: bad arguments", fn);
    if (n > EC_PF_MAX) n = EC_PF_MAX;        // as the reference clamps (ecache.c:406)
    const qma_cuda_moe_weights &w = m->L[layer].moe;
    const size_t gu = size_t(MOE_FF) * (MOE_EMBD / 256) * Q4K_BYTES;
    const size_t dn = packed_bytes(w.down_type, MOE_EMBD, MOE_FF);
    EcRange r{};
    int k = 0;
    for (int i = 0; i < n; i++) {
        QMA_REQUIRE(ids[i] >= 0 && ids[i] < MOE_NEXP, "%s: expert id %d", fn, ids[i]);
        r.p[k] = static_cast<const uint8_t *>(w.gate_exps) + gu * ids[i];
        r.bytes[k++] = uint32_t(gu);
        r.p[k] = static_cast<const uint8_t *>(w.up_exps) + gu * ids[i];
        r.bytes[k++] = uint32_t(gu);
        r.p[k] = static_cast<const uint8_t *>(w.down_exps) + dn * ids[i];
        r.bytes[k++] = uint32_t(dn);
    }
    if (!k) return QMA_CUDA_OK;
    QMA_CHECK_CUDA(cudaSetDevice(m->device));
    ecache_l2_fill_kernel<<<1, 3 * EC_PF_MAX, 0, as_stream(stream)>>>(r, k);
    QMA_CHECK_LAUNCH();
    return QMA_CUDA_OK;
}

}  // namespace qma

int qma_cuda_ecache_hint(const qma_cuda_model *m, int layer, const int *ids, int n, void *stream) {
    qma::clear_error();
    return qma::ecache_fill(m, layer, ids, n, stream, "qma_cuda_ecache_hint");
}

int qma_cuda_ecache_prefetch(const qma_cuda_model *m, int layer, const int *ids, int n, void *stream) {
    qma::clear_error();
    return qma::ecache_fill(m, layer, ids, n, stream, "qma_cuda_ecache_prefetch");
}

int qma_cuda_ecache_hold(qma_cuda_model *m, int layer, int expert, const void **gate, const void **up,
                         const void **down) {
    qma::clear_error();
    QMA_REQUIRE(m, "qma_cuda_ecache_hold: null model");
    {
        std::lock_guard<std::mutex> lock(m->ec_mu);
        if (m->ec_held >= qma::EC_PF_MAX) {
            qma::set_error("qma_cuda_ecache_hold: %d records held already (at most %d until a release)",
                           m->ec_held, qma::EC_PF_MAX);
            return QMA_CUDA_ERR_STATE;
        }
        const int rc = qma_cuda_ecache_get(m, layer, expert, gate, up, down);
        if (rc) return rc;
        m->ec_held++;
    }
    return QMA_CUDA_OK;
}

int qma_cuda_ecache_release(qma_cuda_model *m) {
    qma::clear_error();
    QMA_REQUIRE(m, "qma_cuda_ecache_release: null model");
    std::lock_guard<std::mutex> lock(m->ec_mu);
    m->ec_held = 0;
    return QMA_CUDA_OK;
}

int qma_cuda_ecache_held(const qma_cuda_model *m) {
    if (!m) return -1;
    std::lock_guard<std::mutex> lock(const_cast<qma_cuda_model *>(m)->ec_mu);
    return m->ec_held;
}

int qma_cuda_model_set_router_bias(qma_cuda_model *m, int layer, const float *bias) {
    qma::clear_error();
    QMA_REQUIRE(m && layer >= 0 && layer < qma::NLAYER, "qma_cuda_model_set_router_bias: bad arguments");
    m->L[layer].moe.router_bias = bias;
    return QMA_CUDA_OK;
}

int qma_cuda_model_moe_weights(const qma_cuda_model *m, int layer, qma_cuda_moe_weights *out) {
    qma::clear_error();
    QMA_REQUIRE(m && out && layer >= 0 && layer < qma::NLAYER, "qma_cuda_model_moe_weights: bad layer %d", layer);
    *out = m->L[layer].moe;
    return QMA_CUDA_OK;
}

int qma_cuda_state_create(qma_cuda_model *m, int n_ctx, qma_cuda_state **out) {
    qma::clear_error();
    return qma::create_state(m, n_ctx, out);
}

int qma_cuda_state_free(qma_cuda_state *s) {
    qma::clear_error();
    if (!s) return QMA_CUDA_OK;
    cudaSetDevice(s->m->device);
    cudaStreamSynchronize(s->st);
    if (s->graph) cudaGraphExecDestroy(s->graph);
    for (void *p : s->allocs) cudaFree(p);
    for (float *p : {s->scores, s->cmax, s->opart, s->lpart}) if (p) cudaFreeAsync(p, s->st);
    cudaStreamSynchronize(s->st);
    if (s->sp_host) cudaFreeHost(s->sp_host);
    for (float *p : {s->h_sal, s->h_qf, s->h_pin_sal}) if (p) cudaFreeHost(p);
    if (s->h_tok) cudaFreeHost(s->h_tok);
    cudaStreamSynchronize(s->side);
    cudaEventDestroy(s->ev_fork);
    cudaEventDestroy(s->ev_join);
    if (!s->shared_stream) {
        cudaStreamDestroy(s->side);
        cudaStreamDestroy(s->st);
    }
    delete s;
    return QMA_CUDA_OK;
}

int qma_cuda_state_n_pos(const qma_cuda_state *s) { return s ? s->n_pos : -1; }

void *qma_cuda_state_stream(const qma_cuda_state *s) { return s ? static_cast<void *>(s->st) : nullptr; }

int qma_cuda_state_kv_slot(const qma_cuda_state *s, int lay, int head, int slot, uint8_t *out) {
    qma::clear_error();
    QMA_REQUIRE(s && out && lay >= 0 && lay < qma::NATTN && head >= 0 && head < 2 * qma::NHEAD_KV &&
                    slot >= 0 && slot < s->n_ctx,
                "qma_cuda_state_kv_slot: bad arguments");
    QMA_CHECK_CUDA(cudaStreamSynchronize(s->st));
    QMA_CHECK_CUDA(cudaMemcpy(out, s->kv[lay] + (size_t(head) * s->n_ctx + slot) * qma::KVQ_SLOT,
                              qma::KVQ_SLOT, cudaMemcpyDeviceToHost));
    return QMA_CUDA_OK;
}

int qma_cuda_state_stats(const qma_cuda_state *s, int *graph_kernels, uint64_t *state_bytes) {
    qma::clear_error();
    QMA_REQUIRE(s, "qma_cuda_state_stats: null state");
    if (graph_kernels) *graph_kernels = s->graph_kernels;
    if (state_bytes) *state_bytes = s->state_bytes;
    return QMA_CUDA_OK;
}

int qma_cuda_eval(qma_cuda_model *m, qma_cuda_state *s, const int *tokens, int n_tokens,
                  float *logits, int logits_all) {
    qma::clear_error();
    QMA_REQUIRE(m && s && s->m == m && tokens && n_tokens > 0, "qma_cuda_eval: bad arguments");
    for (int i = 0; i < n_tokens; i++)
        QMA_REQUIRE(tokens[i] >= 0 && tokens[i] < m->n_vocab, "qma_cuda_eval: token %d out of range",
                    tokens[i]);
    return qma::eval(s, tokens, n_tokens, logits, logits_all);
}

int qma_cuda_eval_hidden(qma_cuda_model *m, qma_cuda_state *s, const int *tokens, int n_tokens,
                         int n_layers, float *hidden) {
    qma::clear_error();
    QMA_REQUIRE(m && s && s->m == m && tokens && n_tokens > 0 && hidden && n_layers >= -qma::NLAYER &&
                    n_layers <= qma::NLAYER,
                "qma_cuda_eval_hidden: bad arguments");
    s->stop_before_moe = n_layers < 0;
    const int rc = qma::eval(s, tokens, n_tokens, nullptr, 0, n_layers < 0 ? -n_layers : n_layers, hidden);
    s->stop_before_moe = false;
    return rc;
}

int qma_cuda_gdn_step(qma_cuda_state *s, int layer, const float *x, int n_tokens, float *x_out, int advance) {
    qma::clear_error();
    QMA_REQUIRE(s && x && x_out && layer >= 0 && layer < qma::NLAYER && !qma::is_attn(layer) && n_tokens >= 1 &&
                    n_tokens <= qma::MAX_CHUNK,
                "qma_cuda_gdn_step: bad arguments (layer %d must be a gated-delta-net layer, 1..%d tokens)", layer,
                qma::MAX_CHUNK);
    return qma::mixer_call(s, layer, x, n_tokens, x_out, advance != 0);
}

int qma_cuda_gdn_decode(qma_cuda_state *s, int layer, const float *x, int n_tokens, float *x_out) {
    qma::clear_error();
    QMA_REQUIRE(s && x && x_out && layer >= 0 && layer < qma::NLAYER && !qma::is_attn(layer) && n_tokens >= 1,
                "qma_cuda_gdn_decode: bad arguments (layer %d must be a gated-delta-net layer)", layer);
    return qma::gdn_decode_call(s, layer, x, n_tokens, x_out);
}

int qma_cuda_attn_decode(qma_cuda_state *s, int layer, const float *x, int n_tokens, float *x_out, int advance) {
    qma::clear_error();
    QMA_REQUIRE(s && x && x_out && layer >= 0 && layer < qma::NLAYER && qma::is_attn(layer) && n_tokens >= 1 &&
                    n_tokens <= qma::MAX_CHUNK,
                "qma_cuda_attn_decode: bad arguments (layer %d must be an attention layer, 1..%d tokens)", layer,
                qma::MAX_CHUNK);
    return qma::mixer_call(s, layer, x, n_tokens, x_out, advance != 0);
}

int qma_cuda_decode_greedy(qma_cuda_model *m, qma_cuda_state *s, int token, int n_steps,
                           int *tokens_out, float *logits) {
    qma::clear_error();
    QMA_REQUIRE(m && s && s->m == m && n_steps > 0 && token >= 0 && token < m->n_vocab,
                "qma_cuda_decode_greedy: bad arguments");
    return qma::decode_greedy(s, token, n_steps, tokens_out, logits);
}

}  // extern "C"

// ---------------------------------------------------------------- session --
// A sequence's state saved to and restored from the files
// qma's session keeps (agent.c:409-416, 765-816), byte for byte in the
// reference's formats:
//   state    runstate_save / runstate_load (nn.c:2011-2042): int32 n_pos, then
//            per gated-delta-net layer the conv state float [8192][3] and the
//            recurrent state float [32][128][128] (row j of head h holds
//            S[i][j] at j * 128 + i);
//   kv       the KV slab file of runstate_init_kv (nn.c:1878-1935): per
//            attention layer [K head 0, K head 1, V head 0, V head 1][n_ctx]
//            240-byte records;
//   salience hcm_save / hcm_load (nn.c:1156-1209): uint32 n_ctx, salience
//            float [10][n_ctx], arena positions int32 [2048], arena salience
//            float [10][2048], arena records [10][4][2048][240].
// The engine's device buffers already use these layouts, so a save is one
// device-to-host copy per section.  A load also resets the heavy-hitter
// bookkeeping the way a fresh qma process starts (hcm_init, nn.c:947-970):
// tiers, live index and quantisation scores cleared, the next rebuild due at
// position 128, so the first eval after it rebuilds the live index from the
// restored salience and arena.
namespace qma {
namespace {

struct File {
    FILE *f = nullptr;
    explicit File(const char *path, const char *mode) { f = fopen(path, mode); }
    ~File() {
        if (f) fclose(f);
    }
};

// device -> file, through a bounded host buffer
int write_dev(FILE *f, const void *dev, size_t bytes, cudaStream_t st) {
    static constexpr size_t CH = size_t(64) << 20;
    std::vector<uint8_t> h(bytes < CH ? bytes : CH);
    for (size_t o = 0; o < bytes; o += CH) {
        const size_t n = bytes - o < CH ? bytes - o : CH;
        QMA_CHECK_CUDA(cudaMemcpyAsync(h.data(), static_cast<const uint8_t *>(dev) + o, n, cudaMemcpyDeviceToHost,
                                       st));
        QMA_CHECK_CUDA(cudaStreamSynchronize(st));
        if (fwrite(h.data(), 1, n, f) != n) {
            set_error("session: write failed");
            return QMA_CUDA_ERR_INVALID;
        }
    }
    return QMA_CUDA_OK;
}

// file -> device; returns 1 (and copies nothing more) if the file ends early
int read_dev(FILE *f, void *dev, size_t bytes, cudaStream_t st, bool *short_read) {
    static constexpr size_t CH = size_t(64) << 20;
    std::vector<uint8_t> h(bytes < CH ? bytes : CH);
    for (size_t o = 0; o < bytes; o += CH) {
        const size_t n = bytes - o < CH ? bytes - o : CH;
        if (fread(h.data(), 1, n, f) != n) {
            *short_read = true;
            return QMA_CUDA_OK;
        }
        QMA_CHECK_CUDA(cudaMemcpyAsync(static_cast<uint8_t *>(dev) + o, h.data(), n, cudaMemcpyHostToDevice, st));
        QMA_CHECK_CUDA(cudaStreamSynchronize(st));
    }
    return QMA_CUDA_OK;
}

size_t conv_bytes() { return sizeof(float) * size_t(CONV_DIM) * 3; }
size_t ssm_bytes() { return sizeof(float) * size_t(VHEADS) * SSTATE * SSTATE; }
size_t kv_layer_bytes(int n_ctx) { return size_t(2) * NHEAD_KV * n_ctx * KVQ_SLOT; }
size_t arena_layer_bytes() { return size_t(2) * NHEAD_KV * HCM_H_PIN * KVQ_SLOT; }

int save_state(const qma_cuda_state *s, const char *path) {
    File f(path, "wb");
    if (!f.f) {
        set_error("session: cannot write %s", path);
        return QMA_CUDA_ERR_INVALID;
    }
    const int32_t np = s->n_pos;
    if (fwrite(&np, 4, 1, f.f) != 1) {
        set_error("session: write failed");
        return QMA_CUDA_ERR_INVALID;
    }
    int rc;
    for (int il = 0; il < NLAYER; il++) {
        if (is_attn(il)) continue;
        if ((rc = write_dev(f.f, s->conv[il], conv_bytes(), s->st))) return rc;
        if ((rc = write_dev(f.f, s->ssm[il], ssm_bytes(), s->st))) return rc;
    }
    return QMA_CUDA_OK;
}

int save_kv(const qma_cuda_state *s, const char *path) {
    File f(path, "wb");
    if (!f.f) {
        set_error("session: cannot write %s", path);
        return QMA_CUDA_ERR_INVALID;
    }
    int rc;
    for (int a = 0; a < NATTN; a++)
        if ((rc = write_dev(f.f, s->kv[a], kv_layer_bytes(s->n_ctx), s->st))) return rc;
    return QMA_CUDA_OK;
}

int save_salience(const qma_cuda_state *s, const char *path) {
    File f(path, "wb");
    if (!f.f) {
        set_error("session: cannot write %s", path);
        return QMA_CUDA_ERR_INVALID;
    }
    const uint32_t nc = uint32_t(s->n_ctx);
    if (fwrite(&nc, 4, 1, f.f) != 1) {
        set_error("session: write failed");
        return QMA_CUDA_ERR_INVALID;
    }
    int rc;
    if ((rc = write_dev(f.f, s->sal, sizeof(float) * size_t(NATTN) * s->n_ctx, s->st))) return rc;
    if (fwrite(s->pin_pos.data(), sizeof(int32_t), HCM_H_PIN, f.f) != size_t(HCM_H_PIN)) {
        set_error("session: write failed");
        return QMA_CUDA_ERR_INVALID;
    }
    if ((rc = write_dev(f.f, s->pin_sal, sizeof(float) * size_t(NATTN) * HCM_H_PIN, s->st))) return rc;
    for (int a = 0; a < NATTN; a++)
        if ((rc = write_dev(f.f, s->arena[a], arena_layer_bytes(), s->st))) return rc;
    return QMA_CUDA_OK;
}

int load_state(qma_cuda_state *s, const char *path) {
    File f(path, "rb");
    if (!f.f) {
        set_error("session: cannot read %s", path);
        return QMA_CUDA_ERR_INVALID;
    }
    int32_t np = 0;
    if (fread(&np, 4, 1, f.f) != 1 || np < 0) {
        set_error("session: %s: no position count", path);
        return QMA_CUDA_ERR_INVALID;
    }
    int rc;
    bool short_read = false;
    for (int il = 0; il < NLAYER && !short_read; il++) {
        if (is_attn(il)) continue;
        if ((rc = read_dev(f.f, s->conv[il], conv_bytes(), s->st, &short_read))) return rc;
        if (!short_read && (rc = read_dev(f.f, s->ssm[il], ssm_bytes(), s->st, &short_read))) return rc;
    }
    if (short_read) {
        set_error("session: %s is shorter than the recurrent state", path);
        return QMA_CUDA_ERR_INVALID;
    }
    s->n_pos = np;
    return QMA_CUDA_OK;
}

int load_kv(qma_cuda_state *s, const char *path) {
    File f(path, "rb");
    if (!f.f) {
        set_error("session: cannot read %s", path);
        return QMA_CUDA_ERR_INVALID;
    }
    fseek(f.f, 0, SEEK_END);
    const long size = ftell(f.f);
    fseek(f.f, 0, SEEK_SET);
    if (size < 0 || size_t(size) != NATTN * kv_layer_bytes(s->n_ctx)) {
        set_error("session: %s holds %ld bytes, a KV slab of n_ctx %d holds %zu", path, size, s->n_ctx,
                  NATTN * kv_layer_bytes(s->n_ctx));
        return QMA_CUDA_ERR_INVALID;
    }
    int rc;
    bool short_read = false;
    for (int a = 0; a < NATTN && !short_read; a++)
        if ((rc = read_dev(f.f, s->kv[a], kv_layer_bytes(s->n_ctx), s->st, &short_read))) return rc;
    if (short_read) {
        set_error("session: %s: read failed", path);
        return QMA_CUDA_ERR_INVALID;
    }
    return QMA_CUDA_OK;
}

// hcm_load (nn.c:1173-1209): salience required; the arena sections are
// optional (older files end after the salience: no pinned entries)
int load_salience(qma_cuda_state *s, const char *path) {
    File f(path, "rb");
    if (!f.f) {
        set_error("session: cannot read %s", path);
        return QMA_CUDA_ERR_INVALID;
    }
    uint32_t nc = 0;
    if (fread(&nc, 4, 1, f.f) != 1 || int(nc) != s->n_ctx) {
        set_error("session: %s was saved for another n_ctx", path);
        return QMA_CUDA_ERR_INVALID;
    }
    int rc;
    bool short_read = false;
    if ((rc = read_dev(f.f, s->sal, sizeof(float) * size_t(NATTN) * s->n_ctx, s->st, &short_read))) return rc;
    if (short_read) {
        set_error("session: %s: salience cut short", path);
        return QMA_CUDA_ERR_INVALID;
    }
    std::vector<int32_t> pos(HCM_H_PIN);
    const bool have_pos = fread(pos.data(), sizeof(int32_t), HCM_H_PIN, f.f) == size_t(HCM_H_PIN);
    if (have_pos) {
        std::vector<float> psal(size_t(NATTN) * HCM_H_PIN);
        std::vector<uint8_t> rec(arena_layer_bytes());
        bool ok = fread(psal.data(), sizeof(float), psal.size(), f.f) == psal.size();
        if (ok) {
            QMA_CHECK_CUDA(cudaMemcpyAsync(s->pin_sal, psal.data(), psal.size() * sizeof(float),
                                           cudaMemcpyHostToDevice, s->st));
            for (int a = 0; a < NATTN && ok; a++) {
                ok = fread(rec.data(), 1, rec.size(), f.f) == rec.size();
                if (ok) {
                    QMA_CHECK_CUDA(cudaMemcpyAsync(s->arena[a], rec.data(), rec.size(), cudaMemcpyHostToDevice,
                                                   s->st));
                    QMA_CHECK_CUDA(cudaStreamSynchronize(s->st));
                }
            }
        }
        // a cut-short arena section leaves no pinned entries (nn.c:1193-1203)
        s->pin_pos = ok ? pos : std::vector<int32_t>(HCM_H_PIN, -1);
    } else {
        s->pin_pos.assign(HCM_H_PIN, -1);
    }
    QMA_CHECK_CUDA(cudaStreamSynchronize(s->st));
    return QMA_CUDA_OK;
}

// the heavy-hitter bookkeeping of a fresh process (hcm_init, nn.c:947-970)
int reset_hcm(qma_cuda_state *s) {
    s->live.assign(s->n_ctx, 0);
    s->tier.assign(s->n_ctx, 0);
    s->live_n = s->n4 = s->n_ring_q4 = 0;
    s->rebuilt_at = 0;
    s->next_rebuild = qma_cuda_state::HCM_REBUILD_INIT;
    QMA_CHECK_CUDA(cudaMemsetAsync(s->qf, 0, sizeof(float) * size_t(s->n_ctx), s->st));
    if (s->graph) {
        cudaGraphExecDestroy(s->graph);
        s->graph = nullptr;
    }
    QMA_CHECK_CUDA(cudaStreamSynchronize(s->st));
    return QMA_CUDA_OK;
}

}  // namespace
}  // namespace qma

extern "C" {

int qma_cuda_state_save(const qma_cuda_state *s, const char *state_path, const char *kv_path,
                        const char *salience_path) {
    using namespace qma;
    clear_error();
    QMA_REQUIRE(s, "qma_cuda_state_save: null state");
    QMA_CHECK_CUDA(cudaSetDevice(s->m->device));
    QMA_CHECK_CUDA(cudaStreamSynchronize(s->st));
    QMA_CHECK_CUDA(cudaStreamSynchronize(s->side));
    int rc;
    if (state_path && (rc = save_state(s, state_path))) return rc;
    if (kv_path && (rc = save_kv(s, kv_path))) return rc;
    if (salience_path && (rc = save_salience(s, salience_path))) return rc;
    return QMA_CUDA_OK;
}

int qma_cuda_state_load(qma_cuda_state *s, const char *state_path, const char *kv_path,
                        const char *salience_path) {
    using namespace qma;
    clear_error();
    QMA_REQUIRE(s, "qma_cuda_state_load: null state");
    QMA_CHECK_CUDA(cudaSetDevice(s->m->device));
    QMA_CHECK_CUDA(cudaStreamSynchronize(s->st));
    QMA_CHECK_CUDA(cudaStreamSynchronize(s->side));
    int rc;
    if (state_path && (rc = load_state(s, state_path))) return rc;
    if (kv_path && (rc = load_kv(s, kv_path))) return rc;
    if ((rc = reset_hcm(s))) return rc;
    if (salience_path && (rc = load_salience(s, salience_path))) return rc;
    return QMA_CUDA_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ batch --
// n_seq sequences decoded together (the multi-sequence state of a serving
// loop; the reference's runstate_t, qma.h:254-276, is one sequence, and
// qma_eval, nn.c:2056-2308, runs one).  Each sequence is a full state of
// its own (KV ring, recurrent state, HCM tiers) on the batch's stream.  A
// step of one token from each of T sequences runs the token-parallel work
// once over all T rows: the RMSNorms, the input and output projections
// (the tensor-core GEMM from 8 rows on), the router and experts (the
// grouped path from 16 rows on, or the expert-parallel exchange), the LM
// head; the mixers run per sequence: the conv and gated-delta recurrence as
// one launch that looks up each row's own state through a pointer table,
// attention (its KV ring, live index and salience) once per sequence.
// Sequences given several tokens in one call are prefilled through their
// own state (the single-sequence chunked path).
struct qma_cuda_batch {
    qma_cuda_model *m = nullptr;
    int n_seq = 0, n_ctx = 0, t_step = 0;        // t_step: rows per batched step
    cudaStream_t st = nullptr;
    std::vector<qma_cuda_state *> seqs;
    qma_cuda_state *work = nullptr;              // activations of a batched step
    std::vector<void *> allocs;
    float **conv_tab = nullptr, **ssm_tab = nullptr;   // device [NLAYER][n_seq]
    int *seq_dev = nullptr;                      // device [t_step] sequence of each row
    qma::StepParams *sp_dev = nullptr;           // device [n_seq]: sequence i's kernels read entry i
    qma::StepParams *sp_host = nullptr;          // pinned [n_seq]
    int *h_tok = nullptr, *h_seq = nullptr;      // pinned [t_step]
    float *logits = nullptr;                     // device [t_step][n_vocab]
    int *greedy_dev = nullptr;                   // device [t_step]
    float *h_row = nullptr;                      // pinned [n_vocab], a prefilled sequence's logits
    qma::AttnRow *rows_dev = nullptr, *rows_host = nullptr;   // [NATTN][t_step] attention arguments of a step
    qma_cuda_ep *ep = nullptr;                   // expert-parallel MoE blocks, when set
    std::vector<qma_cuda_moe_weights> ep_w;      // this rank's shard views, per layer
};

namespace qma {

// Greedy id of each logits row: one CTA per row, ties to the lowest id.
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float *__restrict__ logits, int n, int *out) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *x = logits + size_t(row) * n;
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = tid; i < n; i += blockDim.x) {
        const float xv = x[i];
        if (xv > v) { v = xv; idx = i; }
    }
    for (int o = 16; o > 0; o >>= 1)
        argmax_merge(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
    if (lane == 0) { bv[warp] = v; bi[warp] = idx; }
    __syncthreads();
    if (warp) return;
    v = lane < int(blockDim.x >> 5) ? bv[lane] : -INFINITY;
    idx = lane < int(blockDim.x >> 5) ? bi[lane] : 0x7fffffff;
    for (int o = 16; o > 0; o >>= 1)
        argmax_merge(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
    if (lane == 0) out[row] = idx;
}

static int batch_free(qma_cuda_batch *b) {
    if (!b) return QMA_CUDA_OK;
    cudaSetDevice(b->m->device);
    if (b->st) cudaStreamSynchronize(b->st);
    for (qma_cuda_state *c : b->seqs) qma_cuda_state_free(c);
    if (b->work) qma_cuda_state_free(b->work);
    for (void *p : b->allocs) cudaFree(p);
    for (void *p : {static_cast<void *>(b->sp_host), static_cast<void *>(b->h_tok), static_cast<void *>(b->h_seq),
                    static_cast<void *>(b->h_row), static_cast<void *>(b->rows_host)})
        if (p) cudaFreeHost(p);
    if (b->st) cudaStreamDestroy(b->st);
    delete b;
    return QMA_CUDA_OK;
}

static int batch_create(qma_cuda_model *m, int n_seq, int n_ctx, qma_cuda_batch **out) {
    QMA_CHECK_CUDA(cudaSetDevice(m->device));
    qma_cuda_batch *b = new qma_cuda_batch();
    b->m = m;
    b->n_seq = n_seq;
    b->n_ctx = n_ctx;
    b->t_step = n_seq < MAX_CHUNK ? n_seq : MAX_CHUNK;
    int rc = QMA_CUDA_OK;
    auto dalloc = [&](void **p, size_t bytes) -> int {
        QMA_CHECK_CUDA(cudaMalloc(p, bytes));
        b->allocs.push_back(*p);
        QMA_CHECK_CUDA(cudaMemset(*p, 0, bytes));
        return QMA_CUDA_OK;
    };
    auto fail = [&](int e) {
        batch_free(b);
        return e;
    };
    if (cudaStreamCreateWithFlags(&b->st, cudaStreamNonBlocking) != cudaSuccess) {
        set_error("batch: stream creation failed");
        return fail(QMA_CUDA_ERR_CUDA);
    }
    if ((rc = dalloc(reinterpret_cast<void **>(&b->sp_dev), sizeof(StepParams) * n_seq))) return fail(rc);
    for (int i = 0; i < n_seq; i++) {
        qma_cuda_state *c = nullptr;
        if ((rc = create_state(m, n_ctx, &c, b->st))) return fail(rc);
        b->seqs.push_back(c);
        c->sp_dev = b->sp_dev + i;       // its own kernels read its entry of the batch's array
    }
    if ((rc = create_state(m, HCM_SINK + 2, &b->work, b->st))) return fail(rc);
    std::vector<float *> tab(size_t(NLAYER) * n_seq, nullptr);
    if ((rc = dalloc(reinterpret_cast<void **>(&b->conv_tab), sizeof(float *) * tab.size()))) return fail(rc);
    if ((rc = dalloc(reinterpret_cast<void **>(&b->ssm_tab), sizeof(float *) * tab.size()))) return fail(rc);
    for (int il = 0; il < NLAYER; il++)
        for (int i = 0; i < n_seq; i++) tab[size_t(il) * n_seq + i] = b->seqs[i]->conv[il];
    if (cudaMemcpy(b->conv_tab, tab.data(), sizeof(float *) * tab.size(), cudaMemcpyHostToDevice) != cudaSuccess)
        return fail(QMA_CUDA_ERR_CUDA);
    for (int il = 0; il < NLAYER; il++)
        for (int i = 0; i < n_seq; i++) tab[size_t(il) * n_seq + i] = b->seqs[i]->ssm[il];
    if (cudaMemcpy(b->ssm_tab, tab.data(), sizeof(float *) * tab.size(), cudaMemcpyHostToDevice) != cudaSuccess)
        return fail(QMA_CUDA_ERR_CUDA);
    if ((rc = dalloc(reinterpret_cast<void **>(&b->seq_dev), sizeof(int) * b->t_step))) return fail(rc);
    if ((rc = dalloc(reinterpret_cast<void **>(&b->greedy_dev), sizeof(int) * b->t_step))) return fail(rc);
    if ((rc = dalloc(reinterpret_cast<void **>(&b->logits), sizeof(float) * size_t(b->t_step) * m->n_vocab)))
        return fail(rc);
    if ((rc = dalloc(reinterpret_cast<void **>(&b->rows_dev), sizeof(AttnRow) * NATTN * b->t_step))) return fail(rc);
    if (cudaMallocHost(&b->rows_host, sizeof(AttnRow) * NATTN * b->t_step) != cudaSuccess ||
        cudaMallocHost(&b->sp_host, sizeof(StepParams) * n_seq) != cudaSuccess ||
        cudaMallocHost(&b->h_tok, sizeof(int) * b->t_step) != cudaSuccess ||
        cudaMallocHost(&b->h_seq, sizeof(int) * b->t_step) != cudaSuccess ||
        cudaMallocHost(&b->h_row, sizeof(float) * m->n_vocab) != cudaSuccess) {
        set_error("batch: pinned host allocation failed");
        return fail(QMA_CUDA_ERR_NOMEM);
    }
    memset(b->sp_host, 0, sizeof(StepParams) * n_seq);
    if (cudaStreamSynchronize(b->st) != cudaSuccess) return fail(QMA_CUDA_ERR_CUDA);
    *out = b;
    return QMA_CUDA_OK;
}

// One token from each of T distinct sequences (rows t of the step; row t
// is row rows[t] of the caller's logits / greedy / hidden).  n_layers <
// NLAYER stops after that many layers and returns the residual stream in
// hidden (host [n][2048]), the layer-level parity point.
static int batch_step(qma_cuda_batch *b, const int *seq_ids, const int *tokens, int T, float *logits_host,
                      int64_t logits_ld, const int *rows, int *greedy, int n_layers, float *hidden) {
    qma_cuda_model *m = b->m;
    qma_cuda_state *w = b->work;
    cudaStream_t st = b->st;
    int rc;
#define TRY(x) do { if ((rc = (x))) return rc; } while (0)
    std::vector<int> nk(T);
    for (int t = 0; t < T; t++) {
        qma_cuda_state *c = b->seqs[seq_ids[t]];
        const int pos = c->n_pos;
        if (pos + 1 > c->n_ctx - HCM_SINK) {
            set_error("batch: sequence %d is full (%d positions of a ring of %d)", seq_ids[t], pos, c->n_ctx);
            return QMA_CUDA_ERR_UNSUPPORTED;
        }
        TRY(maybe_rebuild(c, pos));
        c->tier[hcm_slot(pos, c->n_ctx)] = 2;      // kv_append
        nk[t] = nk_upper(c, pos, 1, false);
        TRY(ensure_attn_scratch(c, 1, nk[t], attn_span(1, nk[t])));
    }
    // the previous step ended with a synchronize: the pinned buffers are free
    for (int t = 0; t < T; t++) {
        qma_cuda_state *c = b->seqs[seq_ids[t]];
        fill_params(c, b->sp_host[seq_ids[t]], c->n_pos, 1, tokens[t]);
        b->h_tok[t] = tokens[t];
        b->h_seq[t] = seq_ids[t];
    }
    // the attention arguments of every (attention layer, row): one launch per
    // kernel serves all rows while every span fits the decode kernel
    // (QMA_CUDA_ATTN_PER_SEQ=1 in the environment: one sequence at a time,
    // the same kernels and results, as a cross-check)
    const char *per_seq = getenv("QMA_CUDA_ATTN_PER_SEQ");
    bool rows_ok = !(per_seq && atoi(per_seq) != 0);
    int max_nchunk = 1, max_nk = 1;
    for (int t = 0; t < T; t++) {
        const int span = attn_span(1, nk[t]);
        rows_ok = rows_ok && span <= ATTN_ROWS_MAX_SPAN;
        max_nchunk = std::max(max_nchunk, (nk[t] + span - 1) / span);
        max_nk = std::max(max_nk, nk[t]);
    }
    if (rows_ok) {
        for (int lay = 0; lay < NATTN; lay++)
            for (int t = 0; t < T; t++) {
                qma_cuda_state *c = b->seqs[seq_ids[t]];
                AttnRow &r = b->rows_host[size_t(lay) * b->t_step + t];
                r.sp = c->sp_dev;
                r.proj = w->proj + size_t(t) * m->L[4 * lay + 3].in_rows;
                r.rope = c->rope;
                r.qr = c->qr; r.z = c->z;
                r.kv = c->kv[lay]; r.arena = c->arena[lay]; r.live = c->live_dev;
                r.qf = c->qf; r.sal_all = c->sal;
                r.scores = c->scores; r.cmax = c->cmax; r.lpart = c->lpart; r.opart = c->opart; r.ml = c->ml;
                r.xq = w->xq + size_t(t) * WO_DIM;
                r.xd = w->xd + size_t(t) * (WO_DIM / 256);
                r.xs = w->xs + size_t(t) * (WO_DIM / 16);
                r.sal = c->sal + size_t(lay) * c->n_ctx;
                r.pin_sal = c->pin_sal + size_t(lay) * HCM_H_PIN;
                r.nk_max = nk[t];
                r.span = attn_span(1, nk[t]);
                r.nchunk = (nk[t] + r.span - 1) / r.span;
            }
        for (int lay = 0; lay < NATTN; lay++)
            QMA_CHECK_CUDA(cudaMemcpyAsync(b->rows_dev + size_t(lay) * b->t_step,
                                           b->rows_host + size_t(lay) * b->t_step, sizeof(AttnRow) * T,
                                           cudaMemcpyHostToDevice, st));
    }
    QMA_CHECK_CUDA(cudaMemcpyAsync(w->tokens_dev, b->h_tok, sizeof(int) * T, cudaMemcpyHostToDevice, st));
    QMA_CHECK_CUDA(cudaMemcpyAsync(b->seq_dev, b->h_seq, sizeof(int) * T, cudaMemcpyHostToDevice, st));
    QMA_CHECK_CUDA(cudaMemcpyAsync(b->sp_dev, b->sp_host, sizeof(StepParams) * b->n_seq, cudaMemcpyHostToDevice, st));
    TRY(launch_embed(m->embd, m->embd_type, m->n_vocab, w->tokens_dev, b->sp_dev, T, w->x, st));
    for (int il = 0; il < n_layers; il++) {
        const LayerW &L = m->L[il];
        const int ld = L.in_rows;
        TRY(launch_rmsnorm_quant(w->x, L.attn_norm, T, EMBD, w->xq, w->xd, w->xs, st, layer_plan(m, il)));
        TRY(matvec(L.in_type, L.in_proj, EMBD, ld, T, w->xq, w->xd, w->xs, w->proj, st));
        if (is_attn(il) && rows_ok) {
            TRY(launch_attention_rows(b->rows_dev + size_t(il / 4) * b->t_step, T, ld, L.q_norm, L.k_norm, max_nchunk,
                                      max_nk, st));
            TRY(matvec(L.out_type, L.out_proj, WO_DIM, EMBD, T, w->xq, w->xd, w->xs, w->x2, st, w->x));
        } else if (is_attn(il)) {
            // a sequence past 16384 attended positions: the general kernels, one sequence at a time
            const int lay = il / 4;
            for (int t = 0; t < T; t++) {
                qma_cuda_state *c = b->seqs[seq_ids[t]];
                TRY(launch_qk_prep_append(w->proj + size_t(t) * ld, ld, L.q_norm, L.k_norm, c->rope, c->sp_dev, 1,
                                          c->qr, c->z, c->kv[lay], c->qf, c->sal, st));
                AttnArgs a;
                a.qr = c->qr; a.kv = c->kv[lay]; a.arena = c->arena[lay]; a.live = c->live_dev;
                a.sp = c->sp_dev; a.T = 1; a.nk_max = nk[t]; a.pv_chunk = attn_span(1, nk[t]);
                a.scores = c->scores; a.cmax = c->cmax; a.opart = c->opart; a.lpart = c->lpart;
                a.ml = c->ml; a.z = c->z;
                a.xq = w->xq + size_t(t) * WO_DIM;
                a.xd = w->xd + size_t(t) * (WO_DIM / 256);
                a.xs = w->xs + size_t(t) * (WO_DIM / 16);
                a.sal = c->sal + size_t(lay) * c->n_ctx;
                a.pin_sal = c->pin_sal + size_t(lay) * HCM_H_PIN;
                TRY(launch_attention(a, st));
                TRY(launch_salience(a, st));
            }
            TRY(matvec(L.out_type, L.out_proj, WO_DIM, EMBD, T, w->xq, w->xd, w->xs, w->x2, st, w->x));
        } else {
            const SeqTable conv{b->conv_tab + size_t(il) * b->n_seq, b->seq_dev};
            const SeqTable ssm{b->ssm_tab + size_t(il) * b->n_seq, b->seq_dev};
            TRY(launch_conv1d_seqs(w->proj, ld, L.conv1d, conv, T, w->conv_out, st));
            TRY(launch_gdn_seqs(w->conv_out, w->proj, ld, CONV_DIM + VAL_DIM, CONV_DIM + VAL_DIM + VHEADS, L.dt, L.a,
                                ssm, T, w->gdo, st));
            TRY(launch_gated_norm_quant(w->gdo, w->proj + CONV_DIM, ld, L.ssm_norm, T, w->xq, w->xd, w->xs, st));
            TRY(matvec(L.out_type, L.out_proj, VAL_DIM, EMBD, T, w->xq, w->xd, w->xs, w->x2, st, w->x));
        }
        // x = x2 + moe(rms_norm(x2) * post_norm)
        if (b->ep)
            TRY(qma_cuda_ep_moe_layer(b->ep, &b->ep_w[il], w->x2, T, w->x, nullptr, nullptr, st));
        else
            TRY(moe_layer(L.moe, w->x2, T, w->x, nullptr, nullptr, w->moe_scratch, st, false, nullptr));
    }
    if (hidden)
        for (int t = 0; t < T; t++)
            QMA_CHECK_CUDA(cudaMemcpyAsync(hidden + size_t(rows[t]) * EMBD, w->x + size_t(t) * EMBD,
                                           sizeof(float) * EMBD, cudaMemcpyDeviceToHost, st));
    if (n_layers == NLAYER && (logits_host || greedy)) {
        TRY(launch_rmsnorm_quant(w->x, m->out_norm, T, EMBD, w->xq, w->xd, w->xs, st));
        TRY(matvec(m->out_type, m->out, EMBD, m->n_vocab, T, w->xq, w->xd, w->xs, b->logits, st));
        if (greedy) {
            argmax_rows_kernel<<<T, 1024, 0, st>>>(b->logits, m->n_vocab, b->greedy_dev);
            QMA_CHECK_LAUNCH();
            QMA_CHECK_CUDA(cudaMemcpyAsync(b->h_tok, b->greedy_dev, sizeof(int) * T, cudaMemcpyDeviceToHost, st));
        }
        if (logits_host)
            for (int t = 0; t < T; t++)
                QMA_CHECK_CUDA(cudaMemcpyAsync(logits_host + rows[t] * logits_ld, b->logits + size_t(t) * m->n_vocab,
                                               sizeof(float) * m->n_vocab, cudaMemcpyDeviceToHost, st));
    }
    if (b->ep)
        TRY(qma_cuda_ep_sync(b->ep, st));      // bounded: a dead peer fails the step instead of hanging it
    else
        QMA_CHECK_CUDA(cudaStreamSynchronize(st));
    if (greedy)
        for (int t = 0; t < T; t++) greedy[rows[t]] = b->h_tok[t];
    for (int t = 0; t < T; t++) b->seqs[seq_ids[t]]->n_pos += 1;
#undef TRY
    return check_wait_timeouts();
}

// tokens[i] extends sequence seq_ids[i]; see qma_cuda_batch_eval.
static int batch_eval(qma_cuda_batch *b, const int *seq_ids, const int *tokens, int n, float *logits, int *greedy,
                      int n_layers, float *hidden) {
    qma_cuda_model *m = b->m;
    QMA_CHECK_CUDA(cudaSetDevice(m->device));
    std::vector<std::vector<int>> rows_of(b->n_seq);
    for (int i = 0; i < n; i++) rows_of[seq_ids[i]].push_back(i);
    std::vector<int> one_seq, one_tok, one_row;
    int rc;
    for (int q = 0; q < b->n_seq; q++) {
        const std::vector<int> &r = rows_of[q];
        if (r.empty()) continue;
        if (r.size() == 1) {
            one_seq.push_back(q);
            one_tok.push_back(tokens[r[0]]);
            one_row.push_back(r[0]);
            continue;
        }
        if (hidden || b->ep) {
            set_error("batch: %s takes one token per sequence (sequence %d has %d)",
                      hidden ? "the hidden-state entry point" : "an expert-parallel batch", q, int(r.size()));
            return QMA_CUDA_ERR_UNSUPPORTED;
        }
        // a prompt: the sequence's own chunked prefill, logits of its last token
        std::vector<int> toks(r.size());
        for (size_t k = 0; k < r.size(); k++) toks[k] = tokens[r[k]];
        const bool want = logits || greedy;
        if ((rc = eval(b->seqs[q], toks.data(), int(toks.size()), want ? b->h_row : nullptr, 0))) return rc;
        if (logits) memcpy(logits + int64_t(r.back()) * m->n_vocab, b->h_row, sizeof(float) * m->n_vocab);
        if (greedy) {
            int best = 0;
            for (int v = 1; v < m->n_vocab; v++)
                if (b->h_row[v] > b->h_row[best]) best = v;
            greedy[r.back()] = best;
        }
    }
    for (size_t i0 = 0; i0 < one_seq.size(); i0 += b->t_step) {
        const int T = int(std::min(one_seq.size() - i0, size_t(b->t_step)));
        if (b->ep && i0 > 0) {
            set_error("batch: an expert-parallel step takes at most %d sequences", b->t_step);
            return QMA_CUDA_ERR_UNSUPPORTED;
        }
        if ((rc = batch_step(b, one_seq.data() + i0, one_tok.data() + i0, T, logits, m->n_vocab, one_row.data() + i0,
                             greedy, n_layers, hidden)))
            return rc;
    }
    return QMA_CUDA_OK;
}

}  // namespace qma

extern "C" {

int qma_cuda_batch_create(qma_cuda_model *m, int n_seq, int n_ctx, qma_cuda_batch **out) {
    qma::clear_error();
    QMA_REQUIRE(m && out && n_seq >= 1 && n_seq <= 4096 && n_ctx > qma::HCM_SINK + 1,
                "qma_cuda_batch_create: bad arguments (n_seq %d, n_ctx %d)", n_seq, n_ctx);
    *out = nullptr;
    return qma::batch_create(m, n_seq, n_ctx, out);
}

int qma_cuda_batch_free(qma_cuda_batch *b) {
    qma::clear_error();
    return qma::batch_free(b);
}

qma_cuda_state *qma_cuda_batch_seq(qma_cuda_batch *b, int seq) {
    return b && seq >= 0 && seq < b->n_seq ? b->seqs[seq] : nullptr;
}

int qma_cuda_batch_n_seq(const qma_cuda_batch *b) { return b ? b->n_seq : 0; }

int qma_cuda_batch_set_ep(qma_cuda_batch *b, qma_cuda_ep *ep, const qma_cuda_moe_weights *shard) {
    qma::clear_error();
    QMA_REQUIRE(b && (!ep || shard), "qma_cuda_batch_set_ep: bad arguments");
    b->ep = ep;
    b->ep_w.clear();
    if (ep) b->ep_w.assign(shard, shard + qma::NLAYER);
    return QMA_CUDA_OK;
}

static int batch_args(const qma_cuda_batch *b, const int *seq_ids, const int *tokens, int n, const char *fn) {
    QMA_REQUIRE(b && seq_ids && tokens && n > 0, "%s: bad arguments", fn);
    for (int i = 0; i < n; i++) {
        QMA_REQUIRE(seq_ids[i] >= 0 && seq_ids[i] < b->n_seq, "%s: sequence id %d out of range (0..%d)", fn,
                    seq_ids[i], b->n_seq - 1);
        QMA_REQUIRE(tokens[i] >= 0 && tokens[i] < b->m->n_vocab, "%s: token %d out of range", fn, tokens[i]);
    }
    return QMA_CUDA_OK;
}

int qma_cuda_batch_eval(qma_cuda_batch *b, const int *seq_ids, const int *tokens, int n_tokens, float *logits,
                        int *greedy) {
    qma::clear_error();
    int rc;
    if ((rc = batch_args(b, seq_ids, tokens, n_tokens, "qma_cuda_batch_eval"))) return rc;
    return qma::batch_eval(b, seq_ids, tokens, n_tokens, logits, greedy, qma::NLAYER, nullptr);
}

int qma_cuda_batch_eval_hidden(qma_cuda_batch *b, const int *seq_ids, const int *tokens, int n_tokens, int n_layers,
                               float *hidden) {
    qma::clear_error();
    int rc;
    if ((rc = batch_args(b, seq_ids, tokens, n_tokens, "qma_cuda_batch_eval_hidden"))) return rc;
    QMA_REQUIRE(hidden && n_layers >= 0 && n_layers <= qma::NLAYER, "qma_cuda_batch_eval_hidden: bad arguments");
    return qma::batch_eval(b, seq_ids, tokens, n_tokens, nullptr, nullptr, n_layers, hidden);
}

const float *qma_cuda_batch_logits(const qma_cuda_batch *b) { return b ? b->logits : nullptr; }

}  // extern "C"
