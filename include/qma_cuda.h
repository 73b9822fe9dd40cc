/*
 * qma_cuda.h -- C ABI of the B200 (sm_100a) engine for qma's qwen35moe
 * model-engine hot path.
 *
 * Plain C: pointers, sizes and int status codes; no CUDA or C++ types in any
 * signature (a CUDA stream is passed as void*, NULL = the legacy default
 * stream).  Every entry point returns QMA_CUDA_OK (0) or a negative
 * qma_cuda_status; qma_cuda_last_error() describes the last failure on the
 * calling thread.  Nothing here ever calls exit().
 *
 * Pointer conventions: arguments documented "device" are CUDA device
 * pointers; "host" are ordinary host pointers.  Device buffers are read
 * with 16-byte vector loads: activation, weight and output buffers must be
 * 16-byte aligned and scratch buffers 256-byte aligned (cudaMalloc's
 * alignment satisfies both); a misaligned pointer is refused with
 * QMA_CUDA_ERR_INVALID.  Weight type ids are GGML's (qma.h:67-69):
 * 12 = Q4_K, 14 = Q6_K, plus 8 = Q8_0.
 *
 * Each entry point names the reference interface it replaces (qma sources,
 * file:line).
 */
#ifndef QMA_CUDA_H
#define QMA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QMA_CUDA_ABI_VERSION 2

typedef enum {
    QMA_CUDA_OK = 0,
    QMA_CUDA_ERR_INVALID = -1,     /* bad argument (null pointer, size, type) */
    QMA_CUDA_ERR_NOMEM = -2,       /* device or host allocation failed        */
    QMA_CUDA_ERR_CUDA = -3,        /* a CUDA runtime call failed              */
    QMA_CUDA_ERR_UNSUPPORTED = -4, /* shape or type the engine does not handle */
    QMA_CUDA_ERR_STATE = -5,       /* call out of order (e.g. no weights)     */
    QMA_CUDA_ERR_TIMEOUT = -6      /* a bounded device-side wait gave up      */
} qma_cuda_status;

#define QMA_TYPE_F32  0
#define QMA_TYPE_Q8_0 8
#define QMA_TYPE_Q4_K 12
#define QMA_TYPE_Q6_K 14

/* ---- library ---------------------------------------------------------- */
int         qma_cuda_abi_version(void);
/* Message of the last failed call on this thread ("" if none). */
const char *qma_cuda_last_error(void);
/* Select the CUDA device for this thread and check it is sm_100. */
int         qma_cuda_init(int device);

/* ---- Q8_K activation quantization --------------------------------------
 * Replaces qma_q8k_quant (qma.h:359, q8k.c:280; kernel quantize_row_q8k,
 * q8k.c:34-85).  x: device float [rows][n], n a multiple of 256.  Outputs
 * (device): xq int8 [rows][n], xd float [rows][n/256], xsum int16
 * [rows][n/16].  Bit-identical to the reference. */
int qma_cuda_q8k_quant(const float *x, int rows, int n, int8_t *xq, float *xd,
                       int16_t *xsum, void *stream);

/* ---- weight layout ------------------------------------------------------
 * The engine keeps Q4_K weights in GGUF block order (144 B blocks are
 * 16-byte aligned).  Q6_K (210 B blocks) and Q8_0 (34 B blocks) are not
 * 16-byte aligned, so they are repacked once, at load time, into planes per
 * matrix: Q6_K -> [ql rows*n/2][qh rows*n/4][scales rows*n/16][d rows*n/256
 * fp16]; Q8_0 -> [q rows*n][d rows*n/32 fp16].  Within each (row,
 * super-block) of the ql and qh planes the 16-byte chunks are permuted
 * (chunk c of segment s = row*(n/256)+sb at c ^ (s & 3) in ql, c ^ ((s>>1) & 1)
 * in qh) so that warps read them from shared memory without bank conflicts.
 * Byte-for-byte the same values; only their order changes (the reference's
 * own load-time repack is qma_align_model, gguf.c:674).  qma_cuda_packed_bytes() gives the size of a
 * packed matrix (equal to the GGUF size, rounded up to 16 per plane). */
size_t qma_cuda_packed_bytes(int wtype, int rows, int n);
/* src: device GGUF-layout matrix [rows][n]; dst: device packed buffer of
 * qma_cuda_packed_bytes() bytes (for Q4_K a plain copy). */
int qma_cuda_repack(int wtype, const void *src, int rows, int n, void *dst,
                    void *stream);

/* ---- super-block GEMV / small-batch GEMM --------------------------------
 * Replaces matmul / mm_worker (nn.c:261-345) and the row dot dispatch
 * qma_q8k_dot (qma.h:360, q8k.c:305-316) for Q4_K (dot_q4_K_q8k,
 * q8k.c:89-131), Q6_K (dot_q6_K_q8k, q8k.c:210-262) and Q8_0 (no reference
 * kernel; the reference rejects Q8_0 weights, gguf.c:272-287).
 *   out[t][r] = <dequant(W[r]), x_t>,  t < T, r < n_out
 * W: device packed weights (see above), n_out rows of n_in; the activation
 * is the Q8_K quantization of T rows (xq [T][n_in], xd [T][n_in/256], xsum
 * [T][n_in/16], device); out: device float [T][n_out].  n_in a multiple of
 * 256; any T >= 1.  fp32 results agree with the reference to ~1e-6
 * relative (the integer super-block partials are exact; only the fp32
 * summation order differs). */
int qma_cuda_matvec(int wtype, const void *W, int n_in, int n_out, int T,
                    const int8_t *xq, const float *xd, const int16_t *xsum,
                    float *out, void *stream);

/* Debug/parity: the exact int32 partial sums behind one token's row dots.
 * Q4_K / Q8_0: per 32-lane block, sum(q * xq) -> isum [n_out][n_in/32];
 * Q6_K: per super-block, sum_g scale_g * sum16((q - 32) * xq) -> isum
 * [n_out][n_in/256].  Matches the oracle's integer partials bit for bit. */
int qma_cuda_dot_partials(int wtype, const void *W, int n_in, int n_out,
                          const int8_t *xq, int32_t *isum, void *stream);

/* ---- synthetic weights ----------------------------------------------------
 * Random-init weights generated on the device, in GGUF block order: element
 * i of tensor `name` is a seeded Irwin-Hall(4) normal (a pure function of
 * seed, name and i; N(0, 0.02) for projections, 1 + N(0, 0.05) for norms,
 * negative for ssm_a), then quantized to `type` by the engine's quantizer.
 * Byte-identical to the CPU generator the parity tests use.  No reference
 * counterpart: the reference loads a GGUF file (qma_load, gguf.c:104). */
int qma_cuda_synth_tensor(const char *name, int type, uint64_t nelem, uint64_t seed,
                          void *dst, void *stream);

/* ---- model and sequence state (the qma_eval boundary) ---------------------
 * One tensor of a GGUF data section, the layout of tensor_t (qma.h:155-161):
 * ne[0] is the row length, ne[1] the rows, ne[2] the experts; `off` is the
 * byte offset in the data section.  Names are the reference's GGUF names
 * (gguf.c:308-345); types F32 / Q4_K / Q6_K / Q8_0. */
typedef struct {
    char     name[64];
    uint32_t type;
    int64_t  ne[3];
    uint64_t off;
    uint64_t nbytes;
} qma_cuda_tensor;

typedef struct qma_cuda_model qma_cuda_model;   /* device-resident weights */
typedef struct qma_cuda_state qma_cuda_state;   /* one sequence's state    */

/* Replaces qma_load (gguf.c:104-513) for the weights: uploads every tensor
 * the forward uses from a host data section (e.g. an mmapped GGUF) into HBM
 * in the engine's layout.  The hyper-parameters are qwen35moe's (qma.h:28-64);
 * n_vocab comes from token_embd.weight. */
int qma_cuda_model_load(int device, const qma_cuda_tensor *tensors, uint32_t n,
                        const void *host_data, uint64_t data_size, qma_cuda_model **out);
/* The parsing half of qma_load (gguf.c:104-316) on a GGUF v2/v3 file: the
 * tensor infos (host array of `cap` entries; *n_tensors receives the count,
 * so cap 0 sizes the array), the file offset of the aligned data section
 * and the tokenizer's token count (0 if the file has none).  Checks what
 * qma_load checks: magic, metadata, qwen35moe hyper-parameters (40 layers,
 * embedding 2048, heads 16/2, 64 rotary dims in sections 11/11/10, after
 * dropping the "qwen35moe." / "qwen35." key prefix), supported types, whole
 * blocks per row, every tensor inside the file.  Unlike qma_load it also
 * accepts Q8_0 tensors.  Host only: touches no device. */
int qma_cuda_gguf_scan(const char *path, qma_cuda_tensor *tensors, uint32_t cap,
                       uint32_t *n_tensors, uint64_t *data_offset, uint64_t *n_tokens);
/* qma_cuda_gguf_scan + qma_cuda_model_load on the file's data section
 * (mapped read-only, unmapped before returning). */
int qma_cuda_model_load_gguf(int device, const char *path, qma_cuda_model **out);
/* Same model with random-init weights generated on the device
 * (qma_cuda_synth_tensor per tensor): no host copy of the weights. */
int qma_cuda_model_synth(int device, const qma_cuda_tensor *tensors, uint32_t n,
                         uint64_t seed, qma_cuda_model **out);
/* The table check qma_cuda_model_load and qma_cuda_model_synth run before
 * allocating anything, on its own (host only, touches no device): every
 * tensor the forward uses is present with the shape the kernels are written
 * for (qma.h:28-64: e.g. ffn_gate_exps [2048][512][256], norm vectors of
 * 2048 / 256 / 128) and a supported type, and, with data_size > 0, lies in
 * a data section of data_size bytes.  The reference's qma_load checks the
 * hyper-parameters only (gguf.c:226-234) and trusts the shapes. */
int qma_cuda_model_check(const qma_cuda_tensor *tensors, uint32_t n, uint64_t data_size);
int qma_cuda_model_free(qma_cuda_model *m);
int qma_cuda_model_n_vocab(const qma_cuda_model *m);
/* ---- expert cache (ecache.h:87-123) ---------------------------------------
 * Every expert record of the model is HBM-resident, so the cache API keeps
 * its contract with no slot pool behind it: lookups never miss, records
 * never move, and the read-ahead calls become L2 residency hints (the
 * record's bytes requested into the 126 MB L2 ahead of the kernels that
 * read them). */
/* Replaces qma_ecache_get (ecache.h:95, ecache.c:414-498): device pointers
 * to the gate / up (Q4_K rows) and down (packed) matrices of expert
 * `expert` of layer `layer`.  Never fails for valid ids. */
int qma_cuda_ecache_get(const qma_cuda_model *m, int layer, int expert, const void **gate,
                        const void **up, const void **down);
/* Replaces qma_ecache_hint (ecache.h:119, ecache.c:399-410): the records
 * this layer is about to read, in order (host ids, n clamped to 64 as the
 * reference does).  Asks L2 for their bytes on `stream` (no wait, no
 * completion to observe); results never depend on it. */
int qma_cuda_ecache_hint(const qma_cuda_model *m, int layer, const int *ids, int n, void *stream);
/* Replaces qma_ecache_prefetch (ecache.h:123, ecache.c:378-397): a
 * speculative fill for a layer that has not routed yet; the same L2
 * request as a hint (nothing is pinned or counted here either). */
int qma_cuda_ecache_prefetch(const qma_cuda_model *m, int layer, const int *ids, int n, void *stream);
/* Replace qma_ecache_hold / qma_ecache_release (ecache.h:97-104,
 * ecache.c:500-520): hold is get() with the record claimed until the next
 * release; at most 64 holds between releases (QMA_CUDA_ERR_STATE past
 * that, where the reference returns NULL), and one release ends them all.
 * The pointers stay valid for the model's life either way (nothing is ever
 * evicted); the count keeps callers written against the reference's
 * contract honest.  qma_cuda_ecache_held returns the current count. */
int qma_cuda_ecache_hold(qma_cuda_model *m, int layer, int expert, const void **gate, const void **up,
                         const void **down);
int qma_cuda_ecache_release(qma_cuda_model *m);
int qma_cuda_ecache_held(const qma_cuda_model *m);

/* Replaces runstate_init_kv (nn.c:1878-1979) plus the HCM statics
 * (nn.c:912-937): KV ring of n_ctx slots (4-bit + 2-bit records, 240 B per
 * head and position), conv/ssm state, salience and heavy-hitter arena, all in
 * HBM, zero-initialised. */
int qma_cuda_state_create(qma_cuda_model *m, int n_ctx, qma_cuda_state **out);
int qma_cuda_state_free(qma_cuda_state *s);
int qma_cuda_state_n_pos(const qma_cuda_state *s);

/* Replaces qma_eval (qma.h:327-328, nn.c:2056-2308): runs n_tokens host
 * token ids through the model in chunks of up to 512, appending to the KV
 * ring and recurrent state; writes the last token's logits (n_vocab floats,
 * host) or, with logits_all, every token's (n_tokens * n_vocab).  logits may
 * be NULL. */
int qma_cuda_eval(qma_cuda_model *m, qma_cuda_state *s, const int *tokens, int n_tokens,
                  float *logits, int logits_all);
/* A single token with last-token logits replays the state's captured decode
 * step (a CUDA graph, the kernels qma_cuda_decode_greedy runs); with
 * QMA_CUDA_EAGER=1 in the environment every kernel is launched one by one
 * instead (same results; for debugging). */

/* Greedy decode kept on the device: feeds `token`, then each step's argmax
 * (lowest id on ties), for n_steps steps; step i's input token goes to
 * tokens_out[i] (host, optional) and the last step's logits to logits
 * (host, optional).  Each step is one replay of a captured CUDA graph; the
 * host intervenes only when the HCM live index is rebuilt (every 128
 * positions, nn.c:2074-2088).  The tokens are staged in pinned memory the
 * state owns and reach tokens_out when the call returns, so tokens_out may
 * be ordinary (pageable) memory without making the steps wait on the host. */
int qma_cuda_decode_greedy(qma_cuda_model *m, qma_cuda_state *s, int token, int n_steps,
                           int *tokens_out, float *logits);

/* Parity entry point: like qma_cuda_eval but runs only the first n_layers
 * layers (0..40; 0 = the embedding rows) and writes the hidden state after
 * them (T x 2048 floats, host); n_layers < 0 runs |n_layers| layers but
 * stops the last one after its mixer (GDN or attention) and residual,
 * before the MoE block.  The state advances as in qma_cuda_eval.  No reference
 * counterpart (the reference's closest hook is its QMA_DUMP_L1 debug dump,
 * nn.c:2253-2266). */
int qma_cuda_eval_hidden(qma_cuda_model *m, qma_cuda_state *s, const int *tokens,
                         int n_tokens, int n_layers, float *hidden);

/* ---- multi-sequence state ------------------------------------------------
 * n_seq sequences of n_ctx positions each, decoded together: the state of a
 * serving loop with many concurrent sequences (each sequence is a full
 * runstate_t, qma.h:254-276, with its own KV ring, recurrent state and HCM
 * tiers; the reference runs one sequence per process).  All sequences of a
 * batch run on one stream. */
typedef struct qma_cuda_batch qma_cuda_batch;
int qma_cuda_batch_create(qma_cuda_model *m, int n_seq, int n_ctx, qma_cuda_batch **out);
int qma_cuda_batch_free(qma_cuda_batch *b);
int qma_cuda_batch_n_seq(const qma_cuda_batch *b);
/* Sequence seq's own state (owned by the batch; qma_cuda_state_n_pos,
 * _save, _load and qma_cuda_eval work on it), or NULL. */
qma_cuda_state *qma_cuda_batch_seq(qma_cuda_batch *b, int seq);

/* qma_eval over several sequences (nn.c:2056-2308 per sequence):
 * tokens[i] is appended to sequence seq_ids[i] (0..n_seq-1), each
 * sequence's tokens in the order given.  The sequences given one token are
 * evaluated together in batched steps of up to 512 (one token per
 * sequence: the projections, router, experts and LM head run once over all
 * rows; the conv, gated-delta recurrence and attention of each row use its
 * own sequence's state); a sequence given several tokens (a prompt) is
 * prefilled through its own state first.  For the last token of each
 * sequence in the call, row i of logits (host [n_tokens][n_vocab],
 * optional) receives its logits and greedy[i] (host int [n_tokens],
 * optional) its argmax (lowest id on ties); other rows are left as they
 * are.  Sequences are independent: a sequence's results do not depend on
 * which others share its steps, as long as the steps have the same kind
 * of rows (16 or more, the grouped expert path). */
int qma_cuda_batch_eval(qma_cuda_batch *b, const int *seq_ids, const int *tokens, int n_tokens,
                        float *logits, int *greedy);
/* Parity entry point: one token per sequence, the first n_layers layers
 * (0..40) of a batched step; hidden (host [n_tokens][2048]) receives the
 * residual stream after them, row i for tokens[i].  The sequences advance
 * as in qma_cuda_batch_eval. */
int qma_cuda_batch_eval_hidden(qma_cuda_batch *b, const int *seq_ids, const int *tokens, int n_tokens,
                               int n_layers, float *hidden);
/* Device logits [rows][n_vocab] of the last batched step (row t for its
 * t-th sequence in ascending id order). */
const float *qma_cuda_batch_logits(const qma_cuda_batch *b);

/* ---- layer-level parity points -------------------------------------------
 * One layer's mixer (the half before the MoE block) on caller activations,
 * against the state's per-layer memory.  x: device float [n_tokens][2048],
 * the residual stream entering layer `layer` at the state's positions
 * n_pos .. n_pos + n_tokens - 1 (1..512 tokens); x_out: device float
 * [n_tokens][2048], the residual after the mixer (x + mixer(rms_norm(x) *
 * attn_norm)).  With advance != 0 the call also does what qma_eval does at
 * a chunk start and end for these positions: the heavy-hitter live index is
 * rebuilt first when one is due (nn.c:2074-2088), and n_pos moves on by
 * n_tokens afterwards; with advance 0 the state's position is left as is
 * (several layers may then be run for the same positions).  Synchronous on
 * the state's stream.
 *
 * qma_cuda_gdn_step replaces a gated-delta-net layer's mixer (nn.c:2164-2244:
 * projections, conv1d_layer nn.c:717-741, l2norm_skv nn.c:744-761,
 * gdn_worker nn.c:784-833, the gated norm and ssm_out); the layer's conv
 * and recurrent state in `s` advance.  qma_cuda_attn_decode replaces an
 * attention layer's (nn.c:2110-2163: projections, q/k norm, rope_imrope
 * nn.c:841-861, kv_append nn.c:1455-1509, attn_worker nn.c:1215-1446 over
 * the live index and the tail since the last rebuild, the gate and
 * attn_output); the K/V records are appended to the layer's ring and the
 * layer's salience is updated. */
int qma_cuda_gdn_step(qma_cuda_state *s, int layer, const float *x, int n_tokens, float *x_out, int advance);
/* n_tokens single-token steps of gated-delta-net layer `layer` in order,
 * each through the decode kernels (as qma_eval's decode runs the layer,
 * one token at a time), queued back to back with one synchronisation at
 * the end; the same arguments as qma_cuda_gdn_step with advance 1 and any
 * n_tokens.  (qma_cuda_gdn_step with n_tokens > 1 runs them as one prefill
 * chunk instead.) */
int qma_cuda_gdn_decode(qma_cuda_state *s, int layer, const float *x, int n_tokens, float *x_out);
int qma_cuda_attn_decode(qma_cuda_state *s, int layer, const float *x, int n_tokens, float *x_out, int advance);

/* Copies the 240-byte KV slot (q4 record + q2 record, kvq.h:22-29) of
 * attention layer `lay` (0..9, model layer 4*lay+3), head `head` (0, 1 = K
 * heads, 2, 3 = V heads) and ring slot `slot` to host `out`. */
int qma_cuda_state_kv_slot(const qma_cuda_state *s, int lay, int head, int slot, uint8_t *out);

/* The CUDA stream (cudaStream_t as void*) every call on this state runs on,
 * for callers that time or order work against it. */
void *qma_cuda_state_stream(const qma_cuda_state *s);
/* Kernel launches in one captured decode step (0 before the first capture),
 * and the bytes of device memory the state holds. */
int qma_cuda_state_stats(const qma_cuda_state *s, int *graph_kernels, uint64_t *state_bytes);
/* Session files in the reference's byte formats (agent.c:409-416 writes
 * them, agent.c:765-816 resumes from them): state_path as runstate_save
 * (nn.c:2011-2025: int32 n_pos, then per gated-delta-net layer the conv
 * state [8192][3] and recurrent state [32][128][128] floats), kv_path as
 * the KV slab file (nn.c:1878-1935: per attention layer [4 heads][n_ctx]
 * 240-byte records), salience_path as hcm_save (nn.c:1156-1171).  Any path
 * may be NULL to skip that file.  Load checks sizes and n_ctx, and leaves
 * the heavy-hitter bookkeeping as a fresh qma process has it after
 * hcm_load (nn.c:947-970, 1173-1209): tiers, live index and quantisation
 * scores cleared, the next rebuild at the first eval from position 128 on;
 * a salience file whose arena sections are missing or cut short loads with
 * no pinned entries, as hcm_load does. */
int qma_cuda_state_save(const qma_cuda_state *s, const char *state_path, const char *kv_path,
                        const char *salience_path);
int qma_cuda_state_load(qma_cuda_state *s, const char *state_path, const char *kv_path,
                        const char *salience_path);
/* Device pointer of the state's logits [n_vocab]: the last position's
 * logits after a single-token qma_cuda_eval (also with logits NULL, which
 * skips their copy to the host), after qma_cuda_decode_greedy, or after an
 * eval of several tokens that returned the last token's logits
 * (logits_all 0). */
const float *qma_cuda_state_logits(const qma_cuda_state *s);

/* ---- MoE FFN block ------------------------------------------------------
 * Replaces moe_ffn (nn.c:509-649) with its q8k expert kernels
 * (moe_expert_one_q8k nn.c:412-439, moe_shared_q8k nn.c:446-473, the
 * (token, expert) task loop moe_xpar_worker nn.c:652-707) and the residual
 * around it in qma_eval (nn.c:2246-2252):
 *   xn    = rms_norm(x2) * post_attention_norm
 *   top-8 = router(xn)  (fp32 logits, softmax, top-8, renormalise)
 *   x_out = x2 + sum_k w_k * down_k(q8k(silu(gate_k.xn) * up_k.xn))
 *              + sigmoid(shexp_gate . q8k(xn)) * down_sh(...)
 * Routing is bit-exact with the reference: every logit is known to within a
 * proven bound of the reference's sequential fp32 sum, and any expert whose
 * rank that bound cannot settle is recomputed in exactly the reference's
 * order.  All pointers are device pointers.  gate/up expert tensors are in
 * GGUF order ([256][512 rows][2048], Q4_K); down_exps holds one packed
 * [2048 rows][512] matrix per expert (qma_cuda_packed_bytes(down_type,
 * 2048, 512) bytes each, see qma_cuda_repack). */
typedef struct {
    const float *post_norm;        /* blk.N.post_attention_norm.weight [2048] */
    const float *gate_inp;         /* blk.N.ffn_gate_inp.weight [256][2048]    */
    const void  *gate_exps;        /* blk.N.ffn_gate_exps.weight, Q4_K         */
    const void  *up_exps;          /* blk.N.ffn_up_exps.weight, Q4_K           */
    const void  *down_exps;        /* blk.N.ffn_down_exps.weight, packed       */
    const float *gate_inp_shexp;   /* blk.N.ffn_gate_inp_shexp.weight [2048]   */
    const void  *gate_shexp;       /* blk.N.ffn_gate_shexp.weight, Q4_K        */
    const void  *up_shexp;         /* blk.N.ffn_up_shexp.weight, Q4_K          */
    const void  *down_shexp;       /* blk.N.ffn_down_shexp.weight, packed      */
    int down_type;                 /* QMA_TYPE_Q6_K or QMA_TYPE_Q4_K           */
    int down_shexp_type;
    /* Optional device float [256] added to the router's fp32 logits before
     * the softmax and the top-8 (l_e = fl(s_e + bias_e)); NULL for none.
     * qwen35moe has no router bias: this carries a serving workload's
     * per-expert prior (configs[4]'s Zipf prior), and the reference has no
     * counterpart. */
    const float *router_bias;
} qma_cuda_moe_weights;

/* The MoE block weights of model layer `layer` (0..39) as device pointers
 * into the model, in the form qma_cuda_moe_layer takes them: the resolved
 * per-layer ffn_* pointers and weight types of qma_t's layers[]
 * (qma.h:202-212) that moe_ffn reads (nn.c:509-649). */
int qma_cuda_model_moe_weights(const qma_cuda_model *m, int layer, qma_cuda_moe_weights *out);
/* Set (or, with NULL, clear) the router bias of layer `layer`'s MoE block
 * for every later evaluation with this model (device float [256], owned by
 * the caller, see qma_cuda_moe_weights.router_bias).  A state's captured
 * decode step keeps the pointer it was captured with: set the bias before
 * the first single-token evaluation of a state. */
int qma_cuda_model_set_router_bias(qma_cuda_model *m, int layer, const float *bias);

/* Device scratch bytes qma_cuda_moe_layer needs for T tokens. */
size_t qma_cuda_moe_scratch_bytes(int T);

/* x2: device [T][2048] residual stream after attention; x_out: device
 * [T][2048] (may alias x2).  sel (int32 [T][8]) and wts (float [T][8]),
 * optional device outputs, receive the routing in selection order.  scratch:
 * device buffer of qma_cuda_moe_scratch_bytes(T) bytes, owned by the caller;
 * calls that share a scratch buffer must not overlap on the GPU. */
int qma_cuda_moe_layer(const qma_cuda_moe_weights *w, const float *x2, int T,
                       float *x_out, int32_t *sel, float *wts, void *scratch,
                       size_t scratch_bytes, void *stream);

/* MoE FFN block that allocates nothing, for callers that cannot allocate
 * device memory: a host that has reserved the device's memory for its own
 * pools and lets no library allocate, or a step loop that cannot afford
 * cudaMalloc's implicit synchronisation.  This entry point has no
 * counterpart in the reference (the reference's moe_ffn mallocs host
 * buffers per call, nn.c:604).  Same computation and arguments as
 * qma_cuda_moe_layer minus the scratch, which lives in a fixed device array
 * inside the library (512 KB, held on every device that loads the library
 * until the process exits).  At most QMA_CUDA_MOE_NOALLOC_MAX_T tokens per
 * call; larger T is rejected with QMA_CUDA_ERR_INVALID.  The first call on
 * each device looks up that device's copy of the array (make it before any
 * stream capture on the device); the address is kept for the life of the
 * process, so after a cudaDeviceReset() of a device this entry point must
 * not be called on that device again.  All calls share the array: calls
 * that overlap on the GPU race and must not be issued. */
#define QMA_CUDA_MOE_NOALLOC_MAX_T 4
int qma_cuda_moe_layer_noalloc(const qma_cuda_moe_weights *w, const float *x2, int T,
                               float *x_out, int32_t *sel, float *wts, void *stream);

/* Diagnostics of the last routing on a scratch buffer: how many tokens
 * needed the exact sequential recompute (host int, read after the stream
 * is synchronised). */
int qma_cuda_moe_exact_fallbacks(const void *scratch, int T, int *count);

/* ---- sampling -------------------------------------------------------------
 * The first phase of qma's sampler on the GPU: repeat penalty, temperature
 * and the top-k candidates, replacing sampler_candidates (sampler.c:36-95)
 * so that k candidates instead of the logits cross to the host, where the
 * grammar mask and sampler_pick (sampler.c:100-134) run unchanged.
 * logits: device float [n_vocab] (e.g. qma_cuda_state_logits after a
 * single-token qma_cuda_eval with logits NULL); last_tokens: host, the
 * sampler's last n_last (0..64) tokens, oldest first; k = top_k clamped to
 * 1..min(n_vocab, max_k), max_k 1..QMA_CUDA_SAMPLE_MAX_K.  Outputs (host):
 * ids / lgs [k], the candidates' token ids and scaled logits, largest
 * first, and *n_out = k.  The scaled logits are bit-identical to the
 * reference's; candidates of equal value are ordered by token id (the
 * reference's qsort leaves that order unspecified).  When several tokens tie
 * exactly at the k-th value, the engine keeps the lowest ids among them; the
 * reference's min-heap (strict '>', sampler.c:74-85) keeps whichever tied
 * tokens its insertion order leaves, so the candidate SET can differ from
 * the reference's in that case only.  -0.0 and +0.0 rank as equal.  Blocks
 * until done.
 * Calls share a fixed device result array: they must not overlap. */
#define QMA_CUDA_SAMPLE_MAX_K 64
int qma_cuda_sample_candidates(const float *logits, int n_vocab, const int32_t *last_tokens,
                               int n_last, float repeat_penalty, float temp, int top_k, int max_k,
                               int32_t *ids, float *lgs, int *n_out, void *stream);

/* ---- expert parallelism --------------------------------------------------
 * The MoE block with the 256 experts of each layer sharded over N ranks (one
 * process per GPU; rank r owns experts r*256/N .. (r+1)*256/N - 1); the
 * router, the shared expert and the combine run where the token lives.  New
 * in this engine: the reference runs every expert of moe_ffn on one host
 * (its (token, expert) task loop, moe_xpar_worker nn.c:652-707, and the
 * ordered combine, nn.c:604-629, are what the exchange distributes).  Per
 * layer the ranks exchange, over NCCL point-to-point transfers, one Q8_K
 * row (2336 bytes) per (token, owning rank) and one fp32 [2048] down
 * projection per (token, expert) pair; the result is bit-identical to
 * qma_cuda_moe_layer on the same tokens (16 or more per call, its grouped
 * path).  The exchange has a fixed capacity: every rank sends every rank a
 * block of t_max rows (padding rows carry no expert) and gets each block's
 * slot partials back whole, so no count has to reach the host and a call
 * only queues work on the stream (a step of layers runs back to back and
 * can be captured in a CUDA graph); qma_cuda_ep_sync waits for it with the
 * handle's wall-clock limit.  QMA_CUDA_EP_COUNTED=1 in the environment
 * switches to exact-size transfers (the [N][2] counts all-gathered and read
 * on the host: one host synchronisation per call, fewer bytes on NVLink,
 * the same results). */
#define QMA_CUDA_EP_UID_BYTES 128
typedef struct qma_cuda_ep qma_cuda_ep;

/* Rank 0 makes the communicator id (host bytes [QMA_CUDA_EP_UID_BYTES]) and
 * hands it to every rank out of band. */
int qma_cuda_ep_unique_id(uint8_t *uid);

/* Collective over the N ranks: selects `device`, joins the communicator and
 * allocates the exchange buffers for up to t_max tokens per rank and call
 * (1..256, t_max * n_ranks <= 512). */
int qma_cuda_ep_init(int device, const uint8_t *uid, int rank, int n_ranks, int t_max,
                     qma_cuda_ep **out);
/* qma_cuda_ep_init with a wall-clock limit (milliseconds) on every host-side
 * wait of the handle: joining the communicator (a rank that never joins),
 * and each qma_cuda_ep_moe_layer's exchange.  Past the limit the
 * communicator is aborted (its peers' pending transfers fail rather than
 * wait) and the call returns QMA_CUDA_ERR_TIMEOUT; an aborted handle only
 * accepts qma_cuda_ep_free.  qma_cuda_ep_init takes the limit from
 * QMA_CUDA_EP_TIMEOUT_MS in the environment, default 300000.  The reference
 * has no counterpart (it runs on one host). */
int qma_cuda_ep_init_timeout(int device, const uint8_t *uid, int rank, int n_ranks, int t_max,
                             int timeout_ms, qma_cuda_ep **out);
int qma_cuda_ep_free(qma_cuda_ep *ep);

/* Collective: every rank calls it for the same layer, each with its own
 * tokens (0..t_max of them; a rank with none still serves its experts).
 * Arguments as qma_cuda_moe_layer, except that w->gate_exps, up_exps and
 * down_exps point at this rank's shard of the expert tables (its first
 * expert at offset 0) and the down projections must be Q6_K. */
int qma_cuda_ep_moe_layer(qma_cuda_ep *ep, const qma_cuda_moe_weights *w, const float *x2,
                          int T, float *x_out, int32_t *sel, float *wts, void *stream);

/* Route the MoE blocks of a batch's steps through the expert-parallel
 * exchange: shard points at 40 per-layer weight views (this rank's expert
 * shard, as qma_cuda_ep_moe_layer takes them).  Every rank then calls
 * qma_cuda_batch_eval in lockstep, one token for each of at most t_max
 * sequences per call (a data-parallel share of the sequences per rank);
 * ep NULL goes back to the local MoE block. */
int qma_cuda_batch_set_ep(qma_cuda_batch *b, qma_cuda_ep *ep, const qma_cuda_moe_weights *shard);

/* The stream's work done, exchanges with the other ranks included, waiting
 * at most the handle's wall-clock limit: past it, or on a communicator
 * error, the communicator is aborted (the peers' pending transfers fail)
 * and the call returns QMA_CUDA_ERR_TIMEOUT / QMA_CUDA_ERR_CUDA.  Use it
 * instead of a plain stream synchronisation after expert-parallel calls, so
 * that a rank that died does not hang the others. */
int qma_cuda_ep_sync(qma_cuda_ep *ep, void *stream);

/* Bytes this rank sent and received in its last qma_cuda_ep_moe_layer call
 * (itself included) and the rows its experts served (-1 with the
 * fixed-capacity exchange, whose count stays on the device). */
int qma_cuda_ep_stats(const qma_cuda_ep *ep, uint64_t *sent_bytes, uint64_t *recv_bytes,
                      int *rows_in);

#ifdef __cplusplus
}
#endif
#endif /* QMA_CUDA_H */
