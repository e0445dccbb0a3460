// llama.cu -- the Llama decoder on the device (cn_llama_*).
//
// Replaces LlamaModel (Models/Llama/LlamaModel.cs): the constructor's KV
// cache and scratch (:48-88) become device buffers, and Forward (:93-238)
// becomes one decode step enqueued on the context's stream:
//
//   embed -> per layer [RMSNorm, Q/K/V GEMVs, RoPE + KV store, GQA
//   attention, O GEMV, residual add, RMSNorm, gate/up GEMVs, SiLU*up,
//   down GEMV, residual add] -> final RMSNorm -> lm_head GEMV -> argmax
//
// The step reads token ids and positions from device memory, so one CUDA
// graph per batch size replays every step; the host only copies ids and
// positions in and logits / argmax out.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <new>
#include <vector>

#include "cn_common.cuh"
#include "cn_internal.h"
#include "ops.h"
#include "synth.cuh"

namespace cn {

enum { T_EMB = 0, T_OUT = 1, T_ONORM = 2 };
enum { L_ANORM = 0, L_Q, L_K, L_V, L_O, L_FNORM, L_GATE, L_UP, L_DOWN };
constexpr int kMaxBatch = 32;
// Prompts of at least m->prefill_min tokens (0: never) take the prefill
// matmul in cn_llama_forward: from kPrefillMin tokens by default.
constexpr int kPrefillMin = 16;  // the default and the smallest threshold cn_llama_set_prefill accepts

struct Step {
    bool built = false;
    std::vector<GemvOp> ops;  // [layer * 7 + {q,k,v,o,gate,up,down}], then lm_head
    // per layer: q/k/v and gate/up as single launches (n == 0: run apart)
    std::vector<GemvGroup> qkv, gu;
    AttnPlan ap;
    cudaGraphExec_t graph = nullptr;
};

}  // namespace cn

struct cn_llama {
    cn_ctx* ctx = nullptr;
    cn_llama_config cfg;
    std::vector<const cn_tensor*> t;
    int kvdim = 0;
    size_t kv_elem = 4;
    int64_t seq_stride = 0;  // KV elements per sequence slot
    void* kc = nullptr;
    void* vc = nullptr;
    float2* rope = nullptr;
    // x / x2: the residual stream, ping-ponged by the fused add + norm
    float *x = nullptr, *x2 = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr,
          *att = nullptr, *tmp = nullptr, *gate = nullptr, *up = nullptr, *logits = nullptr, *part = nullptr;
    int* attn_ctr = nullptr;  // [max_batch][n_kv] attention merge counters
    // tensor parallelism: this rank's share of heads, FFN rows and vocabulary
    cn_tp* tp = nullptr;
    int nh = 0, nkv = 0, qdim = 0, hid = 0, vocab_l = 0, tp_rank = 0;
    bool logits_owned = true;
    int *tokens = nullptr, *pos = nullptr, *amax = nullptr;
    int *h_tokens = nullptr, *h_pos = nullptr, *h_amax = nullptr;
    cn::GemvBufs gb{nullptr, nullptr, nullptr, nullptr, nullptr};
    size_t counter_bytes = 0;
    cn::Step steps[cn::kMaxBatch + 1];
    bool use_graph = true;
    // prompt processing (prefill) scratch for up to pf_cap tokens, allocated
    // on first use: residual stream, q/k/v, gate/up (fp32), the fp16
    // operand of the next matmul, fp16 copies of the new k/v rows, token ids
    int pf_cap = 0;
    int prefill_min = cn::kPrefillMin;  // cn_llama_forward's prefill threshold (0: sequential steps)
    // cn_llama_set_prefill_precision: 0 every prefill operand rounded to fp16
    // once; 1 the attention path (q/k/v and O projections, and the attention's
    // operands) on split (hi + lo fp16) operands; 2 (the default) every
    // projection split as well
    int prefill_split = 2;
    std::vector<float> pf_ws;  // split scales, [layer * 9 + slot] (projection slots; empty: not yet computed)
    // low halves: of the current matmul input rows, and of the new k and v
    // rows (fp32 caches)
    __half *pf_hl = nullptr, *pf_kl = nullptr, *pf_vl = nullptr;
    // norm_offset models: the RMSNorm weights + 1 ([layer][2][dim], then the
    // output norm), so every norm kernel runs unchanged
    float* normw = nullptr;
    float *pf_x = nullptr, *pf_q = nullptr, *pf_k = nullptr, *pf_v = nullptr, *pf_g = nullptr,
          *pf_u = nullptr;
    __half *pf_h = nullptr, *pf_kh = nullptr, *pf_vh = nullptr;
    int* pf_tok = nullptr;
    float* pf_xs = nullptr;  // [pf_cap] inverse row scales of pf_h
    // row-padded copies of projections whose rows are not 16-byte multiples
    // (pad_rows); they replace the caller's tensors in t
    std::vector<cn_tensor*> pads;
};

namespace cn {

static const cn_tensor* LT(const cn_llama* m, int l, int j) { return m->t[3 + 9 * l + j]; }

// RMSNorm weights: layer l's attn_norm (which 0) or ffn_norm (1), or the
// output norm (l < 0) -- the model's (w + 1) copies for norm_offset models.
static const float* norm_w(const cn_llama* m, int l, int which) {
    const int dim = m->cfg.dim;
    if (m->normw) return m->normw + (l < 0 ? (size_t)2 * m->cfg.n_layers * dim : ((size_t)2 * l + which) * dim);
    return static_cast<const float*>(l < 0 ? m->t[2]->d : LT(m, l, which ? 5 : 0)->d);
}

static int check_shape(const cn_tensor* t, const char* name, int64_t rows, int64_t cols,
                       bool f32_vector) {
    CN_CHECK(t != nullptr, CN_ERR_NOT_FOUND, "Tensor not found: %s", name);
    if (f32_vector) {
        CN_CHECK(t->type == CN_TYPE_F32 && t->rows * t->cols == cols, CN_ERR_INVALID_ARG,
                 "%s must be F32 with %lld values", name, (long long)cols);
        return CN_OK;
    }
    CN_CHECK(t->rows == rows && t->cols == cols, CN_ERR_INVALID_ARG,
             "%s is [%lld, %lld], expected [%lld, %lld]", name, (long long)t->rows,
             (long long)t->cols, (long long)rows, (long long)cols);
    return CN_OK;
}

static int dmalloc(void** p, size_t bytes, bool zero = true) {
    CN_CUDA(cudaMalloc(p, bytes < 256 ? 256 : bytes));
    if (zero) CN_CUDA(cudaMemset(*p, 0, bytes < 256 ? 256 : bytes));
    return CN_OK;
}

// Builds the per-batch GEMV ops and attention plan.
static int build_step(cn_llama* m, int B) {
    Step& st = m->steps[B];
    if (st.built) return CN_OK;
    const cn_llama_config& c = m->cfg;
    st.ops.clear();
    static const int wj[7] = {L_Q, L_K, L_V, L_O, L_GATE, L_UP, L_DOWN};
    for (int l = 0; l < c.n_layers; l++)
        for (int j = 0; j < 7; j++) {
            const cn_tensor* w = LT(m, l, wj[j]);
            GemvOp op;
            int rc = gemv_make(m->ctx, w->type, w->d, w->rows, w->cols, w->has_map ? &w->map : nullptr,
                               B, &op, w->row_bytes);
            if (rc) return rc;
            st.ops.push_back(op);
        }
    {
        const cn_tensor* w = m->t[T_OUT];
        GemvOp op;
        int rc = gemv_make(m->ctx, w->type, w->d, w->rows, w->cols, w->has_map ? &w->map : nullptr,
                           B, &op, w->row_bytes);
        if (rc) return rc;
        st.ops.push_back(op);
    }
    st.qkv.assign(c.n_layers, GemvGroup());
    st.gu.assign(c.n_layers, GemvGroup());
    for (int l = 0; l < c.n_layers; l++) {
        const GemvOp* o = &st.ops[(size_t)l * 7];
        if (gemv_group_make(m->ctx, o, 3, &st.qkv[l]) != CN_OK) st.qkv[l].n = 0;
        if (gemv_group_make(m->ctx, o + 4, 2, &st.gu[l]) != CN_OK) st.gu[l].n = 0;
    }
    set_error(CN_OK, "");
    int rc = attention_plan(m->nh, m->nkv, c.head_dim, c.ctx_len, B, m->ctx->sms,
                            c.kv_dtype == CN_KV_F16, &st.ap);
    if (rc) return rc;
    if ((rc = attention_prepare(st.ap))) return rc;
    st.built = true;
    return CN_OK;
}

// Tracks which activation vector (and in which form: Q4_K's pre-scaled
// second k-step and chunk sums, the plain one, or the tensor-core digit
// records) the fragment buffer holds.
struct PrepCache {
    const float* x = nullptr;
    int kind = -1;
    int nt = 0;
    int64_t cols = 0;
    void set(const float* x_, const GemvOp& op) {
        x = x_;
        kind = gemv_prep_kind(op);
        nt = op.plan.nt;
        cols = op.cols;
    }
    bool holds(const float* x_, const GemvOp& op) const {
        return x == x_ && kind == gemv_prep_kind(op) && nt == op.plan.nt && cols == op.cols;
    }
};

// A GEMV group (prep shared by its members, which read the same x).
static int gemv_g(cn_llama* m, cudaStream_t s, const GemvGroup& g, const float* x, float* const* y,
                  PrepCache& pc) {
    if (!pc.holds(x, g.ops[0])) {
        int rc = gemv_prep(s, m->ctx->sms, g.ops[0], x, m->gb);
        if (rc) return rc;
        pc.set(x, g.ops[0]);
    }
    return gemv_group_run(m->ctx, s, g, m->gb, y);
}

static int gemv(cn_llama* m, cudaStream_t s, const GemvOp& op, const float* x, float* y,
                PrepCache& pc, const XchgOut* xo = nullptr) {
    if (op.tma && !pc.holds(x, op)) {
        int rc = gemv_prep(s, m->ctx->sms, op, x, m->gb);
        if (rc) return rc;
        pc.set(x, op);
    }
    return gemv_run(m->ctx, s, op, x, m->gb, y, xo);
}

// Residual add of the pending delta (if any) into the stream, RMSNorm into
// xn, and the records of the GEMV that reads xn next, in one kernel.  *x is
// the current stream; with a delta it moves to the other buffer.
// (With tensor parallelism the pending delta is the exchange `xin`: the
// sum of every rank's partial output.)
static int norm(cn_llama* m, cudaStream_t s, const float* w, int B, const GemvOp& next, float** x,
                const float** delta, PrepCache& pc, const XchgIn* xin = nullptr) {
    const bool add = *delta || (xin && xin->size > 1);
    float* out = add ? (*x == m->x ? m->x2 : m->x) : nullptr;
    int rc = add_norm_prep(s, *x, xin && xin->size > 1 ? nullptr : *delta, out, w, m->xn,
                           m->cfg.dim, B, m->cfg.rms_eps, &next, m->gb, xin);
    if (rc) return rc;
    if (add) *x = out;
    *delta = nullptr;
    pc = PrepCache();
    if (next.tma && m->cfg.dim % 256 == 0) pc.set(m->xn, next);
    return CN_OK;
}

// Enqueues one decode step for B sequences (tokens/positions already in
// m->tokens / m->pos).
// Per-launch profiling of an eagerly enqueued step (cn_llama_profile_step):
// when set, every stage of enqueue_step records an event after its launches.
struct StepProfile {
    std::vector<cudaEvent_t> ev;
    std::vector<int> kind;
};
static StepProfile* g_prof = nullptr;
enum { P_START = 0, P_TP, P_EMBED, P_NORM, P_QKV, P_ROPE, P_ATTN, P_O, P_GATEUP, P_SILU, P_DOWN, P_HEAD,
       P_WAIT, P_ARGMAX, P_KINDS };
static int mark(cudaStream_t s, int kind) {
    if (!g_prof) return CN_OK;
    cudaEvent_t e;
    CN_CUDA(cudaEventCreate(&e));
    CN_CUDA(cudaEventRecord(e, s));
    g_prof->ev.push_back(e);
    g_prof->kind.push_back(kind);
    return CN_OK;
}

static int enqueue_step(cn_llama* m, int B, cudaStream_t s) {
    const cn_llama_config& c = m->cfg;
    Step& st = m->steps[B];
    const int hid = m->hid, kvd = m->kvdim, qdim = m->qdim;
    const cn_tensor* emb = m->t[T_EMB];
    // tensor parallelism: exchanges per step (O and down of every layer,
    // then lm_head); this step's sequence numbers derive from a counter the
    // first kernel bumps
    const bool tp = m->tp && m->tp->size > 1;
    const uint32_t uses = 2u * (uint32_t)c.n_layers + 1u;
    int rc;
    if (tp && ((rc = tp_step_launch(m->tp, s)) || (rc = mark(s, P_TP)))) return rc;
    rc = launch_embed(emb->type, emb->d, emb->row_bytes, m->tokens, c.vocab, c.dim, B, m->x,
                      m->ctx->dev_err, s);
    if (rc || (rc = mark(s, P_EMBED))) return rc;
    PrepCache pc;
    float* x = m->x;
    const float* delta = nullptr;  // output of the last projection, not yet added to x
    XchgIn xin;                    // tensor parallel: the exchange that delivers it
    for (int l = 0; l < c.n_layers; l++) {
        const GemvOp* ops = &st.ops[(size_t)l * 7];
        if ((rc = norm(m, s, norm_w(m, l, 0), B, ops[0], &x, &delta, pc, &xin)) || (rc = mark(s, P_NORM)))
            return rc;
        xin = XchgIn();
        if (st.qkv[l].n) {
            float* ys[3] = {m->q, m->k, m->v};
            if ((rc = gemv_g(m, s, st.qkv[l], m->xn, ys, pc))) return rc;
        } else {
            if ((rc = gemv(m, s, ops[0], m->xn, m->q, pc))) return rc;
            if ((rc = gemv(m, s, ops[1], m->xn, m->k, pc))) return rc;
            if ((rc = gemv(m, s, ops[2], m->xn, m->v, pc))) return rc;
        }
        if ((rc = mark(s, P_QKV))) return rc;
        AttnArgs aa;
        aa.q = m->q;
        aa.kcache = m->kc;
        aa.vcache = m->vc;
        aa.pos_dev = m->pos;
        aa.pos_host = 0;
        aa.batch = B;
        aa.n_heads = m->nh;
        aa.n_kv = m->nkv;
        aa.hd = c.head_dim;
        aa.q_stride = qdim;
        aa.cache_seq_stride = m->seq_stride;
        aa.cache_layer_off = (int64_t)l * c.ctx_len * kvd;
        aa.kv_f16 = c.kv_dtype == CN_KV_F16;
        aa.ctx_len = c.ctx_len;
        aa.part = m->part;
        aa.counters = m->attn_ctr;
        aa.out = m->att;
        aa.out_stride = qdim;
        aa.prep = prep_target(&ops[3], m->gb);
        // TensorMath.ApplyRoPE of q and the new k row, and the new k/v rows'
        // cache store, run inside the attention kernel
        aa.rope.k = m->k;
        aa.rope.v = m->v;
        aa.rope.rope = m->rope;
        aa.rope.kv_stride = kvd;
        aa.rope.on = 1;
        aa.rope.neox = c.rope_neox;
        if ((m->nh / m->nkv) * c.head_dim % 256 != 0) aa.prep.kind = -1;
        if ((rc = launch_attention(aa, st.ap, s)) || (rc = mark(s, P_ATTN))) return rc;
        pc = PrepCache();
        if (aa.prep.kind >= 0) pc.set(m->att, ops[3]);
        if (tp) {
            const XchgOut xo = tp_reduce_out(m->tp, uses, 2u * l, 0);
            if ((rc = gemv(m, s, ops[3], m->att, m->tmp, pc, &xo))) return rc;
            xin = tp_reduce_in(m->tp, uses, 2u * l, m->ctx->dev_err);
        } else {
            if ((rc = gemv(m, s, ops[3], m->att, m->tmp, pc))) return rc;
            delta = m->tmp;
        }
        if ((rc = mark(s, P_O))) return rc;
        if ((rc = norm(m, s, norm_w(m, l, 1), B, ops[4], &x, &delta, pc, &xin)) || (rc = mark(s, P_NORM)))
            return rc;
        xin = XchgIn();
        if (st.gu[l].n) {
            float* ys[2] = {m->gate, m->up};
            if ((rc = gemv_g(m, s, st.gu[l], m->xn, ys, pc))) return rc;
        } else {
            if ((rc = gemv(m, s, ops[4], m->xn, m->gate, pc))) return rc;
            if ((rc = gemv(m, s, ops[5], m->xn, m->up, pc))) return rc;
        }
        if ((rc = mark(s, P_GATEUP))) return rc;
        const PrepTarget spt = prep_target(&ops[6], m->gb);
        if ((rc = launch_silu_prep(m->gate, m->up, hid, B, spt, s, c.act_gelu)) || (rc = mark(s, P_SILU))) return rc;
        pc = PrepCache();
        if (spt.kind >= 0 && hid % 256 == 0) pc.set(m->gate, ops[6]);
        if (tp) {
            const XchgOut xo = tp_reduce_out(m->tp, uses, 2u * l + 1u, 1);
            if ((rc = gemv(m, s, ops[6], m->gate, m->tmp, pc, &xo))) return rc;
            xin = tp_reduce_in(m->tp, uses, 2u * l + 1u, m->ctx->dev_err);
        } else {
            if ((rc = gemv(m, s, ops[6], m->gate, m->tmp, pc))) return rc;
            delta = m->tmp;
        }
        if ((rc = mark(s, P_DOWN))) return rc;
    }
    const GemvOp& head = st.ops[(size_t)c.n_layers * 7];
    if ((rc = norm(m, s, norm_w(m, -1, 0), B, head, &x, &delta, pc, &xin)) || (rc = mark(s, P_NORM))) return rc;
    if (tp) {
        // lm_head rows of this rank go to every rank's logits (all-gather)
        const XchgOut xo = tp_gather_out(m->tp, m->vocab_l, uses, uses - 1u, 2);
        if ((rc = gemv(m, s, head, m->xn, m->tmp, pc, &xo)) || (rc = mark(s, P_HEAD))) return rc;
        if ((rc = xchg_wait(s, tp_gather_in(m->tp, uses, uses - 1u, m->ctx->dev_err))) || (rc = mark(s, P_WAIT)))
            return rc;
    } else {
        if ((rc = gemv(m, s, head, m->xn, m->logits, pc)) || (rc = mark(s, P_HEAD))) return rc;
    }
    if ((rc = launch_argmax(m->logits, c.vocab, B, m->amax, s))) return rc;
    return mark(s, P_ARGMAX);
}

// Builds the step for B sequences and, with graphs on, captures it once.
static int prepare_step(cn_llama* m, int B) {
    cudaStream_t s = m->ctx->stream;
    int rc = build_step(m, B);
    if (rc) return rc;
    Step& st = m->steps[B];
    if (!m->use_graph || st.graph) return CN_OK;
    {
        cudaGraph_t g = nullptr;
        CN_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        rc = enqueue_step(m, B, s);
        cudaError_t e = cudaStreamEndCapture(s, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (e != cudaSuccess) return cuda_error(e, "cudaStreamEndCapture");
        e = cudaGraphInstantiate(&st.graph, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) {
            st.graph = nullptr;
            return cuda_error(e, "cudaGraphInstantiate");
        }
    }
    return CN_OK;
}

static int run_step(cn_llama* m, int B) {
    int rc = prepare_step(m, B);
    if (rc) return rc;
    if (!m->use_graph) return enqueue_step(m, B, m->ctx->stream);
    CN_CUDA(cudaGraphLaunch(m->steps[B].graph, m->ctx->stream));
    return CN_OK;
}

static int check_dev_err_reset(cn_llama* m) {
    uint32_t e = 0;
    CN_CUDA(cudaMemcpy(&e, m->ctx->dev_err, 4, cudaMemcpyDeviceToHost));
    if (!e) return CN_OK;
    CN_CUDA(cudaMemset(m->ctx->dev_err, 0, 4));
    CN_CUDA(cudaMemset(m->gb.counters, 0, m->counter_bytes));
    if (e & kErrTimeout) return set_error(CN_ERR_TIMEOUT, "a kernel gave up waiting (0x%x)", e);
    return set_error(CN_ERR_INVALID_ARG, "token id or position out of range (0x%x)", e);
}

// Fills the cache's first npos positions with the generator's values of the
// WHOLE model's cache ([layers*ctx, kvd_full]): a tensor-parallel rank holds
// columns [col0, col0 + kvd) of it.
__global__ void kv_synth_kernel(uint64_t seed, int layers, int npos, int ctx, int kvd, int kvd_full, int col0,
                                int f16, void* out) {
    const int64_t n = (int64_t)layers * npos * kvd;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t l = i / ((int64_t)npos * kvd);
        int64_t r = i % ((int64_t)npos * kvd);
        int64_t idx = (l * ctx + r / kvd) * kvd + r % kvd;
        int64_t g = (l * ctx + r / kvd) * kvd_full + col0 + r % kvd;
        float v = synth::normal_elem(seed, (uint64_t)g);
        if (f16) reinterpret_cast<__half*>(out)[idx] = __float2half_rn(v);
        else reinterpret_cast<float*>(out)[idx] = v;
    }
}

// Q6_K projections whose rows are not whole 16-byte units (an inner
// dimension that is not a multiple of 2048: Llama-2-7B's ffn_down at 11008
// columns has 9030-byte rows) cannot be tiled by TMA.  The model keeps a
// copy of each such matrix with every row padded to the next 16-byte
// boundary (zero bytes after the row's blocks, never decoded) and puts it in
// place of the caller's tensor, so the decode GEMV and the prefill matmul
// both take their tiled paths.  The split-variant scale is taken from the
// caller's packed tensor.
static int pad_rows(cn_llama* m) {
    cudaStream_t s = m->ctx->stream;
    for (size_t i = 3; i < m->t.size(); i++) {
        const int j = (int)((i - 3) % 9);
        const cn_tensor* w = m->t[i];
        if (j == L_ANORM || j == L_FNORM || w->type != CN_TYPE_Q6_K || w->row_bytes % 16 == 0 || w->cols % 256)
            continue;
        cn_tensor* p = new (std::nothrow) cn_tensor();
        CN_CHECK(p, CN_ERR_OOM, "host allocation failed");
        *p = *w;
        p->d = nullptr;
        p->owns = true;
        p->has_map = false;
        p->row_bytes = (w->row_bytes + 15) / 16 * 16;
        p->bytes = p->row_bytes * (uint64_t)w->rows;
        cudaError_t e = cudaMalloc(&p->d, p->bytes);
        if (e != cudaSuccess) {
            delete p;
            return cuda_error(e, "padded weight copy");
        }
        m->pads.push_back(p);
        e = cudaMemsetAsync(p->d, 0, p->bytes, s);
        if (e == cudaSuccess)
            e = cudaMemcpy2DAsync(p->d, p->row_bytes, w->d, w->row_bytes, w->row_bytes, (size_t)w->rows,
                                  cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return cuda_error(e, "padded weight copy");
        if (encode_weight_map(p->type, p->d, p->rows, p->row_bytes, &p->map) == CN_OK) p->has_map = true;
        set_error(CN_OK, "");
        cn_tensor packed = *w;
        float ws = 0.f;
        int rc = matmul_split_scale(&packed, s, &ws);
        if (rc) return rc;
        p->split_scale = ws;
        m->t[i] = p;
    }
    CN_CUDA(cudaStreamSynchronize(s));
    return CN_OK;
}

static void free_model(cn_llama* m) {
    for (int b = 0; b <= kMaxBatch; b++)
        if (m->steps[b].graph) cudaGraphExecDestroy(m->steps[b].graph);
    if (!m->logits_owned) m->logits = nullptr;
    void* bufs[] = {m->kc, m->vc, m->rope, m->x, m->x2, m->attn_ctr, m->xn, m->q, m->k, m->v, m->att, m->tmp,
                    m->gate, m->up, m->logits, m->part, m->tokens, m->pos, m->amax,
                    m->gb.xfrag, m->gb.xsum, m->gb.partials, m->gb.counters, m->gb.xinv,
                    m->pf_x, m->pf_q, m->pf_k, m->pf_v, m->pf_g, m->pf_u, m->pf_h, m->pf_kh, m->pf_vh,
                    m->pf_tok, m->pf_xs, m->pf_hl, m->pf_kl, m->pf_vl, m->normw};
    for (void* p : bufs) cudaFree(p);
    for (cn_tensor* p : m->pads) {
        cudaFree(p->d);
        delete p;
    }
    cudaFreeHost(m->h_tokens);
    cudaFreeHost(m->h_pos);
    cudaFreeHost(m->h_amax);
    delete m;
}

// ---- prefill: n tokens through the decoder at once (tcgen05 matmul) ----------

// A weight tensor's TMA descriptor, or null (the matmul then encodes one).
static const CUtensorMap* wmap(const cn_tensor* t) { return t->has_map ? &t->map : nullptr; }

// Whether the model's projections can run on the prefill matmul (Q4_0, Q4_K
// or Q6_K -- Q6_K rows that are not 16-byte multiples were padded by
// pad_rows --, inner dimensions multiples of 256, one GPU).
static bool prefill_supported(const cn_llama* m) {
    if (m->tp && m->tp->size > 1) return false;
    const cn_llama_config& c = m->cfg;
    if (c.dim % 256 != 0 || c.hidden_dim % 256 != 0 || (c.head_dim != 64 && c.head_dim != 128))
        return false;
    for (int l = 0; l < c.n_layers; l++)
        for (int j : {L_Q, L_K, L_V, L_O, L_GATE, L_UP, L_DOWN}) {
            const cn_tensor* t = LT(m, l, j);
            if (!matmul_type_ok(t->type) || (t->type == CN_TYPE_Q6_K && t->row_bytes % 16 != 0)) return false;
        }
    return true;
}

// One launch group of layer l's projections (q/k/v, o, gate/up or down, all
// with inner dimension K) on the fp16 rows m->pf_h, whose inverse row scales
// are m->pf_xs when `scaled`: one matmul launch per run of matrices of the
// same weight type (a single launch when the group's types agree).  The first
// `nsplit` matrices run the split variant (low halves of the rows in
// m->pf_hl, weight scales m->pf_ws), the rest the fp16 one.  With
// count_only, returns the number of launches instead.
static int mm_group(cn_llama* m, int l, int nmat, const int* slots, const int64_t* rows, int64_t K, int n,
                    float* const* y, const int64_t* ldy, bool accumulate, bool scaled, bool count_only = false,
                    int nsplit = 0) {
    int launches = 0;
    for (int i = 0; i < nmat;) {
        const int type = LT(m, l, slots[i])->type;
        const bool split = i < nsplit;
        int j = i + 1;
        while (j < nmat && LT(m, l, slots[j])->type == type && (j < nsplit) == split) j++;
        launches++;
        if (!count_only) {
            const void* w[3];
            const CUtensorMap* wm[3];
            float ws[3] = {1.f, 1.f, 1.f};
            for (int k = i; k < j; k++) {
                w[k - i] = LT(m, l, slots[k])->d;
                wm[k - i] = wmap(LT(m, l, slots[k]));
                if (split) ws[k - i] = m->pf_ws[(size_t)l * 9 + slots[k]];
            }
            int rc = matmul_quant(m->ctx->stream, m->ctx->dev_err, type, j - i, w, wm, rows + i, K, m->pf_h,
                                  scaled ? m->pf_xs : nullptr, n, y + i, ldy + i, accumulate,
                                  split ? m->pf_hl : nullptr, split ? ws : nullptr);
            if (rc) return rc;
        }
        i = j;
    }
    return count_only ? launches : CN_OK;
}

static const int kSlotsQKV[3] = {L_Q, L_K, L_V}, kSlotsO[1] = {L_O}, kSlotsGU[2] = {L_GATE, L_UP},
                 kSlotsDown[1] = {L_DOWN};

// Every projection's split-variant expansion scale, computed once
// (synchronises the stream; cached in the tensors as well).
static int prefill_scales(cn_llama* m) {
    if (!m->pf_ws.empty()) return CN_OK;
    const int L = m->cfg.n_layers;
    std::vector<float> ws(9 * (size_t)L, 1.f);
    for (int l = 0; l < L; l++)
        for (int j : {L_Q, L_K, L_V, L_O, L_GATE, L_UP, L_DOWN}) {
            int rc = matmul_split_scale(const_cast<cn_tensor*>(LT(m, l, j)), m->ctx->stream, &ws[9 * (size_t)l + j]);
            if (rc) return rc;
        }
    m->pf_ws.swap(ws);
    return CN_OK;
}

// Matrices of each projection group that run the split variant at the
// model's prefill precision: {q/k/v, o, gate/up, down}.
static void split_counts(const cn_llama* m, int (&ns)[4]) {
    const int p = m->prefill_split;
    ns[0] = p >= 1 ? 3 : 0;
    ns[1] = p >= 1 ? 1 : 0;
    ns[2] = p >= 2 ? 2 : 0;
    ns[3] = p >= 2 ? 1 : 0;
}

static int prefill_reserve(cn_llama* m, int n) {
    if (n <= m->pf_cap) return CN_OK;
    CN_CUDA(cudaStreamSynchronize(m->ctx->stream));
    void* old[] = {m->pf_x, m->pf_q, m->pf_k, m->pf_v, m->pf_g, m->pf_u, m->pf_h, m->pf_kh, m->pf_vh,
                   m->pf_tok, m->pf_xs, m->pf_hl, m->pf_kl, m->pf_vl};
    for (void* p : old) cudaFree(p);
    m->pf_x = m->pf_q = m->pf_k = m->pf_v = m->pf_g = m->pf_u = nullptr;
    m->pf_h = m->pf_kh = m->pf_vh = m->pf_hl = m->pf_kl = m->pf_vl = nullptr;
    m->pf_tok = nullptr;
    m->pf_xs = nullptr;
    m->pf_cap = 0;
    const cn_llama_config& c = m->cfg;
    const size_t N = (size_t)n;
    const size_t hmax = (size_t)(c.hidden_dim > c.dim ? c.hidden_dim : c.dim);
    int rc;
    if ((rc = dmalloc((void**)&m->pf_x, N * c.dim * 4, false)) ||
        (rc = dmalloc((void**)&m->pf_q, N * m->qdim * 4, false)) ||
        (rc = dmalloc((void**)&m->pf_k, N * m->kvdim * 4, false)) ||
        (rc = dmalloc((void**)&m->pf_v, N * m->kvdim * 4, false)) ||
        (rc = dmalloc((void**)&m->pf_g, N * c.hidden_dim * 4, false)) ||
        (rc = dmalloc((void**)&m->pf_u, N * c.hidden_dim * 4, false)) ||
        (rc = dmalloc((void**)&m->pf_h, N * hmax * 2, false)) ||
        (rc = dmalloc((void**)&m->pf_kh, N * m->kvdim * 2, false)) ||
        (rc = dmalloc((void**)&m->pf_vh, N * m->kvdim * 2, false)) ||
        (rc = dmalloc((void**)&m->pf_tok, N * 4, false)) ||
        (rc = dmalloc((void**)&m->pf_xs, N * 4, false)) ||
        (rc = dmalloc((void**)&m->pf_hl, N * hmax * 2, false)) ||
        (rc = dmalloc((void**)&m->pf_kl, N * m->kvdim * 2, false)) ||
        (rc = dmalloc((void**)&m->pf_vl, N * m->kvdim * 2, false)))
        return rc;
    m->pf_cap = n;
    return CN_OK;
}

// Runs the hidden states m->pf_x [n][dim] (positions pos..pos+n-1 of
// sequence slot 0) through every layer, in place; the layers' K/V rows land
// in the cache.  Per layer: RmsNorm -> q/k/v matmul (one launch) -> RoPE and
// cache store -> causal attention -> O matmul added into the residual ->
// RmsNorm -> gate/up matmul (one launch) -> SiLU * up -> down matmul added
// into the residual (LlamaModel.Forward, Models/Llama/LlamaModel.cs:93-238,
// for n tokens at once).
static int prefill_layers(cn_llama* m, int n, int pos) {
    const cn_llama_config& c = m->cfg;
    cudaStream_t s = m->ctx->stream;
    const int qd = m->qdim, kvd = m->kvdim, hid = c.hidden_dim;
    const bool kv16 = c.kv_dtype == CN_KV_F16;
    int ns[4];
    split_counts(m, ns);
    const bool attn_split = ns[0] > 0, ffn_split = ns[2] > 0;
    __half* kl = attn_split && !kv16 ? m->pf_kl : nullptr;
    __half* vl = attn_split && !kv16 ? m->pf_vl : nullptr;
    int rc;
    if ((attn_split || ffn_split) && (rc = prefill_scales(m))) return rc;
    for (int l = 0; l < c.n_layers; l++) {
        const int64_t cache_off = (int64_t)l * c.ctx_len * kvd;  // sequence slot 0
        if ((rc = prefill_norm(s, m->pf_x, norm_w(m, l, 0), m->pf_h, m->pf_xs, c.dim, n,
                               c.rms_eps, attn_split ? m->pf_hl : nullptr)))
            return rc;
        {
            const int64_t rows[3] = {qd, kvd, kvd};
            float* y[3] = {m->pf_q, m->pf_k, m->pf_v};
            if ((rc = mm_group(m, l, 3, kSlotsQKV, rows, c.dim, n, y, rows, false, true, false, ns[0]))) return rc;
        }
        if ((rc = prefill_rope(s, m->pf_q, m->pf_k, m->pf_v, m->rope, pos, n, qd, kvd, c.head_dim, m->kc, m->vc,
                               cache_off, kv16, m->pf_kh, m->pf_vh, kl, vl, c.rope_neox)))
            return rc;
        if ((rc = prefill_attention(s, m->pf_q, qd, m->kc, m->vc, kv16, cache_off, m->nh, m->nkv, c.head_dim, n,
                                    pos, m->pf_kh, m->pf_vh, m->pf_h, qd, attn_split, kl, vl,
                                    attn_split ? m->pf_hl : nullptr)))
            return rc;
        {
            const int64_t rows = c.dim;
            if ((rc = mm_group(m, l, 1, kSlotsO, &rows, qd, n, &m->pf_x, &rows, true, false, false, ns[1]))) return rc;
        }
        if ((rc = prefill_norm(s, m->pf_x, norm_w(m, l, 1), m->pf_h, m->pf_xs, c.dim, n,
                               c.rms_eps, ffn_split ? m->pf_hl : nullptr)))
            return rc;
        {
            const int64_t rows[2] = {hid, hid};
            float* y[2] = {m->pf_g, m->pf_u};
            if ((rc = mm_group(m, l, 2, kSlotsGU, rows, c.dim, n, y, rows, false, true, false, ns[2]))) return rc;
        }
        if ((rc = prefill_silu(s, m->pf_g, m->pf_u, m->pf_h, m->pf_xs, hid, n, ffn_split ? m->pf_hl : nullptr,
                               c.act_gelu)))
            return rc;
        {
            const int64_t rows = c.dim;
            if ((rc = mm_group(m, l, 1, kSlotsDown, &rows, hid, n, &m->pf_x, &rows, true, true, false, ns[3])))
                return rc;
        }
    }
    return CN_OK;
}

// Kernels one prefill_layers call launches: 6 per layer besides the matmuls,
// and one matmul per same-type run of each projection group (4 per layer
// when every group's types agree).
static int prefill_kernels(const cn_llama* m) {
    cn_llama* mm = const_cast<cn_llama*>(m);
    const int64_t r[3] = {0, 0, 0};
    float* y[3] = {nullptr, nullptr, nullptr};
    int k = 0, ns[4];
    split_counts(m, ns);
    for (int l = 0; l < m->cfg.n_layers; l++)
        k += 6 + mm_group(mm, l, 3, kSlotsQKV, r, 0, 0, y, r, false, false, true, ns[0]) +
             mm_group(mm, l, 1, kSlotsO, r, 0, 0, y, r, false, false, true, ns[1]) +
             mm_group(mm, l, 2, kSlotsGU, r, 0, 0, y, r, false, false, true, ns[2]) +
             mm_group(mm, l, 1, kSlotsDown, r, 0, 0, y, r, false, false, true, ns[3]);
    return k;
}

}  // namespace cn

using namespace cn;

extern "C" {

static int create_model(cn_ctx* ctx, const cn_llama_config* cfg, cn_tensor* const* tensors, int n_tensors,
                        cn_tp* tp, cn_llama** out) {
    CN_CHECK(ctx && cfg && tensors && out, CN_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    const cn_llama_config c = *cfg;
    const int W = tp ? tp->size : 1, R = tp ? tp->rank : 0;
    CN_CHECK(c.n_layers > 0 && c.dim > 0 && c.hidden_dim > 0 && c.n_heads > 0 && c.n_kv_heads > 0 &&
                 c.head_dim > 0 && c.vocab > 0 && c.ctx_len > 0,
             CN_ERR_INVALID_ARG, "non-positive hyper-parameter");
    CN_CHECK(c.n_heads * c.head_dim == c.dim, CN_ERR_INVALID_ARG,
             "n_heads * head_dim (%d) != dim (%d)", c.n_heads * c.head_dim, c.dim);
    CN_CHECK(c.n_heads % c.n_kv_heads == 0, CN_ERR_INVALID_ARG, "n_heads %% n_kv_heads != 0");
    CN_CHECK(c.max_batch >= 1 && c.max_batch <= kMaxBatch, CN_ERR_INVALID_ARG,
             "max_batch %d outside [1, %d]", c.max_batch, kMaxBatch);
    CN_CHECK(c.kv_dtype == CN_KV_F32 || c.kv_dtype == CN_KV_F16, CN_ERR_INVALID_ARG,
             "bad kv_dtype %d", c.kv_dtype);
    CN_CHECK((c.rope_neox == 0 || c.rope_neox == 1) && (c.act_gelu == 0 || c.act_gelu == 1) &&
                 (c.norm_offset == 0 || c.norm_offset == 1),
             CN_ERR_INVALID_ARG, "rope_neox, act_gelu and norm_offset are 0 or 1");
    CN_CHECK(!c.rope_neox || c.head_dim % 8 == 0, CN_ERR_UNSUPPORTED, "split-half RoPE needs head_dim %% 8 == 0");
    CN_CHECK(n_tensors == CN_LLAMA_TENSORS(c.n_layers), CN_ERR_INVALID_ARG,
             "expected %d tensors, got %d", CN_LLAMA_TENSORS(c.n_layers), n_tensors);
    if (tp) {
        CN_CHECK(tp->ctx == ctx && (W == 1 || tp->connected), CN_ERR_INVALID_ARG,
                 "tensor-parallel group not connected on this context");
        CN_CHECK(c.n_kv_heads % W == 0 && c.hidden_dim % W == 0 && c.vocab % W == 0, CN_ERR_INVALID_ARG,
                 "kv heads, hidden_dim and vocab must divide by the group size %d", W);
        CN_CHECK(tp->dim == c.dim && tp->vocab == c.vocab && tp->max_batch >= c.max_batch, CN_ERR_INVALID_ARG,
                 "tensor-parallel buffers sized for another model");
    }
    // this rank's share (the whole model when W == 1)
    const int nh = c.n_heads / W, nkv = c.n_kv_heads / W, hid = c.hidden_dim / W, vocab_l = c.vocab / W;
    const int qdim = nh * c.head_dim;
    const int kvd = nkv * c.head_dim;
    int rc;
    if ((rc = check_shape(tensors[T_EMB], "token_embd.weight", c.vocab, c.dim, false))) return rc;
    if ((rc = check_shape(tensors[T_OUT], "output.weight", vocab_l, c.dim, false))) return rc;
    if ((rc = check_shape(tensors[T_ONORM], "output_norm.weight", 1, c.dim, true))) return rc;
    for (int l = 0; l < c.n_layers; l++) {
        const cn_tensor* const* L = tensors + 3 + 9 * l;
        if ((rc = check_shape(L[L_ANORM], "attn_norm.weight", 1, c.dim, true))) return rc;
        if ((rc = check_shape(L[L_Q], "attn_q.weight", qdim, c.dim, false))) return rc;
        if ((rc = check_shape(L[L_K], "attn_k.weight", kvd, c.dim, false))) return rc;
        if ((rc = check_shape(L[L_V], "attn_v.weight", kvd, c.dim, false))) return rc;
        if ((rc = check_shape(L[L_O], "attn_output.weight", c.dim, qdim, false))) return rc;
        if ((rc = check_shape(L[L_FNORM], "ffn_norm.weight", 1, c.dim, true))) return rc;
        if ((rc = check_shape(L[L_GATE], "ffn_gate.weight", hid, c.dim, false))) return rc;
        if ((rc = check_shape(L[L_UP], "ffn_up.weight", hid, c.dim, false))) return rc;
        if ((rc = check_shape(L[L_DOWN], "ffn_down.weight", c.dim, hid, false))) return rc;
    }
    for (int i = 0; i < n_tensors; i++)
        CN_CHECK(tensors[i]->ctx == ctx, CN_ERR_INVALID_ARG, "tensor %d belongs to another context", i);
    {
        AttnPlan ap;
        if ((rc = attention_plan(nh, nkv, c.head_dim, c.ctx_len, c.max_batch, ctx->sms,
                                 c.kv_dtype == CN_KV_F16, &ap)))
            return rc;
    }

    cudaSetDevice(ctx->device);
    cn_llama* m = new (std::nothrow) cn_llama();
    CN_CHECK(m, CN_ERR_OOM, "host allocation failed");
    m->ctx = ctx;
    m->cfg = c;
    m->t.assign(tensors, tensors + n_tensors);
    m->tp = (tp && W > 1) ? tp : nullptr;
    m->tp_rank = R;
    m->nh = nh;
    m->nkv = nkv;
    m->qdim = qdim;
    m->hid = hid;
    m->vocab_l = vocab_l;
    m->kvdim = kvd;
    m->kv_elem = c.kv_dtype == CN_KV_F16 ? 2 : 4;
    m->seq_stride = (int64_t)c.n_layers * c.ctx_len * kvd;
    m->use_graph = getenv("CN_NO_GRAPH") == nullptr;
    const int B = c.max_batch;
    const size_t kvbytes = (size_t)B * m->seq_stride * m->kv_elem;
    auto fail = [&](int code) {
        free_model(m);
        return code;
    };
    if ((rc = dmalloc(&m->kc, kvbytes)) || (rc = dmalloc(&m->vc, kvbytes))) return fail(rc);
    // RoPE table, computed with the reference's formula and the host libm
    // (TensorMath.ApplyRoPE, TensorMath.cs:418-432).
    {
        const int half = c.head_dim / 2;
        std::vector<float2> tab((size_t)c.ctx_len * half);
        const float neg_log_base = -logf(c.rope_base);
        const float dim_inv = 1.0f / (float)c.head_dim;
        for (int p = 0; p < c.ctx_len; p++)
            for (int i = 0; i < c.head_dim; i += 2) {
                float theta = (float)p * expf((float)i * dim_inv * neg_log_base);
                tab[(size_t)p * half + i / 2] = make_float2(cosf(theta), sinf(theta));
            }
        if ((rc = dmalloc((void**)&m->rope, tab.size() * sizeof(float2), false))) return fail(rc);
        cudaError_t e = cudaMemcpy(m->rope, tab.data(), tab.size() * sizeof(float2),
                                   cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return fail(cuda_error(e, "rope upload"));
    }
    if (c.norm_offset) {
        // RmsNormWithOffset (TensorMath.cs:335-394) scales by (weight + 1): the
        // sums are formed once here, in fp32 as the reference forms them
        const size_t per = (size_t)c.dim;
        if ((rc = dmalloc((void**)&m->normw, (2 * (size_t)c.n_layers + 1) * per * 4, false))) return fail(rc);
        for (int l = 0; l <= c.n_layers; l++)
            for (int which = 0; which < (l < c.n_layers ? 2 : 1); which++) {
                const float* src = static_cast<const float*>(l < c.n_layers ? LT(m, l, which ? L_FNORM : L_ANORM)->d
                                                                             : m->t[T_ONORM]->d);
                float* dst = m->normw + (l < c.n_layers ? (2 * (size_t)l + which) * per : 2 * (size_t)c.n_layers * per);
                if ((rc = launch_add_scalar(dst, src, 1.0f, (int64_t)per, ctx->stream))) return fail(rc);
            }
        cudaError_t e0 = cudaStreamSynchronize(ctx->stream);
        if (e0 != cudaSuccess) return fail(cuda_error(e0, "norm offset"));
    }
    if ((rc = pad_rows(m))) return fail(rc);
    const size_t fd = (size_t)B * c.dim * 4, fq = (size_t)B * qdim * 4, fk = (size_t)B * kvd * 4,
                 fh = (size_t)B * hid * 4;
    if (m->tp) {
        m->logits = tp_logits(m->tp);  // all-gathered by the lm_head GEMVs
        m->logits_owned = false;
    }
    if ((rc = dmalloc((void**)&m->x, fd)) || (rc = dmalloc((void**)&m->x2, fd)) ||
        (rc = dmalloc((void**)&m->xn, fd)) ||
        (rc = dmalloc((void**)&m->attn_ctr, (size_t)B * nkv * sizeof(int))) ||
        (rc = dmalloc((void**)&m->q, fq)) || (rc = dmalloc((void**)&m->k, fk)) ||
        (rc = dmalloc((void**)&m->v, fk)) || (rc = dmalloc((void**)&m->att, fq)) ||
        (rc = dmalloc((void**)&m->tmp, fd)) || (rc = dmalloc((void**)&m->gate, fh)) ||
        (rc = dmalloc((void**)&m->up, fh)) ||
        (!m->tp && (rc = dmalloc((void**)&m->logits, (size_t)B * c.vocab * 4))) ||
        (rc = dmalloc((void**)&m->tokens, B * 4)) || (rc = dmalloc((void**)&m->pos, B * 4)) ||
        (rc = dmalloc((void**)&m->amax, B * 4)))
        return fail(rc);
    {
        // split counts depend on the batch size: size for the largest need
        size_t part = 0;
        for (int b = 1; b <= B; b++) {
            AttnPlan ap;
            attention_plan(nh, nkv, c.head_dim, c.ctx_len, b, ctx->sms, c.kv_dtype == CN_KV_F16, &ap);
            if (ap.part_floats > part) part = ap.part_floats;
        }
        if ((rc = dmalloc((void**)&m->part, part * 4))) return fail(rc);
    }
    // GEMV scratch for the largest plan of any batch size up to max_batch
    {
        GemvNeeds need;
        // one batch size per plan class: the Q4_K decode families (1..5,
        // 1..8), then the n-tiles of 4 of the fp16 kernel
        const int reps[5] = {4, 5, 8, 16, 32};
        for (int r = 0; r < 5; r++) {
            int b = reps[r] < B ? reps[r] : B;
            for (int i = 0; i < n_tensors; i++) {
                const cn_tensor* w = m->t[i];
                if (w->type == CN_TYPE_F32 && (i == T_ONORM || (i >= 3 && (i - 3) % 9 == L_ANORM) ||
                                               (i >= 3 && (i - 3) % 9 == L_FNORM)))
                    continue;
                GemvOp op;
                if ((rc = gemv_make(ctx, w->type, w->d, w->rows, w->cols, w->has_map ? &w->map : nullptr,
                                    b, &op, w->row_bytes)))
                    return fail(rc);
                gemv_reserve(op.plan, &need);
            }
            // the grouped launches (q/k/v, gate/up) of any layer: same shapes
            if (c.n_layers > 0) {
                static const int wj[5] = {L_Q, L_K, L_V, L_GATE, L_UP};
                GemvOp o[5];
                for (int j = 0; j < 5; j++) {
                    const cn_tensor* w = m->t[3 + wj[j]];
                    if ((rc = gemv_make(ctx, w->type, w->d, w->rows, w->cols, w->has_map ? &w->map : nullptr,
                                        b, &o[j], w->row_bytes)))
                        return fail(rc);
                }
                GemvGroup g;
                if (gemv_group_make(ctx, o, 3, &g) == CN_OK) gemv_reserve(g.plan, &need);
                if (gemv_group_make(ctx, o + 3, 2, &g) == CN_OK) gemv_reserve(g.plan, &need);
                set_error(CN_OK, "");
            }
            if (reps[r] >= B) break;
        }
        if ((rc = dmalloc((void**)&m->gb.xfrag, need.xfrag_bytes, true)) ||
            (rc = dmalloc((void**)&m->gb.xsum, need.xsum_bytes, true)) ||
            (rc = dmalloc((void**)&m->gb.partials, need.partial_bytes, false)) ||
            (rc = dmalloc((void**)&m->gb.counters, need.counters * 4 + 256, true)) ||
            (rc = dmalloc((void**)&m->gb.xinv, need.xinv_bytes, true)))
            return fail(rc);
        m->counter_bytes = need.counters * 4 + 256;
    }
    cudaError_t e = cudaMallocHost((void**)&m->h_tokens, B * 4);
    if (e == cudaSuccess) e = cudaMallocHost((void**)&m->h_pos, B * 4);
    if (e == cudaSuccess) e = cudaMallocHost((void**)&m->h_amax, B * 4);
    if (e != cudaSuccess) return fail(cuda_error(e, "cudaMallocHost"));
    set_error(CN_OK, "");
    *out = m;
    return CN_OK;
}

int cn_llama_create(cn_ctx* ctx, const cn_llama_config* cfg, cn_tensor* const* tensors,
                    int n_tensors, cn_llama** out) {
    return create_model(ctx, cfg, tensors, n_tensors, nullptr, out);
}

int cn_llama_create_tp(cn_ctx* ctx, const cn_llama_config* cfg, cn_tensor* const* tensors, int n_tensors,
                       cn_tp* tp, cn_llama** out) {
    CN_CHECK(tp, CN_ERR_INVALID_ARG, "null tensor-parallel group");
    return create_model(ctx, cfg, tensors, n_tensors, tp, out);
}

int cn_llama_prepare(cn_llama* m, int batch) {
    CN_CHECK(m, CN_ERR_INVALID_ARG, "null model");
    CN_CHECK(batch >= 1 && batch <= m->cfg.max_batch, CN_ERR_INVALID_ARG,
             "batch %d outside [1, %d]", batch, m->cfg.max_batch);
    cudaSetDevice(m->ctx->device);
    return prepare_step(m, batch);
}

int cn_llama_prefill_hidden_dev(cn_llama* m, const float* x_dev, int n, int pos, float* out_dev) {
    CN_CHECK(m && x_dev && out_dev, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(n >= 1 && pos >= 0 && pos + n <= m->cfg.ctx_len, CN_ERR_INVALID_ARG,
             "positions [%d, %d) outside the context of %d", pos, pos + n, m->cfg.ctx_len);
    CN_CHECK(prefill_supported(m), CN_ERR_UNSUPPORTED,
             "prefill (LlamaModel.Forward over a prompt) needs Q4_0, Q4_K or Q6_K projections, dim and hidden_dim multiples of 256, head_dim 64 or 128, one GPU");
    cudaSetDevice(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    int rc = prefill_reserve(m, n);
    if (rc) return rc;
    const size_t bytes = (size_t)n * m->cfg.dim * 4;
    CN_CUDA(cudaMemcpyAsync(m->pf_x, x_dev, bytes, cudaMemcpyDeviceToDevice, s));
    if ((rc = prefill_layers(m, n, pos))) return rc;
    CN_CUDA(cudaMemcpyAsync(out_dev, m->pf_x, bytes, cudaMemcpyDeviceToDevice, s));
    return CN_OK;
}

int cn_llama_prefill_kernels(cn_llama* m, int* n_kernels) {
    CN_CHECK(m && n_kernels, CN_ERR_INVALID_ARG, "null argument");
    *n_kernels = prefill_kernels(m);
    return CN_OK;
}

int cn_llama_destroy(cn_llama* m) {
    if (!m) return CN_OK;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    free_model(m);
    return CN_OK;
}

int cn_llama_decode(cn_llama* m, const int* tokens, const int* pos, int batch, float* logits_host,
                    int* argmax_host) {
    CN_CHECK(m && tokens && pos, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(batch >= 1 && batch <= m->cfg.max_batch, CN_ERR_INVALID_ARG,
             "batch %d outside [1, %d]", batch, m->cfg.max_batch);
    for (int b = 0; b < batch; b++) {
        CN_CHECK(tokens[b] >= 0 && tokens[b] < m->cfg.vocab, CN_ERR_INVALID_ARG,
                 "token id %d outside [0, %d)", tokens[b], m->cfg.vocab);
        CN_CHECK(pos[b] >= 0 && pos[b] < m->cfg.ctx_len, CN_ERR_INVALID_ARG,
                 "position %d outside [0, %d)", pos[b], m->cfg.ctx_len);
    }
    cudaSetDevice(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    memcpy(m->h_tokens, tokens, batch * 4);
    memcpy(m->h_pos, pos, batch * 4);
    CN_CUDA(cudaMemcpyAsync(m->tokens, m->h_tokens, batch * 4, cudaMemcpyHostToDevice, s));
    CN_CUDA(cudaMemcpyAsync(m->pos, m->h_pos, batch * 4, cudaMemcpyHostToDevice, s));
    int rc = run_step(m, batch);
    if (rc) return rc;
    if (logits_host)
        CN_CUDA(cudaMemcpyAsync(logits_host, m->logits, (size_t)batch * m->cfg.vocab * 4,
                                cudaMemcpyDeviceToHost, s));
    if (argmax_host) CN_CUDA(cudaMemcpyAsync(m->h_amax, m->amax, batch * 4, cudaMemcpyDeviceToHost, s));
    CN_CUDA(cudaStreamSynchronize(s));
    if ((rc = check_dev_err_reset(m))) return rc;
    if (argmax_host) memcpy(argmax_host, m->h_amax, batch * 4);
    return CN_OK;
}

int cn_llama_set_prefill(cn_llama* m, int min_tokens) {
    CN_CHECK(m, CN_ERR_INVALID_ARG, "null model");
    CN_CHECK(min_tokens == 0 || min_tokens >= kPrefillMin, CN_ERR_INVALID_ARG,
             "prefill threshold %d: 0 or at least %d", min_tokens, kPrefillMin);
    m->prefill_min = min_tokens;
    return CN_OK;
}

int cn_llama_set_prefill_precision(cn_llama* m, int split) {
    CN_CHECK(m, CN_ERR_INVALID_ARG, "null model");
    CN_CHECK(split >= 0 && split <= 2, CN_ERR_INVALID_ARG, "prefill precision %d: 0, 1 or 2", split);
    m->prefill_split = split;
    return CN_OK;
}

int cn_llama_sample(cn_llama* m, int batch, float temperature, int top_k, float top_p, const float* r_host,
                    int* tokens_host) {
    CN_CHECK(m, CN_ERR_INVALID_ARG, "null model");
    CN_CHECK(batch >= 1 && batch <= m->cfg.max_batch, CN_ERR_INVALID_ARG, "batch %d outside [1, %d]", batch,
             m->cfg.max_batch);
    cudaSetDevice(m->ctx->device);
    return sample_launch(m->ctx, m->logits, m->cfg.vocab, batch, temperature, top_k, top_p, r_host, tokens_host);
}

int cn_llama_set_inputs(cn_llama* m, const int* tokens, const int* pos, int batch) {
    CN_CHECK(m && tokens && pos, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(batch >= 1 && batch <= m->cfg.max_batch, CN_ERR_INVALID_ARG,
             "batch %d outside [1, %d]", batch, m->cfg.max_batch);
    for (int b = 0; b < batch; b++) {
        CN_CHECK(tokens[b] >= 0 && tokens[b] < m->cfg.vocab, CN_ERR_INVALID_ARG,
                 "token id %d outside [0, %d)", tokens[b], m->cfg.vocab);
        CN_CHECK(pos[b] >= 0 && pos[b] < m->cfg.ctx_len, CN_ERR_INVALID_ARG,
                 "position %d outside [0, %d)", pos[b], m->cfg.ctx_len);
    }
    cudaSetDevice(m->ctx->device);
    CN_CUDA(cudaStreamSynchronize(m->ctx->stream));
    CN_CUDA(cudaMemcpy(m->tokens, tokens, batch * 4, cudaMemcpyHostToDevice));
    CN_CUDA(cudaMemcpy(m->pos, pos, batch * 4, cudaMemcpyHostToDevice));
    return CN_OK;
}

int cn_llama_step(cn_llama* m, int batch) {
    CN_CHECK(m, CN_ERR_INVALID_ARG, "null model");
    CN_CHECK(batch >= 1 && batch <= m->cfg.max_batch, CN_ERR_INVALID_ARG,
             "batch %d outside [1, %d]", batch, m->cfg.max_batch);
    cudaSetDevice(m->ctx->device);
    return run_step(m, batch);
}

int cn_llama_step_kernels(cn_llama* m, int batch, int* out_count) {
    CN_CHECK(m && out_count, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(batch >= 1 && batch <= m->cfg.max_batch, CN_ERR_INVALID_ARG, "bad batch");
    cudaSetDevice(m->ctx->device);
    int rc = build_step(m, batch);
    if (rc) return rc;
    cudaStream_t s = m->ctx->stream;
    cudaGraph_t g = nullptr;
    CN_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    rc = enqueue_step(m, batch, s);
    cudaError_t e = cudaStreamEndCapture(s, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return cuda_error(e, "cudaStreamEndCapture");
    size_t n = 0;
    e = cudaGraphGetNodes(g, nullptr, &n);
    std::vector<cudaGraphNode_t> nodes(n);
    if (e == cudaSuccess && n) e = cudaGraphGetNodes(g, nodes.data(), &n);
    int kernels = 0;
    for (size_t i = 0; e == cudaSuccess && i < n; i++) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) kernels++;
    }
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_error(e, "cudaGraphGetNodes");
    *out_count = kernels;
    return CN_OK;
}

int cn_llama_time_gemv(cn_llama* m, int proj, int batch, int iters, float* us_per_launch,
                       double* bytes_per_launch) {
    CN_CHECK(m && us_per_launch && bytes_per_launch, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(proj >= 0 && proj <= 9 && iters >= 1, CN_ERR_INVALID_ARG, "bad proj/iters");
    CN_CHECK(batch >= 1 && batch <= m->cfg.max_batch, CN_ERR_INVALID_ARG, "bad batch");
    cudaSetDevice(m->ctx->device);
    int rc = build_step(m, batch);
    if (rc) return rc;
    Step& st = m->steps[batch];
    const int L = m->cfg.n_layers;
    if (proj >= 8) {
        // the grouped launch the step runs: q/k/v (8) or gate/up (9) in one GEMV
        const std::vector<GemvGroup>& gs = proj == 8 ? st.qkv : st.gu;
        CN_CHECK(L > 0 && gs[0].n > 0, CN_ERR_UNSUPPORTED, "this model runs those projections as separate launches");
        float* ys[3] = {proj == 8 ? m->q : m->gate, proj == 8 ? m->k : m->up, m->v};
        cudaStream_t s = m->ctx->stream;
        if ((rc = gemv_prep(s, m->ctx->sms, gs[0].ops[0], m->xn, m->gb))) return rc;
        for (int i = 0; i < 3; i++)
            if ((rc = gemv_group_run(m->ctx, s, gs[i % L], m->gb, ys))) return rc;
        cudaEvent_t e0, e1;
        CN_CUDA(cudaEventCreate(&e0));
        CN_CUDA(cudaEventCreate(&e1));
        CN_CUDA(cudaEventRecord(e0, s));
        for (int i = 0; i < iters; i++)
            if ((rc = gemv_group_run(m->ctx, s, gs[(i + 3) % L], m->gb, ys))) return rc;
        CN_CUDA(cudaEventRecord(e1, s));
        CN_CUDA(cudaEventSynchronize(e1));
        float ms = 0.f;
        CN_CUDA(cudaEventElapsedTime(&ms, e0, e1));
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        *us_per_launch = ms * 1000.f / iters;
        double bytes = 4.0 * batch * gs[0].ops[0].cols;
        for (int k = 0; k < gs[0].n; k++)
            bytes += (double)gs[0].ops[k].rb * gs[0].ops[k].rows + 4.0 * batch * gs[0].ops[k].rows;
        *bytes_per_launch = bytes;
        return check_dev_err_reset(m);
    }
    auto op_of = [&](int i) -> const GemvOp& {
        return proj == 7 ? st.ops[(size_t)L * 7] : st.ops[(size_t)(i % L) * 7 + proj];
    };
    const GemvOp& op0 = op_of(0);
    const float* x = (proj == 3) ? m->att : (proj == 6) ? m->gate : m->xn;
    float* y = (proj == 0 || proj == 3 || proj == 6) ? m->tmp
               : (proj == 1) ? m->k : (proj == 2) ? m->v : (proj == 7) ? m->logits : m->up;
    cudaStream_t s = m->ctx->stream;
    if ((rc = gemv_prep(s, m->ctx->sms, op0, x, m->gb))) return rc;
    // warm-up, then timed launches cycling through the layers (cold L2)
    for (int i = 0; i < 3; i++)
        if ((rc = gemv_run(m->ctx, s, op_of(i), x, m->gb, y))) return rc;
    cudaEvent_t e0, e1;
    CN_CUDA(cudaEventCreate(&e0));
    CN_CUDA(cudaEventCreate(&e1));
    CN_CUDA(cudaEventRecord(e0, s));
    for (int i = 0; i < iters; i++)
        if ((rc = gemv_run(m->ctx, s, op_of(i + 3), x, m->gb, y))) return rc;
    CN_CUDA(cudaEventRecord(e1, s));
    CN_CUDA(cudaEventSynchronize(e1));
    float ms = 0.f;
    CN_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *us_per_launch = ms * 1000.f / iters;
    *bytes_per_launch = (double)op0.rb * op0.rows + 4.0 * batch * (op0.rows + op0.cols);
    return check_dev_err_reset(m);
}

int cn_llama_profile_step(cn_llama* m, int batch, float* us_by_stage, int n_stages) {
    CN_CHECK(m && us_by_stage && n_stages >= 1, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(batch >= 1 && batch <= m->cfg.max_batch, CN_ERR_INVALID_ARG, "bad batch");
    cudaSetDevice(m->ctx->device);
    int rc = build_step(m, batch);
    if (rc) return rc;
    cudaStream_t s = m->ctx->stream;
    CN_CUDA(cudaStreamSynchronize(s));
    StepProfile prof;
    g_prof = &prof;
    rc = mark(s, P_START);
    if (!rc) rc = enqueue_step(m, batch, s);
    g_prof = nullptr;
    if (!rc) {
        const cudaError_t e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) rc = cuda_error(e, "profile step");
    }
    for (int k = 0; k < n_stages; k++) us_by_stage[k] = 0.f;
    for (size_t i = 1; !rc && i < prof.ev.size(); i++) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, prof.ev[i - 1], prof.ev[i]);
        const int k = prof.kind[i];
        if (k < n_stages) us_by_stage[k] += ms * 1000.f;
    }
    for (cudaEvent_t e : prof.ev) cudaEventDestroy(e);
    if (rc) return rc;
    return check_dev_err_reset(m);
}

int cn_llama_time_matmul(cn_llama* m, int group, int n, int iters, float* us_per_launch,
                         double* flops_per_launch) {
    CN_CHECK(m && us_per_launch && flops_per_launch, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(group >= 0 && group <= 3 && iters >= 1 && n >= 1, CN_ERR_INVALID_ARG, "bad group/n/iters");
    CN_CHECK(prefill_supported(m), CN_ERR_UNSUPPORTED, "model cannot run the prefill matmul");
    cudaSetDevice(m->ctx->device);
    int rc = prefill_reserve(m, n);
    if (rc) return rc;
    const cn_llama_config& c = m->cfg;
    const int64_t qd = m->qdim, kvd = m->kvdim, hid = c.hidden_dim, dim = c.dim;
    cudaStream_t s = m->ctx->stream;
    CN_CUDA(cudaMemsetAsync(m->pf_h, 0, (size_t)n * (hid > dim ? hid : dim) * 2, s));
    CN_CUDA(cudaMemsetAsync(m->pf_x, 0, (size_t)n * dim * 4, s));
    CN_CUDA(cudaMemsetAsync(m->pf_xs, 0, (size_t)n * 4, s));
    CN_CUDA(cudaMemsetAsync(m->pf_hl, 0, (size_t)n * (hid > dim ? hid : dim) * 2, s));
    int ns[4];
    split_counts(m, ns);
    if ((ns[0] || ns[2]) && (rc = prefill_scales(m))) return rc;
    const int L = c.n_layers;
    double flops = 0;
    auto launch = [&](int i) -> int {
        const int l = i % L;
        if (group == 0) {
            const int64_t rows[3] = {qd, kvd, kvd};
            float* y[3] = {m->pf_q, m->pf_k, m->pf_v};
            flops = 2.0 * n * (double)(qd + 2 * kvd) * dim;  // algorithmic (the split's extra MMAs not counted)
            return mm_group(m, l, 3, kSlotsQKV, rows, dim, n, y, rows, false, true, false, ns[0]);
        }
        if (group == 2) {
            const int64_t rows[2] = {hid, hid};
            float* y[2] = {m->pf_g, m->pf_u};
            flops = 2.0 * n * (double)(2 * hid) * dim;
            return mm_group(m, l, 2, kSlotsGU, rows, dim, n, y, rows, false, true, false, ns[2]);
        }
        const int64_t rows = dim, K = group == 1 ? qd : hid;
        flops = 2.0 * n * (double)dim * K;
        return mm_group(m, l, 1, group == 1 ? kSlotsO : kSlotsDown, &rows, K, n, &m->pf_x, &rows, true, group == 3,
                        false, group == 1 ? ns[1] : ns[3]);
    };
    for (int i = 0; i < 3; i++)
        if ((rc = launch(i))) return rc;
    cudaEvent_t e0, e1;
    CN_CUDA(cudaEventCreate(&e0));
    CN_CUDA(cudaEventCreate(&e1));
    CN_CUDA(cudaEventRecord(e0, s));
    for (int i = 0; i < iters; i++)
        if ((rc = launch(i + 3))) return rc;
    CN_CUDA(cudaEventRecord(e1, s));
    CN_CUDA(cudaEventSynchronize(e1));
    float ms = 0.f;
    CN_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    *us_per_launch = ms * 1000.f / iters;
    *flops_per_launch = flops;
    return check_dev_err_reset(m);
}

int cn_llama_forward(cn_llama* m, const int* tokens, int n, int pos, float* logits_host) {
    CN_CHECK(m && tokens && logits_host, CN_ERR_INVALID_ARG, "null argument");
    CN_CHECK(n >= 1, CN_ERR_INVALID_ARG, "no tokens");
    CN_CHECK(pos >= 0 && pos + n <= m->cfg.ctx_len, CN_ERR_INVALID_ARG,
             "positions [%d, %d) outside the context of %d", pos, pos + n, m->cfg.ctx_len);
    if (m->prefill_min > 0 && n >= m->prefill_min && prefill_supported(m)) {
        // the prompt in one pass: embed n tokens, all layers on the matmul,
        // then the head of the last token through the decode GEMV
        for (int t = 0; t < n; t++)
            CN_CHECK(tokens[t] >= 0 && tokens[t] < m->cfg.vocab, CN_ERR_INVALID_ARG,
                     "token id %d outside [0, %d)", tokens[t], m->cfg.vocab);
        cudaSetDevice(m->ctx->device);
        cudaStream_t s = m->ctx->stream;
        const cn_llama_config& c = m->cfg;
        int rc = prefill_reserve(m, n);
        if (rc) return rc;
        CN_CUDA(cudaMemcpyAsync(m->pf_tok, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, s));
        const cn_tensor* emb = m->t[T_EMB];
        if ((rc = launch_embed(emb->type, emb->d, emb->row_bytes, m->pf_tok, c.vocab, c.dim, n, m->pf_x,
                               m->ctx->dev_err, s)))
            return rc;
        if ((rc = prefill_layers(m, n, pos))) return rc;
        if ((rc = launch_rmsnorm(m->pf_x + (size_t)(n - 1) * c.dim, norm_w(m, -1, 0), m->xn,
                                 c.dim, 1, c.rms_eps, s)))
            return rc;
        const cn_tensor* w = m->t[T_OUT];
        if ((rc = gemv_launch(m->ctx, w->type, w->d, w->rows, w->cols, w->has_map ? &w->map : nullptr, m->xn,
                              m->logits, 1)))
            return rc;
        CN_CUDA(cudaMemcpyAsync(logits_host, m->logits, (size_t)c.vocab * 4, cudaMemcpyDeviceToHost, s));
        CN_CUDA(cudaStreamSynchronize(s));
        return check_dev_err_reset(m);
    }
    for (int t = 0; t < n; t++) {
        int p = pos + t;
        int rc = cn_llama_decode(m, tokens + t, &p, 1, t == n - 1 ? logits_host : nullptr, nullptr);
        if (rc) return rc;
    }
    return CN_OK;
}

static int kv_check(cn_llama* m, int seq, int layer, int pos0, int npos) {
    CN_CHECK(m, CN_ERR_INVALID_ARG, "null model");
    CN_CHECK(seq >= 0 && seq < m->cfg.max_batch, CN_ERR_INVALID_ARG, "seq %d out of range", seq);
    CN_CHECK(layer >= 0 && layer < m->cfg.n_layers, CN_ERR_INVALID_ARG, "layer %d out of range", layer);
    CN_CHECK(pos0 >= 0 && npos >= 0 && pos0 + npos <= m->cfg.ctx_len, CN_ERR_INVALID_ARG,
             "positions out of range");
    return CN_OK;
}

int cn_llama_kv_write(cn_llama* m, int seq, int layer, int pos0, int npos, const void* k_host,
                      const void* v_host) {
    int rc = kv_check(m, seq, layer, pos0, npos);
    if (rc) return rc;
    cudaSetDevice(m->ctx->device);
    size_t off = ((size_t)seq * m->seq_stride + ((size_t)layer * m->cfg.ctx_len + pos0) * m->kvdim) *
                 m->kv_elem;
    size_t bytes = (size_t)npos * m->kvdim * m->kv_elem;
    CN_CUDA(cudaStreamSynchronize(m->ctx->stream));
    if (k_host) CN_CUDA(cudaMemcpy((uint8_t*)m->kc + off, k_host, bytes, cudaMemcpyHostToDevice));
    if (v_host) CN_CUDA(cudaMemcpy((uint8_t*)m->vc + off, v_host, bytes, cudaMemcpyHostToDevice));
    return CN_OK;
}

int cn_llama_kv_read(cn_llama* m, int seq, int layer, int pos0, int npos, void* k_host,
                     void* v_host) {
    int rc = kv_check(m, seq, layer, pos0, npos);
    if (rc) return rc;
    cudaSetDevice(m->ctx->device);
    size_t off = ((size_t)seq * m->seq_stride + ((size_t)layer * m->cfg.ctx_len + pos0) * m->kvdim) *
                 m->kv_elem;
    size_t bytes = (size_t)npos * m->kvdim * m->kv_elem;
    CN_CUDA(cudaStreamSynchronize(m->ctx->stream));
    if (k_host) CN_CUDA(cudaMemcpy(k_host, (uint8_t*)m->kc + off, bytes, cudaMemcpyDeviceToHost));
    if (v_host) CN_CUDA(cudaMemcpy(v_host, (uint8_t*)m->vc + off, bytes, cudaMemcpyDeviceToHost));
    return CN_OK;
}

int cn_llama_kv_synth(cn_llama* m, int seq, int npos, uint64_t seed_k, uint64_t seed_v) {
    int rc = kv_check(m, seq, 0, 0, npos);
    if (rc) return rc;
    cudaSetDevice(m->ctx->device);
    cudaStream_t s = m->ctx->stream;
    const size_t seq_bytes = (size_t)m->seq_stride * m->kv_elem;
    uint8_t* kb = (uint8_t*)m->kc + (size_t)seq * seq_bytes;
    uint8_t* vb = (uint8_t*)m->vc + (size_t)seq * seq_bytes;
    CN_CUDA(cudaMemsetAsync(kb, 0, seq_bytes, s));
    CN_CUDA(cudaMemsetAsync(vb, 0, seq_bytes, s));
    if (npos > 0) {
        int64_t n = (int64_t)m->cfg.n_layers * npos * m->kvdim;
        int blocks = (int)((n + 255) / 256 > 148 * 64 ? 148 * 64 : (n + 255) / 256);
        int f16 = m->cfg.kv_dtype == CN_KV_F16;
        const int kvd_full = m->cfg.n_kv_heads * m->cfg.head_dim, col0 = m->tp_rank * m->kvdim;
        kv_synth_kernel<<<blocks, 256, 0, s>>>(seed_k, m->cfg.n_layers, npos, m->cfg.ctx_len, m->kvdim,
                                               kvd_full, col0, f16, kb);
        kv_synth_kernel<<<blocks, 256, 0, s>>>(seed_v, m->cfg.n_layers, npos, m->cfg.ctx_len, m->kvdim,
                                               kvd_full, col0, f16, vb);
        CN_CUDA(cudaGetLastError());
    }
    CN_CUDA(cudaStreamSynchronize(s));
    return CN_OK;
}

}  // extern "C"
