/* tgai_forward.c -- whole-model forward on a B200 around the KV path.
 *
 * Host C.  The block structure and its order follow the engine's CPU forward
 * (src/tgai_engine.c:3821-4358 transformer_block, :4361-4507 tg_forward):
 *
 *   x = emb[ids]                                       (ids out of range -> unk)
 *   per layer:  ln = rmsnorm(x, ln1);  qkv = ln . [Wq; Wk; Wv]^T (+ biases)
 *               RoPE(q, k) at positions pos.., K/V appended to the layer cache
 *               attn = causal GQA attention over the cache
 *               x += attn . Wo^T
 *               ln = rmsnorm(x, ln2)
 *               dense: x += (silu(clamp(ln.W1^T)) * ln.W2^T) . W3^T
 *               MoE:   top-k of ln.Wr^T (+ bias), softmax over the k,
 *                      x += sum_k w_k * W3_e (silu(W1_e ln) * W2_e ln)
 *   logits = rmsnorm(x_last, final_norm) . emb^T
 *
 * The device side is one stream per sequence ("slot", keyed by the caller's
 * pointer as cuda/tgai_cuda.cu:1656-1672 keys them): our kernels
 * (tgkv_forward.cu), the KV path's RoPE+append and attention kernels, and
 * for the prefill projections and the router our tensor-core GEMM
 * (tgkv_gemm.cu) at fp32-product accuracy, where the reference bridge calls
 * cublasSgemm (cuda/tgai_cuda.cu:473-479); no library GEMM is used.  The
 * only host synchronisation per forward is the final logits copy; the MoE
 * routing stays on the device (the reference bridge copies the top-k ids to
 * the host once per layer, cuda/tgai_cuda.cu:1532-1590).
 *
 * Slot rules of the reference bridge: at most TGAI_CUDA_KV_SLOTS slots
 * (default 16, 1..64; cuda/tgai_cuda.cu:790-800), a request beyond them is
 * rejected and counted; a forward whose cache_pos is past the slot's last
 * written position clears the slot's KV first (:1674-1711); otherwise the
 * rows [0, cache_pos) are kept and the new tokens overwrite from cache_pos on
 * (LCP truncate + re-append).  Each slot's KV holds max_seq_len positions
 * from its first use (the reference grows by relayout from 2048; 180 GB of
 * HBM makes the fixed capacity the simpler choice).
 */
#include "tgai_engine_bridge.h"
#include "tgai_cuda_bridge.h"
#include "tgai_gpu_dispatch.h"
#include "tgai_kv_cache.h"
#include "tgkv_forward.h"

#include <dlfcn.h>
#include <math.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define HIDDEN __attribute__((visibility("hidden")))

static _Thread_local char t_err[256] = "fwd: no error";
static _Thread_local uint32_t t_launches;

static void set_err(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
}

const char* tg_fwd_last_error(void) { return t_err; }
uint32_t tg_fwd_last_launches(void) { return t_launches; }

/* ---- model and slots ------------------------------------------------------ */
typedef struct {
    float* ln1;        /* [d] */
    float* ln2;        /* [d] */
    float* wqkv;       /* [q_dim + 2 kv_dim][d]: Wq rows, Wk rows, Wv rows */
    float* bqkv;       /* [q_dim + 2 kv_dim] or NULL */
    float* wo;         /* [d][q_dim] */
    float* w12;        /* dense [2 dff][d]; MoE [ne][2 dff][d]: W1 rows then W2 rows */
    float* w3;         /* dense [d][dff];   MoE [ne][d][dff] */
    float* router;     /* [ne][d] */
    float* qb;         /* [ne] or NULL */
    /* the prefill GEMMs' operands: each weight as its tf32-rounded part and
     * the exact remainder (tgkv_split_tf32), same shapes */
    float *wqkv_b, *wqkv_s, *wo_b, *wo_s, *router_b, *router_s;
    float *w12_b, *w12_s, *w3_b, *w3_s;   /* the FFN's (a dense one, or every expert's) */
} Layer;

typedef struct Slot {
    const void* key;
    int used;
    int id;
    TGKvCache** kv;          /* one per layer */
    int last_pos;            /* positions [0, last_pos) written by this slot; -1 none */
    int kv_hi;
    void* stream;
    uint32_t cap;            /* token rows the workspaces hold */
    float *x, *ln, *qkv, *q, *attn, *ab, *h, *router, *top_w, *y, *logits;
    float *abig, *asmall;    /* a prefill GEMM's input rows, split (tgkv_split_tf32) */
    uint32_t *moe_off, *moe_rows;   /* MoE prefill: experts' first packed rows, row -> pair */
    int32_t *top_ids, *ids;
    uint32_t *counts, *lists;
    int32_t* h_ids;          /* page-locked */
    float* h_logits;         /* page-locked [vocab] */
    /* one-launch decode step (tgkv_decode_step.cu), allocated at its first use */
    float** step_kvc;        /* device [n_layers]: this slot's cache buffers */
    float* step_part;        /* attention partials */
    uint32_t* step_state;    /* barrier count, error word */
    int32_t* h_step;         /* page-locked copy of the error word */
} Slot;

struct TGFwdModel {
    TGFwdConfig c;
    uint32_t hd, nkv, q_dim, kv_dim, qkv_dim, rows;
    Layer* L;
    float *emb, *fnorm, *cs, *sn;
    float *emb_b, *emb_s;          /* split embedding, only where the LM head needs the GEMM */
    TGFwdStepLayer* step_layers;   /* device [n_layers], when the one-launch step fits */
    int step_refused;              /* the device refused the step's grid: per-layer launches */
    uint64_t wbytes;
    pthread_mutex_t mu;
    Slot* slots;
    uint32_t max_slots, live;
    long long rejects;
    /* one-token decodes of different slots gathered into one pass (below) */
    pthread_mutex_t bmu;           /* the request queue and the leader flag */
    pthread_cond_t bcv;
    struct BatchReq* bq_head;
    struct BatchReq* bq_tail;
    int b_leader;                  /* a thread is running a batch */
    pthread_mutex_t pmu;           /* the batch workspace and plans, held while a batch runs */
    Slot bs;                       /* the batch's stream and workspaces (no KV) */
    float *b_knew, *b_vnew;        /* [rows][kv_dim]: K/V rows for the fused append */
    uint32_t *b_pos, *bh_pos;      /* positions, device and page-locked [rows] */
    float *b_logits, *bh_logits;   /* [rows][vocab], device and page-locked */
    struct BatchPlan* plans;       /* [kPlanCache] */
    uint64_t plan_clock;
    long long batched_tokens, batches;
};

/* ---- batched decode across slots: types ----------------------------------- */
enum { kPlanCache = 16 };
/* One batch composition (slot ids in ascending order) and, per layer, a
 * batch plan over those slots' caches of that layer. */
struct BatchPlan {
    uint32_t n;
    int ids[8];
    TGKvBatch** b;                 /* [n_layers], NULL when the entry is empty */
    uint64_t used;
};
/* A one-token decode waiting in the queue, run by whichever thread leads. */
typedef struct BatchReq {
    Slot* s;
    int32_t id;
    uint32_t pos;
    int state;                     /* 0 queued, 1 taken, 2 done */
    int ok;
    uint32_t launches;
    char err[256];
    struct BatchReq* next;
} BatchReq;

static void plan_drop(TGFwdModel* m, struct BatchPlan* bp) {
    if (bp->b) {
        for (uint32_t l = 0; l < m->c.n_layers; l++) tg_kv_batch_destroy(bp->b[l]);
        free(bp->b);
    }
    memset(bp, 0, sizeof(*bp));
}

/* Plans that hold slot `id`'s caches (all plans for id < 0). */
static void plans_drop_slot(TGFwdModel* m, int id) {
    if (!m->plans) return;
    for (int i = 0; i < kPlanCache; i++) {
        struct BatchPlan* bp = &m->plans[i];
        if (!bp->b) continue;
        int hit = id < 0;
        for (uint32_t j = 0; j < bp->n && !hit; j++) hit = bp->ids[j] == id;
        if (hit) plan_drop(m, bp);
    }
}

static void slot_release_mem(TGFwdModel* m, Slot* s);

static void batch_release(TGFwdModel* m) {
    plans_drop_slot(m, -1);
    free(m->plans);
    m->plans = NULL;
    slot_release_mem(m, &m->bs);
    tg_cuda_kv_free(m->b_knew);
    tg_cuda_kv_free(m->b_vnew);
    tg_cuda_kv_free(m->b_pos);
    tg_cuda_kv_free(m->b_logits);
    tgkv_fwd_host_free(m->bh_pos);
    tgkv_fwd_host_free(m->bh_logits);
    m->b_knew = m->b_vnew = m->b_logits = m->bh_logits = NULL;
    m->b_pos = m->bh_pos = NULL;
}


/* The fused decode kernels stage R token rows of K floats in shared memory. */
static int decode_fits(uint32_t R, uint32_t K) {
    return R <= tgkv_fwd_decode_rows() && (uint64_t)R * K * 4 + 1024 <= 200 * 1024;
}

/* Device copy of n floats from host (blocking). */
static float* upload(TGFwdModel* m, const float* src, uint64_t n) {
    float* d = (float*)tg_cuda_kv_malloc(n * sizeof(float));
    if (!d) { set_err("device allocation of %llu bytes failed", (unsigned long long)(n * 4)); return NULL; }
    if (!tg_cuda_kv_h2d(d, src, n * sizeof(float), NULL)) {
        set_err("weight upload failed: %s", tg_cuda_kv_last_error());
        tg_cuda_kv_free(d);
        return NULL;
    }
    m->wbytes += n * sizeof(float);
    return d;
}

/* The prefill GEMM's form of a device weight [rows][cols]: its tf32-rounded
 * part and the exact remainder, in two new device buffers (queued on the
 * default stream; creation synchronises before it returns). */
static int split_weight(TGFwdModel* m, const float* w, uint64_t rows, uint64_t cols,
                        float** big, float** small) {
    const uint64_t n = rows * cols;
    *big = (float*)tg_cuda_kv_malloc(n * sizeof(float));
    *small = (float*)tg_cuda_kv_malloc(n * sizeof(float));
    if (!*big || !*small) {
        set_err("device allocation of %llu bytes failed", (unsigned long long)(2 * n * 4));
        return 0;
    }
    const int e = tgkv_split_tf32(w, cols, *big, *small, cols, (uint32_t)rows, (uint32_t)cols,
                                  NULL);
    if (e) { set_err("weight split failed (CUDA error %d)", e); return 0; }
    m->wbytes += 2 * n * sizeof(float);
    return 1;
}

/* A tensor of exactly rows x cols elements (cols 1 for 1-D), or NULL. */
static const float* tensor(TGFwdWeightFn get, void* ctx, const char* name, uint32_t rows,
                           uint32_t cols, int required) {
    uint32_t shape[2] = {0, 0};
    const float* p = get(ctx, name, shape);
    if (!p) {
        if (required) set_err("missing weight %s", name);
        return NULL;
    }
    if ((uint64_t)shape[0] * shape[1] != (uint64_t)rows * cols) {
        set_err("weight %s has shape [%u, %u], expected [%u, %u]", name, shape[0], shape[1],
                rows, cols);
        return NULL;
    }
    return p;
}

/* An optional tensor: NULL and *bad = 0 when absent, NULL and *bad = 1 when
 * present with the wrong size. */
static const float* optional(TGFwdWeightFn get, void* ctx, const char* name, uint32_t rows,
                             uint32_t cols, int* bad) {
    uint32_t shape[2] = {0, 0};
    *bad = 0;
    if (!get(ctx, name, shape)) return NULL;
    const float* p = tensor(get, ctx, name, rows, cols, 1);
    if (!p) *bad = 1;
    return p;
}

static void free_layer(Layer* l) {
    tg_cuda_kv_free(l->ln1);
    tg_cuda_kv_free(l->ln2);
    tg_cuda_kv_free(l->wqkv);
    tg_cuda_kv_free(l->bqkv);
    tg_cuda_kv_free(l->wo);
    tg_cuda_kv_free(l->w12);
    tg_cuda_kv_free(l->w3);
    tg_cuda_kv_free(l->router);
    tg_cuda_kv_free(l->qb);
    float* sp[] = {l->wqkv_b, l->wqkv_s, l->wo_b, l->wo_s, l->router_b, l->router_s,
                   l->w12_b, l->w12_s, l->w3_b, l->w3_s};
    for (size_t i = 0; i < sizeof(sp) / sizeof(sp[0]); i++) tg_cuda_kv_free(sp[i]);
}

static void slot_release_mem(TGFwdModel* m, Slot* s);

void tg_fwd_destroy(TGFwdModel* m) {
    if (!m) return;
    batch_release(m);
    if (m->slots)
        for (uint32_t i = 0; i < m->max_slots; i++) slot_release_mem(m, &m->slots[i]);
    free(m->slots);
    if (m->L) {
        for (uint32_t l = 0; l < m->c.n_layers; l++) free_layer(&m->L[l]);
        free(m->L);
    }
    tg_cuda_kv_free(m->emb);
    tg_cuda_kv_free(m->emb_b);
    tg_cuda_kv_free(m->emb_s);
    tg_cuda_kv_free(m->fnorm);
    tg_cuda_kv_free(m->cs);
    tg_cuda_kv_free(m->sn);
    tg_cuda_kv_free(m->step_layers);
    pthread_mutex_destroy(&m->mu);
    pthread_mutex_destroy(&m->bmu);
    pthread_mutex_destroy(&m->pmu);
    pthread_cond_destroy(&m->bcv);
    free(m);
}

/* Concatenate row blocks into one host buffer and upload it. */
static float* upload_cat(TGFwdModel* m, const float* const* parts, const uint64_t* n, int k) {
    uint64_t tot = 0;
    for (int i = 0; i < k; i++) tot += n[i];
    float* h = (float*)malloc(tot * sizeof(float));
    if (!h) { set_err("host allocation failed"); return NULL; }
    uint64_t o = 0;
    for (int i = 0; i < k; i++) {
        if (parts[i]) memcpy(h + o, parts[i], n[i] * sizeof(float));
        else memset(h + o, 0, n[i] * sizeof(float));
        o += n[i];
    }
    float* d = upload(m, h, tot);
    free(h);
    return d;
}

static int moe_gemm_on(void) {
    const char* e = getenv("TGKV_MOE_GEMM");
    return !(e && e[0] == '0');
}

static int load_layer(TGFwdModel* m, uint32_t l, TGFwdWeightFn get, void* ctx) {
    const uint32_t d = m->c.d_model, dff = m->c.d_ff, ne = m->c.n_experts;
    Layer* L = &m->L[l];
    char name[160];
    int bad = 0;
#define NAME(...) (snprintf(name, sizeof(name), __VA_ARGS__), name)
    const float* p;
    if (!(p = tensor(get, ctx, NAME("blocks.%u.ln1.weight", l), d, 1, 1)) || !(L->ln1 = upload(m, p, d)))
        return 0;
    if (!(p = tensor(get, ctx, NAME("blocks.%u.ln2.weight", l), d, 1, 1)) || !(L->ln2 = upload(m, p, d)))
        return 0;
    {
        const float* w[3];
        const float* b[3];
        uint64_t nw[3] = {(uint64_t)m->q_dim * d, (uint64_t)m->kv_dim * d, (uint64_t)m->kv_dim * d};
        uint64_t nb[3] = {m->q_dim, m->kv_dim, m->kv_dim};
        static const char* pn[3] = {"q_proj", "k_proj", "v_proj"};
        int any_bias = 0;
        for (int i = 0; i < 3; i++) {
            if (!(w[i] = tensor(get, ctx, NAME("blocks.%u.attn.%s.weight", l, pn[i]),
                                (uint32_t)(nb[i]), d, 1)))
                return 0;
            b[i] = optional(get, ctx, NAME("blocks.%u.attn.%s.bias", l, pn[i]), (uint32_t)nb[i], 1, &bad);
            if (bad) return 0;
            any_bias |= b[i] != NULL;
        }
        if (!(L->wqkv = upload_cat(m, w, nw, 3))) return 0;
        if (any_bias && !(L->bqkv = upload_cat(m, b, nb, 3))) return 0;
        if (!split_weight(m, L->wqkv, m->qkv_dim, d, &L->wqkv_b, &L->wqkv_s)) return 0;
    }
    if (!(p = tensor(get, ctx, NAME("blocks.%u.attn.out_proj.weight", l), d, m->q_dim, 1)) ||
        !(L->wo = upload(m, p, (uint64_t)d * m->q_dim)) ||
        !split_weight(m, L->wo, d, m->q_dim, &L->wo_b, &L->wo_s))
        return 0;
    if (ne == 0) {
        const float* w[2];
        uint64_t nw[2] = {(uint64_t)dff * d, (uint64_t)dff * d};
        if (!(w[0] = tensor(get, ctx, NAME("blocks.%u.ffn.w1.weight", l), dff, d, 1))) return 0;
        if (!(w[1] = tensor(get, ctx, NAME("blocks.%u.ffn.w2.weight", l), dff, d, 1))) return 0;
        if (!(L->w12 = upload_cat(m, w, nw, 2)) ||
            !split_weight(m, L->w12, 2 * (uint64_t)dff, d, &L->w12_b, &L->w12_s))
            return 0;
        if (!(p = tensor(get, ctx, NAME("blocks.%u.ffn.w3.weight", l), d, dff, 1)) ||
            !(L->w3 = upload(m, p, (uint64_t)d * dff)) ||
            !split_weight(m, L->w3, d, dff, &L->w3_b, &L->w3_s))
            return 0;
        return 1;
    }
    if (!(p = tensor(get, ctx, NAME("blocks.%u.moe.router.weight", l), ne, d, 1)) ||
        !(L->router = upload(m, p, (uint64_t)ne * d)) ||
        !split_weight(m, L->router, ne, d, &L->router_b, &L->router_s))
        return 0;
    p = optional(get, ctx, NAME("blocks.%u.moe._qb_bias", l), ne, 1, &bad);
    if (bad || (p && !(L->qb = upload(m, p, ne)))) return 0;
    const uint64_t per = (uint64_t)dff * d;
    const float** w12 = (const float**)calloc(2 * ne, sizeof(float*));
    const float** w3 = (const float**)calloc(ne, sizeof(float*));
    uint64_t* n12 = (uint64_t*)calloc(2 * ne, sizeof(uint64_t));
    int ok = w12 && w3 && n12;
    if (!ok) set_err("host allocation failed");
    for (uint32_t e = 0; ok && e < ne; e++) {
        n12[2 * e] = n12[2 * e + 1] = per;
        ok = (w12[2 * e] = tensor(get, ctx, NAME("blocks.%u.moe.experts.%u.w1.weight", l, e), dff, d, 1)) &&
             (w12[2 * e + 1] = tensor(get, ctx, NAME("blocks.%u.moe.experts.%u.w2.weight", l, e), dff, d, 1)) &&
             (w3[e] = tensor(get, ctx, NAME("blocks.%u.moe.experts.%u.w3.weight", l, e), d, dff, 1));
    }
    if (ok) ok = (L->w12 = upload_cat(m, w12, n12, (int)(2 * ne))) != NULL;
    if (ok) {
        for (uint32_t e = 0; e < ne; e++) n12[e] = per;
        ok = (L->w3 = upload_cat(m, w3, n12, (int)ne)) != NULL;
    }
    /* the experts' split form for the prefill's grouped GEMMs (twice the
     * experts' bytes); TGKV_MOE_GEMM=0 keeps the CUDA-core expert kernels */
    if (ok && moe_gemm_on())
        ok = split_weight(m, L->w12, (uint64_t)ne * 2 * dff, d, &L->w12_b, &L->w12_s) &&
             split_weight(m, L->w3, (uint64_t)ne * d, dff, &L->w3_b, &L->w3_s);
    free(w12);
    free(w3);
    free(n12);
#undef NAME
    return ok;
}

TGFwdModel* tg_fwd_create(const TGFwdConfig* cfg, TGFwdWeightFn get, void* ctx) {
    if (!cfg || !get) { set_err("null argument"); return NULL; }
    TGFwdConfig c = *cfg;
    if (!c.n_kv_heads) c.n_kv_heads = c.n_heads;
    if (!c.n_layers || !c.d_model || !c.n_heads || !c.vocab_size || !c.max_seq_len) {
        set_err("n_layers, d_model, n_heads, vocab_size and max_seq_len must be positive");
        return NULL;
    }
    if (!c.head_dim) c.head_dim = c.d_model / c.n_heads;
    if (c.n_kv_heads > c.n_heads || c.n_heads % c.n_kv_heads) {
        set_err("n_heads %u is not a multiple of n_kv_heads %u", c.n_heads, c.n_kv_heads);
        return NULL;
    }
    if (!tg_cuda_kv_attn_supported(0, c.head_dim)) {
        set_err("head_dim %u has no fp32 attention kernel (32, 64 or 128)", c.head_dim);
        return NULL;
    }
    if (c.d_model % 4 || !c.d_ff || c.d_ff % 4) {
        set_err("d_model and d_ff must be positive multiples of 4");
        return NULL;
    }
    if (c.n_experts > 16 || (c.n_experts && (!c.n_activated || c.n_activated > 8 ||
                                             c.n_activated > c.n_experts))) {
        set_err("MoE needs 1..16 experts and top-1..8 (got %u, %u)", c.n_experts, c.n_activated);
        return NULL;
    }
    if (!(c.rope_theta > 0.f)) { set_err("rope_theta must be positive"); return NULL; }
    if (!tg_gpu_backend_init() || !tg_cuda_kv_init()) {
        set_err("no CUDA device: %s", tg_gpu_backend_reason());
        return NULL;
    }

    TGFwdModel* m = (TGFwdModel*)calloc(1, sizeof(TGFwdModel));
    if (!m) { set_err("host allocation failed"); return NULL; }
    pthread_mutex_init(&m->mu, NULL);
    pthread_mutex_init(&m->bmu, NULL);
    pthread_mutex_init(&m->pmu, NULL);
    pthread_cond_init(&m->bcv, NULL);
    m->c = c;
    m->hd = c.head_dim;
    m->nkv = c.n_kv_heads;
    m->q_dim = c.n_heads * c.head_dim;
    m->kv_dim = c.n_kv_heads * c.head_dim;
    m->qkv_dim = m->q_dim + 2 * m->kv_dim;
    m->max_slots = 16;
    {
        const char* e = getenv("TGAI_CUDA_KV_SLOTS");
        if (e && e[0]) { int v = atoi(e); if (v >= 1 && v <= 64) m->max_slots = (uint32_t)v; }
    }
    m->slots = (Slot*)calloc(m->max_slots, sizeof(Slot));
    m->L = (Layer*)calloc(c.n_layers, sizeof(Layer));
    if (!m->slots || !m->L) { set_err("host allocation failed"); goto fail; }

    {   /* embedding: rows beyond vocab_size are never read (tgai_engine.c:4397-4412) */
        uint32_t shape[2] = {0, 0};
        const float* e = get(ctx, "token_embedding.weight", shape);
        if (!e) { set_err("missing weight token_embedding.weight"); goto fail; }
        if (shape[1] != c.d_model || !shape[0]) {
            set_err("token_embedding.weight has shape [%u, %u], expected [*, %u]", shape[0],
                    shape[1], c.d_model);
            goto fail;
        }
        m->rows = shape[0] < c.vocab_size ? shape[0] : c.vocab_size;
        if (c.unk_id < 0 || (uint32_t)c.unk_id >= m->rows) {
            set_err("unk_id %d is outside the %u embedding rows", c.unk_id, m->rows);
            goto fail;
        }
        if (!(m->emb = upload(m, e, (uint64_t)m->rows * c.d_model))) goto fail;
        /* the LM head is a GEMV of the staged row where d fits; else the GEMM */
        if (!decode_fits(1, c.d_model) &&
            !split_weight(m, m->emb, m->rows, c.d_model, &m->emb_b, &m->emb_s))
            goto fail;
        const float* f = tensor(get, ctx, "final_norm.weight", c.d_model, 1, 1);
        if (!f || !(m->fnorm = upload(m, f, c.d_model))) goto fail;
    }
    for (uint32_t l = 0; l < c.n_layers; l++)
        if (!load_layer(m, l, get, ctx)) goto fail;
    {   /* RoPE tables of every position, the engine's formula (no context extension) */
        const uint64_t n = (uint64_t)c.max_seq_len * (c.head_dim / 2);
        float* cs = (float*)malloc(n * sizeof(float));
        float* sn = (float*)malloc(n * sizeof(float));
        int ok = cs && sn &&
                 tg_kv_rope_tables(c.rope_theta, c.head_dim, 0, c.max_seq_len, 0, c.max_seq_len,
                                   cs, sn, NULL);
        if (ok) ok = (m->cs = upload(m, cs, n)) && (m->sn = upload(m, sn, n));
        else set_err("RoPE tables: %s", tg_kv_last_error());
        free(cs);
        free(sn);
        if (!ok) goto fail;
    }
    if (tgkv_fwd_step_supported(c.d_model, c.n_heads, m->nkv, m->hd, c.d_ff, c.n_experts,
                                c.n_activated)) {
        /* the layer table of the one-launch decode step */
        TGFwdStepLayer* t = (TGFwdStepLayer*)calloc(c.n_layers, sizeof(TGFwdStepLayer));
        if (!t) { set_err("host allocation failed"); goto fail; }
        for (uint32_t l = 0; l < c.n_layers; l++) {
            const Layer* L = &m->L[l];
            t[l] = (TGFwdStepLayer){L->ln1, L->ln2, L->wqkv, L->bqkv, L->wo, L->w12, L->w3,
                                    L->router, L->qb};
        }
        const size_t b = (size_t)c.n_layers * sizeof(TGFwdStepLayer);
        m->step_layers = (TGFwdStepLayer*)tg_cuda_kv_malloc(b);
        const int ok = m->step_layers && tg_cuda_kv_h2d(m->step_layers, t, b, NULL);
        free(t);
        if (!ok) { set_err("step layer table: %s", tg_cuda_kv_last_error()); goto fail; }
    }
    /* the weight splits ran on the default stream; the slots' streams do not
     * wait for it */
    if (!tg_cuda_kv_sync(NULL)) { set_err("weight split: %s", tg_cuda_kv_last_error()); goto fail; }
    return m;
fail:
    tg_fwd_destroy(m);
    return NULL;
}

uint64_t tg_fwd_weight_bytes(const TGFwdModel* m) { return m ? m->wbytes : 0; }

/* ---- slots ---------------------------------------------------------------- */
static void slot_free_ws(Slot* s) {
    float** f[] = {&s->x, &s->ln, &s->qkv, &s->q, &s->attn, &s->ab, &s->h, &s->router,
                   &s->top_w, &s->y, &s->abig, &s->asmall};
    for (size_t i = 0; i < sizeof(f) / sizeof(f[0]); i++) { tg_cuda_kv_free(*f[i]); *f[i] = NULL; }
    tg_cuda_kv_free(s->top_ids);
    tg_cuda_kv_free(s->ids);
    tg_cuda_kv_free(s->counts);
    tg_cuda_kv_free(s->lists);
    tg_cuda_kv_free(s->moe_off);
    tg_cuda_kv_free(s->moe_rows);
    s->top_ids = s->ids = NULL;
    s->counts = s->lists = s->moe_off = s->moe_rows = NULL;
    tgkv_fwd_host_free(s->h_ids);
    s->h_ids = NULL;
    s->cap = 0;
}

static void slot_release_mem(TGFwdModel* m, Slot* s) {
    if (s->stream) tg_cuda_kv_sync(s->stream);
    slot_free_ws(s);
    tg_cuda_kv_free(s->step_kvc);
    tg_cuda_kv_free(s->step_part);
    tg_cuda_kv_free(s->step_state);
    tgkv_fwd_host_free(s->h_step);
    s->step_kvc = NULL;
    s->step_part = NULL;
    s->step_state = NULL;
    s->h_step = NULL;
    if (s->kv) {
        for (uint32_t l = 0; l < m->c.n_layers; l++) tg_kv_destroy(s->kv[l]);
        free(s->kv);
        s->kv = NULL;
    }
    tg_cuda_kv_free(s->logits);
    s->logits = NULL;
    tgkv_fwd_host_free(s->h_logits);
    s->h_logits = NULL;
    if (s->stream) tg_cuda_kv_stream_destroy(s->stream);
    s->stream = NULL;
    s->used = 0;
    s->key = NULL;
}

/* Workspaces for `need` token rows (grown by doubling, never shrunk). */
static int slot_reserve(TGFwdModel* m, Slot* s, uint32_t need) {
    if (need <= s->cap) return 1;
    uint32_t cap = s->cap ? s->cap : 16;
    while (cap < need) cap *= 2;
    if (s->stream) tg_cuda_kv_sync(s->stream);
    slot_free_ws(s);
    const uint64_t d = m->c.d_model, dff = m->c.d_ff, ne = m->c.n_experts, na = m->c.n_activated;
    const uint64_t pairs = (uint64_t)cap * (ne ? na : 1);
    s->x = (float*)tg_cuda_kv_malloc(cap * d * 4);
    s->ln = (float*)tg_cuda_kv_malloc(cap * d * 4);
    s->qkv = (float*)tg_cuda_kv_malloc((uint64_t)cap * m->qkv_dim * 4);
    s->q = (float*)tg_cuda_kv_malloc((uint64_t)cap * m->q_dim * 4);
    s->attn = (float*)tg_cuda_kv_malloc((uint64_t)cap * m->q_dim * 4);
    s->h = (float*)tg_cuda_kv_malloc(pairs * dff * 4);
    s->ids = (int32_t*)tg_cuda_kv_malloc((uint64_t)cap * 4);
    s->h_ids = (int32_t*)tgkv_fwd_host_alloc((uint64_t)cap * 4);
    uint64_t kmax = d > m->q_dim ? d : m->q_dim;
    if (dff > kmax) kmax = dff;
    /* split GEMM inputs: token rows, or the MoE's packed (token, expert) rows */
    s->abig = (float*)tg_cuda_kv_malloc(pairs * kmax * 4);
    s->asmall = (float*)tg_cuda_kv_malloc(pairs * kmax * 4);
    int ok = s->x && s->ln && s->qkv && s->q && s->attn && s->h && s->ids && s->h_ids &&
             s->abig && s->asmall;
    if (ne == 0) {
        s->ab = (float*)tg_cuda_kv_malloc(cap * 2 * dff * 4);
        ok = ok && s->ab;
    } else {
        s->router = (float*)tg_cuda_kv_malloc(cap * ne * 4);
        s->top_w = (float*)tg_cuda_kv_malloc(pairs * 4);
        s->top_ids = (int32_t*)tg_cuda_kv_malloc(pairs * 4);
        s->y = (float*)tg_cuda_kv_malloc(pairs * d * 4);
        s->counts = (uint32_t*)tg_cuda_kv_malloc(ne * 4);
        s->lists = (uint32_t*)tg_cuda_kv_malloc(ne * pairs * 4);
        ok = ok && s->router && s->top_w && s->top_ids && s->y && s->counts && s->lists;
        if (m->L[0].w12_b) {              /* the grouped expert GEMMs' workspaces */
            s->ab = (float*)tg_cuda_kv_malloc(pairs * 2 * dff * 4);
            s->moe_off = (uint32_t*)tg_cuda_kv_malloc(16 * 4);
            s->moe_rows = (uint32_t*)tg_cuda_kv_malloc(pairs * 4);
            ok = ok && s->ab && s->moe_off && s->moe_rows;
        }
    }
    if (!ok) {
        slot_free_ws(s);
        set_err("workspace for %u tokens: allocation failed", cap);
        return 0;
    }
    s->cap = cap;
    return 1;
}

static int slot_init(TGFwdModel* m, Slot* s) {
    s->stream = tg_cuda_kv_stream_create();
    if (!s->stream) { set_err("stream: %s", tg_cuda_kv_last_error()); return 0; }
    s->kv = (TGKvCache**)calloc(m->c.n_layers, sizeof(TGKvCache*));
    if (!s->kv) { set_err("host allocation failed"); return 0; }
    for (uint32_t l = 0; l < m->c.n_layers; l++) {
        s->kv[l] = tg_kv_create_ex(m->c.max_seq_len, m->nkv, m->hd, TG_KV_F32);
        if (!s->kv[l]) { set_err("KV cache of layer %u: %s", l, tg_kv_last_error()); return 0; }
    }
    s->logits = (float*)tg_cuda_kv_malloc((uint64_t)m->c.vocab_size * 4);
    s->h_logits = (float*)tgkv_fwd_host_alloc((uint64_t)m->c.vocab_size * 4);
    if (!s->logits || !s->h_logits) { set_err("logits buffers: allocation failed"); return 0; }
    memset(s->h_logits, 0, (size_t)m->c.vocab_size * 4);
    s->last_pos = -1;
    s->kv_hi = 0;
    return slot_reserve(m, s, 16);
}

static Slot* find_slot(const TGFwdModel* m, const void* key) {
    for (uint32_t i = 0; i < m->max_slots; i++)
        if (m->slots[i].used && m->slots[i].key == key) return &m->slots[i];
    return NULL;
}

static Slot* slot_get(TGFwdModel* m, const void* key) {
    pthread_mutex_lock(&m->mu);
    Slot* s = find_slot(m, key);
    if (!s) {
        int had_room = 0;
        for (uint32_t i = 0; i < m->max_slots; i++) {
            if (m->slots[i].used) continue;
            had_room = 1;
            s = &m->slots[i];
            memset(s, 0, sizeof(*s));
            s->used = 1;
            s->key = key;
            s->id = (int)i;
            if (slot_init(m, s)) {
                m->live++;
            } else {
                slot_release_mem(m, s);         /* slot_init's message stands */
                s = NULL;
            }
            break;
        }
        if (!s) {
            if (!had_room) set_err("no free slot (%u live of %u)", m->live, m->max_slots);
            m->rejects++;
        }
    }
    pthread_mutex_unlock(&m->mu);
    return s;
}

/* Zero the slot's KV and forget its positions. */
static int slot_clear(TGFwdModel* m, Slot* s) {
    for (uint32_t l = 0; l < m->c.n_layers; l++) {
        if (!tg_cuda_kv_memset(tg_kv_device_handle(s->kv[l]), 0, (size_t)tg_kv_bytes(s->kv[l]),
                               s->stream)) {
            set_err("KV clear: %s", tg_cuda_kv_last_error());
            return 0;
        }
        tg_kv_reset(s->kv[l]);
    }
    s->last_pos = -1;
    s->kv_hi = 0;
    return 1;
}

int tg_fwd_reset_slot(TGFwdModel* m, const void* key) {
    if (!m) return 0;
    pthread_mutex_lock(&m->mu);
    Slot* s = find_slot(m, key);
    int ok = s && slot_clear(m, s) && tg_cuda_kv_sync(s->stream);
    pthread_mutex_unlock(&m->mu);
    return ok;
}

int tg_fwd_free_slot(TGFwdModel* m, const void* key) {
    if (!m) return 0;
    pthread_mutex_lock(&m->pmu);        /* no batch is running over its caches */
    pthread_mutex_lock(&m->mu);
    Slot* s = find_slot(m, key);
    if (s) {
        plans_drop_slot(m, s->id);
        slot_release_mem(m, s);
        m->live--;
    }
    pthread_mutex_unlock(&m->mu);
    pthread_mutex_unlock(&m->pmu);
    return s != NULL;
}

void tg_fwd_reset_all(TGFwdModel* m) {
    if (!m) return;
    pthread_mutex_lock(&m->mu);
    for (uint32_t i = 0; i < m->max_slots; i++)
        if (m->slots[i].used && slot_clear(m, &m->slots[i])) tg_cuda_kv_sync(m->slots[i].stream);
    pthread_mutex_unlock(&m->mu);
}

uint32_t tg_fwd_slot_count(const TGFwdModel* m) { return m ? m->live : 0; }

int tg_fwd_slot_last_pos(const TGFwdModel* m, const void* key) {
    if (!m) return -1;
    pthread_mutex_lock((pthread_mutex_t*)&m->mu);
    const Slot* s = find_slot(m, key);
    const int r = s ? s->last_pos : -1;
    pthread_mutex_unlock((pthread_mutex_t*)&m->mu);
    return r;
}

/* Slot index of key, or -1; and the rejected-request count (the reference
 * bridge's tg_gpu_kv_slot_of / _rejects). */
HIDDEN int tgkv_fwd_slot_index(TGFwdModel* m, const void* key) {
    if (!m) return -1;
    pthread_mutex_lock(&m->mu);
    const Slot* s = find_slot(m, key);
    const int r = s ? s->id : -1;
    pthread_mutex_unlock(&m->mu);
    return r;
}
HIDDEN long long tgkv_fwd_rejects(const TGFwdModel* m) { return m ? m->rejects : 0; }
HIDDEN uint32_t tgkv_fwd_max_slots(const TGFwdModel* m) { return m ? m->max_slots : 0; }

/* ---- forward -------------------------------------------------------------- */
#define CHECK_LAUNCH(expr)                                                      \
    do {                                                                        \
        const int _e = (expr);                                                  \
        t_launches++;                                                           \
        if (_e) { set_err("%s failed (CUDA error %d)", #expr, _e); return 0; }  \
    } while (0)

/* out[M][N] (row stride ldo) = x[M][K] (row stride ldx) . W[N][K]^T, or +=,
 * on the tensor cores at fp32-product accuracy (tgkv_gemm.cu): x is split
 * into its tf32 part and remainder in the slot's workspace, W comes split
 * (wb, ws) from model creation. */
static int gemm(Slot* s, uint32_t M, uint32_t N, uint32_t K, const float* x, uint32_t ldx,
                const float* wb, const float* ws, float* out, uint32_t ldo, int accumulate) {
    CHECK_LAUNCH(tgkv_split_tf32(x, ldx, s->abig, s->asmall, K, M, K, s->stream));
    TGGemmParams p;
    if (!tgkv_gemm_encode(&p, s->abig, s->asmall, K, wb, ws, K, out, ldo, M, N, K, accumulate,
                          tgkv_bridge_err_word())) {
        set_err("GEMM %u x %u x %u: unsupported shape or tensor map", M, N, K);
        return 0;
    }
    CHECK_LAUNCH(tgkv_gemm_launch(&p, s->stream));
    return 1;
}

/* Attention half of a layer: q/k/v, RoPE + KV append, attention.  Leaves the
 * attention output in s->attn. */
/* A decode step's launches may prefetch the weights of a later launch into
 * L2.  TGKV_PREFETCH is a mask of the sites: 1 Wo (by the Q/K/V launch),
 * 2 the routed experts' W3 (by the W1/W2 launch), 4 the next layer's Q/K/V
 * (by the W3 launch), 8 the dense FFN's W1/W2 and W3; unset or 0: none.
 * NULL when the site is off. */
static const float* pf(const float* w, int site) {
    static int mask = -1;
    int v = __atomic_load_n(&mask, __ATOMIC_RELAXED);
    if (v < 0) {
        const char* e = getenv("TGKV_PREFETCH");
        v = e && e[0] ? atoi(e) & 15 : 0;
        __atomic_store_n(&mask, v, __ATOMIC_RELAXED);
    }
    return (v & site) ? w : NULL;
}

static int attn_half(TGFwdModel* m, Slot* s, const Layer* L, TGKvCache* kv, uint32_t seq,
                     uint32_t pos, int decode) {
    const TGFwdConfig* c = &m->c;
    const uint32_t d = c->d_model;
    void* st = s->stream;
    if (decode) {
        /* norm + projection + bias + RoPE + KV append in one launch; it
         * prefetches Wo for the out projection after the attention */
        CHECK_LAUNCH(tgkv_fwd_dec_qkv_rope(L->wqkv, s->x, L->ln1, L->bqkv, m->cs, m->sn, s->q,
                                           (float*)tg_kv_device_handle(kv), seq, d, m->q_dim,
                                           m->kv_dim, m->hd, pos, c->max_seq_len, pf(L->wo, 1),
                                           (uint64_t)d * m->q_dim, st));
    } else {
        CHECK_LAUNCH(tgkv_fwd_rmsnorm(s->ln, s->x, L->ln1, seq, d, d, d, 1e-6f, st));
        if (!gemm(s, seq, m->qkv_dim, d, s->ln, d, L->wqkv_b, L->wqkv_s, s->qkv, m->qkv_dim, 0)) return 0;
        if (L->bqkv) CHECK_LAUNCH(tgkv_fwd_bias(s->qkv, L->bqkv, seq, m->qkv_dim, st));
        t_launches++;
        if (!tg_cuda_kv_rope_append(TG_KV_F32, s->qkv, m->cs, m->sn, tg_kv_device_handle(kv),
                                    s->q, seq, c->n_heads, m->nkv, m->hd, pos, c->max_seq_len,
                                    st)) {
            set_err("RoPE + append: %s", tg_cuda_kv_last_error());
            return 0;
        }
    }
    tg_kv_advance(kv, seq);
    if (!tg_kv_attention(kv, s->q, s->attn, c->n_heads, seq, st)) {
        set_err("attention: %s", tg_kv_last_error());
        return 0;
    }
    t_launches += tg_cuda_kv_attn_last_launches();
    return 1;
}

/* The rest of a decode layer after the attention (attention output in
 * s->attn, R token rows): out projection + residual, then the FFN, each with
 * its norm fused; each launch prefetches the weights of a later one (the
 * routed experts' W3 once the router has chosen; the next layer's Q/K/V). */
static int decode_tail(TGFwdModel* m, Slot* s, uint32_t l, uint32_t R) {
    const Layer* L = &m->L[l];
    const TGFwdConfig* c = &m->c;
    const uint32_t d = c->d_model, dff = c->d_ff, ne = c->n_experts, na = c->n_activated;
    void* st = s->stream;
    const Layer* Ln = l + 1 < c->n_layers ? &m->L[l + 1] : NULL;
    const float* next_qkv = Ln ? pf(Ln->wqkv, 4) : NULL;
    const uint64_t next_qkv_n = (uint64_t)m->qkv_dim * d;
    if (ne == 0) {
        CHECK_LAUNCH(tgkv_fwd_dec_gemv(1, L->wo, s->attn, m->q_dim, NULL, NULL, s->x, d, R, d,
                                       m->q_dim, 0, pf(L->w12, 8), (uint64_t)2 * dff * d, st));
        CHECK_LAUNCH(tgkv_fwd_dec_gemv(2, L->w12, s->x, d, L->ln2, NULL, s->h, dff, R, dff,
                                       d, 1, pf(L->w3, 8), (uint64_t)d * dff, st));
        CHECK_LAUNCH(tgkv_fwd_dec_gemv(1, L->w3, s->h, dff, NULL, NULL, s->x, d, R, d, dff,
                                       0, next_qkv, next_qkv_n, st));
        return 1;
    }
    CHECK_LAUNCH(tgkv_fwd_dec_gemv(1, L->wo, s->attn, m->q_dim, NULL, NULL, s->x, d, R, d,
                                   m->q_dim, 0, NULL, 0, st));
    CHECK_LAUNCH(tgkv_fwd_dec_moe_w12(s->x, L->ln2, L->router, L->qb, L->w12, s->top_ids,
                                      s->top_w, s->h, R, d, dff, ne, na, pf(L->w3, 2), st));
    CHECK_LAUNCH(tgkv_fwd_dec_w3_combine(L->w3, s->h, s->top_ids, s->top_w, s->x, R, d, dff,
                                         ne, na, next_qkv, next_qkv_n, st));
    return 1;
}

static int run_layer(TGFwdModel* m, Slot* s, uint32_t l, uint32_t seq, uint32_t pos) {
    const Layer* L = &m->L[l];
    const TGFwdConfig* c = &m->c;
    const uint32_t d = c->d_model, dff = c->d_ff, ne = c->n_experts, na = c->n_activated;
    void* st = s->stream;
    const int decode = decode_fits(seq, d) && decode_fits(seq, m->q_dim) && decode_fits(seq, dff);
    if (!attn_half(m, s, L, s->kv[l], seq, pos, decode)) return 0;
    if (decode) return decode_tail(m, s, l, seq);
    if (!gemm(s, seq, d, m->q_dim, s->attn, m->q_dim, L->wo_b, L->wo_s, s->x, d, 1)) return 0;
    CHECK_LAUNCH(tgkv_fwd_rmsnorm(s->ln, s->x, L->ln2, seq, d, d, d, 1e-6f, st));
    if (ne == 0) {
        if (!gemm(s, seq, 2 * dff, d, s->ln, d, L->w12_b, L->w12_s, s->ab, 2 * dff, 0)) return 0;
        CHECK_LAUNCH(tgkv_fwd_silu_mul(s->h, s->ab, seq, dff, 1, st));
        return gemm(s, seq, d, dff, s->h, dff, L->w3_b, L->w3_s, s->x, d, 1);
    }
    if (!gemm(s, seq, ne, d, s->ln, d, L->router_b, L->router_s, s->router, ne, 0)) return 0;
    if (!tg_cuda_kv_memset(s->counts, 0, (size_t)ne * 4, st)) {
        set_err("memset: %s", tg_cuda_kv_last_error());
        return 0;
    }
    CHECK_LAUNCH(tgkv_fwd_route(s->router, L->qb, s->top_ids, s->top_w, s->counts, s->lists,
                                seq, ne, na, st));
    if (L->w12_b) {
        /* the experts on the tensor cores: the (token, expert) pairs packed by
         * expert, one grouped GEMM for W1/W2, SiLU, one for W3 whose rows
         * land at their pair's row of y */
        const uint32_t pr = seq * na;
        TGGemmParams gp;
        CHECK_LAUNCH(tgkv_moe_pack_split(s->counts, s->lists, s->ln, d, seq, ne, na, s->abig,
                                         s->asmall, s->moe_off, s->moe_rows, st));
        if (!tgkv_gemm_encode_grouped(&gp, s->abig, s->asmall, pr, L->w12_b, L->w12_s, ne,
                                      2 * dff, d, s->ab, 2 * dff, s->counts, s->moe_off, NULL,
                                      seq, tgkv_bridge_err_word())) {
            set_err("expert GEMM (W1/W2): tensor map encode failed");
            return 0;
        }
        CHECK_LAUNCH(tgkv_gemm_launch(&gp, st));
        CHECK_LAUNCH(tgkv_moe_silu_split(s->ab, s->counts, ne, pr, dff, s->abig, s->asmall, st));
        if (!tgkv_gemm_encode_grouped(&gp, s->abig, s->asmall, pr, L->w3_b, L->w3_s, ne, d, dff,
                                      s->y, d, s->counts, s->moe_off, s->moe_rows, seq,
                                      tgkv_bridge_err_word())) {
            set_err("expert GEMM (W3): tensor map encode failed");
            return 0;
        }
        CHECK_LAUNCH(tgkv_gemm_launch(&gp, st));
    } else {
        CHECK_LAUNCH(tgkv_fwd_expert_w12(L->w12, s->ln, s->h, s->counts, s->lists, seq, ne, na,
                                         d, dff, st));
        CHECK_LAUNCH(tgkv_fwd_expert_w3(L->w3, s->h, s->y, s->counts, s->lists, seq, ne, na, d,
                                        dff, st));
    }
    CHECK_LAUNCH(tgkv_fwd_moe_combine(s->x, s->y, s->top_ids, s->top_w, seq, d, ne, na, st));
    return 1;
}

/* One-token decode steps run as one cooperative launch over all layers
 * (tgkv_fwd_decode_step) where the model fits it; TGKV_FWD_STEP=0 takes them
 * through the per-layer launches instead. */
static int step_on(void) {
    const char* e = getenv("TGKV_FWD_STEP");
    return !(e && e[0] == '0');
}

/* All layers of one decode token at position pos (x holds its embedding);
 * the error word comes back with the logits.  1 queued, 0 failed, -1 the
 * device refused the grid (nothing queued but a zeroing of the step state;
 * the caller runs the per-layer launches). */
static int run_step(TGFwdModel* m, Slot* s, uint32_t pos) {
    const TGFwdConfig* c = &m->c;
    void* st = s->stream;
    const uint32_t state_n = kTgStepStateWords;
    if (!s->step_kvc) {
        float** h = (float**)malloc(c->n_layers * sizeof(float*));
        if (!h) { set_err("host allocation failed"); return 0; }
        for (uint32_t l = 0; l < c->n_layers; l++) h[l] = (float*)tg_kv_device_handle(s->kv[l]);
        s->step_kvc = (float**)tg_cuda_kv_malloc(c->n_layers * sizeof(float*));
        int ok = s->step_kvc && tg_cuda_kv_h2d(s->step_kvc, h, c->n_layers * sizeof(float*), NULL);
        free(h);
        s->step_part = (float*)tg_cuda_kv_malloc(
            tgkv_fwd_step_part_floats(c->n_heads, m->nkv, m->hd) * sizeof(float));
        s->step_state = (uint32_t*)tg_cuda_kv_malloc(state_n * 4);
        s->h_step = (int32_t*)tgkv_fwd_host_alloc(16);
        if (!ok || !s->step_part || !s->step_state || !s->h_step) {
            /* all or nothing: a later call allocates them again from scratch */
            tg_cuda_kv_free(s->step_kvc);
            tg_cuda_kv_free(s->step_part);
            tg_cuda_kv_free(s->step_state);
            tgkv_fwd_host_free(s->h_step);
            s->step_kvc = NULL;
            s->step_part = NULL;
            s->step_state = NULL;
            s->h_step = NULL;
            set_err("decode step buffers: allocation failed");
            return 0;
        }
    }
    if (!tg_cuda_kv_memset(s->step_state, 0, state_n * 4, st)) {
        set_err("memset: %s", tg_cuda_kv_last_error());
        return 0;
    }
    TGFwdStepParams p;
    memset(&p, 0, sizeof(p));
    p.layers = m->step_layers;
    p.kvc = s->step_kvc;
    p.x = s->x;
    p.q = s->q;
    p.attn = s->attn;
    p.h = s->h;
    p.part = s->step_part;
    p.state = s->step_state;
    p.cs = m->cs;
    p.sn = m->sn;
    p.n_layers = c->n_layers;
    p.d = c->d_model;
    p.n_heads = c->n_heads;
    p.n_kv_heads = m->nkv;
    p.head_dim = m->hd;
    p.dff = c->d_ff;
    p.ne = c->n_experts;
    p.na = c->n_activated;
    p.pos = pos;
    p.max_seq = c->max_seq_len;
    p.sx_floats = c->d_model > m->q_dim ? c->d_model : m->q_dim;
    p.scale = 1.0f / sqrtf((float)m->hd);
    const int e = tgkv_fwd_decode_step(&p, st);
    if (e < 0) {
        __atomic_store_n(&m->step_refused, 1, __ATOMIC_RELAXED);
        return -1;
    }
    t_launches++;
    if (e) { set_err("decode step launch failed (CUDA error %d)", e); return 0; }
    for (uint32_t l = 0; l < c->n_layers; l++) tg_kv_advance(s->kv[l], 1);
    s->h_step[0] = -1;
    if (!tg_cuda_kv_d2h(s->h_step, s->step_state + 1, 4, st)) {
        set_err("decode step status: %s", tg_cuda_kv_last_error());
        return 0;
    }
    return 1;
}

static int run_forward(TGFwdModel* m, Slot* s, const int32_t* ids, uint32_t seq, uint32_t pos) {
    const TGFwdConfig* c = &m->c;
    const uint32_t d = c->d_model;
    void* st = s->stream;
    if (!slot_reserve(m, s, seq)) return 0;
    /* a gap (positions the slot never wrote) clears it: cuda/tgai_cuda.cu:1703-1711 */
    if (s->kv_hi > 0 && (int)pos > s->last_pos && !slot_clear(m, s)) return 0;
    for (uint32_t l = 0; l < c->n_layers; l++) {   /* keep [0, pos): the LCP of the caller */
        tg_kv_reset(s->kv[l]);
        tg_kv_advance(s->kv[l], pos);
    }
    memcpy(s->h_ids, ids, (size_t)seq * 4);
    if (!tg_cuda_kv_h2d(s->ids, s->h_ids, (size_t)seq * 4, st)) {
        set_err("ids upload: %s", tg_cuda_kv_last_error());
        return 0;
    }
    CHECK_LAUNCH(tgkv_fwd_embed(s->x, m->emb, s->ids, seq, d, m->rows, c->unk_id, st));
    /* The step's attention splits a KV head's context into at most
     * kTgStepMaxTasks warp tasks; past 32 positions a task (4096 in all) the
     * tasks grow long and few warps stream the cache, where the per-layer
     * path's split attention kernel keeps HBM busy instead. */
    int step = seq == 1 && m->step_layers && step_on() &&
               (uint64_t)pos + 1 <= (uint64_t)kTgStepMaxTasks * 32 &&
               !__atomic_load_n(&m->step_refused, __ATOMIC_RELAXED);
    if (step) {
        const int r = run_step(m, s, pos);
        if (!r) return 0;
        step = r > 0;
    }
    if (!step)
        for (uint32_t l = 0; l < c->n_layers; l++)
            if (!run_layer(m, s, l, seq, pos)) return 0;
    /* final norm of the last row, then the tied-embedding LM head */
    const float* xl = s->x + (uint64_t)(seq - 1) * d;
    if (decode_fits(1, d)) {
        CHECK_LAUNCH(tgkv_fwd_dec_gemv(0, m->emb, xl, d, m->fnorm, NULL, s->logits, m->rows, 1,
                                       m->rows, d, 0, NULL, 0, st));
    } else {
        CHECK_LAUNCH(tgkv_fwd_rmsnorm(s->ln, xl, m->fnorm, 1, d, d, d, 1e-6f, st));
        if (!gemm(s, 1, m->rows, d, s->ln, d, m->emb_b, m->emb_s, s->logits, m->rows, 0)) return 0;
    }
    if (!tg_cuda_kv_d2h(s->h_logits, s->logits, (size_t)m->rows * 4, st) || !tg_cuda_kv_sync(st)) {
        set_err("forward: %s", tg_cuda_kv_last_error());
        return 0;
    }
    if (step && s->h_step[0] != 0) {
        set_err("decode step: grid barrier timed out (status %d)", s->h_step[0]);
        return 0;
    }
    s->last_pos = (int)(pos + seq);
    if (s->last_pos > s->kv_hi) s->kv_hi = s->last_pos;
    return 1;
}

/* ---- batched decode across slots -------------------------------------------
 * The reference bridge runs every slot on its own stream with no lock on
 * forward (cuda/tgai_cuda_bridge.c:147-162), so sequences served from
 * several threads decode side by side, each reading all the weights.  Here a
 * one-token forward joins a queue; the first thread to find no batch running
 * leads: it takes up to tgkv_fwd_decode_rows() queued requests of different
 * slots and runs them as ONE pass over the weights -- R token rows through
 * the per-layer decode kernels, the attention as one ragged launch over the
 * slots' caches with the K/V append fused in -- then wakes their threads.
 * A request that finds itself alone takes the single-sequence path (the
 * one-launch decode step).  Requests that arrive while a batch runs form the
 * next one, so a busy server batches by itself and an idle one adds no wait.
 * TGKV_FWD_BATCH=0 turns it off (every request runs alone, as before). */
static int batch_on(const TGFwdModel* m) {
    static int v = -1;
    int on = __atomic_load_n(&v, __ATOMIC_RELAXED);
    if (on < 0) {
        const char* e = getenv("TGKV_FWD_BATCH");
        on = !(e && e[0] == '0');
        __atomic_store_n(&v, on, __ATOMIC_RELAXED);
    }
    const uint32_t R = tgkv_fwd_decode_rows();
    return on && R >= 2 && decode_fits(R, m->c.d_model) && decode_fits(R, m->q_dim) &&
           decode_fits(R, m->c.d_ff);
}

/* The batch workspace, made by the first batch (caller holds pmu). */
static int batch_ready(TGFwdModel* m) {
    if (m->plans) return 1;
    const uint32_t R = tgkv_fwd_decode_rows();
    Slot* b = &m->bs;
    if (!b->stream && !(b->stream = tg_cuda_kv_stream_create())) {
        set_err("batch stream: %s", tg_cuda_kv_last_error());
        return 0;
    }
    if (!slot_reserve(m, b, R)) return 0;
    m->b_knew = (float*)tg_cuda_kv_malloc((uint64_t)R * m->kv_dim * 4);
    m->b_vnew = (float*)tg_cuda_kv_malloc((uint64_t)R * m->kv_dim * 4);
    m->b_pos = (uint32_t*)tg_cuda_kv_malloc((uint64_t)R * 4);
    m->b_logits = (float*)tg_cuda_kv_malloc((uint64_t)R * m->rows * 4);
    m->bh_pos = (uint32_t*)tgkv_fwd_host_alloc((uint64_t)R * 4);
    m->bh_logits = (float*)tgkv_fwd_host_alloc((uint64_t)R * m->rows * 4);
    struct BatchPlan* plans = (struct BatchPlan*)calloc(kPlanCache, sizeof(struct BatchPlan));
    if (!m->b_knew || !m->b_vnew || !m->b_pos || !m->b_logits || !m->bh_pos || !m->bh_logits ||
        !plans) {
        free(plans);
        set_err("batch workspace: allocation failed");
        return 0;
    }
    m->plans = plans;
    return 1;
}

/* The per-layer plans over the caches of slots rq[0..n) (ascending ids),
 * from the cache or made now (caller holds pmu). */
static TGKvBatch** batch_plans(TGFwdModel* m, BatchReq** rq, uint32_t n) {
    struct BatchPlan* lru = &m->plans[0];
    for (int i = 0; i < kPlanCache; i++) {
        struct BatchPlan* bp = &m->plans[i];
        if (bp->b && bp->n == n) {
            uint32_t j = 0;
            while (j < n && bp->ids[j] == rq[j]->s->id) j++;
            if (j == n) {
                bp->used = ++m->plan_clock;
                return bp->b;
            }
        }
        if (!bp->b || (lru->b && bp->used < lru->used)) lru = bp;
    }
    plan_drop(m, lru);
    lru->b = (TGKvBatch**)calloc(m->c.n_layers, sizeof(TGKvBatch*));
    if (!lru->b) { set_err("host allocation failed"); return NULL; }
    TGKvCache* cs[8];
    for (uint32_t l = 0; l < m->c.n_layers; l++) {
        for (uint32_t j = 0; j < n; j++) cs[j] = rq[j]->s->kv[l];
        if (!(lru->b[l] = tg_kv_batch_create(cs, n, m->c.n_heads))) {
            set_err("batch plan: %s", tg_kv_last_error());
            plan_drop(m, lru);
            return NULL;
        }
    }
    lru->n = n;
    for (uint32_t j = 0; j < n; j++) lru->ids[j] = rq[j]->s->id;
    lru->used = ++m->plan_clock;
    return lru->b;
}

/* One token of each of the n >= 2 requests (distinct slots, ascending ids)
 * through every layer in one pass; each slot's h_logits receives its row.
 * Caller holds pmu. */
static int run_batch(TGFwdModel* m, BatchReq** rq, uint32_t n) {
    const TGFwdConfig* c = &m->c;
    const uint32_t d = c->d_model;
    if (!batch_ready(m)) return 0;
    Slot* b = &m->bs;
    void* st = b->stream;
    for (uint32_t j = 0; j < n; j++) {
        Slot* s = rq[j]->s;
        const uint32_t pos = rq[j]->pos;
        /* each sequence's gap rule and LCP, as run_forward applies them */
        if (s->kv_hi > 0 && (int)pos > s->last_pos &&
            !(slot_clear(m, s) && tg_cuda_kv_sync(s->stream)))
            return 0;
        for (uint32_t l = 0; l < c->n_layers; l++) {
            tg_kv_reset(s->kv[l]);
            tg_kv_advance(s->kv[l], pos);
        }
        b->h_ids[j] = rq[j]->id;
        m->bh_pos[j] = pos;
    }
    TGKvBatch** plan = batch_plans(m, rq, n);
    if (!plan) return 0;
    if (!tg_cuda_kv_h2d(b->ids, b->h_ids, (size_t)n * 4, st) ||
        !tg_cuda_kv_h2d(m->b_pos, m->bh_pos, (size_t)n * 4, st)) {
        set_err("batch upload: %s", tg_cuda_kv_last_error());
        return 0;
    }
    CHECK_LAUNCH(tgkv_fwd_embed(b->x, m->emb, b->ids, n, d, m->rows, c->unk_id, st));
    for (uint32_t l = 0; l < c->n_layers; l++) {
        const Layer* L = &m->L[l];
        /* norm + Q/K/V rows + bias + RoPE at each row's position; K/V rows
         * for the attention launch, which appends them to each slot's cache */
        CHECK_LAUNCH(tgkv_fwd_dec_qkv_rows(L->wqkv, b->x, L->ln1, L->bqkv, m->cs, m->sn, b->q,
                                           m->b_knew, m->b_vnew, n, d, m->q_dim, m->kv_dim, m->hd,
                                           m->b_pos, c->max_seq_len, pf(L->wo, 1),
                                           (uint64_t)d * m->q_dim, st));
        if (!tg_kv_batch_decode(plan[l], b->q, m->b_knew, m->b_vnew, b->attn, st)) {
            set_err("batch attention: %s", tg_kv_last_error());
            return 0;
        }
        t_launches += tg_kv_batch_last_launches(plan[l]);
        if (!decode_tail(m, b, l, n)) return 0;
    }
    CHECK_LAUNCH(tgkv_fwd_dec_gemv(0, m->emb, b->x, d, m->fnorm, NULL, m->b_logits, m->rows, n,
                                   m->rows, d, 0, NULL, 0, st));
    if (!tg_cuda_kv_d2h(m->bh_logits, m->b_logits, (size_t)n * m->rows * 4, st) ||
        !tg_cuda_kv_sync(st)) {
        set_err("batch: %s", tg_cuda_kv_last_error());
        return 0;
    }
    for (uint32_t j = 0; j < n; j++) {
        Slot* s = rq[j]->s;
        memcpy(s->h_logits, m->bh_logits + (uint64_t)j * m->rows, (size_t)m->rows * 4);
        s->last_pos = (int)(rq[j]->pos + 1);
        if (s->last_pos > s->kv_hi) s->kv_hi = s->last_pos;
    }
    m->batched_tokens += n;
    m->batches++;
    return 1;
}

/* Run the taken requests: alone through run_forward, else as one batch. */
static void run_taken(TGFwdModel* m, BatchReq** rq, uint32_t n) {
    int ok;
    t_launches = 0;
    if (n == 1) {
        ok = run_forward(m, rq[0]->s, &rq[0]->id, 1, rq[0]->pos);
        if (!ok) tg_cuda_kv_sync(rq[0]->s->stream);
    } else {
        /* ascending slot ids: one plan per set of slots */
        for (uint32_t i = 1; i < n; i++)
            for (uint32_t j = i; j > 0 && rq[j - 1]->s->id > rq[j]->s->id; j--) {
                BatchReq* t = rq[j];
                rq[j] = rq[j - 1];
                rq[j - 1] = t;
            }
        pthread_mutex_lock(&m->pmu);
        ok = run_batch(m, rq, n);
        pthread_mutex_unlock(&m->pmu);
        if (!ok) tg_cuda_kv_sync(m->bs.stream);
    }
    for (uint32_t j = 0; j < n; j++) {
        rq[j]->ok = ok;
        rq[j]->launches = t_launches;
        if (!ok) snprintf(rq[j]->err, sizeof(rq[j]->err), "%s", t_err);
    }
}

static const float* forward_one(TGFwdModel* m, Slot* s, int32_t id, uint32_t pos) {
    BatchReq r;
    memset(&r, 0, sizeof(r));
    r.s = s;
    r.id = id;
    r.pos = pos;
    const uint32_t R = tgkv_fwd_decode_rows();
    pthread_mutex_lock(&m->bmu);
    for (BatchReq* q = m->bq_head; q; q = q->next)
        if (q->s == s) {
            pthread_mutex_unlock(&m->bmu);
            set_err("slot %d already has a forward in flight", s->id);
            return NULL;
        }
    if (m->bq_tail) m->bq_tail->next = &r;
    else m->bq_head = &r;
    m->bq_tail = &r;
    while (r.state != 2) {
        if (!m->b_leader && m->bq_head) {
            /* lead: take up to R requests from the head of the queue */
            m->b_leader = 1;
            BatchReq* take[8];
            uint32_t n = 0;
            while (m->bq_head && n < R && n < 8) {
                BatchReq* q = m->bq_head;
                m->bq_head = q->next;
                if (!m->bq_head) m->bq_tail = NULL;
                q->next = NULL;
                q->state = 1;
                take[n++] = q;
            }
            pthread_mutex_unlock(&m->bmu);
            run_taken(m, take, n);
            pthread_mutex_lock(&m->bmu);
            for (uint32_t j = 0; j < n; j++) take[j]->state = 2;
            m->b_leader = 0;
            pthread_cond_broadcast(&m->bcv);
            continue;
        }
        pthread_cond_wait(&m->bcv, &m->bmu);
    }
    pthread_mutex_unlock(&m->bmu);
    t_launches = r.launches;
    if (!r.ok) {
        set_err("%s", r.err);
        return NULL;
    }
    return s->h_logits;
}

const float* tg_fwd_forward(TGFwdModel* m, const void* key, const int32_t* ids,
                            uint32_t seq_len, uint32_t cache_pos) {
    t_launches = 0;
    if (!m || !ids || !seq_len) { set_err("null argument or empty sequence"); return NULL; }
    if ((uint64_t)cache_pos + seq_len > m->c.max_seq_len) {
        set_err("positions %u..%u exceed max_seq_len %u", cache_pos, cache_pos + seq_len - 1,
                m->c.max_seq_len);
        return NULL;
    }
    Slot* s = slot_get(m, key);
    if (!s) return NULL;
    if (seq_len == 1 && batch_on(m)) return forward_one(m, s, ids[0], cache_pos);
    if (!run_forward(m, s, ids, seq_len, cache_pos)) {
        tg_cuda_kv_sync(s->stream);
        return NULL;
    }
    return s->h_logits;
}

/* Tokens decoded in batches of two or more, and the number of those batches
 * (a report for tests and the bench). */
void tg_fwd_batch_stats(const TGFwdModel* m, uint64_t* tokens, uint64_t* batches) {
    if (tokens) *tokens = m ? (uint64_t)m->batched_tokens : 0;
    if (batches) *batches = m ? (uint64_t)m->batches : 0;
}

int tg_fwd_gemm_f32(uint32_t M, uint32_t N, uint32_t K, const float* x, uint32_t ldx,
                    const float* w, uint32_t ldw, float* out, uint32_t ldo, int accumulate,
                    void* stream) {
    t_launches = 0;
    if (!x || !w || !out || !M || !N || !K) { set_err("null argument or empty shape"); return 0; }
    if (K % 4 || ldx % 4 || ldw % 4 || ldx < K || ldw < K || ldo < N) {
        set_err("K, ldx and ldw must be multiples of 4, ldx, ldw >= K and ldo >= N");
        return 0;
    }
    if (!tg_cuda_kv_init()) { set_err("no CUDA device: %s", tg_cuda_kv_last_error()); return 0; }
    float* buf[4] = {NULL, NULL, NULL, NULL};
    const uint64_t na = (uint64_t)M * K, nw = (uint64_t)N * K;
    buf[0] = (float*)tg_cuda_kv_malloc(na * 4);
    buf[1] = (float*)tg_cuda_kv_malloc(na * 4);
    buf[2] = (float*)tg_cuda_kv_malloc(nw * 4);
    buf[3] = (float*)tg_cuda_kv_malloc(nw * 4);
    int ok = buf[0] && buf[1] && buf[2] && buf[3];
    if (!ok) set_err("split operands: device allocation failed");
    int e = 0;
    if (ok && ((e = tgkv_split_tf32(x, ldx, buf[0], buf[1], K, M, K, stream)) ||
               (e = tgkv_split_tf32(w, ldw, buf[2], buf[3], K, N, K, stream)))) {
        set_err("split failed (CUDA error %d)", e);
        ok = 0;
    }
    TGGemmParams p;
    if (ok && !tgkv_gemm_encode(&p, buf[0], buf[1], K, buf[2], buf[3], K, out, ldo, M, N, K,
                                accumulate, tgkv_bridge_err_word())) {
        set_err("GEMM %u x %u x %u: tensor map encode failed", M, N, K);
        ok = 0;
    }
    if (ok && (e = tgkv_gemm_launch(&p, stream))) {
        set_err("GEMM launch failed (CUDA error %d)", e);
        ok = 0;
    }
    t_launches = ok ? 3 : 0;
    if (!tg_cuda_kv_sync(stream) && ok) {
        set_err("GEMM: %s", tg_cuda_kv_last_error());
        ok = 0;
    }
    for (int i = 0; i < 4; i++) tg_cuda_kv_free(buf[i]);
    return ok;
}
