/*
 * llama-dense fixture runner for the CPU oracle.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Runs one Engine::step exactly as the reference CpuDevice would execute the
 * llama-dense command buffer, op by op, through the restated reference
 * kernels. The op sequence is the llama-dense lowering contract
 * (docs/ARCH-0006:157-211, op usage docs/ARCH-0004:252-276):
 *
 *   Gather(embed, ids)
 *   per layer i:
 *     RmsNorm(attn_norm) -> MatMulNT(q), MatMulNT(k), MatMulNT(v)
 *     -> SplitHeads x3 -> Rope(Neox) on q and k
 *     -> CausalAttention{layer=i, scale=1/sqrt(head_dim)} (writes the KV state)
 *     -> MergeHeads -> MatMulNT(o) -> Add(residual)
 *     -> RmsNorm(mlp_norm) -> SwiGlu(gate, up, down) -> Add(residual)
 *   RmsNorm(final_norm) -> LastToken(seq_len) -> MatMulNT(lm_head) -> logits
 *
 * MatMulNT with a [B, T, K] activation and an [N, K] weight follows
 * CpuDevice's broadcast rule (device.rs:1301-1407: one matmul_nt per batch
 * index against the shared weight). With a quantized config every matrix
 * weight is quantized by quant.c and the dequantized f32 copy is what the
 * reference f32 kernels consume ("sl-precision dequantize, then backend-cpu
 * matmul_nt"). The embedding table stays f32 because the Gather port is f32
 * (device.rs:910-946).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

enum {
    ROLE_EMBED = 0, ROLE_ATTN_NORM, ROLE_Q, ROLE_K, ROLE_V, ROLE_O,
    ROLE_MLP_NORM, ROLE_GATE, ROLE_UP, ROLE_DOWN, ROLE_FINAL_NORM, ROLE_LM_HEAD,
    ROLE_COUNT
};

typedef struct {
    float *w;          /* f32 weight (dequantized when quantized) */
    float *src;        /* the weight before quantization (quantized roles) */
    uint8_t *codes;    /* quantized payload or NULL */
    float *scales;
    size_t rows, cols; /* logical [rows, cols]; 1-D weights have rows == 1 */
} weight_t;

struct orc_llama {
    orc_llama_config cfg;
    weight_t *weights;  /* indexed by slot(role, layer) */
    size_t nslots;
    float *cache;
    size_t cache_len;
};

static int is_layer_role(int role) { return role >= ROLE_ATTN_NORM && role <= ROLE_DOWN; }

static size_t slot_of(const orc_llama *m, int role, uint32_t layer) {
    if (role == ROLE_EMBED) return 0;
    if (is_layer_role(role)) return 1 + (size_t)layer * 9 + (size_t)(role - ROLE_ATTN_NORM);
    return 1 + (size_t)m->cfg.layers * 9 + (size_t)(role - ROLE_FINAL_NORM);
}

static void role_shape(const orc_llama_config *c, int role, size_t *rows, size_t *cols) {
    size_t H = c->hidden, Q = (size_t)c->heads * c->head_dim, KV = (size_t)c->kv_heads * c->head_dim;
    switch (role) {
    case ROLE_EMBED: *rows = c->vocab; *cols = H; break;
    case ROLE_ATTN_NORM: case ROLE_MLP_NORM: case ROLE_FINAL_NORM: *rows = 1; *cols = H; break;
    case ROLE_Q: *rows = Q; *cols = H; break;
    case ROLE_K: case ROLE_V: *rows = KV; *cols = H; break;
    case ROLE_O: *rows = H; *cols = Q; break;
    case ROLE_GATE: case ROLE_UP: *rows = c->inter; *cols = H; break;
    case ROLE_DOWN: *rows = H; *cols = c->inter; break;
    default: *rows = c->vocab; *cols = H; break; /* lm_head */
    }
}

static int is_matrix_role(int role) {
    return role == ROLE_Q || role == ROLE_K || role == ROLE_V || role == ROLE_O ||
           role == ROLE_GATE || role == ROLE_UP || role == ROLE_DOWN || role == ROLE_LM_HEAD;
}

orc_llama *orc_llama_create(const orc_llama_config *cfg) {
    orc_llama *m = (orc_llama *)calloc(1, sizeof(orc_llama));
    if (!m) return NULL;
    m->cfg = *cfg;
    m->nslots = 1 + (size_t)cfg->layers * 9 + 2;
    m->weights = (weight_t *)calloc(m->nslots, sizeof(weight_t));
    for (int role = 0; role < ROLE_COUNT; role++) {
        uint32_t nl = is_layer_role(role) ? cfg->layers : 1;
        for (uint32_t l = 0; l < nl; l++) {
            weight_t *w = &m->weights[slot_of(m, role, l)];
            role_shape(cfg, role, &w->rows, &w->cols);
            w->w = (float *)calloc(w->rows * w->cols, sizeof(float));
            w->src = (float *)calloc(w->rows * w->cols, sizeof(float));
            if (cfg->quant_format >= 0 && is_matrix_role(role)) {
                w->codes = (uint8_t *)calloc(w->rows * orc_quant_row_bytes(cfg->quant_format, w->cols), 1);
                w->scales = (float *)calloc(w->rows * orc_quant_groups(w->cols, cfg->group_size), sizeof(float));
            }
        }
    }
    m->cache_len = (size_t)cfg->batch * cfg->layers * 2 * cfg->max_seq * cfg->kv_heads * cfg->head_dim;
    m->cache = (float *)calloc(m->cache_len, sizeof(float));
    return m;
}

void orc_llama_destroy(orc_llama *m) {
    if (!m) return;
    for (size_t i = 0; i < m->nslots; i++) {
        free(m->weights[i].w);
        free(m->weights[i].src);
        free(m->weights[i].codes);
        free(m->weights[i].scales);
    }
    free(m->weights);
    free(m->cache);
    free(m);
}

size_t orc_llama_weight_len(const orc_llama *m, int role, uint32_t layer) {
    const weight_t *w = &m->weights[slot_of(m, role, layer)];
    return w->rows * w->cols;
}

float *orc_llama_weight(orc_llama *m, int role, uint32_t layer) {
    return m->weights[slot_of(m, role, layer)].w;
}

const float *orc_llama_weight_source(const orc_llama *m, int role, uint32_t layer) {
    return m->weights[slot_of(m, role, layer)].src;
}

const uint8_t *orc_llama_codes(const orc_llama *m, int role, uint32_t layer) {
    return m->weights[slot_of(m, role, layer)].codes;
}

const float *orc_llama_scales(const orc_llama *m, int role, uint32_t layer) {
    return m->weights[slot_of(m, role, layer)].scales;
}

static void finish_weight(orc_llama *m, weight_t *w) {
    memcpy(w->src, w->w, w->rows * w->cols * sizeof(float));
    if (!w->codes) return;
    orc_quantize(m->cfg.quant_format, w->w, w->rows, w->cols, m->cfg.group_size,
                 w->codes, w->scales, NULL);
    orc_dequantize(m->cfg.quant_format, w->codes, w->scales, w->rows, w->cols,
                   m->cfg.group_size, w->w, NULL);
}

/* One LCG stream in role order: embed; per layer attn_norm, q, k, v, o,
 * mlp_norm, gate, up, down; final_norm; lm_head. Matrices and the embedding
 * draw N(0, std); norm weights draw N(1, 0.1). */
void orc_llama_init_random(orc_llama *m, uint64_t seed, float std) {
    orc_lcg lcg = {seed};
    for (size_t s = 0; s < m->nslots; s++) {
        weight_t *w = &m->weights[s];
        int norm = (w->rows == 1);
        orc_lcg_fill_normal(&lcg, w->w, w->rows * w->cols, norm ? 1.0f : 0.0f, norm ? 0.1f : std);
        finish_weight(m, w);
    }
}

void orc_llama_reset_cache(orc_llama *m) { memset(m->cache, 0, m->cache_len * sizeof(float)); }

const float *orc_llama_cache(const orc_llama *m, size_t *len) {
    if (len) *len = m->cache_len;
    return m->cache;
}

uint32_t orc_argmax(const float *row, size_t len) {
    uint32_t best = 0;
    for (size_t i = 1; i < len; i++)
        if (row[i] > row[best]) best = (uint32_t)i;
    return best;
}

/* MatMulNT of [rows_a, k] activations against an [n, k] weight shared across
 * the batch prefix: CpuDevice calls matmul_nt once per batch index. */
static int mm_nt(const float *a, size_t batch, size_t m_rows, size_t k, const weight_t *w,
                 float *out, orc_err *err) {
    for (size_t b = 0; b < batch; b++) {
        int rc = orc_matmul_nt(a + b * m_rows * k, m_rows * k, w->w, w->rows * w->cols,
                               out + b * m_rows * w->rows, m_rows * w->rows, 1, m_rows, k,
                               w->rows, err);
        if (rc) return rc;
    }
    return ORC_OK;
}

#define TRY(expr) do { int rc_ = (expr); if (rc_) { status = rc_; goto done; } } while (0)

int orc_llama_step(orc_llama *m, const uint32_t *ids, const uint32_t *positions,
                   uint32_t seq, uint32_t past_len, float *logits, orc_err *err) {
    const orc_llama_config *c = &m->cfg;
    const size_t B = c->batch, T = seq, H = c->hidden, D = c->head_dim;
    const size_t Hq = c->heads, Hkv = c->kv_heads, I = c->inter, V = c->vocab;
    const size_t BT = B * T, QW = Hq * D, KW = Hkv * D;
    const float scale = (float)(1.0 / sqrt((double)D));
    int status = ORC_OK;

    float *x = (float *)malloc(BT * H * sizeof(float));
    float *x1 = (float *)malloc(BT * H * sizeof(float));
    float *h = (float *)malloc(BT * H * sizeof(float));
    float *tmp = (float *)malloc(BT * H * sizeof(float));
    float *q = (float *)malloc(BT * QW * sizeof(float));
    float *k = (float *)malloc(BT * KW * sizeof(float));
    float *v = (float *)malloc(BT * KW * sizeof(float));
    float *qs = (float *)malloc(BT * QW * sizeof(float));
    float *ks = (float *)malloc(BT * KW * sizeof(float));
    float *vs = (float *)malloc(BT * KW * sizeof(float));
    float *att = (float *)malloc(BT * QW * sizeof(float));
    float *last = (float *)malloc(B * H * sizeof(float));
    (void)I;

    const weight_t *W = m->weights;
    TRY(orc_gather(W[slot_of(m, ROLE_EMBED, 0)].w, V * H, ids, BT, x, BT * H, V, H, BT, err));
    for (uint32_t l = 0; l < c->layers; l++) {
        const weight_t *an = &W[slot_of(m, ROLE_ATTN_NORM, l)];
        TRY(orc_rms_norm(x, BT * H, an->w, H, h, BT * H, BT, H, c->eps, err));
        TRY(mm_nt(h, B, T, H, &W[slot_of(m, ROLE_Q, l)], q, err));
        TRY(mm_nt(h, B, T, H, &W[slot_of(m, ROLE_K, l)], k, err));
        TRY(mm_nt(h, B, T, H, &W[slot_of(m, ROLE_V, l)], v, err));
        TRY(orc_split_heads(q, BT * QW, qs, BT * QW, B, T, Hq, D, err));
        TRY(orc_split_heads(k, BT * KW, ks, BT * KW, B, T, Hkv, D, err));
        TRY(orc_split_heads(v, BT * KW, vs, BT * KW, B, T, Hkv, D, err));
        /* Rope writes a new value (copy_into then rotate, device.rs:857-877). */
        TRY(orc_rope_neox(qs, BT * QW, positions, BT, B, Hq, T, D, c->theta, err));
        TRY(orc_rope_neox(ks, BT * KW, positions, BT, B, Hkv, T, D, c->theta, err));
        TRY(orc_causal_attention(qs, BT * QW, ks, BT * KW, vs, BT * KW, m->cache, m->cache_len,
                                 att, BT * QW, B, c->layers, l, Hq, Hkv, T, past_len, D,
                                 c->max_seq, scale, err));
        TRY(orc_merge_heads(att, BT * QW, q, BT * QW, B, T, Hq, D, err));
        TRY(mm_nt(q, B, T, QW, &W[slot_of(m, ROLE_O, l)], tmp, err));
        TRY(orc_add(x, BT * H, tmp, BT * H, x1, BT * H, BT * H, err));
        const weight_t *mn = &W[slot_of(m, ROLE_MLP_NORM, l)];
        TRY(orc_rms_norm(x1, BT * H, mn->w, H, h, BT * H, BT, H, c->eps, err));
        const weight_t *g = &W[slot_of(m, ROLE_GATE, l)];
        const weight_t *u = &W[slot_of(m, ROLE_UP, l)];
        const weight_t *d = &W[slot_of(m, ROLE_DOWN, l)];
        TRY(orc_swiglu(h, BT * H, g->w, g->rows * g->cols, u->w, u->rows * u->cols, d->w,
                       d->rows * d->cols, tmp, BT * H, BT, H, g->rows, err));
        TRY(orc_add(x1, BT * H, tmp, BT * H, x, BT * H, BT * H, err));
    }
    const weight_t *fn = &W[slot_of(m, ROLE_FINAL_NORM, 0)];
    TRY(orc_rms_norm(x, BT * H, fn->w, H, h, BT * H, BT, H, c->eps, err));
    TRY(orc_last_token(h, BT * H, last, B * H, B, T, H, T, err));
    TRY(mm_nt(last, 1, B, H, &W[slot_of(m, ROLE_LM_HEAD, 0)], logits, err));

done:
    free(x); free(x1); free(h); free(tmp); free(q); free(k); free(v);
    free(qs); free(ks); free(vs); free(att); free(last);
    return status;
}
