/*
 * CPU oracle: restatement of the scalar reference kernels of
 * crates/backends/backend-cpu/src/reference/ (all modules) (SeekStarAI/StarLight).
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h). Compiled with -ffp-contract=off so
 * every f32 multiply and add rounds separately, as the Rust reference does.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Thread count for the loops below. Parallel loops only ever split
 * independent outputs, so every output element sees exactly the reference's
 * sequence of f32 operations and the result does not depend on the thread
 * count. */
void orc_set_threads(int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

/* ---- helpers (reference/mod.rs:81-110) --------------------------------- */

static int set_err(orc_err *err, int code, size_t expected, size_t actual,
                   const char *reason) {
    if (err) {
        err->code = code;
        err->expected = expected;
        err->actual = actual;
        err->reason = reason;
    }
    return code;
}

static int ok(orc_err *err) { return set_err(err, ORC_OK, 0, 0, 0); }

/* shape_len, mod.rs:82-88: checked product. */
static int shape_len(const size_t *dims, size_t n, size_t *out) {
    size_t product = 1;
    for (size_t i = 0; i < n; i++) {
        if (dims[i] != 0 && product > SIZE_MAX / dims[i]) return 0;
        product *= dims[i];
    }
    *out = product;
    return 1;
}

#define SHAPE(out, ...)                                                        \
    do {                                                                       \
        const size_t dims_[] = {__VA_ARGS__};                                  \
        if (!shape_len(dims_, sizeof(dims_) / sizeof(dims_[0]), &(out)))       \
            return set_err(err, ORC_SHAPE_OVERFLOW, 0, 0, 0);                  \
    } while (0)

/* expect_len, mod.rs:91-97. */
#define EXPECT_LEN(actual, expected)                                           \
    do {                                                                       \
        if ((actual) != (expected))                                            \
            return set_err(err, ORC_LENGTH_MISMATCH, (expected), (actual), 0); \
    } while (0)

#define INVALID(reason) return set_err(err, ORC_INVALID_SHAPE, 0, 0, (reason))

/* dot, mod.rs:103-110: sequential f32 sum, left to right. */
static float dot(const float *left, const float *right, size_t len) {
    float sum = 0.0f;
    for (size_t i = 0; i < len; i++) sum += left[i] * right[i];
    return sum;
}

/* ---- LCG, mod.rs:118-148 ------------------------------------------------ */

uint32_t orc_lcg_next_u32(orc_lcg *lcg) {
    lcg->state = lcg->state * 6364136223846793005ULL + 1442695040888963407ULL;
    return (uint32_t)(lcg->state >> 33);
}

float orc_lcg_uniform(orc_lcg *lcg, float low, float high) {
    double unit = (double)orc_lcg_next_u32(lcg) / (double)UINT32_MAX;
    return low + (high - low) * (float)unit;
}

void orc_lcg_fill(orc_lcg *lcg, float *values, size_t len, float low, float high) {
    for (size_t i = 0; i < len; i++) values[i] = orc_lcg_uniform(lcg, low, high);
}

size_t orc_lcg_below(orc_lcg *lcg, size_t upper) {
    if (upper == 0) return 0;
    return (size_t)orc_lcg_next_u32(lcg) % upper;
}

/* Box-Muller on two LCG draws, evaluated in f64 and rounded once to f32.
 * u1 is shifted by one so that log(u1) is finite. This transform is this
 * project's definition for N(mean, std) synthetic inputs; the reference has
 * no normal generator. */
float orc_lcg_normal(orc_lcg *lcg, float mean, float std) {
    double u1 = ((double)orc_lcg_next_u32(lcg) + 1.0) / 4294967296.0;
    double u2 = (double)orc_lcg_next_u32(lcg) / 4294967296.0;
    double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
    return (float)((double)mean + (double)std * z);
}

void orc_lcg_fill_normal(orc_lcg *lcg, float *values, size_t len, float mean, float std) {
    for (size_t i = 0; i < len; i++) values[i] = orc_lcg_normal(lcg, mean, std);
}

/* ---- matmul.rs ---------------------------------------------------------- */

/* matmul_nt, matmul.rs:29-59: batch -> row m -> column n -> k ascending. */
int orc_matmul_nt(const float *a, size_t a_len, const float *b, size_t b_len,
                  float *out, size_t out_len, size_t batch, size_t m, size_t k,
                  size_t n, orc_err *err) {
    size_t al, bl, ol;
    SHAPE(al, batch, m, k);
    SHAPE(bl, batch, n, k);
    SHAPE(ol, batch, m, n);
    EXPECT_LEN(a_len, al);
    EXPECT_LEN(b_len, bl);
    EXPECT_LEN(out_len, ol);
    for (size_t bi = 0; bi < batch; bi++) {
        const float *ab = a + bi * m * k;
        const float *bb = b + bi * n * k;
        float *ob = out + bi * m * n;
        long long total = (long long)(m * n);
#pragma omp parallel for schedule(static)
        for (long long idx = 0; idx < total; idx++) {
            size_t row = (size_t)idx / n, col = (size_t)idx % n;
            ob[row * n + col] = dot(ab + row * k, bb + col * k, k);
        }
    }
    return ok(err);
}

/* matmul_nn, matmul.rs:77-110. */
int orc_matmul_nn(const float *a, size_t a_len, const float *b, size_t b_len,
                  float *out, size_t out_len, size_t batch, size_t m, size_t k,
                  size_t n, orc_err *err) {
    size_t al, bl, ol;
    SHAPE(al, batch, m, k);
    SHAPE(bl, batch, k, n);
    SHAPE(ol, batch, m, n);
    EXPECT_LEN(a_len, al);
    EXPECT_LEN(b_len, bl);
    EXPECT_LEN(out_len, ol);
    for (size_t bi = 0; bi < batch; bi++) {
        const float *ab = a + bi * m * k;
        const float *bb = b + bi * k * n;
        float *ob = out + bi * m * n;
        for (size_t row = 0; row < m; row++)
            for (size_t col = 0; col < n; col++) {
                float sum = 0.0f;
                for (size_t d = 0; d < k; d++) sum += ab[row * k + d] * bb[d * n + col];
                ob[row * n + col] = sum;
            }
    }
    return ok(err);
}

/* ---- softmax.rs --------------------------------------------------------- */

/* softmax, softmax.rs:19-42. The maximum is a left fold of f32::max starting
 * at -inf; exp is libm expf; the sum runs left to right. */
int orc_softmax(float *x, size_t x_len, size_t rows, size_t cols, orc_err *err) {
    if (rows == 0 || cols == 0) INVALID("softmax requires nonzero rows and cols");
    size_t total;
    SHAPE(total, rows, cols);
    EXPECT_LEN(x_len, total);
    for (size_t r = 0; r < rows; r++) {
        float *row = x + r * cols;
        float maximum = -INFINITY;
        for (size_t c = 0; c < cols; c++) maximum = fmaxf(maximum, row[c]);
        float sum = 0.0f;
        for (size_t c = 0; c < cols; c++) {
            row[c] = expf(row[c] - maximum);
            sum += row[c];
        }
        float inverse_sum = 1.0f / sum;
        for (size_t c = 0; c < cols; c++) row[c] *= inverse_sum;
    }
    return ok(err);
}

/* softmax_causal, softmax.rs:61-114. */
int orc_softmax_causal(float *x, size_t x_len, size_t rows, size_t cols,
                       size_t seq, size_t past_len, orc_err *err) {
    if (rows == 0 || cols == 0) INVALID("softmax_causal requires nonzero rows and cols");
    if (seq == 0) INVALID("softmax_causal requires a nonzero seq");
    if (past_len > SIZE_MAX - seq) return set_err(err, ORC_SHAPE_OVERFLOW, 0, 0, 0);
    if (cols != past_len + seq) INVALID("softmax_causal requires cols == past_len + seq");
    if (rows % seq != 0) INVALID("softmax_causal requires rows to be a multiple of seq");
    size_t total;
    SHAPE(total, rows, cols);
    EXPECT_LEN(x_len, total);
    for (size_t r = 0; r < rows; r++) {
        size_t last_visible = past_len + r % seq;
        float *row = x + r * cols;
        float maximum = -INFINITY;
        for (size_t c = 0; c <= last_visible; c++) maximum = fmaxf(maximum, row[c]);
        float sum = 0.0f;
        for (size_t c = 0; c <= last_visible; c++) {
            row[c] = expf(row[c] - maximum);
            sum += row[c];
        }
        float inverse_sum = 1.0f / sum;
        for (size_t c = 0; c <= last_visible; c++) row[c] *= inverse_sum;
        for (size_t c = last_visible + 1; c < cols; c++) row[c] = 0.0f;
    }
    return ok(err);
}

/* ---- norm.rs ------------------------------------------------------------ */

/* rms_norm, norm.rs:27-60: left-to-right f32 sum of squares, one
 * 1/sqrt(mean + eps), then value * inverse_rms * scale per element. */
int orc_rms_norm(const float *x, size_t x_len, const float *weight,
                 size_t weight_len, float *out, size_t out_len, size_t rows,
                 size_t hidden, float eps, orc_err *err) {
    if (hidden == 0) INVALID("rms_norm requires a nonzero hidden size");
    size_t total;
    SHAPE(total, rows, hidden);
    EXPECT_LEN(x_len, total);
    EXPECT_LEN(weight_len, hidden);
    EXPECT_LEN(out_len, total);
    for (size_t r = 0; r < rows; r++) {
        const float *xr = x + r * hidden;
        float *or_ = out + r * hidden;
        float sum_of_squares = 0.0f;
        for (size_t i = 0; i < hidden; i++) sum_of_squares += xr[i] * xr[i];
        float mean_square = sum_of_squares / (float)hidden;
        float inverse_rms = 1.0f / sqrtf(mean_square + eps);
        for (size_t i = 0; i < hidden; i++) or_[i] = xr[i] * inverse_rms * weight[i];
    }
    return ok(err);
}

/* ---- rope.rs ------------------------------------------------------------ */

/* validate_rope, rope.rs:9-25. */
static int validate_rope(size_t x_len, size_t positions_len, size_t batch,
                         size_t heads, size_t seq, size_t head_dim, orc_err *err) {
    if (head_dim == 0 || head_dim % 2 != 0) INVALID("head_dim must be a positive even number");
    size_t xl, pl;
    SHAPE(xl, batch, heads, seq, head_dim);
    EXPECT_LEN(x_len, xl);
    SHAPE(pl, batch, seq);
    EXPECT_LEN(positions_len, pl);
    return ORC_OK;
}

/* rope_angle, rope.rs:31-35: position / theta^(2*pair/head_dim) in f64. */
static double rope_angle(double position, size_t pair, size_t head_dim, double theta) {
    double exponent = 2.0 * (double)pair / (double)head_dim;
    return position / pow(theta, exponent);
}

static int rope_apply(float *x, size_t x_len, const uint32_t *positions,
                      size_t positions_len, size_t batch, size_t heads,
                      size_t seq, size_t head_dim, float theta_f, int gptj,
                      orc_err *err) {
    int rc = validate_rope(x_len, positions_len, batch, heads, seq, head_dim, err);
    if (rc != ORC_OK) return rc;
    size_t half = head_dim / 2;
    double theta = (double)theta_f;
    for (size_t b = 0; b < batch; b++)
        for (size_t t = 0; t < seq; t++) {
            double position = (double)positions[b * seq + t];
            for (size_t pair = 0; pair < half; pair++) {
                double angle = rope_angle(position, pair, head_dim, theta);
                float sine = (float)sin(angle);
                float cosine = (float)cos(angle);
                for (size_t h = 0; h < heads; h++) {
                    size_t base = ((b * heads + h) * seq + t) * head_dim;
                    size_t i0 = gptj ? base + 2 * pair : base + pair;
                    size_t i1 = gptj ? base + 2 * pair + 1 : base + pair + half;
                    float first = x[i0];
                    float second = x[i1];
                    x[i0] = first * cosine - second * sine;
                    x[i1] = first * sine + second * cosine;
                }
            }
        }
    return ok(err);
}

/* rope_neox, rope.rs:55-88: pairs (x[i], x[i + head_dim/2]). */
int orc_rope_neox(float *x, size_t x_len, const uint32_t *positions,
                  size_t positions_len, size_t batch, size_t heads, size_t seq,
                  size_t head_dim, float theta, orc_err *err) {
    return rope_apply(x, x_len, positions, positions_len, batch, heads, seq,
                      head_dim, theta, 0, err);
}

/* rope_gptj, rope.rs:108-141: pairs (x[2i], x[2i+1]). */
int orc_rope_gptj(float *x, size_t x_len, const uint32_t *positions,
                  size_t positions_len, size_t batch, size_t heads, size_t seq,
                  size_t head_dim, float theta, orc_err *err) {
    return rope_apply(x, x_len, positions, positions_len, batch, heads, seq,
                      head_dim, theta, 1, err);
}

/* ---- elementwise.rs ----------------------------------------------------- */

/* silu_scalar, elementwise.rs:10-12: x * (1 / (1 + exp(-x))). */
float orc_silu_scalar(float value) { return value * (1.0f / (1.0f + expf(-value))); }

int orc_silu(float *x, size_t len, orc_err *err) {
    for (size_t i = 0; i < len; i++) x[i] = orc_silu_scalar(x[i]);
    return ok(err);
}

/* mul, elementwise.rs:35-44. */
int orc_mul(const float *a, size_t a_len, const float *b, size_t b_len,
            float *out, size_t out_len, size_t len, orc_err *err) {
    EXPECT_LEN(a_len, len);
    EXPECT_LEN(b_len, len);
    EXPECT_LEN(out_len, len);
    for (size_t i = 0; i < len; i++) out[i] = a[i] * b[i];
    return ok(err);
}

/* add, elementwise.rs:53-61. */
int orc_add(const float *a, size_t a_len, const float *b, size_t b_len,
            float *out, size_t out_len, size_t len, orc_err *err) {
    EXPECT_LEN(a_len, len);
    EXPECT_LEN(b_len, len);
    EXPECT_LEN(out_len, len);
    for (size_t i = 0; i < len; i++) out[i] = a[i] + b[i];
    return ok(err);
}

/* scale, elementwise.rs:69-74. */
int orc_scale(float *x, size_t len, float factor, orc_err *err) {
    for (size_t i = 0; i < len; i++) x[i] *= factor;
    return ok(err);
}

/* ---- layout.rs ---------------------------------------------------------- */

/* gather, layout.rs:25-52: every id is validated before the first write. */
int orc_gather(const float *table, size_t table_len, const uint32_t *ids,
               size_t ids_len, float *out, size_t out_len, size_t vocab,
               size_t hidden, size_t rows, orc_err *err) {
    size_t tl, ol;
    SHAPE(tl, vocab, hidden);
    EXPECT_LEN(table_len, tl);
    EXPECT_LEN(ids_len, rows);
    SHAPE(ol, rows, hidden);
    EXPECT_LEN(out_len, ol);
    for (size_t r = 0; r < rows; r++)
        if ((size_t)ids[r] >= vocab) INVALID("id out of range");
    for (size_t r = 0; r < rows; r++)
        memcpy(out + r * hidden, table + (size_t)ids[r] * hidden, hidden * sizeof(float));
    return ok(err);
}

/* last_token, layout.rs:71-95. */
int orc_last_token(const float *input, size_t input_len, float *out,
                   size_t out_len, size_t batch, size_t seq, size_t hidden,
                   size_t seq_len, orc_err *err) {
    if (seq_len < 1 || seq_len > seq) INVALID("last_token requires 1 <= seq_len <= seq");
    size_t il, ol;
    SHAPE(il, batch, seq, hidden);
    EXPECT_LEN(input_len, il);
    SHAPE(ol, batch, hidden);
    EXPECT_LEN(out_len, ol);
    size_t position = seq_len - 1;
    for (size_t b = 0; b < batch; b++)
        memcpy(out + b * hidden, input + (b * seq + position) * hidden, hidden * sizeof(float));
    return ok(err);
}

/* split_heads, layout.rs:107-128: [B,S,H*D] -> [B,H,S,D]. */
int orc_split_heads(const float *input, size_t input_len, float *out,
                    size_t out_len, size_t batch, size_t seq, size_t heads,
                    size_t head_dim, orc_err *err) {
    size_t total;
    SHAPE(total, batch, seq, heads, head_dim);
    EXPECT_LEN(input_len, total);
    EXPECT_LEN(out_len, total);
    for (size_t b = 0; b < batch; b++)
        for (size_t t = 0; t < seq; t++)
            for (size_t h = 0; h < heads; h++)
                memcpy(out + ((b * heads + h) * seq + t) * head_dim,
                       input + ((b * seq + t) * heads + h) * head_dim,
                       head_dim * sizeof(float));
    return ok(err);
}

/* merge_heads, layout.rs:144-168: [B,H,S,D] -> [B,S,H*D]. */
int orc_merge_heads(const float *input, size_t input_len, float *out,
                    size_t out_len, size_t batch, size_t seq, size_t heads,
                    size_t head_dim, orc_err *err) {
    size_t total;
    SHAPE(total, batch, seq, heads, head_dim);
    EXPECT_LEN(input_len, total);
    EXPECT_LEN(out_len, total);
    for (size_t b = 0; b < batch; b++)
        for (size_t t = 0; t < seq; t++)
            for (size_t h = 0; h < heads; h++)
                memcpy(out + ((b * seq + t) * heads + h) * head_dim,
                       input + ((b * heads + h) * seq + t) * head_dim,
                       head_dim * sizeof(float));
    return ok(err);
}

/* ---- attention.rs ------------------------------------------------------- */

/* kv_append, attention.rs:33-83. Cache [B, L, 2, max_seq, Hkv, D]; all checks
 * run before the first write. */
int orc_kv_append(const float *k, size_t k_len, const float *v, size_t v_len,
                  float *cache, size_t cache_len, size_t batch, size_t layers,
                  size_t layer, size_t kv_heads, size_t head_dim,
                  size_t max_seq, size_t past_len, size_t seq, orc_err *err) {
    size_t kvl, cl;
    SHAPE(kvl, batch, kv_heads, seq, head_dim);
    SHAPE(cl, batch, layers, 2, max_seq, kv_heads, head_dim);
    EXPECT_LEN(k_len, kvl);
    EXPECT_LEN(v_len, kvl);
    EXPECT_LEN(cache_len, cl);
    if (layer >= layers) INVALID("layer out of range");
    if (past_len > SIZE_MAX - seq) return set_err(err, ORC_SHAPE_OVERFLOW, 0, 0, 0);
    if (past_len + seq > max_seq) INVALID("past_len + seq exceeds max_seq");
    size_t time_stride = kv_heads * head_dim;
    size_t parity_stride = max_seq * time_stride;
    size_t layer_stride = 2 * parity_stride;
    size_t batch_stride = layers * layer_stride;
    for (size_t b = 0; b < batch; b++)
        for (size_t h = 0; h < kv_heads; h++)
            for (size_t t = 0; t < seq; t++) {
                size_t src = ((b * kv_heads + h) * seq + t) * head_dim;
                size_t dst = b * batch_stride + layer * layer_stride +
                             (past_len + t) * time_stride + h * head_dim;
                memcpy(cache + dst, k + src, head_dim * sizeof(float));
                memcpy(cache + dst + parity_stride, v + src, head_dim * sizeof(float));
            }
    return ok(err);
}

/* causal_attention, attention.rs:129-219: append, then per (b, h, t) three
 * passes over keys 0..=past+t (max, denominator, weighted values). */
int orc_causal_attention(const float *q, size_t q_len, const float *k_new,
                         size_t k_len, const float *v_new, size_t v_len,
                         float *cache, size_t cache_len, float *out,
                         size_t out_len, size_t batch, size_t layers,
                         size_t layer, size_t heads, size_t kv_heads,
                         size_t seq, size_t past_len, size_t head_dim,
                         size_t max_seq, float scale, orc_err *err) {
    if (kv_heads == 0) INVALID("kv_heads must be nonzero");
    if (heads == 0) INVALID("heads must be nonzero");
    if (heads % kv_heads != 0) INVALID("heads must be a multiple of kv_heads");
    size_t ql;
    SHAPE(ql, batch, heads, seq, head_dim);
    EXPECT_LEN(q_len, ql);
    EXPECT_LEN(out_len, ql);
    int rc = orc_kv_append(k_new, k_len, v_new, v_len, cache, cache_len, batch,
                           layers, layer, kv_heads, head_dim, max_seq, past_len,
                           seq, err);
    if (rc != ORC_OK) return rc;
    size_t group = heads / kv_heads;
    size_t time_stride = kv_heads * head_dim;
    size_t parity_stride = max_seq * time_stride;
    size_t layer_stride = 2 * parity_stride;
    size_t batch_stride = layers * layer_stride;
#pragma omp parallel for schedule(static)
    for (long long bh = 0; bh < (long long)(batch * heads); bh++) {
        size_t b = (size_t)bh / heads, h = (size_t)bh % heads;
        {
            size_t kv_head = h / group;
            for (size_t t = 0; t < seq; t++) {
                size_t key_count = past_len + t + 1;
                size_t query_base = ((b * heads + h) * seq + t) * head_dim;
                const float *query = q + query_base;
                size_t key_base = b * batch_stride + layer * layer_stride + kv_head * head_dim;
                size_t value_base = key_base + parity_stride;
                float maximum = -INFINITY;
                for (size_t j = 0; j < key_count; j++) {
                    float score = dot(query, cache + key_base + j * time_stride, head_dim) * scale;
                    if (score > maximum) maximum = score;
                }
                float denominator = 0.0f;
                for (size_t j = 0; j < key_count; j++) {
                    float score = dot(query, cache + key_base + j * time_stride, head_dim) * scale;
                    denominator += expf(score - maximum);
                }
                float inverse_denominator = 1.0f / denominator;
                float *orow = out + query_base;
                for (size_t d = 0; d < head_dim; d++) orow[d] = 0.0f;
                for (size_t j = 0; j < key_count; j++) {
                    float score = dot(query, cache + key_base + j * time_stride, head_dim) * scale;
                    float probability = expf(score - maximum) * inverse_denominator;
                    const float *vrow = cache + value_base + j * time_stride;
                    for (size_t d = 0; d < head_dim; d++) orow[d] += probability * vrow[d];
                }
            }
        }
    }
    return ok(err);
}

/* ---- swiglu.rs ---------------------------------------------------------- */

/* swiglu, swiglu.rs:40-84: per row, for each intermediate i accumulate
 * out[j] += silu(x.gate_i) * (x.up_i) * down[j, i]. */
int orc_swiglu(const float *x, size_t x_len, const float *w_gate,
               size_t gate_len, const float *w_up, size_t up_len,
               const float *w_down, size_t down_len, float *out,
               size_t out_len, size_t rows, size_t hidden, size_t inter,
               orc_err *err) {
    if (hidden == 0) INVALID("swiglu requires a nonzero hidden size");
    if (inter == 0) INVALID("swiglu requires a nonzero inter size");
    size_t tl, wl, dl;
    SHAPE(tl, rows, hidden);
    EXPECT_LEN(x_len, tl);
    SHAPE(wl, inter, hidden);
    EXPECT_LEN(gate_len, wl);
    EXPECT_LEN(up_len, wl);
    SHAPE(dl, hidden, inter);
    EXPECT_LEN(down_len, dl);
    EXPECT_LEN(out_len, tl);
    /* The reference walks i outer, j inner, adding weight_i * down[j, i] into
     * out[j]. Computing every weight_i first and then walking j outer, i inner
     * performs the same f32 operations in the same order for each out[j]. */
    float *weights = (float *)malloc((inter ? inter : 1) * sizeof(float));
    for (size_t r = 0; r < rows; r++) {
        const float *xr = x + r * hidden;
        float *or_ = out + r * hidden;
#pragma omp parallel for schedule(static)
        for (long long i = 0; i < (long long)inter; i++) {
            float gate = orc_silu_scalar(dot(xr, w_gate + i * hidden, hidden));
            float up = dot(xr, w_up + i * hidden, hidden);
            weights[i] = gate * up;
        }
#pragma omp parallel for schedule(static)
        for (long long j = 0; j < (long long)hidden; j++) {
            float acc = 0.0f;
            for (size_t i = 0; i < inter; i++) acc += weights[i] * w_down[j * inter + i];
            or_[j] = acc;
        }
    }
    free(weights);
    return ok(err);
}

/* ---- fused.rs ----------------------------------------------------------- */

/* rms_norm_matmul, fused.rs:41-90: sum += x[i] * inverse_rms * weight[i] * w[i]
 * evaluated left to right as ((x*inv)*weight)*w. */
int orc_rms_norm_matmul(const float *x, size_t x_len, const float *weight,
                        size_t weight_len, const float *w, size_t w_len,
                        float *out, size_t out_len, size_t rows, size_t hidden,
                        size_t out_features, float eps, orc_err *err) {
    if (hidden == 0) INVALID("rms_norm_matmul requires a nonzero hidden size");
    if (out_features == 0) INVALID("rms_norm_matmul requires a nonzero out_features");
    size_t xl, ol, wl;
    SHAPE(xl, rows, hidden);
    SHAPE(ol, rows, out_features);
    EXPECT_LEN(x_len, xl);
    EXPECT_LEN(weight_len, hidden);
    SHAPE(wl, out_features, hidden);
    EXPECT_LEN(w_len, wl);
    EXPECT_LEN(out_len, ol);
    for (size_t r = 0; r < rows; r++) {
        const float *xr = x + r * hidden;
        float sum_of_squares = 0.0f;
        for (size_t i = 0; i < hidden; i++) sum_of_squares += xr[i] * xr[i];
        float mean_square = sum_of_squares / (float)hidden;
        float inverse_rms = 1.0f / sqrtf(mean_square + eps);
        for (size_t c = 0; c < out_features; c++) {
            const float *wr = w + c * hidden;
            float sum = 0.0f;
            for (size_t i = 0; i < hidden; i++) sum += xr[i] * inverse_rms * weight[i] * wr[i];
            out[r * out_features + c] = sum;
        }
    }
    return ok(err);
}
