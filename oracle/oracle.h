/*
 * CPU oracle for the StarLight backend-cuda hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * backend: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * and reference legs may load it. The product path (libslc.so) never links,
 * loads or calls it.
 *
 * Every function is a plain-C restatement of the scalar Rust reference kernels
 * in crates/backends/backend-cpu/src/reference/ (SeekStarAI/StarLight). The
 * loop order, the accumulation order and the f32/f64 split are kept identical,
 * and the library is compiled with -ffp-contract=off (no FMA contraction), so
 * on the same libm it reproduces the reference bit for bit. Citations are
 * given per function in oracle.c.
 *
 * Parity pins: tests/test_oracle.py checks this library against every
 * known-answer test and every LCG-seeded f64-oracle case in the reference's
 * own unit tests (restated from the Rust test modules) and against the
 * starlight-runtime end-to-end fixture (tests/end_to_end.rs:38-68).
 * The INT4/INT8 quantizer (quant.c) has no reference source in the checkout
 * (sl-precision is an empty submodule): its parity is unpinned.
 */
#ifndef STARLIGHT_ORACLE_H
#define STARLIGHT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* KernelError (reference/mod.rs:44-61). */
enum {
    ORC_OK = 0,
    ORC_LENGTH_MISMATCH = 1,
    ORC_SHAPE_OVERFLOW = 2,
    ORC_INVALID_SHAPE = 3,
    ORC_UNSUPPORTED = 4,
};

typedef struct {
    int code;
    size_t expected;
    size_t actual;
    const char *reason;
} orc_err;

/* OpenMP thread count for the oracle's parallel loops (results do not depend
 * on it). */
void orc_set_threads(int threads);

/* ---- deterministic LCG (reference/mod.rs:118-148) ---------------------- */
typedef struct { uint64_t state; } orc_lcg;
uint32_t orc_lcg_next_u32(orc_lcg *lcg);
float orc_lcg_uniform(orc_lcg *lcg, float low, float high);
void orc_lcg_fill(orc_lcg *lcg, float *values, size_t len, float low, float high);
size_t orc_lcg_below(orc_lcg *lcg, size_t upper);
/* Box-Muller normal draw on top of the LCG (this project's definition). */
float orc_lcg_normal(orc_lcg *lcg, float mean, float std);
void orc_lcg_fill_normal(orc_lcg *lcg, float *values, size_t len, float mean, float std);

/* ---- kernels ----------------------------------------------------------- */
int orc_matmul_nt(const float *a, size_t a_len, const float *b, size_t b_len,
                  float *out, size_t out_len, size_t batch, size_t m, size_t k,
                  size_t n, orc_err *err);
int orc_matmul_nn(const float *a, size_t a_len, const float *b, size_t b_len,
                  float *out, size_t out_len, size_t batch, size_t m, size_t k,
                  size_t n, orc_err *err);
int orc_softmax(float *x, size_t x_len, size_t rows, size_t cols, orc_err *err);
int orc_softmax_causal(float *x, size_t x_len, size_t rows, size_t cols,
                       size_t seq, size_t past_len, orc_err *err);
int orc_rms_norm(const float *x, size_t x_len, const float *weight,
                 size_t weight_len, float *out, size_t out_len, size_t rows,
                 size_t hidden, float eps, orc_err *err);
int orc_rope_neox(float *x, size_t x_len, const uint32_t *positions,
                  size_t positions_len, size_t batch, size_t heads, size_t seq,
                  size_t head_dim, float theta, orc_err *err);
int orc_rope_gptj(float *x, size_t x_len, const uint32_t *positions,
                  size_t positions_len, size_t batch, size_t heads, size_t seq,
                  size_t head_dim, float theta, orc_err *err);
float orc_silu_scalar(float value);
int orc_silu(float *x, size_t len, orc_err *err);
int orc_mul(const float *a, size_t a_len, const float *b, size_t b_len,
            float *out, size_t out_len, size_t len, orc_err *err);
int orc_add(const float *a, size_t a_len, const float *b, size_t b_len,
            float *out, size_t out_len, size_t len, orc_err *err);
int orc_scale(float *x, size_t len, float factor, orc_err *err);
int orc_gather(const float *table, size_t table_len, const uint32_t *ids,
               size_t ids_len, float *out, size_t out_len, size_t vocab,
               size_t hidden, size_t rows, orc_err *err);
int orc_last_token(const float *input, size_t input_len, float *out,
                   size_t out_len, size_t batch, size_t seq, size_t hidden,
                   size_t seq_len, orc_err *err);
int orc_split_heads(const float *input, size_t input_len, float *out,
                    size_t out_len, size_t batch, size_t seq, size_t heads,
                    size_t head_dim, orc_err *err);
int orc_merge_heads(const float *input, size_t input_len, float *out,
                    size_t out_len, size_t batch, size_t seq, size_t heads,
                    size_t head_dim, orc_err *err);
int orc_kv_append(const float *k, size_t k_len, const float *v, size_t v_len,
                  float *cache, size_t cache_len, size_t batch, size_t layers,
                  size_t layer, size_t kv_heads, size_t head_dim,
                  size_t max_seq, size_t past_len, size_t seq, orc_err *err);
int orc_causal_attention(const float *q, size_t q_len, const float *k_new,
                         size_t k_len, const float *v_new, size_t v_len,
                         float *cache, size_t cache_len, float *out,
                         size_t out_len, size_t batch, size_t layers,
                         size_t layer, size_t heads, size_t kv_heads,
                         size_t seq, size_t past_len, size_t head_dim,
                         size_t max_seq, float scale, orc_err *err);
int orc_swiglu(const float *x, size_t x_len, const float *w_gate,
               size_t gate_len, const float *w_up, size_t up_len,
               const float *w_down, size_t down_len, float *out,
               size_t out_len, size_t rows, size_t hidden, size_t inter,
               orc_err *err);
int orc_rms_norm_matmul(const float *x, size_t x_len, const float *weight,
                        size_t weight_len, const float *w, size_t w_len,
                        float *out, size_t out_len, size_t rows, size_t hidden,
                        size_t out_features, float eps, orc_err *err);

/* ---- symmetric grouped INT4/INT8 quantization (quant.c) ---------------- */
enum { ORC_INT4 = 0, ORC_INT8 = 1 };
size_t orc_quant_row_bytes(int format, size_t k);
size_t orc_quant_groups(size_t k, size_t group);
int orc_quantize(int format, const float *w, size_t n, size_t k, size_t group,
                 uint8_t *codes, float *scales, orc_err *err);
int orc_dequantize(int format, const uint8_t *codes, const float *scales,
                   size_t n, size_t k, size_t group, float *w, orc_err *err);
int32_t orc_code_at(int format, const uint8_t *codes, size_t k, size_t row,
                    size_t col);

/* ---- llama-dense fixture runner (llama.c) ------------------------------ */
typedef struct {
    uint32_t layers, hidden, heads, kv_heads, head_dim, inter, vocab;
    uint32_t max_seq, batch;
    float eps, theta;
    int quant_format;      /* -1 dense f32, ORC_INT4, ORC_INT8 */
    uint32_t group_size;
} orc_llama_config;

typedef struct orc_llama orc_llama;
orc_llama *orc_llama_create(const orc_llama_config *cfg);
void orc_llama_destroy(orc_llama *model);
/* Weight roles in lowering order; see llama.c. Returns element count. */
size_t orc_llama_weight_len(const orc_llama *model, int role, uint32_t layer);
float *orc_llama_weight(orc_llama *model, int role, uint32_t layer);
/* Random-init N(0, std) for matrices and N(1, 0.1) norms; quantizes matrices
 * when the config asks for it and keeps the dequantized copy for matmul. */
void orc_llama_init_random(orc_llama *model, uint64_t seed, float std);
/* The weight as drawn, before quantization (what a model file would hold). */
const float *orc_llama_weight_source(const orc_llama *model, int role, uint32_t layer);
/* Quantized payload of one matrix role (codes row-major, scales [n, groups]). */
const uint8_t *orc_llama_codes(const orc_llama *model, int role, uint32_t layer);
const float *orc_llama_scales(const orc_llama *model, int role, uint32_t layer);
/* One Engine::step: ids/positions [batch, seq]; logits [batch, vocab]. */
int orc_llama_step(orc_llama *model, const uint32_t *ids,
                   const uint32_t *positions, uint32_t seq, uint32_t past_len,
                   float *logits, orc_err *err);
void orc_llama_reset_cache(orc_llama *model);
const float *orc_llama_cache(const orc_llama *model, size_t *len);
/* Argmax with ties broken towards the lowest index. */
uint32_t orc_argmax(const float *row, size_t len);

#ifdef __cplusplus
}
#endif
#endif
