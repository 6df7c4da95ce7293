/*
 * starlight_engine.h -- the llama-dense engine driven through backend-cuda.
 *
 * The reference's caller of the device is sl-core::Engine (contract in
 * docs/ARCH-0007 section 3.2: Engine::build / Engine::step) fed by the
 * llama-dense lowering of sl-model-adapters (docs/ARCH-0006 sections 3-5).
 * Both crates are empty submodules in the StarLight checkout, so this is a
 * C++ stand-in with the same contract, used to run the fixture and the
 * benchmark configurations end to end:
 *
 *   slc_llama_create  ~ lowering (prefill + decode programs) + Engine::build
 *   slc_llama_step    ~ Engine::step (upload ids/positions, one slc_dispatch
 *                       per command, synchronize, download logits)
 *   slc_llama_generate  the greedy loop the reference leaves to a future
 *                       sl-daemon (docs/ARCH-0005:118): prefill, then decode
 *                       steps feeding back the argmax (ties -> lowest id).
 *
 * Every command goes through slc_dispatch with the same validation as any
 * other caller. Tensor parallelism (tp_world > 1) shards q/k/v/gate/up/
 * lm_head by output rows and o/down by input columns and inserts an
 * all-reduce after o and down and an all-gather of the logits; the device
 * must have been joined to a communicator with slc_comm_init.
 */
#ifndef STARLIGHT_ENGINE_H
#define STARLIGHT_ENGINE_H

#include <stdint.h>

#include "starlight_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef struct slc_llama slc_llama;

typedef struct {
    uint32_t layers, hidden, heads, kv_heads, head_dim, inter, vocab;
    uint32_t batch;       /* sequences per step */
    uint32_t prefill_len; /* tokens per sequence in a prefill step (program shape) */
    uint32_t max_seq;     /* KV cache positions */
    float eps;            /* RmsNorm eps */
    float theta;          /* RoPE (NeoX) theta */
    int32_t quant_format; /* -1 dense f32 matrices, else slc_quant_format */
    uint32_t group_size;  /* quantization group along K */
    int32_t tp_rank, tp_world;
    uint32_t decompose_swiglu; /* 1: MatMulNT x2, Silu, Mul, MatMulNT instead of SwiGlu */
} slc_llama_config;

/* Weight roles (docs/ARCH-0006 section 4). Matrices are [out, in]. */
typedef enum {
    SLC_W_EMBED = 0, SLC_W_ATTN_NORM = 1, SLC_W_Q = 2, SLC_W_K = 3, SLC_W_V = 4, SLC_W_O = 5,
    SLC_W_MLP_NORM = 6, SLC_W_GATE = 7, SLC_W_UP = 8, SLC_W_DOWN = 9, SLC_W_FINAL_NORM = 10,
    SLC_W_LM_HEAD = 11
} slc_weight_role;

typedef enum { SLC_STEP_PREFILL = 0, SLC_STEP_DECODE = 1 } slc_step_mode;

int slc_llama_create(slc_device *device, const slc_llama_config *config, slc_llama **out);
void slc_llama_destroy(slc_llama *model);
/* Uploads the FULL (unsharded) f32 weight of a role; the engine keeps this
 * rank's shard, quantized on the device when the config asks for it. */
int slc_llama_set_weight(slc_llama *model, int role, uint32_t layer, const float *full,
                         uint64_t len);
/* The same role from already quantized weights in the model's format and
 * group size (the sl-precision format: payload rows of ceil(K/2) (INT4) or K
 * bytes, scales [N, ceil(K/group)] f32), full unsharded matrices: this
 * rank's shard is sliced out (whole rows, or whole groups of columns) and
 * stored as it is, without quantizing again. */
int slc_llama_set_quant_weight(slc_llama *model, int role, uint32_t layer, const uint8_t *codes,
                               uint64_t codes_bytes, const float *scales, uint64_t scales_len);
/* Synthetic weights generated on the device: matrices and the embedding
 * N(0, std), norm weights N(1, 0.1), one stream per (role, layer) derived
 * from `seed`; element (r, c) of the full matrix is draw r * cols + c, so
 * every tensor-parallel split sees the same model. */
int slc_llama_init_random(slc_llama *model, uint64_t seed, float std);
/* Engine::step. ids/positions: batch * seq values (seq = prefill_len or 1);
 * seq_len: real tokens per sequence (LastToken); logits: batch * vocab. */
int slc_llama_step(slc_llama *model, int mode, const uint32_t *ids, const uint32_t *positions,
                   uint32_t seq_len, uint32_t past_len, float *logits, uint64_t logits_len);
/* Greedy generation: prompt is batch * prefill_len ids; writes
 * batch * (steps + 1) ids (row-major per step: out[s * batch + b]) and, if
 * margins is not NULL, the top-1 minus top-2 logit of every choice. */
int slc_llama_generate(slc_llama *model, const uint32_t *prompt, uint32_t steps,
                       uint32_t *out_ids, float *margins);
/* Introspection for tests and benchmarks. */
int slc_llama_kv_buffer(const slc_llama *model, uint32_t *buffer, uint64_t *elements);
int slc_llama_command_count(const slc_llama *model, int mode, uint64_t *count);
int slc_llama_weight_bytes(const slc_llama *model, uint64_t *bytes);
/* The BufferRef and Value a command would pass for a weight (this rank's
 * shard), so a caller can dispatch single operators on the model's weights. */
int slc_llama_weight_ref(const slc_llama *model, int role, uint32_t layer, slc_buffer_ref *ref,
                         slc_value *value);
/* Device time (CUDA events on the device stream) from the first to the last
 * command of the most recent slc_llama_step, in milliseconds. */
int slc_llama_last_step_ms(const slc_llama *model, float *ms);
/* Steps (since creation) that relaunched their program's captured graph
 * directly: with command capture on, once a program's commands have run as
 * one graph, later steps of that program fill the graph's scalar table
 * (seq_len, past_len) and relaunch it instead of dispatching every command
 * again. Results are those of the dispatched step. */
int slc_llama_memo_steps(const slc_llama *model, uint64_t *count);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif
