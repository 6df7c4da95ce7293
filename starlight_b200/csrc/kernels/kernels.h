// Host-side launchers of the backend-cuda kernels. Every launcher enqueues
// on `stream`, performs no allocation and returns the launch status.
// Shapes have been validated by the device layer before any call.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace slc {
namespace k {

// ---- elementwise (elementwise.cu) ------------------------------------------
cudaError_t add(cudaStream_t s, const float *a, const float *b, float *out, size_t n);
cudaError_t mul(cudaStream_t s, const float *a, const float *b, float *out, size_t n);
cudaError_t scale(cudaStream_t s, const float *x, float factor, float *out, size_t n);
cudaError_t silu(cudaStream_t s, const float *x, float *out, size_t n);
// out = silu(a) * b (SwiGLU gate epilogue).
cudaError_t silu_mul(cudaStream_t s, const float *a, const float *b, float *out, size_t n);
// out[r, c] = a[r, c] + b[r, c] + bias[c]  (residual add with a broadcast bias)
cudaError_t add_bias(cudaStream_t s, const float *a, const float *b, const float *bias,
                     float *out, size_t rows, size_t cols);
cudaError_t copy_f32(cudaStream_t s, const float *src, float *dst, size_t n);

// ---- reductions (norm.cu, softmax.cu) --------------------------------------
cudaError_t rms_norm(cudaStream_t s, const float *x, const float *w, float *out, size_t rows,
                     size_t hidden, float eps);
// Residual Add then RmsNorm in one launch: sum = a + b, out = rms_norm(sum).
// Supported where rms_norm itself keeps a row in registers.
bool add_rms_norm_supported(const float *a, const float *b, const float *sum, const float *w,
                            const float *out, size_t rows, size_t hidden);
cudaError_t add_rms_norm(cudaStream_t s, const float *a, const float *b, float *sum,
                         const float *w, float *out, size_t rows, size_t hidden, float eps);
cudaError_t softmax(cudaStream_t s, const float *x, float *out, size_t rows, size_t cols);
cudaError_t softmax_causal(cudaStream_t s, const float *x, float *out, size_t rows, size_t cols,
                           size_t seq, size_t past_len);

// ---- rope.cu ----------------------------------------------------------------
cudaError_t rope(cudaStream_t s, const float *x, const uint32_t *positions, float *out,
                 size_t batch, size_t heads, size_t seq, size_t head_dim, float theta,
                 int gptj);

// ---- layout.cu ---------------------------------------------------------------
cudaError_t gather(cudaStream_t s, const float *table, const uint32_t *ids, float *out,
                   size_t vocab, size_t hidden, size_t rows, uint32_t *error_flag);
// d_seq_len: device copy of seq_len (graph replay) or null; err: error word.
cudaError_t last_token(cudaStream_t s, const float *x, float *out, size_t batch, size_t seq,
                       size_t hidden, size_t seq_len, const uint32_t *d_seq_len = nullptr,
                       uint32_t *err = nullptr);
cudaError_t split_heads(cudaStream_t s, const float *x, float *out, size_t batch, size_t seq,
                        size_t heads, size_t head_dim);
cudaError_t merge_heads(cudaStream_t s, const float *x, float *out, size_t batch, size_t seq,
                        size_t heads, size_t head_dim);
// dst[r, b * cols + c] = src[b, r, c] for b < blocks (rank blocks -> rows).
cudaError_t interleave_blocks(cudaStream_t s, const float *src, float *dst, size_t blocks,
                              size_t rows, size_t cols);

// ---- attention.cu --------------------------------------------------------------
struct KvGeometry {
    size_t batch, layers, layer, kv_heads, head_dim, max_seq;
};
cudaError_t kv_append(cudaStream_t s, const float *k, const float *v, float *cache,
                      const KvGeometry &g, size_t past_len, size_t seq,
                      const uint32_t *d_past = nullptr);
// Workspace needed by causal_attention for the given shape (bytes);
// device_past: past_len will be read from device memory (planned for max_seq).
size_t attention_workspace_bytes(size_t batch, size_t heads, size_t kv_heads, size_t seq,
                                 size_t past_len, size_t head_dim, size_t max_seq,
                                 bool device_past);
struct AttnScratch {
    void *workspace;        // chunk partials
    size_t workspace_bytes;
    unsigned *tickets;      // zeroed, reset by the kernels
    size_t ticket_count;
    uint32_t *err;          // device error word
};
// Appends k / v at past_len and attends (attention.rs:129-219). d_past, if
// set, is a device copy of past_len (read by the kernels).
cudaError_t causal_attention(cudaStream_t s, const float *q, const float *k, const float *v,
                             float *cache, float *out, const KvGeometry &g, size_t heads,
                             size_t seq, size_t past_len, float scale, const AttnScratch &scr,
                             const uint32_t *d_past = nullptr);

// Decode (seq 1) attention block: SplitHeads q/k/v, Rope q/k, causal
// attention with the KV append, MergeHeads, as two launches that leave every
// output buffer as the seven commands would (attention.cu). early_cache:
// no kernel that may still run writes this KV cache, so its cached keys may
// be read before the programmatic dependency wait.
struct DecodeBlockIo {
    const float *q, *k, *v;  // [B, 1, H * D], [B, 1, Hkv * D] x 2
    const uint32_t *pos;     // [B, 1]
    float *qs, *ks, *vs, *qr, *kr;
    float *out, *out_merged;
    float *scratch;          // decode_block_scratch_floats(...) floats, private
};
size_t decode_block_scratch_floats(size_t batch, size_t heads, size_t kv_heads, size_t head_dim);
bool decode_block_supported(size_t batch, size_t heads, size_t kv_heads, size_t head_dim,
                            size_t keys_max, size_t ticket_count);
cudaError_t decode_attention_block(cudaStream_t s, const DecodeBlockIo &io, float *cache,
                                   const KvGeometry &g, size_t heads, size_t past_len, float scale,
                                   float theta, int gptj, const AttnScratch &scr,
                                   const uint32_t *d_past, bool early_cache);

// ---- matmul_f32.cu --------------------------------------------------------------
// out[b] = a[b or 0] . w[b or 0]^T (NT) or a . w (NN), batch broadcast when a
// batch count is 1 (device.rs:1301-1407).
cudaError_t matmul_f32(cudaStream_t s, const float *a, const float *w, float *out,
                       size_t batch_a, size_t batch_b, size_t m, size_t k, size_t n,
                       bool transposed);

// ---- gemv_quant.cu ---------------------------------------------------------------
struct QuantWeight {
    const uint8_t *codes;  // payload, rows of row_bytes
    const float *scales;   // [n, groups]
    size_t n, k, group, groups, row_bytes;
    int format;            // 0 INT4, 1 INT8
};
// Prefill GEMM on the tcgen05 tensor cores (gemm_tc.cu): activations split
// into bf16 hi/lo planes in `workspace` (rows processed in passes that fit),
// codes expanded to bf16 in shared memory, group scales applied per group.
bool qgemm_tc_supported(const QuantWeight &w);
size_t qgemm_tc_rows_per_pass(const QuantWeight &w, size_t workspace_bytes);
cudaError_t qgemm_tc(cudaStream_t s, const float *x, size_t m, const QuantWeight &w, float *out,
                     void *workspace, size_t workspace_bytes, uint32_t *err);
// Tiled SIMT GEMM with the weight dequantized on load (prefill-sized m).
cudaError_t qgemm_f32(cudaStream_t s, const float *a, size_t m, const QuantWeight &w, float *out);
size_t qmatmul_workspace_bytes(const QuantWeight &w, size_t m);
// out[m, n] = x[m, k] . dequant(w)[n, k]^T. `err` (optional) receives the
// error code of a kernel whose bounded wait gave up.
cudaError_t qmatmul(cudaStream_t s, const float *x, size_t m, const QuantWeight &w, float *out,
                    void *workspace, size_t workspace_bytes, uint32_t *err = nullptr);
// TMA-fed decode GEMV (gemv_tma.cu), small m; x must be 16-byte aligned.
// A group is up to 4 matrices with the same input, K and format, streamed by
// one launch; with x2 set the input is silu(x) * x2 (SwiGLU), computed while
// it is staged.
struct QuantSeg {
    QuantWeight w;
    float *out;  // [m, w.n]
};
// Decode GEMV for M <= 2 (gemv_lane.cu): whole 16-row tiles per CTA, no
// workspace; used by qgemv_tma_group where its plan fits.
bool qgemv_lane_supported(const QuantSeg *segs, int nseg, size_t m);
cudaError_t qgemv_lane_group(cudaStream_t s, const float *x, const float *x2, size_t m,
                             const QuantSeg *segs, int nseg, uint32_t *err);
bool qgemv_tma_group_supported(const QuantSeg *segs, int nseg, size_t m);
size_t qgemv_tma_group_workspace_bytes(const QuantSeg *segs, int nseg, size_t m);
cudaError_t qgemv_tma_group(cudaStream_t s, const float *x, const float *x2, size_t m,
                            const QuantSeg *segs, int nseg, void *workspace, uint32_t *err);
bool qgemv_tma_supported(const QuantWeight &w, size_t m);
bool qgemv_tma_x_aligned(const float *x);
size_t qgemv_tma_workspace_bytes(const QuantWeight &w, size_t m);
cudaError_t qgemv_tma(cudaStream_t s, const float *x, size_t m, const QuantWeight &w, float *out,
                      void *workspace, uint32_t *err);
cudaError_t quantize(cudaStream_t s, const float *w, size_t n, size_t k, size_t group,
                     int format, uint8_t *codes, float *scales);
cudaError_t dequantize(cudaStream_t s, const QuantWeight &w, float *out);

// ---- fused (fused.cu) -------------------------------------------------------------
// Row-wise inverse RMS of x: inv[r] = 1 / sqrt(mean(x[r]^2) + eps).
cudaError_t rms_inverse(cudaStream_t s, const float *x, float *inv, size_t rows, size_t hidden,
                        float eps);
// y[r, i] = (x[r, i] * inv[r]) * w[i]
cudaError_t rms_apply(cudaStream_t s, const float *x, const float *inv, const float *w,
                      float *out, size_t rows, size_t hidden);

// ---- init.cu ----------------------------------------------------------------
// out[i] = N(mean, std) draw number offset + i of the stream `seed`.
cudaError_t fill_normal(cudaStream_t s, float *out, size_t n, uint64_t seed, uint64_t offset,
                        float mean, float std);

// ---- comm_fused.cu ------------------------------------------------------------
// Tensor-parallel all-reduce of `partial` over NVLink peer memory, fused with
// the residual Add and RmsNorm that follow it (one CTA per row). The peer
// exchange buffers are set up by the communicator (comm.cpp).
constexpr int kMaxPeers = 8;
struct PeerReduceArgs {
    float *peer_data[kMaxPeers];       // data region of each rank's exchange buffer (mapped)
    uint32_t *peer_flags[kMaxPeers];   // flag region of each rank's exchange buffer (mapped)
    const float *local_data;           // this rank's data region
    const uint32_t *local_flags;       // this rank's flag region
    uint32_t *counters;                // [max_rows] call epochs, this rank
    int rank, world;
    size_t max_rows, max_hidden;
    float *partial;                    // [rows, hidden]: partial in, rank-order sum out
    const float *residual;             // [rows, hidden]
    float *sum_out;                    // residual + sum
    float *out;                        // rms_norm(sum_out) * weight
    const float *weight;               // [hidden]
    size_t rows, hidden;
    float eps;
    uint32_t *err;
};
bool allreduce_add_rms_supported(const PeerReduceArgs &a);
cudaError_t allreduce_add_rms(cudaStream_t s, const PeerReduceArgs &a);

// ---- decode_layers.cu ------------------------------------------------------------
// Persistent decode of a run of llama-dense layers at batch 1 (one
// cooperative launch; see decode_layers.cu). Outputs of a layer's sixteen
// commands, in command order:
//   RmsNorm h, MatMulNT q k v, SplitHeads qs ks vs, Rope qr kr,
//   CausalAttention a, MergeHeads am, MatMulNT o, Add x1, RmsNorm h2,
//   SwiGlu f, Add xn.
constexpr int kDlCmds = 16;
enum DlCmd {
    kDlH = 0, kDlQ, kDlK, kDlV, kDlQs, kDlKs, kDlVs, kDlQr, kDlKr, kDlA, kDlAm, kDlO, kDlX1,
    kDlH2, kDlF, kDlXn
};
struct DlLayerIo {
    QuantWeight w[7];          // q, k, v, o, gate, up, down
    const float *wn1, *wn2;    // attention / MLP RmsNorm weights
    float eps1, eps2, scale;   // RmsNorm eps, attention scale
    uint32_t cache_layer;      // the CausalAttention's layer attribute
    uint32_t past;             // host past_len (eager)
    const uint32_t *d_past;    // device past_len (graph replay) or null
    float *cmd[kDlCmds];       // command output buffers
};
// Tensor parallelism of a run (world 1: none). The o and down projections
// hold this rank's columns (partial sums); the kernel all-reduces them over
// peer memory: words[parity][source rank][kDlTpHidden] of {f32 bits, epoch}
// in every rank's exchange region, mapped into all ranks (comm.cpp).
constexpr int kDlTpHidden = 16384;
struct DlPeers {
    int rank = 0, world = 1;
    uint64_t *words[kMaxPeers] = {};
    // This rank's count of fused launches so far (advanced by the last CTA
    // of every launch; it lives with the words, so the exchanges' epochs
    // never repeat while the exchange region exists).
    uint32_t *launches = nullptr;
};
struct DlRun {
    uint32_t layers, hidden, heads, kv_heads, head_dim, inter;
    int format;                // 0 INT4, 1 INT8
    uint32_t group;
    int gptj;
    float theta;
    const float *x0;           // input of the first layer's RmsNorm
    const uint32_t *pos;       // [1] position of the decode token
    float *cache;              // KV state [1, cache_layers, 2, max_seq, kv_heads, head_dim]
    uint32_t cache_layers, max_seq;
    const DlLayerIo *layer;    // [layers]
    DlPeers tp;                // heads, kv_heads, inter and the o / down columns are this rank's
};
bool decode_layers_supported(const DlRun &r);
size_t decode_layers_image_bytes(int layers);
size_t decode_layers_scratch_bytes(const DlRun &r);
// Writes the run's program image (TMA tensor maps of every weight and the
// layer table) into host memory; the caller copies it to dev_image.
bool decode_layers_image(const DlRun &r, void *host_image, size_t bytes, const void *dev_image);
// sync: zeroed device words (kDecodeSyncWords), left zeroed by the kernel
// except the last four: the device global-timer stamps (ns) of the latest
// launch's start (CTA 0 at entry) and end (the last CTA to exit), two u64
// at word kDecodeStampWord.
constexpr int kDecodeSyncWords = 2048;
constexpr int kDecodeStampWord = kDecodeSyncWords - 4;
cudaError_t decode_layers(cudaStream_t s, const DlRun &r, const void *dev_image, void *scratch,
                          size_t scratch_bytes, unsigned *sync, uint32_t *err);

// Whether launches on this thread may overlap their predecessor
// (programmatic dependent launch; on by default).
bool pdl_enabled();
void set_pdl_enabled(bool on);

// Launch counter (incremented by every launcher).
uint64_t launch_count();
void count_launch();
void add_launches(int64_t n);  // graph replays (n > 0) and aborted captures (n < 0)

}  // namespace k
}  // namespace slc
