// Internal state of a backend-cuda device (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>

#include <unordered_map>
#include <vector>

#include "../../include/starlight_cuda.h"
#include "kernels/kernels.h"

struct DeviceBuffer {
    void *alloc = nullptr;  // cudaMalloc result
    char *ptr = nullptr;    // aligned start of element 0
    uint64_t elements = 0;
    bool u32 = false;
    std::vector<uint32_t> shadow;  // host copy of a U32 buffer (written only by upload)
};

struct QuantBinding {
    uint32_t scales;
    uint32_t format;
    uint32_t group;
};

struct CaptureState;  // command capture and graph replay (capture.cpp)
struct CommState;     // NCCL communicator (comm.cpp)
struct DecodeRunState;  // persistent decode-layer fusion (decode_run.cpp)

struct slc_device {
    int ordinal = 0;
    cudaStream_t stream = nullptr;
    std::vector<DeviceBuffer> buffers;
    std::unordered_map<uint32_t, QuantBinding> quant;
    char *workspace = nullptr;
    uint64_t workspace_bytes = 0;
    char *staging = nullptr;
    uint64_t staging_bytes = 0;
    uint32_t *host_flag = nullptr;    // mapped pinned word: kernel error code (0 = none)
    uint32_t *device_flag = nullptr;  // its device address
    slc_error last{};
    CaptureState *capture = nullptr;
    CommState *comm = nullptr;
    DecodeRunState *decode = nullptr;
};

// Device workspace layout (reserved once at creation; dispatch never
// allocates). W = workspace_bytes.
//   [0, 256 KiB)              split-K tickets of the quantized GEMV
//   [256 KiB, W/2 - 64 KiB)   kernel scratch, used by one kernel at a time:
//                             GEMV partial sums, attention chunk partials,
//                             all-gather staging
//   [W/2 - 64 KiB, W/2)       tickets of the decode attention
//   [W/2, W)                  operator intermediates (SwiGlu, RmsNormMatMul)
// Tickets start at zero and every kernel that takes one resets it.
constexpr uint64_t kGemvTicketBytes = 64 * 1024 * sizeof(unsigned);
constexpr uint64_t kAttnTicketBytes = 16 * 1024 * sizeof(unsigned);
inline char *ws_scratch(slc_device *d) { return d->workspace + kGemvTicketBytes; }
inline uint64_t ws_scratch_bytes(slc_device *d) {
    return d->workspace_bytes / 2 - kAttnTicketBytes - kGemvTicketBytes;
}
inline unsigned *ws_attn_tickets(slc_device *d) {
    return reinterpret_cast<unsigned *>(d->workspace + d->workspace_bytes / 2 - kAttnTicketBytes);
}

// Error helpers shared by the operator layer.
int slc_fail(slc_device *d, int status, const char *msg);
int slc_fail_buffer(slc_device *d, uint32_t buffer);
int slc_fail_range(slc_device *d, uint32_t buffer, uint64_t offset, uint64_t len);
int slc_quant_view(slc_device *d, uint32_t codes_buffer, uint64_t offset_words, uint64_t rows,
                   uint64_t k, uint32_t format, uint32_t group, slc::k::QuantWeight *w);

// Capture hooks: flush_capture launches any recorded-but-unlaunched work (a
// no-op when capture is off) and must run before any host-visible effect.
int flush_capture(slc_device *d);
void release_capture(slc_device *d);
// Drops captured graphs (they hold device pointers and quantization views).
void invalidate_capture(slc_device *d);
// Launch one validated command (used by the capture layer). dyn_scalars, if
// set, is a device copy of `scalars` that the kernels read instead (graph
// capture). Returns an slc_status.
int slc_launch_command(slc_device *d, const slc_op *op, const slc_buffer_ref *in,
                       const slc_value *iv, uint64_t n_in, const slc_buffer_ref *out,
                       const slc_value *ov, uint64_t n_out, const uint32_t *scalars,
                       uint64_t n_scalars, const uint32_t *dyn_scalars);
// Consecutive validated MatMulNT commands on the same input (quantized
// weights, decode-sized): launched as one grouped GEMV when the TMA kernel
// takes them (*launched = true); otherwise nothing is launched.
struct MatmulMember {
    const slc_buffer_ref *in;
    const slc_value *iv;
    const slc_buffer_ref *out;
    const slc_value *ov;
};
int slc_launch_matmul_group(slc_device *d, const MatmulMember *mm, int n, bool *launched);
// The seven-command decode attention block (SplitHeads q, k, v; Rope q, k;
// CausalAttention; MergeHeads), each command already validated: launched as
// the fused decode block when its conditions hold (*launched = true);
// otherwise nothing is launched.
struct BlockMember {
    const slc_op *op;
    const slc_buffer_ref *in;
    const slc_value *iv;
    uint64_t n_in;
    const slc_buffer_ref *out;
    const slc_value *ov;
    const uint32_t *scalars;
    uint64_t n_scalars;
};
// early_cache: no command before the block in its segment writes the KV
// state, so the attention kernel may read cached keys before its dependency
// wait.
int slc_launch_attention_block(slc_device *d, const BlockMember *bm, const uint32_t *dyn_past,
                               bool early_cache, bool *launched);
// Add(a, b) -> sum followed by RmsNorm(sum, w) -> out, both validated:
// launched as one kernel when the shapes and buffer reuse allow it.
int slc_launch_add_rmsnorm(slc_device *d, const BlockMember *add, const BlockMember *rms,
                           bool *launched);
// Step memo (capture.cpp): lets a caller that dispatches the same command
// list every step relaunch that list's captured graph without dispatching
// the commands again; only the dynamic scalars change. Owned by the caller.
struct StepMemo {
    uint64_t graph_id = 0;            // 0: empty
    std::vector<uint32_t> slot_src;   // per device-table slot: index of its scalar source
    uint64_t commands = 0;
};
// True when the memo's graph can be relaunched now.
bool capture_memo_valid(slc_device *d, const StepMemo *m);
// Fills the device table from src[0..n_src) and relaunches the memo's graph.
int capture_memo_replay(slc_device *d, StepMemo *m, const uint32_t *src, size_t n_src);
// flush_capture, after which the memo holds the flushed segment's graph if
// the segment was exactly the caller's n_cmds commands (command i taking
// src_count[i] scalars from sources src_flat[...], in order) and ran as a
// graph; empty otherwise.
int capture_flush_memo(slc_device *d, StepMemo *m, const int *src_flat, const uint32_t *src_count,
                       size_t n_cmds);
// Try to record a validated command for graph replay. Returns 1 if the
// command was recorded (launch deferred), 0 if it must be launched now.
int capture_record(slc_device *d, const slc_op *op, const slc_buffer_ref *in,
                   const slc_value *iv, uint64_t n_in, const slc_buffer_ref *out,
                   const slc_value *ov, uint64_t n_out, const uint32_t *scalars,
                   uint64_t n_scalars);

// NCCL hooks (comm.cpp).
void release_comm(slc_device *d);
// Fills the peer-exchange fields of `a` (false when the communicator has no
// peer exchange: world 1, switched off, or setup failed on some rank).
bool comm_peer_args(slc_device *d, slc::k::PeerReduceArgs *a);
// The persistent decode kernel's exchange regions (false: no tensor
// parallelism, peer mappings off, or decode fusion off on some rank).
bool comm_decode_peers(slc_device *d, slc::k::DlPeers *out);
// AllReduce(partial) -> Add(residual, partial) -> RmsNorm(sum), validated:
// launched as the fused peer-memory kernel when its conditions hold.
int slc_launch_allreduce_add_rmsnorm(slc_device *d, const BlockMember *ar, const BlockMember *add,
                                     const BlockMember *rms, bool *launched);
int comm_all_reduce(slc_device *d, float *data, uint64_t count);
int comm_all_gather(slc_device *d, const float *in, float *out, uint64_t rows, uint64_t cols);

// Persistent decode-layer fusion (decode_run.cpp), created with capture.
int decode_run_create(slc_device *d);
void decode_run_release(slc_device *d);
int decode_run_stats(const slc_device *d, slc_decode_fusion_info *out);
// Drops the program images of captured graphs (with the graphs).
void decode_run_invalidate(slc_device *d);
// Commands at the start of cmds[0..n) that form whole decoder layers the
// persistent kernel can run (0: none).
size_t decode_run_match(slc_device *d, const BlockMember *cmds, size_t n);
// Launches the matched run cmds[0..n) (n from decode_run_match). dyn: device
// copies of each command's scalars (graph capture) or null. prepare_only:
// upload a graph's program image before its capture begins, launch nothing.
int decode_run_launch(slc_device *d, const BlockMember *cmds, size_t n, const uint32_t *const *dyn,
                      bool prepare_only, bool *launched);
