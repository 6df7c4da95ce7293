/*
 * starlight_cuda.h -- C ABI of backend-cuda, the B200 (sm_100a) compute
 * backend for StarLight.
 *
 * The core of this header is a one-to-one C rendering of the frozen
 * `sl_device::Device` trait (docs/ARCH-0007 section 3.1, lines 48-97 of the
 * StarLight checkout; CPU implementation crates/backends/backend-cpu/src/
 * device.rs:114-213). A Rust `backend-cuda` crate implements `impl Device`
 * by forwarding each trait method to the function named beside it:
 *
 *   Device::allocate_f32  -> slc_allocate_f32   (device.rs:115-117)
 *   Device::allocate_u32  -> slc_allocate_u32   (device.rs:119-121)
 *   Device::upload_f32    -> slc_upload_f32     (device.rs:123-134)
 *   Device::upload_u32    -> slc_upload_u32     (device.rs:136-147)
 *   Device::download_f32  -> slc_download_f32   (device.rs:149-160)
 *   Device::download_u32  -> slc_download_u32   (device.rs:162-173)
 *   Device::dispatch      -> slc_dispatch       (device.rs:175-208)
 *   Device::synchronize   -> slc_synchronize    (device.rs:210-212)
 *   CpuDevice::new        -> slc_device_create  (device.rs:43-45)
 *
 * Conventions (identical to the trait):
 *   - a BufferId is an opaque u32 index; a BufferRef addresses `len`
 *     ELEMENTS at element `offset` of a buffer;
 *   - `dispatch` runs one operator; completion means "enqueued", the caller
 *     must call slc_synchronize before reading results (docs/ARCH-0004:356);
 *   - `dispatch` never allocates; every validation runs before any work is
 *     enqueued; nothing aborts the process;
 *   - every function returns an slc_status mirroring the DeviceError variant
 *     (docs/ARCH-0007:63-71); slc_last_error() returns its payload.
 *
 * Extensions beyond the trait (the reference has no quantized execution and
 * no multi-device support) are marked EXTENSION and are documented where
 * declared.
 */
#ifndef STARLIGHT_CUDA_H
#define STARLIGHT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define SLC_ABI_VERSION 1u
/* sl-ir IR_VERSION this backend implements (docs/ARCH-0007:44). */
#define SLC_IR_VERSION 2u
#define SLC_MAX_RANK 8u          /* device.rs:29 */
#define SLC_MAX_INPUTS 4u        /* device.rs:26 */
#define SLC_MAX_OUTPUTS 1u       /* device.rs:27 */
#define SLC_MIN_BUFFER_ALIGN 64u /* docs/ARCH-0004:147-151, runtime.rs:55 */

typedef struct slc_device slc_device;

/* DeviceError variants (docs/ARCH-0007:63-71). */
typedef enum {
    SLC_OK = 0,
    SLC_ERR_OUT_OF_MEMORY = 1,  /* OutOfMemory { requested }            */
    SLC_ERR_INVALID_BUFFER = 2, /* InvalidBuffer(BufferId)              */
    SLC_ERR_INVALID_RANGE = 3,  /* InvalidRange { buffer, offset, len } */
    SLC_ERR_UNSUPPORTED_OP = 4, /* UnsupportedOp(OpCode)                */
    SLC_ERR_SHAPE_OVERFLOW = 5, /* ShapeOverflow                        */
    SLC_ERR_EXECUTION = 6,      /* Execution(&'static str)              */
    SLC_ERR_UNIMPLEMENTED = 7   /* Unimplemented(&'static str)          */
} slc_status;

/* Payload of the last error returned on a device. `message` points to a
 * static string (never freed, valid for the life of the process). */
typedef struct {
    int32_t status;
    uint32_t buffer;    /* InvalidBuffer, InvalidRange */
    uint64_t offset;    /* InvalidRange (elements)     */
    uint64_t len;       /* InvalidRange (elements)     */
    uint64_t requested; /* OutOfMemory (elements)      */
    uint32_t opcode;    /* UnsupportedOp               */
    const char *message;
} slc_error;

/* sl_ir::DType, declaration order (docs/ARCH-0004:82). */
typedef enum {
    SLC_F32 = 0, SLC_F16 = 1, SLC_BF16 = 2, SLC_U32 = 3, SLC_I32 = 4, SLC_U8 = 5, SLC_I8 = 6
} slc_dtype;

/* sl_ir::ValueRole, declaration order (docs/ARCH-0004:104-111). */
typedef enum {
    SLC_ROLE_INPUT = 0, SLC_ROLE_SCALAR = 1, SLC_ROLE_OUTPUT = 2,
    SLC_ROLE_PARAM = 3, SLC_ROLE_STATE = 4, SLC_ROLE_TEMP = 5
} slc_role;

/* sl_ir::TensorEncoding (docs/ARCH-0004:120-131). */
typedef enum { SLC_ENC_DENSE = 0, SLC_ENC_GROUPWISE = 1, SLC_ENC_OPAQUE = 2 } slc_encoding;
typedef enum { SLC_QUANT_INT4 = 0, SLC_QUANT_INT8 = 1 } slc_quant_format;

/* sl_ir::Value with its shape resolved to constants (a CommandBuffer holds
 * no Dim::Sym, docs/ARCH-0004:339). `dims[0..rank)` are the extents. */
typedef struct {
    uint32_t dtype;        /* slc_dtype */
    uint32_t role;         /* slc_role */
    uint32_t rank;         /* <= SLC_MAX_RANK */
    uint32_t dims[SLC_MAX_RANK];
    uint32_t encoding;     /* slc_encoding */
    uint32_t quant_format; /* slc_quant_format, GROUPWISE only */
    uint32_t group_size;   /* GROUPWISE only */
} slc_value;

/* sl_device::BufferRef (docs/ARCH-0007:55-60): offset and len in elements. */
typedef struct {
    uint32_t buffer;
    uint32_t reserved;
    uint64_t offset;
    uint64_t len;
} slc_buffer_ref;

/* sl_ir::OpCode. The discriminants are the #[repr(u16)] declaration order of
 * docs/ARCH-0004:226-235 and are part of the ABI (never reused, :522). */
typedef enum {
    SLC_OP_MATMUL_NT = 0,
    SLC_OP_MATMUL_NN = 1,
    SLC_OP_SOFTMAX = 2,
    SLC_OP_SOFTMAX_CAUSAL = 3,
    SLC_OP_RMS_NORM = 4,
    SLC_OP_ROPE = 5,
    SLC_OP_SILU = 6,
    SLC_OP_MUL = 7,
    SLC_OP_ADD = 8,
    SLC_OP_SCALE = 9,
    SLC_OP_GATHER = 10,
    SLC_OP_LAST_TOKEN = 11,
    SLC_OP_KV_APPEND = 12,
    SLC_OP_SPLIT_HEADS = 13,
    SLC_OP_MERGE_HEADS = 14,
    SLC_OP_CAUSAL_ATTENTION = 15,
    SLC_OP_SWIGLU = 16,
    SLC_OP_RMS_NORM_MATMUL = 17,
    /* EXTENSION: tensor-parallel collectives, outside the sl-ir opcode space.
     * ALL_REDUCE: in-place sum of one F32 value over the communicator set up
     * by slc_comm_init (one input port, no output). ALL_GATHER: gathers each
     * rank's [rows, cols] F32 input into an output [rows, world * cols]
     * (rank r's block at columns [r*cols, (r+1)*cols)). */
    SLC_OP_EXT_ALL_REDUCE = 0x8000,
    SLC_OP_EXT_ALL_GATHER = 0x8001,
    /* EXTENSION: residual add with a broadcast bias (no sl-ir counterpart;
     * the benchmark's elementwise sweep): inputs a, b of one shape
     * [..., cols] and bias [cols]; output of a's shape,
     * out = (a + b) + bias[col], each sum rounded as f32 (bit-exact). */
    SLC_OP_EXT_ADD_BIAS = 0x8002
} slc_opcode;

typedef enum { SLC_ROPE_NEOX = 0, SLC_ROPE_GPTJ = 1 } slc_rope_variant;

/* sl_ir::Op: the opcode plus the attributes of its variant
 * (docs/ARCH-0004:237-258). Unused attributes are ignored. */
typedef struct {
    uint16_t code;         /* slc_opcode */
    uint16_t rope_variant; /* Rope */
    uint32_t layer;        /* KvAppend, CausalAttention */
    uint32_t heads;        /* SplitHeads, MergeHeads, CausalAttention */
    uint32_t kv_heads;     /* CausalAttention */
    uint32_t head_dim;     /* SplitHeads, MergeHeads, CausalAttention */
    float eps;             /* RmsNorm, RmsNormMatMul */
    float theta;           /* Rope */
    float scale;           /* CausalAttention */
    float factor;          /* Scale */
} slc_op;

/* sl_ir::DeviceCapabilities (docs/ARCH-0004:396-408). Op sets are bit masks
 * over opcodes 0..63; dtypes is a bit mask over slc_dtype. */
typedef struct {
    uint32_t ir_version;
    uint64_t core_ops;
    uint64_t composite_ops;
    uint32_t dtypes;
    uint32_t min_buffer_align;
    uint64_t max_scratchpad_bytes;
    uint64_t max_value_bytes;
    uint32_t head_dim_multiple_of;
    uint32_t matmul_k_multiple_of;
    uint32_t max_heads;
    uint32_t quant_formats; /* EXTENSION: bit mask over slc_quant_format */
} slc_capabilities;

typedef struct {
    /* Device scratch for split-K partial results, reserved once at creation
     * because dispatch must not allocate. 0 selects the default (256 MiB). */
    uint64_t workspace_bytes;
    /* Host staging buffer (pinned) for upload/download. 0: default 16 MiB. */
    uint64_t staging_bytes;
} slc_device_options;

/* ---- device lifetime (CpuDevice::new, device.rs:43) --------------------- */
int slc_device_create(int ordinal, slc_device **out);
int slc_device_create_ex(int ordinal, const slc_device_options *options, slc_device **out);
void slc_device_destroy(slc_device *device);
int slc_last_error(const slc_device *device, slc_error *out);
int slc_get_capabilities(const slc_device *device, slc_capabilities *out);
/* Static description of a status code. */
const char *slc_status_name(int status);

/* ---- Device trait (docs/ARCH-0007:73-90) -------------------------------- */
int slc_allocate_f32(slc_device *device, uint64_t elements, uint64_t align, uint32_t *out_buffer);
int slc_allocate_u32(slc_device *device, uint64_t elements, uint64_t align, uint32_t *out_buffer);
int slc_upload_f32(slc_device *device, uint32_t buffer, const float *data, uint64_t len);
int slc_upload_u32(slc_device *device, uint32_t buffer, const uint32_t *data, uint64_t len);
int slc_download_f32(slc_device *device, uint32_t buffer, float *out, uint64_t len);
int slc_download_u32(slc_device *device, uint32_t buffer, uint32_t *out, uint64_t len);
int slc_dispatch(slc_device *device, const slc_op *op,
                 const slc_buffer_ref *inputs, const slc_value *input_values, uint64_t n_inputs,
                 const slc_buffer_ref *outputs, const slc_value *output_values, uint64_t n_outputs,
                 const uint32_t *scalars, uint64_t n_scalars);
int slc_synchronize(slc_device *device);

/* ---- EXTENSION: quantized weights (gap G-16, docs/ARCH-0008:122) ---------
 * A GroupwiseQuantized Param (docs/ARCH-0004:120-131, scale tensor a
 * separate Param, docs/ARCH-0006 section 3.1) is stored in a U32 buffer
 * holding the packed payload; its BufferRef.len counts u32 words
 * (ceil(rows * row_bytes / 4)). row_bytes = ceil(K/2) for INT4 (two's
 * complement nibbles, even k in the low nibble) and K for INT8 (signed
 * bytes). The scales are an F32 buffer [rows, ceil(K / group)], scale =
 * max|w| / qmax over each group along K. slc_bind_quant tells the device
 * which scale buffer belongs to a payload buffer; MatMulNT, SwiGlu and
 * RmsNormMatMul consume such a weight through the dequant-fused kernels. */
int slc_bind_quant(slc_device *device, uint32_t codes_buffer, uint32_t scales_buffer,
                   uint32_t quant_format, uint32_t group_size);
/* Quantizes an F32 [rows, k] matrix already on the device into a payload
 * buffer and a scale buffer (the sl-precision format above); bit-exact with
 * the format's CPU definition. */
int slc_quantize(slc_device *device, slc_buffer_ref weights, uint64_t rows, uint64_t k,
                 uint32_t quant_format, uint32_t group_size, uint32_t codes_buffer,
                 uint32_t scales_buffer);
/* Writes (float)code * scale for every element into an F32 [rows, k] ref. */
int slc_dequantize(slc_device *device, uint32_t codes_buffer, uint32_t scales_buffer,
                   uint64_t rows, uint64_t k, uint32_t quant_format, uint32_t group_size,
                   slc_buffer_ref out);

/* ---- EXTENSION: device-resident data ------------------------------------
 * Copies `len` f32 from device memory (e.g. a framework-owned tensor on the
 * same GPU) into a buffer at element `offset`, stream-ordered. */
int slc_copy_f32_from_device(slc_device *device, uint32_t buffer, uint64_t offset,
                             const void *device_src, uint64_t len);
/* Releases a buffer's device memory; its BufferId becomes invalid. The
 * Device trait has no deallocation; this exists for temporaries created
 * outside the step path (weight conversion scratch). */
int slc_release(slc_device *device, uint32_t buffer);
/* Fills an F32 ref with N(mean, std) draws number offset.. of the stream
 * `seed` (splitmix64 of the element index + Box-Muller): synthetic weights
 * for models too large to build on the host. */
int slc_fill_normal(slc_device *device, slc_buffer_ref out, uint64_t seed, uint64_t offset,
                    float mean, float std);
/* Device address of element 0 of a buffer (interop and tests). */
int slc_buffer_device_ptr(slc_device *device, uint32_t buffer, void **out);
/* The CUDA stream (cudaStream_t) every dispatch is enqueued on. */
int slc_device_stream(slc_device *device, void **out_stream);
/* Number of kernels this device has launched (for launch accounting). */
uint64_t slc_kernel_launch_count(const slc_device *device);

/* ---- EXTENSION: command capture and replay -------------------------------
 * With capture enabled, dispatches are validated as usual (errors are still
 * returned by slc_dispatch) but their launches are deferred until the next
 * call that makes their effects observable (synchronize, flush, upload,
 * download, ...). When the same sequence of operators on the same buffer
 * ranges repeats (only the seq_len / past_len scalars of LastToken,
 * KvAppend and CausalAttention may change), it is replayed as one CUDA graph
 * launch with the new scalars: captured the second time it is seen, replayed
 * from the third. Results are those of eager execution. Off by default. */
int slc_set_capture(slc_device *device, int enabled);
/* Submits deferred work to the device stream without waiting for it. */
int slc_flush(slc_device *device);
typedef struct {
    uint64_t captures;           /* graphs captured */
    uint64_t replays;            /* graph replays */
    uint64_t replayed_commands;  /* commands executed inside graphs */
    uint64_t eager_commands;     /* commands launched one by one */
} slc_capture_info;
int slc_capture_stats(const slc_device *device, slc_capture_info *out);

/* ---- EXTENSION: persistent decode-layer fusion ----------------------------
 * With capture enabled, a run of batch-1 llama-dense layers (the sixteen
 * commands per layer of the llama-dense lowering, one token, one sequence,
 * no tensor parallelism) executes as one cooperative kernel launch. The
 * environment variable SLC_DECODE_FUSION=0, read when capture is enabled,
 * keeps the per-command kernels. slc_decode_fusion_stats reports the fused
 * launches the library enqueued (a launch captured into a graph counts once,
 * however often the graph replays), those the runtime refused (the commands
 * then ran unfused) and the device time of the most recent execution in
 * milliseconds (-1 when none finished), from the kernel's own global-timer
 * stamps of its start and end; it waits for the device stream. */
typedef struct {
    uint64_t launched;
    uint64_t refused;
    float last_ms;
    float reserved;
} slc_decode_fusion_info;
int slc_decode_fusion_stats(const slc_device *device, slc_decode_fusion_info *out);

/* ---- EXTENSION: tensor parallelism over NCCL -----------------------------
 * slc_comm_unique_id fills 128 bytes on one rank (an ncclUniqueId) that the
 * caller broadcasts; every rank then calls slc_comm_init with it. NCCL is
 * loaded at run time (libnccl.so.2). */
int slc_comm_unique_id(uint8_t out_id[128]);
int slc_comm_init(slc_device *device, const uint8_t unique_id[128], int rank, int world);
int slc_comm_world(const slc_device *device, int *rank, int *world);
/* Whether the peer-memory paths are on (all ranks agreed at slc_comm_init):
 * the fused all-reduce + Add + RmsNorm kernel, and persistent decode-layer
 * fusion under tensor parallelism (exchanges inside the kernel). Off when any
 * rank failed to map its peers or set SLC_PEER_ALLREDUCE=0 (both) or
 * SLC_DECODE_FUSION=0 (the second); NCCL carries the all-reduces then. */
int slc_comm_peer_status(const slc_device *device, int *peer_allreduce, int *decode_fusion);
/* The communicator's asynchronous error (ncclCommGetAsyncError): SLC_OK while
 * healthy, SLC_ERR_EXECUTION once NCCL reports a failure or after
 * slc_comm_abort. */
int slc_comm_async_error(slc_device *device);
/* Tears this rank's communicator down without waiting for the other ranks
 * (ncclCommAbort), e.g. after a host-side check found that a peer left
 * between steps; captured graphs and peer mappings are dropped, and later
 * collectives on this device fail with SLC_ERR_EXECUTION instead of waiting
 * for the missing rank. */
int slc_comm_abort(slc_device *device);

/* ---- EXTENSION (no counterpart in the reference): quantized matmul that
 * allocates nothing ---------------------------------------------------------
 * out[m, n] = x[m, k] . dequant(codes, scales)[n, k]^T, the computation of
 * slc_dispatch(MatMulNT) on a GroupwiseQuantized weight, on device pointers
 * the caller owns and a stream the caller names. For callers that cannot let
 * a library allocate device memory: a host whose allocator or memory pool
 * owns the GPU, a fixed memory budget, or a latency-critical loop in which
 * cudaMalloc/cudaFree would synchronize the device. Such callers cannot create
 * an slc_device (creation reserves a workspace).
 *
 * x: f32 [m, k]; codes: rows of ceil(k/2) bytes (INT4) or k bytes (INT8) in
 * the slc_bind_quant format; scales: f32 [n, ceil(k/group_size)]; out: f32
 * [m, n]; stream: a cudaStream_t (NULL = legacy default stream). The call is
 * asynchronous on that stream.
 *
 * Scratch: one fixed device array of SLC_NOALLOC_SCRATCH_BYTES inside the
 * library (on each device that uses it). Decode-sized calls (m <= 64) keep
 * the split-K tickets and partial sums there; prefill-sized calls (m > 64)
 * keep the tcgen05 GEMM's bf16 hi/lo copies of x there, as many rows per
 * pass as fit. The tickets must start at zero: each call clears them on the
 * stream before its kernels. A decode-sized problem whose partial sums would
 * exceed the array (large n times its split factor) is rejected with
 * SLC_ERR_OUT_OF_MEMORY and a message rather than run on a slower GEMV that
 * needs less scratch. The first call on each device (with that device
 * current) looks up the array's device address; make that first call
 * outside any stream capture. Every call, whatever its size, shares the
 * array: calls that overlap in time on one device (several streams or host
 * threads) race; serialize them, e.g. on one stream.
 *
 * error_word: device-accessible memory (device memory, or mapped pinned host
 * memory) that a kernel sets to a nonzero code if one of its bounded waits
 * gives up (the output is then incomplete). The library only ever sets it;
 * the caller clears it and reads it after synchronizing the stream. NULL:
 * such a failure is not reported.
 * Returns an slc_status; *error_message (if not NULL) is set to a static
 * string on failure. */
#define SLC_NOALLOC_SCRATCH_BYTES (8u << 20)
int slc_qmatmul_noalloc(const float *x, uint64_t m, const void *codes, const float *scales,
                        uint64_t n, uint64_t k, uint32_t quant_format, uint32_t group_size,
                        float *out, void *stream, uint32_t *error_word,
                        const char **error_message);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif
#endif
