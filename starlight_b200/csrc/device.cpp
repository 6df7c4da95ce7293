// backend-cuda device: the C-ABI implementation of sl_device::Device
// (docs/ARCH-0007 section 3.1) on one B200.
//
// Mirrors crates/backends/backend-cpu/src/device.rs: the same port checks
// (validate_call :224-286, validate_port :288-324, check_disjoint
// :341-377), the same per-operator geometry checks and messages (run_op
// :773-1227, geometry helpers :1301-1488), with the scalar reference kernels
// replaced by sm_100a CUDA kernels enqueued on one stream. All validation
// finishes before the first kernel is enqueued, so a rejected command
// changes nothing. No function allocates device memory on the dispatch path:
// buffers, the split-K workspace and the pinned staging area are created
// by slc_device_create / slc_allocate_*.
//
// U32 buffers can only be written by upload (a U32 command output is
// illegal, device.rs:311-316), so the device keeps a host shadow of every
// U32 buffer. Gather validates token ids on the host from that shadow before
// any write, exactly as reference::gather does (layout.rs:25-52).
#include <cuda_runtime.h>
#include <string.h>

#include <algorithm>
#include <new>
#include <unordered_map>
#include <vector>

#include "../../include/starlight_cuda.h"
#include "device_internal.h"
#include "kernels/kernels.h"

using namespace slc;

namespace {

constexpr uint64_t kDefaultWorkspace = 256ull << 20;
constexpr uint64_t kDefaultStaging = 16ull << 20;

int set_error(slc_device *d, int status, const char *msg) {
    d->last = slc_error{};
    d->last.status = status;
    d->last.message = msg;
    return status;
}

int exec_err(slc_device *d, const char *msg) { return set_error(d, SLC_ERR_EXECUTION, msg); }
int unimpl(slc_device *d, const char *msg) { return set_error(d, SLC_ERR_UNIMPLEMENTED, msg); }
int overflow(slc_device *d) {
    return set_error(d, SLC_ERR_SHAPE_OVERFLOW, "tensor shape product overflows");
}
int invalid_buffer(slc_device *d, uint32_t buffer) {
    set_error(d, SLC_ERR_INVALID_BUFFER, "invalid buffer");
    d->last.buffer = buffer;
    return SLC_ERR_INVALID_BUFFER;
}
int invalid_range(slc_device *d, uint32_t buffer, uint64_t offset, uint64_t len) {
    set_error(d, SLC_ERR_INVALID_RANGE, "invalid range");
    d->last.buffer = buffer;
    d->last.offset = offset;
    d->last.len = len;
    return SLC_ERR_INVALID_RANGE;
}
int oom(slc_device *d, uint64_t requested) {
    set_error(d, SLC_ERR_OUT_OF_MEMORY, "out of device memory");
    d->last.requested = requested;
    return SLC_ERR_OUT_OF_MEMORY;
}
int cuda_err(slc_device *d, cudaError_t e) {
    (void)e;
    return exec_err(d, "CUDA kernel launch failed");
}

bool mul_ok(uint64_t a, uint64_t b, uint64_t *out) {
    if (a != 0 && b > UINT64_MAX / a) return false;
    *out = a * b;
    return true;
}

// ---- Dims (device.rs:709-770) -------------------------------------------

struct Dims {
    uint32_t rank = 0;
    uint64_t ext[SLC_MAX_RANK] = {};
};

struct Status {
    int code = SLC_OK;
    const char *msg = nullptr;
    bool ok() const { return code == SLC_OK; }
};

Status st_exec(const char *m) { return Status{SLC_ERR_EXECUTION, m}; }
Status st_overflow() { return Status{SLC_ERR_SHAPE_OVERFLOW, nullptr}; }

Status dims_of(const slc_value &v, Dims *d) {
    if (v.rank > SLC_MAX_RANK) return st_overflow();
    d->rank = v.rank;
    for (uint32_t i = 0; i < v.rank; i++) d->ext[i] = v.dims[i];
    return {};
}

Status dim(const Dims &d, uint32_t i, uint64_t *out) {
    if (i < d.rank) {
        *out = d.ext[i];
        return {};
    }
    return st_exec("operator rank is too small");
}

Status last_dim(const Dims &d, uint64_t *out) {
    if (d.rank == 0) return st_exec("operator requires at least one dimension");
    *out = d.ext[d.rank - 1];
    return {};
}

Status product(const Dims &d, uint32_t end, uint64_t *out) {
    if (end > d.rank) return st_exec("operator rank is too small");
    uint64_t p = 1;
    for (uint32_t i = 0; i < end; i++)
        if (!mul_ok(p, d.ext[i], &p)) return st_overflow();
    *out = p;
    return {};
}

bool same_as(const Dims &a, const Dims &b) {
    if (a.rank != b.rank) return false;
    for (uint32_t i = 0; i < a.rank; i++)
        if (a.ext[i] != b.ext[i]) return false;
    return true;
}

#define TRY(expr)                          \
    do {                                   \
        Status s_ = (expr);                \
        if (!s_.ok()) return s_;           \
    } while (0)

// ---- signatures (docs/ARCH-0004 section 5.2) -------------------------------

struct Sig {
    int inputs, scalars, outputs;
    bool stateful;
};

bool signature(uint32_t code, Sig *s) {
    switch (code) {
    case SLC_OP_MATMUL_NT: case SLC_OP_MATMUL_NN: *s = {2, 0, 1, false}; return true;
    case SLC_OP_SOFTMAX: *s = {1, 0, 1, false}; return true;
    case SLC_OP_SOFTMAX_CAUSAL: *s = {3, 2, 1, false}; return true;
    case SLC_OP_RMS_NORM: *s = {2, 0, 1, false}; return true;
    case SLC_OP_ROPE: *s = {2, 0, 1, false}; return true;
    case SLC_OP_SILU: *s = {1, 0, 1, false}; return true;
    case SLC_OP_MUL: case SLC_OP_ADD: *s = {2, 0, 1, false}; return true;
    case SLC_OP_SCALE: *s = {1, 0, 1, false}; return true;
    case SLC_OP_GATHER: *s = {2, 0, 1, false}; return true;
    case SLC_OP_LAST_TOKEN: *s = {2, 1, 1, false}; return true;
    case SLC_OP_KV_APPEND: *s = {3, 1, 0, true}; return true;
    case SLC_OP_SPLIT_HEADS: case SLC_OP_MERGE_HEADS: *s = {1, 0, 1, false}; return true;
    case SLC_OP_CAUSAL_ATTENTION: *s = {4, 1, 1, true}; return true;
    case SLC_OP_SWIGLU: *s = {4, 0, 1, false}; return true;
    case SLC_OP_RMS_NORM_MATMUL: *s = {3, 0, 1, false}; return true;
    case SLC_OP_EXT_ALL_REDUCE: *s = {1, 0, 0, false}; return true;
    case SLC_OP_EXT_ALL_GATHER: *s = {1, 0, 1, false}; return true;
    case SLC_OP_EXT_ADD_BIAS: *s = {3, 0, 1, false}; return true;
    default: return false;
    }
}

// Storage (in u32 words) of a quantized value of logical shape [..., n, k].
Status quant_storage_words(const slc_value &v, const Dims &d, uint64_t *words, uint64_t *rows,
                           uint64_t *k, uint64_t *row_bytes) {
    if (d.rank < 1) return st_exec("operator requires at least one dimension");
    uint64_t kk = d.ext[d.rank - 1], rr;
    TRY(product(d, d.rank - 1, &rr));
    uint64_t rb = v.quant_format == SLC_QUANT_INT4 ? (kk + 1) / 2 : kk;
    uint64_t bytes;
    if (!mul_ok(rr, rb, &bytes)) return st_overflow();
    *words = (bytes + 3) / 4;
    *rows = rr;
    *k = kk;
    *row_bytes = rb;
    return {};
}

}  // namespace

// ==== device lifetime ========================================================

extern "C" int slc_device_create(int ordinal, slc_device **out) {
    return slc_device_create_ex(ordinal, nullptr, out);
}

extern "C" int slc_device_create_ex(int ordinal, const slc_device_options *opt,
                                    slc_device **out) {
    if (!out) return SLC_ERR_EXECUTION;
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || ordinal < 0 || ordinal >= count)
        return SLC_ERR_EXECUTION;
    if (cudaSetDevice(ordinal) != cudaSuccess) return SLC_ERR_EXECUTION;
    slc_device *d = new (std::nothrow) slc_device();
    if (!d) return SLC_ERR_OUT_OF_MEMORY;
    d->ordinal = ordinal;
    uint64_t ws = opt && opt->workspace_bytes ? opt->workspace_bytes : kDefaultWorkspace;
    uint64_t stg = opt && opt->staging_bytes ? opt->staging_bytes : kDefaultStaging;
    if (cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&d->workspace, ws) != cudaSuccess ||
        cudaMemset(d->workspace, 0, ws) != cudaSuccess ||
        cudaMallocHost(&d->staging, stg) != cudaSuccess ||
        cudaHostAlloc(&d->host_flag, sizeof(uint32_t), cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer(reinterpret_cast<void **>(&d->device_flag), d->host_flag, 0) !=
            cudaSuccess) {
        slc_device_destroy(d);
        return SLC_ERR_OUT_OF_MEMORY;
    }
    d->workspace_bytes = ws;
    d->staging_bytes = stg;
    *out = d;
    return SLC_OK;
}

extern "C" void slc_device_destroy(slc_device *d) {
    if (!d) return;
    cudaSetDevice(d->ordinal);
    if (d->stream) cudaStreamSynchronize(d->stream);
    release_capture(d);
    release_comm(d);
    for (auto &b : d->buffers)
        if (b.alloc) cudaFree(b.alloc);
    if (d->workspace) cudaFree(d->workspace);
    if (d->host_flag) cudaFreeHost(d->host_flag);
    if (d->staging) cudaFreeHost(d->staging);
    if (d->stream) cudaStreamDestroy(d->stream);
    delete d;
}

extern "C" int slc_last_error(const slc_device *d, slc_error *out) {
    if (!d || !out) return SLC_ERR_EXECUTION;
    *out = d->last;
    return SLC_OK;
}

extern "C" const char *slc_status_name(int status) {
    switch (status) {
    case SLC_OK: return "Ok";
    case SLC_ERR_OUT_OF_MEMORY: return "OutOfMemory";
    case SLC_ERR_INVALID_BUFFER: return "InvalidBuffer";
    case SLC_ERR_INVALID_RANGE: return "InvalidRange";
    case SLC_ERR_UNSUPPORTED_OP: return "UnsupportedOp";
    case SLC_ERR_SHAPE_OVERFLOW: return "ShapeOverflow";
    case SLC_ERR_EXECUTION: return "Execution";
    case SLC_ERR_UNIMPLEMENTED: return "Unimplemented";
    default: return "Unknown";
    }
}

extern "C" int slc_get_capabilities(const slc_device *d, slc_capabilities *c) {
    if (!d || !c) return SLC_ERR_EXECUTION;
    *c = slc_capabilities{};
    c->ir_version = SLC_IR_VERSION;
    for (uint32_t op = SLC_OP_MATMUL_NT; op <= SLC_OP_MERGE_HEADS; op++) c->core_ops |= 1ull << op;
    c->composite_ops = (1ull << SLC_OP_CAUSAL_ATTENTION) | (1ull << SLC_OP_SWIGLU) |
                       (1ull << SLC_OP_RMS_NORM_MATMUL);
    c->dtypes = (1u << SLC_F32) | (1u << SLC_U32);
    c->min_buffer_align = SLC_MIN_BUFFER_ALIGN;
    c->max_scratchpad_bytes = 1ull << 40;
    c->max_value_bytes = 1ull << 40;
    c->head_dim_multiple_of = 2;
    c->matmul_k_multiple_of = 1;
    c->max_heads = 1u << 16;
    c->quant_formats = (1u << SLC_QUANT_INT4) | (1u << SLC_QUANT_INT8);
    return SLC_OK;
}

// ==== buffers (device.rs:56-83, :114-173) ====================================

static int allocate(slc_device *d, uint64_t elements, uint64_t align, bool u32,
                    uint32_t *out_buffer) {
    if (!d || !out_buffer) return SLC_ERR_EXECUTION;
    flush_capture(d);
    if (align == 0 || (align & (align - 1)) != 0)
        return exec_err(d, "alignment must be a nonzero power of two");
    if (d->buffers.size() >= UINT32_MAX) return oom(d, elements);
    uint64_t bytes;
    if (!mul_ok(elements, 4, &bytes) || bytes > (1ull << 46)) return oom(d, elements);
    uint64_t pad = align > 256 ? align : 0;
    void *p = nullptr;
    if (cudaSetDevice(d->ordinal) != cudaSuccess ||
        cudaMalloc(&p, (bytes ? bytes : 4) + pad) != cudaSuccess) {
        cudaGetLastError();
        return oom(d, elements);
    }
    if (cudaMemsetAsync(p, 0, (bytes ? bytes : 4) + pad, d->stream) != cudaSuccess) {
        cudaFree(p);
        return oom(d, elements);
    }
    DeviceBuffer b;
    b.alloc = p;
    uintptr_t base = reinterpret_cast<uintptr_t>(p);
    if (pad) base = (base + align - 1) & ~(uintptr_t)(align - 1);
    b.ptr = reinterpret_cast<char *>(base);
    b.elements = elements;
    b.u32 = u32;
    if (u32) b.shadow.assign(elements, 0u);
    d->buffers.push_back(std::move(b));
    *out_buffer = (uint32_t)(d->buffers.size() - 1);
    return SLC_OK;
}

extern "C" int slc_allocate_f32(slc_device *d, uint64_t elements, uint64_t align, uint32_t *out) {
    return allocate(d, elements, align, false, out);
}

extern "C" int slc_allocate_u32(slc_device *d, uint64_t elements, uint64_t align, uint32_t *out) {
    return allocate(d, elements, align, true, out);
}

static DeviceBuffer *slot(slc_device *d, uint32_t id, bool u32) {
    if (id >= d->buffers.size()) return nullptr;
    DeviceBuffer &b = d->buffers[id];
    if (!b.alloc || b.u32 != u32) return nullptr;
    return &b;
}

// Host <-> device copy through the pinned staging area (chunked).
static int copy_h2d(slc_device *d, char *dst, const void *src, uint64_t bytes) {
    const char *s = static_cast<const char *>(src);
    while (bytes) {
        uint64_t n = std::min<uint64_t>(bytes, d->staging_bytes);
        memcpy(d->staging, s, n);
        if (cudaMemcpyAsync(dst, d->staging, n, cudaMemcpyHostToDevice, d->stream) != cudaSuccess ||
            cudaStreamSynchronize(d->stream) != cudaSuccess)
            return exec_err(d, "host to device copy failed");
        dst += n;
        s += n;
        bytes -= n;
    }
    return SLC_OK;
}

static int copy_d2h(slc_device *d, void *dst, const char *src, uint64_t bytes) {
    char *o = static_cast<char *>(dst);
    while (bytes) {
        uint64_t n = std::min<uint64_t>(bytes, d->staging_bytes);
        if (cudaMemcpyAsync(d->staging, src, n, cudaMemcpyDeviceToHost, d->stream) != cudaSuccess ||
            cudaStreamSynchronize(d->stream) != cudaSuccess)
            return exec_err(d, "device to host copy failed");
        memcpy(o, d->staging, n);
        o += n;
        src += n;
        bytes -= n;
    }
    return SLC_OK;
}

static int upload(slc_device *d, uint32_t buffer, const void *data, uint64_t len, bool u32) {
    if (!d) return SLC_ERR_EXECUTION;
    flush_capture(d);
    DeviceBuffer *b = slot(d, buffer, u32);
    if (!b) return invalid_buffer(d, buffer);
    if (b->elements != len) return invalid_range(d, buffer, 0, len);
    if (len && !data) return exec_err(d, "null host pointer");
    if (cudaSetDevice(d->ordinal) != cudaSuccess) return exec_err(d, "cudaSetDevice failed");
    int rc = copy_h2d(d, b->ptr, data, len * 4);
    if (rc == SLC_OK && u32 && len) memcpy(b->shadow.data(), data, len * 4);
    return rc;
}

static int download(slc_device *d, uint32_t buffer, void *out, uint64_t len, bool u32) {
    if (!d) return SLC_ERR_EXECUTION;
    int rc = flush_capture(d);
    if (rc != SLC_OK) return rc;
    DeviceBuffer *b = slot(d, buffer, u32);
    if (!b) return invalid_buffer(d, buffer);
    if (b->elements != len) return invalid_range(d, buffer, 0, len);
    if (len && !out) return exec_err(d, "null host pointer");
    if (cudaSetDevice(d->ordinal) != cudaSuccess) return exec_err(d, "cudaSetDevice failed");
    return copy_d2h(d, out, b->ptr, len * 4);
}

extern "C" int slc_upload_f32(slc_device *d, uint32_t buffer, const float *data, uint64_t len) {
    return upload(d, buffer, data, len, false);
}
extern "C" int slc_upload_u32(slc_device *d, uint32_t buffer, const uint32_t *data, uint64_t len) {
    return upload(d, buffer, data, len, true);
}
extern "C" int slc_download_f32(slc_device *d, uint32_t buffer, float *out, uint64_t len) {
    return download(d, buffer, out, len, false);
}
extern "C" int slc_download_u32(slc_device *d, uint32_t buffer, uint32_t *out, uint64_t len) {
    return download(d, buffer, out, len, true);
}

// Kernels record failures (a gather id out of range, a bounded wait that gave
// up, a device-resident scalar out of bounds) in a mapped host word; the host
// reads and clears it after every synchronization.
static int check_device_flag(slc_device *d) {
    volatile uint32_t *flag = d->host_flag;
    const uint32_t code = *flag;
    if (code == 0) return SLC_OK;
    *flag = 0;
    switch (code) {
    case 1:
        return exec_err(d, "id out of range");
    case 2:
        return exec_err(d, "a kernel's bounded wait timed out");
    case 3:
        return exec_err(d, "a device-resident scalar was out of bounds");
    default:
        return exec_err(d, "a kernel reported an error");
    }
}

extern "C" int slc_flush(slc_device *d) {
    if (!d) return SLC_ERR_EXECUTION;
    return flush_capture(d);
}

extern "C" int slc_synchronize(slc_device *d) {
    if (!d) return SLC_ERR_EXECUTION;
    int rc = flush_capture(d);
    if (rc != SLC_OK) return rc;
    cudaSetDevice(d->ordinal);
    cudaError_t e = cudaStreamSynchronize(d->stream);
    if (e != cudaSuccess) return exec_err(d, "stream synchronization failed");
    return check_device_flag(d);
}

extern "C" int slc_copy_f32_from_device(slc_device *d, uint32_t buffer, uint64_t offset,
                                        const void *src, uint64_t len) {
    if (!d) return SLC_ERR_EXECUTION;
    flush_capture(d);
    DeviceBuffer *b = slot(d, buffer, false);
    if (!b) return invalid_buffer(d, buffer);
    if (offset > b->elements || len > b->elements - offset)
        return invalid_range(d, buffer, offset, len);
    if (len == 0) return SLC_OK;
    if (cudaMemcpyAsync(b->ptr + offset * 4, src, len * 4, cudaMemcpyDeviceToDevice, d->stream) !=
        cudaSuccess)
        return exec_err(d, "device to device copy failed");
    return SLC_OK;
}

extern "C" int slc_release(slc_device *d, uint32_t buffer) {
    if (!d) return SLC_ERR_EXECUTION;
    int rc = flush_capture(d);
    if (rc != SLC_OK) return rc;
    if (buffer >= d->buffers.size() || !d->buffers[buffer].alloc) return invalid_buffer(d, buffer);
    cudaStreamSynchronize(d->stream);
    invalidate_capture(d);  // graphs hold device pointers
    cudaFree(d->buffers[buffer].alloc);
    d->buffers[buffer] = DeviceBuffer{};
    d->quant.erase(buffer);
    return SLC_OK;
}

extern "C" int slc_fill_normal(slc_device *d, slc_buffer_ref out, uint64_t seed, uint64_t offset,
                               float mean, float stdev) {
    if (!d) return SLC_ERR_EXECUTION;
    flush_capture(d);
    DeviceBuffer *b = slot(d, out.buffer, false);
    if (!b) return invalid_buffer(d, out.buffer);
    if (out.offset > b->elements || out.len > b->elements - out.offset)
        return invalid_range(d, out.buffer, out.offset, out.len);
    cudaError_t e = k::fill_normal(d->stream, reinterpret_cast<float *>(b->ptr) + out.offset, out.len,
                                   seed, offset, mean, stdev);
    // Completes before returning: the quantized GEMV streams weights (codes
    // and scales) ahead of its predecessor kernel, so nothing that writes
    // them may still be running when a dispatch is enqueued.
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    return e == cudaSuccess ? SLC_OK : cuda_err(d, e);
}

extern "C" int slc_buffer_device_ptr(slc_device *d, uint32_t buffer, void **out) {
    if (!d || !out) return SLC_ERR_EXECUTION;
    if (buffer >= d->buffers.size() || !d->buffers[buffer].alloc) return invalid_buffer(d, buffer);
    *out = d->buffers[buffer].ptr;
    return SLC_OK;
}

extern "C" int slc_device_stream(slc_device *d, void **out) {
    if (!d || !out) return SLC_ERR_EXECUTION;
    *out = d->stream;
    return SLC_OK;
}

extern "C" uint64_t slc_kernel_launch_count(const slc_device *) { return k::launch_count(); }

// ==== quantized weights =======================================================

extern "C" int slc_bind_quant(slc_device *d, uint32_t codes_buffer, uint32_t scales_buffer,
                              uint32_t format, uint32_t group) {
    if (!d) return SLC_ERR_EXECUTION;
    int rc = flush_capture(d);
    if (rc != SLC_OK) return rc;
    invalidate_capture(d);  // graphs hold quantization views
    if (!slot(d, codes_buffer, true)) return invalid_buffer(d, codes_buffer);
    if (!slot(d, scales_buffer, false)) return invalid_buffer(d, scales_buffer);
    if (format != SLC_QUANT_INT4 && format != SLC_QUANT_INT8)
        return unimpl(d, "unknown quantization format");
    if (group == 0) return exec_err(d, "quantization group size must be nonzero");
    d->quant[codes_buffer] = QuantBinding{scales_buffer, format, group};
    return SLC_OK;
}

static int quant_view(slc_device *d, uint32_t codes_buffer, uint64_t codes_offset_words,
                      uint64_t rows, uint64_t k, uint32_t format, uint32_t group,
                      k::QuantWeight *w) {
    auto it = d->quant.find(codes_buffer);
    if (it == d->quant.end())
        return exec_err(d, "quantized weight buffer has no scale binding");
    if (it->second.format != format || it->second.group != group)
        return exec_err(d, "quantized weight encoding does not match its binding");
    DeviceBuffer *cb = slot(d, codes_buffer, true);
    DeviceBuffer *sb = slot(d, it->second.scales, false);
    if (!cb) return invalid_buffer(d, codes_buffer);
    if (!sb) return invalid_buffer(d, it->second.scales);
    uint64_t row_bytes = format == SLC_QUANT_INT4 ? (k + 1) / 2 : k;
    uint64_t groups = (k + group - 1) / group, nscales, bytes;
    if (!mul_ok(rows, groups, &nscales) || !mul_ok(rows, row_bytes, &bytes)) return overflow(d);
    if (nscales > sb->elements) return invalid_range(d, it->second.scales, 0, nscales);
    if (codes_offset_words > cb->elements || (bytes + 3) / 4 > cb->elements - codes_offset_words)
        return invalid_range(d, codes_buffer, codes_offset_words, (bytes + 3) / 4);
    w->codes = reinterpret_cast<const uint8_t *>(cb->ptr + codes_offset_words * 4);
    w->scales = reinterpret_cast<const float *>(sb->ptr);
    w->n = rows;
    w->k = k;
    w->group = group;
    w->groups = groups;
    w->row_bytes = row_bytes;
    w->format = (int)format;
    return SLC_OK;
}

extern "C" int slc_quantize(slc_device *d, slc_buffer_ref weights, uint64_t rows, uint64_t kk,
                            uint32_t format, uint32_t group, uint32_t codes_buffer,
                            uint32_t scales_buffer) {
    if (!d) return SLC_ERR_EXECUTION;
    flush_capture(d);
    if (format != SLC_QUANT_INT4 && format != SLC_QUANT_INT8)
        return unimpl(d, "unknown quantization format");
    if (group == 0) return exec_err(d, "quantization group size must be nonzero");
    DeviceBuffer *wb = slot(d, weights.buffer, false);
    if (!wb) return invalid_buffer(d, weights.buffer);
    uint64_t n_el;
    if (!mul_ok(rows, kk, &n_el)) return overflow(d);
    if (weights.len != n_el)
        return exec_err(d, "BufferRef length does not match the value element count");
    if (weights.offset > wb->elements || weights.len > wb->elements - weights.offset)
        return invalid_range(d, weights.buffer, weights.offset, weights.len);
    DeviceBuffer *cb = slot(d, codes_buffer, true);
    DeviceBuffer *sb = slot(d, scales_buffer, false);
    if (!cb) return invalid_buffer(d, codes_buffer);
    if (!sb) return invalid_buffer(d, scales_buffer);
    uint64_t row_bytes = format == SLC_QUANT_INT4 ? (kk + 1) / 2 : kk;
    uint64_t groups = (kk + group - 1) / group, nscales, bytes;
    if (!mul_ok(rows, groups, &nscales) || !mul_ok(rows, row_bytes, &bytes)) return overflow(d);
    if ((bytes + 3) / 4 > cb->elements) return invalid_range(d, codes_buffer, 0, (bytes + 3) / 4);
    if (nscales > sb->elements) return invalid_range(d, scales_buffer, 0, nscales);
    cudaError_t e = k::quantize(d->stream, reinterpret_cast<const float *>(wb->ptr) + weights.offset,
                                rows, kk, group, (int)format, reinterpret_cast<uint8_t *>(cb->ptr),
                                reinterpret_cast<float *>(sb->ptr));
    // Completes before returning (see slc_fill_normal).
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->stream);
    if (e != cudaSuccess) return cuda_err(d, e);
    d->quant[codes_buffer] = QuantBinding{scales_buffer, format, group};
    return SLC_OK;
}

extern "C" int slc_dequantize(slc_device *d, uint32_t codes_buffer, uint32_t scales_buffer,
                              uint64_t rows, uint64_t kk, uint32_t format, uint32_t group,
                              slc_buffer_ref out) {
    if (!d) return SLC_ERR_EXECUTION;
    flush_capture(d);
    if (!slot(d, codes_buffer, true)) return invalid_buffer(d, codes_buffer);
    auto it = d->quant.find(codes_buffer);
    if (it == d->quant.end() || it->second.scales != scales_buffer)
        return exec_err(d, "quantized weight buffer has no scale binding");
    k::QuantWeight w{};
    int rc = quant_view(d, codes_buffer, 0, rows, kk, format, group, &w);
    if (rc != SLC_OK) return rc;
    DeviceBuffer *ob = slot(d, out.buffer, false);
    if (!ob) return invalid_buffer(d, out.buffer);
    uint64_t n_el;
    if (!mul_ok(rows, kk, &n_el)) return overflow(d);
    if (out.len != n_el)
        return exec_err(d, "BufferRef length does not match the value element count");
    if (out.offset > ob->elements || out.len > ob->elements - out.offset)
        return invalid_range(d, out.buffer, out.offset, out.len);
    cudaError_t e = k::dequantize(d->stream, w, reinterpret_cast<float *>(ob->ptr) + out.offset);
    return e == cudaSuccess ? SLC_OK : cuda_err(d, e);
}

// ==== dispatch ================================================================

namespace {

struct Port {
    const slc_buffer_ref *ref;
    const slc_value *val;
};

// validate_call, device.rs:224-286.
int validate_call(slc_device *d, const slc_op *op, const slc_value *in_vals, uint64_t n_in,
                  uint64_t n_out, uint64_t n_scalars, Sig *sig_out) {
    if (n_in > SLC_MAX_INPUTS || n_out > SLC_MAX_OUTPUTS)
        return exec_err(d, "too many command ports");
    Sig sig;
    if (!signature(op->code, &sig)) {
        set_error(d, SLC_ERR_UNSUPPORTED_OP, "unsupported operator");
        d->last.opcode = op->code;
        return SLC_ERR_UNSUPPORTED_OP;
    }
    uint64_t state_ports = 0;
    for (uint64_t i = 0; i < n_in; i++)
        if (in_vals[i].role == SLC_ROLE_STATE) state_ports++;
    if (sig.stateful) {
        if (state_ports != 1)
            return exec_err(d, "stateful operator requires exactly one State input");
    } else if (state_ports != 0) {
        return exec_err(d, "stateless operator received a State input");
    }
    if (n_in != (uint64_t)(sig.inputs - sig.scalars) + state_ports)
        return exec_err(d, "input buffer count does not match the operator signature");
    if (n_out != (uint64_t)sig.outputs)
        return exec_err(d, "output count does not match the operator signature");
    if (n_scalars != (uint64_t)sig.scalars)
        return exec_err(d, "scalar count does not match the operator signature");
    *sig_out = sig;
    return SLC_OK;
}

int check_range(slc_device *d, const slc_buffer_ref &r, uint64_t capacity) {
    if (r.offset > UINT64_MAX - r.len) return overflow(d);
    if (r.offset + r.len > capacity) return invalid_range(d, r.buffer, r.offset, r.len);
    return SLC_OK;
}

// validate_port, device.rs:288-324 (plus the quantized-Param storage rule).
int validate_port(slc_device *d, const slc_buffer_ref &r, const slc_value &v, bool output) {
    if (v.role == SLC_ROLE_SCALAR)
        return exec_err(d, "scalar operands must be passed through the scalars argument");
    Dims dm;
    Status s = dims_of(v, &dm);
    if (!s.ok()) return overflow(d);
    uint64_t elements;
    s = product(dm, dm.rank, &elements);
    if (!s.ok()) return overflow(d);
    if (v.encoding == SLC_ENC_OPAQUE)
        return unimpl(d, "opaque quantized encodings cannot be executed");
    if (v.encoding == SLC_ENC_GROUPWISE) {
        if (v.role != SLC_ROLE_PARAM || output)
            return exec_err(d, "only Param values may use a quantized encoding");
        if (v.dtype != SLC_F32) return unimpl(d, "quantized values must have logical dtype F32");
        if (v.quant_format != SLC_QUANT_INT4 && v.quant_format != SLC_QUANT_INT8)
            return unimpl(d, "unknown quantization format");
        if (v.group_size == 0) return exec_err(d, "quantization group size must be nonzero");
        uint64_t words, rows, kk, rb;
        s = quant_storage_words(v, dm, &words, &rows, &kk, &rb);
        if (!s.ok()) return s.code == SLC_ERR_SHAPE_OVERFLOW ? overflow(d) : exec_err(d, s.msg);
        if (words != r.len)
            return exec_err(d, "BufferRef length does not match the quantized payload size");
        DeviceBuffer *b = slot(d, r.buffer, true);
        if (!b) return invalid_buffer(d, r.buffer);
        return check_range(d, r, b->elements);
    }
    if (elements != r.len)
        return exec_err(d, "BufferRef length does not match the value element count");
    if (v.dtype == SLC_F32) {
        DeviceBuffer *b = slot(d, r.buffer, false);
        if (!b) return invalid_buffer(d, r.buffer);
        return check_range(d, r, b->elements);
    }
    if (v.dtype == SLC_U32) {
        if (output) return exec_err(d, "integer command outputs are not supported");
        DeviceBuffer *b = slot(d, r.buffer, true);
        if (!b) return invalid_buffer(d, r.buffer);
        return check_range(d, r, b->elements);
    }
    return unimpl(d, "dtype is not supported by backend-cuda");
}

bool overlap(const slc_buffer_ref &a, const slc_buffer_ref &b) {
    if (a.buffer != b.buffer) return false;
    uint64_t ae = a.offset > UINT64_MAX - a.len ? UINT64_MAX : a.offset + a.len;
    uint64_t be = b.offset > UINT64_MAX - b.len ? UINT64_MAX : b.offset + b.len;
    return a.offset < be && b.offset < ae;
}

// check_disjoint, device.rs:341-377.
int check_disjoint(slc_device *d, const slc_buffer_ref *in, uint64_t n_in,
                   const slc_buffer_ref *out, uint64_t n_out) {
    for (uint64_t i = 0; i < n_in; i++) {
        for (uint64_t j = i + 1; j < n_in; j++)
            if (overlap(in[i], in[j]))
                return exec_err(d, "one command aliases overlapping input ranges");
        for (uint64_t j = 0; j < n_out; j++)
            if (overlap(in[i], out[j]))
                return exec_err(d, "a command output aliases an overlapping input range");
    }
    for (uint64_t i = 0; i < n_out; i++)
        for (uint64_t j = i + 1; j < n_out; j++)
            if (overlap(out[i], out[j]))
                return exec_err(d, "one command aliases overlapping output ranges");
    return SLC_OK;
}

}  // namespace

// Resolved view of one command, shared with the launcher.
int slc_resolve_and_run(slc_device *d, const slc_op *op, const slc_buffer_ref *in,
                        const slc_value *iv, uint64_t n_in, const slc_buffer_ref *out,
                        const slc_value *ov, uint64_t n_out, const uint32_t *scalars,
                        uint64_t n_scalars);

extern "C" int slc_dispatch(slc_device *d, const slc_op *op, const slc_buffer_ref *inputs,
                            const slc_value *input_values, uint64_t n_inputs,
                            const slc_buffer_ref *outputs, const slc_value *output_values,
                            uint64_t n_outputs, const uint32_t *scalars, uint64_t n_scalars) {
    if (!d || !op) return SLC_ERR_EXECUTION;
    if ((n_inputs && (!inputs || !input_values)) || (n_outputs && (!outputs || !output_values)) ||
        (n_scalars && !scalars))
        return exec_err(d, "null port array");
    Sig sig;
    int rc = validate_call(d, op, input_values, n_inputs, n_outputs, n_scalars, &sig);
    if (rc != SLC_OK) return rc;
    for (uint64_t i = 0; i < n_inputs; i++)
        if ((rc = validate_port(d, inputs[i], input_values[i], false)) != SLC_OK) return rc;
    for (uint64_t i = 0; i < n_outputs; i++)
        if ((rc = validate_port(d, outputs[i], output_values[i], true)) != SLC_OK) return rc;
    if ((rc = check_disjoint(d, inputs, n_inputs, outputs, n_outputs)) != SLC_OK) return rc;
    return slc_resolve_and_run(d, op, inputs, input_values, n_inputs, outputs, output_values,
                               n_outputs, scalars, n_scalars);
}

// Used by the operator layer for its error reporting.
int slc_fail(slc_device *d, int status, const char *msg) { return set_error(d, status, msg); }
int slc_fail_buffer(slc_device *d, uint32_t buffer) { return invalid_buffer(d, buffer); }
int slc_fail_range(slc_device *d, uint32_t buffer, uint64_t offset, uint64_t len) {
    return invalid_range(d, buffer, offset, len);
}
int slc_quant_view(slc_device *d, uint32_t codes_buffer, uint64_t offset_words, uint64_t rows,
                   uint64_t kk, uint32_t format, uint32_t group, k::QuantWeight *w) {
    return quant_view(d, codes_buffer, offset_words, rows, kk, format, group, w);
}
