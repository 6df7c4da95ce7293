// slc_qmatmul_noalloc: the quantized (INT4/INT8, group-scaled) matmul for
// callers that must not allocate device memory.
//
// Who needs it: a host whose GPU memory is owned by someone else (an
// inference server or framework with its own pool or caching allocator that
// has reserved the device), a fixed-budget embedded deployment, or a latency
// loop where cudaMalloc/cudaFree would block on or synchronize the device.
// Such callers cannot create an slc_device either, because device creation
// reserves a workspace. This entry point takes their device pointers and
// stream directly and needs no allocation at all: every scratch byte lives
// in a fixed file-scope device array below, loaded with the library on every
// GPU that uses it and kept until the process exits:
//   [0, 256 KiB)   per-row-block tickets of the split-K decode GEMV;
//   [256 KiB, 8 MiB)  the decode GEMV's partial sums (m <= 64), or the
//                  tcgen05 prefill GEMM's bf16 hi/lo activation planes
//                  (m > 64, rows processed in passes that fit).
//
// The computation is the one slc_dispatch(MatMulNT) performs on a
// GroupwiseQuantized weight: the same launcher, plan and kernels.
#include <cuda_runtime.h>

#include <mutex>

#include "../../../include/starlight_cuda.h"
#include "common.cuh"
#include "kernels.h"

namespace {

constexpr size_t kScratchBytes = SLC_NOALLOC_SCRATCH_BYTES;
constexpr size_t kTicketBytes = 64 * 1024 * sizeof(unsigned);  // first part: split-K tickets
constexpr int kMaxDevices = 64;

// The scratch of every call, on every device that loads the library.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void *g_scratch_addr[kMaxDevices] = {};

int fail(const char **msg, int status, const char *text) {
    if (msg) *msg = text;
    return status;
}

}  // namespace

extern "C" int slc_qmatmul_noalloc(const float *x, uint64_t m, const void *codes,
                                   const float *scales, uint64_t n, uint64_t k,
                                   uint32_t quant_format, uint32_t group_size, float *out,
                                   void *stream, uint32_t *error_word,
                                   const char **error_message) {
    if (error_message) *error_message = nullptr;
    if (quant_format != SLC_QUANT_INT4 && quant_format != SLC_QUANT_INT8)
        return fail(error_message, SLC_ERR_UNIMPLEMENTED, "unknown quantization format");
    if (group_size == 0)
        return fail(error_message, SLC_ERR_EXECUTION, "quantization group size must be nonzero");
    if (m == 0 || n == 0) return SLC_OK;
    if (!x || !codes || !scales || !out)
        return fail(error_message, SLC_ERR_EXECUTION, "null device pointer");
    if (n > (1ull << 30) || k > (1ull << 30) || m > (1ull << 30))
        return fail(error_message, SLC_ERR_SHAPE_OVERFLOW, "matrix dimension above 2^30");

    slc::k::QuantWeight w{};
    w.codes = static_cast<const uint8_t *>(codes);
    w.scales = scales;
    w.n = n;
    w.k = k;
    w.group = group_size;
    w.groups = (k + group_size - 1) / group_size;
    w.row_bytes = quant_format == SLC_QUANT_INT4 ? (k + 1) / 2 : k;
    w.format = (int)quant_format;

    // Split-K scratch of the decode path (rows go 32 at a time). The launcher
    // itself would fall back to a slower GEMV that needs less scratch; this
    // entry point rejects the problem instead, so that a caller never gets
    // that slower path without knowing it. Prefill-sized m (> 64) always
    // fits: the GEMM processes as many rows per pass as the array holds.
    size_t need = 0;
    if (m <= 64) {
        for (uint64_t m0 = 0; m0 < m; m0 += 32) {
            uint64_t mb = m - m0 < 32 ? m - m0 : 32;
            size_t b = slc::k::qmatmul_workspace_bytes(w, mb);
            if (b > need) need = b;
        }
    }
    if (need > kScratchBytes)
        return fail(error_message, SLC_ERR_OUT_OF_MEMORY,
                    "problem needs more split-K scratch than SLC_NOALLOC_SCRATCH_BYTES (8 MiB); "
                    "use slc_dispatch on an slc_device instead");

    // Once per device, with that device current: the device address of the
    // scratch array (the host-side symbol is not a device address).
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fail(error_message, SLC_ERR_EXECUTION, "no usable current CUDA device");
    void *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (!g_scratch_addr[dev]) {
            void *ptr = nullptr;
            if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) {
                cudaGetLastError();
                return fail(error_message, SLC_ERR_EXECUTION,
                            "cudaGetSymbolAddress of the no-allocation scratch failed");
            }
            g_scratch_addr[dev] = ptr;
        }
        scratch = g_scratch_addr[dev];
    }

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The tickets must start at zero; a previous call may have been cut short.
    if (cudaMemsetAsync(scratch, 0, kTicketBytes, s) != cudaSuccess)
        return fail(error_message, SLC_ERR_EXECUTION, "clearing the scratch tickets failed");
    // The caller's stream may have just written the weights: no launch
    // overlap with the previous kernel.
    const bool pdl = slc::k::pdl_enabled();
    slc::k::set_pdl_enabled(false);
    cudaError_t e = slc::k::qmatmul(s, x, m, w, out, scratch, kScratchBytes, error_word);
    slc::k::set_pdl_enabled(pdl);
    if (e != cudaSuccess) return fail(error_message, SLC_ERR_EXECUTION, "CUDA kernel launch failed");
    return SLC_OK;
}
