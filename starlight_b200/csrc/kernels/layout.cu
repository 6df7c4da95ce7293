// Data-movement kernels (crates/backends/backend-cpu/src/reference/layout.rs):
// Gather (:25-52), LastToken (:71-95), SplitHeads (:107-128) and MergeHeads
// (:144-168). All are exact copies; the index maps are the reference's.
//
// HBM-bound: each copies its output size once (8 bytes per element moved).
// Rows of `width` floats are copied with 128-bit accesses when the width is
// a multiple of 4 and the pointers are 16-byte aligned.
#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace slc {
namespace k {
namespace {

// Generic row copy: dst row r <- src row map(r). `mode` selects the map.
enum Map { kGather = 0, kLastToken = 1, kSplit = 2, kMerge = 3 };

struct RowMap {
    int mode;
    const uint32_t *ids;
    size_t vocab, batch, seq, heads, seq_len;
    uint32_t *error_flag;
    const uint32_t *d_seq_len;  // LastToken: device copy of seq_len, or null
};

__device__ __forceinline__ bool source_row(const RowMap &m, size_t r, size_t *src) {
    switch (m.mode) {
    case kGather: {
        uint32_t id = m.ids[r];
        if ((size_t)id >= m.vocab) {  // host validated already; guard anyway
            report_error(m.error_flag, kErrGatherId);
            return false;
        }
        *src = id;
        return true;
    }
    case kLastToken: {  // out row b <- input row (b, seq_len - 1)
        const size_t seq_len = m.d_seq_len ? (size_t)*m.d_seq_len : m.seq_len;
        if (seq_len < 1 || seq_len > m.seq) {  // validated on the host; guard anyway
            report_error(m.error_flag, kErrBadScalar);
            return false;
        }
        *src = r * m.seq + (seq_len - 1);
        return true;
    }
    case kSplit: {  // out row (b, h, t) <- input row (b, t, h)
        size_t t = r % m.seq, bh = r / m.seq, h = bh % m.heads, b = bh / m.heads;
        *src = (b * m.seq + t) * m.heads + h;
        return true;
    }
    default: {  // kMerge: out row (b, t, h) <- input row (b, h, t)
        size_t h = r % m.heads, bt = r / m.heads, t = bt % m.seq, b = bt / m.seq;
        *src = (b * m.heads + h) * m.seq + t;
        return true;
    }
    }
}

__global__ void __launch_bounds__(256) copy_rows_vec(const float *__restrict__ src,
                                                     float *__restrict__ dst, size_t rows,
                                                     size_t width, RowMap m) {
    pdl_trigger();
    pdl_wait();
    const size_t w4 = width / 4, total = rows * w4;
    size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        size_t r = i / w4, c = i - r * w4, sr;
        if (!source_row(m, r, &sr)) continue;
        float4 v = ld_stream_f4(src + sr * width + 4 * c);
        st_stream_f4(dst + r * width + 4 * c, v);
    }
}

__global__ void __launch_bounds__(256) copy_rows(const float *__restrict__ src,
                                                 float *__restrict__ dst, size_t rows,
                                                 size_t width, RowMap m) {
    pdl_trigger();
    pdl_wait();
    const size_t total = rows * width;
    size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        size_t r = i / width, c = i - r * width, sr;
        if (!source_row(m, r, &sr)) continue;
        dst[i] = src[sr * width + c];
    }
}

cudaError_t launch(cudaStream_t s, const float *src, float *dst, size_t rows, size_t width,
                   const RowMap &m) {
    if (rows == 0 || width == 0) return cudaSuccess;
    if (width % 4 == 0 && aligned16(src) && aligned16(dst))
        launch_k(copy_rows_vec, grid_for(rows * width / 4, 256), 256, 0, s, src, dst, rows, width, m);
    else
        launch_k(copy_rows, grid_for(rows * width, 256), 256, 0, s, src, dst, rows, width, m);
    count_launch();
    return cudaGetLastError();
}

}  // namespace

cudaError_t gather(cudaStream_t s, const float *table, const uint32_t *ids, float *out,
                   size_t vocab, size_t hidden, size_t rows, uint32_t *error_flag) {
    RowMap m{kGather, ids, vocab, 0, 0, 0, 0, error_flag, nullptr};
    return launch(s, table, out, rows, hidden, m);
}

cudaError_t last_token(cudaStream_t s, const float *x, float *out, size_t batch, size_t seq,
                       size_t hidden, size_t seq_len, const uint32_t *d_seq_len, uint32_t *err) {
    RowMap m{kLastToken, nullptr, 0, batch, seq, 0, seq_len, err, d_seq_len};
    return launch(s, x, out, batch, hidden, m);
}

cudaError_t split_heads(cudaStream_t s, const float *x, float *out, size_t batch, size_t seq,
                        size_t heads, size_t head_dim) {
    RowMap m{kSplit, nullptr, 0, batch, seq, heads, 0, nullptr, nullptr};
    return launch(s, x, out, batch * seq * heads, head_dim, m);
}

cudaError_t merge_heads(cudaStream_t s, const float *x, float *out, size_t batch, size_t seq,
                        size_t heads, size_t head_dim) {
    RowMap m{kMerge, nullptr, 0, batch, seq, heads, 0, nullptr, nullptr};
    return launch(s, x, out, batch * seq * heads, head_dim, m);
}

namespace {
__global__ void __launch_bounds__(256) interleave_kernel(const float *__restrict__ src,
                                                         float *__restrict__ dst, size_t blocks,
                                                         size_t rows, size_t cols) {
    pdl_trigger();
    pdl_wait();
    size_t total = blocks * rows * cols, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        size_t c = i % cols, br = i / cols, r = br % rows, b = br / rows;
        dst[(r * blocks + b) * cols + c] = src[i];
    }
}
}  // namespace

cudaError_t interleave_blocks(cudaStream_t s, const float *src, float *dst, size_t blocks,
                              size_t rows, size_t cols) {
    size_t total = blocks * rows * cols;
    if (total == 0) return cudaSuccess;
    launch_k(interleave_kernel, grid_for(total, 256), 256, 0, s, src, dst, blocks, rows, cols);
    count_launch();
    return cudaGetLastError();
}

}  // namespace k
}  // namespace slc
