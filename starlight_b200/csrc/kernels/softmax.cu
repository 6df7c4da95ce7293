// Row softmax and causal softmax (crates/backends/backend-cpu/src/reference/
// softmax.rs:19-114). Out of place: the device contract forbids in-place
// writes, so the kernels read the input value and write the output value
// (CpuDevice copies then runs in place, device.rs:803-826).
//
// HBM-bound: algorithmic bytes 8 * rows * cols. One warp per row; rows up to
// 2048 columns are held in registers (one HBM read, one write); wider rows
// take three passes, the later two served from L1/L2. Per element the result
// is expf(x - max) * (1 / sum) with IEEE multiply and divide, as in the
// reference; only the summation order of the denominator differs.
#include "common.cuh"
#include "kernels.h"

namespace slc {
namespace k {
namespace {

template <int NV>
__global__ void __launch_bounds__(256) softmax_regs(const float *__restrict__ x,
                                                    float *__restrict__ out, size_t rows,
                                                    size_t cols, size_t seq, size_t past,
                                                    bool causal) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const size_t c4 = cols / 4;
    size_t warps = (size_t)gridDim.x * 8;
    for (size_t row = (size_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += warps) {
        const size_t visible = causal ? past + row % seq + 1 : cols;
        const float *xr = x + row * cols;
        float4 v[NV];
        float m = -INFINITY;
#pragma unroll
        for (int i = 0; i < NV; i++) {
            size_t c = lane + (size_t)i * 32;
            if (c < c4) {
                v[i] = ld_stream_f4(xr + 4 * c);
                size_t e = 4 * c;
                if (e < visible) m = fmaxf(m, v[i].x);
                if (e + 1 < visible) m = fmaxf(m, v[i].y);
                if (e + 2 < visible) m = fmaxf(m, v[i].z);
                if (e + 3 < visible) m = fmaxf(m, v[i].w);
            }
        }
        m = warp_max(m);
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < NV; i++) {
            size_t c = lane + (size_t)i * 32;
            if (c < c4) {
                size_t e = 4 * c;
                v[i].x = e < visible ? expf(__fsub_rn(v[i].x, m)) : 0.f;
                v[i].y = e + 1 < visible ? expf(__fsub_rn(v[i].y, m)) : 0.f;
                v[i].z = e + 2 < visible ? expf(__fsub_rn(v[i].z, m)) : 0.f;
                v[i].w = e + 3 < visible ? expf(__fsub_rn(v[i].w, m)) : 0.f;
                sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
            }
        }
        sum = warp_sum(sum);
        float inv = __fdiv_rn(1.0f, sum);
        float *orow = out + row * cols;
#pragma unroll
        for (int i = 0; i < NV; i++) {
            size_t c = lane + (size_t)i * 32;
            if (c < c4) {
                float4 r = make_float4(__fmul_rn(v[i].x, inv), __fmul_rn(v[i].y, inv),
                                       __fmul_rn(v[i].z, inv), __fmul_rn(v[i].w, inv));
                st_stream_f4(orow + 4 * c, r);
            }
        }
    }
}

__global__ void __launch_bounds__(256) softmax_generic(const float *__restrict__ x,
                                                       float *__restrict__ out, size_t rows,
                                                       size_t cols, size_t seq, size_t past,
                                                       bool causal) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    size_t warps = (size_t)gridDim.x * 8;
    for (size_t row = (size_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += warps) {
        const size_t visible = causal ? past + row % seq + 1 : cols;
        const float *xr = x + row * cols;
        float m = -INFINITY;
        for (size_t c = lane; c < visible; c += 32) m = fmaxf(m, xr[c]);
        m = warp_max(m);
        float sum = 0.f;
        for (size_t c = lane; c < visible; c += 32) sum += expf(__fsub_rn(xr[c], m));
        float inv = __fdiv_rn(1.0f, warp_sum(sum));
        float *orow = out + row * cols;
        for (size_t c = lane; c < cols; c += 32)
            orow[c] = c < visible ? __fmul_rn(expf(__fsub_rn(xr[c], m)), inv) : 0.f;
    }
}

cudaError_t launch(cudaStream_t s, const float *x, float *out, size_t rows, size_t cols,
                   size_t seq, size_t past, bool causal) {
    if (rows == 0 || cols == 0) return cudaSuccess;
    int grid = grid_for(rows, 8, 16);
    bool vec = cols % 4 == 0 && aligned16(x) && aligned16(out);
    size_t per_lane = (cols / 4 + 31) / 32;
    if (vec && per_lane <= 1)
        launch_k(softmax_regs<1>, grid, 256, 0, s, x, out, rows, cols, seq, past, causal);
    else if (vec && per_lane <= 2)
        launch_k(softmax_regs<2>, grid, 256, 0, s, x, out, rows, cols, seq, past, causal);
    else if (vec && per_lane <= 4)
        launch_k(softmax_regs<4>, grid, 256, 0, s, x, out, rows, cols, seq, past, causal);
    else if (vec && per_lane <= 8)
        launch_k(softmax_regs<8>, grid, 256, 0, s, x, out, rows, cols, seq, past, causal);
    else if (vec && per_lane <= 16)
        launch_k(softmax_regs<16>, grid, 256, 0, s, x, out, rows, cols, seq, past, causal);
    else
        launch_k(softmax_generic, grid, 256, 0, s, x, out, rows, cols, seq, past, causal);
    count_launch();
    return cudaGetLastError();
}

}  // namespace

cudaError_t softmax(cudaStream_t s, const float *x, float *out, size_t rows, size_t cols) {
    return launch(s, x, out, rows, cols, 1, 0, false);
}

cudaError_t softmax_causal(cudaStream_t s, const float *x, float *out, size_t rows, size_t cols,
                           size_t seq, size_t past_len) {
    return launch(s, x, out, rows, cols, seq, past_len, true);
}

}  // namespace k
}  // namespace slc
