// Dense f32 MatMulNT / MatMulNN (crates/backends/backend-cpu/src/reference/
// matmul.rs:29-110) with CpuDevice's batch broadcast (device.rs:1301-1407:
// a batch count of 1 on either operand is shared by every output batch).
//
// This is the path for dense (unquantized) f32 weights, which the reference
// fixture uses; the hot path of the quantized models is gemv_quant.cu. A
// shared-memory tiled SIMT GEMM: 64x64 output tile per CTA, k-tile 16, each
// of the 256 threads owns a 4x4 register block and accumulates with FMA in
// ascending k within its tile. f32 accuracy (no TF32).
#include "common.cuh"
#include "kernels.h"

namespace slc {
namespace k {
namespace {

constexpr int BM = 64, BN = 64, BK = 16;

template <bool NT>
__global__ void __launch_bounds__(256) sgemm_kernel(const float *__restrict__ a,
                                                    const float *__restrict__ w,
                                                    float *__restrict__ out, size_t m, size_t k,
                                                    size_t n, size_t a_bstride,
                                                    size_t w_bstride) {
    pdl_trigger();
    pdl_wait();
    __shared__ float As[BK][BM + 4];
    __shared__ float Ws[BK][BN + 4];
    const size_t bz = blockIdx.z;
    const float *ab = a + bz * a_bstride;
    const float *wb = w + bz * w_bstride;
    float *ob = out + bz * m * n;
    const size_t m0 = (size_t)blockIdx.y * BM, n0 = (size_t)blockIdx.x * BN;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    float acc[4][4] = {};
    for (size_t k0 = 0; k0 < k; k0 += BK) {
        for (int i = threadIdx.x; i < BM * BK; i += 256) {
            int mm = i / BK, kk = i % BK;
            size_t gm = m0 + mm, gk = k0 + kk;
            As[kk][mm] = (gm < m && gk < k) ? ab[gm * k + gk] : 0.f;
        }
        for (int i = threadIdx.x; i < BN * BK; i += 256) {
            if (NT) {
                int nn = i / BK, kk = i % BK;
                size_t gn = n0 + nn, gk = k0 + kk;
                Ws[kk][nn] = (gn < n && gk < k) ? wb[gn * k + gk] : 0.f;
            } else {
                int kk = i / BN, nn = i % BN;
                size_t gn = n0 + nn, gk = k0 + kk;
                Ws[kk][nn] = (gn < n && gk < k) ? wb[gk * n + gn] : 0.f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float av[4], wv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) av[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; j++) wv[j] = Ws[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        size_t gm = m0 + ty * 4 + i;
        if (gm >= m) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            size_t gn = n0 + tx * 4 + j;
            if (gn < n) ob[gm * n + gn] = acc[i][j];
        }
    }
}

// Quantized NT GEMM for prefill-sized M: the same tiling, with the weight
// tile dequantized ((float)code * scale, exact) while it is staged.
template <int FMT>
__global__ void __launch_bounds__(256) qgemm_kernel(const float *__restrict__ a,
                                                   const uint8_t *__restrict__ codes,
                                                   const float *__restrict__ scales,
                                                   float *__restrict__ out, size_t m, size_t k,
                                                   size_t n, size_t row_bytes, size_t group,
                                                   size_t groups) {
    pdl_trigger();
    pdl_wait();
    __shared__ float As[BK][BM + 4];
    __shared__ float Ws[BK][BN + 4];
    const size_t m0 = (size_t)blockIdx.y * BM, n0 = (size_t)blockIdx.x * BN;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    float acc[4][4] = {};
    for (size_t k0 = 0; k0 < k; k0 += BK) {
        for (int i = threadIdx.x; i < BM * BK; i += 256) {
            int mm = i / BK, kk = i % BK;
            size_t gm = m0 + mm, gk = k0 + kk;
            As[kk][mm] = (gm < m && gk < k) ? a[gm * k + gk] : 0.f;
        }
        for (int i = threadIdx.x; i < BN * BK; i += 256) {
            int nn = i / BK, kk = i % BK;
            size_t gn = n0 + nn, gk = k0 + kk;
            float w = 0.f;
            if (gn < n && gk < k) {
                int code;
                if (FMT == 0) {
                    uint8_t b = codes[gn * row_bytes + gk / 2];
                    int nib = (gk & 1) ? (b >> 4) : (b & 15);
                    code = nib >= 8 ? nib - 16 : nib;
                } else {
                    code = (int)(int8_t)codes[gn * row_bytes + gk];
                }
                w = __fmul_rn((float)code, scales[gn * groups + gk / group]);
            }
            Ws[kk][nn] = w;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float av[4], wv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) av[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; j++) wv[j] = Ws[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        size_t gm = m0 + ty * 4 + i;
        if (gm >= m) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            size_t gn = n0 + tx * 4 + j;
            if (gn < n) out[gm * n + gn] = acc[i][j];
        }
    }
}

}  // namespace

cudaError_t qgemm_f32(cudaStream_t s, const float *a, size_t m, const QuantWeight &w, float *out) {
    if (m == 0 || w.n == 0) return cudaSuccess;
    dim3 grid((unsigned)((w.n + BN - 1) / BN), (unsigned)((m + BM - 1) / BM));
    if (w.format == 0)
        launch_k(qgemm_kernel<0>, grid, 256, 0, s, a, w.codes, w.scales, out, m, w.k, w.n, w.row_bytes,
                                             w.group, w.groups);
    else
        launch_k(qgemm_kernel<1>, grid, 256, 0, s, a, w.codes, w.scales, out, m, w.k, w.n, w.row_bytes,
                                             w.group, w.groups);
    count_launch();
    return cudaGetLastError();
}

cudaError_t matmul_f32(cudaStream_t s, const float *a, const float *w, float *out,
                       size_t batch_a, size_t batch_b, size_t m, size_t k, size_t n,
                       bool transposed) {
    size_t batch = batch_a > batch_b ? batch_a : batch_b;
    if (batch_a == 0 || batch_b == 0) batch = 0;
    if (batch == 0 || m == 0 || n == 0) return cudaSuccess;
    size_t a_bs = batch_a == 1 ? 0 : m * k;
    size_t w_bs = batch_b == 1 ? 0 : n * k;
    // Fold a broadcast weight into the row dimension: [batch, m, k] x [n, k]
    // is one [batch * m, k] x [n, k] product with a contiguous output.
    if (batch_b == 1 && batch_a == batch) {
        m *= batch;
        batch = 1;
        a_bs = 0;
    }
    dim3 grid((unsigned)((n + BN - 1) / BN), (unsigned)((m + BM - 1) / BM), (unsigned)batch);
    if (transposed)
        launch_k(sgemm_kernel<true>, grid, 256, 0, s, a, w, out, m, k, n, a_bs, w_bs);
    else
        launch_k(sgemm_kernel<false>, grid, 256, 0, s, a, w, out, m, k, n, a_bs, w_bs);
    count_launch();
    return cudaGetLastError();
}

}  // namespace k
}  // namespace slc
