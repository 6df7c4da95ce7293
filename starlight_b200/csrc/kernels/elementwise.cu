// Elementwise kernels: Add, Mul, Scale, Silu (crates/backends/backend-cpu/src/
// reference/elementwise.rs:20-74) plus the fused SiLU x mul and residual +
// broadcast-bias variants used by the SwiGLU epilogue and the op sweep.
//
// HBM-bound: 128-bit streaming loads/stores when every pointer is 16-byte
// aligned, a grid-stride loop over a grid of 148 x 8 CTAs. Each f32 result
// is one correctly rounded IEEE operation (no contraction), so Add, Mul and
// Scale are bit-exact with the reference; Silu differs only by expf's ulps.
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace slc {
namespace k {

static std::atomic<uint64_t> g_launches{0};
uint64_t launch_count() { return g_launches.load(); }
namespace {
thread_local bool t_pdl = true;
}
bool pdl_enabled() { return t_pdl; }
void set_pdl_enabled(bool on) { t_pdl = on; }
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
void add_launches(int64_t n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

namespace {

enum class Op { Add, Mul, Scale, Silu, SiluMul, Copy };

template <Op OP>
__device__ __forceinline__ float apply(float a, float b, float f) {
    if constexpr (OP == Op::Add) return __fadd_rn(a, b);
    if constexpr (OP == Op::Mul) return __fmul_rn(a, b);
    if constexpr (OP == Op::Scale) return __fmul_rn(a, f);
    if constexpr (OP == Op::Silu) return __fmul_rn(a, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-a))));
    if constexpr (OP == Op::SiluMul)
        return __fmul_rn(__fmul_rn(a, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-a)))), b);
    return a;
}

template <Op OP>
__global__ void __launch_bounds__(256) ew_vec(const float *__restrict__ a,
                                              const float *__restrict__ b, float f,
                                              float *__restrict__ out, size_t n4) {
    pdl_trigger();
    pdl_wait();
    size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 x = ld_stream_f4(a + 4 * i);
        float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
        if constexpr (OP == Op::Add || OP == Op::Mul || OP == Op::SiluMul) y = ld_stream_f4(b + 4 * i);
        float4 r;
        r.x = apply<OP>(x.x, y.x, f);
        r.y = apply<OP>(x.y, y.y, f);
        r.z = apply<OP>(x.z, y.z, f);
        r.w = apply<OP>(x.w, y.w, f);
        st_stream_f4(out + 4 * i, r);
    }
}

template <Op OP>
__global__ void __launch_bounds__(256) ew_scalar(const float *__restrict__ a,
                                                 const float *__restrict__ b, float f,
                                                 float *__restrict__ out, size_t begin,
                                                 size_t n) {
    pdl_trigger();
    pdl_wait();
    size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = begin + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float y = 0.f;
        if constexpr (OP == Op::Add || OP == Op::Mul || OP == Op::SiluMul) y = b[i];
        out[i] = apply<OP>(a[i], y, f);
    }
}

template <Op OP>
cudaError_t launch(cudaStream_t s, const float *a, const float *b, float f, float *out,
                   size_t n) {
    if (n == 0) return cudaSuccess;
    bool vec = ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(out) |
                 (b ? reinterpret_cast<uintptr_t>(b) : 0)) & 15u) == 0;
    size_t n4 = vec ? n / 4 : 0;
    if (n4) {
        launch_k(ew_vec<OP>, grid_for(n4, 256), 256, 0, s, a, b, f, out, n4);
        count_launch();
    }
    if (n4 * 4 < n) {
        launch_k(ew_scalar<OP>, grid_for(n - n4 * 4, 256), 256, 0, s, a, b, f, out, n4 * 4, n);
        count_launch();
    }
    return cudaGetLastError();
}

__global__ void __launch_bounds__(256) add_bias_kernel(const float *__restrict__ a,
                                                       const float *__restrict__ b,
                                                       const float *__restrict__ bias,
                                                       float *__restrict__ out, size_t rows,
                                                       size_t cols, bool vec) {
    pdl_trigger();
    pdl_wait();
    size_t stride = (size_t)gridDim.x * blockDim.x;
    if (vec) {
        size_t c4 = cols / 4, n4 = rows * c4;
        for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
            size_t c = (i % c4) * 4;
            float4 x = ld_stream_f4(a + 4 * i), y = ld_stream_f4(b + 4 * i);
            float4 z = *reinterpret_cast<const float4 *>(bias + c);
            float4 r = make_float4(__fadd_rn(__fadd_rn(x.x, y.x), z.x),
                                   __fadd_rn(__fadd_rn(x.y, y.y), z.y),
                                   __fadd_rn(__fadd_rn(x.z, y.z), z.z),
                                   __fadd_rn(__fadd_rn(x.w, y.w), z.w));
            st_stream_f4(out + 4 * i, r);
        }
    } else {
        size_t n = rows * cols;
        for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
            out[i] = __fadd_rn(__fadd_rn(a[i], b[i]), bias[i % cols]);
    }
}

}  // namespace

cudaError_t add(cudaStream_t s, const float *a, const float *b, float *out, size_t n) {
    return launch<Op::Add>(s, a, b, 0.f, out, n);
}
cudaError_t mul(cudaStream_t s, const float *a, const float *b, float *out, size_t n) {
    return launch<Op::Mul>(s, a, b, 0.f, out, n);
}
cudaError_t scale(cudaStream_t s, const float *x, float factor, float *out, size_t n) {
    return launch<Op::Scale>(s, x, nullptr, factor, out, n);
}
cudaError_t silu(cudaStream_t s, const float *x, float *out, size_t n) {
    return launch<Op::Silu>(s, x, nullptr, 0.f, out, n);
}
cudaError_t silu_mul(cudaStream_t s, const float *a, const float *b, float *out, size_t n) {
    return launch<Op::SiluMul>(s, a, b, 0.f, out, n);
}
cudaError_t copy_f32(cudaStream_t s, const float *src, float *dst, size_t n) {
    return launch<Op::Copy>(s, src, nullptr, 0.f, dst, n);
}

cudaError_t add_bias(cudaStream_t s, const float *a, const float *b, const float *bias,
                     float *out, size_t rows, size_t cols) {
    if (rows == 0 || cols == 0) return cudaSuccess;
    bool vec = (cols % 4 == 0) &&
               ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                 reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
    size_t work = vec ? rows * cols / 4 : rows * cols;
    launch_k(add_bias_kernel, grid_for(work, 256), 256, 0, s, a, b, bias, out, rows, cols, vec);
    count_launch();
    return cudaGetLastError();
}

}  // namespace k
}  // namespace slc
