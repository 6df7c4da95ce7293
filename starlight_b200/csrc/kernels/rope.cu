// Rotary position embedding, NeoX (split-half) and GPT-J (interleaved)
// layouts (crates/backends/backend-cpu/src/reference/rope.rs:31-141).
// Out of place: reads the input value, writes the output value.
//
// The angle position / theta^(2*pair/head_dim) and its sine and cosine are
// evaluated in f64 once per (batch, token, pair) and rounded to f32, exactly
// the reference's precision split (rope.rs:31-35, :73-76): an f32 angle
// would lose ~1e-3 rad at position 16384 with theta 500000. The f64
// denominators theta^(2*pair/head_dim) (up to 64 pairs) are computed on the
// host with the C library's pow, the same libm function the reference's
// f64::powf calls, and passed as a kernel parameter; the device does the IEEE
// f64 division and sincos. The rotation is two IEEE multiplies and one
// add/sub per output, in the reference's order.
//
// HBM-bound: algorithmic bytes 8 * batch * heads * seq * head_dim + 4 *
// batch * seq. One CTA per (batch, token): its first head_dim/2 threads
// compute the f64 sin/cos into shared memory, then all threads rotate every
// head of that token (contiguous head_dim-wide rows, coalesced).
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace slc {
namespace k {
namespace {

constexpr int kTablePairs = 64;
struct RopeTable {
    double denom[kTablePairs];  // theta^(2 * pair / head_dim), host libm pow
};

__global__ void __launch_bounds__(256) rope_kernel(const float *__restrict__ x,
                                                   const uint32_t *__restrict__ positions,
                                                   float *__restrict__ out, size_t batch,
                                                   size_t heads, size_t seq, size_t head_dim,
                                                   double theta, int gptj, int use_table,
                                                   const __grid_constant__ RopeTable table) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float trig[];  // [half] sin, then [half] cos
    const size_t half = head_dim / 2;
    for (size_t bt = blockIdx.x; bt < batch * seq; bt += gridDim.x) {
        const size_t b = bt / seq, t = bt - b * seq;
        const double position = (double)positions[bt];
        for (size_t p = threadIdx.x; p < half; p += blockDim.x) {
            double denom;
            if (use_table) {
                denom = table.denom[p];
            } else {
                double exponent = 2.0 * (double)p / (double)head_dim;
                denom = pow(theta, exponent);
            }
            double angle = position / denom;
            double sn, cs;
            sincos(angle, &sn, &cs);
            trig[p] = (float)sn;
            trig[half + p] = (float)cs;
        }
        __syncthreads();
        const size_t work = heads * half;
        for (size_t i = threadIdx.x; i < work; i += blockDim.x) {
            const size_t h = i / half, p = i - h * half;
            const size_t base = ((b * heads + h) * seq + t) * head_dim;
            const size_t i0 = gptj ? base + 2 * p : base + p;
            const size_t i1 = gptj ? base + 2 * p + 1 : base + p + half;
            const float first = x[i0], second = x[i1];
            const float sn = trig[p], cs = trig[half + p];
            out[i0] = __fsub_rn(__fmul_rn(first, cs), __fmul_rn(second, sn));
            out[i1] = __fadd_rn(__fmul_rn(first, sn), __fmul_rn(second, cs));
        }
        __syncthreads();
    }
}

}  // namespace

cudaError_t rope(cudaStream_t s, const float *x, const uint32_t *positions, float *out,
                 size_t batch, size_t heads, size_t seq, size_t head_dim, float theta,
                 int gptj) {
    if (batch == 0 || heads == 0 || seq == 0 || head_dim == 0) return cudaSuccess;
    size_t rows = batch * seq;
    int grid = (int)(rows < (size_t)kSmCount * 16 ? rows : (size_t)kSmCount * 16);
    size_t threads = heads * (head_dim / 2);
    int block = threads >= 256 ? 256 : (threads >= 128 ? 128 : (threads >= 64 ? 64 : 32));
    RopeTable table{};
    const size_t half = head_dim / 2;
    const int use_table = half <= (size_t)kTablePairs;
    if (use_table)
        for (size_t p = 0; p < half; p++)
            table.denom[p] = pow((double)theta, 2.0 * (double)p / (double)head_dim);
    launch_k(rope_kernel, grid, block, head_dim * sizeof(float), s, 
        x, positions, out, batch, heads, seq, head_dim, (double)theta, gptj, use_table, table);
    count_launch();
    return cudaGetLastError();
}

}  // namespace k
}  // namespace slc
