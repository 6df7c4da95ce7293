// Synthetic weight generation on the device (bench and large-model tests):
// element i of a stream is a deterministic function of (seed, offset + i).
// A splitmix64 hash of the element index gives two 32-bit uniforms; a
// Box-Muller transform in f64 gives one N(mean, std) draw rounded to f32.
// Large models (the 8B/70B configurations hold 30-275 GB of f32 weights)
// cannot be generated on the host, so their parity is checked on rows
// reproduced on the host with the same function (tests/gpu_util.py).
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace slc {
namespace k {
namespace {

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

__global__ void __launch_bounds__(256) fill_normal_kernel(float *__restrict__ out, size_t n,
                                                          uint64_t seed, uint64_t offset,
                                                          float mean, float std) {
    pdl_trigger();
    pdl_wait();
    size_t stride = (size_t)gridDim.x * blockDim.x;
    const uint64_t key = splitmix64(seed);
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        uint64_t h = splitmix64(key ^ (offset + i));
        double u1 = ((double)(uint32_t)(h >> 32) + 1.0) * (1.0 / 4294967296.0);
        double u2 = (double)(uint32_t)h * (1.0 / 4294967296.0);
        double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
        out[i] = (float)((double)mean + (double)std * z);
    }
}

}  // namespace

cudaError_t fill_normal(cudaStream_t s, float *out, size_t n, uint64_t seed, uint64_t offset,
                        float mean, float std) {
    if (n == 0) return cudaSuccess;
    launch_k(fill_normal_kernel, grid_for(n, 256), 256, 0, s, out, n, seed, offset, mean, std);
    count_launch();
    return cudaGetLastError();
}

}  // namespace k
}  // namespace slc
