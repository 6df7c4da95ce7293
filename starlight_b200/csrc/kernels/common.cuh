// Shared device helpers for the sm_100a kernels of backend-cuda.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <utility>

namespace slc {

// B200: 148 SMs on two dies. Grids of memory-bound kernels are sized as a
// multiple of this so that every SM gets the same number of resident CTAs.
constexpr int kSmCount = 148;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Streaming 128-bit load that bypasses L1 (data read exactly once).
__device__ __forceinline__ float4 ld_stream_f4(const float *p) {
    float4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Streaming 128-bit store (evict-first).
__device__ __forceinline__ void st_stream_f4(float *p, float4 v) {
    asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}

// L2-coherent load (skips L1): data written by other CTAs of the same launch.
__device__ __forceinline__ float ld_cg_f32(const float *p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

__host__ __device__ __forceinline__ bool aligned16(const void *p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Programmatic dependent launch. Every kernel lets the next kernel of its
// stream launch as soon as all of its own CTAs are resident (pdl_trigger),
// and waits for the previous kernel's completion and memory before its first
// access to data another kernel produced (pdl_wait). Without the launch
// attribute both are no-ops.
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

namespace k {
// Whether launches on this thread may overlap their predecessor (on by
// default; entry points that run on a caller's stream turn it off).
bool pdl_enabled();
void set_pdl_enabled(bool on);
}  // namespace k

// Launches `kernel` on `s`, with programmatic stream serialization when
// enabled, so its prologue overlaps the previous kernel's tail.
template <typename... Params, typename... Args>
cudaError_t launch_k(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t s, Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = k::pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Raises `kernel`'s dynamic shared-memory limit to `bytes` on the current
// device, once per device. The attribute belongs to the device's context, so
// `done` keeps one bit per device ordinal (ordinals >= 64 set it every call).
template <typename Kernel>
cudaError_t set_smem_limit_once(Kernel kernel, int bytes, std::atomic<uint64_t> *done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev >= 0 && dev < 64 ? (1ull << dev) : 0;
    if (bit && (done->load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && bit) done->fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

// Host-side helpers.
inline int grid_for(size_t work_items, int per_cta, int ctas_per_sm = 8) {
    size_t g = (work_items + per_cta - 1) / per_cta;
    size_t cap = (size_t)kSmCount * ctas_per_sm;
    if (g > cap) g = cap;
    if (g < 1) g = 1;
    return (int)g;
}

}  // namespace slc
