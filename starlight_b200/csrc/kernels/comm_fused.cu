// Tensor-parallel all-reduce fused with the residual Add and the RmsNorm
// that follow it (the llama-dense TP layer: o / down projection partial ->
// AllReduce(sum) -> Add(residual) -> RmsNorm), over NVLink peer memory.
//
// Every rank owns an exchange buffer mapped into all its peers (CUDA IPC,
// set up by comm.cpp): data[parity][source rank][row][hidden] f32 and
// flags[parity][source rank][row] u32. One CTA per row:
//   1. writes its row of the partial into every peer's buffer at
//      [parity][own rank][row] (plain peer stores over NVLink);
//   2. after a block barrier, one thread makes the stores visible at system
//      scope and writes the call's epoch to every peer's flag;
//   3. waits (bounded) until every peer's flag for this row carries the
//      epoch, then adds the partials of ranks 0 .. world - 1 in that order
//      (the same order on every rank, so every rank holds identical sums),
//      writes the sum back to the all-reduced buffer, adds the residual and
//      normalises exactly as rms_norm_regs does.
// The epoch is a per-row counter in the local buffer, advanced by the CTA
// of that row once per call (all ranks make the same calls), so the kernel
// needs no host argument that changes between CUDA-graph replays. Data slots
// alternate by epoch parity: a rank writes a slot again only two calls later,
// after every peer has signalled (and therefore finished reading) the call
// in between.
//
// NVLink and HBM: per row and rank, 4 * hidden bytes to each of world - 1
// peers and about 4 * hidden * (world + 3) bytes of local traffic.
#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace slc {
namespace k {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

template <int NV>
__global__ void __launch_bounds__(256) allreduce_add_rms(PeerReduceArgs a) {
    pdl_trigger();
    pdl_wait();
    __shared__ float partial[8];
    __shared__ uint32_t epoch_s;
    __shared__ int ok_s;
    const int row = blockIdx.x;
    const size_t H = a.hidden, h4 = H / 4;
    uint32_t *ctr = a.counters + row;
    if (threadIdx.x == 0) {
        epoch_s = *ctr + 1;
        ok_s = 1;
    }
    __syncthreads();
    const uint32_t epoch = epoch_s;
    const int par = epoch & 1;
    const size_t slot = a.max_rows * a.max_hidden;  // floats per (parity, source)
    const float *mine = a.partial + (size_t)row * H;
    float4 v[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const size_t c = threadIdx.x + (size_t)i * 256;
        if (c < h4) v[i] = *reinterpret_cast<const float4 *>(mine + 4 * c);
    }
    // 1. this rank's row into every peer's buffer.
    for (int p = 0; p < a.world; p++) {
        if (p == a.rank) continue;
        float *dst = a.peer_data[p] + ((size_t)par * a.world + a.rank) * slot +
                     (size_t)row * a.max_hidden;
#pragma unroll
        for (int i = 0; i < NV; i++) {
            const size_t c = threadIdx.x + (size_t)i * 256;
            if (c < h4) *reinterpret_cast<float4 *>(dst + 4 * c) = v[i];
        }
    }
    __syncthreads();
    // 2. publish: the barrier orders every thread's peer stores before this
    // thread's system-scope fence and release stores.
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int p = 0; p < a.world; p++) {
            if (p == a.rank) continue;
            st_release_sys(a.peer_flags[p] + ((size_t)par * a.world + a.rank) * a.max_rows + row,
                           epoch);
        }
    }
    // 3. wait for every peer's row (one thread per peer), bounded.
    if (threadIdx.x < (unsigned)a.world && threadIdx.x != (unsigned)a.rank) {
        const uint32_t *f =
            a.local_flags + ((size_t)par * a.world + threadIdx.x) * a.max_rows + row;
        const uint64_t t0 = global_ns();
        while (ld_acquire_sys(f) != epoch) {
            if (global_ns() - t0 > 1000000000ull) {
                report_error(a.err, kErrWaitTimeout);
                ok_s = 0;
                break;
            }
        }
    }
    __syncthreads();
    if (!ok_s) {
        if (threadIdx.x == 0) *ctr = epoch;
        return;
    }
    // Sum in rank order.
    float4 s[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) s[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < a.world; p++) {
        const float *src = a.local_data + ((size_t)par * a.world + p) * slot +
                           (size_t)row * a.max_hidden;
#pragma unroll
        for (int i = 0; i < NV; i++) {
            const size_t c = threadIdx.x + (size_t)i * 256;
            if (c < h4) {
                const float4 q =
                    p == a.rank ? v[i] : __ldcg(reinterpret_cast<const float4 *>(src + 4 * c));
                s[i] = make_float4(__fadd_rn(s[i].x, q.x), __fadd_rn(s[i].y, q.y),
                                   __fadd_rn(s[i].z, q.z), __fadd_rn(s[i].w, q.w));
            }
        }
    }
    // Residual and sum of squares; every read of the row's inputs precedes
    // the barrier below, every write follows it.
    float ss = 0.f;
    const float *xr = a.residual + (size_t)row * H;
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const size_t c = threadIdx.x + (size_t)i * 256;
        if (c < h4) {
            const float4 r = *reinterpret_cast<const float4 *>(xr + 4 * c);
            v[i] = make_float4(__fadd_rn(r.x, s[i].x), __fadd_rn(r.y, s[i].y),
                               __fadd_rn(r.z, s[i].z), __fadd_rn(r.w, s[i].w));
            ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
        }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) total += partial[i];
    const float mean = __fdiv_rn(total, (float)H);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const size_t c = threadIdx.x + (size_t)i * 256;
        if (c < h4) {
            *reinterpret_cast<float4 *>(a.partial + (size_t)row * H + 4 * c) = s[i];
            *reinterpret_cast<float4 *>(a.sum_out + (size_t)row * H + 4 * c) = v[i];
            const float4 g = *reinterpret_cast<const float4 *>(a.weight + 4 * c);
            *reinterpret_cast<float4 *>(a.out + (size_t)row * H + 4 * c) = make_float4(
                __fmul_rn(__fmul_rn(v[i].x, inv), g.x), __fmul_rn(__fmul_rn(v[i].y, inv), g.y),
                __fmul_rn(__fmul_rn(v[i].z, inv), g.z), __fmul_rn(__fmul_rn(v[i].w, inv), g.w));
        }
    }
    if (threadIdx.x == 0) *ctr = epoch;
}

}  // namespace

bool allreduce_add_rms_supported(const PeerReduceArgs &a) {
    return a.world >= 2 && a.world <= kMaxPeers && a.rows >= 1 && a.rows <= a.max_rows &&
           a.hidden >= 4 && a.hidden <= a.max_hidden && a.hidden % 4 == 0 &&
           a.hidden / 4 <= 2048 && aligned16(a.partial) && aligned16(a.residual) &&
           aligned16(a.sum_out) && aligned16(a.out) && aligned16(a.weight);
}

cudaError_t allreduce_add_rms(cudaStream_t s, const PeerReduceArgs &a) {
    if (!allreduce_add_rms_supported(a)) return cudaErrorInvalidValue;
    const size_t h4 = a.hidden / 4;
    if (h4 <= 256)
        launch_k(allreduce_add_rms<1>, (unsigned)a.rows, 256, 0, s, a);
    else if (h4 <= 512)
        launch_k(allreduce_add_rms<2>, (unsigned)a.rows, 256, 0, s, a);
    else if (h4 <= 1024)
        launch_k(allreduce_add_rms<4>, (unsigned)a.rows, 256, 0, s, a);
    else
        launch_k(allreduce_add_rms<8>, (unsigned)a.rows, 256, 0, s, a);
    count_launch();
    return cudaGetLastError();
}

}  // namespace k
}  // namespace slc
