// Prefill quantized GEMM on the fifth-generation tensor cores (tcgen05):
// out[m, n] = sum_k x[m, k] * w[n, k], w = code * scale[n, k / group], for
// prefill-sized M (a dense contraction). Parity target: dequantize, then
// backend-cpu's f32 matmul_nt (crates/backends/backend-cpu/src/reference/
// matmul.rs:29-59); within the matmul tolerance (summation order and the
// activation split below).
//
// Operands. The MMA kind is f16 with bf16 A and B and f32 accumulation.
//  * A = activations, split once by qgemm_split_kernel into bf16 hi + lo
//    planes (hi = bf16(x), lo = bf16(x - hi): 16 significant bits), each a
//    [M, Kp] row-major tensor read by TMA with the 128-byte swizzle (the
//    canonical K-major SW128 layout). Every output tile is two MMAs per k16
//    step, one per plane, into the same accumulator.
//  * B = codes, read as packed bytes by TMA and expanded by the converter
//    warps into exact bf16 integers in the SW128 layout (INT4: LOP3 under the
//    bf16 exponent of 128 with the sign bit flipped, minus 136; INT8: byte
//    under the f32 exponent of 2^23, minus 2^23 + 128, packed to bf16x2).
//    INT4 yields nibble pairs (i, i + 4), so both operands order the k values
//    of every 8-wide chunk as 0 4 1 5 2 6 3 7 (the split kernel writes A in
//    the same order, INT8 is permuted to match).
//  * Group scales: every quantization group (a multiple of 64 along K) is
//    accumulated in its own TMEM buffer (two buffers of 256 columns, double
//    buffered); the converter warps read a finished buffer (tcgen05.ld) and
//    add scale[n, g] * partial into f32 registers while the MMAs of the next
//    group run.
//
// Tile 128 (M) x 256 (N) x 64 (K), one CTA per SM (TMEM: 512 columns).
// Warp 0: TMA producer of the activation planes. Warp 1: TMEM allocation and
// MMA issue (one thread). Warp 2: TMA producer of the packed codes, running
// ahead of the activation ring on its own ring. Warps 3..18: code
// conversion, scale promotion and the output epilogue; warp w reads TMEM
// lanes 32 (w % 4) .. + 31 and columns 64 ((w - 3) / 4) .. + 63,
// accumulating its 32 rows x 64 columns in registers. Group scales reach a
// warp's lanes by shuffle (no CTA-wide barrier between conversion and
// promotion).
//
// Bound: tensor cores. Algorithmic flops per launch 2 M N K (the hi/lo split
// executes twice that on the tensor pipe).
//
// Every mbarrier wait is bounded (1 s): on timeout the kernel records an
// error for the host, stops issuing work, waits (bounded) for the copies and
// MMAs it issued, frees its TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>

#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "kernels.h"
#include "tensormap.h"
#include "tma.cuh"

namespace slc {
namespace k {
namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kConvWarps = 16;
constexpr int kConv0 = 3;  // first converter warp
constexpr int kThreads = (kConv0 + kConvWarps) * 32;  // 608
constexpr int kABytes = BM * BK * 2;             // 16 KiB per plane
constexpr int kBBytes = BN * BK * 2;             // 32 KiB
constexpr int kSlotBytes = 2 * kABytes + kBBytes;  // 64 KiB
constexpr uint32_t kTmemCols = 512;
// kind::f16, D f32, A bf16, B bf16, both K-major, N = 256, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

template <int FMT>
struct Cfg {
    static constexpr int kStages = FMT == 0 ? 3 : 2;                // bf16 ring
    static constexpr int kPStages = FMT == 0 ? 3 : 4;               // packed-code ring
    static constexpr int kPackedBytes = FMT == 0 ? BN * BK / 2 : BN * BK;  // per stage
    static constexpr int kRing = kStages * kSlotBytes;
    static constexpr int kPacked = kPStages * kPackedBytes;
    static constexpr int kBars = (2 * kStages + 2 * kPStages + 5) * 8 + 16;
    // 1 KiB for aligning the ring to the 1024-byte swizzle atom.
    static constexpr int kSmem = 1024 + kRing + kPacked + kBars;
};
static_assert(Cfg<0>::kSmem <= 227 * 1024, "INT4 shared layout");
static_assert(Cfg<1>::kSmem <= 227 * 1024, "INT8 shared layout");

struct GemmArgs {
    CUtensorMap a_hi, a_lo;  // [M][Kp] bf16, box [64][128], SW128
    CUtensorMap codes;       // [N][row_bytes] u8, box [32 or 64][256]
    const float *scales;     // [N][groups]
    float *out;              // [M][N]
    uint32_t *err;
    int M, N, K, group, groups, nst;
};

// ---- tcgen05 / descriptor helpers ----------------------------------------

// Shared-memory matrix descriptor, K-major with the 128-byte swizzle: start
// address, leading offset 16 B (unused for this layout), stride 1024 B
// between 8-row core groups, descriptor version 1, layout 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

// Arrives on `bar` once every tcgen05 operation this thread issued so far
// has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// 16 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// Bounded wait that ignores the abort word (used to drain work in flight).
__device__ __forceinline__ void drain_wait(uint64_t *bar, uint32_t parity) {
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity) && global_ns() - t0 < 100000000ull) {
    }
}

__device__ __forceinline__ uint32_t lop3_and_xor_b(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;  // (a & b) ^ c
    asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t bsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t prmt_b(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// Eight INT4 codes (low nibble = even k) as bf16 pairs (k, k + 4), k = 0..3.
__device__ __forceinline__ uint4 int4_to_bf16(uint32_t w) {
    const uint32_t magic = 0x43084308u;  // bf16 (136, 136) with the nibble's sign bit flipped
    uint4 r;
    r.x = bsub2(lop3_and_xor_b(w, 0x000F000Fu, magic), magic);
    r.y = bsub2(lop3_and_xor_b(w >> 4, 0x000F000Fu, magic), magic);
    r.z = bsub2(lop3_and_xor_b(w >> 8, 0x000F000Fu, magic), magic);
    r.w = bsub2(lop3_and_xor_b(w >> 12, 0x000F000Fu, magic), magic);
    return r;
}

// Eight INT8 codes (bytes k = 0..7 of lo, hi) as bf16 pairs (k, k + 4).
__device__ __forceinline__ uint32_t int8_pair(uint32_t a, uint32_t b, uint32_t i) {
    // bytes -> f32 2^23 + 128 + code, exact; minus 2^23 + 128.
    const float fa = __uint_as_float(prmt_b(a, 0x4B000000u, 0x7540u + i)) - 8388736.0f;
    const float fb = __uint_as_float(prmt_b(b, 0x4B000000u, 0x7540u + i)) - 8388736.0f;
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(fb), "f"(fa));
    return d;
}

__device__ __forceinline__ uint4 int8_to_bf16(uint2 q) {
    const uint32_t a = q.x ^ 0x80808080u, b = q.y ^ 0x80808080u;
    return make_uint4(int8_pair(a, b, 0), int8_pair(a, b, 1), int8_pair(a, b, 2),
                      int8_pair(a, b, 3));
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

template <int FMT>
__global__ void __launch_bounds__(kThreads, 1) qgemm_tc_kernel(const __grid_constant__ GemmArgs p) {
    using C = Cfg<FMT>;
    constexpr int S = C::kStages;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // Ring at the first 1024-byte boundary (SW128 atoms).
    const uint32_t raw = smem_addr(smem_raw);
    unsigned char *smem = smem_raw + ((1024 - (raw & 1023)) & 1023);
    unsigned char *ring = smem;
    unsigned char *packed = smem + C::kRing;
    uint64_t *bars = reinterpret_cast<uint64_t *>(packed + C::kPacked);
    constexpr int kPStages = C::kPStages;
    uint64_t *full = bars;                // [S]: A bytes + converter warps
    uint64_t *empty = full + S;           // [S]: MMA commit
    uint64_t *pfull = empty + S;          // [P]: packed bytes
    uint64_t *pempty = pfull + kPStages;  // [P]: converter warps
    uint64_t *afull = pempty + kPStages;  // [2]: MMA commit of a group
    uint64_t *aempty = afull + 2;         // [2]: converter warps
    uint64_t *done = aempty + 2;          // [1]: final MMA commit
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    volatile int *abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const int nst = p.nst;
    const int G = p.group;

    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) {
            mbar_init(&full[i], 1 + kConvWarps);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < kPStages; i++) {
            mbar_init(&pfull[i], 1);
            mbar_init(&pempty[i], kConvWarps);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&afull[i], 1);
            mbar_init(&aempty[i], kConvWarps);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        *abort = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- TMA producer of the activation planes.
        if (lane == 0) {
            prefetch_tensormap(&p.a_hi);
            prefetch_tensormap(&p.a_lo);
            pdl_wait();  // activations come from the split kernel
            int issued = 0;
            for (int s = 0; s < nst; s++) {
                const int slot = s % S, ph = (s / S) & 1;
                if (s >= S && !mbar_wait(&empty[slot], ph ^ 1, p.err, abort)) break;
                unsigned char *sl = ring + slot * kSlotBytes;
                mbar_arrive_expect_tx(&full[slot], 2 * kABytes);
                tma_load_2d_nohint(sl, &p.a_hi, s * BK, m0, &full[slot]);
                tma_load_2d_nohint(sl + kABytes, &p.a_lo, s * BK, m0, &full[slot]);
                issued = s + 1;
            }
            // Copies still in flight must land before the CTA's shared memory
            // is released: wait (bounded) for the last stages' barriers.
            for (int s = issued - 1; s >= 0 && s >= issued - S; s--)
                drain_wait(&full[s % S], (s / S) & 1);
        }
    } else if (warp == 2) {
        // ---- TMA producer of the packed codes (weights: no dependency on
        // the previous kernel).
        if (lane == 0) {
            prefetch_tensormap(&p.codes);
            const uint64_t pol_w = policy_evict_first();
            int issued = 0;
            for (int s = 0; s < nst; s++) {
                const int ps = s % kPStages, pph = (s / kPStages) & 1;
                if (s >= kPStages && !mbar_wait(&pempty[ps], pph ^ 1, p.err, abort)) break;
                mbar_arrive_expect_tx(&pfull[ps], C::kPackedBytes);
                tma_load_2d(packed + ps * C::kPackedBytes, &p.codes,
                            FMT == 0 ? s * (BK / 2) : s * BK, n0, &pfull[ps], pol_w);
                issued = s + 1;
            }
            for (int s = issued - 1; s >= 0 && s >= issued - kPStages; s--)
                drain_wait(&pfull[s % kPStages], (s / kPStages) & 1);
        }
    } else if (warp == 1) {
        // ---- MMA issue (one thread).
        if (lane == 0) {
            for (int s = 0; s < nst && !*abort; s++) {
                const int slot = s % S, ph = (s / S) & 1;
                const int kbase = s * BK;
                const int g = kbase / G;
                const bool first = kbase % G == 0;
                const bool last = s == nst - 1 || (kbase + BK) % G == 0;
                const int buf = g & 1;
                if (first && g >= 2 && !mbar_wait(&aempty[buf], ((g >> 1) - 1) & 1, p.err, abort))
                    break;
                if (!mbar_wait(&full[slot], ph, p.err, abort)) break;
                tc_fence_after();
                const uint32_t sa = smem_addr(ring + slot * kSlotBytes);
                const uint32_t d = tmem + (uint32_t)(buf * BN);
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++) {
                    const uint64_t bdesc = sw128_desc(sa + 2 * kABytes + kk * 32);
                    mma_bf16(d, sw128_desc(sa + kk * 32), bdesc, (first && kk == 0) ? 0u : 1u);
                    mma_bf16(d, sw128_desc(sa + kABytes + kk * 32), bdesc, 1u);
                }
                mma_commit(&empty[slot]);
                if (last) mma_commit(&afull[buf]);
            }
            // Every MMA issued must complete before TMEM is freed.
            mma_commit(done);
            drain_wait(done, 0);
        }
    } else {
        // ---- converters / promotion / epilogue (warps 3..18).
        pdl_wait();
        const int cw = warp - kConv0;
        const int tc = cw * 32 + lane;  // 0 .. 511
        const int q = warp & 3;         // TMEM lane quarter
        const int cq = cw >> 2;         // column quarter
        const int cbase = n0 + cq * 64; // this warp's first output column
        float acc[64];
#pragma unroll
        for (int i = 0; i < 64; i++) acc[i] = 0.f;
        // Scales of this warp's columns cbase + lane and cbase + 32 + lane:
        // group `cur` (being accumulated) and the next one (prefetched).
        float cur0 = 0.f, cur1 = 0.f;

        auto promote = [&](int g, float s0, float s1) {
            const int buf = g & 1;
            bool ok = !*abort && mbar_wait(&afull[buf], (g >> 1) & 1, p.err, abort);
            ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld is warp-collective
            if (ok) {
                tc_fence_after();
                const uint32_t ta =
                    tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + cq * 64);
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    float v[16];
                    tmem_ld16(ta + c * 16, v);
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int col = c * 16 + j;  // 0..63: lane col % 32 of s0 / s1
                        const float sj = __shfl_sync(0xffffffffu, col < 32 ? s0 : s1, col & 31);
                        acc[col] = fmaf(v[j], sj, acc[col]);
                    }
                }
                tc_fence_before();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&aempty[buf]);
        };

        for (int s = 0; s < nst; s++) {
            const int kbase = s * BK;
            const int g = kbase / G;
            const bool first = kbase % G == 0;
            float nxt0 = 0.f, nxt1 = 0.f;
            if (first) {
                const int c0 = cbase + lane, c1 = cbase + 32 + lane;
                nxt0 = c0 < p.N ? __ldg(p.scales + (size_t)c0 * p.groups + g) : 0.f;
                nxt1 = c1 < p.N ? __ldg(p.scales + (size_t)c1 * p.groups + g) : 0.f;
            }
            const int slot = s % S, ph = (s / S) & 1;
            const int ps = s % kPStages, pph = (s / kPStages) & 1;
            bool ok = !*abort && mbar_wait(&pfull[ps], pph, p.err, abort);
            if (ok && s >= S) ok = mbar_wait(&empty[slot], ph ^ 1, p.err, abort);
            if (ok) {
                const unsigned char *pk = packed + ps * C::kPackedBytes;
                const uint32_t bb = smem_addr(ring + slot * kSlotBytes + 2 * kABytes);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int item = tc + 512 * j;
                    const int r = item >> 3, c = item & 7;
                    uint4 v;
                    if (FMT == 0)
                        v = int4_to_bf16(*reinterpret_cast<const uint32_t *>(pk + r * 32 + c * 4));
                    else
                        v = int8_to_bf16(*reinterpret_cast<const uint2 *>(pk + r * 64 + c * 8));
                    sts128(bb + r * 128 + ((c ^ (r & 7)) << 4), v);
                }
                fence_proxy_async_smem();
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&full[slot]);
                mbar_arrive(&pempty[ps]);
            }
            if (first) {
                // Promote the previous group while the MMAs of this one run.
                if (g >= 1) promote(g - 1, cur0, cur1);
                cur0 = nxt0;
                cur1 = nxt1;
            }
        }
        promote((nst * BK - 1) / G, cur0, cur1);

        // ---- epilogue: row m0 + 32 q + lane, columns cbase .. cbase + 63.
        const int row = m0 + q * 32 + lane;
        if (row < p.M && !*abort) {
            float *orow = p.out + (size_t)row * p.N;
            if ((p.N & 3) == 0 && cbase + 64 <= p.N) {
#pragma unroll
                for (int i = 0; i < 16; i++)
                    *reinterpret_cast<float4 *>(orow + cbase + 4 * i) =
                        make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
            } else {
#pragma unroll
                for (int i = 0; i < 64; i++)
                    if (cbase + i < p.N) orow[cbase + i] = acc[i];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

// x [rows, K] f32 -> bf16 hi / lo planes [rows, Kp], k of every 8-wide chunk
// in the order 0 4 1 5 2 6 3 7, zero beyond K.
__global__ void qgemm_split_kernel(const float *__restrict__ x, size_t rows, int K, int Kp,
                                   __nv_bfloat16 *__restrict__ hi, __nv_bfloat16 *__restrict__ lo) {
    pdl_trigger();
    pdl_wait();
    const int chunks = Kp / 8;
    const size_t total = rows * (size_t)chunks;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / chunks;
        const int c = (int)(i - r * chunks);
        const float *src = x + r * (size_t)K + c * 8;
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = c * 8 + e < K ? src[e] : 0.f;
        uint32_t h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            // positions 2e, 2e + 1 hold k = e and e + 4
            const float a = v[e], b = v[e + 4];
            const __nv_bfloat16 ah = __float2bfloat16_rn(a), bh = __float2bfloat16_rn(b);
            const float ar = __bfloat162float(ah), br = __bfloat162float(bh);
            const __nv_bfloat16 al = __float2bfloat16_rn(isfinite(ar) ? a - ar : 0.f);
            const __nv_bfloat16 bl = __float2bfloat16_rn(isfinite(br) ? b - br : 0.f);
            h[e] = (uint32_t)__bfloat16_as_ushort(ah) | ((uint32_t)__bfloat16_as_ushort(bh) << 16);
            l[e] = (uint32_t)__bfloat16_as_ushort(al) | ((uint32_t)__bfloat16_as_ushort(bl) << 16);
        }
        *reinterpret_cast<uint4 *>(hi + r * (size_t)Kp + c * 8) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4 *>(lo + r * (size_t)Kp + c * 8) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

struct CodesKey {
    const void *codes;
    size_t n, row_bytes;
    int fmt;
    bool operator==(const CodesKey &o) const {
        return codes == o.codes && n == o.n && row_bytes == o.row_bytes && fmt == o.fmt;
    }
};
struct CodesKeyHash {
    size_t operator()(const CodesKey &k) const {
        return std::hash<const void *>()(k.codes) * 31 + k.n * 7 + k.row_bytes * 3 + k.fmt;
    }
};

bool codes_map(const QuantWeight &w, CUtensorMap *out) {
    static std::mutex mu;
    static std::unordered_map<CodesKey, CUtensorMap, CodesKeyHash> cache;
    const CodesKey key{w.codes, w.n, w.row_bytes, w.format};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return true;
    }
    CUtensorMap m;
    if (!encode_tensor_map(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.codes, w.row_bytes, w.n, w.row_bytes,
                           w.format == 0 ? BK / 2 : BK, BN, false))
        return false;
    if (cache.size() > 8192) cache.clear();
    cache.emplace(key, m);
    *out = m;
    return true;
}

template <int FMT>
cudaError_t launch_gemm(cudaStream_t s, const __nv_bfloat16 *hi, const __nv_bfloat16 *lo,
                        size_t rows, int Kp, const QuantWeight &w, float *out, uint32_t *err) {
    GemmArgs a{};
    if (!encode_tensor_map(&a.a_hi, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, hi, Kp, rows, (size_t)Kp * 2,
                           BK, BM, true) ||
        !encode_tensor_map(&a.a_lo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, lo, Kp, rows, (size_t)Kp * 2,
                           BK, BM, true) ||
        !codes_map(w, &a.codes))
        return cudaErrorInvalidValue;
    a.scales = w.scales;
    a.out = out;
    a.err = err;
    a.M = (int)rows;
    a.N = (int)w.n;
    a.K = (int)w.k;
    a.group = (int)w.group;
    a.groups = (int)w.groups;
    a.nst = (int)((w.k + BK - 1) / BK);
    static std::atomic<uint64_t> smem_set{0};
    set_smem_limit_once(qgemm_tc_kernel<FMT>, Cfg<FMT>::kSmem, &smem_set);
    dim3 grid((unsigned)((rows + BM - 1) / BM), (unsigned)((w.n + BN - 1) / BN));
    launch_k(qgemm_tc_kernel<FMT>, grid, kThreads, Cfg<FMT>::kSmem, s, a);
    count_launch();
    return cudaGetLastError();
}

size_t kpad(size_t k) { return (k + BK - 1) / BK * BK; }

}  // namespace

bool qgemm_tc_supported(const QuantWeight &w) {
    return w.n > 0 && w.k > 0 && w.group % BK == 0 && w.row_bytes % 16 == 0 &&
           aligned16(w.codes) && w.k <= (1u << 24) && w.n <= (1u << 30) &&
           (w.format == 0 ? w.row_bytes == (w.k + 1) / 2 : w.row_bytes == w.k);
}

size_t qgemm_tc_rows_per_pass(const QuantWeight &w, size_t workspace_bytes) {
    const size_t per_row = kpad(w.k) * 4;  // hi + lo bf16
    size_t rows = workspace_bytes / per_row;
    return rows >= BM ? rows / BM * BM : 0;
}

cudaError_t qgemm_tc(cudaStream_t s, const float *x, size_t m, const QuantWeight &w, float *out,
                     void *workspace, size_t workspace_bytes, uint32_t *err) {
    if (m == 0 || w.n == 0) return cudaSuccess;
    const size_t chunk = qgemm_tc_rows_per_pass(w, workspace_bytes);
    if (!qgemm_tc_supported(w) || chunk == 0 || !aligned16(workspace)) return cudaErrorInvalidValue;
    const int Kp = (int)kpad(w.k);
    __nv_bfloat16 *hi = static_cast<__nv_bfloat16 *>(workspace);
    for (size_t r0 = 0; r0 < m; r0 += chunk) {
        const size_t rows = m - r0 < chunk ? m - r0 : chunk;
        __nv_bfloat16 *lo = hi + rows * (size_t)Kp;
        launch_k(qgemm_split_kernel, grid_for(rows * (size_t)(Kp / 8), 256), 256, 0, s,
                 x + r0 * w.k, rows, (int)w.k, Kp, hi, lo);
        count_launch();
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        e = w.format == 0 ? launch_gemm<0>(s, hi, lo, rows, Kp, w, out + r0 * w.n, err)
                          : launch_gemm<1>(s, hi, lo, rows, Kp, w, out + r0 * w.n, err);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace k
}  // namespace slc
