// Decode GEMV for one or two activation rows (M <= 2): out[m, n] =
// sum_k x[m, k] * code[n, k] * scale[n, k / group], INT4 / INT8 codes.
//
// Parity target: dequantize, then backend-cpu's f32 matmul_nt
// (crates/backends/backend-cpu/src/reference/matmul.rs:29-59).
//
// HBM-bound on the payload; algorithmic bytes per launch
//   N * row_bytes + 4 * N * K / group + 4 * M * (K + N).
//
// Built for the fixed cost of a decode launch rather than for the streaming
// rate alone (which the grouped qgemv_imma reaches on large matrices):
//
//  * Work split without cross-CTA sums: the rows (over all matrices of the
//    launch) are cut into 16-row tiles and every CTA owns a contiguous range
//    of whole tiles (balanced to one tile). No partial-sum workspace, no
//    tickets, no tail.
//  * Inside a CTA, consumer warp w owns the contiguous warp-steps (64 bytes
//    of every row: 128 INT4 or 64 INT8 codes) [w R, (w + 1) R) of every
//    tile, R = ceil(warp-steps per row / 16), so each warp reads runs of
//    64 R bytes of every row. It stages
//    the activation digits of exactly those warp-steps itself, in its own
//    shared region, so no CTA-wide barrier precedes the math.
//  * Codes: each lane copies the 16-byte pieces of rows g and g + 8 it will
//    multiply (cp.async, L1 bypassed) into its warp's ring of kDepth items,
//    and reads back only what it copied itself. The first items are issued
//    before the programmatic-dependency wait, so weights stream while the
//    previous kernel finishes.
//  * Scales: one TMA box per tile ([16 rows][groups] f32) into a small ring
//    filled by a producer warp.
//  * Math: the exact s8 tensor-core path of qgemv_imma (INT4 nibbles as
//    16 x code, activations as three 7-bit digits in the MMA's N dimension,
//    integer sums converted exactly, scaled by scale * 2^e * 2^-7d).
//  * Every 4 tiles the 16 warps' row sums meet in shared memory and are
//    added in warp order (deterministic).
//
// All waits are bounded (1 s); on timeout the kernel records an error for
// the host and skips the remaining math.
#include <math.h>

#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "gemv_common.cuh"
#include "kernels.h"
#include "tensormap.h"
#include "tma.cuh"

namespace slc {
namespace k {
namespace {

constexpr int kWarps = 16;                 // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;  // + scale producer warp
constexpr int kDepth = 6;                  // code items in flight per warp
constexpr int kItemBytes = 16 * 64;        // one warp-step of one tile
constexpr int kScaleSlots = 4;
constexpr int kBatch = 4;                  // tiles per reduction
constexpr int kMaxSeg = 4;
constexpr int kSmemLimit = 227 * 1024;

struct LaneArgs {
    CUtensorMap scales_map[kMaxSeg];  // [N][groups] f32, box [groups][16]
    const uint8_t *codes[kMaxSeg];
    float *out[kMaxSeg];
    int N[kMaxSeg];
    int tile_end[kMaxSeg];  // cumulative 16-row tile counts
    int nseg;
    const float *x, *x2;    // x2: SwiGLU up input (staged value silu(x) * x2)
    uint32_t *err;
    long long row_bytes;
    int M, K, spr, groups, gs_shift, tiles;
    int wmax;               // warp-steps per warp (R): ceil(spr / 16)
    int scale_slot_bytes;
    int dig_off, fx_off, ring_off, red_off, bar_off;
};

template <int FMT>
struct Lane;
template <>
struct Lane<0> {
    static constexpr int kKStep = 128;  // k per warp-step
    static constexpr int kWsBytes = 128;  // digit bytes per column per warp-step
    static constexpr int kJ = 4;          // k32 MMAs per warp-step
};
template <>
struct Lane<1> {
    static constexpr int kKStep = 64;
    static constexpr int kWsBytes = 64;
    static constexpr int kJ = 2;
};

// Byte of activation k (within its warp-step) in the [j][t][8 bytes] cell
// layout of the B fragments (bytes 0..3 = b0, 4..7 = b1 of MMA j, lane
// quad t). INT4: quad t holds codes 32t .. 32t + 31, MMA j pairs the even
// nibbles of word j (k = 32t + 8j + 2i) in b0 with the odd ones in b1.
// INT8: quad t holds codes 16t .. 16t + 15; MMA j takes words 2j, 2j + 1.
template <int FMT>
__device__ __forceinline__ int lane_byte(int kl) {
    if (FMT == 0) {
        const int t = kl >> 5, j = (kl >> 3) & 3, i = (kl >> 1) & 3, odd = kl & 1;
        return j * 32 + t * 8 + odd * 4 + i;
    }
    const int t = kl >> 4, j = (kl >> 3) & 1, h = (kl >> 2) & 1, i = kl & 3;
    return j * 32 + t * 8 + h * 4 + i;
}

__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                       uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint2 lds64u(const void *p) {
    uint2 r;
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(a));
    return r;
}

// Exact int -> float for |c| < 2^22.
__device__ __forceinline__ float i2f_small(int c) {
    return __int_as_float(c + 0x4B400000) - 12582912.0f;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(kWarps * 32) : "memory");
}

// Matrix of a (global) tile and the tile's row inside that matrix.
__device__ __forceinline__ int tile_segment(const LaneArgs &p, int tile, int *row) {
    int s = 0;
    while (s + 1 < p.nseg && tile >= p.tile_end[s]) s++;
    *row = (tile - (s ? p.tile_end[s - 1] : 0)) * 16;
    return s;
}

template <int FMT>
__global__ void __launch_bounds__(kThreads, 1) qgemv_lane(const __grid_constant__ LaneArgs p) {
    constexpr int WSB = Lane<FMT>::kWsBytes;
    constexpr int J = Lane<FMT>::kJ;
    constexpr int KSTEP = Lane<FMT>::kKStep;
    constexpr int PER = KSTEP / 32;  // activation values per lane per warp-step
    extern __shared__ __align__(1024) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + p.bar_off);
    uint64_t *empty = full + kScaleSlots;
    volatile int *abort = reinterpret_cast<volatile int *>(empty + kScaleSlots);

    const int G = gridDim.x, c = blockIdx.x;
    const int t0 = (int)((long long)c * p.tiles / G), t1 = (int)((long long)(c + 1) * p.tiles / G);
    const int nt = t1 - t0;

    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int i = 0; i < kScaleSlots; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kWarps);
        }
        fence_mbar_init();
        *abort = 0;
    }
    __syncthreads();

    if (warp == kWarps) {
        // ---- scale producer: one box per tile.
        if (lane == 0) {
            for (int i = 0; i < p.nseg; i++) prefetch_tensormap(&p.scales_map[i]);
            const uint64_t pol = policy_evict_first();
            int issued = 0;
            for (int lt = 0; lt < nt; lt++) {
                const int slot = lt % kScaleSlots, ph = (lt / kScaleSlots) & 1;
                if (lt >= kScaleSlots && !mbar_wait(&empty[slot], ph ^ 1, p.err, abort)) break;
                int row;
                const int sg = tile_segment(p, t0 + lt, &row);
                mbar_arrive_expect_tx(&full[slot], (uint32_t)(16 * p.groups * 4));
                tma_load_2d(smem + slot * p.scale_slot_bytes, &p.scales_map[sg], 0, row, &full[slot],
                            pol);
                issued = lt + 1;
            }
            // Boxes still in flight land before the CTA exits (bounded).
            for (int lt = issued - 1; lt >= 0 && lt >= issued - kScaleSlots; lt--) {
                const uint64_t st = global_ns();
                while (!mbar_try_wait(&full[lt % kScaleSlots], (lt / kScaleSlots) & 1) &&
                       global_ns() - st < 100000000ull) {
                }
            }
        }
        return;
    }

    // ---- consumers. Warp w owns warp-steps ws0 .. ws0 + nw - 1.
    const int ws0 = warp * p.wmax;
    const int nw = max(0, min(p.wmax, p.spr - ws0));
    const int n_items = nt * nw;
    unsigned char *ring = smem + p.ring_off + warp * (kDepth * kItemBytes);
    const uint32_t ring_s = smem_addr(ring);
    auto issue = [&](int it) {
        if (it < n_items) {
            const int lt = it / nw, q = it - lt * nw;
            int row;
            const int sg = tile_segment(p, t0 + lt, &row);
            const uint8_t *src = p.codes[sg] + (long long)(row + g) * p.row_bytes +
                                 (long long)(ws0 + q) * 64 + t * 16;
            const uint32_t dst = ring_s + (it % kDepth) * kItemBytes + g * 64 + t * 16;
            cp_async16(dst, src);
            cp_async16(dst + 8 * 64, src + 8 * p.row_bytes);
        }
        cp_commit();  // one group per item (empty past the end)
    };
    // Weights do not depend on the previous kernel: start streaming now.
#pragma unroll
    for (int i = 0; i < kDepth - 1; i++) issue(i);

    pdl_wait();
    // ---- this warp's activation digits and factors. The loads of up to
    // kStageBatch warp-steps are issued before any conversion, so staging
    // costs about one load latency per batch.
    int8_t *dig = reinterpret_cast<int8_t *>(smem + p.dig_off) + warp * (p.wmax * 3 * p.M * WSB);
    float *fxw = reinterpret_cast<float *>(smem + p.fx_off) + warp * (p.wmax * 8);
    const int ncol = 3 * p.M;
    constexpr int kStageBatch = 8;
    for (int m = 0; m < p.M; m++) {
        for (int q0 = 0; q0 < nw; q0 += kStageBatch) {
            float v[kStageBatch][PER], u[kStageBatch][PER];
#pragma unroll
            for (int qq = 0; qq < kStageBatch; qq++) {
                const int q = q0 + qq;
                if (q >= nw) break;
                const long long off = (long long)m * p.K + (ws0 + q) * KSTEP + lane * PER;
                if constexpr (PER == 4) {
                    const float4 a = __ldg(reinterpret_cast<const float4 *>(p.x + off));
                    v[qq][0] = a.x, v[qq][1] = a.y, v[qq][2] = a.z, v[qq][3] = a.w;
                    if (p.x2) {
                        const float4 b = __ldg(reinterpret_cast<const float4 *>(p.x2 + off));
                        u[qq][0] = b.x, u[qq][1] = b.y, u[qq][2] = b.z, u[qq][3] = b.w;
                    }
                } else {
                    const float2 a = __ldg(reinterpret_cast<const float2 *>(p.x + off));
                    v[qq][0] = a.x, v[qq][1] = a.y;
                    if (p.x2) {
                        const float2 b = __ldg(reinterpret_cast<const float2 *>(p.x2 + off));
                        u[qq][0] = b.x, u[qq][1] = b.y;
                    }
                }
            }
#pragma unroll
            for (int qq = 0; qq < kStageBatch; qq++) {
                const int q = q0 + qq;
                if (q >= nw) break;
                if (p.x2) {
                    // SwiGLU: silu(gate) * up, the elementwise silu_mul expression.
#pragma unroll
                    for (int i = 0; i < PER; i++)
                        v[qq][i] = __fmul_rn(
                            __fmul_rn(v[qq][i], __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v[qq][i])))),
                            u[qq][i]);
                }
                float mx = 0.f;
                bool bad = false;
#pragma unroll
                for (int i = 0; i < PER; i++) {
                    const float a = fabsf(v[qq][i]);
                    bad |= !(a <= 3.402823466e38f);
                    mx = fmaxf(mx, a);
                }
                mx = warp_max(mx);
                bad = __any_sync(0xffffffffu, bad);
                int e = 0;
                if (mx > 0.f && !bad) {
                    int ex;
                    frexpf(mx, &ex);
                    e = ex - 6;  // |x / 2^e| < 64
                }
                // Digits: y = x / 2^e exactly (power-of-two multiply; ldexpf
                // outside the normal exponent range), then
                // d = rint(y), y' = (y - d) * 128 = fma(d, -128, 128 y), exact.
                float sc;
                const bool direct = e >= -126 && e <= 126;
                sc = __int_as_float((127 - e) << 23);
                uint32_t db[3][PER];  // digit + 1.5 * 2^23, low byte = two's complement
#pragma unroll
                for (int i = 0; i < PER; i++) {
                    float y = 0.f;
                    if (!bad) y = direct ? v[qq][i] * sc : ldexpf(v[qq][i], -e);
                    const float d0 = rintf(y);
                    const float r1 = fmaf(d0, -128.f, y * 128.f);
                    const float d1 = rintf(r1);
                    const float r2 = fmaf(d1, -128.f, r1 * 128.f);
                    const float d2 = rintf(r2);
                    db[0][i] = __float_as_uint(d0 + 12582912.0f);
                    db[1][i] = __float_as_uint(d1 + 12582912.0f);
                    db[2][i] = __float_as_uint(d2 + 12582912.0f);
                }
                unsigned char *d0p =
                    reinterpret_cast<unsigned char *>(dig + ((q * ncol) + 3 * m) * WSB);
#pragma unroll
                for (int dd = 0; dd < 3; dd++) {
                    if (FMT == 0) {
                        // Values i = 0, 2 -> bytes B, B + 1; i = 1, 3 -> B + 4, B + 5.
                        const int b = lane_byte<FMT>(lane * PER);
                        *reinterpret_cast<uint16_t *>(d0p + dd * WSB + b) =
                            (uint16_t)prmt(db[dd][0], db[dd][2], 0x0040u);
                        *reinterpret_cast<uint16_t *>(d0p + dd * WSB + b + 4) =
                            (uint16_t)prmt(db[dd][1], db[dd][3 % PER], 0x0040u);
                    } else {
                        // Values i = 0, 1 -> adjacent bytes.
                        const int b = lane_byte<FMT>(lane * PER);
                        *reinterpret_cast<uint16_t *>(d0p + dd * WSB + b) =
                            (uint16_t)prmt(db[dd][0], db[dd][1 % PER], 0x0040u);
                    }
                }
                if (lane < 3) {
                    float f = bad ? __int_as_float(0x7fc00000) : ldexpf(FMT == 0 ? 0.0625f : 1.0f, e);
                    f *= lane == 0 ? 1.0f : (lane == 1 ? 0.0078125f : 6.103515625e-05f);
                    fxw[q * 8 + 3 * m + lane] = f;
                }
            }
        }
    }
    for (int q = 0; q < nw; q++)
        if (lane >= ncol && lane < 8) fxw[q * 8 + lane] = 0.f;
    __syncwarp();

    float *red = reinterpret_cast<float *>(smem + p.red_off);  // [kBatch][kWarps][32]
    float res[kBatch][4];
#pragma unroll
    for (int b = 0; b < kBatch; b++)
#pragma unroll
        for (int i = 0; i < 4; i++) res[b][i] = 0.f;

    int it = 0;
    for (int lt = 0; lt < nt; lt++) {
        const int slot = lt % kScaleSlots, ph = (lt / kScaleSlots) & 1;
        const bool ready = !*abort && mbar_wait(&full[slot], ph, p.err, abort);
        const float *sc = reinterpret_cast<const float *>(smem + slot * p.scale_slot_bytes);
        const int bl = lt % kBatch;
        for (int q = 0; q < nw; q++, it++) {
            issue(it + kDepth - 1);
            cp_wait<kDepth - 1>();  // item `it` has landed (this lane's copies)
            if (!ready) continue;
            const unsigned char *item = ring + (it % kDepth) * kItemBytes;
            const uint4 wa = lds128(item + g * 64 + t * 16);
            const uint4 wb = lds128(item + (g + 8) * 64 + t * 16);
            const uint32_t qa[4] = {wa.x, wa.y, wa.z, wa.w}, qb[4] = {wb.x, wb.y, wb.z, wb.w};
            uint32_t ag[2 * J], a8[2 * J];
            if (FMT == 0) {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    ag[2 * j] = (qa[j] << 4) & 0xF0F0F0F0u;
                    ag[2 * j + 1] = qa[j] & 0xF0F0F0F0u;
                    a8[2 * j] = (qb[j] << 4) & 0xF0F0F0F0u;
                    a8[2 * j + 1] = qb[j] & 0xF0F0F0F0u;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    ag[j] = qa[j];
                    a8[j] = qb[j];
                }
            }
            int acc[4] = {0, 0, 0, 0};
            const int8_t *cell = dig + (q * ncol + g) * WSB + t * 8;
#pragma unroll
            for (int j = 0; j < J; j++) {
                uint2 b = make_uint2(0u, 0u);
                if (g < ncol) b = lds64u(cell + j * 32);
                mma_s8(acc, ag[2 * j], a8[2 * j], ag[2 * j + 1], a8[2 * j + 1], b.x, b.y);
            }
            const int gi = (ws0 + q) >> p.gs_shift;
            const float s0 = sc[g * p.groups + gi], s1 = sc[(g + 8) * p.groups + gi];
            const float2 f = *reinterpret_cast<const float2 *>(fxw + q * 8 + 2 * t);
            res[bl][0] = fmaf(i2f_small(acc[0]), s0 * f.x, res[bl][0]);
            res[bl][1] = fmaf(i2f_small(acc[1]), s0 * f.y, res[bl][1]);
            res[bl][2] = fmaf(i2f_small(acc[2]), s1 * f.x, res[bl][2]);
            res[bl][3] = fmaf(i2f_small(acc[3]), s1 * f.y, res[bl][3]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);

        if (bl == kBatch - 1 || lt == nt - 1) {
            // ---- batch reduction: per warp, rows (g, g + 8) x digit column
            // 2t + {0, 1}; digits of column m sit in columns 3m .. 3m + 2.
            // Lane (g, t) publishes rows g and g + 8 of columns 2t, 2t + 1.
#pragma unroll
            for (int b = 0; b < kBatch; b++) {
                if (b <= bl) {
                    float *rw = red + (b * kWarps + warp) * 128;  // [16 rows][8 cols]
                    rw[g * 8 + 2 * t] = res[b][0];
                    rw[g * 8 + 2 * t + 1] = res[b][1];
                    rw[(g + 8) * 8 + 2 * t] = res[b][2];
                    rw[(g + 8) * 8 + 2 * t + 1] = res[b][3];
                }
#pragma unroll
                for (int i = 0; i < 4; i++) res[b][i] = 0.f;
            }
            consumers_sync();
            const int first = lt - bl;
            for (int o = threadIdx.x; o < (bl + 1) * 16 * p.M; o += kWarps * 32) {
                const int m = o / ((bl + 1) * 16), r2 = o - m * (bl + 1) * 16;
                const int b = r2 >> 4, r = r2 & 15;
                float v = 0.f;
                for (int w = 0; w < kWarps; w++) {
                    const float *q3 = red + (b * kWarps + w) * 128 + r * 8 + 3 * m;
                    v += (q3[0] + q3[1]) + q3[2];
                }
                int row;
                const int sg = tile_segment(p, t0 + first + b, &row);
                if (ready) p.out[sg][(long long)m * p.N[sg] + row + r] = v;
            }
            consumers_sync();
        }
    }
    cp_wait<0>();
}

struct LanePlan {
    bool ok = false;
    int tiles = 0, grid = 0, spr = 0, wmax = 0, scale_slot = 0;
    int dig_off = 0, fx_off = 0, ring_off = 0, red_off = 0, bar_off = 0;
    size_t smem = 0;
};

size_t up16(size_t v) { return (v + 15) / 16 * 16; }

LanePlan make_plan(const QuantSeg *segs, int nseg, size_t m) {
    LanePlan pl;
    if (nseg < 1 || nseg > kMaxSeg || m < 1 || m > 2) return pl;
    const QuantWeight &w0 = segs[0].w;
    const int kstep = w0.format == 0 ? 128 : 64;
    long long tiles = 0;
    for (int i = 0; i < nseg; i++) {
        const QuantWeight &w = segs[i].w;
        if (w.n == 0 || w.n % 16 != 0 || w.k != w0.k || w.format != w0.format ||
            w.group != w0.group || w.k % kstep != 0 || w.group % kstep != 0 ||
            w.row_bytes % 64 != 0 || w.groups % 4 != 0 || w.groups > 256 || !aligned16(w.codes) ||
            !aligned16(w.scales) || w.n > (1u << 24))
            return pl;
        tiles += (long long)(w.n / 16);
    }
    const size_t gsteps = w0.group / kstep;
    // Launches of at most three tiles per SM, where the fixed cost of a
    // launch dominates; larger ones stream better through qgemv_imma's
    // 128-row TMA boxes. Long rows (K > 8192) also go there: every CTA here
    // stages the digits of all of K, qgemv_imma's only those of its K slice.
    if ((gsteps & (gsteps - 1)) != 0 || tiles > 3LL * kSmCount || w0.k > 8192) return pl;
    pl.tiles = (int)tiles;
    pl.grid = (int)std::min<long long>(tiles, kSmCount);
    pl.spr = (int)(w0.row_bytes / 64);
    pl.wmax = (pl.spr + kWarps - 1) / kWarps;
    const int wsb = w0.format == 0 ? 128 : 64;
    pl.scale_slot = (int)up16((size_t)16 * w0.groups * 4);
    size_t off = (size_t)kScaleSlots * pl.scale_slot;
    pl.dig_off = (int)off;
    off = up16(off + (size_t)kWarps * pl.wmax * 3 * m * wsb);
    pl.fx_off = (int)off;
    off = up16(off + (size_t)kWarps * pl.wmax * 8 * 4);
    off = (off + 127) / 128 * 128;
    pl.ring_off = (int)off;
    off += (size_t)kWarps * kDepth * kItemBytes;
    pl.red_off = (int)off;
    off += (size_t)kBatch * kWarps * 128 * 4;
    pl.bar_off = (int)off;
    off += 2 * kScaleSlots * 8 + 16;
    pl.smem = off;
    pl.ok = pl.smem <= (size_t)kSmemLimit;
    return pl;
}

struct ScaleKey {
    const void *scales;
    size_t n, groups;
    bool operator==(const ScaleKey &o) const {
        return scales == o.scales && n == o.n && groups == o.groups;
    }
};
struct ScaleKeyHash {
    size_t operator()(const ScaleKey &k) const {
        return std::hash<const void *>()(k.scales) * 31 + k.n * 7 + k.groups;
    }
};

bool scale_map(const QuantWeight &w, CUtensorMap *out) {
    static std::mutex mu;
    static std::unordered_map<ScaleKey, CUtensorMap, ScaleKeyHash> cache;
    const ScaleKey key{w.scales, w.n, w.groups};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return true;
    }
    CUtensorMap m;
    if (!encode_tensor_map_2d(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.scales, w.groups, w.n,
                              w.groups * 4, (uint32_t)w.groups, 16))
        return false;
    if (cache.size() > 8192) cache.clear();
    cache.emplace(key, m);
    *out = m;
    return true;
}

template <int FMT>
cudaError_t launch_lane(cudaStream_t s, const float *x, const float *x2, size_t m,
                        const QuantSeg *segs, int nseg, const LanePlan &pl, uint32_t *err) {
    LaneArgs a{};
    int tiles = 0;
    for (int i = 0; i < nseg; i++) {
        if (!scale_map(segs[i].w, &a.scales_map[i])) return cudaErrorInvalidValue;
        a.codes[i] = segs[i].w.codes;
        a.out[i] = segs[i].out;
        a.N[i] = (int)segs[i].w.n;
        tiles += (int)(segs[i].w.n / 16);
        a.tile_end[i] = tiles;
    }
    const QuantWeight &w = segs[0].w;
    a.nseg = nseg;
    a.x = x;
    a.x2 = x2;
    a.err = err;
    a.row_bytes = (long long)w.row_bytes;
    a.M = (int)m;
    a.K = (int)w.k;
    a.spr = pl.spr;
    a.groups = (int)w.groups;
    a.gs_shift = 0;
    while ((1u << a.gs_shift) < w.group / (size_t)Lane<FMT>::kKStep) a.gs_shift++;
    a.tiles = pl.tiles;
    a.wmax = pl.wmax;
    a.scale_slot_bytes = pl.scale_slot;
    a.dig_off = pl.dig_off;
    a.fx_off = pl.fx_off;
    a.ring_off = pl.ring_off;
    a.red_off = pl.red_off;
    a.bar_off = pl.bar_off;
    static std::atomic<uint64_t> smem_set{0};
    set_smem_limit_once(qgemv_lane<FMT>, kSmemLimit, &smem_set);
    launch_k(qgemv_lane<FMT>, pl.grid, kThreads, pl.smem, s, a);
    count_launch();
    return cudaGetLastError();
}

}  // namespace

bool qgemv_lane_supported(const QuantSeg *segs, int nseg, size_t m) {
    return make_plan(segs, nseg, m).ok;
}

cudaError_t qgemv_lane_group(cudaStream_t s, const float *x, const float *x2, size_t m,
                             const QuantSeg *segs, int nseg, uint32_t *err) {
    LanePlan pl = make_plan(segs, nseg, m);
    if (!pl.ok || !aligned16(x) || (x2 && !aligned16(x2))) return cudaErrorInvalidValue;
    return segs[0].w.format == 0 ? launch_lane<0>(s, x, x2, m, segs, nseg, pl, err)
                                 : launch_lane<1>(s, x, x2, m, segs, nseg, pl, err);
}

}  // namespace k
}  // namespace slc
