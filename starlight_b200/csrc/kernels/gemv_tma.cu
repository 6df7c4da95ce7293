// Decode GEMV for group-quantized weights, fed by bulk asynchronous copies
// (TMA) into a shared-memory ring: out[m, n] = sum_k x[m, k] * w[n, k] with
// w = code * scale[n, k / group], small M (decode batch).
//
// Parity target: dequantize, then backend-cpu's f32 matmul_nt
// (crates/backends/backend-cpu/src/reference/matmul.rs:29-59).
//
// HBM-bound on the payload; algorithmic bytes per launch
//   N * row_bytes + 4 * N * K / group + 4 * M * (K + N).
//
// Work decomposition. The weight matrix is cut into tiles of 16 rows (one
// mma.sync M tile) and every tile into warp-steps of 64 bytes per row (128
// INT4 or 64 INT8 codes, always inside one quantization group). The
// n_tiles * steps_per_row warp-steps are ordered tile-major and split into
// one contiguous, balanced range per CTA (persistent grid, one CTA per SM),
// so every CTA streams the same number of bytes to within one warp-step.
//
// Per CTA, warp 8 is the producer: it cuts its range into stages of at most
// 32 warp-steps (16 rows x <= 2 KiB) that never cross a tile, and copies
// each row of a stage with one cp.async.bulk into a ring slot (row pitch
// 2 KiB + 64 B, so that the consumers' 16-byte reads of two rows per phase
// are conflict-free), completing on the slot's "full" mbarrier. Bulk copies
// are issued per row of up to 2 KiB because their throughput is bounded by
// the copy count (measured on B200: 256 B copies reach 1.3 TB/s, >= 2 KiB
// copies the full HBM rate).
//
// Warps 0..7 consume: warp w takes warp-steps w, w + 8, ... of the stage;
// each lane reads 16-byte chunks of rows g and g + 8, turns codes into exact
// f16 integers (magic-number LOP3 / byte permute + one packed subtraction)
// and multiplies them with the activations on the tensor cores (mma.sync
// m16n8k16, f16 x f16 -> f32), activations split into f16 hi + lo after a
// power-of-two prescale per column; the group scale is applied after every
// warp-step. Each warp releases the slot on its "empty" mbarrier. All waits
// are bounded (1 s), after which the kernel records an error for the host
// and skips the rest of its work.
//
// Activations are staged once per CTA (all of K, the permuted f16 layout of
// gemv_common.cuh); shapes whose activations do not fit next to the ring
// use the register-streaming kernel of gemv_quant.cu.
//
// Results: at the end of a tile's run the 8 warps' sums are added in warp
// order through shared memory. A CTA that covered the whole tile writes the
// output; otherwise each contributing CTA writes a partial to a workspace
// slot (its rank among the tile's contributors) and the last one to arrive
// (atomic ticket, no waiting) adds the slots in ascending order, so results
// are deterministic for a given shape.
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

constexpr int kTiles = 8;                         // 16-row tiles per block
constexpr int kTileRows = 16;                     // rows per tile (mma M)
constexpr int kBlockRows = kTileRows * kTiles;    // 128 rows per block
constexpr int kStepBytes = 64;                    // bytes per row per warp-step
constexpr int kRun = 5;                           // warp-steps per stage
constexpr int kPitch = kRun * kStepBytes;         // 320 bytes: = 64 mod 128, so the 16-byte
                                                  // reads of rows g and g + 1 never collide
constexpr int kScaleBox = 8;                      // scale groups per row per stage (box)
constexpr int kCodeBytes = kBlockRows * kPitch;   // 40 KiB
constexpr int kScaleBytes = kBlockRows * kScaleBox * 4;
constexpr int kSlotBytes = kCodeBytes + kScaleBytes;  // 44 KiB
constexpr int kMaxStages = 5;
constexpr int kMinStages = 3;
constexpr int kSmemLimit = 227 * 1024;

constexpr int kMaxSeg = 4;  // weight matrices per launch (same x, same K)

struct TmaArgs {
    CUtensorMap codes_map[kMaxSeg];   // [N][row_bytes / 8] u64, box [128][kRun * 8]
    CUtensorMap scales_map[kMaxSeg];  // [N][groups] f32, box [128][8]
    const float *x;         // [M, K]
    const float *x2;        // SwiGLU: the staged activation is silu(x) * x2; else null
    float *out[kMaxSeg];    // [M, N_s]
    int N[kMaxSeg];         // rows of each matrix
    int blk_end[kMaxSeg];   // cumulative 128-row block counts
    int nseg;
    float *partials;        // [slots][M][n_blocks * 128]
    unsigned *tickets;      // [n_blocks]
    uint32_t *err;          // device error word or null
    int M, K, groups;
    int gs_shift;           // log2(warp-steps per quantization group)
    long long row_bytes;
    long long spr;          // warp-steps per row
    long long total;        // n_blocks * spr
    long long units;        // n_blocks * split: the work units CTAs are given
    int split;              // K slices per block (1: every CTA owns whole blocks)
    long long prow;         // n_blocks * 128: row stride of the partial slots
    int nstage;
    int S;                  // 16-byte units per staged activation column (padded)
    int ring_bytes;         // shared offset of the activation planes
    int unscale_floats;     // M * spr rounded up to an even count
    // Integer consumer (qgemv_imma) only:
    int Sn;                 // bytes per digit column (= 32 mod 128)
    int ncol;               // digit columns: 3 * M
    int xd_off, fx_off, red_off;  // shared offsets of digits, factors, block sums
    // K slices (qgemv_imma): CTA c works on warp-steps [s * spr, (s + 1) * spr)
    // of every row, s = c / (gridDim.x / nslice); spr, total and units then
    // describe one slice. 1 everywhere else.
    int nslice;
};

// Matrix of a (global) block and the block's index inside it.
__device__ __forceinline__ int block_segment(const TmaArgs &p, long long blk, int *local) {
    int sgi = 0;
    while (sgi + 1 < p.nseg && blk >= p.blk_end[sgi]) sgi++;
    *local = (int)(blk - (sgi ? p.blk_end[sgi - 1] : 0));
    return sgi;
}

template <int CW>
__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(CW * 32) : "memory");
}

// Work split. A unit is one K slice of one 128-row block: slice r of a block
// covers warp-steps [r * spr / split, (r + 1) * spr / split). CTA c gets
// units [c * units / grid, (c + 1) * units / grid), so with split == 1 it
// owns whole blocks and never shares one (no partial sums).
__device__ __forceinline__ long long unit_start(const TmaArgs &p, long long i) {
    if (i >= p.units) return p.total;
    const long long blk = i / p.split;
    const long long r = i - blk * p.split;
    return blk * p.spr + (r * p.spr) / p.split;
}

// CTA whose range contains warp-step u.
__device__ __forceinline__ long long owner(const TmaArgs &p, long long u, long long grid) {
    const long long blk = u / p.spr, st = u - blk * p.spr;
    const long long r = (st * p.split + p.split - 1) / p.spr;  // slice holding step st
    const long long i = blk * p.split + r;
    return ((i + 1) * grid - 1) / p.units;
}

__device__ __forceinline__ int prescale_exponent(float mx) {
    int e = 0;
    if (mx > 0.f) {
        int ex;
        frexpf(mx, &ex);
        e = 14 - ex;
        e = e > 126 ? 126 : (e < -126 ? -126 : e);
    }
    return e;
}

// Position of activation k of column col in the f16 planes. INT4: lane quad
// t of a warp-step reads codes 32t .. 32t + 31 as four words q of eight
// codes, so the 8-value unit (ws, q, t) sits at ws * 16 + 4q + t: the four
// quads read consecutive 16-byte units (conflict-free), and within a unit
// value e sits at the f16 slot of the nibble pair (i, i + 4) that int4_pairs
// produces. INT8: natural order (lane quads read units 2t, 2t + 1).
template <int FMT>
__device__ __forceinline__ int tma_slot(int kr, int S, int col) {
    if (FMT == 0) {
        const int unit = (kr >> 7) * 16 + ((kr >> 3) & 3) * 4 + ((kr >> 5) & 3);
        const int e = kr & 7;
        return (col * S + unit) * 8 + (e < 4 ? 2 * e : 2 * (e - 4) + 1);
    }
    return (col * S + (kr >> 3)) * 8 + (kr & 7);
}

// Stages all of x into the permuted f16 hi/lo planes (consumer warps only).
// Every block of one warp-step's k values (128 for INT4, 64 for INT8) of a
// column gets its own power-of-two prescale, computed by one warp from one
// vectorised load per lane, so staging needs no CTA-wide reduction; the
// inverse (`unscale[col][step]`) is applied after the step's MMAs.
template <int FMT, int CW>
__device__ void stage_x(const TmaArgs &p, __half *xh, __half *xl, float *unscale) {
    constexpr int KSTEP = Fmt<FMT>::kStep;
    constexpr int PER = KSTEP / 32;  // values per lane: 4 (INT4) or 2 (INT8)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int spr = (int)p.spr;
    const int blocks = p.M * spr;
    for (int b = warp; b < blocks; b += CW) {
        const int col = b / spr, st = b - col * spr;
        const int k0 = st * KSTEP + lane * PER;
        const float *src = p.x + (long long)col * p.K + k0;
        float v[PER];
        if constexpr (PER == 4) {
            const float4 q = __ldg(reinterpret_cast<const float4 *>(src));
            v[0] = q.x;
            v[1] = q.y;
            v[2] = q.z;
            v[3] = q.w;
        } else {
            const float2 q = __ldg(reinterpret_cast<const float2 *>(src));
            v[0] = q.x;
            v[1] = q.y;
        }
        if (p.x2) {
            // SwiGLU: silu(gate) * up, the exact expression of the
            // elementwise silu_mul kernel (so the product is bit-identical).
            const float *src2 = p.x2 + (long long)col * p.K + k0;
            float u[PER];
            if constexpr (PER == 4) {
                const float4 q = __ldg(reinterpret_cast<const float4 *>(src2));
                u[0] = q.x;
                u[1] = q.y;
                u[2] = q.z;
                u[3] = q.w;
            } else {
                const float2 q = __ldg(reinterpret_cast<const float2 *>(src2));
                u[0] = q.x;
                u[1] = q.y;
            }
#pragma unroll
            for (int i = 0; i < PER; i++)
                v[i] = __fmul_rn(__fmul_rn(v[i], __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v[i])))),
                                 u[i]);
        }
        float mx = 0.f;
#pragma unroll
        for (int i = 0; i < PER; i++) mx = fmaxf(mx, fabsf(v[i]));
        const int e = prescale_exponent(warp_max(mx));
        const float up = ldexpf(1.0f, e);
#pragma unroll
        for (int i = 0; i < PER; i++) {
            const float y = v[i] * up;
            const __half hi = __float2half_rn(y);
            const __half lo = __float2half_rn(y - __half2float(hi));
            const int slot = tma_slot<FMT>(k0 + i, p.S, col);
            xh[slot] = hi;
            xl[slot] = lo;
        }
        if (lane == 0) unscale[b] = ldexpf(1.0f, -e);
    }
    consumer_sync<CW>();
}

// One warp-step (64 bytes of rows g and g + 8 per lane quad) into acc. The
// MMAs go to four independent accumulator chains (hi / lo activation part x
// even / odd chunk) that are added at the end, so that consecutive MMAs do
// not wait on each other's results.
template <int FMT, int NT>
__device__ __forceinline__ void warp_step(const unsigned char *tile, int pitch, int ws,
                                          const __half *xh, const __half *xl, int S, int Mc,
                                          int g, int t, float (&acc)[NT][4]) {
    float ch[4][NT][4];
#pragma unroll
    for (int c = 0; c < 4; c++)
#pragma unroll
        for (int jn = 0; jn < NT; jn++)
#pragma unroll
            for (int i = 0; i < 4; i++) ch[c][jn][i] = 0.f;
    const uint4 wg = lds128(tile);
    const uint4 wg8 = lds128(tile + 8 * pitch);
    const uint32_t wa[4] = {wg.x, wg.y, wg.z, wg.w};
    const uint32_t wb[4] = {wg8.x, wg8.y, wg8.z, wg8.w};
    if (FMT == 0) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
            uint32_t pa[4], pb[4];
            int4_pairs(wa[q], pa);
            int4_pairs(wb[q], pb);
            const int phys = ws * 16 + 4 * q + t;
            const int c = (q & 1) * 2;
#pragma unroll
            for (int jn = 0; jn < NT; jn++) {
                const int col = g + 8 * jn;
                uint4 bh = make_uint4(0, 0, 0, 0), bl = bh;
                if (col < Mc) {
                    bh = lds128(xh + ((size_t)col * S + phys) * 8);
                    bl = lds128(xl + ((size_t)col * S + phys) * 8);
                }
                mma16816(ch[c][jn], pa[0], pb[0], pa[1], pb[1], bh.x, bh.y);
                mma16816(ch[c + 1][jn], pa[0], pb[0], pa[1], pb[1], bl.x, bl.y);
                mma16816(ch[c][jn], pa[2], pb[2], pa[3], pb[3], bh.z, bh.w);
                mma16816(ch[c + 1][jn], pa[2], pb[2], pa[3], pb[3], bl.z, bl.w);
            }
        }
    } else {
#pragma unroll
        for (int qq = 0; qq < 2; qq++) {
            uint32_t lo_a[2], hi_a[2], lo_b[2], hi_b[2];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t xa = wa[2 * qq + h] ^ 0x80808080u;
                const uint32_t xb = wb[2 * qq + h] ^ 0x80808080u;
                lo_a[h] = hsub2(prmt(xa, 0x64646464u, 0x4140u), 0x64806480u);
                hi_a[h] = hsub2(prmt(xa, 0x64646464u, 0x4342u), 0x64806480u);
                lo_b[h] = hsub2(prmt(xb, 0x64646464u, 0x4140u), 0x64806480u);
                hi_b[h] = hsub2(prmt(xb, 0x64646464u, 0x4342u), 0x64806480u);
            }
            const int unit = ws * 8 + 2 * t + qq;
#pragma unroll
            for (int jn = 0; jn < NT; jn++) {
                const int col = g + 8 * jn;
                uint4 bh = make_uint4(0, 0, 0, 0), bl = bh;
                if (col < Mc) {
                    bh = lds128(xh + ((size_t)col * S + unit) * 8);
                    bl = lds128(xl + ((size_t)col * S + unit) * 8);
                }
                mma16816(ch[0][jn], lo_a[0], lo_b[0], hi_a[0], hi_b[0], bh.x, bh.y);
                mma16816(ch[1][jn], lo_a[0], lo_b[0], hi_a[0], hi_b[0], bl.x, bl.y);
                mma16816(ch[2][jn], lo_a[1], lo_b[1], hi_a[1], hi_b[1], bh.z, bh.w);
                mma16816(ch[3][jn], lo_a[1], lo_b[1], hi_a[1], hi_b[1], bl.z, bl.w);
            }
        }
    }
#pragma unroll
    for (int jn = 0; jn < NT; jn++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[jn][i] = (ch[0][jn][i] + ch[2][jn][i]) + (ch[1][jn][i] + ch[3][jn][i]);
}

// The warp-steps j = h, h + SPLIT, ... of a stage for one warp (tile rows at
// `base`), scaled into res. FULL: the stage holds all kRun steps (no guards,
// so the compiler can interleave the steps).
template <int FMT, int NT, int SPLIT, bool FULL>
__device__ __forceinline__ void stage_math(const TmaArgs &p, const unsigned char *base,
                                           const float *ssl, int step0, int run, int h,
                                           const __half *xh, const __half *xl,
                                           const float *unscale, int g, int t,
                                           float (&res)[NT][4]) {
    const int g4 = (step0 >> p.gs_shift) & ~3;
    const int Mc = p.M;
#pragma unroll
    for (int jj = 0; jj < (kRun + SPLIT - 1) / SPLIT; jj++) {
        const int j = jj * SPLIT + h;
        if (j < kRun && (FULL || j < run)) {
            float acc[NT][4];
            const int sw = step0 + j;
            warp_step<FMT, NT>(base + j * kStepBytes, kPitch, sw, xh, xl, p.S, Mc, g, t, acc);
            const int gi = (sw >> p.gs_shift) - g4;
            const float s0 = ssl[gi], s1 = ssl[8 * kScaleBox + gi];
#pragma unroll
            for (int jn = 0; jn < NT; jn++) {
                const int c0 = 2 * t + 8 * jn, c1 = c0 + 1;
                const float u0s = c0 < Mc ? unscale[c0 * (int)p.spr + sw] : 0.f;
                const float u1s = c1 < Mc ? unscale[c1 * (int)p.spr + sw] : 0.f;
                res[jn][0] = fmaf(s0 * u0s, acc[jn][0], res[jn][0]);
                res[jn][1] = fmaf(s0 * u1s, acc[jn][1], res[jn][1]);
                res[jn][2] = fmaf(s1 * u0s, acc[jn][2], res[jn][2]);
                res[jn][3] = fmaf(s1 * u1s, acc[jn][3], res[jn][3]);
            }
        }
    }
}

// Producer (one thread): per stage one box of codes (128 rows x 320 bytes
// from warp-step step0) and one box of scales (128 rows x groups g4 ..
// g4 + 7, g4 rounded down to 4 groups = 16 bytes) into the next ring slot.
__device__ __forceinline__ void produce(const TmaArgs &p, unsigned char *ring, uint64_t *full,
                                        uint64_t *empty, volatile int *abort, long long u0,
                                        long long u1, int kbase) {
    for (int i = 0; i < p.nseg; i++) {
        prefetch_tensormap(&p.codes_map[i]);
        prefetch_tensormap(&p.scales_map[i]);
    }
    const uint64_t pol = policy_evict_first();
    int slot = 0, phase = 0;
    bool first_pass = true;
    for (long long u = u0; u < u1;) {
        const long long blk = u / p.spr;
        const long long run_end = min(u1, (blk + 1) * p.spr);
        int lblk;
        const int sgi = block_segment(p, blk, &lblk);
        while (u < run_end) {
            const int run = (int)min((long long)kRun, run_end - u);
            if (!first_pass && !mbar_wait(&empty[slot], phase ^ 1, p.err, abort)) return;
            const long long step0 = u - blk * p.spr + kbase;  // warp-step within the row
            const int g4 = (int)(step0 >> p.gs_shift) & ~3;
            unsigned char *sl = ring + slot * kSlotBytes;
            mbar_arrive_expect_tx(&full[slot], (uint32_t)kSlotBytes);
            tma_load_2d(sl, &p.codes_map[sgi], (int)(step0 * (kStepBytes / 8)),
                        lblk * kBlockRows, &full[slot], pol);
            tma_load_2d(sl + kCodeBytes, &p.scales_map[sgi], g4, lblk * kBlockRows, &full[slot],
                        pol);
            u += run;
            if (++slot == p.nstage) {
                slot = 0;
                phase ^= 1;
                first_pass = false;
            }
        }
    }
}

// SPLIT consumer warps share each 16-row tile (warp w: tile w % 8, steps
// h = w / 8, h + SPLIT, ... of every stage); their sums meet in shared
// memory at the end of a block's run.
template <int FMT, int NT, int SPLIT>
__global__ void __launch_bounds__((kTiles * SPLIT + 1) * 32, 1)
    qgemv_tma(const __grid_constant__ TmaArgs p) {
    constexpr int CW = kTiles * SPLIT;  // consumer warps
    extern __shared__ __align__(1024) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int tile = warp % kTiles, h = warp / kTiles;
    const int Mc = p.M;

    unsigned char *ring = smem;
    __half *xh = reinterpret_cast<__half *>(smem + p.ring_bytes);
    __half *xl = xh + (size_t)Mc * p.S * 8;
    float *unscale = reinterpret_cast<float *>(xl + (size_t)Mc * p.S * 8);  // [M][spr]
    float *red = unscale + p.unscale_floats;  // [kTiles][32 lanes][16] (SPLIT > 1)
    uint64_t *full = reinterpret_cast<uint64_t *>(red + (SPLIT > 1 ? kTiles * 32 * 16 : 0));
    uint64_t *empty = full + kMaxStages;
    int *last_flag = reinterpret_cast<int *>(empty + kMaxStages);
    volatile int *abort = last_flag + 1;  // set when a wait timed out

    const long long grid = gridDim.x, cta = blockIdx.x;
    const long long u0 = unit_start(p, cta * p.units / grid);
    const long long u1 = unit_start(p, (cta + 1) * p.units / grid);

    // The producer streams weights before the previous kernel has finished
    // (weights are written only by uploads and quantization, which complete
    // before any dispatch); consumers wait for it before reading x.
    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nstage; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], CW);
        }
        fence_mbar_init();
        *abort = 0;
    }
    __syncthreads();

    if (warp == CW) {
        if (lane == 0) produce(p, ring, full, empty, abort, u0, u1, 0);
        return;
    }

    // ---- consumers.
    pdl_wait();
    stage_x<FMT, CW>(p, xh, xl, unscale);
    float res[NT][4];
    int slot = 0, phase = 0;
    for (long long u = u0; u < u1;) {
        const long long blk = u / p.spr;
        const long long run_end = min(u1, (blk + 1) * p.spr);
        int lblk;
        const int sgi = block_segment(p, blk, &lblk);
        const int n_seg = p.N[sgi];
        const int row0 = lblk * kBlockRows + tile * kTileRows;  // row in this matrix
        const bool active = row0 < n_seg;
#pragma unroll
        for (int jn = 0; jn < NT; jn++)
#pragma unroll
            for (int i = 0; i < 4; i++) res[jn][i] = 0.f;
        while (u < run_end) {
            const int run = (int)min((long long)kRun, run_end - u);
            const int step0 = (int)(u - blk * p.spr);  // warp-step index within the row
            // After a timed-out wait the CTA keeps its control flow (every
            // named barrier is still reached) but skips waits and math.
            const bool ready = !*abort && mbar_wait(&full[slot], phase, p.err, abort);
            if (ready && active) {
                const unsigned char *sl = ring + slot * kSlotBytes;
                const unsigned char *base = sl + (tile * kTileRows + g) * kPitch + t * 16;
                const float *ssl = reinterpret_cast<const float *>(sl + kCodeBytes) +
                                   (tile * kTileRows + g) * kScaleBox;
                if (run == kRun)
                    stage_math<FMT, NT, SPLIT, true>(p, base, ssl, step0, run, h, xh, xl, unscale,
                                                     g, t, res);
                else
                    stage_math<FMT, NT, SPLIT, false>(p, base, ssl, step0, run, h, xh, xl,
                                                      unscale, g, t, res);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            u += run;
            if (++slot == p.nstage) {
                slot = 0;
                phase ^= 1;
            }
        }

        // ---- end of this CTA's run over the block.
        if (SPLIT > 1) {
            // Warps h > 0 hand their sums to warp h = 0 of the same tile.
            float *rl = red + (tile * 32 + lane) * 16;
            if (h > 0) {
#pragma unroll
                for (int jn = 0; jn < NT; jn++)
#pragma unroll
                    for (int i = 0; i < 4; i++) rl[jn * 4 + i] = res[jn][i];
            }
            consumer_sync<CW>();
            if (h == 0) {
#pragma unroll
                for (int jn = 0; jn < NT; jn++)
#pragma unroll
                    for (int i = 0; i < 4; i++) res[jn][i] += rl[jn * 4 + i];
            }
            consumer_sync<CW>();
        }
        const long long first = owner(p, blk * p.spr, grid);
        const long long last = owner(p, (blk + 1) * p.spr - 1, grid);
        const int count = (int)(last - first + 1);
        // Direct output, or this CTA's partial slot (rows indexed over all
        // matrices' blocks).
        float *dst;
        long long ld, r0;
        if (count == 1) {
            dst = p.out[sgi];
            ld = n_seg;
            r0 = row0;
        } else {
            dst = p.partials + (cta - first) * (long long)Mc * p.prow;
            ld = p.prow;
            r0 = blk * kBlockRows + tile * kTileRows;
        }
        if (active && h == 0) {
#pragma unroll
            for (int jn = 0; jn < NT; jn++) {
                const int c0 = 2 * t + 8 * jn, c1 = c0 + 1;
                if (c0 < Mc) {
                    dst[c0 * ld + r0 + g] = res[jn][0];
                    dst[c0 * ld + r0 + g + 8] = res[jn][2];
                }
                if (c1 < Mc) {
                    dst[c1 * ld + r0 + g] = res[jn][1];
                    dst[c1 * ld + r0 + g + 8] = res[jn][3];
                }
            }
        }
        if (count > 1) {
            __threadfence();
            consumer_sync<CW>();
            if (threadIdx.x == 0) {
                const unsigned ticket = atomicAdd(&p.tickets[blk], 1u);
                *last_flag = ticket == (unsigned)(count - 1);
            }
            consumer_sync<CW>();
            const bool is_last = *last_flag;
            consumer_sync<CW>();  // last_flag is rewritten by the next shared block
            if (is_last) {
                __threadfence();
                const int rows_here = min(kBlockRows, n_seg - lblk * kBlockRows);
                for (int i = threadIdx.x; i < Mc * rows_here; i += CW * 32) {
                    const int c = i / rows_here, r = i % rows_here;
                    const float *src = p.partials + (long long)c * p.prow + blk * kBlockRows + r;
                    const long long slot_stride = (long long)Mc * p.prow;
                    float v = 0.f;
#pragma unroll 8
                    for (int sl = 0; sl < count; sl++) v += __ldcg(src + sl * slot_stride);
                    p.out[sgi][(long long)c * n_seg + lblk * kBlockRows + r] = v;
                }
                if (threadIdx.x == 0) p.tickets[blk] = 0u;  // ready for the next launch
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Exact-integer consumer (qgemv_imma). The same producer, ring, work split and
// partial-sum protocol as qgemv_tma, with the products formed by the s8 tensor
// path (mma.sync m16n8k32, s8 x s8 -> s32) instead of f16:
//
//  * Codes become s8 without arithmetic: an INT4 nibble moved to the top of
//    its byte is 16 x code (odd nibbles are masked in place, even nibbles
//    shifted up by 4), INT8 bytes are used as they are.
//  * Every activation block of one warp-step (128 k for INT4, 64 for INT8)
//    of column m is written as x = 2^e * (d0 + d1 / 128 + d2 / 16384) with
//    digits d in [-64, 64] (e from the block's largest magnitude, so that
//    |x / 2^e| < 64): about 20 significant bits relative to the block's
//    largest value, every step exact in f32.
//  * The digits are the MMA's N dimension: column n = 3m + d, so one n8 tile
//    carries the three digits of two activation columns and M = 1 or 2 costs
//    4 (INT4) or 2 (INT8) MMAs per 16 rows x one warp-step.
//  * Integer sums of one warp-step (|sum| < 2^21) convert to f32 exactly
//    and are scaled by scale[n, group] * 2^e * 2^-7d (x 1/16 for INT4).
// Column sums of the three digits are added at the end of a block.
template <int FMT>
struct Imma;
template <>
struct Imma<0> {
    static constexpr int kWsBytes = 128;  // digit bytes per column per warp-step
    static constexpr int kJ = 4;          // k32 MMAs per warp-step
};
template <>
struct Imma<1> {
    static constexpr int kWsBytes = 64;
    static constexpr int kJ = 2;
};

// Byte of activation k (within its warp-step) inside the column's warp-step
// block, laid out [j][t][8 bytes] so that lane (g, t) reads the B fragment
// of MMA j with one 8-byte load: bytes 0..3 = register b0, 4..7 = b1.
// INT4: lane quad t holds codes 32t .. 32t + 31; MMA j pairs the even
// nibbles of word j (k = 32t + 8j + 2i) in b0 with the odd ones in b1.
// INT8: lane quad t holds codes 16t .. 16t + 15; MMA j takes words 2j and
// 2j + 1 (k = 16t + 8j + i and 16t + 8j + 4 + i).
template <int FMT>
__device__ __forceinline__ int imma_byte(int kl) {
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

__device__ __forceinline__ uint2 lds64(const void *p) {
    uint2 r;
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(a));
    return r;
}

// Exact int -> float for |c| < 2^22 on the integer and FP32 pipes.
__device__ __forceinline__ float i2f_small(int c) {
    return __int_as_float(c + 0x4B400000) - 12582912.0f;
}

// Stages the activation digit planes of warp-steps ws0 .. ws0 + nws - 1
// (mod spr: the ones this CTA's range touches) for every column (consumer
// warps only). Block (m, ws) is converted by one warp, each lane taking 4
// (INT4) or 2 (INT8) values; a warp issues the loads of up to kBatch blocks
// before converting any, so staging costs about one load latency.
template <int FMT, int CW, int NT>
__device__ void stage_digits(const TmaArgs &p, int8_t *xd, float *fx, int ws0, int nws,
                             int kbase) {
    constexpr int KSTEP = Fmt<FMT>::kStep;
    constexpr int PER = KSTEP / 32;
    constexpr int WSB = Imma<FMT>::kWsBytes;
    constexpr int kBatch = 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int spr = (int)p.spr;
    const int blocks = p.M * nws;
    for (int b0 = warp; b0 < blocks; b0 += CW * kBatch) {
        float v[kBatch][PER], u[kBatch][PER];
#pragma unroll
        for (int q = 0; q < kBatch; q++) {
            const int b = b0 + q * CW;
            if (b >= blocks) break;
            const int col = b / nws;
            int st = ws0 + (b - col * nws);
            if (st >= spr) st -= spr;
            const long long off = (long long)col * p.K + (long long)(kbase + st) * KSTEP + lane * PER;
            if constexpr (PER == 4) {
                const float4 a = __ldg(reinterpret_cast<const float4 *>(p.x + off));
                v[q][0] = a.x;
                v[q][1] = a.y;
                v[q][2] = a.z;
                v[q][3] = a.w;
                if (p.x2) {
                    const float4 c = __ldg(reinterpret_cast<const float4 *>(p.x2 + off));
                    u[q][0] = c.x;
                    u[q][1] = c.y;
                    u[q][2] = c.z;
                    u[q][3] = c.w;
                }
            } else {
                const float2 a = __ldg(reinterpret_cast<const float2 *>(p.x + off));
                v[q][0] = a.x;
                v[q][1] = a.y;
                if (p.x2) {
                    const float2 c = __ldg(reinterpret_cast<const float2 *>(p.x2 + off));
                    u[q][0] = c.x;
                    u[q][1] = c.y;
                }
            }
        }
#pragma unroll
        for (int q = 0; q < kBatch; q++) {
            const int b = b0 + q * CW;
            if (b >= blocks) break;
            const int col = b / nws;
            int st = ws0 + (b - col * nws);
            if (st >= spr) st -= spr;
            if (p.x2) {
                // SwiGLU: silu(gate) * up, the exact expression of the
                // elementwise silu_mul kernel.
#pragma unroll
                for (int i = 0; i < PER; i++)
                    v[q][i] = __fmul_rn(
                        __fmul_rn(v[q][i], __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v[q][i])))),
                        u[q][i]);
            }
            float mx = 0.f;
            bool bad = false;
#pragma unroll
            for (int i = 0; i < PER; i++) {
                const float a = fabsf(v[q][i]);
                bad |= !(a <= 3.402823466e38f);  // inf or nan
                mx = fmaxf(mx, a);
            }
            mx = warp_max(mx);
            bad = __any_sync(0xffffffffu, bad);
            int e = 0;
            if (mx > 0.f && !bad) {
                int ex;
                frexpf(mx, &ex);
                e = ex - 6;  // |x| < 2^ex, so |x / 2^e| < 64
            }
            // Digits by exact power-of-two scaling (ldexpf outside the normal
            // exponent range) and d = rint(y), y' = fma(d, -128, 128 y).
            int8_t *dst = xd + (3 * col) * p.Sn + st * WSB;
            const bool direct = e >= -126 && e <= 126;
            const float sc = __int_as_float((127 - e) << 23);
#pragma unroll
            for (int i = 0; i < PER; i++) {
                float y = 0.f;
                if (!bad) y = direct ? v[q][i] * sc : ldexpf(v[q][i], -e);
                const float d0 = rintf(y);
                const float r1 = fmaf(d0, -128.f, y * 128.f);
                const float d1 = rintf(r1);
                const float r2 = fmaf(d1, -128.f, r1 * 128.f);
                const float d2 = rintf(r2);
                const int off = imma_byte<FMT>(lane * PER + i);
                dst[off] = (int8_t)(int)d0;
                dst[p.Sn + off] = (int8_t)(int)d1;
                dst[2 * p.Sn + off] = (int8_t)(int)d2;
            }
            if (lane < 3) {
                // 2^e, times 1/16 for the INT4 codes' byte position;
                // non-finite input makes the column's outputs NaN.
                float f = bad ? __int_as_float(0x7fc00000) : ldexpf(FMT == 0 ? 0.0625f : 1.0f, e);
                f *= lane == 0 ? 1.0f : (lane == 1 ? 0.0078125f : 6.103515625e-05f);
                fx[st * (8 * NT) + 3 * col + lane] = f;
            }
        }
    }
    // Padding columns 3M .. 8 NT - 1 contribute nothing.
    const int pad = 8 * NT - 3 * p.M;
    for (int i = threadIdx.x; i < nws * pad; i += CW * 32) {
        int st = ws0 + i / pad;
        if (st >= spr) st -= spr;
        fx[st * (8 * NT) + 3 * p.M + i % pad] = 0.f;
    }
    consumer_sync<CW>();
}

// One warp-step of one 16-row tile: integer sums c[nt] of the tile's rows
// (g, g + 8) with the lane's digit columns (8 nt + 2t, + 1).
template <int FMT, int NT>
__device__ __forceinline__ void imma_step(const unsigned char *rowg, int pitch,
                                          const unsigned char *xcell, int Sn, int ncol, int g,
                                          int (&c)[NT][4]) {
    constexpr int J = Imma<FMT>::kJ;
    uint32_t ag[2 * J], a8[2 * J];  // per MMA j: (a0 | a2) of row g and (a1 | a3) of row g + 8
    const uint4 wa = lds128(rowg);
    const uint4 wb = lds128(rowg + 8 * pitch);
    const uint32_t qa[4] = {wa.x, wa.y, wa.z, wa.w}, qb[4] = {wb.x, wb.y, wb.z, wb.w};
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
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
#pragma unroll
        for (int i = 0; i < 4; i++) c[nt][i] = 0;
        const int n = 8 * nt + g;
#pragma unroll
        for (int j = 0; j < J; j++) {
            uint2 b = make_uint2(0u, 0u);
            if (n < ncol) b = lds64(xcell + n * Sn + j * 32);
            mma_s8(c[nt], ag[2 * j], a8[2 * j], ag[2 * j + 1], a8[2 * j + 1], b.x, b.y);
        }
    }
}

template <int FMT, int NT, int SPLIT, bool FULL>
__device__ __forceinline__ void imma_stage(const TmaArgs &p, const unsigned char *base,
                                           const float *ssl, int step0, int run, int h,
                                           const unsigned char *xd, const float *fx, int g, int t,
                                           int kbase, float (&res)[NT][4]) {
    constexpr int WSB = Imma<FMT>::kWsBytes;
    // Digits and factors are indexed by the warp-step within the slice,
    // scales by the warp-step within the row.
    const int g4 = ((step0 + kbase) >> p.gs_shift) & ~3;
#pragma unroll
    for (int jj = 0; jj < (kRun + SPLIT - 1) / SPLIT; jj++) {
        const int j = jj * SPLIT + h;
        if (j < kRun && (FULL || j < run)) {
            int c[NT][4];
            const int sw = step0 + j;
            imma_step<FMT, NT>(base + j * kStepBytes, kPitch, xd + sw * WSB + t * 8, p.Sn,
                               p.ncol, g, c);
            const int gi = ((sw + kbase) >> p.gs_shift) - g4;
            const float s0 = ssl[gi], s1 = ssl[8 * kScaleBox + gi];
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const float2 f = *reinterpret_cast<const float2 *>(fx + sw * (8 * NT) + 8 * nt + 2 * t);
                res[nt][0] = fmaf(i2f_small(c[nt][0]), s0 * f.x, res[nt][0]);
                res[nt][1] = fmaf(i2f_small(c[nt][1]), s0 * f.y, res[nt][1]);
                res[nt][2] = fmaf(i2f_small(c[nt][2]), s1 * f.x, res[nt][2]);
                res[nt][3] = fmaf(i2f_small(c[nt][3]), s1 * f.y, res[nt][3]);
            }
        }
    }
}

template <int FMT, int NT, int SPLIT>
__global__ void __launch_bounds__((kTiles * SPLIT + 1) * 32, 1)
    qgemv_imma(const __grid_constant__ TmaArgs p) {
    constexpr int CW = kTiles * SPLIT;  // consumer warps
    constexpr int NC = 8 * NT;          // digit columns per lane tile row
    extern __shared__ __align__(1024) unsigned char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int tile = warp % kTiles, h = warp / kTiles;
    const int Mc = p.M;

    unsigned char *ring = smem;
    int8_t *xd = reinterpret_cast<int8_t *>(smem + p.xd_off);
    float *fx = reinterpret_cast<float *>(smem + p.fx_off);
    float *red = reinterpret_cast<float *>(smem + p.red_off);  // [CW][16][NC]
    uint64_t *full = reinterpret_cast<uint64_t *>(red + CW * 16 * NC);
    uint64_t *empty = full + kMaxStages;
    int *last_flag = reinterpret_cast<int *>(empty + kMaxStages);
    volatile int *abort = last_flag + 1;

    // This CTA's K slice and its index among the slice's CTAs.
    const long long grid = gridDim.x / p.nslice;
    const long long ks = blockIdx.x / grid, cta = blockIdx.x - ks * grid;
    const int kbase = (int)(ks * p.spr);
    const long long u0 = unit_start(p, cta * p.units / grid);
    const long long u1 = unit_start(p, (cta + 1) * p.units / grid);

    pdl_trigger();
    if (threadIdx.x == 0) {
        for (int i = 0; i < p.nstage; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], CW);
        }
        fence_mbar_init();
        *abort = 0;
    }
    __syncthreads();

    if (warp == CW) {
        if (lane == 0) produce(p, ring, full, empty, abort, u0, u1, kbase);
        return;
    }

    pdl_wait();
    // Only the warp-steps this CTA's range touches (contiguous mod spr).
    const bool all_ws = u1 - u0 >= p.spr;
    stage_digits<FMT, CW, NT>(p, xd, fx, all_ws ? 0 : (int)(u0 % p.spr),
                              all_ws ? (int)p.spr : (int)(u1 - u0), kbase);
    float res[NT][4];
    int slot = 0, phase = 0;
    for (long long u = u0; u < u1;) {
        const long long blk = u / p.spr;
        const long long run_end = min(u1, (blk + 1) * p.spr);
        int lblk;
        const int sgi = block_segment(p, blk, &lblk);
        const int n_seg = p.N[sgi];
        const int row0 = lblk * kBlockRows + tile * kTileRows;
        const bool active = row0 < n_seg;
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) res[nt][i] = 0.f;
        while (u < run_end) {
            const int run = (int)min((long long)kRun, run_end - u);
            const int step0 = (int)(u - blk * p.spr);
            const bool ready = !*abort && mbar_wait(&full[slot], phase, p.err, abort);
            if (ready && active) {
                const unsigned char *sl = ring + slot * kSlotBytes;
                const unsigned char *base = sl + (tile * kTileRows + g) * kPitch + t * 16;
                const float *ssl = reinterpret_cast<const float *>(sl + kCodeBytes) +
                                   (tile * kTileRows + g) * kScaleBox;
                if (run == kRun)
                    imma_stage<FMT, NT, SPLIT, true>(p, base, ssl, step0, run, h,
                                                     reinterpret_cast<const unsigned char *>(xd),
                                                     fx, g, t, kbase, res);
                else
                    imma_stage<FMT, NT, SPLIT, false>(p, base, ssl, step0, run, h,
                                                      reinterpret_cast<const unsigned char *>(xd),
                                                      fx, g, t, kbase, res);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            u += run;
            if (++slot == p.nstage) {
                slot = 0;
                phase ^= 1;
            }
        }

        // ---- end of this CTA's run over the block: every warp's column
        // sums meet in shared memory; output (m, row) = sum over the SPLIT
        // warps of the tile, then over the three digit columns, in order.
        float *rw = red + warp * 16 * NC;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const int c0 = 8 * nt + 2 * t;
            rw[g * NC + c0] = res[nt][0];
            rw[g * NC + c0 + 1] = res[nt][1];
            rw[(g + 8) * NC + c0] = res[nt][2];
            rw[(g + 8) * NC + c0 + 1] = res[nt][3];
        }
        consumer_sync<CW>();
        // CTAs sharing the block: `shared` per K slice (the same in every
        // slice); partial slots in slice order, then CTA order.
        const long long first = owner(p, blk * p.spr, grid);
        const long long last = owner(p, (blk + 1) * p.spr - 1, grid);
        const int shared = (int)(last - first + 1);
        const int count = shared * p.nslice;
        float *dst;
        long long ld, rbase;
        if (count == 1) {
            dst = p.out[sgi];
            ld = n_seg;
            rbase = (long long)lblk * kBlockRows;
        } else {
            dst = p.partials + (ks * shared + (cta - first)) * (long long)Mc * p.prow;
            ld = p.prow;
            rbase = blk * kBlockRows;
        }
        for (int i = threadIdx.x; i < Mc * kBlockRows; i += CW * 32) {
            const int m = i / kBlockRows, tr = i - m * kBlockRows;
            const int tl = tr >> 4, r = tr & 15;
            if (lblk * kBlockRows + tr >= n_seg) continue;
            float v = 0.f;
#pragma unroll
            for (int hh = 0; hh < SPLIT; hh++) {
                const float *q = red + ((hh * kTiles + tl) * 16 + r) * NC + 3 * m;
                v += (q[0] + q[1]) + q[2];
            }
            dst[m * ld + rbase + tr] = v;
        }
        if (count > 1) {
            // The barrier orders every thread's partial stores before thread
            // 0's fence and ticket (release); thread 0's second fence orders
            // the ticket before the barrier that lets the last CTA read the
            // other CTAs' partials (acquire).
            consumer_sync<CW>();
            if (threadIdx.x == 0) {
                __threadfence();
                const unsigned ticket = atomicAdd(&p.tickets[blk], 1u);
                *last_flag = ticket == (unsigned)(count - 1);
                __threadfence();
            }
            consumer_sync<CW>();
            const bool is_last = *last_flag;
            if (is_last) {
                const int rows_here = min(kBlockRows, n_seg - lblk * kBlockRows);
                for (int i = threadIdx.x; i < Mc * rows_here; i += CW * 32) {
                    const int c = i / rows_here, r = i % rows_here;
                    const float *src = p.partials + (long long)c * p.prow + blk * kBlockRows + r;
                    const long long slot_stride = (long long)Mc * p.prow;
                    float v = 0.f;
#pragma unroll 8
                    for (int sl = 0; sl < count; sl++) v += __ldcg(src + sl * slot_stride);
                    p.out[sgi][(long long)c * n_seg + lblk * kBlockRows + r] = v;
                }
                if (threadIdx.x == 0) p.tickets[blk] = 0u;
            }
        }
        // red and last_flag are rewritten for the next block.
        consumer_sync<CW>();
    }
}

struct TmaPlan {
    bool ok = false;
    int nstage = 0, S = 0, ring_bytes = 0, grid = 0, slots = 0, unscale_floats = 0, split = 1;
    long long spr = 0, total = 0, n_blocks = 0, units = 0;
    size_t smem = 0;
    // Integer consumer (qgemv_imma), when its activation digits fit.
    bool imma = false;
    int int_nt = 0, int_nstage = 0, Sn = 0, xd_off = 0, fx_off = 0, red_off = 0;
    size_t int_smem = 0;
    // K slices of the integer consumer (1: whole rows with the plan above).
    int int_nslice = 1, int_grid = 0, int_slots = 0;
    long long int_sps = 0;
};

constexpr int kImmaSplit = 2;  // consumer warps per 16-row tile in qgemv_imma

int imma_nt(size_t m) {
    const int nt = (int)((3 * m + 7) / 8);
    return nt <= 3 ? nt : 6;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

constexpr int kMaxSlices = 64;  // at least two CTAs per slice

// Shared layout of qgemv_imma: ring, digit planes [3M][Sn], factors
// [steps][8 NT], block sums [warps][16][8 NT], barriers and flags. The
// digits of whole rows when they fit beside at least two stages; otherwise,
// for at most 8 activation rows, the row is cut into 2, 4, .. 64 K slices
// (each CTA stages the digits of one slice only, beside at least three
// stages) and every slice's CTAs add partial sums. With more rows the slices
// get so short that the per-block partial sums cost more than the weight
// stream (70B-shaped batch-16 step 92 -> 130 ms when they were allowed).
void plan_imma(TmaPlan &pl, int fmt, size_t m) {
    if (m > 16) return;
    const int nt = imma_nt(m);
    const long long wsb = fmt == 0 ? 128 : 64;
    const size_t red = (size_t)kTiles * kImmaSplit * 16 * 8 * nt * 4;
    const int max_slices = nt <= 3 ? kMaxSlices : 1;
    for (int nslice = 1; nslice <= max_slices && pl.spr % nslice == 0; nslice *= 2) {
        const long long sps = pl.spr / nslice;
        const long long sn = (long long)align_up((size_t)(sps * wsb), 128) + 32;
        const size_t xd = (size_t)(3 * m) * (size_t)sn;
        const size_t fx = (size_t)sps * 8 * nt * 4;
        for (int ns = kMaxStages; ns >= (nslice == 1 ? 2 : kMinStages); ns--) {
            const size_t ring = (size_t)ns * kSlotBytes;
            const size_t fx_off = align_up(ring + xd, 16);
            const size_t red_off = align_up(fx_off + fx, 16);
            const size_t total = red_off + red + 2 * kMaxStages * 8 + 16;
            if (total > (size_t)kSmemLimit) continue;
            pl.imma = true;
            pl.int_nt = nt;
            pl.int_nstage = ns;
            pl.Sn = (int)sn;
            pl.xd_off = (int)ring;
            pl.fx_off = (int)fx_off;
            pl.red_off = (int)red_off;
            pl.int_smem = total;
            pl.int_nslice = nslice;
            pl.int_sps = sps;
            if (nslice > 1) {
                const long long g = std::min<long long>(kSmCount / nslice, pl.n_blocks * sps);
                pl.int_grid = (int)(g * nslice);
                pl.int_slots = (int)(nslice * std::min<long long>(g, (g + pl.n_blocks - 1) / pl.n_blocks + 1));
            }
            return;
        }
    }
}

int padded_stride(int fmt, long long units) {
    long long S = units;
    if (fmt == 0) {
        while (S % 8 != 4) S++;
    } else if (S % 2 == 0) {
        S++;
    }
    return (int)S;
}

// One matrix the kernel can stream: shape, format and alignment rules.
bool seg_ok(const QuantWeight &w) {
    const int kstep = w.format == 0 ? Fmt<0>::kStep : Fmt<1>::kStep;
    if (w.n == 0 || w.n % kTileRows != 0 || w.k == 0 || w.k % w.group != 0 ||
        w.group % kstep != 0 || w.row_bytes % kStepBytes != 0 || !aligned16(w.codes) ||
        !aligned16(w.scales) || w.groups % 4 != 0 || w.n > (1u << 24) || w.k > (1u << 24))
        return false;
    const size_t gsteps = w.group / kstep;
    return (gsteps & (gsteps - 1)) == 0;  // power of two: shifts in the hot loop
}

TmaPlan make_tma_plan(const QuantSeg *segs, int nseg, size_t m) {
    TmaPlan pl;
    if (nseg < 1 || nseg > kMaxSeg || m < 1 || m > 32) return pl;
    const QuantWeight &w0 = segs[0].w;
    long long n_blocks = 0;
    for (int i = 0; i < nseg; i++) {
        const QuantWeight &w = segs[i].w;
        if (!seg_ok(w) || w.k != w0.k || w.format != w0.format || w.group != w0.group) return pl;
        n_blocks += (long long)((w.n + kBlockRows - 1) / kBlockRows);
    }
    if (n_blocks > 64 * 1024) return pl;
    pl.n_blocks = n_blocks;
    pl.spr = (long long)(w0.row_bytes / kStepBytes);
    pl.total = n_blocks * pl.spr;
    // One CTA consumes only ~20 GB/s (its dequant + MMA issue rate), so
    // every matrix is spread over all SMs: units are single warp-steps and
    // CTAs that share a block add partial sums. Whole blocks per CTA (no
    // partial sums) only when they balance within 10% (e.g. a vocabulary
    // projection of ~1000 blocks).
    const long long per = (n_blocks + kSmCount - 1) / kSmCount;
    pl.split = (n_blocks >= kSmCount && per * kSmCount * 10 <= n_blocks * 11) ? 1 : (int)pl.spr;
    pl.units = n_blocks * pl.split;
    pl.grid = (int)std::min<long long>(pl.units, kSmCount);
    pl.S = padded_stride(w0.format, (long long)w0.k / 8);
    const size_t xbytes = (size_t)m * pl.S * 16 * 2;
    pl.unscale_floats = (int)(((long long)m * pl.spr + 1) / 2 * 2);
    const size_t fixed = (size_t)pl.unscale_floats * 4 + (size_t)kTiles * 32 * 16 * 4 +
                         2 * kMaxStages * 8 + 16;  // unscale, split sums, barriers, flags
    for (pl.nstage = kMaxStages; pl.nstage >= kMinStages; pl.nstage--) {
        pl.ring_bytes = pl.nstage * kSlotBytes;
        pl.smem = pl.ring_bytes + xbytes + fixed;
        if (pl.smem <= (size_t)kSmemLimit) break;
    }
    plan_imma(pl, w0.format, m);
    if (pl.nstage < kMinStages && !pl.imma) return pl;
    // Partial slots: the most CTAs that share one block.
    pl.slots = pl.split == 1
                   ? 1
                   : (int)std::min<long long>(pl.grid, (pl.grid + n_blocks - 1) / n_blocks + 1);
    if (pl.imma && pl.int_nslice == 1) {
        pl.int_grid = pl.grid;
        pl.int_slots = pl.slots;
    }
    if (pl.imma) pl.slots = std::max(pl.slots, pl.int_slots);
    pl.ok = true;
    return pl;
}

// Tensor maps of a weight, encoded once and cached by everything they encode.
struct MapKey {
    const void *codes, *scales;
    size_t n, row_bytes, groups;
    bool operator==(const MapKey &o) const {
        return codes == o.codes && scales == o.scales && n == o.n && row_bytes == o.row_bytes &&
               groups == o.groups;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey &k) const {
        size_t h = std::hash<const void *>()(k.codes) * 31 + std::hash<const void *>()(k.scales);
        return h * 131 + k.n * 7 + k.row_bytes * 3 + k.groups;
    }
};
struct MapPair {
    CUtensorMap codes, scales;
};

bool tensor_maps(const QuantWeight &w, MapPair *out) {
    static std::mutex mu;
    static std::unordered_map<MapKey, MapPair, MapKeyHash> cache;
    const MapKey key{w.codes, w.scales, w.n, w.row_bytes, w.groups};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return true;
    }
    MapPair mp;
    if (!encode_tensor_map_2d(&mp.codes, CU_TENSOR_MAP_DATA_TYPE_UINT64, w.codes, w.row_bytes / 8,
                              w.n, w.row_bytes, kPitch / 8, kBlockRows) ||
        !encode_tensor_map_2d(&mp.scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, w.scales, w.groups, w.n,
                              w.groups * 4, kScaleBox, kBlockRows))
        return false;
    if (cache.size() > 8192) cache.clear();
    cache.emplace(key, mp);
    *out = mp;
    return true;
}

// Kernel arguments shared by both consumers (tensor maps cached per weight).
bool fill_args(TmaArgs &a, int fmt, const float *x, const float *x2, size_t m,
               const QuantSeg *segs, int nseg, const TmaPlan &pl, void *ws, uint32_t *err) {
    long long blocks = 0;
    for (int i = 0; i < nseg; i++) {
        MapPair maps;
        if (!tensor_maps(segs[i].w, &maps)) return false;
        a.codes_map[i] = maps.codes;
        a.scales_map[i] = maps.scales;
        a.out[i] = segs[i].out;
        a.N[i] = (int)segs[i].w.n;
        blocks += (long long)((segs[i].w.n + kBlockRows - 1) / kBlockRows);
        a.blk_end[i] = (int)blocks;
    }
    const QuantWeight &w = segs[0].w;
    const int kstep = fmt == 0 ? Fmt<0>::kStep : Fmt<1>::kStep;
    a.nseg = nseg;
    a.x = x;
    a.x2 = x2;
    a.M = (int)m;
    a.K = (int)w.k;
    a.groups = (int)w.groups;
    a.gs_shift = 0;
    while ((1u << a.gs_shift) < w.group / kstep) a.gs_shift++;
    a.row_bytes = (long long)w.row_bytes;
    a.spr = pl.spr;
    a.total = pl.total;
    a.units = pl.units;
    a.split = pl.split;
    a.prow = pl.n_blocks * kBlockRows;
    a.nstage = pl.nstage;
    a.S = pl.S;
    a.ring_bytes = pl.ring_bytes;
    a.unscale_floats = pl.unscale_floats;
    a.err = err;
    a.tickets = static_cast<unsigned *>(ws);
    a.partials = reinterpret_cast<float *>(static_cast<char *>(ws) + 64 * 1024 * sizeof(unsigned));
    return true;
}

template <int FMT, int NT, int SPLIT>
cudaError_t launch_tma(cudaStream_t s, const float *x, const float *x2, size_t m,
                       const QuantSeg *segs, int nseg, const TmaPlan &pl, void *ws,
                       uint32_t *err) {
    TmaArgs a{};
    if (!fill_args(a, FMT, x, x2, m, segs, nseg, pl, ws, err)) return cudaErrorInvalidValue;
    static std::atomic<uint64_t> smem_set{0};
    set_smem_limit_once(qgemv_tma<FMT, NT, SPLIT>, kSmemLimit, &smem_set);
    launch_k(qgemv_tma<FMT, NT, SPLIT>, pl.grid, (kTiles * SPLIT + 1) * 32, pl.smem, s, a);
    count_launch();
    return cudaGetLastError();
}

template <int FMT, int NT>
cudaError_t launch_imma(cudaStream_t s, const float *x, const float *x2, size_t m,
                        const QuantSeg *segs, int nseg, const TmaPlan &pl, void *ws,
                        uint32_t *err) {
    TmaArgs a{};
    if (!fill_args(a, FMT, x, x2, m, segs, nseg, pl, ws, err)) return cudaErrorInvalidValue;
    a.nstage = pl.int_nstage;
    a.Sn = pl.Sn;
    a.ncol = (int)(3 * m);
    a.xd_off = pl.xd_off;
    a.fx_off = pl.fx_off;
    a.red_off = pl.red_off;
    a.nslice = pl.int_nslice;
    if (pl.int_nslice > 1) {
        // One slice's geometry: warp-steps as units.
        a.spr = pl.int_sps;
        a.total = pl.n_blocks * pl.int_sps;
        a.units = a.total;
        a.split = (int)pl.int_sps;
    }
    static std::atomic<uint64_t> smem_set{0};
    set_smem_limit_once(qgemv_imma<FMT, NT, kImmaSplit>, kSmemLimit, &smem_set);
    launch_k(qgemv_imma<FMT, NT, kImmaSplit>, pl.int_grid, (kTiles * kImmaSplit + 1) * 32,
             pl.int_smem, s, a);
    count_launch();
    return cudaGetLastError();
}

template <int FMT>
cudaError_t launch_imma_nt(cudaStream_t s, const float *x, const float *x2, size_t m,
                           const QuantSeg *segs, int nseg, const TmaPlan &pl, void *ws,
                           uint32_t *err) {
    switch (pl.int_nt) {
        case 1: return launch_imma<FMT, 1>(s, x, x2, m, segs, nseg, pl, ws, err);
        case 2: return launch_imma<FMT, 2>(s, x, x2, m, segs, nseg, pl, ws, err);
        case 3: return launch_imma<FMT, 3>(s, x, x2, m, segs, nseg, pl, ws, err);
        default: return launch_imma<FMT, 6>(s, x, x2, m, segs, nseg, pl, ws, err);
    }
}

}  // namespace

bool qgemv_tma_group_supported(const QuantSeg *segs, int nseg, size_t m) {
    return make_tma_plan(segs, nseg, m).ok;
}

size_t qgemv_tma_group_workspace_bytes(const QuantSeg *segs, int nseg, size_t m) {
    TmaPlan pl = make_tma_plan(segs, nseg, m);
    if (!pl.ok) return (size_t)-1;
    return 64 * 1024 * sizeof(unsigned) +
           (pl.slots > 1 ? (size_t)pl.slots * m * pl.n_blocks * kBlockRows * 4 : 0);
}

bool qgemv_tma_supported(const QuantWeight &w, size_t m) {
    const QuantSeg seg{w, nullptr};
    return qgemv_tma_group_supported(&seg, 1, m);
}

size_t qgemv_tma_workspace_bytes(const QuantWeight &w, size_t m) {
    const QuantSeg seg{w, nullptr};
    return qgemv_tma_group_workspace_bytes(&seg, 1, m);
}

bool qgemv_tma_x_aligned(const float *x) { return aligned16(x); }

cudaError_t qgemv_tma_group(cudaStream_t s, const float *x, const float *x2, size_t m,
                            const QuantSeg *segs, int nseg, void *workspace, uint32_t *err) {
    // One or two activation rows: whole tiles per CTA (no split-K tail).
    if (m <= 2 && aligned16(x) && (!x2 || aligned16(x2)) && qgemv_lane_supported(segs, nseg, m))
        return qgemv_lane_group(s, x, x2, m, segs, nseg, err);
    TmaPlan pl = make_tma_plan(segs, nseg, m);
    if (!pl.ok || !aligned16(x) || (x2 && !aligned16(x2))) return cudaErrorInvalidValue;
    // The integer consumer wherever its activation digits fit in shared
    // memory; the f16 consumer otherwise.
    if (pl.imma)
        return segs[0].w.format == 0
                   ? launch_imma_nt<0>(s, x, x2, m, segs, nseg, pl, workspace, err)
                   : launch_imma_nt<1>(s, x, x2, m, segs, nseg, pl, workspace, err);
    const int nt = m <= 8 ? 1 : (m <= 16 ? 2 : 4);
    // One column tile: two warps per 16-row tile (17 warps, 96 registers
    // each, no spills); more columns need the registers of one warp per tile.
    if (segs[0].w.format == 0)
        return nt == 1 ? launch_tma<0, 1, 2>(s, x, x2, m, segs, nseg, pl, workspace, err)
             : nt == 2 ? launch_tma<0, 2, 1>(s, x, x2, m, segs, nseg, pl, workspace, err)
                       : launch_tma<0, 4, 1>(s, x, x2, m, segs, nseg, pl, workspace, err);
    return nt == 1 ? launch_tma<1, 1, 2>(s, x, x2, m, segs, nseg, pl, workspace, err)
         : nt == 2 ? launch_tma<1, 2, 1>(s, x, x2, m, segs, nseg, pl, workspace, err)
                   : launch_tma<1, 4, 1>(s, x, x2, m, segs, nseg, pl, workspace, err);
}

cudaError_t qgemv_tma(cudaStream_t s, const float *x, size_t m, const QuantWeight &w, float *out,
                      void *workspace, uint32_t *err) {
    const QuantSeg seg{w, out};
    return qgemv_tma_group(s, x, nullptr, m, &seg, 1, workspace, err);
}

}  // namespace k
}  // namespace slc
