// Group-dequant-fused quantized MatMulNT: out[m, n] = sum_k x[m, k] * w[n, k]
// with w[n, k] = code[n, k] * scale[n, k / group] (symmetric grouped INT4 /
// INT8, the sl-precision format described in include/starlight_cuda.h).
// Parity target: dequantize, then backend-cpu's f32 matmul_nt
// (crates/backends/backend-cpu/src/reference/matmul.rs:29-59).
//
// Decode (M <= 32) is HBM-bound on the payload: algorithmic bytes per launch
//   N * row_bytes + 4 * N * K / group + 4 * M * (K + N).
//
// Fast path (tensor cores, mma.sync.m16n8k16 f16 -> f32):
//  * Weights are the A operand (16 rows per warp tile), the activations the
//    B operand (8 batch columns per n-tile, up to 4 n-tiles). Each lane
//    streams 16-byte chunks of two weight rows with L1-bypassing 128-bit
//    loads, several warp-steps ahead, straight into registers.
//  * Codes become exact small integers in f16 without a multiply: INT4 nibble
//    pairs are masked into the mantissa of 1024.0 (one shift + one LOP3 per
//    two codes, giving 1032 + code), INT8 bytes are placed under 0x64 with a
//    byte permute (1152 + code); one packed f16 subtraction per two codes
//    removes the bias exactly. (Folding the bias into a per-group correction
//    instead would make the MMA accumulate values ~100x larger than the
//    result and amplify its accumulation rounding by the same factor.)
//  * Activations are split into f16 hi + lo (22 significant bits) after a
//    per-CTA, per-column power-of-two prescale that keeps them in f16 range;
//    hi and lo products accumulate into the same f32 accumulator.
//  * Per group: acc * scale[n, group], accumulated in f32 registers. Column
//    prescales are undone exactly at the end.
//  * Split-K across CTAs when N alone cannot fill 148 SMs; partial sums go to
//    the workspace and the last CTA of each row block (atomic ticket, no
//    waiting) adds them in ascending split order, so results are
//    deterministic.
// Any other shape (ragged groups, unaligned rows, N % 16 != 0) takes a
// correct SIMT path with the reference's exact dequantization.
#include <math.h>

#include <utility>

#include "common.cuh"
#include "gemv_common.cuh"
#include "kernels.h"

namespace slc {
namespace k {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRowsPerCta = 16 * kWarps;
constexpr int kPrefetch = 4;
constexpr int kSmemBudget = 160 * 1024;

struct GemvArgs {
    const float *x;         // [M, K]
    const uint8_t *codes;   // [N, row_bytes]
    const float *scales;    // [N, groups]
    float *out;             // [M, N]
    float *partials;        // [ksplit, M, N]
    unsigned *tickets;      // [row_blocks]
    int M, N, K, group, groups, ksplit, slice_k;  // slice_k: k per CTA slice
    int units_stride;       // S: 16-byte units per smem row (padded)
    size_t row_bytes;
};

template <int FMT, int NT>
__global__ void __launch_bounds__(kThreads) qgemv_mma(GemvArgs p) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    constexpr int KSTEP = Fmt<FMT>::kStep;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int row_block = blockIdx.x, kidx = blockIdx.y;
    const int kb0 = kidx * p.slice_k;
    const int klen = min(p.slice_k, p.K - kb0);
    const int nsteps = klen / KSTEP;
    const int group_steps = p.group / KSTEP;
    const int S = p.units_stride;
    const int Mc = p.M;  // real columns (<= 8 * NT)

    __half *xh = reinterpret_cast<__half *>(smem_raw);
    __half *xl = xh + (size_t)Mc * S * 8;
    float *unscale = reinterpret_cast<float *>(xl + (size_t)Mc * S * 8);  // [Mc]
    __shared__ bool is_last;

    // ---- stage activations: warp w handles columns w, w + 8, ...
    for (int col = warp; col < Mc; col += kWarps) {
        const float *xr = p.x + (size_t)col * p.K + kb0;
        float mx = 0.f;
        for (int k = lane; k < klen; k += 32) mx = fmaxf(mx, fabsf(xr[k]));
        mx = warp_max(mx);
        int e = 0;
        if (mx > 0.f) {
            int ex;
            frexpf(mx, &ex);
            e = 14 - ex;
            e = e > 126 ? 126 : (e < -126 ? -126 : e);
        }
        const float up = ldexpf(1.0f, e);
        if (lane == 0) unscale[col] = ldexpf(1.0f, -e);
        for (int k = lane; k < klen; k += 32) {
            float v = xr[k] * up;
            __half hi = __float2half_rn(v);
            __half lo = __float2half_rn(v - __half2float(hi));
            int slot = stage_slot<FMT>(k, S, col);
            xh[slot] = hi;
            xl[slot] = lo;
        }
    }
    __syncthreads();

    const int row0 = row_block * kRowsPerCta + warp * 16;
    float res[NT][4];
#pragma unroll
    for (int j = 0; j < NT; j++)
#pragma unroll
        for (int i = 0; i < 4; i++) res[j][i] = 0.f;

    if (row0 < p.N) {
        const uint8_t *rg = p.codes + (size_t)(row0 + g) * p.row_bytes +
                            (size_t)kb0 * (FMT == 0 ? 1 : 2) / 2 + t * 16;
        const uint8_t *rg8 = rg + 8 * p.row_bytes;
        const size_t step_bytes = FMT == 0 ? KSTEP / 2 : KSTEP;
        const float *sg = p.scales + (size_t)(row0 + g) * p.groups + kb0 / p.group;
        const float *sg8 = sg + 8 * (size_t)p.groups;

        uint4 buf_g[kPrefetch], buf_g8[kPrefetch];
#pragma unroll
        for (int j = 0; j < kPrefetch; j++) {
            if (j < nsteps) {
                buf_g[j] = ld_stream_u4(rg + j * step_bytes);
                buf_g8[j] = ld_stream_u4(rg8 + j * step_bytes);
            }
        }
        float acc[NT][4];
#pragma unroll
        for (int j = 0; j < NT; j++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc[j][i] = 0.f;

        for (int base = 0; base < nsteps; base += kPrefetch) {
#pragma unroll
            for (int j = 0; j < kPrefetch; j++) {
                const int ws = base + j;
                if (ws < nsteps) {
                    const uint4 wg = buf_g[j], wg8 = buf_g8[j];
                    if (ws + kPrefetch < nsteps) {
                        buf_g[j] = ld_stream_u4(rg + (ws + kPrefetch) * step_bytes);
                        buf_g8[j] = ld_stream_u4(rg8 + (ws + kPrefetch) * step_bytes);
                    }
                    const uint32_t wa[4] = {wg.x, wg.y, wg.z, wg.w};
                    const uint32_t wb[4] = {wg8.x, wg8.y, wg8.z, wg8.w};
                    if (FMT == 0) {
#pragma unroll
                        for (int q = 0; q < 4; q++) {
                            uint32_t pa[4], pb[4];
#pragma unroll
                            for (int i = 0; i < 4; i++) {
                                pa[i] = hsub2(lop3_and_xor(wa[q] >> (4 * i), 0x000F000Fu, 0x64086408u),
                                              0x64086408u);
                                pb[i] = hsub2(lop3_and_xor(wb[q] >> (4 * i), 0x000F000Fu, 0x64086408u),
                                              0x64086408u);
                            }
                            const int unit = ws * 16 + 4 * t + q;
                            const int phys = unit ^ ((unit >> 3) & 1);
#pragma unroll
                            for (int jn = 0; jn < NT; jn++) {
                                const int col = g + 8 * jn;
                                uint4 bh = make_uint4(0, 0, 0, 0), bl = make_uint4(0, 0, 0, 0);
                                if (col < Mc) {
                                    bh = lds128(xh + ((size_t)col * S + phys) * 8);
                                    bl = lds128(xl + ((size_t)col * S + phys) * 8);
                                }
                                mma16816(acc[jn], pa[0], pb[0], pa[1], pb[1], bh.x, bh.y);
                                mma16816(acc[jn], pa[0], pb[0], pa[1], pb[1], bl.x, bl.y);
                                mma16816(acc[jn], pa[2], pb[2], pa[3], pb[3], bh.z, bh.w);
                                mma16816(acc[jn], pa[2], pb[2], pa[3], pb[3], bl.z, bl.w);
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
                                uint4 bh = make_uint4(0, 0, 0, 0), bl = make_uint4(0, 0, 0, 0);
                                if (col < Mc) {
                                    bh = lds128(xh + ((size_t)col * S + unit) * 8);
                                    bl = lds128(xl + ((size_t)col * S + unit) * 8);
                                }
                                mma16816(acc[jn], lo_a[0], lo_b[0], hi_a[0], hi_b[0], bh.x, bh.y);
                                mma16816(acc[jn], lo_a[0], lo_b[0], hi_a[0], hi_b[0], bl.x, bl.y);
                                mma16816(acc[jn], lo_a[1], lo_b[1], hi_a[1], hi_b[1], bh.z, bh.w);
                                mma16816(acc[jn], lo_a[1], lo_b[1], hi_a[1], hi_b[1], bl.z, bl.w);
                            }
                        }
                    }
                    // Group epilogue: apply the group scale.
                    if ((ws + 1) % group_steps == 0) {
                        const int gi = ws / group_steps;
                        const float s0 = __ldg(sg + gi), s1 = __ldg(sg8 + gi);
#pragma unroll
                        for (int jn = 0; jn < NT; jn++) {
                            res[jn][0] = fmaf(s0, acc[jn][0], res[jn][0]);
                            res[jn][1] = fmaf(s0, acc[jn][1], res[jn][1]);
                            res[jn][2] = fmaf(s1, acc[jn][2], res[jn][2]);
                            res[jn][3] = fmaf(s1, acc[jn][3], res[jn][3]);
#pragma unroll
                            for (int i = 0; i < 4; i++) acc[jn][i] = 0.f;
                        }
                    }
                }
            }
        }
    }

    // ---- write: directly (one split) or via partials + last-CTA reduction.
    const int r_g = row0 + g, r_g8 = row0 + g + 8;
    if (p.ksplit == 1) {
        if (row0 < p.N) {
#pragma unroll
            for (int jn = 0; jn < NT; jn++) {
                const int c0 = 2 * t + 8 * jn, c1 = c0 + 1;
                if (c0 < Mc) {
                    p.out[(size_t)c0 * p.N + r_g] = res[jn][0] * unscale[c0];
                    p.out[(size_t)c0 * p.N + r_g8] = res[jn][2] * unscale[c0];
                }
                if (c1 < Mc) {
                    p.out[(size_t)c1 * p.N + r_g] = res[jn][1] * unscale[c1];
                    p.out[(size_t)c1 * p.N + r_g8] = res[jn][3] * unscale[c1];
                }
            }
        }
        return;
    }
    float *part = p.partials + (size_t)kidx * p.M * p.N;
    if (row0 < p.N) {
#pragma unroll
        for (int jn = 0; jn < NT; jn++) {
            const int c0 = 2 * t + 8 * jn, c1 = c0 + 1;
            if (c0 < Mc) {
                part[(size_t)c0 * p.N + r_g] = res[jn][0] * unscale[c0];
                part[(size_t)c0 * p.N + r_g8] = res[jn][2] * unscale[c0];
            }
            if (c1 < Mc) {
                part[(size_t)c1 * p.N + r_g] = res[jn][1] * unscale[c1];
                part[(size_t)c1 * p.N + r_g8] = res[jn][3] * unscale[c1];
            }
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned ticket = atomicAdd(&p.tickets[row_block], 1u);
        is_last = (ticket == (unsigned)p.ksplit - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const int rows_here = min(kRowsPerCta, p.N - row_block * kRowsPerCta);
    for (int i = threadIdx.x; i < Mc * rows_here; i += kThreads) {
        const int c = i / rows_here, r = row_block * kRowsPerCta + i % rows_here;
        float s = 0.f;
        for (int ks = 0; ks < p.ksplit; ks++)
            s += ld_cg(p.partials + ((size_t)ks * p.M + c) * p.N + r);
        p.out[(size_t)c * p.N + r] = s;
    }
    if (threadIdx.x == 0) p.tickets[row_block] = 0;  // ready for the next launch
}

// SIMT fallback for any shape: one warp per output row n, all M columns.
// Dequantization is the reference's exact (float)code * scale.
template <int FMT>
__global__ void __launch_bounds__(256) qgemv_simple(const float *__restrict__ x, int M, int K,
                                                    const uint8_t *__restrict__ codes,
                                                    size_t row_bytes,
                                                    const float *__restrict__ scales, int group,
                                                    int groups, float *__restrict__ out, int N) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * 8;
    for (int n = blockIdx.x * 8 + (threadIdx.x >> 5); n < N; n += warps) {
        const uint8_t *cr = codes + (size_t)n * row_bytes;
        const float *sr = scales + (size_t)n * groups;
        for (int m0 = 0; m0 < M; m0 += 8) {
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int k = lane; k < K; k += 32) {
                int code;
                if (FMT == 0) {
                    uint8_t b = cr[k >> 1];
                    int nib = (k & 1) ? (b >> 4) : (b & 15);
                    code = nib >= 8 ? nib - 16 : nib;
                } else {
                    code = (int)(int8_t)cr[k];
                }
                const float w = __fmul_rn((float)code, sr[k / group]);
#pragma unroll
                for (int i = 0; i < 8; i++)
                    if (m0 + i < M) acc[i] = fmaf(x[(size_t)(m0 + i) * K + k], w, acc[i]);
            }
#pragma unroll
            for (int i = 0; i < 8; i++) {
                float v = warp_sum(acc[i]);
                if (lane == 0 && m0 + i < M) out[(size_t)(m0 + i) * N + n] = v;
            }
        }
    }
}

// ---- quantization (sl-precision format) ------------------------------------

__global__ void __launch_bounds__(256) quant_scales(const float *__restrict__ w, size_t n,
                                                    size_t k, size_t group, size_t groups,
                                                    float qmax, float *__restrict__ scales) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    size_t total = n * groups, warps = (size_t)gridDim.x * 8;
    for (size_t i = (size_t)blockIdx.x * 8 + (threadIdx.x >> 5); i < total; i += warps) {
        size_t row = i / groups, gi = i - row * groups;
        size_t begin = gi * group, end = begin + group < k ? begin + group : k;
        float mx = 0.f;
        for (size_t c = begin + lane; c < end; c += 32) mx = fmaxf(mx, fabsf(w[row * k + c]));
        mx = warp_max(mx);
        if (lane == 0) scales[i] = __fdiv_rn(mx, qmax);
    }
}

__device__ __forceinline__ int quant_code(float v, float scale, float qmax) {
    if (scale == 0.f) return 0;
    float q = roundf(__fdiv_rn(v, scale));
    q = fminf(fmaxf(q, -qmax), qmax);
    return (int)q;
}

__global__ void __launch_bounds__(256) quant_codes(const float *__restrict__ w, size_t n,
                                                   size_t k, size_t group, size_t groups,
                                                   size_t row_bytes, int format, float qmax,
                                                   const float *__restrict__ scales,
                                                   uint8_t *__restrict__ codes) {
    pdl_trigger();
    pdl_wait();
    size_t total = n * row_bytes, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        size_t row = i / row_bytes, b = i - row * row_bytes;
        const float *wr = w + row * k;
        const float *sr = scales + row * groups;
        if (format == 1) {
            codes[i] = (uint8_t)(int8_t)quant_code(wr[b], sr[b / group], qmax);
        } else {
            size_t c0 = 2 * b, c1 = 2 * b + 1;
            int lo = quant_code(wr[c0], sr[c0 / group], qmax);
            int hi = c1 < k ? quant_code(wr[c1], sr[c1 / group], qmax) : 0;
            codes[i] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
        }
    }
}

__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t *__restrict__ codes,
                                                      const float *__restrict__ scales,
                                                      size_t n, size_t k, size_t group,
                                                      size_t groups, size_t row_bytes,
                                                      int format, float *__restrict__ out) {
    pdl_trigger();
    pdl_wait();
    size_t total = n * k, stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        size_t row = i / k, c = i - row * k;
        int code;
        if (format == 1) {
            code = (int)(int8_t)codes[row * row_bytes + c];
        } else {
            uint8_t b = codes[row * row_bytes + c / 2];
            int nib = (c & 1) ? (b >> 4) : (b & 15);
            code = nib >= 8 ? nib - 16 : nib;
        }
        out[i] = __fmul_rn((float)code, scales[row * groups + c / group]);
    }
}

struct Plan {
    bool fast;
    int nt, ksplit, slice_k, S, row_blocks;
    size_t smem;
};

Plan make_plan(const QuantWeight &w, size_t m) {
    Plan pl{};
    const int kstep = w.format == 0 ? Fmt<0>::kStep : Fmt<1>::kStep;
    pl.fast = m >= 1 && m <= 32 && w.n % 16 == 0 && w.k % w.group == 0 &&
              w.group % kstep == 0 && w.row_bytes % 16 == 0 &&
              (reinterpret_cast<uintptr_t>(w.codes) & 15u) == 0 && w.n <= (1u << 30) &&
              w.k <= (1u << 30);
    if (!pl.fast) return pl;
    pl.nt = m <= 8 ? 1 : (m <= 16 ? 2 : 4);
    pl.row_blocks = (int)((w.n + kRowsPerCta - 1) / kRowsPerCta);
    const int groups = (int)w.groups;
    int want = (2 * kSmCount + pl.row_blocks - 1) / pl.row_blocks;
    if (want < 1) want = 1;
    if (want > groups) want = groups;
    int groups_per_slice = (groups + want - 1) / want;
    // Keep the staged activations within the shared-memory budget.
    auto smem_for = [&](int gps) {
        int slice_k = gps * (int)w.group;
        int units = slice_k / 8;
        int S = units;
        if (w.format == 0) {
            while (S % 8 != 2) S++;
        } else {
            if (S % 2 == 0) S++;
        }
        return std::make_pair(S, (size_t)m * S * 16 * 2 + (size_t)m * 4);
    };
    while (groups_per_slice > 1 && smem_for(groups_per_slice).second > (size_t)kSmemBudget)
        groups_per_slice = (groups_per_slice + 1) / 2;
    auto sz = smem_for(groups_per_slice);
    if (sz.second > (size_t)kSmemBudget) {
        pl.fast = false;
        return pl;
    }
    pl.slice_k = groups_per_slice * (int)w.group;
    pl.ksplit = (groups + groups_per_slice - 1) / groups_per_slice;
    pl.S = sz.first;
    pl.smem = sz.second;
    return pl;
}

template <int FMT, int NT>
cudaError_t launch_fast(cudaStream_t s, const float *x, size_t m, const QuantWeight &w,
                        float *out, const Plan &pl, void *ws) {
    GemvArgs a{};
    a.x = x;
    a.codes = w.codes;
    a.scales = w.scales;
    a.out = out;
    a.M = (int)m;
    a.N = (int)w.n;
    a.K = (int)w.k;
    a.group = (int)w.group;
    a.groups = (int)w.groups;
    a.ksplit = pl.ksplit;
    a.slice_k = pl.slice_k;
    a.units_stride = pl.S;
    a.row_bytes = w.row_bytes;
    if (pl.ksplit > 1) {
        a.tickets = static_cast<unsigned *>(ws);
        a.partials = reinterpret_cast<float *>(static_cast<char *>(ws) + 64 * 1024 * sizeof(unsigned));
    }
    static std::atomic<uint64_t> smem_set{0};
    set_smem_limit_once(qgemv_mma<FMT, NT>, kSmemBudget, &smem_set);
    dim3 grid((unsigned)pl.row_blocks, (unsigned)pl.ksplit);
    launch_k(qgemv_mma<FMT, NT>, grid, kThreads, pl.smem, s, a);
    count_launch();
    return cudaGetLastError();
}

}  // namespace

// The first 64 Ki unsigned of the workspace are the split-K tickets (zeroed
// once when the device is created and reset by every last CTA); the partial
// sums follow.
namespace {
size_t mma_workspace_bytes(const QuantWeight &w, size_t m) {
    Plan pl = make_plan(w, m);
    if (!pl.fast || pl.ksplit <= 1) return 0;
    if (pl.row_blocks > 64 * 1024) return (size_t)-1;
    return 64 * 1024 * sizeof(unsigned) + (size_t)pl.ksplit * m * w.n * sizeof(float);
}
}  // namespace

size_t qmatmul_workspace_bytes(const QuantWeight &w, size_t m) {
    if (m > 64) return 0;
    size_t most = 0;
    for (size_t m0 = 0; m0 < m; m0 += 32) {
        const size_t mb = m - m0 < 32 ? m - m0 : 32;
        size_t b = qgemv_tma_supported(w, mb) ? qgemv_tma_workspace_bytes(w, mb)
                                              : mma_workspace_bytes(w, mb);
        most = b > most ? b : most;
    }
    return most;
}

cudaError_t qmatmul(cudaStream_t s, const float *x, size_t m, const QuantWeight &w, float *out,
                    void *workspace, size_t workspace_bytes, uint32_t *err) {
    if (m == 0 || w.n == 0) return cudaSuccess;
    if (w.k == 0) return cudaMemsetAsync(out, 0, m * w.n * sizeof(float), s);
    // Prefill-sized inputs: the tcgen05 GEMM (activation planes after the
    // GEMV tickets in the workspace), else the SIMT GEMM.
    if (m > 64) {
        const size_t tickets = 64 * 1024 * sizeof(unsigned);
        if (workspace && workspace_bytes > tickets && qgemm_tc_supported(w) &&
            qgemm_tc_rows_per_pass(w, workspace_bytes - tickets) > 0)
            return qgemm_tc(s, x, m, w, out, static_cast<char *>(workspace) + tickets,
                            workspace_bytes - tickets, err);
        return qgemm_f32(s, x, m, w, out);
    }
    // Decode-sized inputs: the tensor-core GEMV, in blocks of at most 32 rows.
    for (size_t m0 = 0; m0 < m; m0 += 32) {
        size_t mb = m - m0 < 32 ? m - m0 : 32;
        const float *xb = x + m0 * w.k;
        float *ob = out + m0 * w.n;
        if (qgemv_tma_supported(w, mb) && qgemv_tma_x_aligned(xb) &&
            qgemv_tma_workspace_bytes(w, mb) <= workspace_bytes) {
            cudaError_t e = qgemv_tma(s, xb, mb, w, ob, workspace, err);
            if (e != cudaSuccess) return e;
            continue;
        }
        Plan pl = make_plan(w, mb);
        size_t need = mma_workspace_bytes(w, mb);
        if (pl.fast && need <= workspace_bytes) {
            cudaError_t e;
            if (w.format == 0) {
                e = pl.nt == 1 ? launch_fast<0, 1>(s, xb, mb, w, ob, pl, workspace)
                  : pl.nt == 2 ? launch_fast<0, 2>(s, xb, mb, w, ob, pl, workspace)
                               : launch_fast<0, 4>(s, xb, mb, w, ob, pl, workspace);
            } else {
                e = pl.nt == 1 ? launch_fast<1, 1>(s, xb, mb, w, ob, pl, workspace)
                  : pl.nt == 2 ? launch_fast<1, 2>(s, xb, mb, w, ob, pl, workspace)
                               : launch_fast<1, 4>(s, xb, mb, w, ob, pl, workspace);
            }
            if (e != cudaSuccess) return e;
        } else {
            int grid = grid_for(w.n, 8, 16);
            if (w.format == 0)
                launch_k(qgemv_simple<0>, grid, 256, 0, s, xb, (int)mb, (int)w.k, w.codes, w.row_bytes,
                                                     w.scales, (int)w.group, (int)w.groups, ob,
                                                     (int)w.n);
            else
                launch_k(qgemv_simple<1>, grid, 256, 0, s, xb, (int)mb, (int)w.k, w.codes, w.row_bytes,
                                                     w.scales, (int)w.group, (int)w.groups, ob,
                                                     (int)w.n);
            count_launch();
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) return e;
        }
    }
    return cudaSuccess;
}

cudaError_t quantize(cudaStream_t s, const float *w, size_t n, size_t k, size_t group,
                     int format, uint8_t *codes, float *scales) {
    if (n == 0 || k == 0) return cudaSuccess;
    const size_t groups = (k + group - 1) / group;
    const size_t row_bytes = format == 0 ? (k + 1) / 2 : k;
    const float qmax = format == 0 ? 7.0f : 127.0f;
    launch_k(quant_scales, grid_for(n * groups, 8, 16), 256, 0, s, w, n, k, group, groups, qmax, scales);
    count_launch();
    launch_k(quant_codes, grid_for(n * row_bytes, 256), 256, 0, s, w, n, k, group, groups, row_bytes,
                                                             format, qmax, scales, codes);
    count_launch();
    return cudaGetLastError();
}

cudaError_t dequantize(cudaStream_t s, const QuantWeight &w, float *out) {
    if (w.n == 0 || w.k == 0) return cudaSuccess;
    launch_k(dequant_kernel, grid_for(w.n * w.k, 256), 256, 0, s, w.codes, w.scales, w.n, w.k, w.group,
                                                            w.groups, w.row_bytes, w.format, out);
    count_launch();
    return cudaGetLastError();
}

}  // namespace k
}  // namespace slc
