// Persistent decode of a run of llama-dense layers at batch 1: one
// cooperative launch replaces, for every layer of the run, the sixteen
// commands the llama-dense lowering emits per layer
// (sl-model-adapters contract, docs/ARCH-0006 sections 4-5):
//
//   RmsNorm(x) -> h; MatMulNT q, k, v; SplitHeads x3; Rope q, k;
//   CausalAttention (KV append + attention); MergeHeads; MatMulNT o;
//   Add(x, o) -> x1; RmsNorm(x1) -> h2; SwiGlu(h2) -> f; Add(x1, f) -> x'.
//
// Reference arithmetic: crates/backends/backend-cpu/src/reference/
// norm.rs:27-60 (RmsNorm), matmul.rs:29-59 on the dequantized weights,
// rope.rs:55-88 (f64 angle, f32 rotation), attention.rs:33-83 (append) and
// :129-219 (attention), swiglu.rs:40-84 (silu(gate) * up, then down),
// elementwise.rs:53-61 (Add).
//
// Why one kernel: at batch 1 a decode step streams ~4 GB of quantized
// weights through ~260 dependent launches; each launch boundary costs a few
// microseconds in which no weight byte moves (the next kernel's CTAs cannot
// become resident while the previous kernel holds the SMs' shared memory).
// Here the weights never stop streaming: in every CTA a producer warp walks
// the whole run's weight sequence (and the CTA's attention chunk of the KV
// cache) through a shared-memory ring with TMA, waiting only for free slots,
// so the next stage's weights are already on chip when its inputs become
// ready. Stage boundaries are global arrival counters, not launches.
//
// Grid: one CTA per SM (all co-resident: cooperative launch). CTAs
// 0 .. W-1 are workers; CTA W (the last) is the scribe.
//
// Stages of a layer (workers), each ended by an arrival counter (the
// inputs of the GEMV stages are digitized first: their own arrival counters
// DQ, DGU, DD separate digitization from use):
//   QKV   x = x1 + f (previous layer), h = rmsnorm(x); q, k, v GEMVs
//   ATTN  one (kv head, key chunk) item per worker: RoPE of its q heads and
//         of the new key, scores over the chunk's keys (cached keys from the
//         ring, the new key from this step's k / v, appended to the cache by
//         the chunk's owner), online softmax; chunk partials merged in
//         ascending chunk order by the last CTA of each kv head (ticket)
//   O     o GEMV on the attention output
//   GU    x1 = x + o, h2 = rmsnorm(x1); gate and up GEMVs
//   DOWN  down GEMV on silu(gate) * up
// Under tensor parallelism each rank runs its shard (its heads, gate/up
// rows and o/down columns); after the O and DOWN GEMVs every worker
// all-reduces its output rows with the same worker of the other ranks over
// peer memory (tp_reduce_rows) before the stage's arrival.
// The residual stream (x, then x1) lives in every CTA's shared memory and
// is updated redundantly and identically; intermediate activations go
// through a private scratch area that no command aliases.
//
// The scribe writes every command's output buffer, in command order, from
// the private copies (SplitHeads / MergeHeads at one token are element
// copies), so all buffers end as sequential execution leaves them even
// where the memory plan lets outputs reuse the bytes of dead values.
// Workers never read command buffers after the start (only the first
// layer's input, the weights, the positions and the KV cache), and a worker
// overwrites a private buffer of layer l only after the scribe has
// signalled that it has read layer l - 1's copies.
//
// GEMV (the decode GEMV arithmetic of gemv_lane.cu): weights in 16-row
// tiles; each worker owns a contiguous range of whole tiles (no cross-CTA
// sums). A tile is streamed in chunks of [16 rows][C bytes of codes] (one
// 2-D TMA box, C chosen per stage by the host, at most 1 KiB; rows padded
// in shared memory so that neighbouring rows sit 16 banks apart) plus the
// chunk's scales ([16 rows][groups of the chunk], a second box padded
// likewise, or for single-chunk rows one bulk copy of the tile's contiguous
// scale rows); a worker's tiles go in groups of four, chunk by chunk within
// a group. Consumer warp w multiplies two 64-byte warp-steps of every chunk
// (2w and 2w + 1 of a 1 KiB chunk, w and w + 8 of a shorter one) with the
// s8 tensor-core path
// (INT4 nibbles as 16 x code, activations as three exact 7-bit digits per
// value in the MMA's N dimension, integer block sums converted exactly and
// scaled by scale * 2^e * 2^-7d), reusing a chunk's digits for the whole
// group. Warp sums of every tile are added in warp order.
//
// HBM traffic per layer: the quantized weights (codes + scales) once, the
// KV cache rows [0, past) of the layer once, plus activations (KBs). The
// padding boxes also read the first 64 code bytes (16 scale bytes) of the
// row's next chunk, which the next box of the same tile reads again from
// L2; past a row's end they are zero fill.
//
// Every wait is bounded (1 s): a CTA that gives up records kErrWaitTimeout,
// raises the global abort word (every other CTA then stops waiting at its
// next dependency) and finishes without touching the ring, after its
// producer has waited (bounded) for the copies it issued. The last CTA to
// exit resets the counters for the next launch.
#include <math.h>

#include <cuda.h>

#include <string.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "gemv_common.cuh"
#include "kernels.h"
#include "tensormap.h"
#include "tma.cuh"

namespace slc {
namespace k {
namespace {

constexpr int kCons = 8;                     // consumer warps (each takes two warp-steps
                                             // of every chunk; 9 warps leave 168 registers
                                             // a thread, so nothing spills to local memory)
constexpr int kConsThreads = kCons * 32;
// + the producer warpgroup: one warp (lane 0) walks the weights, three stay
// idle. At the start the producer warpgroup lowers its registers to
// kProdRegs and the consumer warpgroups raise theirs to kConsRegs
// (setmaxnreg); the block is launched with 168 a thread, and
// 384 x 168 = 256 x kConsRegs + 128 x kProdRegs, so the raise never waits
// for registers that do not exist.
constexpr int kThreads = kConsThreads + 128;
constexpr int kLaunchRegs = 168, kConsRegs = 224, kProdRegs = 56;
static_assert(kThreads * kLaunchRegs == kConsThreads * kConsRegs + 128 * kProdRegs,
              "register split");
constexpr int kSlots = 8;                    // ring slots
constexpr int kChunk = 1024;                 // code bytes per row per chunk
// A slot holds 16 rows of a chunk; each row is followed by 64 bytes (the
// start of the next chunk, or the zero fill past the row's end) so that
// rows r and r + 1 start 16 banks apart and a quarter-warp's 16-byte loads
// of two rows never share a bank.
constexpr int kRowPad = 64;
constexpr int kSlotCode = 16 * (kChunk + kRowPad);  // codes (or 16 K + 16 V rows)
constexpr int kScalePad = 4;                 // floats after each row's chunk scales
constexpr int kSlotBytes = kSlotCode + 16 * (16 + kScalePad) * 4;  // + scales [16][<= 20]
constexpr int kRedTiles = 4;                 // tiles per group (one cross-warp reduction)
constexpr int kD = 128;                      // head_dim
constexpr int kMaxLayers = 128;
constexpr int kSmemLimit = 227 * 1024;
constexpr uint64_t kWaitNs = 1000000000ull;

// Sync words (unsigned), zero at launch, reset by the last CTA to exit.
constexpr int kSyncAbort = 0, kSyncExit = 1, kSyncScribe = 2, kSyncTickets = 8,
              kSyncStages = 64;
enum Stage { kQKV = 0, kATTN = 1, kO = 2, kGU = 3, kDOWN = 4 };
// Arrival counters of a layer: the three digitize phases (DQ, DGU, DD)
// and the five stages.
enum Ctr { cDQ = 0, cQKV, cATTN, cO, cDGU, cGU, cDD, cDOWN, kCtrs };
static_assert(kSyncStages + kCtrs * kMaxLayers <= kDecodeStampWord, "sync words");
enum { kMq = 0, kMk, kMv, kMo, kMgate, kMup, kMdown };

struct DlLayer {
    int map[7];         // codes tensor map of q k v o gate up down (scales: map + 1)
    int cache_layer;    // layer index in the KV state
    const float *wn1, *wn2;
    float eps1, eps2, scale, pad;
    const uint32_t *d_past;  // device past_len (graph replay) or null
    uint32_t past;           // host past_len otherwise
    uint32_t order;          // bit c: the scribe needs a barrier before output c
    float *cmd[kDlCmds];     // command outputs, in command order
    const float *scales[7];  // scale rows of q k v o gate up down (single-chunk stages)
};

struct alignas(64) DlArgs {
    CUtensorMap kv_map;  // [cache_layers * 2 * max_seq][Hkv][D] f32, box [16][1][D]
    const CUtensorMap *maps;
    const DlLayer *layers;
    const float *x0;
    const uint32_t *pos;
    float *cache;
    float *Q, *Kp, *Vp, *ATT, *O, *Gb, *Ub, *F, *part_o, *part_ml;
    unsigned char *digA, *digO, *digD;  // digit vectors: h / h2, attention output, silu(g) * u
    unsigned *sync;
    uint32_t *err;
    long long par_stride;  // floats from the keys to the values of a cache layer
    long long lay_stride;  // floats between cache layers
    int L, H, Hq, Hkv, I, G, group, gptj, max_seq, W, nchunk_cap;
    int stC[5];                  // code bytes per chunk of stages kQKV .. kDOWN (host choice)
    int tp_rank, tp_world;       // tensor parallelism (world 1: none)
    uint64_t *xwords[kMaxPeers]; // every rank's exchange words [2][world][kDlTpHidden]
    uint32_t *tp_launches;       // this rank's fused launches so far (exchange epochs)
    int dig_bytes, nch_max;
    int off_bar, off_misc, off_resid, off_dig, off_red, off_trig;
    double denom[kD / 2];
};

struct Smem {
    unsigned char *ring;
    uint64_t *full, *empty;
    uint64_t *dbar;       // completion of the digit-vector copy
    volatile int *abort;  // this CTA gave up
    int *flag;
    float *part;          // [kCons] rms partial sums
    float *resid;         // [H]
    int8_t *dig;          // the stage input's digit vector (dig_bytes), or attention scratch
    float *red;           // [kRedTiles][kCons][16]
    float *trig;          // [D]: sin of the D/2 pairs, then cos
};

__device__ __forceinline__ Smem carve(const DlArgs &p, unsigned char *base) {
    Smem s;
    s.ring = base;
    s.full = reinterpret_cast<uint64_t *>(base + p.off_bar);
    s.empty = s.full + kSlots;
    s.dbar = s.empty + kSlots;
    s.abort = reinterpret_cast<volatile int *>(base + p.off_misc);
    s.flag = reinterpret_cast<int *>(base + p.off_misc + 4);
    s.part = reinterpret_cast<float *>(base + p.off_misc + 16);
    s.resid = reinterpret_cast<float *>(base + p.off_resid);
    s.dig = reinterpret_cast<int8_t *>(base + p.off_dig);
    s.red = reinterpret_cast<float *>(base + p.off_red);
    s.trig = reinterpret_cast<float *>(base + p.off_trig);
    return s;
}

// ---- small device helpers -------------------------------------------------------

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *a) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}

// *a += v at GPU scope with release semantics: the writes this CTA made
// before (ordered to this thread by a CTA barrier) are visible to a thread
// that acquires the new value.
__device__ __forceinline__ void red_release_add(unsigned *a, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}

// Ticket: the old value of *a, incremented with acquire-release semantics
// at GPU scope (the last taker sees every earlier taker's writes).
__device__ __forceinline__ unsigned atom_acq_rel_add(unsigned *a, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(a), "r"(v) : "memory");
    return old;
}

// L2 policy for data every CTA reads (the digit vectors).
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void cons_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(kConsThreads) : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const void *tmap, int x, int y, int z,
                                            uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
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
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(smem_addr(p)));
    return r;
}

// Exact int -> float for |c| < 2^22.
__device__ __forceinline__ float i2f_exact(int c) {
    return __int_as_float(c + 0x4B400000) - 12582912.0f;
}

// Thread 0 of the consumers: waits until *ctr >= target and, when `gate`
// is set, *gate >= gate_target (both loads in flight together). False when
// this or another CTA gave up (abort words), or on timeout (recorded, abort
// raised everywhere).
__device__ __forceinline__ bool poll_ge(const DlArgs &p, const Smem &sm, const unsigned *ctr, unsigned target,
                        const unsigned *gate, unsigned gate_target) {
    uint64_t t0 = 0;
    for (int it = 0;; it++) {
        const unsigned a = ld_acquire_u32(ctr);
        const unsigned b = gate ? ld_acquire_u32(gate) : gate_target;
        if (a >= target && b >= gate_target) return true;
        if (*sm.abort || *reinterpret_cast<volatile unsigned *>(p.sync + kSyncAbort)) {
            *sm.abort = 1;
            return false;
        }
        if (it == 0) {
            t0 = global_ns();
        } else if (global_ns() - t0 > kWaitNs) {
            report_error(p.err, kErrWaitTimeout);
            atomicExch(p.sync + kSyncAbort, 1u);
            *sm.abort = 1;
            return false;
        }
        if (it > 64) __nanosleep(32);
    }
}

// All consumer threads: the stage's dependency `*ctr >= target` and, for a
// stage that overwrites a private buffer the scribe copies, the scribe's
// progress `*gate >= gate_target`.
__device__ __forceinline__ void dep_wait(const DlArgs &p, const Smem &sm, const unsigned *ctr,
                                         unsigned target, const unsigned *gate = nullptr,
                                         unsigned gate_target = 0) {
    if (threadIdx.x == 0) poll_ge(p, sm, ctr, target, gate, gate_target);
    cons_sync();
}

// All consumer threads: this CTA's part of a stage is written.
__device__ __forceinline__ void arrive(unsigned *ctr) {
    cons_sync();
    if (threadIdx.x == 0) {
        red_release_add(ctr, 1u);
    }
}

// Consumers: the ring slot `seq` has landed (false: give up, see abort).
__device__ __forceinline__ bool wait_full(uint32_t *err, const Smem sm, unsigned seq) {
    if (*sm.abort) return false;
    return mbar_wait(&sm.full[seq % kSlots], (seq / kSlots) & 1, err,
                     const_cast<volatile int *>(sm.abort), kWaitNs);
}

__device__ __forceinline__ void release(const Smem sm, unsigned seq) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0 && !*sm.abort) mbar_arrive(&sm.empty[seq % kSlots]);
}

// ---- stage geometry (identical in producer and consumers) -----------------------

template <int FMT>
struct Q;
template <>
struct Q<0> {
    static constexpr int kStep = 128;  // codes per warp-step (64 bytes)
    static constexpr int kWsb = 128;   // digit bytes per column per warp-step
    static constexpr int kJ = 4;       // k32 MMAs per warp-step
};
template <>
struct Q<1> {
    static constexpr int kStep = 64;
    static constexpr int kWsb = 64;
    static constexpr int kJ = 2;
};

struct StageGeo {
    int nm;                  // matrices
    int mat0, mat1, mat2;    // kMq ...
    int tend0, tend1;        // cumulative 16-row tiles of the first two
    float *out0, *out1, *out2;  // private outputs
    int tiles, K, rowb, C, nch, wact, gpc;
    int Cp, gps;  // slot row strides: code bytes, scale floats
    int bulk;     // single-chunk tiles: the scales by one bulk copy of the tile's rows
    int wstep0, wstride;  // warp w takes warp-steps wstep0 * w and wstep0 * w + wstride
};

// Slot row strides of a stage with rows of rowb code bytes in chunks of C
// bytes holding gpc scale groups (the boxes the host encodes match).
// Single-chunk rows are copied unpadded (the box never exceeds the row).
__host__ __device__ __forceinline__ int slot_code_stride(int rowb, int C) {
    return (rowb > C && C % 128 == 0) ? C + kRowPad : C;
}
__host__ __device__ __forceinline__ int slot_scale_stride(int rowb, int C, int gpc) {
    return rowb > C ? gpc + kScalePad : gpc;
}

template <int FMT>
__device__ __forceinline__ StageGeo stage_geo(const DlArgs &p, int st) {
    StageGeo g{};
    const int D = kD;
    int r0 = 0, r1 = 0, r2 = 0;
    if (st == kQKV) {
        g.nm = 3;
        g.mat0 = kMq, g.mat1 = kMk, g.mat2 = kMv;
        r0 = p.Hq * D, r1 = p.Hkv * D, r2 = p.Hkv * D;
        g.out0 = p.Q, g.out1 = p.Kp, g.out2 = p.Vp;
        g.K = p.H;
    } else if (st == kO) {
        g.nm = 1;
        g.mat0 = g.mat1 = g.mat2 = kMo;
        r0 = p.H;
        g.out0 = g.out1 = g.out2 = p.O;
        g.K = p.Hq * D;
    } else if (st == kGU) {
        g.nm = 2;
        g.mat0 = kMgate, g.mat1 = g.mat2 = kMup;
        r0 = p.I, r1 = p.I;
        g.out0 = p.Gb, g.out1 = g.out2 = p.Ub;
        g.K = p.H;
    } else {
        g.nm = 1;
        g.mat0 = g.mat1 = g.mat2 = kMdown;
        r0 = p.H;
        g.out0 = g.out1 = g.out2 = p.F;
        g.K = p.I;
    }
    g.tend0 = r0 / 16;
    g.tend1 = g.tend0 + r1 / 16;
    g.tiles = g.tend1 + r2 / 16;
    g.rowb = FMT == 0 ? g.K / 2 : g.K;
    g.C = p.stC[st];
    g.nch = (g.rowb + g.C - 1) / g.C;  // the last chunk may be ragged
    g.wact = g.C / 64;
    g.gpc = g.C * (FMT == 0 ? 2 : 1) / p.group;
    g.Cp = slot_code_stride(g.rowb, g.C);
    g.gps = slot_scale_stride(g.rowb, g.C, g.gpc);
    g.bulk = g.nch == 1;
    // Sixteen warp-steps a chunk: adjacent pairs; fewer: w and w + 8.
    g.wstep0 = g.wact == 16 ? 2 : 1;
    g.wstride = g.wact == 16 ? 1 : 8;
    return g;
}

// Matrix (0, 1, 2) of a tile of the stage and the tile's first row in it.
__device__ __forceinline__ int tile_mat(const StageGeo &g, int tile, int *row) {
    if (g.nm > 1 && tile >= g.tend0) {
        if (g.nm > 2 && tile >= g.tend1) {
            *row = (tile - g.tend1) * 16;
            return 2;
        }
        *row = (tile - g.tend0) * 16;
        return 1;
    }
    *row = tile * 16;
    return 0;
}

__device__ __forceinline__ float *stage_out(const StageGeo &g, int m) {
    return m == 0 ? g.out0 : (m == 1 ? g.out1 : g.out2);
}

__device__ __forceinline__ int stage_mat(const StageGeo &g, int m) {
    return m == 0 ? g.mat0 : (m == 1 ? g.mat1 : g.mat2);
}

// Attention plan of one layer (identical in producer and consumers).
struct AttnPlan {
    int past, nchunk, ck;
};

__device__ __forceinline__ AttnPlan attn_plan(const DlArgs &p, const DlLayer &ly) {
    AttnPlan a;
    int past = ly.d_past ? (int)*ly.d_past : (int)ly.past;
    if (past < 0 || past >= p.max_seq) {  // validated on the host; guard anyway
        report_error(p.err, kErrBadScalar);
        past = 0;
    }
    a.past = past;
    const int nk = past + 1;
    int want = p.nchunk_cap;
    const int by_len = (nk + 15) / 16;
    if (want > by_len) want = by_len;
    if (want < 1) want = 1;
    int ck = (nk + want - 1) / want;
    ck = (ck + 15) / 16 * 16;
    a.ck = ck;
    a.nchunk = (nk + ck - 1) / ck;
    return a;
}

// ---- producer ----------------------------------------------------------------

template <int FMT>
__device__ void producer(const DlArgs &p, const Smem sm) {
    const uint64_t pol = policy_evict_first();
    const int c = blockIdx.x;
    // Kept in registers: a generic load of the kernel parameters (passed
    // by reference to this non-inlined function) on every slot costs more
    // than the slot's copy.
    uint32_t *const err = p.err;
    const CUtensorMap *const maps = p.maps;
    const CUtensorMap *const kvmap = &p.kv_map;
    const int W = p.W, L = p.L, Hkv = p.Hkv, max_seq = p.max_seq;
    unsigned seq = 0;
    bool stop = false;
    // Reserves the next slot for `bytes` of copies; null when giving up.
    auto next_slot = [&](uint32_t bytes) -> unsigned char * {
        if (stop || *sm.abort) {
            stop = true;
            return nullptr;
        }
        const int slot = seq % kSlots;
        if (seq >= (unsigned)kSlots &&
            !mbar_wait(&sm.empty[slot], ((seq / kSlots) - 1) & 1, err,
                       const_cast<volatile int *>(sm.abort), kWaitNs)) {
            stop = true;
            return nullptr;
        }
        mbar_arrive_expect_tx(&sm.full[slot], bytes);
        seq++;
        return sm.ring + slot * kSlotBytes;
    };
    for (int l = 0; l < L && !stop; l++) {
        const DlLayer &ly = p.layers[l];
        for (int st = kQKV; st <= kDOWN && !stop; st++) {
            if (st == kATTN) {
                const AttnPlan ap = attn_plan(p, ly);
                if (c >= Hkv * ap.nchunk) continue;
                const int kvh = c / ap.nchunk, chunk = c - kvh * ap.nchunk;
                const int k0 = chunk * ap.ck, k1 = min(ap.past + 1, k0 + ap.ck);
                const int nsl = (k1 - k0 + 15) / 16;
                const int zk = (ly.cache_layer * 2) * max_seq + k0;
                const int zv = (ly.cache_layer * 2 + 1) * max_seq + k0;
                for (int s = 0; s < nsl; s++) {
                    unsigned char *dst = next_slot(2 * 16 * kD * 4);
                    if (!dst) break;
                    tma_load_3d(dst, kvmap, 0, kvh, zk + 16 * s, &sm.full[(seq - 1) % kSlots], pol);
                    tma_load_3d(dst + 16 * kD * 4, kvmap, 0, kvh, zv + 16 * s,
                                &sm.full[(seq - 1) % kSlots], pol);
                }
                continue;
            }
            // This worker's tiles in groups of kRedTiles, each group chunk by
            // chunk (the consumers reuse a chunk's digits across the group).
            const StageGeo g = stage_geo<FMT>(p, st);
            const int t0 = (int)((long long)c * g.tiles / W);
            const int t1 = (int)((long long)(c + 1) * g.tiles / W);
            const uint32_t bytes = (uint32_t)(16 * g.Cp + 16 * g.gps * 4);
            for (int tg = t0; tg < t1 && !stop; tg += kRedTiles) {
                const int nb = min(kRedTiles, t1 - tg);
                for (int ch = 0; ch < g.nch && !stop; ch++) {
                    for (int b = 0; b < nb; b++) {
                        int row;
                        const int m = tile_mat(g, tg + b, &row);
                        const CUtensorMap *cm = maps + ly.map[stage_mat(g, m)];
                        unsigned char *dst = next_slot(bytes);
                        if (!dst) break;
                        uint64_t *bar = &sm.full[(seq - 1) % kSlots];
                        tma_load_2d(dst, cm, ch * (g.C / 8), row, bar, pol);  // u64 units
                        if (g.bulk)  // the tile's 16 scale rows are contiguous
                            bulk_g2s(dst + kSlotCode,
                                     ly.scales[stage_mat(g, m)] + (size_t)row * g.gpc,
                                     (uint32_t)(16 * g.gpc * 4), bar, pol);
                        else
                            tma_load_2d(dst + kSlotCode, cm + 1, ch * g.gpc, row, bar, pol);
                    }
                }
            }
        }
    }
    // Copies still in flight land before the CTA exits (bounded): the last
    // use of every slot.
    for (int s = 0; s < kSlots; s++) {
        if ((unsigned)s >= seq) break;
        const unsigned last = seq - 1 - ((seq - 1 - s) % kSlots);
        const uint32_t ph = (last / kSlots) & 1;
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(&sm.full[s], ph) && global_ns() - t0 < 100000000ull) {
        }
    }
}

// ---- consumers: activation staging ---------------------------------------------

// Byte of activation k (within its warp-step) in the [j][t][8 bytes] cell
// layout of the MMA B fragments (the layout of gemv_lane.cu).
template <int FMT>
__device__ __forceinline__ int lane_byte(int kl) {
    if (FMT == 0) {
        const int t = kl >> 5, j = (kl >> 3) & 3, i = (kl >> 1) & 3, odd = kl & 1;
        return j * 32 + t * 8 + odd * 4 + i;
    }
    const int t = kl >> 4, j = (kl >> 3) & 1, h = (kl >> 2) & 1, i = kl & 3;
    return j * 32 + t * 8 + h * 4 + i;
}

// One warp-step of the activation row as three exact 7-bit digits
// (x = 2^e (d0 + d1 / 128 + d2 / 16384), |x / 2^e| < 64) plus the digit
// factors 2^e 2^-7d (x 1/16 for INT4 codes held as 16 x code).
template <int FMT>
__device__ __forceinline__ void digits_step(float (&v)[Q<FMT>::kStep / 32], int8_t *dstep,
                                            float *fstep) {
    constexpr int PER = Q<FMT>::kStep / 32;
    constexpr int WSB = Q<FMT>::kWsb;
    const int lane = threadIdx.x & 31;
    float mx = 0.f;
    bool bad = false;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const float a = fabsf(v[i]);
        bad |= !(a <= 3.402823466e38f);
        mx = fmaxf(mx, a);
    }
    mx = warp_max(mx);
    bad = __any_sync(0xffffffffu, bad);
    int e = 0;
    if (mx > 0.f && !bad) {
        int ex;
        frexpf(mx, &ex);
        e = ex - 6;
    }
    const bool direct = e >= -126 && e <= 126;
    const float sc = __int_as_float((127 - e) << 23);
    uint32_t db[3][PER];
#pragma unroll
    for (int i = 0; i < PER; i++) {
        float y = 0.f;
        if (!bad) y = direct ? v[i] * sc : ldexpf(v[i], -e);
        const float d0 = rintf(y);
        const float r1 = fmaf(d0, -128.f, y * 128.f);
        const float d1 = rintf(r1);
        const float r2 = fmaf(d1, -128.f, r1 * 128.f);
        const float d2 = rintf(r2);
        db[0][i] = __float_as_uint(d0 + 12582912.0f);
        db[1][i] = __float_as_uint(d1 + 12582912.0f);
        db[2][i] = __float_as_uint(d2 + 12582912.0f);
    }
    unsigned char *d0p = reinterpret_cast<unsigned char *>(dstep);
    const int b = lane_byte<FMT>(lane * PER);
#pragma unroll
    for (int dd = 0; dd < 3; dd++) {
        if (FMT == 0) {
            *reinterpret_cast<uint16_t *>(d0p + dd * WSB + b) =
                (uint16_t)prmt(db[dd][0], db[dd][2 % PER], 0x0040u);
            *reinterpret_cast<uint16_t *>(d0p + dd * WSB + b + 4) =
                (uint16_t)prmt(db[dd][1 % PER], db[dd][3 % PER], 0x0040u);
        } else {
            *reinterpret_cast<uint16_t *>(d0p + dd * WSB + b) =
                (uint16_t)prmt(db[dd][0], db[dd][1 % PER], 0x0040u);
        }
    }
    if (lane < 8) {
        float f = 0.f;
        if (lane < 3) {
            f = bad ? __int_as_float(0x7fc00000) : ldexpf(FMT == 0 ? 0.0625f : 1.0f, e);
            f *= lane == 0 ? 1.0f : (lane == 1 ? 0.0078125f : 6.103515625e-05f);
        }
        fstep[lane] = f;
    }
}

enum StageIn { kInNorm = 0, kInVec = 1, kInSwiglu = 2, kInShared = 3 };

// A stage input is digitized once per stage (warp-steps spread over the
// workers) into a digit vector in global memory, one record per warp-step:
// [3][WSB] digit bytes, then 8 digit factors. Every worker then copies the
// whole vector into shared memory.
template <int FMT>
struct Rec {
    static constexpr int kDigits = 3 * Q<FMT>::kWsb;
    static constexpr int kBytes = kDigits + 32;
};

// Warp-steps [s0, s1) of a stage input, one per warp: rmsnorm(resid) * w
// (norm.rs arithmetic: two rounded multiplies), a private vector (global,
// or shared memory holding the steps from s0 on), or silu(a) * b (the
// elementwise silu_mul expression).
template <int FMT, int MODE>
__device__ __forceinline__ void digitize_steps(const Smem &sm, int s0, int s1, const float *src,
                                               const float *src2, const float *wn, float inv,
                                               unsigned char *out) {
    constexpr int PER = Q<FMT>::kStep / 32;
    constexpr int kBatch = 4;  // steps of a warp whose loads are in flight together
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int base = s0 + warp; base < s1; base += kCons * kBatch) {
        float x[kBatch][PER], y[kBatch][PER];
#pragma unroll
        for (int q = 0; q < kBatch; q++) {
            const int st = base + q * kCons;
            const int k = st * Q<FMT>::kStep + lane * PER;
#pragma unroll
            for (int i = 0; i < PER; i++) {
                x[q][i] = 0.f, y[q][i] = 0.f;
                if (st < s1) {
                    if (MODE == kInNorm) {
                        x[q][i] = sm.resid[k + i];
                        y[q][i] = __ldg(wn + k + i);
                    } else if (MODE == kInVec) {
                        x[q][i] = __ldcg(src + k + i);
                    } else if (MODE == kInShared) {  // src holds the steps from s0 on
                        x[q][i] = src[k - s0 * Q<FMT>::kStep + i];
                    } else {
                        x[q][i] = __ldcg(src + k + i);
                        y[q][i] = __ldcg(src2 + k + i);
                    }
                }
            }
        }
#pragma unroll
        for (int q = 0; q < kBatch; q++) {
            const int st = base + q * kCons;
            if (st >= s1) break;
            float v[PER];
#pragma unroll
            for (int i = 0; i < PER; i++) {
                if (MODE == kInNorm) {
                    v[i] = __fmul_rn(__fmul_rn(x[q][i], inv), y[q][i]);
                } else if (MODE == kInSwiglu) {
                    const float a = x[q][i];
                    v[i] = __fmul_rn(__fmul_rn(a, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-a)))),
                                     y[q][i]);
                } else {
                    v[i] = x[q][i];
                }
            }
            unsigned char *rec = out + (size_t)st * Rec<FMT>::kBytes;
            digits_step<FMT>(v, reinterpret_cast<int8_t *>(rec),
                             reinterpret_cast<float *>(rec + Rec<FMT>::kDigits));
        }
    }
}

// This worker's share of the warp-steps of a stage input of K values.
template <int FMT>
__device__ __forceinline__ void my_steps(const DlArgs &p, int K, int *s0, int *s1) {
    const int S = K / Q<FMT>::kStep;
    *s0 = (int)((long long)blockIdx.x * S / p.W);
    *s1 = (int)((long long)(blockIdx.x + 1) * S / p.W);
}

// The digit vector of a stage input of K values, into shared memory: one
// bulk copy (TMA) issued by one thread, after a proxy fence that orders the
// other CTAs' digit stores (acquired by the dependency wait) before the
// copy reads them. `fetches` counts this CTA's copies (the barrier phase).
template <int FMT>
__device__ __forceinline__ void fetch_digits(const DlArgs &p, const Smem &sm,
                                             const unsigned char *src, int K, unsigned &fetches) {
    const uint32_t bytes = (uint32_t)(K / Q<FMT>::kStep * Rec<FMT>::kBytes);
    // The destination was last written by ordinary stores (the attention
    // scratch aliases it): order them before the copy.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    cons_sync();
    if (threadIdx.x == 0 && !*sm.abort) {
        asm volatile("fence.proxy.async.global;" ::: "memory");
        mbar_arrive_expect_tx(sm.dbar, bytes);
        bulk_g2s(sm.dig, src, bytes, sm.dbar, policy_evict_last());
    }
    if (!*sm.abort)
        mbar_wait(sm.dbar, fetches & 1, p.err, const_cast<volatile int *>(sm.abort), kWaitNs);
    fetches++;
}

// ---- consumers: GEMV over this worker's tiles -----------------------------------
//
// Warp w multiplies two warp-steps (64 code bytes each) of every chunk
// (StageGeo::wstep0, wstride). A worker's tiles are streamed in groups of kRedTiles tiles,
// chunk by chunk within a group, so a warp loads a chunk's digit fragments
// and factors once and uses them for every tile of the group; each tile
// keeps its own row sums in registers (chunks added in ascending order).

// The digit fragments (B operands) and factors of warp-steps ws0 and
// ws0 + dstep of the stage input, from the shared digit vector.
template <int FMT>
struct StepDigits {
    uint2 bf[2][Q<FMT>::kJ];
    float2 fx[2];
};

template <int FMT>
__device__ __forceinline__ void load_step_digits(const unsigned char *rec0, int dstep, bool has0,
                                                 bool has1, StepDigits<FMT> &d) {
    constexpr int WSB = Q<FMT>::kWsb;
    const int lane = threadIdx.x & 31, gq = lane >> 2, t = lane & 3;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const unsigned char *rec = rec0 + h * dstep * Rec<FMT>::kBytes;
        const bool on = h == 0 ? has0 : has1;
        const int8_t *cell = reinterpret_cast<const int8_t *>(rec) + gq * WSB + t * 8;
#pragma unroll
        for (int j = 0; j < Q<FMT>::kJ; j++)
            d.bf[h][j] = (gq < 3 && on) ? lds64(cell + j * 32) : make_uint2(0u, 0u);
        d.fx[h] = on ? *reinterpret_cast<const float2 *>(
                           reinterpret_cast<const float *>(rec + Rec<FMT>::kDigits) + 2 * t)
                     : make_float2(0.f, 0.f);
    }
}

// One landed slot's part for this warp: the codes of its two warp-steps
// (rows gq and gq + 8) and the four scales they need.
struct SlotLoad {
    uint4 wa[2], wb[2];
    float s[2][2];
};

__device__ __forceinline__ void load_slot(const unsigned char *sl, int Cp, int gps, int ws0,
                                          int dstep, int gi0, int gi1, bool has1, SlotLoad &x) {
    const int lane = threadIdx.x & 31, gq = lane >> 2, t = lane & 3;
    const unsigned char *ra = sl + gq * Cp + ws0 * 64 + t * 16;
    const unsigned char *rb = ra + 8 * Cp;
    x.wa[0] = lds128(ra);
    x.wb[0] = lds128(rb);
    x.wa[1] = has1 ? lds128(ra + dstep * 64) : make_uint4(0u, 0u, 0u, 0u);
    x.wb[1] = has1 ? lds128(rb + dstep * 64) : make_uint4(0u, 0u, 0u, 0u);
    const float *sc = reinterpret_cast<const float *>(sl + kSlotCode);
    x.s[0][0] = sc[gq * gps + gi0];
    x.s[0][1] = sc[(gq + 8) * gps + gi0];
    x.s[1][0] = has1 ? sc[gq * gps + gi1] : 0.f;
    x.s[1][1] = has1 ? sc[(gq + 8) * gps + gi1] : 0.f;
}

// The s8 tensor-core products of a slot's two warp-steps with the digits
// (integer sums, exact).
template <int FMT>
__device__ __forceinline__ void mma_slot(const SlotLoad &x, const StepDigits<FMT> &d,
                                         int (&acc)[2][4]) {
    constexpr int J = Q<FMT>::kJ;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const uint32_t qa[4] = {x.wa[h].x, x.wa[h].y, x.wa[h].z, x.wa[h].w};
        const uint32_t qb[4] = {x.wb[h].x, x.wb[h].y, x.wb[h].z, x.wb[h].w};
        uint32_t ag[8], a8[8];
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
        // One accumulator chain per warp-step (the two warp-steps of each of
        // the two slots in flight give four independent chains a warp).
        int accj[J][4];
#pragma unroll
        for (int j = 0; j < J; j++) {
            accj[j][0] = accj[j][1] = accj[j][2] = accj[j][3] = 0;
            mma_s8(accj[j], ag[2 * j], a8[2 * j], ag[2 * j + 1], a8[2 * j + 1], d.bf[h][j].x,
                   d.bf[h][j].y);
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            acc[h][i] = accj[0][i];
#pragma unroll
            for (int j = 1; j < J; j++) acc[h][i] += accj[j][i];
        }
    }
}

// The integer block sums of a slot scaled (scale * digit factor) into the
// tile's row sums.
template <int FMT>
__device__ __forceinline__ void scale_slot(const SlotLoad &x, const int (&acc)[2][4],
                                           const StepDigits<FMT> &d, bool has1, float (&res)[4]) {
#pragma unroll
    for (int h = 0; h < 2; h++) {
        if (h == 1 && !has1) break;
        const float2 f = d.fx[h];
        res[0] = fmaf(i2f_exact(acc[h][0]), x.s[h][0] * f.x, res[0]);
        res[1] = fmaf(i2f_exact(acc[h][1]), x.s[h][0] * f.y, res[1]);
        res[2] = fmaf(i2f_exact(acc[h][2]), x.s[h][1] * f.x, res[2]);
        res[3] = fmaf(i2f_exact(acc[h][3]), x.s[h][1] * f.y, res[3]);
    }
}

template <int FMT>
__device__ __forceinline__ void gemv_tiles(const DlArgs &p, const Smem &sm, const StageGeo &g,
                                           unsigned &seq) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, t = lane & 3;
    const int c = blockIdx.x;
    const int t0 = (int)((long long)c * g.tiles / p.W);
    const int t1 = (int)((long long)(c + 1) * g.tiles / p.W);
    const unsigned char *digv = reinterpret_cast<const unsigned char *>(sm.dig);
    // The warp's warp-steps of a chunk: ws0 and ws0 + dstep.
    const int ws0 = g.wstep0 * warp, dstep = g.wstride;
    const int gi0 = ws0 * Q<FMT>::kStep / p.group, gi1 = (ws0 + dstep) * Q<FMT>::kStep / p.group;
    uint32_t *const err = p.err;
    const int nch = g.nch, wact = g.wact, Cp = g.Cp, gps = g.gps;
    const int steps = g.rowb / 64;  // warp-steps of a row (a ragged last chunk has fewer)
    static_assert(kRedTiles % 2 == 0, "slot pairs");
    for (int tg = t0; tg < t1; tg += kRedTiles) {
        const int nb = min(kRedTiles, t1 - tg);
        float res[kRedTiles][4];
#pragma unroll
        for (int b = 0; b < kRedTiles; b++) res[b][0] = res[b][1] = res[b][2] = res[b][3] = 0.f;
        for (int ch = 0; ch < nch; ch++) {
            const int wv = min(wact, steps - ch * wact);  // this chunk's warp-steps
            const bool has0 = ws0 < wv, has1 = ws0 + dstep < wv;
            StepDigits<FMT> d;
            load_step_digits<FMT>(digv + (ch * wact + ws0) * Rec<FMT>::kBytes, dstep, has0, has1,
                                  d);
#pragma unroll
            for (int b = 0; b < kRedTiles; b++) {
                if (b < nb) {
                    if (wait_full(err, sm, seq)) {
                        if (has0) {
                            SlotLoad x;
                            load_slot(sm.ring + (seq % kSlots) * kSlotBytes, Cp, gps, ws0,
                                      dstep, gi0, gi1, has1, x);
                            int a[2][4];
                            mma_slot<FMT>(x, d, a);
                            scale_slot<FMT>(x, a, d, has1, res[b]);
                        }
                        release(sm, seq);
                    }
                    seq++;
                }
            }
        }
        // Row sums of this warp: digit columns 0, 1 (lane quad t = 0) and 2
        // (t = 1) of activation row 0; then the warps' sums in warp order.
#pragma unroll
        for (int b = 0; b < kRedTiles; b++) {
            const float ca = __shfl_down_sync(0xffffffffu, res[b][0], 1);
            const float cb = __shfl_down_sync(0xffffffffu, res[b][2], 1);
            if (t == 0 && b < nb) {
                sm.red[(b * kCons + warp) * 16 + gq] = (res[b][0] + res[b][1]) + ca;
                sm.red[(b * kCons + warp) * 16 + gq + 8] = (res[b][2] + res[b][3]) + cb;
            }
        }
        cons_sync();
        if ((int)threadIdx.x < nb * 16) {
            const int b = threadIdx.x >> 4, r = threadIdx.x & 15;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kCons; w++) v += sm.red[(b * kCons + w) * 16 + r];
            int row;
            const int m = tile_mat(g, tg + b, &row);
            if (!*sm.abort) stage_out(g, m)[row + r] = v;
        }
        cons_sync();
    }
}

// ---- consumers: shared-memory vector helpers (all consumer threads) ------------

// 1 / sqrt(sum(x^2) / H + eps) of the residual row.
__device__ __forceinline__ float resid_inv_rms(const DlArgs &p, const Smem &sm, float eps) {
    const int tid = threadIdx.x;
    float ss = 0.f;
    for (int i = tid; i < p.H / 4; i += kConsThreads) {
        const float4 v = reinterpret_cast<const float4 *>(sm.resid)[i];
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) sm.part[tid >> 5] = ss;
    cons_sync();
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kCons; w++) total += sm.part[w];
    cons_sync();
    const float mean = __fdiv_rn(total, (float)p.H);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

// Global -> shared copy of n floats (n % 4 == 0, both 16-byte aligned), the
// loads of up to four float4 per thread issued before their stores.
__device__ __forceinline__ void load_smem(float *dst, const float *src, int n) {
    const int n4 = n / 4;
    for (int b = threadIdx.x; b < n4; b += 4 * kConsThreads) {
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; j++)
            if (b + j * kConsThreads < n4)
                v[j] = __ldcg(reinterpret_cast<const float4 *>(src) + b + j * kConsThreads);
#pragma unroll
        for (int j = 0; j < 4; j++)
            if (b + j * kConsThreads < n4)
                reinterpret_cast<float4 *>(dst)[b + j * kConsThreads] = v[j];
    }
}

// resid += v (the Add command's IEEE add), v in global memory, loads issued
// before the adds.
__device__ __forceinline__ void resid_add(const DlArgs &p, const Smem &sm, const float *v) {
    const int n4 = p.H / 4;
    for (int b = threadIdx.x; b < n4; b += 4 * kConsThreads) {
        float4 x[4];
#pragma unroll
        for (int j = 0; j < 4; j++)
            if (b + j * kConsThreads < n4)
                x[j] = __ldcg(reinterpret_cast<const float4 *>(v) + b + j * kConsThreads);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = b + j * kConsThreads;
            if (i < n4) {
                float4 r = reinterpret_cast<float4 *>(sm.resid)[i];
                r.x = __fadd_rn(r.x, x[j].x);
                r.y = __fadd_rn(r.y, x[j].y);
                r.z = __fadd_rn(r.z, x[j].z);
                r.w = __fadd_rn(r.w, x[j].w);
                reinterpret_cast<float4 *>(sm.resid)[i] = r;
            }
        }
    }
    cons_sync();
}

// ---- the scribe: command outputs from shared memory ------------------------------
//
// A phase loads the private values it needs into shared memory once, then
// writes the outputs of its commands in command order; a barrier precedes an
// output only when it shares bytes with an earlier output of the phase (bit
// c of the layer's `order`, computed on the host).

__device__ __forceinline__ void order_sync(const DlLayer &ly, int c) {
    if (ly.order & (1u << c)) cons_sync();
}

__device__ void put_smem(const DlLayer &ly, int c, const float *src, int n) {
    order_sync(ly, c);
    float *dst = ly.cmd[c];
    if (!dst) return;
    for (int i = threadIdx.x; i < n / 4; i += kConsThreads)
        reinterpret_cast<float4 *>(dst)[i] = reinterpret_cast<const float4 *>(src)[i];
}

__device__ void put_norm(const DlArgs &p, const Smem &sm, const DlLayer &ly, int c,
                         const float *wn, float inv) {
    order_sync(ly, c);
    float *dst = ly.cmd[c];
    if (!dst) return;
    for (int i = threadIdx.x; i < p.H; i += kConsThreads)
        dst[i] = __fmul_rn(__fmul_rn(sm.resid[i], inv), __ldg(wn + i));
}

// resid += v, v in shared memory (the scribe's staged copy).
__device__ void resid_add_smem(const DlArgs &p, const Smem &sm, const float *v) {
    for (int i = threadIdx.x; i < p.H; i += kConsThreads) sm.resid[i] = __fadd_rn(sm.resid[i], v[i]);
    cons_sync();
}

// The scribe has copied the private values of one more phase (called after
// the barrier that follows its loads): workers may overwrite them.
__device__ __forceinline__ void scribe_signal(const DlArgs &p) {
    if (threadIdx.x == 0) {
        red_release_add(p.sync + kSyncScribe, 1u);
    }
}

// RoPE of `rows` rows of D (rope.rs:55-88 pairs; the rope_kernel arithmetic:
// f32 sin / cos of the f64 angle, two IEEE multiplies and an add / sub).
// src: shared memory, or global memory written by other CTAs (global_src).
__device__ __forceinline__ void rope_rows(const DlArgs &p, const Smem &sm, const float *src, float *dst, int rows,
                          bool global_src) {
    const int half = kD / 2;
    for (int i = threadIdx.x; i < rows * half; i += kConsThreads) {
        const int row = i / half, pr = i - row * half;
        const int i0 = p.gptj ? 2 * pr : pr;
        const int i1 = p.gptj ? 2 * pr + 1 : pr + half;
        const float first = global_src ? __ldcg(src + row * kD + i0) : src[row * kD + i0];
        const float second = global_src ? __ldcg(src + row * kD + i1) : src[row * kD + i1];
        const float sn = sm.trig[pr], cs = sm.trig[half + pr];
        dst[row * kD + i0] = __fsub_rn(__fmul_rn(first, cs), __fmul_rn(second, sn));
        dst[row * kD + i1] = __fadd_rn(__fmul_rn(first, sn), __fmul_rn(second, cs));
    }
}

// ---- consumers: attention item ---------------------------------------------------

// Shared scratch of an attention item (aliases the digits, idle during the
// stage), in floats.
template <int G>
struct AttnScratch {
    static constexpr int kQ = 0;                    // [G][D] roped, scaled q
    static constexpr int kK = kQ + G * kD;          // [D] roped new key
    static constexpr int kV = kK + kD;              // [D] new value
    static constexpr int kMo = kV + kD;             // [kCons][G][D] warp partial outputs
    static constexpr int kMl = kMo + kCons * G * kD;  // [kCons][G][2] warp max / sum
    static constexpr int kW = kMl + kCons * G * 2;  // [G][kCons] warp weights
    static constexpr int kRmax = kW + G * kCons;    // [G] row maxima
    static constexpr int kOut = (kRmax + G + 3) / 4 * 4;  // [G][D] this kv head's output rows
    // The chunk merge splits the chunks of every output float4 over kParts
    // threads (all consumer threads busy): [kParts][G][D] partial sums.
    static constexpr int kParts = kConsThreads / (32 * G);
    static constexpr int kPart = kOut + G * kD;
    static constexpr int kEnd = kPart + kParts * G * kD;  // then [G][nchunk] x 2 + [G]
};

// Floats of the attention scratch for GQA group G and at most cap chunks
// per kv head (host and device agree).
__host__ __device__ inline int attn_scratch_floats(int G, int cap) {
    int end = 0;
    switch (G) {
        case 1: end = AttnScratch<1>::kEnd; break;
        case 2: end = AttnScratch<2>::kEnd; break;
        case 4: end = AttnScratch<4>::kEnd; break;
        default: end = AttnScratch<8>::kEnd; break;
    }
    return end + 2 * G * cap + G;
}

// The G attention-output rows of kv head kvh (in the scratch), as digit
// records of the o projection's input.
template <int FMT, int G>
__device__ __forceinline__ void digitize_heads(const DlArgs &p, const Smem &sm, int kvh) {
    cons_sync();  // the rows are in the scratch
    constexpr int kSteps = G * kD / Q<FMT>::kStep;
    const int s0 = kvh * kSteps;
    const float *rows = reinterpret_cast<const float *>(sm.dig) + AttnScratch<G>::kOut;
    digitize_steps<FMT, kInShared>(sm, s0, s0 + kSteps, rows, nullptr, nullptr, 0.f, p.digO);
}

template <int FMT, int G>
__device__ __forceinline__ void attention_item(const DlArgs &p, const Smem &sm, const DlLayer &ly,
                                               const AttnPlan &ap, unsigned &seq) {
    using S = AttnScratch<G>;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int item = blockIdx.x;
    const int kvh = item / ap.nchunk, chunk = item - kvh * ap.nchunk;
    const int k0 = chunk * ap.ck, k1 = min(ap.past + 1, k0 + ap.ck);
    const int nsl = (k1 - k0 + 15) / 16;
    float *scr = reinterpret_cast<float *>(sm.dig);
    float *qsm = scr + S::kQ, *knew = scr + S::kK, *vnew = scr + S::kV;
    // RoPE of the G query heads and of the new key, and the new value: every
    // load issued before any arithmetic (one round trip to L2).
    {
        constexpr int kHalf = kD / 2;
        constexpr int kItems = (G + 1) * kHalf + kD / 4;  // q pairs, k pairs, v float4
        const float *qsrc = p.Q + (long long)kvh * G * kD;
        const float *ksrc = p.Kp + (long long)kvh * kD;
        const float *vsrc = p.Vp + (long long)kvh * kD;
        constexpr int kPer = (kItems + kConsThreads - 1) / kConsThreads;
        float a[kPer], b[kPer];
        float4 v4[kPer];
#pragma unroll
        for (int j = 0; j < kPer; j++) {
            const int i = tid + j * kConsThreads;
            if (i < (G + 1) * kHalf) {
                const int row = i / kHalf, pr = i - row * kHalf;
                const float *src = row < G ? qsrc + row * kD : ksrc;
                const int i0 = p.gptj ? 2 * pr : pr, i1 = p.gptj ? 2 * pr + 1 : pr + kHalf;
                a[j] = __ldcg(src + i0);
                b[j] = __ldcg(src + i1);
            } else if (i < kItems) {
                v4[j] = __ldcg(reinterpret_cast<const float4 *>(vsrc) + (i - (G + 1) * kHalf));
            }
        }
        const float qscale = ly.scale;
#pragma unroll
        for (int j = 0; j < kPer; j++) {
            const int i = tid + j * kConsThreads;
            if (i < (G + 1) * kHalf) {
                const int row = i / kHalf, pr = i - row * kHalf;
                const int i0 = p.gptj ? 2 * pr : pr, i1 = p.gptj ? 2 * pr + 1 : pr + kHalf;
                const float sn = sm.trig[pr], cs = sm.trig[kHalf + pr];
                float r0 = __fsub_rn(__fmul_rn(a[j], cs), __fmul_rn(b[j], sn));
                float r1 = __fadd_rn(__fmul_rn(a[j], sn), __fmul_rn(b[j], cs));
                float *dst = row < G ? qsm + row * kD : knew;
                if (row < G) {  // q pre-scaled, as the attention reference scales scores
                    r0 *= qscale;
                    r1 *= qscale;
                }
                dst[i0] = r0;
                dst[i1] = r1;
            } else if (i < kItems) {
                reinterpret_cast<float4 *>(vnew)[i - (G + 1) * kHalf] = v4[j];
            }
        }
    }
    cons_sync();

    float4 q[G], o[G];
    float m[G], l[G];
#pragma unroll
    for (int r = 0; r < G; r++) {
        q[r] = reinterpret_cast<const float4 *>(qsm + r * kD)[lane];
        o[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        m[r] = -INFINITY;
        l[r] = 0.f;
    }
    const float4 kn = reinterpret_cast<const float4 *>(knew)[lane];
    const float4 vn = reinterpret_cast<const float4 *>(vnew)[lane];
    uint32_t *const err = p.err;
    const int past = ap.past;
    // Rounds of RS slots: warp w takes keys w and w + 8 of each slot of the
    // round (KPW keys, ascending), and the G x KPW scores of the round are
    // reduced across the warp by one transposed butterfly (each stage hands
    // half of the values a lane carries to its partner), after which lane
    // l holds the score of pair l / REP (row r = pair / KPW, key i = pair %
    // KPW).
    constexpr int KPW = (32 / G) < 8 ? (32 / G) : 8;
    constexpr int RS = KPW / 2;
    constexpr int NV = G * KPW, REP = 32 / NV;
    constexpr int LOG = NV == 32 ? 5 : NV == 16 ? 4 : NV == 8 ? 3 : 2;
    static_assert(NV <= 32 && (1 << LOG) == NV && RS >= 1, "pairs per round");
    for (int s0 = 0; s0 < nsl; s0 += RS) {
        const int ns = min(RS, nsl - s0);
        bool ok = true;
        for (int i = 0; i < ns; i++) ok = wait_full(err, sm, seq + i) && ok;
        if (ok) {
            // Keys of the round, ascending: the valid ones are a prefix (nk).
            float v[NV];
            int nk = 0;
#pragma unroll
            for (int i = 0; i < KPW; i++) {
                const int j = k0 + 16 * (s0 + i / 2) + warp + 8 * (i & 1);
                float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
                if (i / 2 < ns && j < k1) {
                    nk = i + 1;
                    if (j == past) {
                        kv = kn;
                    } else {
                        const unsigned char *sl = sm.ring + ((seq + i / 2) % kSlots) * kSlotBytes;
                        kv = reinterpret_cast<const float4 *>(sl + (warp + 8 * (i & 1)) * kD * 4)[lane];
                    }
                }
#pragma unroll
                for (int r = 0; r < G; r++)
                    v[r * KPW + i] = fmaf(q[r].w, kv.w, fmaf(q[r].z, kv.z, fmaf(q[r].y, kv.y, q[r].x * kv.x)));
            }
#pragma unroll
            for (int st = 0; st < LOG; st++) {
                const int half = NV >> (st + 1), sh = 16 >> st;
                const bool upper = (lane & sh) != 0;
#pragma unroll
                for (int k2 = 0; k2 < half; k2++) {
                    const float send = upper ? v[k2] : v[k2 + half];
                    const float keep = upper ? v[k2 + half] : v[k2];
                    v[k2] = keep + __shfl_xor_sync(0xffffffffu, send, sh);
                }
            }
#pragma unroll
            for (int sh = REP / 2; sh >= 1; sh >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], sh);
            const int idx = lane / REP, ri = idx / KPW, ii = idx - ri * KPW;
            const float sc = ii < nk ? v[0] : -INFINITY;
            float mb = sc;
#pragma unroll
            for (int sh = KPW * REP / 2; sh >= 1; sh >>= 1)
                mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, sh));
            float m_new[G];
            float m_own = 0.f;
#pragma unroll
            for (int r = 0; r < G; r++) {
                m_new[r] = fmaxf(m[r], __shfl_sync(0xffffffffu, mb, r * KPW * REP));
                if (r == ri) m_own = m_new[r];
            }
            const float p_own = sc == -INFINITY ? 0.f : expf(sc - m_own);
#pragma unroll
            for (int r = 0; r < G; r++) {
                const float alpha = m[r] == -INFINITY ? 0.f : expf(m[r] - m_new[r]);
                l[r] *= alpha;
                o[r].x *= alpha, o[r].y *= alpha, o[r].z *= alpha, o[r].w *= alpha;
                m[r] = m_new[r];
            }
            // Values are read when they are used.
#pragma unroll
            for (int i = 0; i < KPW; i++) {
                const int j = k0 + 16 * (s0 + i / 2) + warp + 8 * (i & 1);
                float4 vv = make_float4(0.f, 0.f, 0.f, 0.f);
                if (i < nk) {
                    if (j == past) {
                        vv = vn;
                    } else {
                        const unsigned char *sl = sm.ring + ((seq + i / 2) % kSlots) * kSlotBytes;
                        vv = reinterpret_cast<const float4 *>(sl + 16 * kD * 4 + (warp + 8 * (i & 1)) * kD * 4)[lane];
                    }
                }
#pragma unroll
                for (int r = 0; r < G; r++) {
                    const float pj = __shfl_sync(0xffffffffu, p_own, (r * KPW + i) * REP);
                    l[r] += pj;
                    o[r].x = fmaf(pj, vv.x, o[r].x);
                    o[r].y = fmaf(pj, vv.y, o[r].y);
                    o[r].z = fmaf(pj, vv.z, o[r].z);
                    o[r].w = fmaf(pj, vv.w, o[r].w);
                }
            }
        }
        for (int i = 0; i < ns; i++) release(sm, seq + i);
        seq += ns;
    }
    // The chunk holding the new position appends it (attention.rs:61-78
    // index arithmetic, batch 0).
    if (past >= k0 && past < k1 && warp == 0) {
        float *dst = p.cache + (long long)ly.cache_layer * p.lay_stride +
                     (long long)past * p.Hkv * kD + (long long)kvh * kD;
        reinterpret_cast<float4 *>(dst)[lane] = kn;
        reinterpret_cast<float4 *>(dst + p.par_stride)[lane] = vn;
    }
    // Warps merged in ascending order: per (row, warp) weight exp(m_w - M)
    // once, then every output the weighted sum over the warps.
    float *mo = scr + S::kMo, *mml = scr + S::kMl, *wgt = scr + S::kW, *rmax = scr + S::kRmax;
#pragma unroll
    for (int r = 0; r < G; r++) {
        reinterpret_cast<float4 *>(mo + (warp * G + r) * kD)[lane] = o[r];
        if (lane == 0) {
            mml[(warp * G + r) * 2] = m[r];
            mml[(warp * G + r) * 2 + 1] = l[r];
        }
    }
    cons_sync();
    if (tid < G * kCons) {
        const int r = tid / kCons, w = tid - r * kCons;
        float mm = -INFINITY;
#pragma unroll
        for (int x = 0; x < kCons; x++) mm = fmaxf(mm, mml[(x * G + r) * 2]);
        const float mw = mml[(w * G + r) * 2];
        wgt[r * kCons + w] = mw == -INFINITY ? 0.f : expf(mw - mm);
        if (w == 0) rmax[r] = mm;
    }
    cons_sync();
    for (int i = tid; i < G * kD; i += kConsThreads) {
        const int r = i / kD, d = i - r * kD;
        float ll = 0.f, acc = 0.f;
#pragma unroll
        for (int w = 0; w < kCons; w++) {
            const float f = wgt[r * kCons + w];
            ll = fmaf(mml[(w * G + r) * 2 + 1], f, ll);
            acc = fmaf(mo[(w * G + r) * kD + d], f, acc);
        }
        const long long row = (long long)kvh * G + r;
        if (!*sm.abort) {
            if (ap.nchunk == 1) {
                const float out = __fdiv_rn(acc, ll);
                p.ATT[row * kD + d] = out;
                scr[S::kOut + r * kD + d] = out;
            } else {
                p.part_o[(row * ap.nchunk + chunk) * kD + d] = acc;
                if (d == 0) {
                    p.part_ml[(row * ap.nchunk + chunk) * 2] = rmax[r];
                    p.part_ml[(row * ap.nchunk + chunk) * 2 + 1] = ll;
                }
            }
        }
    }
    if (ap.nchunk == 1) {
        digitize_heads<FMT, G>(p, sm, kvh);
        cons_sync();
        return;
    }
    // The last CTA of this kv head merges the chunks in ascending order.
    cons_sync();
    if (tid == 0) {
        const unsigned ticket = atom_acq_rel_add(p.sync + kSyncTickets + kvh, 1u);
        *sm.flag = ticket == (unsigned)(ap.nchunk - 1);
    }
    cons_sync();
    if (!*sm.flag) return;
    float *wt = scr + S::kEnd;        // [G][nchunk] chunk weights
    float *lt = wt + G * ap.nchunk;   // [G][nchunk] chunk denominators
    float *inv = lt + G * ap.nchunk;  // [G]
    const long long row0 = (long long)kvh * G;
    // Every output float4 of the G rows: its chunks split over kParts
    // threads (ascending ranges), the parts then added in ascending order.
    // The first batch of this thread's partials is loaded together with the
    // chunk maxima / sums, before the chunk weights are known.
    constexpr int kItems = G * kD / 4, kParts = S::kParts, kBatch = 16;
    static_assert(kItems * kParts == kConsThreads, "merge threads");
    const int mi = tid % kItems, part = tid / kItems;
    const int r = mi / (kD / 4), d4 = mi - r * (kD / 4);
    const int c0 = part * ap.nchunk / kParts, c1 = (part + 1) * ap.nchunk / kParts;
    const float4 *src =
        reinterpret_cast<const float4 *>(p.part_o + (row0 + r) * ap.nchunk * kD) + d4;
    float4 v[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; j++)
        v[j] = c0 + j < c1 ? __ldcg(src + (size_t)(c0 + j) * (kD / 4))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = tid; i < G * ap.nchunk; i += kConsThreads) {
        const int rr = i / ap.nchunk, cc = i - rr * ap.nchunk;
        const float2 ml = __ldcg(reinterpret_cast<const float2 *>(p.part_ml) + (row0 + rr) * ap.nchunk + cc);
        wt[i] = ml.x;
        lt[i] = ml.y;
    }
    cons_sync();
    if (warp < G) {
        const int rr = warp;
        float mm = -INFINITY;
        for (int cc = lane; cc < ap.nchunk; cc += 32) mm = fmaxf(mm, wt[rr * ap.nchunk + cc]);
        mm = warp_max(mm);
        __syncwarp();
        for (int cc = lane; cc < ap.nchunk; cc += 32) {
            const float mc = wt[rr * ap.nchunk + cc];
            wt[rr * ap.nchunk + cc] = mc == -INFINITY ? 0.f : expf(mc - mm);
        }
        __syncwarp();
        if (lane == 0) {
            float ll = 0.f;
            for (int cc = 0; cc < ap.nchunk; cc++)
                ll = fmaf(lt[rr * ap.nchunk + cc], wt[rr * ap.nchunk + cc], ll);
            inv[rr] = ll;
        }
    }
    cons_sync();
    {
        const float *w = wt + r * ap.nchunk;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int cb = c0; cb < c1; cb += kBatch) {
            if (cb != c0) {
#pragma unroll
                for (int j = 0; j < kBatch; j++)
                    v[j] = cb + j < c1 ? __ldcg(src + (size_t)(cb + j) * (kD / 4))
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int j = 0; j < kBatch; j++) {
                if (cb + j < c1) {
                    const float f = w[cb + j];
                    acc.x = fmaf(v[j].x, f, acc.x);
                    acc.y = fmaf(v[j].y, f, acc.y);
                    acc.z = fmaf(v[j].z, f, acc.z);
                    acc.w = fmaf(v[j].w, f, acc.w);
                }
            }
        }
        reinterpret_cast<float4 *>(scr + S::kPart)[part * kItems + mi] = acc;
        cons_sync();
        if (tid < kItems) {
            const float4 *pp = reinterpret_cast<const float4 *>(scr + S::kPart);
            float4 a = pp[tid];
#pragma unroll
            for (int q = 1; q < kParts; q++) {
                const float4 b = pp[q * kItems + tid];
                a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
            }
            const float den = inv[r];
            const float4 out = make_float4(__fdiv_rn(a.x, den), __fdiv_rn(a.y, den),
                                           __fdiv_rn(a.z, den), __fdiv_rn(a.w, den));
            if (!*sm.abort)
                reinterpret_cast<float4 *>(p.ATT + (row0 + r) * kD)[d4] = out;
            reinterpret_cast<float4 *>(scr + S::kOut + r * kD)[d4] = out;
        }
    }
    if (tid == 0) p.sync[kSyncTickets + kvh] = 0u;
    digitize_heads<FMT, G>(p, sm, kvh);
    cons_sync();
}

// ---- consumers: tensor-parallel all-reduce of a row-parallel stage ---------------
//
// Under tensor parallelism the o and down GEMVs produce partial sums over
// this rank's columns. Every rank uses the same tile partition, so CTA c
// owns the same output rows on every rank. Each value travels as one 8-byte
// word {float bits, exchange epoch} (an aligned 8-byte store is single-copy
// atomic, so a word that carries the current epoch carries its value): CTA
// c stores its rows into its slot in every peer's exchange region (plain
// NVLink stores, no fence, no separate flag), then polls (bounded) the
// peers' words for its rows in its own region and adds the ranks' partials
// in rank order (identical bits on every rank). Slots alternate by epoch
// parity: a rank writes a slot again two exchanges later, after it has
// received every peer's words of the exchange in between, which each peer
// sends only after it has read the slot.

__device__ __forceinline__ void st_u64(uint64_t *a, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t *a) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
    return v;
}

__device__ __noinline__ void tp_reduce_rows(const DlArgs &p, const Smem &sm, float *out, int r0,
                                            int r1, uint32_t epoch) {
    const int tid = threadIdx.x, world = p.tp_world, rank = p.tp_rank;
    const int par = (int)(epoch & 1u);
    const int n = r1 - r0;  // at most kConsThreads (checked on the host): one row a thread
    if (n == 0 || *sm.abort) return;  // the same CTA of every rank has no rows
    const size_t slot = (size_t)kDlTpHidden;  // words per (parity, source rank)
    float own = 0.f, acc = 0.f;
    bool ok = true;
    if (tid < n) {
        // This CTA's row of the partial (written before the CTA barrier that
        // ended the GEMV) into every peer's slot for this rank.
        own = out[r0 + tid];
        const uint64_t w = ((uint64_t)epoch << 32) | __float_as_uint(own);
        for (int q = 0; q < world; q++)
            if (q != rank)
                st_u64(p.xwords[q] + ((size_t)par * world + rank) * slot + r0 + tid, w);
        // The peers' words for the row, added in rank order.
        for (int q = 0; q < world; q++) {
            float v = own;
            if (q != rank) {
                const uint64_t *src = p.xwords[rank] + ((size_t)par * world + q) * slot + r0 + tid;
                uint64_t x = ld_relaxed_sys_u64(src);
                if ((uint32_t)(x >> 32) != epoch && ok) {
                    const uint64_t t0 = global_ns();
                    while ((uint32_t)((x = ld_relaxed_sys_u64(src)) >> 32) != epoch) {
                        if (*sm.abort ||
                            *reinterpret_cast<volatile unsigned *>(p.sync + kSyncAbort)) {
                            ok = false;
                            break;
                        }
                        if (global_ns() - t0 > kWaitNs) {
                            report_error(p.err, kErrWaitTimeout);
                            atomicExch(p.sync + kSyncAbort, 1u);
                            ok = false;
                            break;
                        }
                    }
                }
                v = __uint_as_float((uint32_t)x);
            }
            acc = __fadd_rn(acc, v);
        }
    }
    if (!ok) *sm.abort = 1;
    cons_sync();
    if (!*sm.abort && tid < n) out[r0 + tid] = acc;
}

// ---- consumers: the layer program --------------------------------------------------
//
// The scribe's phases, counted by the scribe word: S1(l) = 4l (the previous
// layer's f and x', this layer's h), ATTN(l) = 4l + 1 (q k v, their split
// and roped copies), O(l) = 4l + 2 (a, am), GU(l) = 4l + 3 (o, x1, h2). The
// word counts phases whose private values are copied, so a worker stage of
// layer l that overwrites such a value waits for the matching phase of
// layer l - 1 (QKV: ATTN, ATTN: O, O: GU) or of layer l (DOWN: S1).

// The scribe's program (the last CTA): every command output in command
// order, from private copies staged in its (idle) ring.
__device__ void scribe_program(const DlArgs &p, const Smem &sm) {
    const unsigned W = (unsigned)p.W;
    const int QD = p.Hq * kD, KD = p.Hkv * kD;
    float *stg = reinterpret_cast<float *>(sm.ring);
    load_smem(sm.resid, p.x0, p.H);
    cons_sync();
    for (int l = 0; l < p.L; l++) {
        const DlLayer &ly = p.layers[l];
        unsigned *ctr = p.sync + kSyncStages + kCtrs * l;
        // S1(l): the previous layer's f and x', then h.
        if (l > 0) {
            const DlLayer &prev = p.layers[l - 1];
            dep_wait(p, sm, ctr - kCtrs + cDOWN, W);
            load_smem(stg, p.F, p.H);
            cons_sync();
            scribe_signal(p);
            put_smem(prev, kDlF, stg, p.H);
            resid_add_smem(p, sm, stg);
            put_smem(prev, kDlXn, sm.resid, p.H);
        } else {
            scribe_signal(p);
        }
        const float inv1 = resid_inv_rms(p, sm, ly.eps1);
        put_norm(p, sm, ly, kDlH, ly.wn1, inv1);
        // ATTN(l): q k v, split copies, roped copies.
        dep_wait(p, sm, ctr + cQKV, W);
        load_smem(stg, p.Q, QD);
        load_smem(stg + QD, p.Kp, KD);
        load_smem(stg + QD + KD, p.Vp, KD);
        cons_sync();
        scribe_signal(p);
        put_smem(ly, kDlQ, stg, QD);
        put_smem(ly, kDlK, stg + QD, KD);
        put_smem(ly, kDlV, stg + QD + KD, KD);
        put_smem(ly, kDlQs, stg, QD);
        put_smem(ly, kDlKs, stg + QD, KD);
        put_smem(ly, kDlVs, stg + QD + KD, KD);
        order_sync(ly, kDlQr);
        if (ly.cmd[kDlQr]) rope_rows(p, sm, stg, ly.cmd[kDlQr], p.Hq, false);
        order_sync(ly, kDlKr);
        if (ly.cmd[kDlKr]) rope_rows(p, sm, stg + QD, ly.cmd[kDlKr], p.Hkv, false);
        // O(l): a, am.
        dep_wait(p, sm, ctr + cATTN, W);
        load_smem(stg, p.ATT, QD);
        cons_sync();
        scribe_signal(p);
        put_smem(ly, kDlA, stg, QD);
        put_smem(ly, kDlAm, stg, QD);
        // GU(l): o, x1, h2.
        dep_wait(p, sm, ctr + cO, W);
        load_smem(stg, p.O, p.H);
        cons_sync();
        scribe_signal(p);
        put_smem(ly, kDlO, stg, p.H);
        resid_add_smem(p, sm, stg);
        put_smem(ly, kDlX1, sm.resid, p.H);
        const float inv2 = resid_inv_rms(p, sm, ly.eps2);
        put_norm(p, sm, ly, kDlH2, ly.wn2, inv2);
    }
    // The last layer's SwiGlu output and final Add.
    const DlLayer &last = p.layers[p.L - 1];
    dep_wait(p, sm, p.sync + kSyncStages + kCtrs * (p.L - 1) + cDOWN, W);
    load_smem(stg, p.F, p.H);
    cons_sync();
    put_smem(last, kDlF, stg, p.H);
    resid_add_smem(p, sm, stg);
    put_smem(last, kDlXn, sm.resid, p.H);
}

// A worker's program: the layer stages, each ended by an arrival. The four
// GEMV stages share one code path (one copy of the GEMV loop and of the
// input digitization: the instruction cache holds the whole layer).
template <int FMT, int G>
__device__ void worker_program(const DlArgs &p, const Smem &sm) {
    const unsigned W = (unsigned)p.W;
    const unsigned *sc = p.sync + kSyncScribe;
    const int QD = p.Hq * kD;
    unsigned seq = 0, fetches = 0;
    // Launches before this one (advanced at the end of every launch; the
    // same count on every rank): numbers this launch's exchanges.
    const unsigned launch =
        p.tp_world > 1 ? *reinterpret_cast<volatile unsigned *>(p.tp_launches) : 0u;
    load_smem(sm.resid, p.x0, p.H);
    cons_sync();
    for (int l = 0; l < p.L; l++) {
        const DlLayer &ly = p.layers[l];
        unsigned *ctr = p.sync + kSyncStages + kCtrs * l;
        const unsigned g0 = 4u * (unsigned)l;
        for (int st = kQKV; st <= kDOWN; st++) {
            if (st == kATTN) {
                // ATTN (the merging CTAs also digitize the output rows).
                dep_wait(p, sm, ctr + cQKV, W, l == 0 ? nullptr : sc, g0 - 1);
                const AttnPlan ap = attn_plan(p, ly);
                if ((int)blockIdx.x < p.Hkv * ap.nchunk) attention_item<FMT, G>(p, sm, ly, ap, seq);
                arrive(ctr + cATTN);
                continue;
            }
            // The stage input as a digit vector in global memory.
            const unsigned char *dsrc;
            int K;
            if (st == kO) {
                dep_wait(p, sm, ctr + cATTN, W, l == 0 ? nullptr : sc, g0);
                dsrc = p.digO;
                K = QD;
            } else {
                // QKV: x = x1 + f, h = rmsnorm(x); GU: x1 = x + o, h2 =
                // rmsnorm(x1); DOWN: silu(gate) * up. Each worker digitizes
                // its share of the warp-steps, then waits for the others.
                if (st == kQKV) {
                    if (l > 0) {
                        dep_wait(p, sm, ctr - kCtrs + cDOWN, W);
                        resid_add(p, sm, p.F);
                    }
                } else if (st == kGU) {
                    dep_wait(p, sm, ctr + cO, W);
                    resid_add(p, sm, p.O);
                } else {
                    dep_wait(p, sm, ctr + cGU, W);
                }
                const bool down = st == kDOWN;
                K = down ? p.I : p.H;
                unsigned char *dst = down ? p.digD : p.digA;
                int s0, s1;
                my_steps<FMT>(p, K, &s0, &s1);
                if (down) {
                    digitize_steps<FMT, kInSwiglu>(sm, s0, s1, p.Gb, p.Ub, nullptr, 0.f, dst);
                } else {
                    const float inv = resid_inv_rms(p, sm, st == kQKV ? ly.eps1 : ly.eps2);
                    digitize_steps<FMT, kInNorm>(sm, s0, s1, nullptr, nullptr,
                                                 st == kQKV ? ly.wn1 : ly.wn2, inv, dst);
                }
                const int cd = st == kQKV ? cDQ : (st == kGU ? cDGU : cDD);
                arrive(ctr + cd);
                // QKV overwrites q k v (scribe phase ATTN(l - 1) read them);
                // DOWN overwrites f (S1(l) read the previous layer's).
                const unsigned *gate = st == kQKV ? (l == 0 ? nullptr : sc) : (down ? sc : nullptr);
                const unsigned gt = st == kQKV ? g0 - 2 : g0 + 1;
                dep_wait(p, sm, ctr + cd, W, gate, gt);
                dsrc = dst;
            }
            fetch_digits<FMT>(p, sm, dsrc, K, fetches);
            const StageGeo g = stage_geo<FMT>(p, st);
            gemv_tiles<FMT>(p, sm, g, seq);
            if (p.tp_world > 1 && (st == kO || st == kDOWN)) {
                // The rows' partial sums over this rank's columns, all-reduced.
                const int t0 = (int)((long long)blockIdx.x * g.tiles / p.W);
                const int t1 = (int)((long long)(blockIdx.x + 1) * g.tiles / p.W);
                tp_reduce_rows(p, sm, g.out0, 16 * t0, 16 * t1,
                               launch * 256u + 2u * (unsigned)l + (st == kDOWN ? 2u : 1u));
            }
            arrive(ctr + (st == kQKV ? cQKV : st == kO ? cO : st == kGU ? cGU : cDOWN));
        }
    }
    // A copy still in flight after giving up lands before the CTA exits
    // (bounded).
    if (threadIdx.x == 0 && fetches > 0) {
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(sm.dbar, (fetches - 1) & 1) && global_ns() - t0 < 100000000ull) {
        }
    }
}

template <int FMT, int G>
__global__ void __launch_bounds__(kThreads, 1) decode_layers_kernel(const __grid_constant__ DlArgs p) {
    extern __shared__ __align__(1024) unsigned char smem[];
    const Smem sm = carve(p, smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0 && blockIdx.x == 0)
        reinterpret_cast<unsigned long long *>(p.sync + kDecodeStampWord)[0] = global_ns();
    if (threadIdx.x == 0) {
        for (int i = 0; i < kSlots; i++) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], kCons);
        }
        mbar_init(sm.dbar, 1);
        fence_mbar_init();
        *sm.abort = 0;
        *sm.flag = 0;
    }
    // f32 sine / cosine of the f64 angles of the decode position (positions
    // are U32 data, written only by uploads).
    if (threadIdx.x < kD / 2) {
        const double angle = (double)p.pos[0] / p.denom[threadIdx.x];
        double sn, cs;
        sincos(angle, &sn, &cs);
        sm.trig[threadIdx.x] = (float)sn;
        sm.trig[kD / 2 + threadIdx.x] = (float)cs;
    }
    __syncthreads();
    if (warp >= kCons) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProdRegs));
        if (warp == kCons && lane == 0 && (int)blockIdx.x < p.W) {
            for (int l = 0; l < p.L && l < 2; l++)
                for (int m = 0; m < 7; m++) {
                    prefetch_tensormap(p.maps + p.layers[l].map[m]);
                }
            producer<FMT>(p, sm);
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsRegs));
        if ((int)blockIdx.x == p.W)
            scribe_program(p, sm);
        else
            worker_program<FMT, G>(p, sm);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned ticket = atomicAdd(p.sync + kSyncExit, 1u);
        if (ticket == gridDim.x - 1) {  // every CTA is past its last wait
            for (int i = 0; i < kSyncStages + kCtrs * p.L; i++)
                *reinterpret_cast<volatile unsigned *>(p.sync + i) = 0u;
            if (p.tp_world > 1) *p.tp_launches += 1u;
            reinterpret_cast<unsigned long long *>(p.sync + kDecodeStampWord)[1] = global_ns();
            __threadfence();
        }
    }
}

// ---- host ------------------------------------------------------------------------

struct Layout {
    int off_bar, off_misc, off_resid, off_dig, off_red, off_trig, dig_bytes, nch_max;
    size_t smem;
    int nchunk_cap;
};

int rowb_of(int fmt, size_t K) { return (int)(fmt == 0 ? K / 2 : K); }

// Code bytes per chunk of a stage whose rows hold K codes (0: the stage is
// not supported): the whole row when it fits one chunk (its scales then come
// by one bulk copy of the tile's contiguous scale rows), else the largest
// multiple of 128 bytes up to 1 KiB that divides the row and whose scale
// groups start 16-byte aligned (the scales' TMA box).
int chunk_bytes(int fmt, size_t K, size_t group) {
    const int kstep = fmt == 0 ? 128 : 64;
    if (K == 0 || K % (size_t)kstep != 0 || group % (size_t)kstep != 0 || K % group != 0)
        return 0;
    const int rowb = rowb_of(fmt, K);
    const int groups = (int)(K / group);
    if (rowb <= kChunk)
        return rowb % 64 == 0 && 16 * groups * 4 <= kSlotBytes - kSlotCode ? rowb : 0;
    if (groups % 4 != 0) return 0;  // the scales' row stride (TMA) is a multiple of 16 bytes
    // 1 KiB chunks, the last one ragged (the boxes read zero fill past the
    // row's end; its missing warp-steps are skipped).
    const int gpc1k = kChunk * (fmt == 0 ? 2 : 1) / (int)group;
    if (gpc1k >= 4 && gpc1k % 4 == 0 && gpc1k <= 16) return kChunk;
    for (int C = kChunk; C >= 128; C -= 128) {
        if (rowb % C != 0) continue;
        const int gpc = C * (fmt == 0 ? 2 : 1) / (int)group;
        if (gpc >= 4 && gpc % 4 == 0 && gpc <= 16) return C;
    }
    return 0;
}

bool stage_ok(int fmt, size_t K, size_t group, int *nch) {
    const int C = chunk_bytes(fmt, K, group);
    if (C == 0) return false;
    *nch = (rowb_of(fmt, K) + C - 1) / C;
    return true;
}

Layout layout_for(const DlRun &r, int sms) {
    Layout L{};
    const int fmt = r.format;
    int nch[4] = {0, 0, 0, 0};
    const size_t Ks[4] = {(size_t)r.hidden, (size_t)r.heads * kD, (size_t)r.hidden,
                          (size_t)r.inter};
    for (int i = 0; i < 4; i++)
        if (!stage_ok(fmt, Ks[i], r.group, &nch[i])) return Layout{};
    L.nch_max = *std::max_element(nch, nch + 4);
    const int wsb = fmt == 0 ? 128 : 64;
    const int kstep = fmt == 0 ? 128 : 64;
    const size_t rec = 3 * (size_t)wsb + 32;
    // The digit vector of the longest stage input (whole-vector copy).
    const size_t kmax = std::max<size_t>(std::max<size_t>(r.hidden, (size_t)r.heads * kD), r.inter);
    L.dig_bytes = (int)(kmax / kstep * rec);
    const int W = sms - 1;
    L.nchunk_cap = W / (int)r.kv_heads;
    const int G = (int)(r.heads / r.kv_heads);
    // The attention scratch (aliasing the digits) must fit as well.
    const size_t attn_floats = (size_t)attn_scratch_floats(G, L.nchunk_cap);
    size_t dig_region = (size_t)L.dig_bytes;
    if (attn_floats * 4 > dig_region) dig_region = attn_floats * 4;
    dig_region = (dig_region + 15) / 16 * 16;
    size_t off = (size_t)kSlots * kSlotBytes;
    L.off_bar = (int)off;
    off += (2 * kSlots + 2) * 8;
    L.off_misc = (int)off;
    off += 16 + kCons * 4 + 16;
    off = (off + 15) / 16 * 16;
    L.off_resid = (int)off;
    off += (size_t)r.hidden * 4;
    L.off_dig = (int)off;
    off += dig_region;
    L.off_red = (int)off;
    off += (size_t)kRedTiles * kCons * 16 * 4;
    L.off_trig = (int)off;
    off += kD * 4;
    L.smem = off;
    return L;
}

bool weight_ok(const QuantWeight &w, size_t n, size_t K, int fmt, size_t group) {
    return w.codes && w.scales && w.n == n && w.k == K && (int)w.format == fmt &&
           w.group == group && w.groups == K / group && w.row_bytes == (size_t)rowb_of(fmt, K) &&
           n % 16 == 0 && aligned16(w.codes) && aligned16(w.scales) && n <= (1u << 24);
}

struct ImageHeader {
    int layers;
};

size_t maps_bytes(int layers) { return (size_t)layers * 14 * sizeof(CUtensorMap); }

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return 0;
    return n;
}

}  // namespace

size_t decode_layers_image_bytes(int layers) {
    return maps_bytes(layers) + (size_t)layers * sizeof(DlLayer);
}

size_t decode_layers_scratch_bytes(const DlRun &r) {
    const int sms = sm_count();
    if (sms < 2) return 0;
    const int nchunk_cap = (sms - 1) / (int)(r.kv_heads ? r.kv_heads : 1);
    const size_t qd = r.heads * kD, kd = r.kv_heads * kD;
    const size_t floats = qd + 2 * kd + qd + r.hidden + 2 * r.inter + r.hidden +
                          qd * nchunk_cap + r.heads * nchunk_cap * 2 + 64 * 16;
    const size_t kstep = r.format == 0 ? 128 : 64, rec = 3 * (r.format == 0 ? 128 : 64) + 32;
    const size_t digit_bytes = (r.hidden + qd + r.inter) / kstep * rec;
    return floats * 4 + digit_bytes + 3 * 256;
}

bool decode_layers_supported(const DlRun &r) {
    const int sms = sm_count();
    if (sms < 2 || r.layers < 1 || r.layers > kMaxLayers || r.head_dim != kD || r.kv_heads == 0 ||
        r.heads % r.kv_heads != 0 || r.kv_heads > 32 || r.format < 0 || r.format > 1)
        return false;
    const size_t G = r.heads / r.kv_heads;
    if (G != 1 && G != 2 && G != 4 && G != 8) return false;
    if (r.hidden % 1024 != 0 || r.hidden > 16384 || r.inter % 16 != 0 || !r.x0 || !r.pos ||
        !r.cache || r.max_seq == 0 || r.max_seq > (1u << 24) || r.cache_layers == 0 ||
        (size_t)r.cache_layers * 2 * r.max_seq > (1u << 30) || (size_t)sms - 1 < r.kv_heads)
        return false;
    const Layout L = layout_for(r, sms);
    if (L.smem == 0 || L.smem > (size_t)kSmemLimit || !aligned16(r.x0)) return false;
    // Tensor parallelism: every rank's exchange region mapped, one flag per
    // CTA, the hidden row within a slot.
    if (r.tp.world > 1) {
        if (r.tp.world > kMaxPeers || r.tp.rank < 0 || r.tp.rank >= r.tp.world ||
            r.hidden > (uint32_t)kDlTpHidden ||
            16 * ((r.hidden / 16 + (sms - 1) - 1) / (sms - 1)) > (uint32_t)kConsThreads)
            return false;  // a worker's rows of o / down: one a consumer thread
        for (int q = 0; q < r.tp.world; q++)
            if (!r.tp.words[q] || !aligned16(r.tp.words[q])) return false;
        if (!r.tp.launches) return false;
    }
    // The scribe stages q, k and v in its (idle) ring.
    if (((size_t)r.heads + 2 * r.kv_heads) * kD * 4 > (size_t)kSlots * kSlotBytes) return false;
    const size_t H = r.hidden, QD = r.heads * kD, KD = r.kv_heads * kD, I = r.inter;
    for (uint32_t l = 0; l < r.layers; l++) {
        const DlLayerIo &io = r.layer[l];
        const size_t n[7] = {QD, KD, KD, H, I, I, H};
        const size_t K[7] = {H, H, H, QD, H, H, I};
        for (int m = 0; m < 7; m++)
            if (!weight_ok(io.w[m], n[m], K[m], r.format, r.group)) return false;
        if (!io.wn1 || !io.wn2 || io.cache_layer >= r.cache_layers ||
            (!io.d_past && io.past >= r.max_seq))
            return false;
        // The scribe stores float4.
        for (int c = 0; c < kDlCmds; c++)
            if (io.cmd[c] && !aligned16(io.cmd[c])) return false;
        // Each layer appends to and reads its own cache layer (an appended
        // key is never read back through TMA in the same launch).
        for (uint32_t j = 0; j < l; j++)
            if (r.layer[j].cache_layer == io.cache_layer) return false;
    }
    return true;
}

bool decode_layers_image(const DlRun &r, void *host_image, size_t bytes, const void *dev_image) {
    if (bytes < decode_layers_image_bytes((int)r.layers)) return false;
    CUtensorMap *maps = static_cast<CUtensorMap *>(host_image);
    DlLayer *layers = reinterpret_cast<DlLayer *>(static_cast<char *>(host_image) +
                                                  maps_bytes((int)r.layers));
    for (uint32_t l = 0; l < r.layers; l++) {
        const DlLayerIo &io = r.layer[l];
        DlLayer &d = layers[l];
        memset(&d, 0, sizeof(d));
        for (int m = 0; m < 7; m++) {
            const QuantWeight &w = io.w[m];
            const int rowb = (int)w.row_bytes;
            const int C = chunk_bytes(r.format, w.k, r.group);
            if (C == 0) return false;
            const int gpc = C * (r.format == 0 ? 2 : 1) / (int)r.group;
            const int idx = (int)(l * 14 + 2 * m);
            // Boxes of the slot row strides (codes in 8-byte units: a padded
            // row of 1088 bytes is 136 elements, within the 256 a box allows).
            // Single-chunk rows take their scales by bulk copy (no map).
            const int Cp = slot_code_stride(rowb, C), gps = slot_scale_stride(rowb, C, gpc);
            if (!encode_tensor_map_2d(&maps[idx], CU_TENSOR_MAP_DATA_TYPE_UINT64, w.codes,
                                      (uint64_t)rowb / 8, w.n, (uint64_t)rowb, (uint32_t)Cp / 8,
                                      16))
                return false;
            memset(&maps[idx + 1], 0, sizeof(CUtensorMap));
            if (rowb > C && !encode_tensor_map_2d(&maps[idx + 1], CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                                                  w.scales, w.groups, w.n, w.groups * 4,
                                                  (uint32_t)gps, 16))
                return false;
            d.scales[m] = w.scales;
            d.map[m] = idx;
        }
        d.cache_layer = (int)io.cache_layer;
        d.wn1 = io.wn1;
        d.wn2 = io.wn2;
        d.eps1 = io.eps1;
        d.eps2 = io.eps2;
        d.scale = io.scale;
        d.d_past = io.d_past;
        d.past = io.past;
        for (int c = 0; c < kDlCmds; c++) d.cmd[c] = io.cmd[c];
    }
    // Barriers the scribe needs: an output that shares bytes with an earlier
    // output of the same scribe phase is written after a barrier.
    const size_t H = r.hidden, QD = (size_t)r.heads * kD, KD = (size_t)r.kv_heads * kD;
    const size_t len[kDlCmds] = {H, QD, KD, KD, QD, KD, KD, QD, KD, QD, QD, H, H, H, H, H};
    auto hit = [&](uint32_t la, int ca, uint32_t lb, int cb) {
        const char *a = reinterpret_cast<const char *>(r.layer[la].cmd[ca]);
        const char *b = reinterpret_cast<const char *>(r.layer[lb].cmd[cb]);
        if (!a || !b) return false;
        return a < b + 4 * len[cb] && b < a + 4 * len[ca];
    };
    for (uint32_t l = 0; l < r.layers; l++) {
        uint32_t order = 0;
        const int phases[3][8] = {{kDlQ, kDlK, kDlV, kDlQs, kDlKs, kDlVs, kDlQr, kDlKr},
                                  {kDlA, kDlAm, -1}, {kDlO, kDlX1, kDlH2, -1}};
        for (const auto &ph : phases)
            for (int i = 1; i < 8 && ph[i] >= 0; i++)
                for (int j = 0; j < i; j++)
                    if (hit(l, ph[i], l, ph[j])) order |= 1u << ph[i];
        // Phase S1(l + 1): this layer's f and x', then the next layer's h.
        if (hit(l, kDlXn, l, kDlF)) order |= 1u << kDlXn;
        if (l > 0 && (hit(l, kDlH, l - 1, kDlF) || hit(l, kDlH, l - 1, kDlXn))) order |= 1u << kDlH;
        layers[l].order = order;
    }
    (void)dev_image;
    return true;
}

cudaError_t decode_layers(cudaStream_t s, const DlRun &r, const void *dev_image, void *scratch,
                          size_t scratch_bytes, unsigned *sync, uint32_t *err) {
    const int sms = sm_count();
    if (!decode_layers_supported(r) || !dev_image || !sync ||
        scratch_bytes < decode_layers_scratch_bytes(r) || !aligned16(scratch))
        return cudaErrorInvalidValue;
    const Layout L = layout_for(r, sms);
    DlArgs a;
    memset(&a, 0, sizeof(a));
    const uint64_t dims[3] = {kD, r.kv_heads, (uint64_t)r.cache_layers * 2 * r.max_seq};
    const uint64_t strides[2] = {(uint64_t)kD * 4, (uint64_t)r.kv_heads * kD * 4};
    const uint32_t box[3] = {kD, 1, 16};
    if (!encode_tensor_map_3d(&a.kv_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, r.cache, dims, strides,
                              box))
        return cudaErrorInvalidValue;
    a.maps = static_cast<const CUtensorMap *>(dev_image);
    a.layers = reinterpret_cast<const DlLayer *>(static_cast<const char *>(dev_image) +
                                                 maps_bytes((int)r.layers));
    a.x0 = r.x0;
    a.pos = r.pos;
    a.cache = r.cache;
    const size_t qd = r.heads * kD, kd = r.kv_heads * kD;
    float *f = static_cast<float *>(scratch);
    auto take = [&](size_t n) {
        float *p = f;
        f += (n + 15) / 16 * 16;
        return p;
    };
    a.Q = take(qd);
    a.Kp = take(kd);
    a.Vp = take(kd);
    a.ATT = take(qd);
    a.O = take(r.hidden);
    a.Gb = take(r.inter);
    a.Ub = take(r.inter);
    a.F = take(r.hidden);
    a.part_o = take(qd * L.nchunk_cap);
    a.part_ml = take((size_t)r.heads * L.nchunk_cap * 2);
    const size_t kstep = r.format == 0 ? 128 : 64, rec = 3 * (r.format == 0 ? 128 : 64) + 32;
    a.digA = reinterpret_cast<unsigned char *>(take(r.hidden / kstep * rec / 4));
    a.digO = reinterpret_cast<unsigned char *>(take(qd / kstep * rec / 4));
    a.digD = reinterpret_cast<unsigned char *>(take(r.inter / kstep * rec / 4));
    a.sync = sync;
    a.err = err;
    a.par_stride = (long long)r.max_seq * r.kv_heads * kD;
    a.lay_stride = 2 * a.par_stride;
    a.L = (int)r.layers;
    a.H = (int)r.hidden;
    a.Hq = (int)r.heads;
    a.Hkv = (int)r.kv_heads;
    a.I = (int)r.inter;
    a.G = (int)(r.heads / r.kv_heads);
    a.group = (int)r.group;
    a.gptj = r.gptj;
    a.max_seq = (int)r.max_seq;
    a.W = sms - 1;
    a.nchunk_cap = L.nchunk_cap;
    a.stC[kQKV] = chunk_bytes(r.format, r.hidden, r.group);
    a.stC[kATTN] = 0;
    a.stC[kO] = chunk_bytes(r.format, qd, r.group);
    a.stC[kGU] = chunk_bytes(r.format, r.hidden, r.group);
    a.stC[kDOWN] = chunk_bytes(r.format, r.inter, r.group);
    a.tp_rank = r.tp.world > 1 ? r.tp.rank : 0;
    a.tp_world = r.tp.world > 1 ? r.tp.world : 1;
    for (int q = 0; q < kMaxPeers; q++) a.xwords[q] = q < a.tp_world ? r.tp.words[q] : nullptr;
    a.tp_launches = a.tp_world > 1 ? r.tp.launches : nullptr;
    a.dig_bytes = L.dig_bytes;
    a.nch_max = L.nch_max;
    a.off_bar = L.off_bar;
    a.off_misc = L.off_misc;
    a.off_resid = L.off_resid;
    a.off_dig = L.off_dig;
    a.off_red = L.off_red;
    a.off_trig = L.off_trig;
    for (int pr = 0; pr < kD / 2; pr++)
        a.denom[pr] = pow((double)r.theta, 2.0 * (double)pr / (double)kD);

    void (*kern)(DlArgs) = nullptr;
    const int G = a.G;
    if (r.format == 0)
        kern = G == 1 ? decode_layers_kernel<0, 1> : G == 2 ? decode_layers_kernel<0, 2>
             : G == 4 ? decode_layers_kernel<0, 4> : decode_layers_kernel<0, 8>;
    else
        kern = G == 1 ? decode_layers_kernel<1, 1> : G == 2 ? decode_layers_kernel<1, 2>
             : G == 4 ? decode_layers_kernel<1, 4> : decode_layers_kernel<1, 8>;
    static std::atomic<uint64_t> smem_set[2][4];
    const int gi = G == 1 ? 0 : G == 2 ? 1 : G == 4 ? 2 : 3;
    cudaError_t e = set_smem_limit_once(kern, kSmemLimit, &smem_set[r.format][gi]);
    if (e != cudaSuccess) return e;
    // One CTA per SM must fit (registers, shared memory), or the cooperative
    // launch is refused.
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, L.smem);
    if (e != cudaSuccess || per_sm < 1) return e != cudaSuccess ? e : cudaErrorInvalidConfiguration;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a);
    count_launch();
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace k
}  // namespace slc
