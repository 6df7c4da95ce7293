// KV-cache append and causal attention with a KV cache
// (crates/backends/backend-cpu/src/reference/attention.rs:33-219).
//
// Cache layout (reference, attention.rs:10-21):
//   cache[batch, layers, 2, max_seq, kv_heads, head_dim]
// index [b, layer, 0, t, h, :] holds keys, [b, layer, 1, t, h, :] values.
// The append writes positions past_len .. past_len + seq of `layer`; the
// index arithmetic is the reference's (attention.rs:61-78), so the cache
// contents are bit-exact.
//
// Attention (split-K, "flash-decoding"): the keys visible to any query of a
// CTA are cut into chunks; one CTA handles one (batch, kv_head, block of
// query heads sharing that kv_head (GQA), block of query positions, key
// chunk). K/V tiles of 32 keys are staged in shared memory once and used by
// every query row of the CTA (all GQA heads), scores and probabilities stay
// in shared memory, and the running max / denominator / weighted sum are
// updated online per tile. With more than one chunk, each CTA writes its
// (max, denominator, unnormalised output) to the workspace and a combine
// kernel merges the chunks in ascending order; with one chunk the CTA
// normalises and writes the output directly.
//
// Decode is HBM-bound on the KV read: algorithmic bytes per layer
// 2 * 4 * batch * kv_heads * (past_len + 1) * head_dim (+ q and out).
//
// Decode (seq == 1, head_dim 64 or 128, up to 8 query heads per KV head)
// has its own kernel, attention_decode: the append and the attention are
// one launch (the CTA whose chunk holds the new key reads it from the k / v
// inputs and writes it to the cache), each lane owns head_dim / 32
// consecutive dimensions of every GQA query row and of the K / V rows it
// streams (128-bit loads, 4 keys per warp in flight), scores are warp sums,
// and the chunks of one (batch, kv_head) are merged in ascending order by the
// last CTA to finish (atomic ticket, no waiting). With a device-resident
// past_len (graph replay) the grid is planned for max_seq and chunks beyond
// the live keys only take their ticket.
#include <math.h>

#include "common.cuh"
#include "kernels.h"
#include "tma.cuh"

namespace slc {
namespace k {
namespace {

constexpr int kThreads = 128;
constexpr int kTileKeys = 32;
constexpr int kMaxRows = 32;  // query rows (GQA heads x positions) per CTA

__global__ void __launch_bounds__(256) kv_append_kernel(const float *__restrict__ k,
                                                        const float *__restrict__ v,
                                                        float *__restrict__ cache, size_t batch,
                                                        size_t layers, size_t layer,
                                                        size_t kv_heads, size_t head_dim,
                                                        size_t max_seq, size_t past_len,
                                                        size_t seq, const uint32_t *d_past,
                                                        uint32_t *err) {
    pdl_trigger();
    pdl_wait();
    if (d_past) {
        past_len = *d_past;
        if (past_len + seq > max_seq) {  // validated on the host; guard anyway
            report_error(err, kErrBadScalar);
            return;
        }
    }
    const size_t time_stride = kv_heads * head_dim;
    const size_t parity_stride = max_seq * time_stride;
    const size_t layer_stride = 2 * parity_stride;
    const size_t batch_stride = layers * layer_stride;
    const size_t total = batch * kv_heads * seq * head_dim;
    size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        size_t d = i % head_dim, r = i / head_dim;
        size_t t = r % seq, bh = r / seq, h = bh % kv_heads, b = bh / kv_heads;
        size_t dst = b * batch_stride + layer * layer_stride + (past_len + t) * time_stride +
                     h * head_dim + d;
        cache[dst] = k[i];
        cache[dst + parity_stride] = v[i];
    }
}

struct AttnParams {
    const float *q;
    const float *cache;
    float *out;
    float *part_o;   // [rows_total][chunks][head_dim]
    float *part_ml;  // [rows_total][chunks][2]
    size_t batch, heads, kv_heads, seq, past_len, head_dim;
    size_t key_base_layer;  // layer * layer_stride
    size_t batch_stride, parity_stride, time_stride;
    size_t group, g_block, t_block, chunk_keys, chunks;
    float scale;
    const uint32_t *d_past;  // device past_len (graph replay) or null
};

__global__ void __launch_bounds__(kThreads) attention_kernel(AttnParams p) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float smem[];
    const size_t D = p.head_dim;
    const int R_MAX = kMaxRows;
    float *q_s = smem;                                  // [R][D]
    float *k_s = q_s + R_MAX * D;                       // [TK][D+1]
    float *v_s = k_s + kTileKeys * (D + 1);             // [TK][D]
    float *s_s = v_s + kTileKeys * D;                   // [R][TK]
    float *o_s = s_s + R_MAX * kTileKeys;               // [R][D]
    float *m_s = o_s + R_MAX * D;                       // [R]
    float *l_s = m_s + R_MAX;                           // [R]
    float *a_s = l_s + R_MAX;                           // [R]

    // Decode the CTA coordinates: x = chunk, y = (g_blk, t_blk), z = (b, kvh).
    const size_t chunk = blockIdx.x;
    const size_t n_gblk = (p.group + p.g_block - 1) / p.g_block;
    const size_t g_blk = blockIdx.y % n_gblk, t_blk = blockIdx.y / n_gblk;
    const size_t b = blockIdx.z / p.kv_heads, kvh = blockIdx.z % p.kv_heads;
    const size_t g0 = g_blk * p.g_block;
    const size_t gn = min(p.g_block, p.group - g0);
    const size_t t0 = t_blk * p.t_block;
    const size_t tn = min(p.t_block, p.seq - t0);
    const int rows = (int)(gn * tn);  // row r = tq * gn + gi

    const size_t past_len = p.d_past ? (size_t)*p.d_past : p.past_len;
    const size_t key_begin = chunk * p.chunk_keys;
    const size_t last_key = past_len + t0 + tn - 1;  // largest visible key of this CTA
    size_t key_end = min(key_begin + p.chunk_keys, last_key + 1);

    // Load the query rows.
    for (size_t i = threadIdx.x; i < (size_t)rows * D; i += kThreads) {
        size_t r = i / D, d = i - r * D;
        size_t gi = r % gn, tq = r / gn;
        size_t h = kvh * p.group + g0 + gi, t = t0 + tq;
        q_s[i] = p.q[((b * p.heads + h) * p.seq + t) * D + d];
    }
    for (size_t i = threadIdx.x; i < (size_t)rows * D; i += kThreads) o_s[i] = 0.f;
    for (int r = threadIdx.x; r < rows; r += kThreads) {
        m_s[r] = -INFINITY;
        l_s[r] = 0.f;
    }
    __syncthreads();

    const float *kbase = p.cache + b * p.batch_stride + p.key_base_layer + kvh * D;
    const float *vbase = kbase + p.parity_stride;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    for (size_t j0 = key_begin; j0 < key_end; j0 += kTileKeys) {
        const int tk = (int)min((size_t)kTileKeys, key_end - j0);
        // Stage K and V tiles (each key row is head_dim contiguous floats).
        for (size_t i = threadIdx.x; i < (size_t)tk * D; i += kThreads) {
            size_t j = i / D, d = i - j * D;
            size_t off = (j0 + j) * p.time_stride + d;
            k_s[j * (D + 1) + d] = kbase[off];
            v_s[j * D + d] = vbase[off];
        }
        __syncthreads();
        // Scores with the causal mask of each row.
        for (int i = threadIdx.x; i < rows * kTileKeys; i += kThreads) {
            int r = i / kTileKeys, j = i - r * kTileKeys;
            size_t tq = (size_t)r / gn;
            size_t limit = past_len + t0 + tq;  // keys 0..=limit visible
            float sc = -INFINITY;
            if (j < tk && j0 + j <= limit) {
                const float *qr = q_s + (size_t)r * D;
                const float *kr = k_s + (size_t)j * (D + 1);
                float acc = 0.f;
                for (size_t d = 0; d < D; d++) acc = fmaf(qr[d], kr[d], acc);
                sc = acc * p.scale;
            }
            s_s[r * kTileKeys + j] = sc;
        }
        __syncthreads();
        // Online softmax update, one warp per row.
        for (int r = warp; r < rows; r += kThreads / 32) {
            float sc = s_s[r * kTileKeys + lane];
            float tile_max = warp_max(sc);
            float m_old = m_s[r];
            float m_new = fmaxf(m_old, tile_max);
            float pj = (sc == -INFINITY) ? 0.f : expf(sc - m_new);
            float psum = warp_sum(pj);
            s_s[r * kTileKeys + lane] = pj;
            if (lane == 0) {
                float alpha = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
                a_s[r] = alpha;
                l_s[r] = l_s[r] * alpha + psum;
                m_s[r] = m_new;
            }
        }
        __syncthreads();
        // O = alpha * O + P . V
        for (size_t i = threadIdx.x; i < (size_t)rows * D; i += kThreads) {
            size_t r = i / D, d = i - r * D;
            const float *pr = s_s + r * kTileKeys;
            float acc = o_s[i] * a_s[r];
            for (int j = 0; j < tk; j++) acc = fmaf(pr[j], v_s[(size_t)j * D + d], acc);
            o_s[i] = acc;
        }
        __syncthreads();
    }

    // Write the result (single chunk) or the chunk partials.
    for (size_t i = threadIdx.x; i < (size_t)rows * D; i += kThreads) {
        size_t r = i / D, d = i - r * D;
        size_t gi = r % gn, tq = r / gn;
        size_t h = kvh * p.group + g0 + gi, t = t0 + tq;
        size_t row = (b * p.heads + h) * p.seq + t;
        if (p.chunks == 1) {
            p.out[row * D + d] = __fdiv_rn(o_s[i], l_s[r]);
        } else {
            p.part_o[(row * p.chunks + chunk) * D + d] = o_s[i];
            if (d == 0) {
                p.part_ml[(row * p.chunks + chunk) * 2 + 0] = m_s[r];
                p.part_ml[(row * p.chunks + chunk) * 2 + 1] = l_s[r];
            }
        }
    }
}

// Merge the chunk partials of every (b, h, t) row, chunks in ascending order.
__global__ void __launch_bounds__(128) attention_combine(const float *__restrict__ part_o,
                                                         const float *__restrict__ part_ml,
                                                         float *__restrict__ out, size_t rows,
                                                         size_t chunks, size_t head_dim) {
    pdl_trigger();
    pdl_wait();
    for (size_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const float *ml = part_ml + row * chunks * 2;
        float m = -INFINITY;
        for (size_t c = 0; c < chunks; c++) m = fmaxf(m, ml[2 * c]);
        float l = 0.f;
        for (size_t c = 0; c < chunks; c++)
            if (ml[2 * c] != -INFINITY) l += ml[2 * c + 1] * expf(ml[2 * c] - m);
        for (size_t d = threadIdx.x; d < head_dim; d += blockDim.x) {
            float acc = 0.f;
            for (size_t c = 0; c < chunks; c++)
                if (ml[2 * c] != -INFINITY)
                    acc = fmaf(part_o[(row * chunks + c) * head_dim + d], expf(ml[2 * c] - m), acc);
            out[row * head_dim + d] = __fdiv_rn(acc, l);
        }
    }
}

struct Plan {
    size_t g_block, t_block, chunk_keys, chunks, grid_y;
    size_t smem;
};

Plan plan(size_t batch, size_t heads, size_t kv_heads, size_t seq, size_t past_len,
          size_t head_dim) {
    Plan pl{};
    size_t group = heads / kv_heads;
    pl.g_block = group < (size_t)kMaxRows ? group : (size_t)kMaxRows;
    pl.t_block = kMaxRows / pl.g_block;
    if (pl.t_block < 1) pl.t_block = 1;
    if (pl.t_block > seq) pl.t_block = seq;
    size_t n_gblk = (group + pl.g_block - 1) / pl.g_block;
    size_t n_tblk = (seq + pl.t_block - 1) / pl.t_block;
    pl.grid_y = n_gblk * n_tblk;
    size_t max_keys = past_len + seq;
    size_t ctas = batch * kv_heads * pl.grid_y;
    // Enough chunks to give every SM two CTAs, each chunk at least 64 keys.
    size_t want = (2 * (size_t)kSmCount + ctas - 1) / ctas;
    size_t by_len = (max_keys + 63) / 64;
    pl.chunks = want < by_len ? want : by_len;
    if (pl.chunks < 1) pl.chunks = 1;
    pl.chunk_keys = (max_keys + pl.chunks - 1) / pl.chunks;
    pl.chunk_keys = (pl.chunk_keys + kTileKeys - 1) / kTileKeys * kTileKeys;
    pl.chunks = (max_keys + pl.chunk_keys - 1) / pl.chunk_keys;
    pl.smem = sizeof(float) * (kMaxRows * head_dim + kTileKeys * (head_dim + 1) +
                               kTileKeys * head_dim + kMaxRows * kTileKeys +
                               kMaxRows * head_dim + 3 * kMaxRows);
    return pl;
}


// ---- decode -------------------------------------------------------------------

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecMaxGroup = 8;
constexpr int kDecKeysPerWarp = 4;  // keys in flight per warp
constexpr int kDecMaxChunks = 128;  // chunks per (batch, kv_head)

struct DecodeParams {
    const float *q;        // [B, H, 1, D]
    const float *k_new;    // [B, Hkv, 1, D]
    const float *v_new;
    float *cache;
    float *out;            // [B, H, 1, D]
    float *out2;           // optional second copy of out (merged heads, same layout at seq 1)
    int early;             // cached keys may be read before the dependency wait
    float *part_o;         // [B * H][chunks][D]
    float *part_ml;        // [B * H][chunks][2]
    unsigned *tickets;     // [B * Hkv]
    const uint32_t *d_past;  // device past_len (graph replay) or null
    uint32_t *err;
    long long batch_stride, layer_off, parity_stride, time_stride;
    int past, max_seq;
    int H, Hkv, G, chunk_keys, chunks;
    float scale;
};

template <int VEC>
struct Vec;
template <>
struct Vec<2> {
    using T = float2;
    __device__ static T ld(const float *p) { return *reinterpret_cast<const float2 *>(p); }
    __device__ static void st(float *p, T v) { *reinterpret_cast<float2 *>(p) = v; }
    __device__ static float dot(T a, T b) { return fmaf(a.y, b.y, a.x * b.x); }
    __device__ static void axpby(T &o, float a, float p, T v) {
        o.x = fmaf(p, v.x, o.x * a);
        o.y = fmaf(p, v.y, o.y * a);
    }
    __device__ static float get(T v, int i) { return i == 0 ? v.x : v.y; }
    __device__ static void set(T &v, int i, float x) { (i == 0 ? v.x : v.y) = x; }
    __device__ static T zero() { return make_float2(0.f, 0.f); }
};
template <>
struct Vec<4> {
    using T = float4;
    __device__ static T ld(const float *p) { return *reinterpret_cast<const float4 *>(p); }
    __device__ static void st(float *p, T v) { *reinterpret_cast<float4 *>(p) = v; }
    __device__ static float dot(T a, T b) {
        return fmaf(a.w, b.w, fmaf(a.z, b.z, fmaf(a.y, b.y, a.x * b.x)));
    }
    __device__ static void axpby(T &o, float a, float p, T v) {
        o.x = fmaf(p, v.x, o.x * a);
        o.y = fmaf(p, v.y, o.y * a);
        o.z = fmaf(p, v.z, o.z * a);
        o.w = fmaf(p, v.w, o.w * a);
    }
    __device__ static float get(T v, int i) {
        return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
    }
    __device__ static void set(T &v, int i, float x) {
        (i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w))) = x;
    }
    __device__ static T zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
};

// G: query heads per KV head; KPW: keys per warp loaded in one batch (all
// of a 32-key chunk for G <= 4).
template <int VEC, int G, int KPW>
__global__ void __launch_bounds__(kDecThreads) attention_decode(DecodeParams p) {
    pdl_trigger();
    using V = Vec<VEC>;
    using T = typename V::T;
    constexpr int D = 32 * VEC;
    __shared__ float sm_o[kDecWarps][G][D];
    __shared__ float sm_ml[kDecWarps][G][2];
    __shared__ int is_last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bh = blockIdx.y, chunk = blockIdx.x;
    const int b = bh / p.Hkv, kvh = bh - b * p.Hkv;
    // past_len: a host scalar or the capture table (written by a copy ahead
    // of the launch), never by a kernel.
    int past = p.past;
    if (p.d_past) {
        past = (int)*p.d_past;
        if (past < 0 || past >= p.max_seq) {  // validated on the host; guard anyway
            report_error(p.err, kErrBadScalar);
            past = 0;
        }
    }
    const int n_keys = past + 1;
    const int k0 = chunk * p.chunk_keys;
    const int k1 = min(n_keys, k0 + p.chunk_keys);
    const float *kbase = p.cache + b * p.batch_stride + p.layer_off + (long long)kvh * D + lane * VEC;

    // This warp's keys of one round (KPW keys kDecWarps apart), cached keys
    // only; the new key (position past) comes from the inputs.
    T kv[KPW], vv[KPW];
    auto load_cached = [&](int j0) {
#pragma unroll
        for (int i = 0; i < KPW; i++) {
            const int j = j0 + i * kDecWarps;
            kv[i] = V::zero();
            vv[i] = V::zero();
            if (j < k1 && j != past) {
                const float *src = kbase + (long long)j * p.time_stride;
                kv[i] = V::ld(src);
                vv[i] = V::ld(src + p.parity_stride);
            }
        }
    };
    int j0 = k0 + warp;
    // With `early`, the first round's cached keys stream while the kernel
    // producing q / k / v finishes (no command before it in its segment
    // writes this cache).
    bool loaded = false;
    if (p.early && j0 < k1) {
        load_cached(j0);
        loaded = true;
    }
    pdl_wait();

    // Query rows of the group (lane slice), pre-scaled.
    T q[G];
#pragma unroll
    for (int r = 0; r < G; r++) {
        const float *qr = p.q + ((long long)(b * p.H + kvh * G + r)) * D + lane * VEC;
        q[r] = V::ld(qr);
#pragma unroll
        for (int i = 0; i < VEC; i++) V::set(q[r], i, V::get(q[r], i) * p.scale);
    }
    float m[G], l[G];
    T o[G];
#pragma unroll
    for (int r = 0; r < G; r++) {
        m[r] = -INFINITY;
        l[r] = 0.f;
        o[r] = V::zero();
    }

    const float *knew = p.k_new + ((long long)b * p.Hkv + kvh) * D + lane * VEC;
    const float *vnew = p.v_new + ((long long)b * p.Hkv + kvh) * D + lane * VEC;
    for (; j0 < k1; j0 += kDecWarps * KPW) {
        if (!loaded) load_cached(j0);
        loaded = false;
        int nk = 0;
#pragma unroll
        for (int i = 0; i < KPW; i++) {
            const int j = j0 + i * kDecWarps;
            if (j < k1) {
                nk = i + 1;
                if (j == past) {
                    // The new key: from the inputs, appended to the cache
                    // (attention.rs:61-78 index arithmetic).
                    kv[i] = V::ld(knew);
                    vv[i] = V::ld(vnew);
                    float *dst = const_cast<float *>(kbase) + (long long)j * p.time_stride;
                    V::st(dst, kv[i]);
                    V::st(dst + p.parity_stride, vv[i]);
                }
            }
        }
        // Scores of the round: the lane's partial dots of every (row r, key
        // i) pair, summed across the warp by a transposed butterfly (each
        // stage hands half of the values a lane carries to its partner), so
        // that lane holds the score of pair idx = lane / REP, idx = r KPW + i.
        constexpr int NV = G * KPW, REP = 32 / NV;
        constexpr int LOG = NV == 32 ? 5 : NV == 16 ? 4 : NV == 8 ? 3 : NV == 4 ? 2 : 1;
        static_assert(NV <= 32 && 32 % NV == 0 && (1 << LOG) == NV, "pairs per round");
        float v[NV];
#pragma unroll
        for (int r = 0; r < G; r++)
#pragma unroll
            for (int i = 0; i < KPW; i++) v[r * KPW + i] = V::dot(q[r], kv[i]);
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
        const float s = ii < nk ? v[0] : -INFINITY;
        // Row maxima over the round's keys (KPW * REP aligned lanes per row).
        float mb = s;
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
        const float p_own = s == -INFINITY ? 0.f : expf(s - m_own);
#pragma unroll
        for (int r = 0; r < G; r++) {
            const float alpha = m[r] == -INFINITY ? 0.f : expf(m[r] - m_new[r]);
            float lsum = l[r] * alpha;
            T acc = o[r];
#pragma unroll
            for (int i = 0; i < VEC; i++) V::set(acc, i, V::get(acc, i) * alpha);
#pragma unroll
            for (int i = 0; i < KPW; i++) {
                const float pj = __shfl_sync(0xffffffffu, p_own, (r * KPW + i) * REP);
                lsum += pj;
                V::axpby(acc, 1.0f, pj, vv[i]);
            }
            o[r] = acc;
            l[r] = lsum;
            m[r] = m_new[r];
        }
    }

    // Merge the warps (ascending warp order) into the CTA's partial.
#pragma unroll
    for (int r = 0; r < G; r++) {
#pragma unroll
        for (int i = 0; i < VEC; i++) sm_o[warp][r][lane * VEC + i] = V::get(o[r], i);
        if (lane == 0) {
            sm_ml[warp][r][0] = m[r];
            sm_ml[warp][r][1] = l[r];
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * D; idx += kDecThreads) {
        const int r = idx / D, d = idx - r * D;
        float mm = -INFINITY;
        for (int w = 0; w < kDecWarps; w++) mm = fmaxf(mm, sm_ml[w][r][0]);
        float ll = 0.f, acc = 0.f;
        for (int w = 0; w < kDecWarps; w++) {
            const float mw = sm_ml[w][r][0];
            if (mw != -INFINITY) {
                const float f = expf(mw - mm);
                ll = fmaf(sm_ml[w][r][1], f, ll);
                acc = fmaf(sm_o[w][r][d], f, acc);
            }
        }
        const long long row = (long long)b * p.H + kvh * G + r;
        if (p.chunks == 1) {
            const float val = __fdiv_rn(acc, ll);
            p.out[row * D + d] = val;
            if (p.out2) p.out2[row * D + d] = val;
        } else {
            p.part_o[(row * p.chunks + chunk) * D + d] = acc;
            if (d == 0) {
                p.part_ml[(row * p.chunks + chunk) * 2 + 0] = mm;
                p.part_ml[(row * p.chunks + chunk) * 2 + 1] = ll;
            }
        }
    }
    if (p.chunks == 1) return;

    // Last CTA of this (batch, kv_head) merges the chunks in ascending order.
    // The barrier orders every thread's partial stores before thread 0's
    // fence and ticket (release); its second fence orders the ticket before
    // the barrier after which the last CTA reads the other partials.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned ticket = atomicAdd(&p.tickets[bh], 1u);
        is_last = ticket == (unsigned)(p.chunks - 1);
        __threadfence();
    }
    __syncthreads();
    if (!is_last) return;
    // Chunk weights exp(m_c - M) per query row from statistics loaded in one
    // parallel pass; then every (row, dim) output adds the live chunks in
    // ascending order, its partial values loaded before the sum.
    __shared__ float sm_w[G][kDecMaxChunks];
    __shared__ float sm_l[G][kDecMaxChunks];
    __shared__ float sm_inv[G];
    const int live = min(p.chunks, (n_keys + p.chunk_keys - 1) / p.chunk_keys);
    const long long row0 = (long long)b * p.H + kvh * G;
    for (int i = threadIdx.x; i < G * live; i += kDecThreads) {
        const int r = i / live, c = i - r * live;
        const float2 ml = __ldcg(reinterpret_cast<const float2 *>(p.part_ml) +
                                 (row0 + r) * p.chunks + c);
        sm_w[r][c] = ml.x;
        sm_l[r][c] = ml.y;
    }
    __syncthreads();
    for (int r = warp; r < G; r += kDecWarps) {
        float mm = -INFINITY;
        for (int c = lane; c < live; c += 32) mm = fmaxf(mm, sm_w[r][c]);
        mm = warp_max(mm);
        __syncwarp();
        for (int c = lane; c < live; c += 32) {
            const float mc = sm_w[r][c];
            sm_w[r][c] = mc == -INFINITY ? 0.f : expf(mc - mm);
        }
        __syncwarp();
        if (lane == 0) {
            float ll = 0.f;
            for (int c = 0; c < live; c++) ll = fmaf(sm_l[r][c], sm_w[r][c], ll);
            sm_inv[r] = ll;
        }
    }
    __syncthreads();
    // Each thread owns kU float4 outputs and keeps the partials of kB chunks
    // in flight per batch; chunks are added in ascending order.
    constexpr int kU = (G * D / 4 + kDecThreads - 1) / kDecThreads;
    constexpr int kB = kU == 1 ? 20 : 10;
    float4 acc[kU];
#pragma unroll
    for (int j = 0; j < kU; j++) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c0 = 0; c0 < live; c0 += kB) {
        float4 v[kB][kU];
#pragma unroll
        for (int cc = 0; cc < kB; cc++)
#pragma unroll
            for (int j = 0; j < kU; j++) {
                const int u = threadIdx.x + j * kDecThreads, c = c0 + cc;
                const int r = (4 * u) / D, d = 4 * u - r * D;
                v[cc][j] = (u < G * D / 4 && c < live)
                               ? __ldcg(reinterpret_cast<const float4 *>(
                                     p.part_o + ((row0 + r) * p.chunks + c) * D + d))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
        for (int cc = 0; cc < kB; cc++)
#pragma unroll
            for (int j = 0; j < kU; j++) {
                const int u = threadIdx.x + j * kDecThreads, c = c0 + cc;
                if (u < G * D / 4 && c < live) {
                    const float w = sm_w[(4 * u) / D][c];
                    acc[j].x = fmaf(v[cc][j].x, w, acc[j].x);
                    acc[j].y = fmaf(v[cc][j].y, w, acc[j].y);
                    acc[j].z = fmaf(v[cc][j].z, w, acc[j].z);
                    acc[j].w = fmaf(v[cc][j].w, w, acc[j].w);
                }
            }
    }
#pragma unroll
    for (int j = 0; j < kU; j++) {
        const int u = threadIdx.x + j * kDecThreads;
        if (u < G * D / 4) {
            const int r = (4 * u) / D, d = 4 * u - r * D;
            const float inv = sm_inv[r];
            const float4 val = make_float4(__fdiv_rn(acc[j].x, inv), __fdiv_rn(acc[j].y, inv),
                                           __fdiv_rn(acc[j].z, inv), __fdiv_rn(acc[j].w, inv));
            *reinterpret_cast<float4 *>(p.out + (row0 + r) * D + d) = val;
            if (p.out2) *reinterpret_cast<float4 *>(p.out2 + (row0 + r) * D + d) = val;
        }
    }
    if (threadIdx.x == 0) p.tickets[bh] = 0u;  // ready for the next launch
}

struct DecodePlan {
    bool ok = false;
    int chunk_keys = 0, chunks = 0;
};

// keys_max: the most keys any replay can see (past_len + 1 for a host
// scalar, max_seq for a device-resident one).
DecodePlan plan_decode(size_t batch, size_t kv_heads, size_t heads, size_t seq, size_t head_dim,
                       size_t keys_max) {
    DecodePlan pl;
    if (seq != 1 || kv_heads == 0 || heads % kv_heads != 0) return pl;
    const size_t group = heads / kv_heads;
    if ((group != 1 && group != 2 && group != 4 && group != 8) ||
        (head_dim != 64 && head_dim != 128))
        return pl;
    if (keys_max > (size_t)INT32_MAX || batch * kv_heads > 65535) return pl;
    const size_t bh = batch * kv_heads;
    // At most one CTA per SM (one wave: the kernel's registers allow one
    // CTA per SM, so a 149th CTA would double the time), each at least 64
    // keys (one round of its 8 warps), so that the last CTA merges few chunk
    // partials.
    size_t want = bh < (size_t)kSmCount ? (size_t)kSmCount / bh : 1;
    size_t by_len = (keys_max + 63) / 64;
    size_t chunks = want < by_len ? want : by_len;
    if (chunks < 1) chunks = 1;
    size_t ck = (keys_max + chunks - 1) / chunks;
    ck = (ck + 15) / 16 * 16;
    pl.chunk_keys = (int)ck;
    pl.chunks = (int)((keys_max + ck - 1) / ck);
    if (pl.chunks > kDecMaxChunks) {  // very long contexts: larger chunks
        ck = (keys_max + kDecMaxChunks - 1) / kDecMaxChunks;
        ck = (ck + 15) / 16 * 16;
        pl.chunk_keys = (int)ck;
        pl.chunks = (int)((keys_max + ck - 1) / ck);
    }
    pl.ok = true;
    return pl;
}

// ---- fused decode attention block (capture-time fusion) ------------------
//
// Replaces, for one decode position (seq 1), the command run
//   SplitHeads(q) -> qs, SplitHeads(k) -> ks, SplitHeads(v) -> vs,
//   Rope(qs) -> qr, Rope(ks) -> kr, CausalAttention(qr, kr, vs) -> a,
//   MergeHeads(a) -> am
// by two launches with the same results in every output buffer:
//  * decode_block_prep (one CTA) reads q, k, v and the positions into shared
//    memory, then writes qs, ks, vs, qr, kr in command order, a block-wide
//    barrier between commands, so outputs that share bytes with each other
//    or with the inputs (the memory plan reuses dead temporaries) end with
//    the values sequential execution leaves. It also writes qr, kr and v to
//    a private scratch area that nothing else aliases.
//  * attention_decode reads only the scratch copies and writes a and am.
// At seq 1, [B, 1, H * D] and [B, H, 1, D] are the same bytes, so the split
// and merge copies are element copies. RoPE is the rope_kernel arithmetic
// (f64 angle from the host-computed f64 denominators, f32 rotation).
struct BlockPrep {
    const float *q, *k, *v;
    const uint32_t *pos;  // [B, 1]
    float *qs, *ks, *vs, *qr, *kr;
    float *sq, *sk, *sv;  // private scratch copies: roped q, roped k, v
    int B, H, Hkv, D, gptj;
    double denom[64];     // theta^(2 p / D), host libm pow
};

__device__ __forceinline__ void rope_pair(const float *x, float *o, int base, int p, int half,
                                          int gptj, const float *trig) {
    const int i0 = gptj ? base + 2 * p : base + p;
    const int i1 = gptj ? base + 2 * p + 1 : base + p + half;
    const float first = x[i0], second = x[i1];
    const float sn = trig[p], cs = trig[half + p];
    o[i0] = __fsub_rn(__fmul_rn(first, cs), __fmul_rn(second, sn));
    o[i1] = __fadd_rn(__fmul_rn(first, sn), __fmul_rn(second, cs));
}

__global__ void __launch_bounds__(1024) decode_block_prep(const __grid_constant__ BlockPrep p) {
    pdl_trigger();
    extern __shared__ float sm[];
    const int D = p.D, half = D / 2;
    const int nq = p.B * p.H * D, nk = p.B * p.Hkv * D;
    float *q = sm, *k = q + nq, *v = k + nk, *trig = v + nk;  // trig [B][D]
    float *rq = trig + p.B * D, *rk = rq + nq;                  // roped q, k
    // Positions are U32 data, written only by uploads (a U32 command output
    // is illegal), so the f64 sine / cosine run before the dependency wait.
    for (int i = threadIdx.x; i < p.B * half; i += blockDim.x) {
        const int b = i / half, pr = i - b * half;
        const double angle = (double)p.pos[b] / p.denom[pr];
        double sn, cs;
        sincos(angle, &sn, &cs);
        trig[b * D + pr] = (float)sn;
        trig[b * D + half + pr] = (float)cs;
    }
    pdl_wait();
    for (int i = threadIdx.x; i < nq; i += blockDim.x) q[i] = p.q[i];
    for (int i = threadIdx.x; i < nk; i += blockDim.x) {
        k[i] = p.k[i];
        v[i] = p.v[i];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < p.B * p.H * half; i += blockDim.x) {
        const int row = i / half, pr = i - row * half;  // row = b * H + h
        rope_pair(q, rq, row * D, pr, half, p.gptj, trig + (row / p.H) * D);
    }
    for (int i = threadIdx.x; i < p.B * p.Hkv * half; i += blockDim.x) {
        const int row = i / half, pr = i - row * half;
        rope_pair(k, rk, row * D, pr, half, p.gptj, trig + (row / p.Hkv) * D);
    }
    __syncthreads();  // rotated rows are read by other threads below
    // Private copies for the attention kernel.
    for (int i = threadIdx.x; i < nq; i += blockDim.x) p.sq[i] = rq[i];
    for (int i = threadIdx.x; i < nk; i += blockDim.x) {
        p.sk[i] = rk[i];
        p.sv[i] = v[i];
    }
    // The five outputs, in command order.
    for (int i = threadIdx.x; i < nq; i += blockDim.x) p.qs[i] = q[i];
    __syncthreads();
    for (int i = threadIdx.x; i < nk; i += blockDim.x) p.ks[i] = k[i];
    __syncthreads();
    for (int i = threadIdx.x; i < nk; i += blockDim.x) p.vs[i] = v[i];
    __syncthreads();
    for (int i = threadIdx.x; i < nq; i += blockDim.x) p.qr[i] = rq[i];
    __syncthreads();
    for (int i = threadIdx.x; i < nk; i += blockDim.x) p.kr[i] = rk[i];
}

size_t block_prep_smem(size_t B, size_t H, size_t Hkv, size_t D) {
    return (2 * B * H * D + 3 * B * Hkv * D + B * D) * sizeof(float);
}

}  // namespace

cudaError_t kv_append(cudaStream_t s, const float *k, const float *v, float *cache,
                      const KvGeometry &g, size_t past_len, size_t seq, const uint32_t *d_past) {
    size_t total = g.batch * g.kv_heads * seq * g.head_dim;
    if (total == 0) return cudaSuccess;
    launch_k(kv_append_kernel, grid_for(total, 256), 256, 0, s, k, v, cache, g.batch, g.layers, g.layer,
                                                          g.kv_heads, g.head_dim, g.max_seq,
                                                          past_len, seq, d_past, nullptr);
    count_launch();
    return cudaGetLastError();
}

size_t attention_workspace_bytes(size_t batch, size_t heads, size_t kv_heads, size_t seq,
                                 size_t past_len, size_t head_dim, size_t max_seq,
                                 bool device_past) {
    if (seq == 0 || batch == 0 || kv_heads == 0) return 0;
    const size_t keys = device_past ? max_seq : past_len + seq;
    DecodePlan dp = plan_decode(batch, kv_heads, heads, seq, head_dim, keys);
    if (dp.ok) return dp.chunks <= 1 ? 0 : batch * heads * dp.chunks * (head_dim + 2) * 4;
    Plan pl = plan(batch, heads, kv_heads, seq, keys - seq, head_dim);
    if (pl.chunks <= 1) return 0;
    return batch * heads * seq * pl.chunks * (head_dim + 2) * sizeof(float);
}

// Decode attention (seq 1) with the append fused: q / k / v rows given,
// out (and, if set, out2) written. Requires the decode plan.
cudaError_t causal_attention_decode_into(cudaStream_t s, const float *q, const float *k,
                                         const float *v, float *cache, float *out, float *out2,
                                         const KvGeometry &g, size_t heads, size_t past_len,
                                         float scale, const AttnScratch &scr,
                                         const uint32_t *d_past, bool early) {
    const size_t keys = d_past ? g.max_seq : past_len + 1;
    const size_t time_stride = g.kv_heads * g.head_dim;
    const size_t parity_stride = g.max_seq * time_stride;
    DecodePlan dp = plan_decode(g.batch, g.kv_heads, heads, 1, g.head_dim, keys);
    if (!dp.ok || g.batch * g.kv_heads > scr.ticket_count) return cudaErrorInvalidValue;
    const size_t need = dp.chunks <= 1 ? 0 : g.batch * heads * dp.chunks * (g.head_dim + 2) * 4;
    if (need > scr.workspace_bytes) return cudaErrorMemoryAllocation;
    DecodeParams p{};
    p.q = q;
    p.k_new = k;
    p.v_new = v;
    p.cache = cache;
    p.out = out;
    p.out2 = out2;
    p.early = early ? 1 : 0;
    p.part_o = static_cast<float *>(scr.workspace);
    p.part_ml = p.part_o + g.batch * heads * dp.chunks * g.head_dim;
    p.tickets = scr.tickets;
    p.d_past = d_past;
    p.err = scr.err;
    p.batch_stride = (long long)(g.layers * 2 * parity_stride);
    p.layer_off = (long long)(g.layer * 2 * parity_stride);
    p.parity_stride = (long long)parity_stride;
    p.time_stride = (long long)time_stride;
    p.past = (int)past_len;
    p.max_seq = (int)g.max_seq;
    p.H = (int)heads;
    p.Hkv = (int)g.kv_heads;
    p.G = (int)(heads / g.kv_heads);
    p.chunk_keys = dp.chunk_keys;
    p.chunks = dp.chunks;
    p.scale = scale;
    dim3 grid((unsigned)dp.chunks, (unsigned)(g.batch * g.kv_heads));
    const bool d128 = g.head_dim == 128;
    switch (p.G) {
    case 1:
        launch_k(d128 ? attention_decode<4, 1, 8> : attention_decode<2, 1, 8>, grid,
                 kDecThreads, 0, s, p);
        break;
    case 2:
        launch_k(d128 ? attention_decode<4, 2, 8> : attention_decode<2, 2, 8>, grid,
                 kDecThreads, 0, s, p);
        break;
    case 4:
        launch_k(d128 ? attention_decode<4, 4, 8> : attention_decode<2, 4, 8>, grid,
                 kDecThreads, 0, s, p);
        break;
    default:
        launch_k(d128 ? attention_decode<4, 8, 4> : attention_decode<2, 8, 4>, grid,
                 kDecThreads, 0, s, p);
        break;
    }
    count_launch();
    return cudaGetLastError();
}

cudaError_t causal_attention(cudaStream_t s, const float *q, const float *k, const float *v,
                             float *cache, float *out, const KvGeometry &g, size_t heads,
                             size_t seq, size_t past_len, float scale, const AttnScratch &scr,
                             const uint32_t *d_past) {
    if (seq == 0 || g.batch == 0) return kv_append(s, k, v, cache, g, past_len, seq, d_past);
    const size_t keys = d_past ? g.max_seq : past_len + seq;
    const size_t time_stride = g.kv_heads * g.head_dim;
    const size_t parity_stride = g.max_seq * time_stride;
    DecodePlan dp = plan_decode(g.batch, g.kv_heads, heads, seq, g.head_dim, keys);
    if (dp.ok && g.batch * g.kv_heads <= scr.ticket_count)
        return causal_attention_decode_into(s, q, k, v, cache, out, nullptr, g, heads, past_len,
                                            scale, scr, d_past, false);
    cudaError_t e = kv_append(s, k, v, cache, g, past_len, seq, d_past);
    if (e != cudaSuccess) return e;
    Plan pl = plan(g.batch, heads, g.kv_heads, seq, keys - seq, g.head_dim);
    size_t rows = g.batch * heads * seq;
    size_t need = rows * pl.chunks * (g.head_dim + 2) * sizeof(float);
    if (pl.chunks > 1 && need > scr.workspace_bytes) return cudaErrorMemoryAllocation;
    AttnParams p{};
    p.q = q;
    p.cache = cache;
    p.out = out;
    p.part_o = static_cast<float *>(scr.workspace);
    p.part_ml = p.part_o + rows * pl.chunks * g.head_dim;
    p.batch = g.batch;
    p.heads = heads;
    p.kv_heads = g.kv_heads;
    p.seq = seq;
    p.past_len = past_len;
    p.head_dim = g.head_dim;
    p.time_stride = time_stride;
    p.parity_stride = parity_stride;
    p.key_base_layer = g.layer * 2 * p.parity_stride;
    p.batch_stride = g.layers * 2 * p.parity_stride;
    p.group = heads / g.kv_heads;
    p.g_block = pl.g_block;
    p.t_block = pl.t_block;
    p.chunk_keys = pl.chunk_keys;
    p.chunks = pl.chunks;
    p.scale = scale;
    p.d_past = d_past;
    static std::atomic<uint64_t> smem_set{0};
    set_smem_limit_once(attention_kernel, 227 * 1024, &smem_set);
    dim3 grid((unsigned)pl.chunks, (unsigned)pl.grid_y, (unsigned)(g.batch * g.kv_heads));
    launch_k(attention_kernel, grid, kThreads, pl.smem, s, p);
    count_launch();
    if (pl.chunks > 1) {
        launch_k(attention_combine, grid_for(rows, 1, 16), 128, 0, s, p.part_o, p.part_ml, out, rows,
                                                                pl.chunks, g.head_dim);
        count_launch();
    }
    return cudaGetLastError();
}

size_t decode_block_scratch_floats(size_t batch, size_t heads, size_t kv_heads, size_t head_dim) {
    return batch * (heads + 2 * kv_heads) * head_dim;
}

bool decode_block_supported(size_t batch, size_t heads, size_t kv_heads, size_t head_dim,
                            size_t keys_max, size_t ticket_count) {
    DecodePlan dp = plan_decode(batch, kv_heads, heads, 1, head_dim, keys_max);
    return dp.ok && head_dim / 2 <= 64 && batch * kv_heads <= ticket_count &&
           block_prep_smem(batch, heads, kv_heads, head_dim) <= 200 * 1024;
}

cudaError_t decode_attention_block(cudaStream_t s, const DecodeBlockIo &io, float *cache,
                                   const KvGeometry &g, size_t heads, size_t past_len, float scale,
                                   float theta, int gptj, const AttnScratch &scr,
                                   const uint32_t *d_past, bool early_cache) {
    BlockPrep bp{};
    bp.q = io.q;
    bp.k = io.k;
    bp.v = io.v;
    bp.pos = io.pos;
    bp.qs = io.qs;
    bp.ks = io.ks;
    bp.vs = io.vs;
    bp.qr = io.qr;
    bp.kr = io.kr;
    const size_t nq = g.batch * heads * g.head_dim, nk = g.batch * g.kv_heads * g.head_dim;
    bp.sq = io.scratch;
    bp.sk = bp.sq + nq;
    bp.sv = bp.sk + nk;
    bp.B = (int)g.batch;
    bp.H = (int)heads;
    bp.Hkv = (int)g.kv_heads;
    bp.D = (int)g.head_dim;
    bp.gptj = gptj;
    for (size_t pr = 0; pr < g.head_dim / 2; pr++)
        bp.denom[pr] = pow((double)theta, 2.0 * (double)pr / (double)g.head_dim);
    const size_t smem = block_prep_smem(g.batch, heads, g.kv_heads, g.head_dim);
    static std::atomic<uint64_t> smem_set{0};
    set_smem_limit_once(decode_block_prep, 200 * 1024, &smem_set);
    launch_k(decode_block_prep, 1, 1024, smem, s, bp);
    count_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return causal_attention_decode_into(s, bp.sq, bp.sk, bp.sv, cache, io.out, io.out_merged, g,
                                        heads, past_len, scale, scr, d_past, early_cache);
}

}  // namespace k
}  // namespace slc
