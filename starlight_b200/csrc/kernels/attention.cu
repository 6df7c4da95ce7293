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
#include <math.h>

#include "common.cuh"
#include "kernels.h"

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
                                                        size_t seq) {
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
};

__global__ void __launch_bounds__(kThreads) attention_kernel(AttnParams p) {
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

    const size_t key_begin = chunk * p.chunk_keys;
    const size_t last_key = p.past_len + t0 + tn - 1;  // largest visible key of this CTA
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
            size_t limit = p.past_len + t0 + tq;  // keys 0..=limit visible
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

}  // namespace

cudaError_t kv_append(cudaStream_t s, const float *k, const float *v, float *cache,
                      const KvGeometry &g, size_t past_len, size_t seq) {
    size_t total = g.batch * g.kv_heads * seq * g.head_dim;
    if (total == 0) return cudaSuccess;
    kv_append_kernel<<<grid_for(total, 256), 256, 0, s>>>(k, v, cache, g.batch, g.layers, g.layer,
                                                          g.kv_heads, g.head_dim, g.max_seq,
                                                          past_len, seq);
    count_launch();
    return cudaGetLastError();
}

size_t attention_workspace_bytes(size_t batch, size_t heads, size_t kv_heads, size_t seq,
                                 size_t past_len, size_t head_dim) {
    if (seq == 0 || batch == 0 || kv_heads == 0) return 0;
    Plan pl = plan(batch, heads, kv_heads, seq, past_len, head_dim);
    if (pl.chunks <= 1) return 0;
    return batch * heads * seq * pl.chunks * (head_dim + 2) * sizeof(float);
}

cudaError_t causal_attention(cudaStream_t s, const float *q, const float *k, const float *v,
                             float *cache, float *out, const KvGeometry &g, size_t heads,
                             size_t seq, size_t past_len, float scale, void *workspace,
                             size_t workspace_bytes) {
    cudaError_t e = kv_append(s, k, v, cache, g, past_len, seq);
    if (e != cudaSuccess || seq == 0 || g.batch == 0) return e;
    Plan pl = plan(g.batch, heads, g.kv_heads, seq, past_len, g.head_dim);
    size_t rows = g.batch * heads * seq;
    size_t need = rows * pl.chunks * (g.head_dim + 2) * sizeof(float);
    if (pl.chunks > 1 && need > workspace_bytes) return cudaErrorMemoryAllocation;
    AttnParams p{};
    p.q = q;
    p.cache = cache;
    p.out = out;
    p.part_o = static_cast<float *>(workspace);
    p.part_ml = p.part_o + rows * pl.chunks * g.head_dim;
    p.batch = g.batch;
    p.heads = heads;
    p.kv_heads = g.kv_heads;
    p.seq = seq;
    p.past_len = past_len;
    p.head_dim = g.head_dim;
    p.time_stride = g.kv_heads * g.head_dim;
    p.parity_stride = g.max_seq * p.time_stride;
    p.key_base_layer = g.layer * 2 * p.parity_stride;
    p.batch_stride = g.layers * 2 * p.parity_stride;
    p.group = heads / g.kv_heads;
    p.g_block = pl.g_block;
    p.t_block = pl.t_block;
    p.chunk_keys = pl.chunk_keys;
    p.chunks = pl.chunks;
    p.scale = scale;
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             227 * 1024);
        configured = true;
    }
    dim3 grid((unsigned)pl.chunks, (unsigned)pl.grid_y, (unsigned)(g.batch * g.kv_heads));
    attention_kernel<<<grid, kThreads, pl.smem, s>>>(p);
    count_launch();
    if (pl.chunks > 1) {
        attention_combine<<<grid_for(rows, 1, 16), 128, 0, s>>>(p.part_o, p.part_ml, out, rows,
                                                                pl.chunks, g.head_dim);
        count_launch();
    }
    return cudaGetLastError();
}

}  // namespace k
}  // namespace slc
