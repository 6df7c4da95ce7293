// llama-dense engine over the backend-cuda C ABI (see include/starlight_engine.h).
//
// Lowering (the sl-model-adapters llama-dense contract, docs/ARCH-0006
// sections 4-5, op usage docs/ARCH-0004:252-276), per step:
//   Gather(embed, ids)
//   per layer i:
//     RmsNorm(attn_norm) -> MatMulNT q, k, v -> SplitHeads x3 -> Rope(Neox) q, k
//     -> CausalAttention{layer=i} (writes the KV state) -> MergeHeads
//     -> MatMulNT o [-> AllReduce] -> Add(residual)
//     -> RmsNorm(mlp_norm) -> SwiGlu(gate, up, down) [-> AllReduce] -> Add(residual)
//   RmsNorm(final_norm) -> LastToken(seq_len) -> MatMulNT lm_head [-> AllGather]
// LastToken precedes the lm_head projection (a row select commutes with it).
//
// Engine::build / step follow docs/ARCH-0007 section 3.2: build allocates the
// scratchpad, KV state and IO buffers through the device and binds every
// value to a BufferRef (Temps at memory-plan offsets, plan built by greedy
// interval reuse over the command order as sl-graph does, docs/ARCH-0004
// section 7); step uploads ids and positions, dispatches every command,
// synchronizes and downloads the logits. step performs no allocation.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <new>
#include <vector>

#include "../../include/starlight_cuda.h"
#include "../../include/starlight_engine.h"
#include "device_internal.h"
#include "kernels/kernels.h"

namespace {

struct Weight {
    int role;
    uint32_t layer;
    uint64_t full_rows, full_cols;  // unsharded logical shape
    uint64_t row0, rows, col0, cols;  // this rank's shard
    bool quant = false;
    uint32_t buf = 0;     // f32 weight, or the u32 payload when quantized
    uint32_t scales = 0;  // f32 scales when quantized
    uint64_t len = 0;     // BufferRef length (elements or payload words)
};

struct Cmd {
    slc_op op;
    std::vector<uint32_t> in, out;
};

struct Ready {
    slc_op op;
    std::vector<slc_buffer_ref> in, out;
    std::vector<slc_value> iv, ov;
    std::vector<int> scalar_src;  // 0: seq_len, 1: past_len
};

struct Program {
    uint64_t seq = 0;
    std::vector<slc_value> values;
    std::vector<int> weight_of;  // value -> weight index, -1 otherwise
    std::vector<Cmd> cmds;
    uint32_t ids = 0, pos = 0, seq_len = 0, past_len = 0, kv = 0, logits = 0;
    std::vector<uint64_t> temp_offset;  // elements into the scratchpad
    uint64_t scratch_elems = 0;
    std::vector<slc_buffer_ref> refs;
    std::vector<Ready> ready;
    // The scalar sources of ready[i] are src_flat[sum(src_count[<i]) ...],
    // src_count[i] of them; the memo relaunches the step's graph directly.
    std::vector<int> src_flat;
    std::vector<uint32_t> src_count;
    StepMemo memo;
};

uint64_t count_of(const slc_value &v) {
    uint64_t n = 1;
    for (uint32_t i = 0; i < v.rank; i++) n *= v.dims[i];
    return n;
}

slc_value make_value(uint32_t dtype, uint32_t role, std::initializer_list<uint64_t> shape) {
    slc_value v{};
    v.dtype = dtype;
    v.role = role;
    v.rank = (uint32_t)shape.size();
    uint32_t i = 0;
    for (uint64_t d : shape) v.dims[i++] = (uint32_t)d;
    v.encoding = SLC_ENC_DENSE;
    return v;
}

uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

}  // namespace

struct slc_llama {
    slc_device *dev = nullptr;
    slc_llama_config cfg{};
    uint64_t hq = 0, hkv = 0, inter = 0, vocab = 0;  // per-rank shard sizes
    std::vector<Weight> weights;
    Program prefill, decode;
    uint32_t scratch = 0, kv = 0, logits_buf = 0;
    uint32_t ids_prefill = 0, pos_prefill = 0, ids_decode = 0, pos_decode = 0;
    uint32_t temp = UINT32_MAX;  // staging for weight shards
    uint64_t temp_elems = 0;
    std::vector<float> host_logits;
    cudaEvent_t ev_begin = nullptr, ev_end = nullptr;
    float last_step_ms = 0.f;
    uint64_t memo_steps = 0;  // steps relaunched from a program's step memo
    bool memo = true;         // SLC_STEP_MEMO=0 at creation: always dispatch
};

namespace {

int weight_index(slc_llama *m, int role, uint32_t layer) {
    for (size_t i = 0; i < m->weights.size(); i++)
        if (m->weights[i].role == role && m->weights[i].layer == layer) return (int)i;
    return -1;
}

void add_weight(slc_llama *m, int role, uint32_t layer, uint64_t fr, uint64_t fc, int shard) {
    // shard: 0 replicated, 1 split rows (output features), 2 split columns (input features)
    const uint64_t world = (uint64_t)m->cfg.tp_world, rank = (uint64_t)m->cfg.tp_rank;
    Weight w{};
    w.role = role;
    w.layer = layer;
    w.full_rows = fr;
    w.full_cols = fc;
    w.rows = shard == 1 ? fr / world : fr;
    w.cols = shard == 2 ? fc / world : fc;
    w.row0 = shard == 1 ? rank * w.rows : 0;
    w.col0 = shard == 2 ? rank * w.cols : 0;
    bool matrix = role == SLC_W_Q || role == SLC_W_K || role == SLC_W_V || role == SLC_W_O ||
                  role == SLC_W_GATE || role == SLC_W_UP || role == SLC_W_DOWN ||
                  role == SLC_W_LM_HEAD;
    w.quant = matrix && m->cfg.quant_format >= 0;
    m->weights.push_back(w);
}

// ---- program construction ---------------------------------------------------

struct Builder {
    slc_llama *m;
    Program &p;

    uint32_t value(const slc_value &v, int weight = -1) {
        p.values.push_back(v);
        p.weight_of.push_back(weight);
        return (uint32_t)(p.values.size() - 1);
    }
    uint32_t temp(std::initializer_list<uint64_t> shape) {
        return value(make_value(SLC_F32, SLC_ROLE_TEMP, shape));
    }
    uint32_t param(int role, uint32_t layer) {
        int wi = weight_index(m, role, layer);
        const Weight &w = m->weights[wi];
        slc_value v = w.rows == 1 && (role == SLC_W_ATTN_NORM || role == SLC_W_MLP_NORM ||
                                      role == SLC_W_FINAL_NORM)
                          ? make_value(SLC_F32, SLC_ROLE_PARAM, {w.cols})
                          : make_value(SLC_F32, SLC_ROLE_PARAM, {w.rows, w.cols});
        if (w.quant) {
            v.encoding = SLC_ENC_GROUPWISE;
            v.quant_format = (uint32_t)m->cfg.quant_format;
            v.group_size = m->cfg.group_size;
        }
        return value(v, wi);
    }
    void emit(const slc_op &op, std::vector<uint32_t> in, std::vector<uint32_t> out) {
        p.cmds.push_back(Cmd{op, std::move(in), std::move(out)});
    }
};

slc_op make_op(uint16_t code) {
    slc_op o{};
    o.code = code;
    return o;
}

void build_program(slc_llama *m, Program &p, uint64_t T) {
    const slc_llama_config &c = m->cfg;
    const uint64_t B = c.batch, H = c.hidden, D = c.head_dim;
    const uint64_t Hq = m->hq, Hkv = m->hkv, I = m->inter, V = m->vocab;
    const bool tp = c.tp_world > 1;
    p = Program{};
    p.seq = T;
    Builder b{m, p};
    p.ids = b.value(make_value(SLC_U32, SLC_ROLE_INPUT, {B, T}));
    p.pos = b.value(make_value(SLC_U32, SLC_ROLE_INPUT, {B, T}));
    p.seq_len = b.value(make_value(SLC_U32, SLC_ROLE_SCALAR, {}));
    p.past_len = b.value(make_value(SLC_U32, SLC_ROLE_SCALAR, {}));
    p.kv = b.value(make_value(SLC_F32, SLC_ROLE_STATE, {B, c.layers, 2, c.max_seq, Hkv, D}));

    slc_op rms = make_op(SLC_OP_RMS_NORM);
    rms.eps = c.eps;
    uint32_t x = b.temp({B, T, H});
    b.emit(make_op(SLC_OP_GATHER), {b.param(SLC_W_EMBED, 0), p.ids}, {x});
    const float scale = (float)(1.0 / sqrt((double)D));
    for (uint32_t l = 0; l < c.layers; l++) {
        uint32_t h = b.temp({B, T, H});
        b.emit(rms, {x, b.param(SLC_W_ATTN_NORM, l)}, {h});
        uint32_t q = b.temp({B, T, Hq * D}), k = b.temp({B, T, Hkv * D}), v = b.temp({B, T, Hkv * D});
        b.emit(make_op(SLC_OP_MATMUL_NT), {h, b.param(SLC_W_Q, l)}, {q});
        b.emit(make_op(SLC_OP_MATMUL_NT), {h, b.param(SLC_W_K, l)}, {k});
        b.emit(make_op(SLC_OP_MATMUL_NT), {h, b.param(SLC_W_V, l)}, {v});
        slc_op sq = make_op(SLC_OP_SPLIT_HEADS), skv = make_op(SLC_OP_SPLIT_HEADS);
        sq.heads = (uint32_t)Hq;
        sq.head_dim = (uint32_t)D;
        skv.heads = (uint32_t)Hkv;
        skv.head_dim = (uint32_t)D;
        uint32_t qs = b.temp({B, Hq, T, D}), ks = b.temp({B, Hkv, T, D}), vs = b.temp({B, Hkv, T, D});
        b.emit(sq, {q}, {qs});
        b.emit(skv, {k}, {ks});
        b.emit(skv, {v}, {vs});
        slc_op rope = make_op(SLC_OP_ROPE);
        rope.rope_variant = SLC_ROPE_NEOX;
        rope.theta = c.theta;
        uint32_t qr = b.temp({B, Hq, T, D}), kr = b.temp({B, Hkv, T, D});
        b.emit(rope, {qs, p.pos}, {qr});
        b.emit(rope, {ks, p.pos}, {kr});
        slc_op att = make_op(SLC_OP_CAUSAL_ATTENTION);
        att.layer = l;
        att.heads = (uint32_t)Hq;
        att.kv_heads = (uint32_t)Hkv;
        att.head_dim = (uint32_t)D;
        att.scale = scale;
        uint32_t a = b.temp({B, Hq, T, D});
        b.emit(att, {qr, kr, vs, p.kv, p.past_len}, {a});
        slc_op mh = make_op(SLC_OP_MERGE_HEADS);
        mh.heads = (uint32_t)Hq;
        mh.head_dim = (uint32_t)D;
        uint32_t am = b.temp({B, T, Hq * D});
        b.emit(mh, {a}, {am});
        uint32_t o = b.temp({B, T, H});
        b.emit(make_op(SLC_OP_MATMUL_NT), {am, b.param(SLC_W_O, l)}, {o});
        if (tp) b.emit(make_op(SLC_OP_EXT_ALL_REDUCE), {o}, {});
        uint32_t x1 = b.temp({B, T, H});
        b.emit(make_op(SLC_OP_ADD), {x, o}, {x1});
        uint32_t h2 = b.temp({B, T, H});
        b.emit(rms, {x1, b.param(SLC_W_MLP_NORM, l)}, {h2});
        uint32_t f = b.temp({B, T, H});
        if (c.decompose_swiglu) {
            // The decomposition sl-graph applies when SwiGlu is not a declared
            // composite (docs/ARCH-0004:285).
            uint32_t g = b.temp({B, T, I}), u = b.temp({B, T, I});
            b.emit(make_op(SLC_OP_MATMUL_NT), {h2, b.param(SLC_W_GATE, l)}, {g});
            b.emit(make_op(SLC_OP_MATMUL_NT), {h2, b.param(SLC_W_UP, l)}, {u});
            uint32_t gs = b.temp({B, T, I}), hm = b.temp({B, T, I});
            b.emit(make_op(SLC_OP_SILU), {g}, {gs});
            b.emit(make_op(SLC_OP_MUL), {gs, u}, {hm});
            b.emit(make_op(SLC_OP_MATMUL_NT), {hm, b.param(SLC_W_DOWN, l)}, {f});
        } else {
            b.emit(make_op(SLC_OP_SWIGLU),
                   {h2, b.param(SLC_W_GATE, l), b.param(SLC_W_UP, l), b.param(SLC_W_DOWN, l)}, {f});
        }
        if (tp) b.emit(make_op(SLC_OP_EXT_ALL_REDUCE), {f}, {});
        uint32_t x2 = b.temp({B, T, H});
        b.emit(make_op(SLC_OP_ADD), {x1, f}, {x2});
        x = x2;
    }
    uint32_t hf = b.temp({B, T, H});
    b.emit(rms, {x, b.param(SLC_W_FINAL_NORM, 0)}, {hf});
    uint32_t last = b.temp({B, H});
    b.emit(make_op(SLC_OP_LAST_TOKEN), {hf, p.seq_len}, {last});
    if (tp) {
        uint32_t part = b.temp({B, V});
        b.emit(make_op(SLC_OP_MATMUL_NT), {last, b.param(SLC_W_LM_HEAD, 0)}, {part});
        p.logits = b.value(make_value(SLC_F32, SLC_ROLE_OUTPUT, {B, V * (uint64_t)c.tp_world}));
        b.emit(make_op(SLC_OP_EXT_ALL_GATHER), {part}, {p.logits});
    } else {
        p.logits = b.value(make_value(SLC_F32, SLC_ROLE_OUTPUT, {B, V}));
        b.emit(make_op(SLC_OP_MATMUL_NT), {last, b.param(SLC_W_LM_HEAD, 0)}, {p.logits});
    }
}

// Greedy interval reuse for Temps over the command order; lifetimes are the
// closed intervals [first use, last use] (docs/ARCH-0004 section 7), so a
// value read by command i never shares bytes with an output of command i.
void plan_memory(Program &p) {
    const size_t nv = p.values.size();
    std::vector<int64_t> first(nv, -1), last(nv, -1);
    for (size_t i = 0; i < p.cmds.size(); i++) {
        for (uint32_t v : p.cmds[i].in) {
            if (first[v] < 0) first[v] = (int64_t)i;
            last[v] = (int64_t)i;
        }
        for (uint32_t v : p.cmds[i].out) {
            if (first[v] < 0) first[v] = (int64_t)i;
            last[v] = std::max(last[v], (int64_t)i);
        }
    }
    struct Block {
        uint64_t off, len;
    };
    std::vector<Block> free_blocks;
    uint64_t top = 0;
    p.temp_offset.assign(nv, 0);
    auto round = [](uint64_t n) { return (n + 15) / 16 * 16; };  // 64-byte alignment
    for (size_t i = 0; i < p.cmds.size(); i++) {
        for (uint32_t v : p.cmds[i].out) {
            if (p.values[v].role != SLC_ROLE_TEMP || first[v] != (int64_t)i) continue;
            uint64_t need = round(std::max<uint64_t>(count_of(p.values[v]), 1));
            int best = -1;
            for (size_t j = 0; j < free_blocks.size(); j++)
                if (free_blocks[j].len >= need &&
                    (best < 0 || free_blocks[j].len < free_blocks[best].len))
                    best = (int)j;
            if (best >= 0) {
                p.temp_offset[v] = free_blocks[best].off;
                free_blocks[best].off += need;
                free_blocks[best].len -= need;
                if (free_blocks[best].len == 0) free_blocks.erase(free_blocks.begin() + best);
            } else {
                p.temp_offset[v] = top;
                top += need;
            }
        }
        for (uint32_t v : p.cmds[i].in) {
            if (p.values[v].role != SLC_ROLE_TEMP || last[v] != (int64_t)i) continue;
            free_blocks.push_back(Block{p.temp_offset[v], round(std::max<uint64_t>(count_of(p.values[v]), 1))});
        }
        // Coalesce adjacent free blocks.
        std::sort(free_blocks.begin(), free_blocks.end(),
                  [](const Block &a, const Block &b) { return a.off < b.off; });
        std::vector<Block> merged;
        for (const Block &blk : free_blocks) {
            if (!merged.empty() && merged.back().off + merged.back().len == blk.off)
                merged.back().len += blk.len;
            else
                merged.push_back(blk);
        }
        free_blocks.swap(merged);
    }
    p.scratch_elems = std::max<uint64_t>(top, 16);
}

void bind(slc_llama *m, Program &p, uint32_t ids_buf, uint32_t pos_buf) {
    const size_t nv = p.values.size();
    p.refs.assign(nv, slc_buffer_ref{});
    for (size_t v = 0; v < nv; v++) {
        const slc_value &val = p.values[v];
        slc_buffer_ref &r = p.refs[v];
        switch (val.role) {
        case SLC_ROLE_PARAM: {
            const Weight &w = m->weights[p.weight_of[v]];
            r = slc_buffer_ref{w.buf, 0, 0, w.len};
            break;
        }
        case SLC_ROLE_STATE: r = slc_buffer_ref{m->kv, 0, 0, count_of(val)}; break;
        case SLC_ROLE_OUTPUT: r = slc_buffer_ref{m->logits_buf, 0, 0, count_of(val)}; break;
        case SLC_ROLE_TEMP: r = slc_buffer_ref{m->scratch, 0, p.temp_offset[v], count_of(val)}; break;
        case SLC_ROLE_INPUT:
            r = slc_buffer_ref{v == p.ids ? ids_buf : pos_buf, 0, 0, count_of(val)};
            break;
        default: break;
        }
    }
    p.ready.clear();
    for (const Cmd &c : p.cmds) {
        Ready rd;
        rd.op = c.op;
        for (uint32_t v : c.in) {
            if (p.values[v].role == SLC_ROLE_SCALAR) {
                rd.scalar_src.push_back(v == p.seq_len ? 0 : 1);
            } else {
                rd.in.push_back(p.refs[v]);
                rd.iv.push_back(p.values[v]);
            }
        }
        for (uint32_t v : c.out) {
            rd.out.push_back(p.refs[v]);
            rd.ov.push_back(p.values[v]);
        }
        p.ready.push_back(std::move(rd));
    }
    p.src_flat.clear();
    p.src_count.clear();
    for (const Ready &r : p.ready) {
        p.src_count.push_back((uint32_t)r.scalar_src.size());
        p.src_flat.insert(p.src_flat.end(), r.scalar_src.begin(), r.scalar_src.end());
    }
    p.memo = StepMemo{};
}

int fail(slc_llama *m, int status, const char *msg) {
    if (m && m->dev) return slc_fail(m->dev, status, msg);
    return status;
}

int alloc_weights(slc_llama *m) {
    slc_device *d = m->dev;
    for (Weight &w : m->weights) {
        int rc;
        if (w.quant) {
            uint64_t row_bytes = m->cfg.quant_format == SLC_QUANT_INT4 ? (w.cols + 1) / 2 : w.cols;
            w.len = (w.rows * row_bytes + 3) / 4;
            uint64_t groups = (w.cols + m->cfg.group_size - 1) / m->cfg.group_size;
            if ((rc = slc_allocate_u32(d, w.len, 256, &w.buf)) != SLC_OK) return rc;
            if ((rc = slc_allocate_f32(d, w.rows * groups, 256, &w.scales)) != SLC_OK) return rc;
            if ((rc = slc_bind_quant(d, w.buf, w.scales, (uint32_t)m->cfg.quant_format,
                                     m->cfg.group_size)) != SLC_OK)
                return rc;
        } else {
            w.len = w.rows * w.cols;
            if ((rc = slc_allocate_f32(d, w.len, 256, &w.buf)) != SLC_OK) return rc;
        }
    }
    return SLC_OK;
}

int ensure_temp(slc_llama *m, uint64_t elems) {
    if (m->temp != UINT32_MAX && m->temp_elems >= elems) return SLC_OK;
    if (m->temp != UINT32_MAX) slc_release(m->dev, m->temp);
    m->temp = UINT32_MAX;
    int rc = slc_allocate_f32(m->dev, elems, 256, &m->temp);
    if (rc == SLC_OK) m->temp_elems = elems;
    return rc;
}

// Moves the f32 shard in m->temp into the weight's storage.
int commit_shard(slc_llama *m, Weight &w) {
    slc_device *d = m->dev;
    slc_buffer_ref src{m->temp, 0, 0, w.rows * w.cols};
    if (w.quant)
        return slc_quantize(d, src, w.rows, w.cols, (uint32_t)m->cfg.quant_format,
                            m->cfg.group_size, w.buf, w.scales);
    return cudaMemcpyAsync(d->buffers[w.buf].ptr, d->buffers[m->temp].ptr, w.len * 4,
                           cudaMemcpyDeviceToDevice, d->stream) == cudaSuccess
               ? SLC_OK
               : fail(m, SLC_ERR_EXECUTION, "device copy failed");
}

}  // namespace

extern "C" int slc_llama_create(slc_device *d, const slc_llama_config *cfg, slc_llama **out) {
    if (!d || !cfg || !out) return SLC_ERR_EXECUTION;
    *out = nullptr;
    const slc_llama_config &c = *cfg;
    if (c.layers == 0 || c.hidden == 0 || c.heads == 0 || c.kv_heads == 0 || c.head_dim == 0 ||
        c.inter == 0 || c.vocab == 0 || c.batch == 0 || c.prefill_len == 0 || c.max_seq == 0)
        return slc_fail(d, SLC_ERR_EXECUTION, "llama config has a zero dimension");
    if (c.heads % c.kv_heads != 0)
        return slc_fail(d, SLC_ERR_EXECUTION, "heads must be a multiple of kv_heads");
    if (c.prefill_len > c.max_seq)
        return slc_fail(d, SLC_ERR_EXECUTION, "prefill_len exceeds max_seq");
    int world = c.tp_world < 1 ? 1 : c.tp_world, rank = c.tp_rank;
    if (rank < 0 || rank >= world) return slc_fail(d, SLC_ERR_EXECUTION, "invalid tensor-parallel rank");
    if (c.heads % world || c.kv_heads % world || c.inter % world || c.vocab % world)
        return slc_fail(d, SLC_ERR_EXECUTION,
                        "heads, kv_heads, inter and vocab must divide by the tensor-parallel world");
    if (world > 1) {
        int r = 0, w = 1;
        slc_comm_world(d, &r, &w);
        if (w != world || r != rank)
            return slc_fail(d, SLC_ERR_EXECUTION, "device communicator does not match tp_rank/tp_world");
    }
    if (c.quant_format >= 0) {
        if (c.quant_format != SLC_QUANT_INT4 && c.quant_format != SLC_QUANT_INT8)
            return slc_fail(d, SLC_ERR_UNIMPLEMENTED, "unknown quantization format");
        if (c.group_size == 0) return slc_fail(d, SLC_ERR_EXECUTION, "group size must be nonzero");
        if (world > 1 && (((uint64_t)c.heads / world * c.head_dim) % c.group_size ||
                          ((uint64_t)c.inter / world) % c.group_size))
            return slc_fail(d, SLC_ERR_EXECUTION,
                            "row-parallel shards must hold whole quantization groups");
    }
    slc_llama *m = new (std::nothrow) slc_llama();
    if (!m) return SLC_ERR_OUT_OF_MEMORY;
    m->dev = d;
    m->cfg = c;
    m->cfg.tp_world = world;
    const char *memo_env = getenv("SLC_STEP_MEMO");
    m->memo = !(memo_env && strcmp(memo_env, "0") == 0);
    m->hq = c.heads / world;
    m->hkv = c.kv_heads / world;
    m->inter = c.inter / world;
    m->vocab = c.vocab / world;
    const uint64_t H = c.hidden, D = c.head_dim;
    add_weight(m, SLC_W_EMBED, 0, c.vocab, H, 0);
    for (uint32_t l = 0; l < c.layers; l++) {
        add_weight(m, SLC_W_ATTN_NORM, l, 1, H, 0);
        add_weight(m, SLC_W_Q, l, (uint64_t)c.heads * D, H, 1);
        add_weight(m, SLC_W_K, l, (uint64_t)c.kv_heads * D, H, 1);
        add_weight(m, SLC_W_V, l, (uint64_t)c.kv_heads * D, H, 1);
        add_weight(m, SLC_W_O, l, H, (uint64_t)c.heads * D, 2);
        add_weight(m, SLC_W_MLP_NORM, l, 1, H, 0);
        add_weight(m, SLC_W_GATE, l, c.inter, H, 1);
        add_weight(m, SLC_W_UP, l, c.inter, H, 1);
        add_weight(m, SLC_W_DOWN, l, H, c.inter, 2);
    }
    add_weight(m, SLC_W_FINAL_NORM, 0, 1, H, 0);
    add_weight(m, SLC_W_LM_HEAD, 0, c.vocab, H, 1);

    build_program(m, m->prefill, c.prefill_len);
    build_program(m, m->decode, 1);
    plan_memory(m->prefill);
    plan_memory(m->decode);

    int rc = alloc_weights(m);
    const uint64_t B = c.batch, T = c.prefill_len;
    uint64_t scratch = std::max(m->prefill.scratch_elems, m->decode.scratch_elems);
    uint64_t kv_elems = B * c.layers * 2 * (uint64_t)c.max_seq * m->hkv * D;
    if (rc == SLC_OK) rc = slc_allocate_f32(d, scratch, 256, &m->scratch);
    if (rc == SLC_OK) rc = slc_allocate_f32(d, kv_elems, 256, &m->kv);
    if (rc == SLC_OK) rc = slc_allocate_f32(d, B * c.vocab, 256, &m->logits_buf);
    if (rc == SLC_OK) rc = slc_allocate_u32(d, B * T, 64, &m->ids_prefill);
    if (rc == SLC_OK) rc = slc_allocate_u32(d, B * T, 64, &m->pos_prefill);
    if (rc == SLC_OK) rc = slc_allocate_u32(d, B, 64, &m->ids_decode);
    if (rc == SLC_OK) rc = slc_allocate_u32(d, B, 64, &m->pos_decode);
    if (rc != SLC_OK) {
        slc_llama_destroy(m);
        return rc;
    }
    bind(m, m->prefill, m->ids_prefill, m->pos_prefill);
    bind(m, m->decode, m->ids_decode, m->pos_decode);
    m->host_logits.assign(B * c.vocab, 0.f);
    cudaEventCreate(&m->ev_begin);
    cudaEventCreate(&m->ev_end);
    *out = m;
    return SLC_OK;
}

extern "C" void slc_llama_destroy(slc_llama *m) {
    if (!m) return;
    // Buffers belong to the device (the Device contract has no free); the
    // conversion staging buffer is the one temporary the engine releases.
    if (m->temp != UINT32_MAX) slc_release(m->dev, m->temp);
    if (m->ev_begin) cudaEventDestroy(m->ev_begin);
    if (m->ev_end) cudaEventDestroy(m->ev_end);
    delete m;
}

extern "C" int slc_llama_set_weight(slc_llama *m, int role, uint32_t layer, const float *full,
                                    uint64_t len) {
    if (!m || !full) return SLC_ERR_EXECUTION;
    int wi = weight_index(m, role, layer);
    if (wi < 0) return fail(m, SLC_ERR_EXECUTION, "unknown weight role or layer");
    Weight &w = m->weights[wi];
    if (len != w.full_rows * w.full_cols)
        return fail(m, SLC_ERR_EXECUTION, "weight length does not match its role shape");
    int rc = ensure_temp(m, w.rows * w.cols);
    if (rc != SLC_OK) return rc;
    std::vector<float> shard(w.rows * w.cols);
    for (uint64_t r = 0; r < w.rows; r++)
        memcpy(&shard[r * w.cols], full + (w.row0 + r) * w.full_cols + w.col0, w.cols * sizeof(float));
    slc_device *d = m->dev;
    if (cudaMemcpyAsync(d->buffers[m->temp].ptr, shard.data(), shard.size() * 4,
                        cudaMemcpyHostToDevice, d->stream) != cudaSuccess)
        return fail(m, SLC_ERR_EXECUTION, "host to device copy failed");
    rc = commit_shard(m, w);
    if (rc == SLC_OK) rc = slc_synchronize(d);
    return rc;
}

extern "C" int slc_llama_set_quant_weight(slc_llama *m, int role, uint32_t layer,
                                          const uint8_t *codes, uint64_t codes_bytes,
                                          const float *scales, uint64_t scales_len) {
    if (!m || !codes || !scales) return SLC_ERR_EXECUTION;
    int wi = weight_index(m, role, layer);
    if (wi < 0) return fail(m, SLC_ERR_EXECUTION, "unknown weight role or layer");
    Weight &w = m->weights[wi];
    if (!w.quant) return fail(m, SLC_ERR_EXECUTION, "weight role is not quantized in this model");
    const bool int4 = m->cfg.quant_format == SLC_QUANT_INT4;
    const uint64_t g = m->cfg.group_size;
    auto row_bytes = [&](uint64_t k) { return int4 ? (k + 1) / 2 : k; };
    const uint64_t full_rb = row_bytes(w.full_cols), full_groups = (w.full_cols + g - 1) / g;
    if (codes_bytes != w.full_rows * full_rb || scales_len != w.full_rows * full_groups)
        return fail(m, SLC_ERR_EXECUTION, "quantized weight sizes do not match its role shape");
    // This rank's shard: whole rows, or whole quantization groups of columns
    // (checked at creation), so the shard's codes and scales are slices.
    if (w.col0 % g != 0 || (int4 && w.col0 % 2 != 0))
        return fail(m, SLC_ERR_EXECUTION, "column shard does not start on a group");
    const uint64_t rb = row_bytes(w.cols), groups = (w.cols + g - 1) / g;
    const uint64_t b0 = int4 ? w.col0 / 2 : w.col0, g0 = w.col0 / g;
    std::vector<uint8_t> payload((w.rows * rb + 3) / 4 * 4, 0);
    std::vector<float> sc(w.rows * groups);
    for (uint64_t r = 0; r < w.rows; r++) {
        memcpy(&payload[r * rb], codes + (w.row0 + r) * full_rb + b0, rb);
        memcpy(&sc[r * groups], scales + (w.row0 + r) * full_groups + g0, groups * sizeof(float));
    }
    slc_device *d = m->dev;
    if (cudaMemcpyAsync(d->buffers[w.buf].ptr, payload.data(), payload.size(),
                        cudaMemcpyHostToDevice, d->stream) != cudaSuccess ||
        cudaMemcpyAsync(d->buffers[w.scales].ptr, sc.data(), sc.size() * sizeof(float),
                        cudaMemcpyHostToDevice, d->stream) != cudaSuccess)
        return fail(m, SLC_ERR_EXECUTION, "host to device copy failed");
    return slc_synchronize(d);
}

extern "C" int slc_llama_init_random(slc_llama *m, uint64_t seed, float stdev) {
    if (!m) return SLC_ERR_EXECUTION;
    slc_device *d = m->dev;
    uint64_t biggest = 0;
    for (const Weight &w : m->weights) biggest = std::max(biggest, w.rows * w.cols);
    int rc = ensure_temp(m, biggest);
    if (rc != SLC_OK) return rc;
    float *tmp = reinterpret_cast<float *>(d->buffers[m->temp].ptr);
    for (Weight &w : m->weights) {
        const bool norm = w.role == SLC_W_ATTN_NORM || w.role == SLC_W_MLP_NORM ||
                          w.role == SLC_W_FINAL_NORM;
        const uint64_t stream = splitmix64(seed ^ splitmix64((uint64_t)w.role * 1000003ull + w.layer));
        // Row r of the shard is row row0 + r of the full matrix: draws
        // (row0 + r) * full_cols + col0 .. + cols.
        if (w.cols == w.full_cols) {
            if (slc::k::fill_normal(d->stream, tmp, w.rows * w.cols, stream, w.row0 * w.full_cols,
                                    norm ? 1.0f : 0.0f, norm ? 0.1f : stdev) != cudaSuccess)
                return fail(m, SLC_ERR_EXECUTION, "weight generation failed");
        } else {
            for (uint64_t r = 0; r < w.rows; r++)
                if (slc::k::fill_normal(d->stream, tmp + r * w.cols, w.cols, stream,
                                        (w.row0 + r) * w.full_cols + w.col0, norm ? 1.0f : 0.0f,
                                        norm ? 0.1f : stdev) != cudaSuccess)
                    return fail(m, SLC_ERR_EXECUTION, "weight generation failed");
        }
        if ((rc = commit_shard(m, w)) != SLC_OK) return rc;
    }
    return slc_synchronize(d);
}

extern "C" int slc_llama_step(slc_llama *m, int mode, const uint32_t *ids,
                              const uint32_t *positions, uint32_t seq_len, uint32_t past_len,
                              float *logits, uint64_t logits_len) {
    if (!m || !ids || !positions) return SLC_ERR_EXECUTION;
    slc_device *d = m->dev;
    const slc_llama_config &c = m->cfg;
    Program &p = mode == SLC_STEP_PREFILL ? m->prefill : m->decode;
    const uint64_t T = p.seq, B = c.batch;
    if (mode != SLC_STEP_PREFILL && mode != SLC_STEP_DECODE)
        return fail(m, SLC_ERR_EXECUTION, "unknown step mode");
    if (seq_len < 1 || seq_len > T) return fail(m, SLC_ERR_EXECUTION, "seq_len exceeds the program");
    if ((uint64_t)past_len + T > c.max_seq) return fail(m, SLC_ERR_EXECUTION, "KV cache is full");
    if (logits && logits_len != B * c.vocab)
        return fail(m, SLC_ERR_EXECUTION, "logits length must be batch * vocab");
    int rc = slc_upload_u32(d, p.refs[p.ids].buffer, ids, B * T);
    if (rc == SLC_OK) rc = slc_upload_u32(d, p.refs[p.pos].buffer, positions, B * T);
    if (rc != SLC_OK) return rc;
    const uint32_t scalars_src[2] = {seq_len, past_len};
    uint32_t sc[4];
    // Device time of the step: with capture the dispatches below only record
    // (the work is submitted by slc_flush), so the begin event goes after them
    // and the events bracket device work only; host-side dispatch cost shows
    // in the caller's wall clock.
    const bool deferred = d->capture != nullptr;
    if (deferred && m->memo && capture_memo_valid(d, &p.memo)) {
        // The program's commands replay as one known graph: relaunch it with
        // this step's scalars instead of dispatching every command again
        // (the checks above are the ones the scalars get at dispatch).
        cudaEventRecord(m->ev_begin, d->stream);
        if ((rc = capture_memo_replay(d, &p.memo, scalars_src, 2)) != SLC_OK) return rc;
        m->memo_steps++;
    } else {
        if (!deferred) cudaEventRecord(m->ev_begin, d->stream);
        for (const Ready &r : p.ready) {
            for (size_t i = 0; i < r.scalar_src.size(); i++) sc[i] = scalars_src[r.scalar_src[i]];
            rc = slc_dispatch(d, &r.op, r.in.data(), r.iv.data(), r.in.size(), r.out.data(),
                              r.ov.data(), r.out.size(), sc, r.scalar_src.size());
            if (rc != SLC_OK) return rc;
        }
        if (deferred) cudaEventRecord(m->ev_begin, d->stream);
        rc = deferred && m->memo ? capture_flush_memo(d, &p.memo, p.src_flat.data(),
                                                      p.src_count.data(), p.ready.size())
                                 : slc_flush(d);
        if (rc != SLC_OK) return rc;
    }
    cudaEventRecord(m->ev_end, d->stream);
    if ((rc = slc_synchronize(d)) != SLC_OK) return rc;
    cudaEventElapsedTime(&m->last_step_ms, m->ev_begin, m->ev_end);
    if (logits) rc = slc_download_f32(d, m->logits_buf, logits, B * c.vocab);
    return rc;
}

extern "C" int slc_llama_generate(slc_llama *m, const uint32_t *prompt, uint32_t steps,
                                  uint32_t *out_ids, float *margins) {
    if (!m || !prompt || !out_ids) return SLC_ERR_EXECUTION;
    const slc_llama_config &c = m->cfg;
    const uint64_t B = c.batch, T = c.prefill_len, V = c.vocab;
    if (T + steps > c.max_seq) return fail(m, SLC_ERR_EXECUTION, "generation exceeds max_seq");
    std::vector<uint32_t> pos(B * T), ids(B), dpos(B);
    for (uint64_t b = 0; b < B; b++)
        for (uint64_t t = 0; t < T; t++) pos[b * T + t] = (uint32_t)t;
    float *lg = m->host_logits.data();
    auto pick = [&](uint32_t s) {
        for (uint64_t b = 0; b < B; b++) {
            const float *row = lg + b * V;
            uint64_t best = 0;
            for (uint64_t i = 1; i < V; i++)
                if (row[i] > row[best]) best = i;
            float second = -INFINITY;
            for (uint64_t i = 0; i < V; i++)
                if (i != best && row[i] > second) second = row[i];
            ids[b] = (uint32_t)best;
            out_ids[(uint64_t)s * B + b] = (uint32_t)best;
            if (margins) margins[(uint64_t)s * B + b] = row[best] - second;
        }
    };
    int rc = slc_llama_step(m, SLC_STEP_PREFILL, prompt, pos.data(), (uint32_t)T, 0, lg, B * V);
    if (rc != SLC_OK) return rc;
    pick(0);
    for (uint32_t s = 0; s < steps; s++) {
        for (uint64_t b = 0; b < B; b++) dpos[b] = (uint32_t)(T + s);
        rc = slc_llama_step(m, SLC_STEP_DECODE, ids.data(), dpos.data(), 1, (uint32_t)(T + s), lg,
                            B * V);
        if (rc != SLC_OK) return rc;
        pick(s + 1);
    }
    return SLC_OK;
}

extern "C" int slc_llama_kv_buffer(const slc_llama *m, uint32_t *buffer, uint64_t *elements) {
    if (!m) return SLC_ERR_EXECUTION;
    if (buffer) *buffer = m->kv;
    if (elements) *elements = m->decode.refs[m->decode.kv].len;
    return SLC_OK;
}

extern "C" int slc_llama_memo_steps(const slc_llama *m, uint64_t *count) {
    if (!m || !count) return SLC_ERR_EXECUTION;
    *count = m->memo_steps;
    return SLC_OK;
}

extern "C" int slc_llama_command_count(const slc_llama *m, int mode, uint64_t *count) {
    if (!m || !count) return SLC_ERR_EXECUTION;
    *count = (mode == SLC_STEP_PREFILL ? m->prefill : m->decode).ready.size();
    return SLC_OK;
}

extern "C" int slc_llama_weight_bytes(const slc_llama *m, uint64_t *bytes) {
    if (!m || !bytes) return SLC_ERR_EXECUTION;
    uint64_t total = 0;
    for (const Weight &w : m->weights) {
        if (w.quant) {
            uint64_t groups = (w.cols + m->cfg.group_size - 1) / m->cfg.group_size;
            total += w.len * 4 + w.rows * groups * 4;
        } else {
            total += w.len * 4;
        }
    }
    *bytes = total;
    return SLC_OK;
}

extern "C" int slc_llama_weight_ref(const slc_llama *m, int role, uint32_t layer,
                                    slc_buffer_ref *ref, slc_value *value) {
    if (!m) return SLC_ERR_EXECUTION;
    for (const Weight &w : m->weights) {
        if (w.role != role || w.layer != layer) continue;
        if (ref) *ref = slc_buffer_ref{w.buf, 0, 0, w.len};
        if (value) {
            bool norm = role == SLC_W_ATTN_NORM || role == SLC_W_MLP_NORM || role == SLC_W_FINAL_NORM;
            *value = norm ? make_value(SLC_F32, SLC_ROLE_PARAM, {w.cols})
                          : make_value(SLC_F32, SLC_ROLE_PARAM, {w.rows, w.cols});
            if (w.quant) {
                value->encoding = SLC_ENC_GROUPWISE;
                value->quant_format = (uint32_t)m->cfg.quant_format;
                value->group_size = m->cfg.group_size;
            }
        }
        return SLC_OK;
    }
    return slc_fail(m->dev, SLC_ERR_EXECUTION, "unknown weight role or layer");
}

extern "C" int slc_llama_last_step_ms(const slc_llama *m, float *ms) {
    if (!m || !ms) return SLC_ERR_EXECUTION;
    *ms = m->last_step_ms;
    return SLC_OK;
}
