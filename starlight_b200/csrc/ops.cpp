// Operator layer of backend-cuda: per-operator geometry validation (the
// checks and messages of run_op, crates/backends/backend-cpu/src/
// device.rs:773-1227, and of the reference kernels it calls) followed by the
// kernel launches. Every check of a command runs before its first launch.
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <algorithm>

#include "device_internal.h"
#include "kernels/kernels.h"

using namespace slc;

namespace {

struct Cmd {
    const slc_op *op;
    const slc_buffer_ref *in;
    const slc_value *iv;
    uint64_t n_in;
    const slc_buffer_ref *out;
    const slc_value *ov;
    uint64_t n_out;
    const uint32_t *scalars;
    uint64_t n_scalars;
    int64_t state_index;
    const uint32_t *dyn_scalars;  // device copies of the scalars (graph replay) or null
};

struct Dims {
    uint32_t rank = 0;
    uint64_t ext[SLC_MAX_RANK] = {};
    uint64_t operator[](uint32_t i) const { return ext[i]; }
};

// A failed check: status + static message.
struct Fail {
    int code;
    const char *msg;
};

struct Checker {
    slc_device *d;
    const Cmd &c;
    bool failed = false;
    int rc = SLC_OK;

    int fail(int code, const char *msg) {
        if (!failed) {
            failed = true;
            rc = slc_fail(d, code, msg);
        }
        return rc;
    }
    int exec(const char *msg) { return fail(SLC_ERR_EXECUTION, msg); }
    int overflow() { return fail(SLC_ERR_SHAPE_OVERFLOW, "tensor shape product overflows"); }

    bool dims(const slc_value &v, Dims *o) {
        if (v.rank > SLC_MAX_RANK) {
            overflow();
            return false;
        }
        o->rank = v.rank;
        for (uint32_t i = 0; i < v.rank; i++) o->ext[i] = v.dims[i];
        return true;
    }
    bool ivalue(uint64_t i, Dims *o) {
        if (i >= c.n_in) {
            exec("operator is missing an input value");
            return false;
        }
        return dims(c.iv[i], o);
    }
    bool ovalue(uint64_t i, Dims *o) {
        if (i >= c.n_out) {
            exec("operator is missing an output value");
            return false;
        }
        return dims(c.ov[i], o);
    }
    bool dim(const Dims &d_, uint32_t i, uint64_t *o) {
        if (i < d_.rank) {
            *o = d_.ext[i];
            return true;
        }
        exec("operator rank is too small");
        return false;
    }
    bool last(const Dims &d_, uint64_t *o) {
        if (d_.rank == 0) {
            exec("operator requires at least one dimension");
            return false;
        }
        *o = d_.ext[d_.rank - 1];
        return true;
    }
    bool product(const Dims &d_, uint32_t end, uint64_t *o) {
        if (end > d_.rank) {
            exec("operator rank is too small");
            return false;
        }
        uint64_t p = 1;
        for (uint32_t i = 0; i < end; i++) {
            if (d_.ext[i] != 0 && p > UINT64_MAX / d_.ext[i]) {
                overflow();
                return false;
            }
            p *= d_.ext[i];
        }
        *o = p;
        return true;
    }
    bool scalar(uint64_t i, uint64_t *o) {
        if (i >= c.n_scalars) {
            exec("operator is missing a scalar input");
            return false;
        }
        *o = c.scalars[i];
        return true;
    }
    bool is_quant(uint64_t i) const {
        return i < c.n_in && (int64_t)i != c.state_index && c.iv[i].encoding == SLC_ENC_GROUPWISE;
    }
    // f32_input / u32_input, device.rs:1244-1264.
    float *f32(uint64_t i) {
        if (i >= c.n_in || (int64_t)i == c.state_index || c.iv[i].dtype != SLC_F32 ||
            c.iv[i].encoding != SLC_ENC_DENSE) {
            exec("operator is missing an f32 input");
            return nullptr;
        }
        return reinterpret_cast<float *>(d->buffers[c.in[i].buffer].ptr) + c.in[i].offset;
    }
    const uint32_t *u32(uint64_t i) {
        if (i >= c.n_in || (int64_t)i == c.state_index || c.iv[i].dtype != SLC_U32) {
            exec("operator is missing a u32 input");
            return nullptr;
        }
        return reinterpret_cast<const uint32_t *>(d->buffers[c.in[i].buffer].ptr) + c.in[i].offset;
    }
    const uint32_t *u32_host(uint64_t i) {
        return d->buffers[c.in[i].buffer].shadow.data() + c.in[i].offset;
    }
    float *output() {
        return reinterpret_cast<float *>(d->buffers[c.out[0].buffer].ptr) + c.out[0].offset;
    }
    float *state() {
        return reinterpret_cast<float *>(d->buffers[c.in[c.state_index].buffer].ptr) +
               c.in[c.state_index].offset;
    }
};

bool same(const Dims &a, const Dims &b) {
    if (a.rank != b.rank) return false;
    for (uint32_t i = 0; i < a.rank; i++)
        if (a.ext[i] != b.ext[i]) return false;
    return true;
}

bool checked_mul(uint64_t a, uint64_t b, uint64_t *o) {
    if (a != 0 && b > UINT64_MAX / a) return false;
    *o = a * b;
    return true;
}

// broadcast_batch, device.rs:1333-1353.
bool broadcast_batch(Checker &ck, uint64_t left, uint64_t right, uint64_t *out) {
    if (left == right) {
        *out = left;
        return true;
    }
    if (left == 0 || right == 0) {
        if (std::max(left, right) <= 1) {
            *out = 0;
            return true;
        }
        ck.exec("matmul batch dimensions are not broadcastable");
        return false;
    }
    if (left == 1) {
        *out = right;
        return true;
    }
    if (right == 1) {
        *out = left;
        return true;
    }
    ck.exec("matmul batch dimensions are not broadcastable");
    return false;
}

// check_state_geometry, device.rs:1466-1488.
bool state_geometry(Checker &ck, const Dims &st, uint64_t batch, uint64_t kv_heads,
                    uint64_t head_dim, uint64_t layer, uint64_t *layers, uint64_t *max_seq) {
    if (st.rank != 6 || st[0] != batch || st[2] != 2 || st[4] != kv_heads || st[5] != head_dim) {
        ck.exec("KV cache shape must be [batch, layers, 2, max_seq, kv_heads, head_dim]");
        return false;
    }
    *layers = st[1];
    if (layer >= *layers) {
        ck.exec("attention layer is out of range");
        return false;
    }
    *max_seq = st[3];
    return true;
}

// Workspace regions: see device_internal.h. The GEMV gets the tickets and
// the scratch behind them (partials at +256 KiB).
void *gemv_workspace(slc_device *d) { return d->workspace; }
uint64_t gemv_workspace_bytes(slc_device *d) { return d->workspace_bytes / 2 - kAttnTicketBytes; }
void *kernel_scratch(slc_device *d) { return ws_scratch(d); }
uint64_t kernel_scratch_bytes(slc_device *d) { return ws_scratch_bytes(d); }
float *intermediates(slc_device *d) {
    return reinterpret_cast<float *>(d->workspace + d->workspace_bytes / 2);
}
uint64_t intermediate_floats(slc_device *d) { return d->workspace_bytes / 2 / sizeof(float); }

// A matmul right-hand side: dense f32 or a bound quantized payload.
struct Weight {
    bool quant = false;
    const float *dense = nullptr;
    k::QuantWeight q{};
};

bool weight_of(Checker &ck, uint64_t i, uint64_t rows, uint64_t kk, Weight *w) {
    if (ck.is_quant(i)) {
        const slc_value &v = ck.c.iv[i];
        w->quant = true;
        int rc = slc_quant_view(ck.d, ck.c.in[i].buffer, ck.c.in[i].offset, rows, kk,
                                v.quant_format, v.group_size, &w->q);
        if (rc != SLC_OK) {
            ck.failed = true;
            ck.rc = rc;
            return false;
        }
        return true;
    }
    w->dense = ck.f32(i);
    return w->dense != nullptr;
}

// y[rows, n] = x[rows, k] . W[n, k]^T for either kind of weight.
cudaError_t matmul_rows(slc_device *d, const float *x, uint64_t rows, uint64_t kk,
                        const Weight &w, uint64_t n, float *y) {
    if (w.quant)
        return k::qmatmul(d->stream, x, rows, w.q, y, gemv_workspace(d), gemv_workspace_bytes(d),
                          d->device_flag);
    return k::matmul_f32(d->stream, x, w.dense, y, 1, 1, rows, kk, n, true);
}

int finish(Checker &ck, cudaError_t e) {
    if (e != cudaSuccess) return ck.exec("CUDA kernel launch failed");
    return SLC_OK;
}

#define REQUIRE(expr)             \
    do {                          \
        if (!(expr)) return ck.rc; \
    } while (0)

int run_op(slc_device *d, const Cmd &c, bool launch) {
    Checker ck{d, c};
    cudaStream_t s = d->stream;
    switch (c.op->code) {
    case SLC_OP_MATMUL_NT:
    case SLC_OP_MATMUL_NN: {
        const bool nt = c.op->code == SLC_OP_MATMUL_NT;
        Dims l, r, o;
        REQUIRE(ck.ivalue(0, &l) && ck.ivalue(1, &r) && ck.ovalue(0, &o));
        // matmul_geometry, device.rs:1301-1331.
        if (l.rank < 2 || r.rank < 2 || o.rank < 2)
            return ck.exec("matmul operands and output must have rank at least 2");
        uint64_t m = l[l.rank - 2], kk = l[l.rank - 1];
        uint64_t rk = nt ? r[r.rank - 1] : r[r.rank - 2];
        uint64_t n = nt ? r[r.rank - 2] : r[r.rank - 1];
        if (kk != rk) return ck.exec("matmul reduction dimensions must match");
        uint64_t ba, bb, batch, ob;
        REQUIRE(ck.product(l, l.rank - 2, &ba) && ck.product(r, r.rank - 2, &bb));
        REQUIRE(broadcast_batch(ck, ba, bb, &batch));
        if (o[o.rank - 2] != m || o[o.rank - 1] != n)
            return ck.exec("matmul output shape must be m x n");
        REQUIRE(ck.product(o, o.rank - 2, &ob));
        if (ob != batch) return ck.exec("matmul output batch must match the operands");
        const float *a = ck.f32(0);
        REQUIRE(a);
        if (ck.is_quant(1)) {
            if (!nt) return ck.fail(SLC_ERR_UNIMPLEMENTED, "quantized weights require MatMulNT");
            if (bb != 1 && batch != 0)
                return ck.fail(SLC_ERR_UNIMPLEMENTED, "quantized matmul weights must not be batched");
            Weight w;
            REQUIRE(weight_of(ck, 1, n, kk, &w));
            if (!launch || batch == 0) return SLC_OK;
            return finish(ck, k::qmatmul(s, a, batch * m, w.q, ck.output(), gemv_workspace(d),
                                         gemv_workspace_bytes(d), d->device_flag));
        }
        const float *w = ck.f32(1);
        REQUIRE(w);
        if (!launch || batch == 0) return SLC_OK;
        if (kk == 0)
            return finish(ck, cudaMemsetAsync(ck.output(), 0, batch * m * n * 4, s));
        return finish(ck, k::matmul_f32(s, a, w, ck.output(), ba, bb, m, kk, n, nt));
    }
    case SLC_OP_SOFTMAX:
    case SLC_OP_SOFTMAX_CAUSAL: {
        const bool causal = c.op->code == SLC_OP_SOFTMAX_CAUSAL;
        Dims x, o;
        REQUIRE(ck.ivalue(0, &x) && ck.ovalue(0, &o));
        if (!same(x, o))
            return ck.exec(causal ? "softmax_causal output shape must match its input"
                                  : "softmax output shape must match its input");
        uint64_t cols, rows, seq = 0, past = 0;
        REQUIRE(ck.last(x, &cols) && ck.product(x, x.rank - 1, &rows));
        if (causal) REQUIRE(ck.scalar(0, &seq) && ck.scalar(1, &past));
        const float *in = ck.f32(0);
        REQUIRE(in);
        // softmax.rs:19-25 / :61-91.
        if (rows == 0 || cols == 0)
            return ck.exec(causal ? "softmax_causal requires nonzero rows and cols"
                                  : "softmax requires nonzero rows and cols");
        if (causal) {
            if (seq == 0) return ck.exec("softmax_causal requires a nonzero seq");
            if (cols != past + seq) return ck.exec("softmax_causal requires cols == past_len + seq");
            if (rows % seq != 0)
                return ck.exec("softmax_causal requires rows to be a multiple of seq");
        }
        if (!launch) return SLC_OK;
        return finish(ck, causal ? k::softmax_causal(s, in, ck.output(), rows, cols, seq, past)
                                 : k::softmax(s, in, ck.output(), rows, cols));
    }
    case SLC_OP_RMS_NORM: {
        Dims x, w, o;
        REQUIRE(ck.ivalue(0, &x) && ck.ivalue(1, &w) && ck.ovalue(0, &o));
        uint64_t hidden, rows;
        REQUIRE(ck.last(x, &hidden) && ck.product(x, x.rank - 1, &rows));
        if (w.rank != 1 || w[0] != hidden)
            return ck.exec("rms_norm weight shape must be [hidden]");
        if (!same(x, o)) return ck.exec("rms_norm output shape must match its input");
        const float *xp = ck.f32(0), *wp = ck.f32(1);
        REQUIRE(xp && wp);
        if (hidden == 0) return ck.exec("rms_norm requires a nonzero hidden size");
        if (!launch) return SLC_OK;
        return finish(ck, k::rms_norm(s, xp, wp, ck.output(), rows, hidden, c.op->eps));
    }
    case SLC_OP_ROPE: {
        Dims x, p, o;
        REQUIRE(ck.ivalue(0, &x) && ck.ivalue(1, &p) && ck.ovalue(0, &o));
        uint64_t b, h, sq, hd;
        // rope_geometry, device.rs:1409-1428.
        if (x.rank == 4) {
            b = x[0]; h = x[1]; sq = x[2]; hd = x[3];
        } else if (x.rank == 3) {
            b = x[0]; h = 1; sq = x[1]; hd = x[2];
        } else {
            return ck.exec("rope input must have rank 3 or 4");
        }
        if (p.rank != 2 || p[0] != b || p[1] != sq)
            return ck.exec("rope positions shape must be [batch, seq]");
        if (!same(x, o)) return ck.exec("rope output shape must match its input");
        const float *xp = ck.f32(0);
        REQUIRE(xp);
        const uint32_t *pos = ck.u32(1);
        REQUIRE(pos);
        if (hd == 0 || hd % 2 != 0) return ck.exec("head_dim must be a positive even number");
        if (c.op->rope_variant > SLC_ROPE_GPTJ)
            return ck.fail(SLC_ERR_UNIMPLEMENTED, "unknown rope variant");
        if (!launch) return SLC_OK;
        return finish(ck, k::rope(s, xp, pos, ck.output(), b, h, sq, hd, c.op->theta,
                                  c.op->rope_variant == SLC_ROPE_GPTJ));
    }
    case SLC_OP_SILU:
    case SLC_OP_SCALE: {
        const bool silu = c.op->code == SLC_OP_SILU;
        Dims x, o;
        REQUIRE(ck.ivalue(0, &x) && ck.ovalue(0, &o));
        if (!same(x, o))
            return ck.exec(silu ? "silu output shape must match its input"
                                : "scale output shape must match its input");
        const float *xp = ck.f32(0);
        REQUIRE(xp);
        uint64_t n;
        REQUIRE(ck.product(x, x.rank, &n));
        if (!launch) return SLC_OK;
        return finish(ck, silu ? k::silu(s, xp, ck.output(), n)
                               : k::scale(s, xp, c.op->factor, ck.output(), n));
    }
    case SLC_OP_MUL:
    case SLC_OP_ADD: {
        Dims a, b, o;
        REQUIRE(ck.ivalue(0, &a) && ck.ivalue(1, &b) && ck.ovalue(0, &o));
        if (!same(a, b) || !same(a, o))
            return ck.exec("mul/add operands and output must have identical shapes");
        uint64_t n;
        REQUIRE(ck.product(a, a.rank, &n));
        const float *ap = ck.f32(0), *bp = ck.f32(1);
        REQUIRE(ap && bp);
        if (!launch) return SLC_OK;
        return finish(ck, c.op->code == SLC_OP_MUL ? k::mul(s, ap, bp, ck.output(), n)
                                                    : k::add(s, ap, bp, ck.output(), n));
    }
    case SLC_OP_GATHER: {
        Dims t, ids, o;
        REQUIRE(ck.ivalue(0, &t) && ck.ivalue(1, &ids) && ck.ovalue(0, &o));
        if (t.rank != 2) return ck.exec("gather table must have shape [vocab, hidden]");
        uint64_t vocab = t[0], hidden = t[1], rows;
        REQUIRE(ck.product(ids, ids.rank, &rows));
        if (o.rank != ids.rank + 1) return ck.exec("gather output rank must be the id rank plus one");
        for (uint32_t i = 0; i < ids.rank; i++)
            if (o[i] != ids[i]) return ck.exec("gather output prefix must match the id shape");
        uint64_t ow;
        REQUIRE(ck.last(o, &ow));
        if (ow != hidden) return ck.exec("gather output width must equal hidden");
        const float *tp = ck.f32(0);
        REQUIRE(tp);
        const uint32_t *idp = ck.u32(1);
        REQUIRE(idp);
        // layout.rs:37-43: every id is checked before the first write.
        const uint32_t *host_ids = ck.u32_host(1);
        for (uint64_t i = 0; i < rows; i++)
            if (host_ids[i] >= vocab) return ck.exec("id out of range");
        if (!launch) return SLC_OK;
        return finish(ck, k::gather(s, tp, idp, ck.output(), vocab, hidden, rows, d->device_flag));
    }
    case SLC_OP_LAST_TOKEN: {
        Dims x, o;
        REQUIRE(ck.ivalue(0, &x) && ck.ovalue(0, &o));
        uint64_t seq_len;
        REQUIRE(ck.scalar(0, &seq_len));
        if (x.rank != 3 || o.rank != 2) return ck.exec("last_token shapes must be [B, M, H] -> [B, H]");
        uint64_t b = x[0], sq = x[1], h = x[2];
        if (o[0] != b || o[1] != h) return ck.exec("last_token output shape must be [batch, hidden]");
        const float *xp = ck.f32(0);
        REQUIRE(xp);
        if (seq_len < 1 || seq_len > sq) return ck.exec("last_token requires 1 <= seq_len <= seq");
        if (!launch) return SLC_OK;
        return finish(ck, k::last_token(s, xp, ck.output(), b, sq, h, seq_len, c.dyn_scalars,
                                        d->device_flag));
    }
    case SLC_OP_KV_APPEND: {
        Dims kd, vd;
        REQUIRE(ck.ivalue(0, &kd) && ck.ivalue(1, &vd));
        uint64_t past;
        REQUIRE(ck.scalar(0, &past));
        const uint64_t layer = c.op->layer;
        // attention_kv_geometry, device.rs:1451-1464.
        if (kd.rank != 4 || vd.rank != 4) return ck.exec("kv_append key/value must have rank 4");
        if (!same(kd, vd)) return ck.exec("kv_append key and value shapes must match");
        uint64_t b = kd[0], hkv = kd[1], sq = kd[2], hd = kd[3];
        Dims st;
        REQUIRE(ck.dims(c.iv[c.state_index], &st));
        uint64_t layers, max_seq;
        REQUIRE(state_geometry(ck, st, b, hkv, hd, layer, &layers, &max_seq));
        const float *kp = ck.f32(0), *vp = ck.f32(1);
        REQUIRE(kp && vp);
        // attention.rs:51-59.
        if (past + sq > max_seq) return ck.exec("past_len + seq exceeds max_seq");
        if (!launch) return SLC_OK;
        k::KvGeometry g{b, layers, layer, hkv, hd, max_seq};
        return finish(ck, k::kv_append(s, kp, vp, ck.state(), g, past, sq, c.dyn_scalars));
    }
    case SLC_OP_SPLIT_HEADS: {
        Dims x, o;
        REQUIRE(ck.ivalue(0, &x) && ck.ovalue(0, &o));
        const uint64_t heads = c.op->heads, hd = c.op->head_dim;
        // split_geometry, device.rs:1430-1449.
        if (x.rank != 3)
            return ck.exec("split_heads input shape must be [batch, seq, heads * head_dim]");
        uint64_t b = x[0], sq = x[1], width;
        if (!checked_mul(heads, hd, &width)) return ck.overflow();
        if (x[2] != width) return ck.exec("split_heads input width must equal heads * head_dim");
        if (o.rank != 4 || o[0] != b || o[1] != heads || o[2] != sq || o[3] != hd)
            return ck.exec("split_heads output shape must be [batch, heads, seq, head_dim]");
        const float *xp = ck.f32(0);
        REQUIRE(xp);
        if (!launch) return SLC_OK;
        return finish(ck, k::split_heads(s, xp, ck.output(), b, sq, heads, hd));
    }
    case SLC_OP_MERGE_HEADS: {
        Dims x, o;
        REQUIRE(ck.ivalue(0, &x) && ck.ovalue(0, &o));
        const uint64_t heads = c.op->heads, hd = c.op->head_dim;
        if (x.rank != 4)
            return ck.exec("merge_heads input shape must be [batch, heads, seq, head_dim]");
        uint64_t b = x[0], sq = x[2];
        if (x[1] != heads || x[3] != hd)
            return ck.exec("merge_heads input does not match its heads/head_dim attributes");
        uint64_t width;
        if (!checked_mul(heads, hd, &width)) return ck.overflow();
        if (o.rank != 3 || o[0] != b || o[1] != sq || o[2] != width)
            return ck.exec("merge_heads output shape must be [batch, seq, heads * head_dim]");
        const float *xp = ck.f32(0);
        REQUIRE(xp);
        if (!launch) return SLC_OK;
        return finish(ck, k::merge_heads(s, xp, ck.output(), b, sq, heads, hd));
    }
    case SLC_OP_CAUSAL_ATTENTION: {
        Dims qd, kd, vd, od;
        REQUIRE(ck.ivalue(0, &qd) && ck.ivalue(1, &kd) && ck.ivalue(2, &vd) && ck.ovalue(0, &od));
        uint64_t past;
        REQUIRE(ck.scalar(0, &past));
        const uint64_t layer = c.op->layer, heads = c.op->heads, kvh = c.op->kv_heads,
                       hd = c.op->head_dim;
        if (qd.rank != 4 || kd.rank != 4 || vd.rank != 4 || od.rank != 4)
            return ck.exec("causal_attention operands must have rank 4");
        uint64_t b = qd[0], sq = qd[2];
        if (qd[1] != heads || qd[3] != hd)
            return ck.exec("causal_attention query shape does not match its attributes");
        if (kd[0] != b || vd[0] != b || kd[1] != kvh || vd[1] != kvh || kd[2] != sq ||
            vd[2] != sq || kd[3] != hd || vd[3] != hd)
            return ck.exec(
                "causal_attention key/value shapes must be [batch, kv_heads, seq, head_dim]");
        if (!same(od, qd)) return ck.exec("causal_attention output shape must match the query shape");
        Dims st;
        REQUIRE(ck.dims(c.iv[c.state_index], &st));
        uint64_t layers, max_seq;
        REQUIRE(state_geometry(ck, st, b, kvh, hd, layer, &layers, &max_seq));
        const float *qp = ck.f32(0), *kp = ck.f32(1), *vp = ck.f32(2);
        REQUIRE(qp && kp && vp);
        // attention.rs:146-156, then kv_append's checks (:51-59).
        if (kvh == 0) return ck.exec("kv_heads must be nonzero");
        if (heads == 0) return ck.exec("heads must be nonzero");
        if (heads % kvh != 0) return ck.exec("heads must be a multiple of kv_heads");
        if (past + sq > max_seq) return ck.exec("past_len + seq exceeds max_seq");
        if (hd > 384) return ck.fail(SLC_ERR_UNIMPLEMENTED, "causal_attention supports head_dim <= 384");
        uint64_t need = k::attention_workspace_bytes(b, heads, kvh, sq, past, hd, max_seq,
                                                     c.dyn_scalars != nullptr);
        if (need > kernel_scratch_bytes(d))
            return ck.exec("device workspace is too small for this attention shape");
        if (!launch) return SLC_OK;
        k::KvGeometry g{b, layers, layer, kvh, hd, max_seq};
        k::AttnScratch scr{kernel_scratch(d), kernel_scratch_bytes(d), ws_attn_tickets(d),
                           kAttnTicketBytes / sizeof(unsigned), d->device_flag};
        return finish(ck, k::causal_attention(s, qp, kp, vp, ck.state(), ck.output(), g, heads, sq,
                                              past, c.op->scale, scr, c.dyn_scalars));
    }
    case SLC_OP_SWIGLU: {
        Dims x, g, u, dn, o;
        REQUIRE(ck.ivalue(0, &x) && ck.ivalue(1, &g) && ck.ivalue(2, &u) && ck.ivalue(3, &dn) &&
                ck.ovalue(0, &o));
        uint64_t hidden, rows;
        REQUIRE(ck.last(x, &hidden) && ck.product(x, x.rank - 1, &rows));
        if (g.rank != 2 || u.rank != 2 || dn.rank != 2)
            return ck.exec("swiglu weights must have rank 2");
        uint64_t inter = g[0];
        if (g[1] != hidden || u[0] != inter || u[1] != hidden || dn[0] != hidden || dn[1] != inter)
            return ck.exec(
                "swiglu weight shapes must be [inter, hidden], [inter, hidden], [hidden, inter]");
        if (!same(x, o)) return ck.exec("swiglu output shape must match its input");
        const float *xp = ck.f32(0);
        REQUIRE(xp);
        Weight wg, wu, wd;
        REQUIRE(weight_of(ck, 1, inter, hidden, &wg) && weight_of(ck, 2, inter, hidden, &wu) &&
                weight_of(ck, 3, hidden, inter, &wd));
        if (hidden == 0) return ck.exec("swiglu requires a nonzero hidden size");
        if (inter == 0) return ck.exec("swiglu requires a nonzero inter size");
        uint64_t chunk = intermediate_floats(d) / (2 * inter);
        if (chunk == 0) return ck.exec("device workspace is too small for this swiglu shape");
        if (!launch || rows == 0) return SLC_OK;
        float *gb = intermediates(d), *ub = gb + chunk * inter;
        float *outp = ck.output();
        // Decode-sized: gate and up in one TMA GEMV launch, then down with
        // silu(gate) * up computed while its input is staged (two launches
        // instead of four; the same arithmetic as the general path below).
        if (wg.quant && wu.quant && wd.quant && rows <= 32 && rows <= chunk) {
            const k::QuantSeg gu[2] = {{wg.q, gb}, {wu.q, ub}};
            const k::QuantSeg dn[1] = {{wd.q, outp}};
            if (k::qgemv_tma_group_supported(gu, 2, rows) &&
                k::qgemv_tma_group_supported(dn, 1, rows) && k::qgemv_tma_x_aligned(xp) &&
                k::qgemv_tma_x_aligned(gb) && k::qgemv_tma_x_aligned(ub) &&
                k::qgemv_tma_group_workspace_bytes(gu, 2, rows) <= gemv_workspace_bytes(d) &&
                k::qgemv_tma_group_workspace_bytes(dn, 1, rows) <= gemv_workspace_bytes(d)) {
                cudaError_t e = k::qgemv_tma_group(s, xp, nullptr, rows, gu, 2, gemv_workspace(d),
                                                   d->device_flag);
                if (e == cudaSuccess)
                    e = k::qgemv_tma_group(s, gb, ub, rows, dn, 1, gemv_workspace(d),
                                           d->device_flag);
                return finish(ck, e);
            }
        }
        for (uint64_t r0 = 0; r0 < rows; r0 += chunk) {
            uint64_t rc = std::min(chunk, rows - r0);
            cudaError_t e = matmul_rows(d, xp + r0 * hidden, rc, hidden, wg, inter, gb);
            if (e == cudaSuccess) e = matmul_rows(d, xp + r0 * hidden, rc, hidden, wu, inter, ub);
            if (e == cudaSuccess) e = k::silu_mul(s, gb, ub, gb, rc * inter);
            if (e == cudaSuccess) e = matmul_rows(d, gb, rc, inter, wd, hidden, outp + r0 * hidden);
            if (e != cudaSuccess) return finish(ck, e);
        }
        return SLC_OK;
    }
    case SLC_OP_RMS_NORM_MATMUL: {
        Dims x, w, mtx, o;
        REQUIRE(ck.ivalue(0, &x) && ck.ivalue(1, &w) && ck.ivalue(2, &mtx) && ck.ovalue(0, &o));
        uint64_t hidden, rows;
        REQUIRE(ck.last(x, &hidden) && ck.product(x, x.rank - 1, &rows));
        if (w.rank != 1 || w[0] != hidden)
            return ck.exec("rms_norm_matmul weight shape must be [hidden]");
        if (mtx.rank != 2 || mtx[1] != hidden)
            return ck.exec("rms_norm_matmul matrix shape must be [out_features, hidden]");
        uint64_t nout = mtx[0];
        if (o.rank != x.rank) return ck.exec("rms_norm_matmul output rank must match its input rank");
        for (uint32_t i = 0; i + 1 < x.rank; i++)
            if (o[i] != x[i]) return ck.exec("rms_norm_matmul output prefix must match its input");
        uint64_t ol;
        REQUIRE(ck.last(o, &ol));
        if (ol != nout) return ck.exec("rms_norm_matmul output width must equal out_features");
        const float *xp = ck.f32(0), *wp = ck.f32(1);
        REQUIRE(xp && wp);
        Weight wm;
        REQUIRE(weight_of(ck, 2, nout, hidden, &wm));
        if (hidden == 0) return ck.exec("rms_norm_matmul requires a nonzero hidden size");
        if (nout == 0) return ck.exec("rms_norm_matmul requires a nonzero out_features");
        uint64_t avail = intermediate_floats(d);
        uint64_t chunk = avail / (hidden + 1);
        if (chunk == 0) return ck.exec("device workspace is too small for this rms_norm_matmul shape");
        if (!launch || rows == 0) return SLC_OK;
        float *inv = intermediates(d), *y = inv + chunk;
        float *outp = ck.output();
        for (uint64_t r0 = 0; r0 < rows; r0 += chunk) {
            uint64_t rc = std::min(chunk, rows - r0);
            cudaError_t e = k::rms_inverse(s, xp + r0 * hidden, inv, rc, hidden, c.op->eps);
            if (e == cudaSuccess) e = k::rms_apply(s, xp + r0 * hidden, inv, wp, y, rc, hidden);
            if (e == cudaSuccess) e = matmul_rows(d, y, rc, hidden, wm, nout, outp + r0 * nout);
            if (e != cudaSuccess) return finish(ck, e);
        }
        return SLC_OK;
    }
    case SLC_OP_EXT_ADD_BIAS: {
        Dims a, b, bias, o;
        REQUIRE(ck.ivalue(0, &a) && ck.ivalue(1, &b) && ck.ivalue(2, &bias) && ck.ovalue(0, &o));
        if (!same(a, b) || !same(a, o))
            return ck.exec("add_bias operands and output must have identical shapes");
        if (a.rank < 1) return ck.exec("operator requires at least one dimension");
        uint64_t cols, rows, nb;
        REQUIRE(ck.last(a, &cols) && ck.product(a, a.rank - 1, &rows));
        REQUIRE(ck.product(bias, bias.rank, &nb));
        if (bias.rank != 1 || nb != cols) return ck.exec("add_bias bias must have shape [cols]");
        const float *ap = ck.f32(0), *bp = ck.f32(1), *zp = ck.f32(2);
        REQUIRE(ap && bp && zp);
        if (!launch) return SLC_OK;
        return finish(ck, k::add_bias(s, ap, bp, zp, ck.output(), rows, cols));
    }
    case SLC_OP_EXT_ALL_REDUCE: {
        Dims x;
        REQUIRE(ck.ivalue(0, &x));
        uint64_t n;
        REQUIRE(ck.product(x, x.rank, &n));
        float *xp = ck.f32(0);
        REQUIRE(xp);
        if (!d->comm) return ck.exec("all_reduce requires slc_comm_init");
        if (!launch) return SLC_OK;
        int rc = comm_all_reduce(d, xp, n);
        return rc == SLC_OK ? SLC_OK : ck.exec("NCCL all_reduce failed");
    }
    case SLC_OP_EXT_ALL_GATHER: {
        Dims x, o;
        REQUIRE(ck.ivalue(0, &x) && ck.ovalue(0, &o));
        if (!d->comm) return ck.exec("all_gather requires slc_comm_init");
        int rank = 0, world = 1;
        slc_comm_world(d, &rank, &world);
        uint64_t cols, rows, ocols, orows;
        REQUIRE(ck.last(x, &cols) && ck.product(x, x.rank - 1, &rows));
        REQUIRE(ck.last(o, &ocols) && ck.product(o, o.rank - 1, &orows));
        if (orows != rows || ocols != cols * (uint64_t)world)
            return ck.exec("all_gather output must be [rows, world * cols]");
        const float *xp = ck.f32(0);
        REQUIRE(xp);
        if (!launch) return SLC_OK;
        int rc = comm_all_gather(d, xp, ck.output(), rows, cols);
        return rc == SLC_OK ? SLC_OK : ck.exec("NCCL all_gather failed");
    }
    default:
        break;
    }
    int rc = slc_fail(d, SLC_ERR_UNSUPPORTED_OP, "unsupported operator");
    d->last.opcode = c.op->code;
    return rc;
}

Cmd make_cmd(const slc_op *op, const slc_buffer_ref *in, const slc_value *iv, uint64_t n_in,
             const slc_buffer_ref *out, const slc_value *ov, uint64_t n_out,
             const uint32_t *scalars, uint64_t n_scalars) {
    Cmd c{op, in, iv, n_in, out, ov, n_out, scalars, n_scalars, -1, nullptr};
    for (uint64_t i = 0; i < n_in; i++)
        if (iv[i].role == SLC_ROLE_STATE) c.state_index = (int64_t)i;
    return c;
}

}  // namespace

int slc_launch_command(slc_device *d, const slc_op *op, const slc_buffer_ref *in,
                       const slc_value *iv, uint64_t n_in, const slc_buffer_ref *out,
                       const slc_value *ov, uint64_t n_out, const uint32_t *scalars,
                       uint64_t n_scalars, const uint32_t *dyn_scalars) {
    Cmd c = make_cmd(op, in, iv, n_in, out, ov, n_out, scalars, n_scalars);
    c.dyn_scalars = dyn_scalars;
    return run_op(d, c, true);
}

namespace {
bool same_ref(const slc_buffer_ref &a, const slc_buffer_ref &b) {
    return a.buffer == b.buffer && a.offset == b.offset && a.len == b.len;
}
bool disjoint(const slc_buffer_ref &a, const slc_buffer_ref &b) {
    return a.buffer != b.buffer || a.offset + a.len <= b.offset || b.offset + b.len <= a.offset;
}
// For kernels whose CTA reads a row of every input before a barrier and
// writes the same row of every output after it: an output may take exactly
// an input's bytes (every row then meets only itself), never a shifted range.
bool row_safe(const slc_buffer_ref &out, const slc_buffer_ref &in) {
    return disjoint(out, in) || same_ref(out, in);
}
}  // namespace

int slc_launch_attention_block(slc_device *d, const BlockMember *bm, const uint32_t *dyn_past,
                               bool early_cache, bool *launched) {
    *launched = false;
    const BlockMember &sq = bm[0], &sk = bm[1], &sv = bm[2], &rq = bm[3], &rk = bm[4],
                      &at = bm[5], &mh = bm[6];
    const uint16_t want[7] = {SLC_OP_SPLIT_HEADS, SLC_OP_SPLIT_HEADS, SLC_OP_SPLIT_HEADS,
                              SLC_OP_ROPE,        SLC_OP_ROPE,        SLC_OP_CAUSAL_ATTENTION,
                              SLC_OP_MERGE_HEADS};
    for (int i = 0; i < 7; i++)
        if (bm[i].op->code != want[i]) return SLC_OK;
    // Dataflow: split outputs feed the ropes / attention, rope outputs feed
    // the attention, the attention output feeds the merge.
    if (sq.n_in != 1 || sk.n_in != 1 || sv.n_in != 1 || rq.n_in != 2 || rk.n_in != 2 ||
        at.n_in != 4 || mh.n_in != 1 || at.n_scalars != 1)
        return SLC_OK;
    if (!same_ref(rq.in[0], sq.out[0]) || !same_ref(rk.in[0], sk.out[0]) ||
        !same_ref(at.in[0], rq.out[0]) || !same_ref(at.in[1], rk.out[0]) ||
        !same_ref(at.in[2], sv.out[0]) || !same_ref(mh.in[0], at.out[0]) ||
        !same_ref(rq.in[1], rk.in[1]) || at.iv[3].role != SLC_ROLE_STATE)
        return SLC_OK;
    if (rq.op->rope_variant != rk.op->rope_variant || rq.op->theta != rk.op->theta ||
        rq.op->rope_variant > SLC_ROPE_GPTJ)
        return SLC_OK;
    const slc_value &qv = at.iv[0];  // [B, H, 1, D]
    if (qv.rank != 4 || qv.dims[2] != 1) return SLC_OK;
    const uint64_t B = qv.dims[0], H = qv.dims[1], D = qv.dims[3];
    const uint64_t Hkv = at.op->kv_heads;
    const slc_value &st = at.iv[3];  // [B, layers, 2, max_seq, Hkv, D]
    if (st.rank != 6) return SLC_OK;
    const uint64_t layers = st.dims[1], max_seq = st.dims[3];
    const uint64_t past = at.scalars[0];
    const uint64_t keys = dyn_past ? max_seq : past + 1;
    if (!k::decode_block_supported(B, H, Hkv, D, keys, kAttnTicketBytes / sizeof(unsigned)))
        return SLC_OK;
    const uint64_t need_scratch = k::decode_block_scratch_floats(B, H, Hkv, D);
    const uint64_t need_part =
        k::attention_workspace_bytes(B, H, Hkv, 1, past, D, max_seq, dyn_past != nullptr);
    if (need_scratch > intermediate_floats(d) || need_part > kernel_scratch_bytes(d))
        return SLC_OK;
    // The merged output is written together with the attention output: it
    // must not share bytes with it (the merge reads it).
    if (!disjoint(mh.out[0], at.out[0])) return SLC_OK;
    auto fp = [&](const slc_buffer_ref &r) {
        return reinterpret_cast<float *>(d->buffers[r.buffer].ptr) + r.offset;
    };
    k::DecodeBlockIo io{};
    io.q = fp(sq.in[0]);
    io.k = fp(sk.in[0]);
    io.v = fp(sv.in[0]);
    io.pos = reinterpret_cast<const uint32_t *>(d->buffers[rq.in[1].buffer].ptr) + rq.in[1].offset;
    io.qs = fp(sq.out[0]);
    io.ks = fp(sk.out[0]);
    io.vs = fp(sv.out[0]);
    io.qr = fp(rq.out[0]);
    io.kr = fp(rk.out[0]);
    io.out = fp(at.out[0]);
    io.out_merged = fp(mh.out[0]);
    io.scratch = intermediates(d);
    k::KvGeometry g{B, layers, at.op->layer, Hkv, D, max_seq};
    k::AttnScratch scr{kernel_scratch(d), kernel_scratch_bytes(d), ws_attn_tickets(d),
                       kAttnTicketBytes / sizeof(unsigned), d->device_flag};
    cudaError_t e = k::decode_attention_block(d->stream, io, fp(at.in[3]), g, H, past,
                                              at.op->scale, rq.op->theta,
                                              rq.op->rope_variant == SLC_ROPE_GPTJ, scr, dyn_past,
                                              early_cache);
    if (e != cudaSuccess) return slc_fail(d, SLC_ERR_EXECUTION, "CUDA kernel launch failed");
    *launched = true;
    return SLC_OK;
}

int slc_launch_add_rmsnorm(slc_device *d, const BlockMember *add, const BlockMember *rms,
                           bool *launched) {
    *launched = false;
    if (add->op->code != SLC_OP_ADD || rms->op->code != SLC_OP_RMS_NORM || add->n_in != 2 ||
        rms->n_in != 2 || !same_ref(rms->in[0], add->out[0]))
        return SLC_OK;
    const slc_value &xv = rms->iv[0];
    if (xv.rank < 1 || xv.dtype != SLC_F32) return SLC_OK;
    const uint64_t hidden = xv.dims[xv.rank - 1];
    uint64_t rows = 1;
    for (uint32_t r = 0; r + 1 < xv.rank; r++) rows *= xv.dims[r];
    // Rows are read before the barrier and written after it by the same
    // CTA; across rows an output may reuse an input's bytes only exactly.
    if (rows != 1 && (!row_safe(rms->out[0], add->in[0]) || !row_safe(rms->out[0], add->in[1]) ||
                      !row_safe(add->out[0], add->in[0]) || !row_safe(add->out[0], add->in[1]) ||
                      !row_safe(rms->out[0], add->out[0])))
        return SLC_OK;
    auto fp = [&](const slc_buffer_ref &r) {
        return reinterpret_cast<float *>(d->buffers[r.buffer].ptr) + r.offset;
    };
    const float *a = fp(add->in[0]), *b = fp(add->in[1]), *w = fp(rms->in[1]);
    float *sum = fp(add->out[0]), *out = fp(rms->out[0]);
    if (!k::add_rms_norm_supported(a, b, sum, w, out, rows, hidden)) return SLC_OK;
    if (k::add_rms_norm(d->stream, a, b, sum, w, out, rows, hidden, rms->op->eps) != cudaSuccess)
        return slc_fail(d, SLC_ERR_EXECUTION, "CUDA kernel launch failed");
    *launched = true;
    return SLC_OK;
}

int slc_launch_allreduce_add_rmsnorm(slc_device *d, const BlockMember *ar, const BlockMember *add,
                                     const BlockMember *rms, bool *launched) {
    *launched = false;
    if (ar->op->code != SLC_OP_EXT_ALL_REDUCE || ar->n_in != 1 || add->op->code != SLC_OP_ADD ||
        rms->op->code != SLC_OP_RMS_NORM || add->n_in != 2 || rms->n_in != 2 ||
        !same_ref(rms->in[0], add->out[0]))
        return SLC_OK;
    // The all-reduced value is one of the Add's operands; the other is the
    // residual.
    int pi = -1;
    if (same_ref(add->in[1], ar->in[0]))
        pi = 1;
    else if (same_ref(add->in[0], ar->in[0]))
        pi = 0;
    if (pi < 0) return SLC_OK;
    const slc_value &xv = rms->iv[0];
    if (xv.rank < 1 || xv.dtype != SLC_F32 || ar->iv[0].dtype != SLC_F32) return SLC_OK;
    const uint64_t hidden = xv.dims[xv.rank - 1];
    uint64_t rows = 1;
    for (uint32_t r = 0; r + 1 < xv.rank; r++) rows *= xv.dims[r];
    if (ar->in[0].len != rows * hidden || add->in[1 - pi].len != rows * hidden) return SLC_OK;
    // Rows are read before the row's barrier and written after it; across
    // rows the outputs may only reuse the inputs' bytes when there is a
    // single row.
    if (rows != 1 &&
        (!disjoint(rms->out[0], add->in[0]) || !disjoint(rms->out[0], add->in[1]) ||
         !disjoint(add->out[0], add->in[0]) || !disjoint(add->out[0], add->in[1]) ||
         !disjoint(rms->out[0], add->out[0])))
        return SLC_OK;
    k::PeerReduceArgs a{};
    if (!comm_peer_args(d, &a)) return SLC_OK;
    auto fp = [&](const slc_buffer_ref &r) {
        return reinterpret_cast<float *>(d->buffers[r.buffer].ptr) + r.offset;
    };
    a.partial = fp(ar->in[0]);
    a.residual = fp(add->in[1 - pi]);
    a.sum_out = fp(add->out[0]);
    a.out = fp(rms->out[0]);
    a.weight = fp(rms->in[1]);
    a.rows = rows;
    a.hidden = hidden;
    a.eps = rms->op->eps;
    a.err = d->device_flag;
    if (!k::allreduce_add_rms_supported(a)) return SLC_OK;
    if (k::allreduce_add_rms(d->stream, a) != cudaSuccess)
        return slc_fail(d, SLC_ERR_EXECUTION, "CUDA kernel launch failed");
    *launched = true;
    return SLC_OK;
}

int slc_launch_matmul_group(slc_device *d, const MatmulMember *mm, int n, bool *launched) {
    *launched = false;
    if (n < 2 || n > 4) return SLC_OK;
    k::QuantSeg segs[4];
    const float *x = nullptr;
    uint64_t m = 0, kk = 0;
    for (int i = 0; i < n; i++) {
        const slc_value &xv = mm[i].iv[0], &wv = mm[i].iv[1], &ov = mm[i].ov[0];
        if (wv.encoding != SLC_ENC_GROUPWISE || xv.rank < 2 || wv.rank != 2 || ov.rank < 2)
            return SLC_OK;
        uint64_t rows = 1;
        for (uint32_t r = 0; r + 1 < xv.rank; r++) rows *= xv.dims[r];
        const uint64_t k_i = xv.dims[xv.rank - 1];
        const float *xp =
            reinterpret_cast<const float *>(d->buffers[mm[i].in[0].buffer].ptr) + mm[i].in[0].offset;
        if (i == 0) {
            x = xp;
            m = rows;
            kk = k_i;
        } else if (xp != x || rows != m || k_i != kk) {
            return SLC_OK;
        }
        if (slc_quant_view(d, mm[i].in[1].buffer, mm[i].in[1].offset, wv.dims[0], kk,
                           wv.quant_format, wv.group_size, &segs[i].w) != SLC_OK) {
            d->last = slc_error{};
            return SLC_OK;
        }
        segs[i].out =
            reinterpret_cast<float *>(d->buffers[mm[i].out[0].buffer].ptr) + mm[i].out[0].offset;
    }
    if (m == 0 || m > 32 || !k::qgemv_tma_x_aligned(x) || !k::qgemv_tma_group_supported(segs, n, m) ||
        k::qgemv_tma_group_workspace_bytes(segs, n, m) > gemv_workspace_bytes(d))
        return SLC_OK;
    cudaError_t e = k::qgemv_tma_group(d->stream, x, nullptr, m, segs, n, gemv_workspace(d),
                                       d->device_flag);
    if (e != cudaSuccess) return slc_fail(d, SLC_ERR_EXECUTION, "CUDA kernel launch failed");
    *launched = true;
    return SLC_OK;
}

int slc_resolve_and_run(slc_device *d, const slc_op *op, const slc_buffer_ref *in,
                        const slc_value *iv, uint64_t n_in, const slc_buffer_ref *out,
                        const slc_value *ov, uint64_t n_out, const uint32_t *scalars,
                        uint64_t n_scalars) {
    Cmd c = make_cmd(op, in, iv, n_in, out, ov, n_out, scalars, n_scalars);
    if (d->capture) {
        int rc = run_op(d, c, false);
        if (rc != SLC_OK) return rc;
        if (capture_record(d, op, in, iv, n_in, out, ov, n_out, scalars, n_scalars)) return SLC_OK;
    }
    cudaSetDevice(d->ordinal);
    return run_op(d, c, true);
}
