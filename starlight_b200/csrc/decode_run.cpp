// Capture-time fusion of whole decode layers into one persistent launch
// (kernels/decode_layers.cu).
//
// A recorded segment that contains, at batch 1 and one token, consecutive
// llama-dense decoder layers -- per layer the sixteen commands
//   RmsNorm, MatMulNT q k v, SplitHeads x3, Rope q k, CausalAttention,
//   MergeHeads, MatMulNT o, Add, RmsNorm, SwiGlu, Add
// (the lowering of docs/ARCH-0006 sections 4-5; operator semantics of
// crates/backends/backend-cpu/src/device.rs:773-1227) with GroupwiseQuantized
// weights -- runs as one cooperative launch that leaves every output buffer
// and the KV state as the commands would. Under tensor parallelism a layer
// is eighteen commands (an in-place AllReduce after MatMulNT o and after
// SwiGlu); the matcher checks their placement and matches the other
// sixteen, and the kernel performs the all-reduces over peer memory (only
// when every rank agreed on it at slc_comm_init).
//
// The kernel reads the command buffers only at its start (the first layer's
// input, weights, norm weights, positions, KV state) and computes from
// private copies; it writes every command output in command order. That is
// equivalent to running the commands one by one when
//   (a) no command output overlaps the weights, norm weights, positions or
//       KV state it reads,
//   (b) no output of a command up to the first layer's residual Add overlaps
//       the first layer's input (read again by that Add), and
//   (c) every value produced inside the run is not overwritten by another
//       command before its last reader in the run.
// These are checked here; a run that fails any check is left to the other
// fusions and the per-command kernels.
//
// Program images (tensor maps + layer table) live in device slots owned by
// this state: slot 0 is rewritten by every eager run (host past_len values),
// slots 1.. hold the images of captured graphs (device past_len pointers),
// uploaded before the capture begins and kept until the graphs are dropped.
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include <new>

#include <string>
#include <unordered_map>
#include <vector>

#include "device_internal.h"
#include "kernels/kernels.h"

namespace {

constexpr int kLayerCmds = 16;
constexpr int kImageSlots = 8;
constexpr size_t kImageSlotBytes = 256 * 1024;

const uint16_t kPattern[kLayerCmds] = {
    SLC_OP_RMS_NORM,    SLC_OP_MATMUL_NT,       SLC_OP_MATMUL_NT,    SLC_OP_MATMUL_NT,
    SLC_OP_SPLIT_HEADS, SLC_OP_SPLIT_HEADS,     SLC_OP_SPLIT_HEADS,  SLC_OP_ROPE,
    SLC_OP_ROPE,        SLC_OP_CAUSAL_ATTENTION, SLC_OP_MERGE_HEADS, SLC_OP_MATMUL_NT,
    SLC_OP_ADD,         SLC_OP_RMS_NORM,        SLC_OP_SWIGLU,       SLC_OP_ADD};
const uint64_t kInputs[kLayerCmds] = {2, 2, 2, 2, 1, 1, 1, 2, 2, 4, 1, 2, 2, 2, 4, 2};

uint64_t fnv1a(const unsigned char *p, size_t n) {
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < n; i++) h = (h ^ p[i]) * 1099511628211ull;
    return h;
}

uint64_t elements(const slc_value &v) {
    uint64_t n = 1;
    for (uint32_t i = 0; i < v.rank; i++) n *= v.dims[i];
    return n;
}

bool same_ref(const slc_buffer_ref &a, const slc_buffer_ref &b) {
    return a.buffer == b.buffer && a.offset == b.offset && a.len == b.len;
}

bool overlaps(const slc_buffer_ref &a, const slc_buffer_ref &b) {
    return a.buffer == b.buffer && a.offset < b.offset + b.len && b.offset < a.offset + a.len;
}

float *fptr(slc_device *d, const slc_buffer_ref &r) {
    return reinterpret_cast<float *>(d->buffers[r.buffer].ptr) + r.offset;
}

bool f32_count(const slc_value &v, uint64_t n) { return v.dtype == SLC_F32 && elements(v) == n; }

// Everything the matcher learns about a run.
struct Match {
    std::vector<slc::k::DlLayerIo> io;
    slc::k::DlRun run{};
    slc_buffer_ref x0{}, pos{}, kv{};
    std::vector<slc_buffer_ref> reads;        // weights, norm weights (element refs)
    std::vector<uint32_t> scale_buffers;      // bound scale buffers (whole buffers)
};

bool quant_weight(slc_device *d, const slc_buffer_ref &ref, const slc_value &v, uint64_t rows,
                  uint64_t k, slc::k::QuantWeight *w) {
    if (v.encoding != SLC_ENC_GROUPWISE || v.rank != 2 || v.dims[0] != rows || v.dims[1] != k)
        return false;
    if (slc_quant_view(d, ref.buffer, ref.offset, rows, k, v.quant_format, v.group_size, w) !=
        SLC_OK) {
        d->last = slc_error{};
        return false;
    }
    return true;
}

// One layer at c[0..16) whose input is `x`; the shapes are learned from the
// first layer and checked on the others.
bool match_layer(slc_device *d, const BlockMember *c, const slc_buffer_ref &x, bool first,
                 Match *m) {
    for (int i = 0; i < kLayerCmds; i++)
        if (c[i].op->code != kPattern[i] || c[i].n_in != kInputs[i]) return false;
    for (int i = 0; i < kLayerCmds; i++)
        if (c[i].n_scalars != (i == 9 ? 1u : 0u)) return false;
    const BlockMember &rms1 = c[0], &mq = c[1], &mk = c[2], &mv = c[3], &sq = c[4], &sk = c[5],
                      &sv = c[6], &rq = c[7], &rk = c[8], &at = c[9], &mh = c[10], &mo = c[11],
                      &add1 = c[12], &rms2 = c[13], &sw = c[14], &add2 = c[15];
    // Dataflow.
    if (!same_ref(rms1.in[0], x) || !same_ref(mq.in[0], rms1.out[0]) ||
        !same_ref(mk.in[0], rms1.out[0]) || !same_ref(mv.in[0], rms1.out[0]) ||
        !same_ref(sq.in[0], mq.out[0]) || !same_ref(sk.in[0], mk.out[0]) ||
        !same_ref(sv.in[0], mv.out[0]) || !same_ref(rq.in[0], sq.out[0]) ||
        !same_ref(rk.in[0], sk.out[0]) || !same_ref(rq.in[1], rk.in[1]) ||
        !same_ref(at.in[0], rq.out[0]) || !same_ref(at.in[1], rk.out[0]) ||
        !same_ref(at.in[2], sv.out[0]) || !same_ref(mh.in[0], at.out[0]) ||
        !same_ref(mo.in[0], mh.out[0]) || !same_ref(rms2.in[0], add1.out[0]) ||
        !same_ref(sw.in[0], rms2.out[0]))
        return false;
    if (!((same_ref(add1.in[0], x) && same_ref(add1.in[1], mo.out[0])) ||
          (same_ref(add1.in[1], x) && same_ref(add1.in[0], mo.out[0]))))
        return false;
    if (!((same_ref(add2.in[0], add1.out[0]) && same_ref(add2.in[1], sw.out[0])) ||
          (same_ref(add2.in[1], add1.out[0]) && same_ref(add2.in[0], sw.out[0]))))
        return false;
    // Shapes: batch 1, one token.
    const slc_value &qv = at.iv[0];  // [1, Hq, 1, D]
    const slc_value &st = at.iv[3];  // [1, layers, 2, max_seq, Hkv, D]
    if (qv.rank != 4 || qv.dims[0] != 1 || qv.dims[2] != 1 || st.rank != 6 || st.dims[0] != 1 ||
        st.role != SLC_ROLE_STATE || st.dtype != SLC_F32)
        return false;
    const uint64_t Hq = qv.dims[1], D = qv.dims[3], Hkv = st.dims[4];
    if (at.op->heads != Hq || at.op->kv_heads != Hkv || at.op->head_dim != D || st.dims[5] != D ||
        at.op->layer >= st.dims[1])
        return false;
    const slc_value &xv = rms1.iv[0];
    if (xv.rank < 1 || xv.dtype != SLC_F32) return false;
    const uint64_t H = xv.dims[xv.rank - 1];
    if (elements(xv) != H) return false;  // one row
    const slc_value &gv = sw.iv[1];
    if (gv.rank != 2) return false;
    const uint64_t I = gv.dims[0];
    slc::k::DlRun &r = m->run;
    if (first) {
        r.hidden = (uint32_t)H;
        r.heads = (uint32_t)Hq;
        r.kv_heads = (uint32_t)Hkv;
        r.head_dim = (uint32_t)D;
        r.inter = (uint32_t)I;
        r.format = (int)mq.iv[1].quant_format;
        r.group = mq.iv[1].group_size;
        r.gptj = rq.op->rope_variant == SLC_ROPE_GPTJ;
        r.theta = rq.op->theta;
        r.cache_layers = st.dims[1];
        r.max_seq = st.dims[3];
        m->kv = at.in[3];
        m->pos = rq.in[1];
        m->x0 = x;
    } else if (H != r.hidden || Hq != r.heads || Hkv != r.kv_heads || D != r.head_dim ||
               I != r.inter || (int)mq.iv[1].quant_format != r.format ||
               mq.iv[1].group_size != r.group || !same_ref(at.in[3], m->kv) ||
               !same_ref(rq.in[1], m->pos) || (rq.op->rope_variant == SLC_ROPE_GPTJ) != (r.gptj != 0) ||
               rq.op->theta != r.theta) {
        return false;
    }
    if (rq.op->rope_variant > SLC_ROPE_GPTJ || rk.op->rope_variant != rq.op->rope_variant ||
        rk.op->theta != rq.op->theta || rq.iv[1].dtype != SLC_U32 || elements(rq.iv[1]) != 1)
        return false;
    if (sq.op->heads != Hq || sq.op->head_dim != D || sk.op->heads != Hkv || sk.op->head_dim != D ||
        sv.op->heads != Hkv || sv.op->head_dim != D || mh.op->heads != Hq || mh.op->head_dim != D)
        return false;
    // Values.
    const uint64_t QD = Hq * D, KD = Hkv * D;
    if (!f32_count(rms1.iv[1], H) || !f32_count(rms2.iv[1], H) || !f32_count(rms1.ov[0], H) ||
        !f32_count(mq.ov[0], QD) || !f32_count(mk.ov[0], KD) || !f32_count(mv.ov[0], KD) ||
        !f32_count(sq.ov[0], QD) || !f32_count(sk.ov[0], KD) || !f32_count(sv.ov[0], KD) ||
        !f32_count(rq.ov[0], QD) || !f32_count(rk.ov[0], KD) || !f32_count(at.ov[0], QD) ||
        !f32_count(mh.ov[0], QD) || !f32_count(mo.ov[0], H) || !f32_count(add1.ov[0], H) ||
        !f32_count(rms2.ov[0], H) || !f32_count(sw.ov[0], H) || !f32_count(add2.ov[0], H))
        return false;
    slc::k::DlLayerIo io{};
    if (!quant_weight(d, mq.in[1], mq.iv[1], QD, H, &io.w[0]) ||
        !quant_weight(d, mk.in[1], mk.iv[1], KD, H, &io.w[1]) ||
        !quant_weight(d, mv.in[1], mv.iv[1], KD, H, &io.w[2]) ||
        !quant_weight(d, mo.in[1], mo.iv[1], H, QD, &io.w[3]) ||
        !quant_weight(d, sw.in[1], sw.iv[1], I, H, &io.w[4]) ||
        !quant_weight(d, sw.in[2], sw.iv[2], I, H, &io.w[5]) ||
        !quant_weight(d, sw.in[3], sw.iv[3], H, I, &io.w[6]))
        return false;
    for (int w = 0; w < 7; w++)
        if ((int)io.w[w].format != r.format || io.w[w].group != r.group) return false;
    io.wn1 = fptr(d, rms1.in[1]);
    io.wn2 = fptr(d, rms2.in[1]);
    io.eps1 = rms1.op->eps;
    io.eps2 = rms2.op->eps;
    io.scale = at.op->scale;
    io.cache_layer = at.op->layer;
    io.past = at.scalars[0];
    for (int i = 0; i < kLayerCmds; i++) io.cmd[i] = fptr(d, c[i].out[0]);
    m->io.push_back(io);
    const BlockMember *wcmds[5] = {&mq, &mk, &mv, &mo, &sw};
    for (const BlockMember *wc : wcmds)
        for (uint64_t q = 1; q < wc->n_in; q++) {
            m->reads.push_back(wc->in[q]);
            auto it = d->quant.find(wc->in[q].buffer);
            if (it != d->quant.end()) m->scale_buffers.push_back(it->second.scales);
        }
    m->reads.push_back(rms1.in[1]);
    m->reads.push_back(rms2.in[1]);
    return true;
}

// Sequential equivalence of the run c[0 .. 16 * layers): conditions (a)-(c)
// of the file comment.
bool run_is_sequential(const BlockMember *c, size_t layers, const Match &m) {
    const size_t n = layers * kLayerCmds;
    auto out_hits = [&](size_t from, size_t to, const slc_buffer_ref &v) {  // outputs of (from, to)
        for (size_t i = from + 1; i < to; i++)
            if (overlaps(c[i].out[0], v)) return true;
        return false;
    };
    for (size_t i = 0; i < n; i++) {
        const slc_buffer_ref &o = c[i].out[0];
        if (overlaps(o, m.pos) || overlaps(o, m.kv)) return false;
        for (const slc_buffer_ref &r : m.reads)
            if (overlaps(o, r)) return false;
        for (uint32_t b : m.scale_buffers)
            if (o.buffer == b) return false;
    }
    // The first layer's input: read by commands 0 and 12.
    for (size_t i = 0; i <= 12; i++)
        if (overlaps(c[i].out[0], m.x0)) return false;
    // Values produced in the run, up to their last reader in the run.
    static const int kEdges[][2] = {{0, 3}, {1, 4}, {2, 5}, {3, 6}, {4, 7}, {5, 8}, {6, 9},
                                    {7, 9}, {8, 9}, {9, 10}, {10, 11}, {11, 12}, {12, 15},
                                    {13, 14}, {14, 15}};
    for (size_t l = 0; l < layers; l++) {
        const size_t b = l * kLayerCmds;
        for (const auto &e : kEdges)
            if (out_hits(b + e[0], b + e[1], c[b + e[0]].out[0])) return false;
        // This layer's output, read by the next layer's commands 0 and 12.
        if (l + 1 < layers && out_hits(b + 15, b + kLayerCmds + 12, c[b + 15].out[0])) return false;
    }
    return true;
}

// Tensor parallelism: a layer is 18 commands, an in-place AllReduce of the o
// projection's output after command 11 and of the SwiGlu output after
// command 15 (the lowering's row-parallel projections). The layers at
// c[0..n) with both all-reduces where they belong, copied without them (the
// persistent kernel performs them), into `out`.
constexpr int kTpLayerCmds = kLayerCmds + 2;

bool all_reduce_of(const BlockMember &ar, const BlockMember &producer) {
    return ar.op->code == SLC_OP_EXT_ALL_REDUCE && ar.n_in == 1 && ar.n_scalars == 0 &&
           same_ref(ar.in[0], producer.out[0]) && ar.iv[0].dtype == SLC_F32;
}

void strip_all_reduces(const BlockMember *c, size_t n, std::vector<BlockMember> *out) {
    out->clear();
    for (size_t b = 0; b + kTpLayerCmds <= n && out->size() < 128 * (size_t)kLayerCmds;
         b += kTpLayerCmds) {
        const BlockMember *l = c + b;
        if (l[11].op->code != SLC_OP_MATMUL_NT || l[15].op->code != SLC_OP_SWIGLU ||
            !all_reduce_of(l[12], l[11]) || !all_reduce_of(l[16], l[15]))
            break;
        for (int i = 0; i < kTpLayerCmds; i++)
            if (i != 12 && i != 16) out->push_back(l[i]);
    }
}

// Matches as many layers as possible at c[0..n).
size_t match_run(slc_device *d, const BlockMember *c, size_t n, Match *m) {
    size_t layers = 0;
    if (n < kLayerCmds || c[0].op->code != SLC_OP_RMS_NORM) return 0;
    slc_buffer_ref x = c[0].in[0];
    while ((layers + 1) * kLayerCmds <= n) {
        const BlockMember *lc = c + layers * kLayerCmds;
        if (!match_layer(d, lc, x, layers == 0, m)) break;
        x = lc[15].out[0];
        layers++;
        if (layers == 128) break;
    }
    if (layers == 0) return 0;
    // Shrink to the longest prefix that is sequentially equivalent.
    while (layers > 0 && !run_is_sequential(c, layers, *m)) layers--;
    m->io.resize(layers);
    return layers;
}

}  // namespace

struct DecodeRunState {
    unsigned *sync = nullptr;     // kDecodeSyncWords, zero between launches
    char *images = nullptr;       // kImageSlots x kImageSlotBytes
    unsigned char *host_image = nullptr;  // pinned staging
    std::unordered_map<uint64_t, int> slot_of;  // image hash -> slot (graph images)
    int next_slot = 1;
    bool disabled = false;
    uint64_t launched = 0, refused = 0;  // launches made / refused by the runtime
};

int decode_run_create(slc_device *d) {
    if (d->decode) return SLC_OK;
    DecodeRunState *s = new (std::nothrow) DecodeRunState();
    if (!s) return slc_fail(d, SLC_ERR_OUT_OF_MEMORY, "decode fusion state allocation failed");
    if (cudaMalloc(&s->sync, slc::k::kDecodeSyncWords * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(s->sync, 0, slc::k::kDecodeSyncWords * sizeof(unsigned)) != cudaSuccess ||
        cudaMalloc(&s->images, kImageSlots * kImageSlotBytes) != cudaSuccess ||
        cudaMallocHost(&s->host_image, kImageSlotBytes) != cudaSuccess) {
        cudaGetLastError();
        if (s->sync) cudaFree(s->sync);
        if (s->images) cudaFree(s->images);
        if (s->host_image) cudaFreeHost(s->host_image);
        delete s;
        return slc_fail(d, SLC_ERR_OUT_OF_MEMORY, "decode fusion state allocation failed");
    }
    // SLC_DECODE_FUSION=0 keeps the per-layer launches (comparison runs).
    const char *env = getenv("SLC_DECODE_FUSION");
    s->disabled = env && env[0] == '0';
    d->decode = s;
    return SLC_OK;
}

void decode_run_release(slc_device *d) {
    DecodeRunState *s = d->decode;
    if (!s) return;
    cudaSetDevice(d->ordinal);
    cudaStreamSynchronize(d->stream);
    cudaFree(s->sync);
    cudaFree(s->images);
    cudaFreeHost(s->host_image);
    delete s;
    d->decode = nullptr;
}

int decode_run_stats(const slc_device *d, slc_decode_fusion_info *out) {
    *out = slc_decode_fusion_info{};
    out->last_ms = -1.f;
    const DecodeRunState *s = d->decode;
    if (!s) return SLC_OK;
    out->launched = s->launched;
    out->refused = s->refused;
    // The kernel's own global-timer stamps of its latest launch (start, end).
    unsigned long long t[2] = {0, 0};
    cudaSetDevice(d->ordinal);
    if (s->launched > 0 && cudaStreamSynchronize(d->stream) == cudaSuccess &&
        cudaMemcpy(t, s->sync + slc::k::kDecodeStampWord, sizeof(t), cudaMemcpyDeviceToHost) ==
            cudaSuccess &&
        t[1] > t[0])
        out->last_ms = (float)((double)(t[1] - t[0]) / 1e6);
    cudaGetLastError();
    return SLC_OK;
}

void decode_run_invalidate(slc_device *d) {
    if (!d->decode) return;
    d->decode->slot_of.clear();
    d->decode->next_slot = 1;
}

// Tensor parallelism of the device (world 1: none); false when the device
// is tensor-parallel but the persistent kernel's exchange is off.
bool run_peers(slc_device *d, slc::k::DlPeers *tp) {
    *tp = slc::k::DlPeers{};
    int rank = 0, world = 1;
    if (d->comm) slc_comm_world(d, &rank, &world);
    if (world <= 1) return true;
    return comm_decode_peers(d, tp);
}

size_t decode_run_match(slc_device *d, const BlockMember *cmds, size_t n) {
    if (!d->decode || (d->decode->disabled && !d->comm)) return 0;
    slc::k::DlPeers tp;
    if (!run_peers(d, &tp)) return 0;
    // Under tensor parallelism every rank decided alike at slc_comm_init.
    if (tp.world == 1 && d->decode->disabled) return 0;
    std::vector<BlockMember> stripped;
    if (tp.world > 1) {
        strip_all_reduces(cmds, n, &stripped);
        cmds = stripped.data();
        n = stripped.size();
    }
    Match m;
    const size_t layers = match_run(d, cmds, n, &m);
    if (layers == 0) return 0;
    m.run.tp = tp;
    m.run.layers = (uint32_t)layers;
    m.run.layer = m.io.data();
    m.run.x0 = fptr(d, m.x0);
    m.run.pos = reinterpret_cast<const uint32_t *>(d->buffers[m.pos.buffer].ptr) + m.pos.offset;
    m.run.cache = fptr(d, m.kv);
    if (!slc::k::decode_layers_supported(m.run) ||
        slc::k::decode_layers_scratch_bytes(m.run) > ws_scratch_bytes(d) ||
        slc::k::decode_layers_image_bytes((int)layers) > kImageSlotBytes)
        return 0;
    return layers * (tp.world > 1 ? kTpLayerCmds : kLayerCmds);
}

int decode_run_launch(slc_device *d, const BlockMember *cmds, size_t n, const uint32_t *const *dyn,
                      bool prepare_only, bool *launched) {
    *launched = false;
    DecodeRunState *s = d->decode;
    if (!s) return SLC_OK;
    slc::k::DlPeers tp;
    if (!run_peers(d, &tp)) return SLC_OK;
    if (tp.world == 1 && s->disabled) return SLC_OK;
    const size_t stride = tp.world > 1 ? kTpLayerCmds : kLayerCmds;
    const size_t n_orig = n;
    std::vector<BlockMember> stripped;
    if (tp.world > 1) {
        strip_all_reduces(cmds, n, &stripped);
        cmds = stripped.data();
        n = stripped.size();
    }
    Match m;
    const size_t layers = match_run(d, cmds, n, &m);
    if (layers == 0 || layers * stride != n_orig) return SLC_OK;
    m.run.tp = tp;
    m.run.layers = (uint32_t)layers;
    m.run.layer = m.io.data();
    m.run.x0 = fptr(d, m.x0);
    m.run.pos = reinterpret_cast<const uint32_t *>(d->buffers[m.pos.buffer].ptr) + m.pos.offset;
    m.run.cache = fptr(d, m.kv);
    const bool graph = dyn != nullptr;
    for (size_t l = 0; l < layers; l++) {
        m.io[l].d_past = graph ? dyn[l * stride + 9] : nullptr;
        if (graph && !m.io[l].d_past) return SLC_OK;
    }
    if (!slc::k::decode_layers_supported(m.run)) return SLC_OK;
    const size_t bytes = slc::k::decode_layers_image_bytes((int)layers);
    if (bytes > kImageSlotBytes || slc::k::decode_layers_scratch_bytes(m.run) > ws_scratch_bytes(d))
        return SLC_OK;
    // Eager runs use slot 0 (rewritten each time); graph images get a slot
    // of their own before the capture begins (prepare_only) and are found
    // by content during it.
    int slot = 0;
    if (graph) {
        memset(s->host_image, 0, bytes);
        // The image's content depends on its own address only through the
        // tensor maps' neighbours; build it once for slot lookup.
        if (!slc::k::decode_layers_image(m.run, s->host_image, bytes, nullptr)) return SLC_OK;
        const uint64_t h = fnv1a(s->host_image, bytes);
        auto it = s->slot_of.find(h);
        if (it != s->slot_of.end()) {
            slot = it->second;
        } else {
            if (!prepare_only) return SLC_OK;  // inside a capture: no uploads
            if (s->next_slot >= kImageSlots) return SLC_OK;
            slot = s->next_slot++;
            if (cudaMemcpy(s->images + (size_t)slot * kImageSlotBytes, s->host_image, bytes,
                           cudaMemcpyHostToDevice) != cudaSuccess) {
                cudaGetLastError();
                return SLC_OK;
            }
            s->slot_of.emplace(h, slot);
        }
        if (prepare_only) return SLC_OK;
    } else {
        if (prepare_only) return SLC_OK;
        // The previous eager launch may still read slot 0.
        if (cudaStreamSynchronize(d->stream) != cudaSuccess) {
            cudaGetLastError();
            return slc_fail(d, SLC_ERR_EXECUTION, "stream synchronization failed");
        }
        memset(s->host_image, 0, bytes);
        if (!slc::k::decode_layers_image(m.run, s->host_image, bytes, s->images) ||
            cudaMemcpy(s->images, s->host_image, bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
            cudaGetLastError();
            return SLC_OK;
        }
    }
    cudaError_t e = slc::k::decode_layers(d->stream, m.run, s->images + (size_t)slot * kImageSlotBytes,
                                          ws_scratch(d), ws_scratch_bytes(d), s->sync,
                                          d->device_flag);
    if (e == cudaErrorInvalidValue || e == cudaErrorInvalidConfiguration ||
        e == cudaErrorCooperativeLaunchTooLarge) {
        // Refused before anything was enqueued (a tensor map the driver does
        // not accept, or one CTA per SM does not fit): the commands run
        // through the other kernels instead -- except under tensor
        // parallelism, where the other ranks' kernels expect this rank's
        // exchanges and the per-command path would enter collectives they
        // never join: the step fails here instead (their exchange waits end
        // with a timeout error).
        cudaGetLastError();
        s->refused++;
        if (tp.world > 1)
            return slc_fail(d, SLC_ERR_EXECUTION,
                            "persistent decode kernel refused under tensor parallelism");
        return SLC_OK;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return slc_fail(d, SLC_ERR_EXECUTION, "persistent decode kernel launch failed");
    }
    s->launched++;
    *launched = true;
    return SLC_OK;
}
