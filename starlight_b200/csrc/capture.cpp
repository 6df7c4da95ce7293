// Command capture and CUDA-graph replay (slc_set_capture).
//
// With capture on, slc_dispatch validates a command exactly as before (every
// error is still reported by the dispatch call itself) and records it instead
// of launching it. The recorded segment runs at the next point where its
// effects could be observed (synchronize, upload, download, flush, any other
// call that touches the stream or device data):
//
//  * the segment's key is everything that determines its kernels: operators
//    and their attributes, buffer references, values, and the scalars of
//    operators that cannot take them from device memory. The scalars of
//    LastToken, KvAppend and CausalAttention (seq_len, past_len) are not part
//    of the key: their kernels read them from a device table, written from
//    pinned host memory before each replay;
//  * the first time a key is seen the segment runs eagerly (launch by
//    launch); the second time it is captured into a CUDA graph (kernels read
//    the table) and instantiated; from then on it is replayed with one graph
//    launch. Up to kMaxGraphs graphs are kept (least recently used evicted).
//    A segment that fails to capture runs eagerly and is not tried again.
//
// Results are those of eager execution: the same kernels run on the same
// buffers in the same order. Graphs hold device pointers, so the cache is
// dropped whenever a buffer is released or a quantization binding changes.
#include <cuda_runtime.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <list>
#include <unordered_map>
#include <vector>

#include "device_internal.h"

namespace {

constexpr size_t kMaxGraphs = 8;
constexpr uint32_t kTableSlots = 1 << 14;  // device scalars per segment
constexpr size_t kMaxPorts = 8;

struct Rec {
    slc_op op;
    uint32_t n_in, n_out, n_scalars;
    slc_buffer_ref in[kMaxPorts], out[kMaxPorts];
    slc_value iv[kMaxPorts], ov[kMaxPorts];
    uint32_t scalars[kMaxPorts];
    int32_t slot;  // first device-table slot of its scalars, or -1
};

struct Graph {
    cudaGraphExec_t exec = nullptr;
    std::vector<unsigned char> key;
    uint64_t launches = 0;  // kernels per replay
    uint64_t id = 0;        // unique in the process (step memos name graphs by it)
};

std::atomic<uint64_t> g_next_graph_id{1};

bool dynamic_scalars(uint16_t code) {
    return code == SLC_OP_LAST_TOKEN || code == SLC_OP_KV_APPEND ||
           code == SLC_OP_CAUSAL_ATTENTION;
}

// Hash of a command-list key (a decode step of an 8B model is ~200 KB of
// key, rebuilt and hashed every step). Four independent lanes over 8-byte
// words (multiply, then fold the high bits down) keep it at memory speed; a
// byte-serial FNV-1a took ~0.25 ms a step. A hit is confirmed by comparing
// the whole key, so the hash only has to spread keys, not be collision-free.
uint64_t key_hash(const unsigned char *p, size_t n) {
    constexpr uint64_t kMul = 0x9e3779b97f4a7c15ull;
    uint64_t h[4] = {0x243f6a8885a308d3ull, 0x13198a2e03707344ull, 0xa4093822299f31d0ull,
                     0x082efa98ec4e6c89ull};
    size_t i = 0;
    for (; i + 32 <= n; i += 32)
        for (int l = 0; l < 4; l++) {
            uint64_t w;
            memcpy(&w, p + i + 8 * l, 8);
            h[l] = (h[l] ^ w) * kMul;
            h[l] ^= h[l] >> 31;
        }
    uint64_t r = n * kMul;
    for (; i < n; i++) r = (r ^ p[i]) * 1099511628211ull;
    for (int l = 0; l < 4; l++) {
        r = (r ^ h[l]) * kMul;
        r ^= r >> 29;
    }
    return r;
}

}  // namespace

struct CaptureState {
    std::vector<Rec> pending;
    std::vector<unsigned char> key;
    uint32_t table_used = 0;
    uint32_t *h_table = nullptr;  // pinned
    uint32_t *d_table = nullptr;
    cudaEvent_t table_done = nullptr;
    bool table_pending = false;
    std::unordered_map<uint64_t, std::list<Graph>::iterator> by_hash;
    std::list<Graph> graphs;  // front = most recently used
    std::unordered_map<uint64_t, int> seen;  // key hash -> times run (-1: never capture)
    slc_capture_info stats{};
};

static void append_key(CaptureState *cs, const void *p, size_t n) {
    const unsigned char *b = static_cast<const unsigned char *>(p);
    cs->key.insert(cs->key.end(), b, b + n);
}

static void drop_graphs(CaptureState *cs) {
    for (Graph &g : cs->graphs)
        if (g.exec) cudaGraphExecDestroy(g.exec);
    cs->graphs.clear();
    cs->by_hash.clear();
}

void invalidate_capture(slc_device *d) {
    if (d->capture) drop_graphs(d->capture);
    decode_run_invalidate(d);
}

extern "C" int slc_set_capture(slc_device *d, int enabled) {
    if (!d) return SLC_ERR_EXECUTION;
    int rc = flush_capture(d);
    if (rc != SLC_OK) return rc;
    if (!enabled) {
        release_capture(d);
        return SLC_OK;
    }
    if (d->capture) return SLC_OK;
    cudaSetDevice(d->ordinal);
    CaptureState *cs = new (std::nothrow) CaptureState();
    if (!cs) return slc_fail(d, SLC_ERR_OUT_OF_MEMORY, "capture state allocation failed");
    if (cudaMallocHost(&cs->h_table, kTableSlots * sizeof(uint32_t)) != cudaSuccess ||
        cudaMalloc(&cs->d_table, kTableSlots * sizeof(uint32_t)) != cudaSuccess ||
        cudaEventCreateWithFlags(&cs->table_done, cudaEventDisableTiming) != cudaSuccess) {
        if (cs->h_table) cudaFreeHost(cs->h_table);
        if (cs->d_table) cudaFree(cs->d_table);
        delete cs;
        return slc_fail(d, SLC_ERR_OUT_OF_MEMORY, "capture scalar table allocation failed");
    }
    cs->pending.reserve(1024);
    cs->key.reserve(1 << 20);
    d->capture = cs;
    return decode_run_create(d);
}

extern "C" int slc_capture_stats(const slc_device *d, slc_capture_info *out) {
    if (!d || !out) return SLC_ERR_EXECUTION;
    *out = d->capture ? d->capture->stats : slc_capture_info{};
    return SLC_OK;
}

extern "C" int slc_decode_fusion_stats(const slc_device *d, slc_decode_fusion_info *out) {
    if (!d || !out) return SLC_ERR_EXECUTION;
    return decode_run_stats(d, out);
}

void release_capture(slc_device *d) {
    CaptureState *cs = d->capture;
    if (!cs) return;
    cudaSetDevice(d->ordinal);
    cudaStreamSynchronize(d->stream);
    drop_graphs(cs);
    decode_run_release(d);
    if (cs->h_table) cudaFreeHost(cs->h_table);
    if (cs->d_table) cudaFree(cs->d_table);
    if (cs->table_done) cudaEventDestroy(cs->table_done);
    delete cs;
    d->capture = nullptr;
}

int capture_record(slc_device *d, const slc_op *op, const slc_buffer_ref *in,
                   const slc_value *iv, uint64_t n_in, const slc_buffer_ref *out,
                   const slc_value *ov, uint64_t n_out, const uint32_t *scalars,
                   uint64_t n_scalars) {
    CaptureState *cs = d->capture;
    const bool dyn = dynamic_scalars(op->code);
    if (n_in > kMaxPorts || n_out > kMaxPorts || n_scalars > kMaxPorts ||
        (dyn && cs->table_used + n_scalars > kTableSlots)) {
        // Not recordable: run what is pending, then this command eagerly.
        flush_capture(d);
        return 0;
    }
    cs->pending.emplace_back();  // built in place: a Rec is ~1.4 KB
    Rec &r = cs->pending.back();
    memset(&r, 0, sizeof(r));  // the key is built from raw bytes
    r.op = *op;
    r.n_in = (uint32_t)n_in;
    r.n_out = (uint32_t)n_out;
    r.n_scalars = (uint32_t)n_scalars;
    for (uint64_t i = 0; i < n_in; i++) {
        r.in[i] = in[i];
        r.in[i].reserved = 0;
        r.iv[i] = iv[i];
    }
    for (uint64_t i = 0; i < n_out; i++) {
        r.out[i] = out[i];
        r.out[i].reserved = 0;
        r.ov[i] = ov[i];
    }
    for (uint64_t i = 0; i < n_scalars; i++) r.scalars[i] = scalars[i];
    r.slot = -1;
    if (dyn && n_scalars) {
        r.slot = (int32_t)cs->table_used;
        cs->table_used += (uint32_t)n_scalars;
    }
    // Key: everything but the values of dynamic scalars.
    append_key(cs, &r.op, sizeof(r.op));
    append_key(cs, &r.n_in, sizeof(uint32_t) * 3);
    append_key(cs, r.in, sizeof(slc_buffer_ref) * n_in);
    append_key(cs, r.iv, sizeof(slc_value) * n_in);
    append_key(cs, r.out, sizeof(slc_buffer_ref) * n_out);
    append_key(cs, r.ov, sizeof(slc_value) * n_out);
    if (!dyn) append_key(cs, r.scalars, sizeof(uint32_t) * n_scalars);
    return 1;
}

static bool overlaps(const slc_buffer_ref &a, const slc_buffer_ref &b) {
    return a.buffer == b.buffer && a.offset < b.offset + b.len && b.offset < a.offset + a.len;
}

// Length of the run of MatMulNT commands starting at i that read the same
// input with quantized weights and write pairwise disjoint outputs (which
// then do not depend on each other): such a run can be one grouped launch.
static int matmul_run(const std::vector<Rec> &v, size_t i) {
    const Rec &a = v[i];
    if (a.op.code != SLC_OP_MATMUL_NT || a.n_in != 2 || a.n_out != 1 ||
        a.iv[1].encoding != SLC_ENC_GROUPWISE)
        return 1;
    size_t j = i + 1;
    for (; j < v.size() && j - i < 4; j++) {
        const Rec &b = v[j];
        if (b.op.code != SLC_OP_MATMUL_NT || b.n_in != 2 || b.n_out != 1 ||
            b.iv[1].encoding != SLC_ENC_GROUPWISE || memcmp(&b.in[0], &a.in[0], sizeof(a.in[0])) ||
            memcmp(&b.iv[0], &a.iv[0], sizeof(a.iv[0])))
            break;
        bool clash = false;
        for (size_t t = i; t < j; t++)
            if (overlaps(v[t].out[0], b.out[0]) || overlaps(v[t].out[0], b.in[1]) ||
                overlaps(b.out[0], a.in[0]))
                clash = true;
        if (clash) break;
    }
    return (int)(j - i);
}

// Whether a command before position i writes bytes of layer `layer` of the
// KV state `st`: as an output, or as the State input of an attention / append
// command on the same layer (those write only their own layer's slice).
static bool written_before(const std::vector<Rec> &v, size_t i, const slc_buffer_ref &st,
                           uint32_t layer) {
    for (size_t t = 0; t < i; t++) {
        const Rec &r = v[t];
        for (uint32_t o = 0; o < r.n_out; o++)
            if (overlaps(r.out[o], st)) return true;
        for (uint32_t q = 0; q < r.n_in; q++) {
            if (r.iv[q].role != SLC_ROLE_STATE || !overlaps(r.in[q], st)) continue;
            const bool layered = r.op.code == SLC_OP_CAUSAL_ATTENTION || r.op.code == SLC_OP_KV_APPEND;
            if (!layered || r.op.layer == layer || memcmp(&r.in[q], &st, sizeof(st)) != 0)
                return true;
        }
    }
    return false;
}

// BlockMember views of the recorded commands (the operator layer's form).
static void members(const std::vector<Rec> &v, std::vector<BlockMember> *bm) {
    bm->clear();
    bm->reserve(v.size());
    for (const Rec &r : v)
        bm->push_back(BlockMember{&r.op, r.in, r.iv, r.n_in, r.out, r.ov, r.scalars, r.n_scalars});
}

// Runs of whole decoder layers that go out as one persistent launch:
// (first command, command count), in order, non-overlapping.
static std::vector<std::pair<size_t, size_t>> decode_runs(slc_device *d,
                                                          const std::vector<BlockMember> &bm) {
    std::vector<std::pair<size_t, size_t>> runs;
    if (!d->decode) return runs;
    for (size_t i = 0; i < bm.size();) {
        const size_t n =
            bm[i].op->code == SLC_OP_RMS_NORM ? decode_run_match(d, &bm[i], bm.size() - i) : 0;
        if (n) {
            runs.emplace_back(i, n);
            i += n;
        } else {
            i++;
        }
    }
    return runs;
}

// Device copies of the scalars of commands [first, first + n) (graph
// capture), or null for commands without dynamic scalars.
static std::vector<const uint32_t *> dyn_scalars(const CaptureState *cs, size_t first, size_t n) {
    std::vector<const uint32_t *> out(n, nullptr);
    for (size_t j = 0; j < n; j++) {
        const Rec &r = cs->pending[first + j];
        if (r.slot >= 0) out[j] = cs->d_table + r.slot;
    }
    return out;
}

// Restores the programmatic-launch setting of this thread on scope exit.
struct PdlScope {
    bool saved = slc::k::pdl_enabled();
    ~PdlScope() { slc::k::set_pdl_enabled(saved); }
};

// Runs the pending commands; dyn = kernels read the device scalar table
// (graph capture). Runs of MatMulNT on one input go out as grouped GEMVs;
// the decode attention block (SplitHeads x3, Rope x2, CausalAttention,
// MergeHeads at seq 1) goes out as the fused two-launch block, a residual
// Add followed by the RmsNorm of its sum as one launch, and a tensor-parallel
// AllReduce feeding that pair as one peer-memory launch.
static int run_pending(slc_device *d, CaptureState *cs, bool dyn) {
    const std::vector<Rec> &v = cs->pending;
    std::vector<BlockMember> all;
    members(v, &all);
    const auto runs = decode_runs(d, all);
    size_t next_run = 0;
    // The first command of a segment does not overlap earlier work: kernels
    // that read data before their dependency wait can then only overlap
    // commands of their own segment.
    PdlScope pdl;
    for (size_t i = 0; i < v.size();) {
        slc::k::set_pdl_enabled(pdl.saved && i > 0);
        if (next_run < runs.size() && runs[next_run].first == i) {
            const size_t n = runs[next_run].second;
            next_run++;
            const auto ds = dyn_scalars(cs, i, n);
            bool launched = false;
            int rc = decode_run_launch(d, &all[i], n, dyn ? ds.data() : nullptr, false, &launched);
            if (rc != SLC_OK) return rc;
            if (launched) {
                i += n;
                continue;
            }
        }
        // Other fusions end before the next decode run begins.
        const size_t limit = next_run < runs.size() ? runs[next_run].first : v.size();
        if (v[i].op.code == SLC_OP_SPLIT_HEADS && i + 7 <= limit &&
            v[i + 5].op.code == SLC_OP_CAUSAL_ATTENTION) {
            BlockMember bm[7];
            for (int t = 0; t < 7; t++) {
                const Rec &r = v[i + t];
                bm[t] = BlockMember{&r.op, r.in, r.iv, r.n_in, r.out, r.ov, r.scalars, r.n_scalars};
            }
            const Rec &at = v[i + 5];
            const uint32_t *ds = (dyn && at.slot >= 0) ? cs->d_table + at.slot : nullptr;
            bool launched = false;
            const bool early = !written_before(v, i, at.in[3], at.op.layer);
            int rc = slc_launch_attention_block(d, bm, ds, early, &launched);
            if (rc != SLC_OK) return rc;
            if (launched) {
                i += 7;
                continue;
            }
        }
        if (v[i].op.code == SLC_OP_EXT_ALL_REDUCE && i + 3 <= limit &&
            v[i + 1].op.code == SLC_OP_ADD && v[i + 2].op.code == SLC_OP_RMS_NORM) {
            BlockMember bm[3];
            for (int t = 0; t < 3; t++) {
                const Rec &r = v[i + t];
                bm[t] = BlockMember{&r.op, r.in, r.iv, r.n_in, r.out, r.ov, r.scalars, r.n_scalars};
            }
            bool launched = false;
            int rc = slc_launch_allreduce_add_rmsnorm(d, &bm[0], &bm[1], &bm[2], &launched);
            if (rc != SLC_OK) return rc;
            if (launched) {
                i += 3;
                continue;
            }
        }
        if (v[i].op.code == SLC_OP_ADD && i + 2 <= limit &&
            v[i + 1].op.code == SLC_OP_RMS_NORM) {
            const Rec &ra = v[i], &rr = v[i + 1];
            const BlockMember add{&ra.op, ra.in, ra.iv, ra.n_in, ra.out, ra.ov, ra.scalars,
                                  ra.n_scalars};
            const BlockMember rms{&rr.op, rr.in, rr.iv, rr.n_in, rr.out, rr.ov, rr.scalars,
                                  rr.n_scalars};
            bool launched = false;
            int rc = slc_launch_add_rmsnorm(d, &add, &rms, &launched);
            if (rc != SLC_OK) return rc;
            if (launched) {
                i += 2;
                continue;
            }
        }
        const int run = (int)std::min<size_t>((size_t)matmul_run(v, i), limit - i);
        if (run > 1) {
            MatmulMember mm[4];
            for (int t = 0; t < run; t++)
                mm[t] = MatmulMember{v[i + t].in, v[i + t].iv, v[i + t].out, v[i + t].ov};
            bool launched = false;
            int rc = slc_launch_matmul_group(d, mm, run, &launched);
            if (rc != SLC_OK) return rc;
            if (launched) {
                i += run;
                continue;
            }
        }
        const Rec &r = v[i];
        const uint32_t *ds = (dyn && r.slot >= 0) ? cs->d_table + r.slot : nullptr;
        int rc = slc_launch_command(d, &r.op, r.in, r.iv, r.n_in, r.out, r.ov, r.n_out,
                                    r.scalars, r.n_scalars, ds);
        if (rc != SLC_OK) return rc;
        i++;
    }
    return SLC_OK;
}

// The previous table copy must have read the pinned table before it changes.
static int table_wait(slc_device *d, CaptureState *cs) {
    if (cs->table_pending && cudaEventSynchronize(cs->table_done) != cudaSuccess)
        return slc_fail(d, SLC_ERR_EXECUTION, "capture scalar table synchronization failed");
    cs->table_pending = false;
    return SLC_OK;
}

// Copies slots [0, n) of the pinned table to the device table (stream-ordered).
static int table_send(slc_device *d, CaptureState *cs, uint32_t n) {
    if (cudaMemcpyAsync(cs->d_table, cs->h_table, sizeof(uint32_t) * n, cudaMemcpyHostToDevice,
                        d->stream) != cudaSuccess ||
        cudaEventRecord(cs->table_done, d->stream) != cudaSuccess)
        return slc_fail(d, SLC_ERR_EXECUTION, "capture scalar table upload failed");
    cs->table_pending = true;
    return SLC_OK;
}

// Copies the segment's dynamic scalars to the device table (stream-ordered).
static int upload_table(slc_device *d, CaptureState *cs) {
    if (cs->table_used == 0) return SLC_OK;
    const int rc = table_wait(d, cs);
    if (rc != SLC_OK) return rc;
    for (const Rec &r : cs->pending)
        if (r.slot >= 0)
            memcpy(cs->h_table + r.slot, r.scalars, sizeof(uint32_t) * r.n_scalars);
    return table_send(d, cs, cs->table_used);
}

static bool try_capture(slc_device *d, CaptureState *cs, Graph *g) {
    // Program images of decode runs are uploaded now: nothing may be copied
    // to the device while the stream is being captured.
    if (d->decode) {
        std::vector<BlockMember> all;
        members(cs->pending, &all);
        for (const auto &run : decode_runs(d, all)) {
            const auto ds = dyn_scalars(cs, run.first, run.second);
            bool launched = false;
            if (decode_run_launch(d, &all[run.first], run.second, ds.data(), true, &launched) !=
                SLC_OK)
                d->last = slc_error{};
        }
    }
    const uint64_t before = slc::k::launch_count();
    if (cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    const int rc = run_pending(d, cs, true);
    cudaGraph_t graph = nullptr;
    const cudaError_t end = cudaStreamEndCapture(d->stream, &graph);
    const uint64_t launched = slc::k::launch_count() - before;
    slc::k::add_launches(-(int64_t)launched);  // nothing ran yet
    bool ok = rc == SLC_OK && end == cudaSuccess && graph;
    if (ok && cudaGraphInstantiate(&g->exec, graph, 0) != cudaSuccess) ok = false;
    if (graph) cudaGraphDestroy(graph);
    if (!ok) {
        cudaGetLastError();
        g->exec = nullptr;
        d->last = slc_error{};  // a failed capture is not the caller's error
        return false;
    }
    g->launches = launched;
    return true;
}

// Runs the pending segment (replay, capture or eager); *graph_id names the
// graph it ran as, 0 when it ran eagerly or failed.
static int flush_segment(slc_device *d, uint64_t *graph_id) {
    *graph_id = 0;
    CaptureState *cs = d ? d->capture : nullptr;
    if (!cs || cs->pending.empty()) return SLC_OK;
    cudaSetDevice(d->ordinal);
    int rc = SLC_OK;
    auto hit = cs->graphs.end();
    uint64_t h = 0;
    if (!cs->graphs.empty() && cs->graphs.front().key == cs->key) {
        // Repeated steps replay the most recently used graph: comparing the
        // keys settles it without hashing.
        hit = cs->graphs.begin();
    } else {
        h = key_hash(cs->key.data(), cs->key.size());
        auto it = cs->by_hash.find(h);
        if (it != cs->by_hash.end() && it->second->key == cs->key) hit = it->second;
    }
    if (hit != cs->graphs.end()) {
        // Replay.
        cs->graphs.splice(cs->graphs.begin(), cs->graphs, hit);
        Graph &g = cs->graphs.front();
        rc = upload_table(d, cs);
        if (rc == SLC_OK && cudaGraphLaunch(g.exec, d->stream) != cudaSuccess)
            rc = slc_fail(d, SLC_ERR_EXECUTION, "CUDA graph launch failed");
        if (rc == SLC_OK) {
            slc::k::add_launches((int64_t)g.launches);
            cs->stats.replays++;
            cs->stats.replayed_commands += cs->pending.size();
            *graph_id = g.id;
        }
    } else {
        if (cs->seen.size() > 4096) cs->seen.clear();  // bound the history of keys
        int &count = cs->seen[h];
        bool captured = false;
        if (count >= 1) {
            Graph g;
            g.key = cs->key;
            rc = upload_table(d, cs);
            if (rc == SLC_OK && try_capture(d, cs, &g)) {
                g.id = g_next_graph_id.fetch_add(1);
                if (cs->graphs.size() >= kMaxGraphs) {
                    Graph &old = cs->graphs.back();
                    cs->by_hash.erase(key_hash(old.key.data(), old.key.size()));
                    if (old.exec) cudaGraphExecDestroy(old.exec);
                    cs->graphs.pop_back();
                }
                cs->graphs.push_front(std::move(g));
                cs->by_hash[h] = cs->graphs.begin();
                Graph &ng = cs->graphs.front();
                if (cudaGraphLaunch(ng.exec, d->stream) != cudaSuccess) {
                    rc = slc_fail(d, SLC_ERR_EXECUTION, "CUDA graph launch failed");
                } else {
                    slc::k::add_launches((int64_t)ng.launches);
                    cs->stats.captures++;
                    cs->stats.replayed_commands += cs->pending.size();
                    *graph_id = ng.id;
                }
                captured = true;
            } else if (rc == SLC_OK) {
                count = -1;  // does not capture; stay eager
            }
        }
        if (!captured && rc == SLC_OK) {
            if (count >= 0) count++;
            rc = run_pending(d, cs, false);
            cs->stats.eager_commands += cs->pending.size();
        }
    }
    cs->pending.clear();
    cs->key.clear();
    cs->table_used = 0;
    return rc;
}

int flush_capture(slc_device *d) {
    uint64_t graph_id;
    return flush_segment(d, &graph_id);
}

// Step memo. A caller that dispatches the same command list every step
// (an engine program: the same operators on the same buffers, only seq_len
// and past_len changing) builds the same segment key every time, so the
// segment always replays the same graph; only the device table of dynamic
// scalars differs. After a step whose commands were flushed as exactly one
// segment that ran as a graph, the memo keeps that graph's id and, for every
// table slot, which of the caller's scalar sources fills it. The next steps
// then skip dispatching (validating, recording, keying) their commands:
// they fill the table from the sources and relaunch the graph. Validation is
// not lost: every check of a command depends only on its buffers, values
// and the caller's scalars; buffers and quantization bindings cannot change
// without dropping every graph (which empties the memo: its graph is no
// longer found), and the scalars' range checks are the caller's, done before
// each step (seq_len within the program, past_len + seq within the cache).
// Only on a device without a communicator: a tensor-parallel step keeps the
// per-command path.
static std::list<Graph>::iterator memo_graph(CaptureState *cs, const StepMemo *m) {
    if (!m->graph_id) return cs->graphs.end();
    for (auto it = cs->graphs.begin(); it != cs->graphs.end(); ++it)
        if (it->id == m->graph_id) return it;
    return cs->graphs.end();
}

bool capture_memo_valid(slc_device *d, const StepMemo *m) {
    CaptureState *cs = d ? d->capture : nullptr;
    return cs && !d->comm && cs->pending.empty() && memo_graph(cs, m) != cs->graphs.end();
}

int capture_memo_replay(slc_device *d, StepMemo *m, const uint32_t *src, size_t n_src) {
    CaptureState *cs = d->capture;
    auto it = memo_graph(cs, m);
    if (it == cs->graphs.end() || !cs->pending.empty())
        return slc_fail(d, SLC_ERR_EXECUTION, "step memo replayed without its graph");
    for (uint32_t s : m->slot_src)
        if (s >= n_src) return slc_fail(d, SLC_ERR_EXECUTION, "step memo scalar source out of range");
    cudaSetDevice(d->ordinal);
    const uint32_t n = (uint32_t)m->slot_src.size();
    int rc = SLC_OK;
    if (n) {
        if ((rc = table_wait(d, cs)) != SLC_OK) return rc;
        for (uint32_t i = 0; i < n; i++) cs->h_table[i] = src[m->slot_src[i]];
        if ((rc = table_send(d, cs, n)) != SLC_OK) return rc;
    }
    cs->graphs.splice(cs->graphs.begin(), cs->graphs, it);
    Graph &g = cs->graphs.front();
    if (cudaGraphLaunch(g.exec, d->stream) != cudaSuccess)
        return slc_fail(d, SLC_ERR_EXECUTION, "CUDA graph launch failed");
    slc::k::add_launches((int64_t)g.launches);
    cs->stats.replays++;
    cs->stats.replayed_commands += m->commands;
    return SLC_OK;
}

int capture_flush_memo(slc_device *d, StepMemo *m, const int *src_flat, const uint32_t *src_count,
                       size_t n_cmds) {
    m->graph_id = 0;
    CaptureState *cs = d ? d->capture : nullptr;
    if (!cs) return flush_capture(d);
    // Which source fills each table slot, read off the recorded commands
    // before the flush clears them. Eligible only when the pending segment
    // is exactly the caller's commands and every scalar is a device-table
    // scalar (a scalar in the key would make the next step's key differ).
    bool ok = !d->comm && cs->pending.size() == n_cmds;
    std::vector<uint32_t> slot_src;
    if (ok) {
        slot_src.assign(cs->table_used, UINT32_MAX);
        size_t off = 0;
        for (size_t i = 0; i < n_cmds && ok; i++) {
            const Rec &r = cs->pending[i];
            if (r.n_scalars != src_count[i] || (r.n_scalars && r.slot < 0)) {
                ok = false;
                break;
            }
            for (uint32_t j = 0; j < r.n_scalars; j++)
                slot_src[(size_t)r.slot + j] = (uint32_t)src_flat[off + j];
            off += src_count[i];
        }
        for (uint32_t s : slot_src) ok = ok && s != UINT32_MAX;
    }
    uint64_t graph_id;
    const int rc = flush_segment(d, &graph_id);
    if (rc == SLC_OK && ok && graph_id) {
        m->graph_id = graph_id;
        m->slot_src = std::move(slot_src);
        m->commands = n_cmds;
    }
    return rc;
}
