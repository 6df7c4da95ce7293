// Tensor-parallel collectives for backend-cuda: one NCCL communicator per
// device, collectives enqueued on the device stream (so they order with the
// kernels and can sit inside a captured CUDA graph).
//
// NCCL is loaded at run time with dlopen("libnccl.so.2"): when the host
// process already carries an NCCL (PyTorch bundles one) the same library is
// reused, and the product library has no link-time NCCL dependency.
// The reference has no distributed communication at all (README.md:107);
// this is the Megatron-style tensor parallelism the llama-dense layer
// admits: an all-reduce after the row-parallel o/down projections and an
// all-gather of vocabulary-split logits.
//
// Peer exchange: for the decode-sized all-reduce (fused with the residual
// Add and RmsNorm, comm_fused.cu) every rank allocates an exchange buffer at
// init, shares its CUDA IPC handle through an NCCL all-gather and maps its
// peers' buffers; the path is used only when every rank succeeded (agreed by
// an NCCL min-reduction), otherwise the NCCL all-reduce serves all sizes.
// SLC_PEER_ALLREDUCE=0 in the environment of any rank switches it off. The
// same buffer holds the persistent decode kernel's exchange words and its
// launch count; that kernel is used under tensor parallelism only when every
// rank also allows decode fusion (SLC_DECODE_FUSION, same agreement).
//
// Failures: slc_comm_abort tears the communicator down without the other
// ranks (ncclCommAbort) once a host-side check found that a peer left;
// slc_comm_async_error polls ncclCommGetAsyncError.
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "device_internal.h"
#include "kernels/kernels.h"

namespace {

struct NcclApi {
    void *handle = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
                               ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*abort)(ncclComm_t) = nullptr;
    ncclResult_t (*async_error)(ncclComm_t, ncclResult_t *) = nullptr;
    bool ok = false;
};

NcclApi &api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        const char *names[] = {"libnccl.so.2", "libnccl.so"};
        for (const char *n : names) {
            a.handle = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
            if (a.handle) break;
        }
        if (!a.handle) return;
        a.get_unique_id = (decltype(a.get_unique_id))dlsym(a.handle, "ncclGetUniqueId");
        a.init_rank = (decltype(a.init_rank))dlsym(a.handle, "ncclCommInitRank");
        a.all_reduce = (decltype(a.all_reduce))dlsym(a.handle, "ncclAllReduce");
        a.all_gather = (decltype(a.all_gather))dlsym(a.handle, "ncclAllGather");
        a.destroy = (decltype(a.destroy))dlsym(a.handle, "ncclCommDestroy");
        a.abort = (decltype(a.abort))dlsym(a.handle, "ncclCommAbort");
        a.async_error = (decltype(a.async_error))dlsym(a.handle, "ncclCommGetAsyncError");
        a.ok = a.get_unique_id && a.init_rank && a.all_reduce && a.all_gather && a.destroy &&
               a.abort && a.async_error;
    });
    return a;
}

}  // namespace

// Exchange buffer geometry (rows x hidden per source rank and parity).
constexpr size_t kXRows = 32, kXHidden = 8192;

struct CommState {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    bool peer_ok = false;
    bool decode_ok = false;                      // every rank fuses decode layers (peer exchange)
    char *xbuf = nullptr;                        // this rank's exchange buffer
    char *peer_base[slc::k::kMaxPeers] = {};     // every rank's buffer (own = xbuf)
    size_t data_bytes = 0, flag_bytes = 0;
    size_t dec_data_off = 0, dec_count_off = 0;   // the persistent decode kernel's words, launch count
};

namespace {

void release_peers(CommState *c) {
    for (int p = 0; p < c->world && p < slc::k::kMaxPeers; p++)
        if (p != c->rank && c->peer_base[p]) cudaIpcCloseMemHandle(c->peer_base[p]);
    if (c->xbuf) cudaFree(c->xbuf);
    for (auto &b : c->peer_base) b = nullptr;
    c->xbuf = nullptr;
    c->peer_ok = false;
    c->decode_ok = false;
}

bool decode_fusion_requested() {
    const char *e = getenv("SLC_DECODE_FUSION");
    return !(e && e[0] == '0');
}

bool peer_exchange_requested() {
    const char *e = getenv("SLC_PEER_ALLREDUCE");
    return !(e && strcmp(e, "0") == 0);
}

// Collective over all ranks: every rank calls it from slc_comm_init and takes
// the same NCCL steps whatever fails (or is switched off) locally.
void setup_peers(slc_device *d, CommState *c) {
    NcclApi &a = api();
    if (c->world < 2 || c->world > slc::k::kMaxPeers) return;
    c->data_bytes = 2 * (size_t)c->world * kXRows * kXHidden * sizeof(float);
    c->flag_bytes = 2 * (size_t)c->world * kXRows * sizeof(uint32_t);
    // Then the persistent decode kernel's region: words [2][world][kDlTpHidden]
    // of {f32, epoch} (decode_layers.cu) and this rank's count of fused
    // decode launches.
    c->dec_data_off = (c->data_bytes + c->flag_bytes + kXRows * sizeof(uint32_t) + 255) / 256 * 256;
    c->dec_count_off = c->dec_data_off + 2 * (size_t)c->world * slc::k::kDlTpHidden * sizeof(uint64_t);
    const size_t total = c->dec_count_off + 16;
    bool ok = peer_exchange_requested() && cudaMalloc(&c->xbuf, total) == cudaSuccess &&
              cudaMemset(c->xbuf, 0, total) == cudaSuccess &&
              cudaDeviceSynchronize() == cudaSuccess;
    cudaIpcMemHandle_t mine{};
    if (ok) ok = cudaIpcGetMemHandle(&mine, c->xbuf) == cudaSuccess;
    // Gather the handles through NCCL; staging in the kernel scratch.
    char *dh = ws_scratch(d);
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    static_assert(sizeof(cudaIpcMemHandle_t) <= 64, "IPC handle size");
    char handles[slc::k::kMaxPeers][64];
    const bool gathered =
        cudaMemcpyAsync(dh + (size_t)c->rank * 64, &mine, hb, cudaMemcpyHostToDevice, d->stream) ==
            cudaSuccess &&
        a.all_gather(dh + (size_t)c->rank * 64, dh, 64, ncclUint8, c->comm, d->stream) ==
            ncclSuccess &&
        cudaMemcpyAsync(handles, dh, 64 * (size_t)c->world, cudaMemcpyDeviceToHost, d->stream) ==
            cudaSuccess &&
        cudaStreamSynchronize(d->stream) == cudaSuccess;
    ok = ok && gathered;
    for (int p = 0; ok && p < c->world; p++) {
        if (p == c->rank) {
            c->peer_base[p] = c->xbuf;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, handles[p], hb);
        void *ptr = nullptr;
        ok = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
        c->peer_base[p] = static_cast<char *>(ptr);
    }
    cudaGetLastError();
    // Agreement: on only if every rank succeeded (2: every rank also fuses
    // decode layers, whose exchanges must then happen on all ranks alike).
    int32_t flag = ok ? (decode_fusion_requested() ? 3 : 1) : 0;
    int32_t *df = reinterpret_cast<int32_t *>(dh);
    const bool agreed =
        cudaMemcpyAsync(df, &flag, 4, cudaMemcpyHostToDevice, d->stream) == cudaSuccess &&
        a.all_reduce(df, df, 1, ncclInt32, ncclMin, c->comm, d->stream) == ncclSuccess &&
        cudaMemcpyAsync(&flag, df, 4, cudaMemcpyDeviceToHost, d->stream) == cudaSuccess &&
        cudaStreamSynchronize(d->stream) == cudaSuccess && flag >= 1;
    cudaGetLastError();
    if (agreed) {
        c->peer_ok = true;
        c->decode_ok = flag == 3;
    } else {
        release_peers(c);
    }
}

}  // namespace

bool comm_peer_args(slc_device *d, slc::k::PeerReduceArgs *a) {
    CommState *c = d ? d->comm : nullptr;
    if (!c || !c->peer_ok) return false;
    for (int p = 0; p < c->world; p++) {
        a->peer_data[p] = reinterpret_cast<float *>(c->peer_base[p]);
        a->peer_flags[p] = reinterpret_cast<uint32_t *>(c->peer_base[p] + c->data_bytes);
    }
    a->local_data = reinterpret_cast<const float *>(c->xbuf);
    a->local_flags = reinterpret_cast<const uint32_t *>(c->xbuf + c->data_bytes);
    a->counters = reinterpret_cast<uint32_t *>(c->xbuf + c->data_bytes + c->flag_bytes);
    a->rank = c->rank;
    a->world = c->world;
    a->max_rows = kXRows;
    a->max_hidden = kXHidden;
    return true;
}

bool comm_decode_peers(slc_device *d, slc::k::DlPeers *out) {
    CommState *c = d ? d->comm : nullptr;
    if (!c || !c->peer_ok || !c->decode_ok) return false;
    out->rank = c->rank;
    out->world = c->world;
    for (int p = 0; p < c->world; p++)
        out->words[p] = reinterpret_cast<uint64_t *>(c->peer_base[p] + c->dec_data_off);
    out->launches = reinterpret_cast<uint32_t *>(c->xbuf + c->dec_count_off);
    return true;
}

extern "C" int slc_comm_peer_status(const slc_device *d, int *peer_allreduce, int *decode_fusion) {
    if (!d) return SLC_ERR_EXECUTION;
    const CommState *c = d->comm;
    if (peer_allreduce) *peer_allreduce = c && c->peer_ok ? 1 : 0;
    if (decode_fusion) *decode_fusion = c && c->peer_ok && c->decode_ok ? 1 : 0;
    return SLC_OK;
}

extern "C" int slc_comm_unique_id(uint8_t out_id[128]) {
    if (!out_id) return SLC_ERR_EXECUTION;
    NcclApi &a = api();
    if (!a.ok) return SLC_ERR_UNIMPLEMENTED;
    ncclUniqueId id;
    if (a.get_unique_id(&id) != ncclSuccess) return SLC_ERR_EXECUTION;
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    memcpy(out_id, &id, 128);
    return SLC_OK;
}

extern "C" int slc_comm_init(slc_device *d, const uint8_t unique_id[128], int rank, int world) {
    if (!d || !unique_id) return SLC_ERR_EXECUTION;
    if (world < 1 || rank < 0 || rank >= world) return slc_fail(d, SLC_ERR_EXECUTION, "invalid rank");
    NcclApi &a = api();
    if (!a.ok) return slc_fail(d, SLC_ERR_UNIMPLEMENTED, "libnccl.so.2 could not be loaded");
    int rc = flush_capture(d);
    if (rc != SLC_OK) return rc;
    invalidate_capture(d);  // graphs hold the communicator
    release_comm(d);
    ncclUniqueId id;
    memcpy(&id, unique_id, 128);
    cudaSetDevice(d->ordinal);
    CommState *c = new CommState();
    c->rank = rank;
    c->world = world;
    if (a.init_rank(&c->comm, world, id, rank) != ncclSuccess) {
        delete c;
        return slc_fail(d, SLC_ERR_EXECUTION, "ncclCommInitRank failed");
    }
    d->comm = c;
    setup_peers(d, c);
    return SLC_OK;
}

extern "C" int slc_comm_async_error(slc_device *d) {
    if (!d) return SLC_ERR_EXECUTION;
    CommState *c = d->comm;
    if (!c) return SLC_OK;
    if (!c->comm) return slc_fail(d, SLC_ERR_EXECUTION, "the communicator was aborted");
    ncclResult_t r = ncclSuccess;
    if (api().async_error(c->comm, &r) != ncclSuccess || (r != ncclSuccess && r != ncclInProgress))
        return slc_fail(d, SLC_ERR_EXECUTION, "the communicator reported an asynchronous error");
    return SLC_OK;
}

extern "C" int slc_comm_abort(slc_device *d) {
    if (!d) return SLC_ERR_EXECUTION;
    CommState *c = d->comm;
    if (!c || !c->comm) return SLC_OK;
    cudaSetDevice(d->ordinal);
    // Captured graphs hold the communicator and the peer mappings.
    invalidate_capture(d);
    release_peers(c);
    api().abort(c->comm);
    c->comm = nullptr;
    cudaGetLastError();
    return SLC_OK;
}

extern "C" int slc_comm_world(const slc_device *d, int *rank, int *world) {
    if (!d) return SLC_ERR_EXECUTION;
    if (rank) *rank = d->comm ? d->comm->rank : 0;
    if (world) *world = d->comm ? d->comm->world : 1;
    return SLC_OK;
}

void release_comm(slc_device *d) {
    if (!d->comm) return;
    cudaSetDevice(d->ordinal);
    release_peers(d->comm);
    if (d->comm->comm && api().ok) api().destroy(d->comm->comm);  // null after slc_comm_abort
    delete d->comm;
    d->comm = nullptr;
}

int comm_all_reduce(slc_device *d, float *data, uint64_t count) {
    if (!d->comm || (d->comm->world > 1 && !d->comm->comm)) return SLC_ERR_EXECUTION;
    if (count == 0 || d->comm->world == 1) return SLC_OK;
    ncclResult_t r = api().all_reduce(data, data, count, ncclFloat32, ncclSum, d->comm->comm,
                                      d->stream);
    slc::k::count_launch();
    return r == ncclSuccess ? SLC_OK : SLC_ERR_EXECUTION;
}

int comm_all_gather(slc_device *d, const float *in, float *out, uint64_t rows, uint64_t cols) {
    if (!d->comm || (d->comm->world > 1 && !d->comm->comm)) return SLC_ERR_EXECUTION;
    const uint64_t world = (uint64_t)d->comm->world;
    if (rows == 0 || cols == 0) return SLC_OK;
    if (world == 1) return slc::k::copy_f32(d->stream, in, out, rows * cols) == cudaSuccess
                              ? SLC_OK : SLC_ERR_EXECUTION;
    // NCCL gathers rank blocks contiguously ([world][rows][cols]); with one
    // row that already is [rows, world * cols], otherwise interleave.
    // Staging in the kernel-scratch region of the workspace.
    float *dst = rows == 1 ? out : reinterpret_cast<float *>(ws_scratch(d));
    if (rows > 1 && world * rows * cols * sizeof(float) > ws_scratch_bytes(d))
        return SLC_ERR_EXECUTION;
    ncclResult_t r = api().all_gather(in, dst, rows * cols, ncclFloat32, d->comm->comm, d->stream);
    slc::k::count_launch();
    if (r != ncclSuccess) return SLC_ERR_EXECUTION;
    if (rows > 1 &&
        slc::k::interleave_blocks(d->stream, dst, out, world, rows, cols) != cudaSuccess)
        return SLC_ERR_EXECUTION;
    return SLC_OK;
}
