// Expert-parallel driver over NCCL: one rank's whole configuration-4 step behind the C ABI.
//
// The reference has no expert-parallel exchange on this path (its MoE layer runs on one host);
// this is the C++ side that the per-rank pieces of vlb_abi.cu (route, half-row plan, given-routes
// forward, pack, combine) were built for:
//
//   route -> plan (expert-sorted send rows, one host read of the per-slot offsets)
//   -> counts all-to-all -> rows + meta all-to-all -> own rows for the shared expert
//   -> group forward (routed experts of this rank + the shared expert, tensor-core path)
//   -> pack fp16 results -> results all-to-all -> combine in slot order.
//
// The exchanges are grouped ncclSend / ncclRecv on the caller's stream, ordered with the kernels
// without host synchronisation except where sizes are needed. With two or more ranks whose GPUs
// reach each other (CUDA IPC over NVLink), the two large payloads - the dispatched fp16 rows and
// the fp16 results coming back - move instead by peer stores: every rank maps its peers' receive
// buffers at layer creation and one copy kernel writes each peer's rows straight into place (the
// full count matrix, exchanged first, gives every rank its offsets in every peer's buffer). The
// small meta / scale exchange that follows on the same stream is the fence: a receiver's NCCL
// receive completes only after the sender's NCCL call ran, which is after its copy kernel (whose
// stores end with a system-scope fence). The next step's counts exchange orders the reuse of the
// buffers the same way. VLB_EP_EXCHANGE=nccl keeps everything on NCCL. NCCL is loaded at run time (dlopen
// of $VLB_NCCL_LIBRARY, else libnccl.so.2, reusing the copy the process already has), so the
// library itself loads and runs its other entry points without NCCL.
//
// Failure handling: the communicator is non-blocking, and every host wait (communicator set-up,
// the count read-back, the end of a step) polls both the CUDA event and ncclCommGetAsyncError
// under the communicator's time limit. A peer that fails, leaves or never arrives makes the wait
// run out (or NCCL report an error); the driver then aborts the communicator (which ends NCCL's
// kernels on this GPU) and marks the layer failed with the phase's name ("counts", "dispatch",
// "return"); every later forward is refused. Rebuild the communicator and the layer to go on.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "vlb200.h"

namespace vlb {
void set_thread_error(const std::string& msg);  // vlb_abi.cu
}

namespace {

// ---- NCCL entry points, resolved once per process ----------------------------------------------
struct NcclApi {
    bool ok = false;
    std::string why;
    int version = 0;
    ncclResult_t (*GetVersion)(int*) = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
};

template <class F>
bool bind(void* lib, const char* name, F& f) {
    f = reinterpret_cast<F>(dlsym(lib, name));
    return f != nullptr;
}

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* env = std::getenv("VLB_NCCL_LIBRARY");
        void* lib = nullptr;
        if (env && *env) {
            lib = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
        } else {
            lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);  // the process's copy
            if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        }
        if (!lib) {
            const char* e = dlerror();
            api.why = std::string("NCCL library not found: ") + (e ? e : "dlopen failed");
            return;
        }
        bool all = bind(lib, "ncclGetVersion", api.GetVersion) && bind(lib, "ncclGetUniqueId", api.GetUniqueId) &&
                   bind(lib, "ncclCommInitRankConfig", api.CommInitRankConfig) &&
                   bind(lib, "ncclCommFinalize", api.CommFinalize) && bind(lib, "ncclCommDestroy", api.CommDestroy) &&
                   bind(lib, "ncclCommAbort", api.CommAbort) &&
                   bind(lib, "ncclCommGetAsyncError", api.CommGetAsyncError) &&
                   bind(lib, "ncclGetErrorString", api.GetErrorString) && bind(lib, "ncclGroupStart", api.GroupStart) &&
                   bind(lib, "ncclGroupEnd", api.GroupEnd) && bind(lib, "ncclSend", api.Send) &&
                   bind(lib, "ncclRecv", api.Recv);
        if (!all) {
            api.why = "the NCCL library lacks an entry point this driver needs (NCCL >= 2.18 is required)";
            return;
        }
        if (api.GetVersion(&api.version) != ncclSuccess || api.version < 21800) {
            api.why = "NCCL >= 2.18 is required (non-blocking communicators with finalize)";
            return;
        }
        api.ok = true;
    });
    return api;
}

int fail(int code, const std::string& msg) {
    vlb::set_thread_error(msg);
    return code;
}

std::string nccl_msg(const char* op, ncclResult_t r) {
    return std::string("NCCL call failed: ") + op + " (status=" + std::to_string((int)r) + ", " +
           nccl().GetErrorString(r) + ")";
}

std::string cuda_msg(const char* op, cudaError_t e) {
    return std::string("CUDA call failed: ") + op + " (status=" + std::to_string((int)e) + ", " +
           cudaGetErrorName(e) + ": " + cudaGetErrorString(e) + ")";
}

int handle_fail(vlb_handle* h, int st) {
    char buf[512];
    vlb_last_error(h, buf, sizeof(buf));
    return fail(st, buf);
}

using Clock = std::chrono::steady_clock;

}  // namespace

struct vlb_ep_comm {
    vlb_handle* h = nullptr;
    int device = 0;
    ncclComm_t comm = nullptr;
    int rank = 0, world = 0;
    uint32_t timeout_ms = 0;
    bool aborted = false;

    // Polls the communicator until its pending NCCL calls are issued (ncclInProgress ends) or it
    // reports an error; bounded by the time limit.
    int settle(const char* what) {
        const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
        for (;;) {
            ncclResult_t st = ncclSuccess;
            ncclResult_t r = nccl().CommGetAsyncError(comm, &st);
            if (r != ncclSuccess) return abort_with(VLB_ERR_IO_ERROR, std::string(what) + ": " + nccl_msg("ncclCommGetAsyncError", r));
            if (st == ncclSuccess) return VLB_OK;
            if (st != ncclInProgress) return abort_with(VLB_ERR_IO_ERROR, std::string(what) + ": " + nccl_msg("async", st));
            if (Clock::now() > deadline)
                return abort_with(VLB_ERR_IO_ERROR, std::string(what) + ": no progress within the communicator time limit");
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        }
    }
    // Waits for `ev` (recorded after the work to wait for) while watching the communicator.
    int wait(cudaEvent_t ev, const char* what) {
        const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
        for (;;) {
            cudaError_t q = cudaEventQuery(ev);
            if (q == cudaSuccess) return VLB_OK;
            if (q != cudaErrorNotReady) return abort_with(VLB_ERR_IO_ERROR, std::string(what) + ": " + cuda_msg("cudaEventQuery", q));
            ncclResult_t st = ncclSuccess;
            nccl().CommGetAsyncError(comm, &st);
            if (st != ncclSuccess && st != ncclInProgress)
                return abort_with(VLB_ERR_IO_ERROR, std::string(what) + ": " + nccl_msg("async", st));
            if (Clock::now() > deadline)
                return abort_with(VLB_ERR_IO_ERROR,
                                  std::string(what) + ": a peer did not complete the exchange within the time limit");
            std::this_thread::sleep_for(std::chrono::microseconds(20));
        }
    }
    int abort_with(int code, const std::string& msg) {
        if (comm && !aborted) {
            nccl().CommAbort(comm);  // ends this rank's NCCL kernels; the communicator is unusable after
            aborted = true;
        }
        return fail(code, msg);
    }
};

struct vlb_ep_layer {
    vlb_handle* h = nullptr;
    vlb_ep_comm* c = nullptr;
    uint32_t H = 0, I = 0, E = 0, k = 0, epr = 0, max_tokens = 0;
    int score = 0;
    float route_scale = 1.f;
    vlb_moe_layer_desc group_desc{};
    std::vector<vlb_matrix*> w1, w3, w2;  // this rank's experts + the shared expert last
    std::vector<float> zero_router;
    vlb_layer* group = nullptr;
    uint32_t capacity = 0;  // rows the group layer and receive buffers hold
    std::string failed;     // the exchange that failed, once one has
    // device buffers (vlb_alloc: the governor sees them)
    std::vector<void*> owned;
    float* bias = nullptr;
    uint32_t* slots = nullptr;
    uint32_t* idx = nullptr;
    float* w = nullptr;
    uint32_t* offsets = nullptr;
    void* ws = nullptr;
    uint16_t* send_rows = nullptr;
    uint32_t* send_meta = nullptr;
    uint32_t* elem_row = nullptr;
    uint16_t* own_rows = nullptr;
    uint32_t* own_meta = nullptr;
    uint64_t* counts_dev = nullptr;  // [2 x world]: send counts, then received counts
    uint16_t* back_yh = nullptr;
    float* back_ys = nullptr;
    uint16_t* group_rows = nullptr;
    uint32_t* group_meta = nullptr;
    float* group_y = nullptr;
    uint16_t* group_yh = nullptr;
    float* group_ys = nullptr;
    std::vector<void*> group_owned;
    // peer mode: this rank's receive buffer for dispatched rows (fixed, the worst case of every
    // rank sending it all its pairs) and every rank's receive buffers mapped here (IPC)
    bool peer = false;
    uint16_t* peer_rows = nullptr;
    uint64_t peer_rows_cap = 0;          // rows of peer_rows
    std::vector<uint16_t*> rows_at;      // [W] each rank's dispatch receive buffer
    std::vector<uint16_t*> back_at;      // [W] each rank's results receive buffer (back_yh)
    std::vector<uint64_t> rows_cap_at, back_cap_at;
    std::vector<void*> ipc_opened;
    // pinned host words
    uint32_t* offsets_host = nullptr;
    uint64_t* counts_host = nullptr;     // [W]: send counts, [W]: received counts, [W x W]: matrix
    cudaEvent_t sync_ev = nullptr;
    cudaEvent_t phase[6] = {};
    bool have_phases = false;
    uint64_t last_rows[2] = {0, 0};

    int alloc(size_t bytes, const char* tag, void** p, std::vector<void*>& list) {
        int st = vlb_alloc(h, bytes ? bytes : 16, tag, p);
        if (st != VLB_OK) return handle_fail(h, st);
        list.push_back(*p);
        return VLB_OK;
    }
    void free_list(std::vector<void*>& list) {
        for (void* p : list) vlb_free(h, p);
        list.clear();
    }
    // Receive side for `rows` group rows (received pairs + this rank's own rows for the shared
    // expert): the group layer's workspace and the row buffers, regrown with headroom.
    int reserve(uint32_t rows) {
        if (rows <= capacity) return VLB_OK;
        const uint32_t cap = (uint32_t)((uint64_t)rows * 5 / 4 + 16);
        if (group) {
            vlb_layer_destroy(h, group);
            group = nullptr;
        }
        free_list(group_owned);
        capacity = 0;
        vlb_moe_layer_desc d = group_desc;
        d.max_tokens = cap;
        int st = vlb_layer_create(h, &d, &group);
        if (st != VLB_OK) return handle_fail(h, st);
        const size_t hr = (size_t)cap * H;
        if (peer) group_rows = peer_rows;  // fixed: its peers write into it
        if ((!peer && (st = alloc(hr * 2, "vlb-ep-group-rows", (void**)&group_rows, group_owned))) ||
            (st = alloc((size_t)cap * 12, "vlb-ep-group-meta", (void**)&group_meta, group_owned)) ||
            (st = alloc(hr * 4, "vlb-ep-group-y", (void**)&group_y, group_owned)) ||
            (st = alloc(hr * 2, "vlb-ep-group-yh", (void**)&group_yh, group_owned)) ||
            (st = alloc((size_t)cap * 4, "vlb-ep-group-ys", (void**)&group_ys, group_owned)))
            return st;
        capacity = cap;
        return VLB_OK;
    }
    void release() {
        for (void* q : ipc_opened) cudaIpcCloseMemHandle(q);
        ipc_opened.clear();
        if (group) vlb_layer_destroy(h, group);
        group = nullptr;
        free_list(group_owned);
        free_list(owned);
        if (offsets_host) cudaFreeHost(offsets_host);
        if (counts_host) cudaFreeHost(counts_host);
        offsets_host = nullptr;
        counts_host = nullptr;
        if (sync_ev) cudaEventDestroy(sync_ev);
        for (cudaEvent_t& e : phase)
            if (e) cudaEventDestroy(e);
    }
};

namespace {

// One grouped exchange: to every peer p, send_count[p] rows of `row_bytes` from `send` (rows in
// peer order), from every peer recv_count[p] rows into `recv`; zero counts are skipped on both
// sides (the counts were exchanged, so both ends agree).
int exchange_rows(vlb_ep_comm* c, const void* send, const uint64_t* send_count, void* recv,
                  const uint64_t* recv_count, size_t row_bytes, cudaStream_t s, const char* what) {
    const NcclApi& n = nccl();
    ncclResult_t r = n.GroupStart();
    if (r != ncclSuccess) return c->abort_with(VLB_ERR_IO_ERROR, std::string(what) + ": " + nccl_msg("ncclGroupStart", r));
    size_t so = 0, ro = 0;
    for (int p = 0; p < c->world && r == ncclSuccess; ++p) {
        const size_t sb = send_count[p] * row_bytes, rb = recv_count[p] * row_bytes;
        if (sb) r = n.Send(static_cast<const char*>(send) + so, sb, ncclUint8, p, c->comm, s);
        if (r == ncclSuccess && rb) r = n.Recv(static_cast<char*>(recv) + ro, rb, ncclUint8, p, c->comm, s);
        so += sb;
        ro += rb;
    }
    ncclResult_t e = n.GroupEnd();
    if (r != ncclSuccess && r != ncclInProgress) return c->abort_with(VLB_ERR_IO_ERROR, std::string(what) + ": " + nccl_msg("ncclSend/ncclRecv", r));
    if (e != ncclSuccess && e != ncclInProgress) return c->abort_with(VLB_ERR_IO_ERROR, std::string(what) + ": " + nccl_msg("ncclGroupEnd", e));
    return c->settle(what);
}

// ---- peer-store exchange --------------------------------------------------------------------
constexpr uint32_t kPeerMaxRanks = 16;
struct PeerSegs {
    const uint4* src[kPeerMaxRanks];
    uint4* dst[kPeerMaxRanks];
    uint64_t n16[kPeerMaxRanks];
    uint32_t count;
};

// Copies every segment (local source, a peer's mapped memory or this GPU's as destination), all
// CTAs striding over one segment after another, four 16-byte loads in flight per thread; the
// stores are made visible system-wide before the kernel ends.
__global__ void __launch_bounds__(256) peer_copy_kernel(PeerSegs g) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint32_t sgi = 0; sgi < g.count; ++sgi) {
        const uint4* __restrict__ src = g.src[sgi];
        uint4* dst = g.dst[sgi];
        const uint64_t n = g.n16[sgi];
        uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
        for (; i + 3u * stride < n; i += 4u * stride) {
            const uint4 a = src[i], b = src[i + stride], c = src[i + 2u * stride], d = src[i + 3u * stride];
            dst[i] = a;
            dst[i + stride] = b;
            dst[i + 2u * stride] = c;
            dst[i + 3u * stride] = d;
        }
        for (; i < n; i += stride) dst[i] = src[i];
    }
    __threadfence_system();
}

int launch_peer_copy(const PeerSegs& g, cudaStream_t s) {
    bool any = false;
    for (uint32_t i = 0; i < g.count; ++i) any = any || g.n16[i] != 0;
    if (!any) return VLB_OK;
    int sms = 148;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    peer_copy_kernel<<<(unsigned)sms * 4u, 256, 0, s>>>(g);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? VLB_OK : fail(VLB_ERR_IO_ERROR, cuda_msg("peer_copy_kernel", e));
}

// Maps every peer's receive buffers (CUDA IPC handles exchanged over the communicator) and agrees
// with every peer on using them: peer mode only if every rank mapped every peer. Collective: every
// rank of the communicator calls it at layer creation.
int enable_peer_exchange(vlb_ep_layer* l) {
    vlb_ep_comm* c = l->c;
    const uint32_t W = (uint32_t)c->world, me = (uint32_t)c->rank;
    const char* env = std::getenv("VLB_EP_EXCHANGE");
    bool want = W > 1 && W <= kPeerMaxRanks && !(env && std::string(env) == "nccl");
    // this rank's record: two IPC handles, the two capacities, and whether it wants peer mode
    struct Rec {
        cudaIpcMemHandle_t rows, back;
        uint64_t rows_cap, back_cap;
        uint64_t ok;
    };
    static_assert(sizeof(Rec) % 8 == 0, "record size");
    Rec mine{};
    const uint64_t n = (uint64_t)l->max_tokens * l->k;
    if (want) {
        l->peer_rows_cap = (uint64_t)W * n + l->max_tokens;
        void* p = nullptr;
        if (l->alloc(l->peer_rows_cap * l->H * 2, "vlb-ep-peer-rows", &p, l->owned) != VLB_OK) {
            want = false;
            l->peer_rows_cap = 0;
        } else {
            l->peer_rows = static_cast<uint16_t*>(p);
        }
    }
    if (want && (cudaIpcGetMemHandle(&mine.rows, l->peer_rows) != cudaSuccess ||
                 cudaIpcGetMemHandle(&mine.back, l->back_yh) != cudaSuccess)) {
        (void)cudaGetLastError();
        want = false;
    }
    mine.rows_cap = l->peer_rows_cap;
    mine.back_cap = n;
    mine.ok = want ? 1u : 0u;
    // everyone's record to everyone (the same record to every peer)
    std::vector<Rec> all(W), out(W, mine);
    void* dev_buf = nullptr;
    int st = l->alloc(sizeof(Rec) * W * 2, "vlb-ep-ipc", &dev_buf, l->owned);
    if (st != VLB_OK) return st;
    cudaStream_t s = static_cast<cudaStream_t>(vlb_stream(l->h));
    char* d = static_cast<char*>(dev_buf);
    cudaError_t ce = cudaMemcpyAsync(d, out.data(), sizeof(Rec) * W, cudaMemcpyHostToDevice, s);
    if (ce != cudaSuccess) return fail(VLB_ERR_IO_ERROR, cuda_msg("cudaMemcpyAsync(ipc records)", ce));
    std::vector<uint64_t> ones(W, sizeof(Rec));
    if ((st = exchange_rows(c, d, ones.data(), d + sizeof(Rec) * W, ones.data(), 1, s, "setup")) != VLB_OK) return st;
    ce = cudaMemcpyAsync(all.data(), d + sizeof(Rec) * W, sizeof(Rec) * W, cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess) ce = cudaEventRecord(l->sync_ev, s);
    if (ce != cudaSuccess) return fail(VLB_ERR_IO_ERROR, cuda_msg("ipc records", ce));
    if ((st = c->wait(l->sync_ev, "setup")) != VLB_OK) return st;
    bool every = true;
    for (uint32_t q = 0; q < W; ++q) every = every && all[q].ok;
    l->rows_at.assign(W, nullptr);
    l->back_at.assign(W, nullptr);
    l->rows_cap_at.assign(W, 0);
    l->back_cap_at.assign(W, 0);
    uint64_t mapped = 1;
    for (uint32_t q = 0; q < W && every; ++q) {
        l->rows_cap_at[q] = all[q].rows_cap;
        l->back_cap_at[q] = all[q].back_cap;
        if (q == me) {
            l->rows_at[q] = l->peer_rows;
            l->back_at[q] = l->back_yh;
            continue;
        }
        void* pr = nullptr;
        void* pb = nullptr;
        if (cudaIpcOpenMemHandle(&pr, all[q].rows, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            (void)cudaGetLastError();
            mapped = 0;
            break;
        }
        l->ipc_opened.push_back(pr);
        if (cudaIpcOpenMemHandle(&pb, all[q].back, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            (void)cudaGetLastError();
            mapped = 0;
            break;
        }
        l->ipc_opened.push_back(pb);
        l->rows_at[q] = static_cast<uint16_t*>(pr);
        l->back_at[q] = static_cast<uint16_t*>(pb);
    }
    if (!every) mapped = 0;
    // agree: peer mode only if every rank mapped every peer
    std::vector<uint64_t> flags(W, mapped), got(W, 0);
    uint64_t* fd = reinterpret_cast<uint64_t*>(d);
    ce = cudaMemcpyAsync(fd, flags.data(), 8 * W, cudaMemcpyHostToDevice, s);
    if (ce != cudaSuccess) return fail(VLB_ERR_IO_ERROR, cuda_msg("cudaMemcpyAsync(peer flags)", ce));
    std::vector<uint64_t> eights(W, 8);
    if ((st = exchange_rows(c, fd, eights.data(), fd + W, eights.data(), 1, s, "setup")) != VLB_OK) return st;
    ce = cudaMemcpyAsync(got.data(), fd + W, 8 * W, cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess) ce = cudaEventRecord(l->sync_ev, s);
    if (ce != cudaSuccess) return fail(VLB_ERR_IO_ERROR, cuda_msg("peer flags", ce));
    if ((st = c->wait(l->sync_ev, "setup")) != VLB_OK) return st;
    bool all_mapped = true;
    for (uint32_t q = 0; q < W; ++q) all_mapped = all_mapped && got[q] == 1;
    if (!all_mapped) {
        for (void* q : l->ipc_opened) cudaIpcCloseMemHandle(q);
        l->ipc_opened.clear();
        l->rows_at.clear();
        l->back_at.clear();
        return VLB_OK;  // NCCL carries the rows
    }
    l->peer = true;
    return VLB_OK;
}

int layer_refuse(vlb_ep_layer* l) {
    return fail(VLB_ERR_IO_ERROR, "an earlier exchange (" + l->failed +
                                      ") of this expert-parallel layer failed; rebuild the communicator and the layer");
}

}  // namespace

extern "C" {

int vlb_ep_nccl_version(int* version) {
    const NcclApi& n = nccl();
    if (!n.ok) return fail(VLB_ERR_UNSUPPORTED, n.why);
    if (version) *version = n.version;
    return VLB_OK;
}

int vlb_ep_unique_id(uint8_t* id) {
    const NcclApi& n = nccl();
    if (!n.ok) return fail(VLB_ERR_UNSUPPORTED, n.why);
    if (!id) return fail(VLB_ERR_INVALID_ARGUMENT, "null unique id buffer");
    static_assert(sizeof(ncclUniqueId) == VLB_EP_UNIQUE_ID_BYTES, "ncclUniqueId size");
    ncclUniqueId u;
    ncclResult_t r = n.GetUniqueId(&u);
    if (r != ncclSuccess) return fail(VLB_ERR_IO_ERROR, nccl_msg("ncclGetUniqueId", r));
    std::memcpy(id, &u, sizeof(u));
    return VLB_OK;
}

int vlb_ep_comm_init(vlb_handle* h, const uint8_t* id, int rank, int world, uint32_t timeout_ms,
                     vlb_ep_comm** out) {
    const NcclApi& n = nccl();
    if (!n.ok) return fail(VLB_ERR_UNSUPPORTED, n.why);
    if (!h || !id || !out || world < 1 || rank < 0 || rank >= world || timeout_ms == 0)
        return fail(VLB_ERR_INVALID_ARGUMENT, "invalid expert-parallel communicator argument");
    *out = nullptr;
    // the communicator binds to the current device: make it the handle's for the set-up
    int dev = 0, prev = 0;
    cudaError_t ce = cudaStreamGetDevice(static_cast<cudaStream_t>(vlb_stream(h)), &dev);
    if (ce == cudaSuccess) ce = cudaGetDevice(&prev);
    if (ce == cudaSuccess) ce = cudaSetDevice(dev);
    if (ce != cudaSuccess) return fail(VLB_ERR_IO_ERROR, cuda_msg("selecting the handle's device", ce));
    vlb_ep_comm* c = new (std::nothrow) vlb_ep_comm();
    if (!c) return fail(VLB_ERR_RESOURCE_EXHAUSTED, "unable to allocate the communicator record");
    c->h = h;
    c->device = dev;
    c->rank = rank;
    c->world = world;
    c->timeout_ms = timeout_ms;
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // every wait on it is the driver's own, bounded one
    ncclResult_t r = n.CommInitRankConfig(&c->comm, world, u, rank, &cfg);
    int st = VLB_OK;
    if (r != ncclSuccess && r != ncclInProgress) {
        st = fail(VLB_ERR_IO_ERROR, nccl_msg("ncclCommInitRankConfig", r));
        if (c->comm) n.CommAbort(c->comm);
        c->comm = nullptr;
    } else {
        st = c->settle("communicator set-up");
    }
    cudaSetDevice(prev);
    if (st != VLB_OK) {
        delete c;
        return st;
    }
    *out = c;
    return VLB_OK;
}

int vlb_ep_comm_destroy(vlb_ep_comm* c) {
    if (!c) return VLB_OK;
    int st = VLB_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    if (c->comm && !c->aborted) {
        // finalize flushes the communicator's outstanding work (bounded), then destroy frees it
        ncclResult_t r = nccl().CommFinalize(c->comm);
        if (r == ncclSuccess || r == ncclInProgress) st = c->settle("communicator finalize");
        else st = c->abort_with(VLB_ERR_IO_ERROR, nccl_msg("ncclCommFinalize", r));
        if (!c->aborted) nccl().CommDestroy(c->comm);
    }
    cudaSetDevice(prev);
    delete c;
    return st;
}

int vlb_ep_comm_abort(vlb_ep_comm* c) {
    if (!c) return fail(VLB_ERR_INVALID_ARGUMENT, "null communicator");
    c->abort_with(VLB_ERR_IO_ERROR, "communicator aborted by its caller");
    return VLB_OK;
}

int vlb_ep_all_to_all_device(vlb_ep_comm* c, const void* send_dev, const uint64_t* send_bytes, void* recv_dev,
                             const uint64_t* recv_bytes, void* stream) {
    if (!c || !send_bytes || !recv_bytes) return fail(VLB_ERR_INVALID_ARGUMENT, "invalid all-to-all argument");
    if (c->aborted) return fail(VLB_ERR_IO_ERROR, "the communicator was aborted");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : static_cast<cudaStream_t>(vlb_stream(c->h));
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    int st = exchange_rows(c, send_dev, send_bytes, recv_dev, recv_bytes, 1, s, "all-to-all");
    cudaSetDevice(prev);
    return st;
}

int vlb_ep_layer_create(vlb_handle* h, vlb_ep_comm* c, const vlb_ep_layer_desc* d, vlb_ep_layer** out) {
    if (!h || !c || !d || !out) return fail(VLB_ERR_INVALID_ARGUMENT, "null expert-parallel layer argument");
    *out = nullptr;
    if (c->h != h) return fail(VLB_ERR_INVALID_ARGUMENT, "the communicator belongs to another handle");
    const uint32_t W = (uint32_t)c->world;
    if (d->experts == 0 || d->experts % W || d->experts > 512 || d->top_k == 0 || d->top_k > 16 ||
        d->top_k > d->experts || d->hidden == 0 || d->hidden % 256 || d->intermediate == 0 ||
        d->intermediate % 256 || d->max_tokens == 0 || !d->w1 || !d->w3 || !d->w2)
        return fail(VLB_ERR_INVALID_ARGUMENT, "expert-parallel layer dimensions are invalid");
    if (d->score < VLB_SCORE_SQRT_SOFTPLUS || d->score > VLB_SCORE_SOFTMAX_F64_NORM)
        return fail(VLB_ERR_INVALID_ARGUMENT, "unknown router score mode");
    if (d->routed_swiglu_limit != d->shared_swiglu_limit)
        return fail(VLB_ERR_UNSUPPORTED,
                    "the expert group applies one SwiGLU limit to the routed and the shared expert");
    vlb_ep_layer* l = new (std::nothrow) vlb_ep_layer();
    if (!l) return fail(VLB_ERR_RESOURCE_EXHAUSTED, "unable to allocate the expert-parallel layer");
    l->h = h;
    l->c = c;
    l->H = d->hidden;
    l->I = d->intermediate;
    l->E = d->experts;
    l->k = d->top_k;
    l->epr = d->experts / W;
    l->max_tokens = d->max_tokens;
    l->score = d->score;
    l->route_scale = d->route_scale;
    const uint32_t el = l->epr + 1;  // this rank's routed experts, then the shared expert
    for (uint32_t e = 0; e < el; ++e) {
        if (!d->w1[e] || !d->w3[e] || !d->w2[e]) {
            delete l;
            return fail(VLB_ERR_INVALID_ARGUMENT, "an expert matrix of this rank is missing");
        }
        l->w1.push_back(d->w1[e]);
        l->w3.push_back(d->w3[e]);
        l->w2.push_back(d->w2[e]);
    }
    l->zero_router.assign((size_t)el * l->H, 0.f);
    vlb_moe_layer_desc& g = l->group_desc;
    g.hidden = l->H;
    g.intermediate = l->I;
    g.experts = el;
    g.top_k = 1;
    g.score = d->score;
    g.hash_routing = 0;
    g.weight_after_down = d->weight_after_down;
    g.route_scale = 1.f;
    g.routed_swiglu_limit = d->routed_swiglu_limit;
    g.shared_swiglu_limit = d->shared_swiglu_limit;
    g.router = l->zero_router.data();  // the group forward takes its routes from the rows' meta words
    g.w1 = l->w1.data();
    g.w3 = l->w3.data();
    g.w2 = l->w2.data();

    const size_t T = d->max_tokens, n = T * d->top_k, Hs = l->H;
    int st = VLB_OK;
    auto& o = l->owned;
    if ((st = l->alloc(n * 4, "vlb-ep-idx", (void**)&l->idx, o)) || (st = l->alloc(n * 4, "vlb-ep-w", (void**)&l->w, o)) ||
        (st = l->alloc(((size_t)l->E + 2) * 4, "vlb-ep-offsets", (void**)&l->offsets, o)) ||
        (st = l->alloc(vlb_ep_workspace_bytes((uint32_t)T, l->k, l->E), "vlb-ep-plan", &l->ws, o)) ||
        (st = l->alloc(n * Hs * 2, "vlb-ep-send-rows", (void**)&l->send_rows, o)) ||
        (st = l->alloc(n * 12, "vlb-ep-send-meta", (void**)&l->send_meta, o)) ||
        (st = l->alloc(n * 4, "vlb-ep-elem-row", (void**)&l->elem_row, o)) ||
        (st = l->alloc(T * Hs * 2, "vlb-ep-own-rows", (void**)&l->own_rows, o)) ||
        (st = l->alloc(T * 12, "vlb-ep-own-meta", (void**)&l->own_meta, o)) ||
        (st = l->alloc((size_t)W * W * 16 + (size_t)W * 16, "vlb-ep-counts", (void**)&l->counts_dev, o)) ||
        (st = l->alloc(n * Hs * 2, "vlb-ep-back-rows", (void**)&l->back_yh, o)) ||
        (st = l->alloc(n * 4, "vlb-ep-back-scales", (void**)&l->back_ys, o))) {
        l->release();
        delete l;
        return st;
    }
    if (d->bias) {
        if ((st = l->alloc((size_t)l->E * 4, "vlb-ep-bias", (void**)&l->bias, o)) ||
            (st = vlb_memcpy_h2d(h, l->bias, d->bias, (size_t)l->E * 4))) {
            if (st) handle_fail(h, st);
            l->release();
            delete l;
            return st;
        }
    }
    if (d->expert_slot) {
        std::vector<uint8_t> seen(l->E, 0);
        for (uint32_t e = 0; e < l->E; ++e) {
            if (d->expert_slot[e] >= l->E || seen[d->expert_slot[e]]) {
                l->release();
                delete l;
                return fail(VLB_ERR_INVALID_ARGUMENT, "expert_slot is not a permutation of the experts");
            }
            seen[d->expert_slot[e]] = 1;
        }
        if ((st = l->alloc((size_t)l->E * 4, "vlb-ep-slots", (void**)&l->slots, o)) ||
            (st = vlb_memcpy_h2d(h, l->slots, d->expert_slot, (size_t)l->E * 4))) {
            if (st) handle_fail(h, st);
            l->release();
            delete l;
            return st;
        }
    }
    cudaError_t ce = cudaHostAlloc((void**)&l->offsets_host, ((size_t)l->E + 1) * 4, cudaHostAllocDefault);
    if (ce == cudaSuccess) ce = cudaHostAlloc((void**)&l->counts_host, (size_t)W * 16 + (size_t)W * W * 8, cudaHostAllocDefault);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&l->sync_ev, cudaEventDisableTiming);
    for (int i = 0; i < 6 && ce == cudaSuccess; ++i) ce = cudaEventCreate(&l->phase[i]);
    if (ce != cudaSuccess) {
        l->release();
        delete l;
        return fail(VLB_ERR_IO_ERROR, cuda_msg("expert-parallel host buffers", ce));
    }
    if ((st = enable_peer_exchange(l)) != VLB_OK) {
        l->release();
        delete l;
        return st;
    }
    // receive side sized for the balanced load with headroom; a heavier step regrows it
    st = l->reserve((uint32_t)((n + W - 1) / W + T));
    if (st != VLB_OK) {
        l->release();
        delete l;
        return st;
    }
    *out = l;
    return VLB_OK;
}

int vlb_ep_layer_destroy(vlb_handle* h, vlb_ep_layer* l) {
    if (!l) return VLB_OK;
    if (l->h != h) return fail(VLB_ERR_INVALID_ARGUMENT, "the layer belongs to another handle");
    vlb_synchronize(h);
    l->release();
    delete l;
    return VLB_OK;
}

int vlb_ep_forward_device(vlb_handle* h, vlb_ep_layer* l, const float* x, const float* logits, uint32_t T,
                          float* out, void* stream) {
    if (!h || !l || l->h != h || !x || !logits || !out)
        return fail(VLB_ERR_INVALID_ARGUMENT, "invalid expert-parallel forward argument");
    if (T > l->max_tokens) return fail(VLB_ERR_INVALID_ARGUMENT, "more tokens than the layer was sized for");
    if (!l->failed.empty()) return layer_refuse(l);
    vlb_ep_comm* c = l->c;
    if (c->aborted) {
        l->failed = "communicator";
        return layer_refuse(l);
    }
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : static_cast<cudaStream_t>(vlb_stream(h));
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    struct Restore {
        int d;
        ~Restore() { cudaSetDevice(d); }
    } restore{prev};
    const uint32_t W = (uint32_t)c->world, k = l->k, H = l->H, epr = l->epr;
    const size_t n = (size_t)T * k;
    l->have_phases = false;
    int st;
    cudaEventRecord(l->phase[0], s);
    // route and plan (the plan synchronises once: its offsets size the exchange)
    if ((st = vlb_route_device(h, l->score, 0, logits, l->bias, nullptr, nullptr, 0, T, l->E, k, l->route_scale,
                               l->idx, l->w, s)) != VLB_OK)
        return handle_fail(h, st);
    if ((st = vlb_ep_plan_half_device(h, l->idx, l->w, T, k, l->E, epr, l->slots, x, H, l->ws, l->offsets,
                                      l->offsets_host, l->send_rows, l->send_meta, l->elem_row, l->own_rows,
                                      l->own_meta, s)) != VLB_OK)
        return handle_fail(h, st);
    uint64_t* send_count = l->counts_host;
    uint64_t* recv_count = l->counts_host + W;
    for (uint32_t p = 0; p < W; ++p)
        send_count[p] = (uint64_t)l->offsets_host[(p + 1) * epr] - l->offsets_host[p * epr];
    // counts: one u64 to and from every rank; in peer mode every rank's whole send-count vector
    // to every rank (matrix[q][p] = rows rank q sends rank p), which gives each rank its offsets
    // in every peer's receive buffers
    uint64_t* matrix = l->counts_host + 2 * W;
    cudaError_t ce = cudaSuccess;
    if (l->peer) {
        for (uint32_t p = 0; p < W; ++p) std::memcpy(matrix + (size_t)p * W, send_count, (size_t)W * 8);
        ce = cudaMemcpyAsync(l->counts_dev, matrix, (size_t)W * W * 8, cudaMemcpyHostToDevice, s);
    } else {
        ce = cudaMemcpyAsync(l->counts_dev, send_count, (size_t)W * 8, cudaMemcpyHostToDevice, s);
    }
    if (ce != cudaSuccess) return fail(VLB_ERR_IO_ERROR, cuda_msg("cudaMemcpyAsync(counts)", ce));
    {
        const uint64_t per = l->peer ? (uint64_t)W * 8 : 8;
        std::vector<uint64_t> sizes(W, per);
        st = exchange_rows(c, l->counts_dev, sizes.data(), l->counts_dev + (size_t)W * (per / 8), sizes.data(), 1, s,
                           "counts");
        if (st == VLB_OK) {
            ce = cudaMemcpyAsync(l->peer ? matrix : recv_count, l->counts_dev + (size_t)W * (per / 8),
                                 (size_t)W * per, cudaMemcpyDeviceToHost, s);
            if (ce == cudaSuccess) ce = cudaEventRecord(l->sync_ev, s);
            st = ce != cudaSuccess ? fail(VLB_ERR_IO_ERROR, cuda_msg("cudaMemcpyAsync(counts)", ce))
                                   : c->wait(l->sync_ev, "counts");
        }
    }
    if (st != VLB_OK) {
        l->failed = "counts";
        return st;
    }
    if (l->peer) {
        for (uint32_t q = 0; q < W; ++q) recv_count[q] = matrix[(size_t)q * W + (uint32_t)c->rank];
        if (matrix[(size_t)c->rank * W + 0] != send_count[0]) {
            l->failed = "counts";
            return fail(VLB_ERR_INTERNAL_ERROR, "counts: the exchanged count matrix does not hold this rank's own row");
        }
    }
    uint64_t R = 0;
    for (uint32_t p = 0; p < W; ++p) R += recv_count[p];
    if (R + T > 0xffffffffull || (l->peer && R + T > l->peer_rows_cap)) {
        l->failed = "counts";
        return fail(VLB_ERR_RESOURCE_EXHAUSTED, "too many received rows");
    }
    if ((st = l->reserve((uint32_t)(R + T))) != VLB_OK) return st;
    cudaEventRecord(l->phase[1], s);
    // dispatch: fp16 rows (peer stores, or NCCL), then their meta words (NCCL; in peer mode also
    // the fence that makes the stored rows safe to read on every receiver)
    const uint32_t me = (uint32_t)c->rank;
    if (l->peer) {
        PeerSegs g{};
        g.count = W;
        uint64_t so = 0;
        for (uint32_t p = 0; p < W; ++p) {
            uint64_t off = 0;  // rows of ranks before this one in p's receive buffer
            for (uint32_t q = 0; q < me; ++q) off += matrix[(size_t)q * W + p];
            if (off + send_count[p] > l->rows_cap_at[p]) {
                l->failed = "dispatch";
                return fail(VLB_ERR_RESOURCE_EXHAUSTED, "dispatch: a peer's receive buffer is too small for this step");
            }
            g.src[p] = reinterpret_cast<const uint4*>(l->send_rows + so * H);
            g.dst[p] = reinterpret_cast<uint4*>(l->rows_at[p] + off * H);
            g.n16[p] = send_count[p] * H * 2 / 16;
            so += send_count[p];
        }
        st = launch_peer_copy(g, s);
    } else {
        st = exchange_rows(c, l->send_rows, send_count, l->group_rows, recv_count, (size_t)H * 2, s, "dispatch");
    }
    if (st == VLB_OK)
        st = exchange_rows(c, l->send_meta, send_count, l->group_meta, recv_count, 12, s, "dispatch");
    if (st != VLB_OK) {
        l->failed = "dispatch";
        return st;
    }
    // this rank's own tokens for its shared expert (local expert epr) after the received rows
    ce = cudaMemcpyAsync(l->group_rows + R * H, l->own_rows, (size_t)T * H * 2, cudaMemcpyDeviceToDevice, s);
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(l->group_meta + R * 3, l->own_meta, (size_t)T * 12, cudaMemcpyDeviceToDevice, s);
    if (ce != cudaSuccess) return fail(VLB_ERR_IO_ERROR, cuda_msg("cudaMemcpyAsync(own rows)", ce));
    cudaEventRecord(l->phase[2], s);
    if ((st = vlb_layer_forward_rows_half_device(h, l->group, l->group_rows, l->group_meta, (uint32_t)(R + T),
                                                 l->group_y, s)) != VLB_OK)
        return handle_fail(h, st);
    cudaEventRecord(l->phase[3], s);
    // results back as fp16 rows with a power-of-two scale each
    if ((st = vlb_ep_pack_half_device(h, l->group_y, (uint32_t)R, H, l->group_yh, l->group_ys, s)) != VLB_OK)
        return handle_fail(h, st);
    if (l->peer) {
        // the results of rank q's rows go back into q's results buffer after the rows q sent to
        // ranks before this one (q's send order)
        PeerSegs g{};
        g.count = W;
        uint64_t ro = 0;
        for (uint32_t q = 0; q < W; ++q) {
            uint64_t off = 0;
            for (uint32_t p = 0; p < me; ++p) off += matrix[(size_t)q * W + p];
            if (off + recv_count[q] > l->back_cap_at[q]) {
                l->failed = "return";
                return fail(VLB_ERR_RESOURCE_EXHAUSTED, "return: a peer's results buffer is too small for this step");
            }
            g.src[q] = reinterpret_cast<const uint4*>(l->group_yh + ro * H);
            g.dst[q] = reinterpret_cast<uint4*>(l->back_at[q] + off * H);
            g.n16[q] = recv_count[q] * H * 2 / 16;
            ro += recv_count[q];
        }
        st = launch_peer_copy(g, s);
    } else {
        st = exchange_rows(c, l->group_yh, recv_count, l->back_yh, send_count, (size_t)H * 2, s, "return");
    }
    if (st == VLB_OK) st = exchange_rows(c, l->group_ys, recv_count, l->back_ys, send_count, 4, s, "return");
    if (st != VLB_OK) {
        l->failed = "return";
        return st;
    }
    cudaEventRecord(l->phase[4], s);
    if ((st = vlb_ep_combine_half_device(h, l->back_yh, l->back_ys, l->elem_row, T, k, l->group_y + R * H, H, out,
                                         s)) != VLB_OK)
        return handle_fail(h, st);
    cudaEventRecord(l->phase[5], s);
    // end of step: the exchanges completed (bounded wait), then the group forward's error bits
    cudaEventRecord(l->sync_ev, s);
    if ((st = c->wait(l->sync_ev, "return")) != VLB_OK) {
        l->failed = "return";
        return st;
    }
    if ((st = vlb_layer_status(h, l->group, s)) != VLB_OK) return handle_fail(h, st);
    l->have_phases = true;
    l->last_rows[0] = R;
    l->last_rows[1] = n;
    return VLB_OK;
}

int vlb_ep_last_phases(vlb_ep_layer* l, float* ms, uint64_t* rows) {
    if (!l || !ms) return fail(VLB_ERR_INVALID_ARGUMENT, "invalid phase query");
    if (!l->have_phases) return fail(VLB_ERR_NOT_FOUND, "no completed forward to report");
    for (int i = 0; i < 5; ++i) {
        cudaError_t e = cudaEventElapsedTime(&ms[i], l->phase[i], l->phase[i + 1]);
        if (e != cudaSuccess) return fail(VLB_ERR_IO_ERROR, cuda_msg("cudaEventElapsedTime", e));
    }
    if (rows) {
        rows[0] = l->last_rows[0];
        rows[1] = l->last_rows[1];
    }
    return VLB_OK;
}

}  // extern "C"
