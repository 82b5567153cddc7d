// Tensor-parallel plumbing: an NCCL communicator (libnccl.so.2 is opened at run time,
// so the library loads on machines without NCCL and only the TP entry points need it)
// and the host-side sharding of packed GGUF tensors.  The reference runs on one GPU;
// the partitioning follows the Megatron split of a Llama layer: q/k/v and gate/up rows
// by head / FFN column, o_proj and down input columns on block boundaries, the output
// head by vocabulary rows.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <chrono>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "comm.cuh"
#include "common.cuh"

namespace ib {

namespace {

struct Nccl {
    void* so = nullptr;
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
    decltype(&ncclCommGetAsyncError) get_async_error = nullptr;
    decltype(&ncclCommAbort) abort = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};

int nccl_load(Nccl** out) {
    static Nccl n;
    static std::once_flag once;
    static std::string err;
    std::call_once(once, [] {
        n.so = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!n.so) {
            err = std::string("NCCL: cannot open libnccl.so.2: ") + dlerror();
            return;
        }
        n.get_unique_id = (decltype(n.get_unique_id))dlsym(n.so, "ncclGetUniqueId");
        n.init_rank_config = (decltype(n.init_rank_config))dlsym(n.so, "ncclCommInitRankConfig");
        n.get_async_error = (decltype(n.get_async_error))dlsym(n.so, "ncclCommGetAsyncError");
        n.abort = (decltype(n.abort))dlsym(n.so, "ncclCommAbort");
        n.all_reduce = (decltype(n.all_reduce))dlsym(n.so, "ncclAllReduce");
        n.all_gather = (decltype(n.all_gather))dlsym(n.so, "ncclAllGather");
        n.destroy = (decltype(n.destroy))dlsym(n.so, "ncclCommDestroy");
        n.error_string = (decltype(n.error_string))dlsym(n.so, "ncclGetErrorString");
        if (!n.get_unique_id || !n.init_rank_config || !n.get_async_error || !n.abort ||
            !n.all_reduce || !n.all_gather || !n.destroy || !n.error_string)
            err = "NCCL: libnccl.so.2 lacks an expected symbol";
    });
    if (!err.empty()) {
        set_error(err);
        return IB_ERR_COMM;
    }
    *out = &n;
    return IB_OK;
}

using Clock = std::chrono::steady_clock;

long long ms_since(Clock::time_point t0) {
    return std::chrono::duration_cast<std::chrono::milliseconds>(Clock::now() - t0).count();
}

}  // namespace

// A communicator in NCCL's non-blocking mode: every call returns at once, and a call
// that reports ncclInProgress is polled (ncclCommGetAsyncError) until it settles or the
// communicator's deadline passes.  A failed or expired call aborts the communicator
// (ncclCommAbort also ends NCCL kernels waiting for a rank that never comes), after
// which every call on it fails at once.
struct Comm {
    ncclComm_t nc = nullptr;
    int rank = 0, world = 1, device = 0;
    long long timeout_ms = IB_COMM_DEFAULT_TIMEOUT_MS;
    bool failed = false;
};

namespace {

void comm_abort(Nccl* n, Comm* c) {
    if (c->nc) n->abort(c->nc);
    c->nc = nullptr;
    c->failed = true;
}

// Settles a non-blocking NCCL call's result r (see Comm).
int nccl_settle(Nccl* n, Comm* c, ncclResult_t r, const char* what) {
    const Clock::time_point t0 = Clock::now();
    int spins = 0;
    while (r == ncclInProgress) {
        if (ms_since(t0) > c->timeout_ms) {
            comm_abort(n, c);
            set_error(std::string("NCCL: ") + what + " did not complete within " +
                      std::to_string(c->timeout_ms) + " ms (a rank did not join); communicator aborted");
            return IB_ERR_TIMEOUT;
        }
        if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(200));
        ncclResult_t st = ncclSuccess;
        const ncclResult_t q = n->get_async_error(c->nc, &st);
        r = q != ncclSuccess ? q : st;
    }
    if (r != ncclSuccess) {
        const std::string msg = n->error_string(r);
        comm_abort(n, c);
        set_error(std::string("NCCL: ") + what + " failed: " + msg + "; communicator aborted");
        return IB_ERR_COMM;
    }
    return IB_OK;
}

int comm_usable(Comm* c, Nccl** n) {
    int r = nccl_load(n);
    if (r) return r;
    if (c->failed) {
        set_error("NCCL: the communicator was aborted after an earlier failure");
        return IB_ERR_COMM;
    }
    return IB_OK;
}

// Waits for `st` with the communicator's deadline; on expiry aborts the communicator
// (its kernels then return) and reports IB_ERR_TIMEOUT.
int stream_settle(Nccl* n, Comm* c, cudaStream_t st, const char* what) {
    const Clock::time_point t0 = Clock::now();
    int spins = 0;
    for (;;) {
        const cudaError_t e = cudaStreamQuery(st);
        if (e == cudaSuccess) return IB_OK;
        if (e != cudaErrorNotReady) {
            set_error(std::string(what) + ": " + cudaGetErrorString(e));
            return IB_ERR_CUDA;
        }
        if (ms_since(t0) > c->timeout_ms) {
            comm_abort(n, c);
            set_error(std::string(what) + " did not complete within " +
                      std::to_string(c->timeout_ms) + " ms; communicator aborted");
            return IB_ERR_TIMEOUT;
        }
        if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

}  // namespace

int comm_rank(const Comm* c) { return c ? c->rank : 0; }
int comm_world(const Comm* c) { return c ? c->world : 1; }

int comm_allreduce_sum_f32(Comm* c, float* buf, size_t n, cudaStream_t st) {
    if (!c || c->world == 1 || n == 0) return IB_OK;
    Nccl* nc;
    int r = comm_usable(c, &nc);
    if (r) return r;
    return nccl_settle(nc, c, nc->all_reduce(buf, buf, n, ncclFloat32, ncclSum, c->nc, st),
                       "ncclAllReduce");
}

int comm_allreduce_max_u64(Comm* c, unsigned long long* buf, size_t n, cudaStream_t st) {
    if (!c || c->world == 1 || n == 0) return IB_OK;
    Nccl* nc;
    int r = comm_usable(c, &nc);
    if (r) return r;
    return nccl_settle(nc, c, nc->all_reduce(buf, buf, n, ncclUint64, ncclMax, c->nc, st),
                       "ncclAllReduce");
}

// ---- peer memory set-up: every rank fails together or none does ----------------------
// Round 1: every rank exports its buffer (status, IPC handle) and all records are
// gathered, so a rank whose allocation or export failed -- or that arrives with a
// failure from earlier in its set-up -- is seen by all.  Round 2: every rank maps the
// others' buffers and the map statuses are gathered; any failure releases every
// mapping on every rank.  Each rank joins both gathers whatever happened locally, so no
// rank is left waiting in a collective.
int peer_setup(int rank, int world, void* local, int local_status, const PeerIpc& ipc,
               const PeerGather& gather, void** peers) {
    for (int q = 0; q < world; ++q) peers[q] = nullptr;
    struct Rec {
        int32_t status;  // 0 ok, 1 failed before the set-up, 2 export failed
        uint8_t handle[kPeerHandleBytes];
    };
    Rec mine = {};
    mine.status = local_status != 0 ? 1 : 0;
    std::string export_err;
    if (mine.status == 0 && ipc.handle(ipc.ctx, local, mine.handle, kPeerHandleBytes, &export_err))
        mine.status = 2;
    std::vector<Rec> all(world);
    int r = gather.all(gather.ctx, (const uint8_t*)&mine, (uint8_t*)all.data(), sizeof(Rec));
    if (r) return r;  // the gather's failure ends every rank's gather (aborted or timed out)
    for (int q = 0; q < world; ++q) {
        if (all[q].status == 0) continue;
        if (q == rank && mine.status == 1) return local_status;  // keep the local message
        if (q == rank) {
            set_error("peer memory: cannot export this rank's buffer: " + export_err);
        } else {
            set_error("peer memory: rank " + std::to_string(q) +
                      (all[q].status == 1 ? " failed before the peer set-up"
                                          : " could not export its buffer") +
                      "; every rank stops");
        }
        return IB_ERR_COMM;
    }
    // round 2
    int32_t map_status = 0;  // 0 ok, else 1 + the first peer that could not be mapped
    std::string map_err;
    for (int q = 0; q < world && map_status == 0; ++q) {
        if (q == rank) continue;
        if (ipc.open(ipc.ctx, q, all[q].handle, kPeerHandleBytes, &peers[q], &map_err)) {
            peers[q] = nullptr;
            map_status = 1 + q;
        }
    }
    std::vector<int32_t> maps(world);
    r = gather.all(gather.ctx, (const uint8_t*)&map_status, (uint8_t*)maps.data(), 4);
    int bad = -1;
    for (int q = 0; q < world && r == IB_OK; ++q)
        if (maps[q] != 0 && bad < 0) bad = q;
    if (r == IB_OK && bad < 0) {
        peers[rank] = local;
        return IB_OK;
    }
    for (int q = 0; q < world; ++q) {
        if (peers[q] && q != rank) ipc.close(ipc.ctx, peers[q]);
        peers[q] = nullptr;
    }
    if (r) return r;
    if (bad == rank)
        set_error("peer memory: cannot map rank " + std::to_string(maps[bad] - 1) +
                  "'s buffer: " + map_err);
    else
        set_error("peer memory: rank " + std::to_string(bad) + " could not map rank " +
                  std::to_string(maps[bad] - 1) + "'s buffer; every rank stops");
    return IB_ERR_COMM;
}

namespace {

// CUDA IPC and an NCCL all-gather: the production layers of the set-up above.
int cuda_handle(void*, void* local, uint8_t* out, size_t bytes, std::string* err) {
    static_assert(sizeof(cudaIpcMemHandle_t) <= kPeerHandleBytes, "IPC handle size");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, local);
    if (e != cudaSuccess) {
        *err = std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e);
        return 1;
    }
    memset(out, 0, bytes);
    memcpy(out, &h, sizeof(h));
    return 0;
}

int cuda_open(void*, int, const uint8_t* handle, size_t, void** ptr, std::string* err) {
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        *err = std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e);
        cudaGetLastError();
        return 1;
    }
    return 0;
}

void cuda_close(void*, void* ptr) { cudaIpcCloseMemHandle(ptr); }

int nccl_gather(void* ctx, const uint8_t* mine, uint8_t* all, size_t bytes) {
    Comm* c = (Comm*)ctx;
    Nccl* nc;
    int r = comm_usable(c, &nc);
    if (r) return r;
    const int W = c->world;
    uint8_t* dev = nullptr;
    cudaStream_t st = nullptr;
    IB_CUDA_CHECK(cudaMalloc(&dev, bytes * (W + 1)));
    cudaError_t e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dev + bytes * W, mine, bytes, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) {
        r = nccl_settle(nc, c, nc->all_gather(dev + bytes * W, dev, bytes, ncclUint8, c->nc, st),
                        "ncclAllGather (peer set-up)");
        if (r == IB_OK) r = stream_settle(nc, c, st, "peer set-up all-gather");
        if (r == IB_OK && cudaMemcpy(all, dev, bytes * W, cudaMemcpyDeviceToHost) != cudaSuccess) {
            set_error("peer set-up: copy of the gathered records failed");
            r = IB_ERR_CUDA;
        }
    } else {
        set_error(std::string("peer set-up: ") + cudaGetErrorString(e));
        r = IB_ERR_CUDA;
    }
    if (st) cudaStreamDestroy(st);
    cudaFree(dev);
    return r;
}

}  // namespace

int comm_peer_alloc(Comm* c, size_t bytes, int local_status, void** local, void** peers) {
    IB_REQUIRE(c && local && peers && bytes > 0, "bad peer allocation arguments");
    const int W = c->world;
    *local = nullptr;
    for (int q = 0; q < W; ++q) peers[q] = nullptr;
    int st = local_status;
    if (st == IB_OK) {
        cudaError_t e = cudaMalloc(local, bytes);
        if (e == cudaSuccess) e = cudaMemset(*local, 0, bytes);
        if (e != cudaSuccess) {
            set_error(std::string("peer memory: ") + cudaGetErrorString(e));
            st = IB_ERR_CUDA;
        }
    }
    if (W == 1) {
        if (st == IB_OK) peers[0] = *local;
    } else {
        const PeerIpc ipc{nullptr, cuda_handle, cuda_open, cuda_close};
        const PeerGather gather{c, nccl_gather};
        const int r = peer_setup(c->rank, W, *local, st, ipc, gather, peers);
        if (st == IB_OK) st = r;
    }
    if (st != IB_OK && *local) {
        cudaFree(*local);
        *local = nullptr;
    }
    return st;
}

void comm_peer_free(int world, void* local, void** peers) {
    const int W = world;
    for (int q = 0; q < W; ++q) {
        if (peers[q] && peers[q] != local) cudaIpcCloseMemHandle(peers[q]);
        peers[q] = nullptr;
    }
    if (local) cudaFree(local);
}

int comm_allgather_f32(Comm* c, const float* send, float* recv, size_t n_per_rank,
                       cudaStream_t st) {
    if (!c || c->world == 1) {
        if (send != recv)
            IB_CUDA_CHECK(cudaMemcpyAsync(recv, send, n_per_rank * 4, cudaMemcpyDeviceToDevice, st));
        return IB_OK;
    }
    Nccl* nc;
    int r = comm_usable(c, &nc);
    if (r) return r;
    return nccl_settle(nc, c, nc->all_gather(send, recv, n_per_rank, ncclFloat32, c->nc, st),
                       "ncclAllGather");
}

}  // namespace ib

using namespace ib;

extern "C" int ib_comm_unique_id(uint8_t* id128) {
    IB_REQUIRE(id128, "null pointer argument");
    Nccl* nc;
    int r = nccl_load(&nc);
    if (r) return r;
    ncclUniqueId id;
    if (nc->get_unique_id(&id) != ncclSuccess) {
        set_error("NCCL: ncclGetUniqueId failed");
        return IB_ERR_COMM;
    }
    memcpy(id128, id.internal, NCCL_UNIQUE_ID_BYTES);
    return IB_OK;
}

extern "C" int ib_comm_init_timeout(int rank, int world, const uint8_t* id128, int device,
                                    int64_t timeout_ms, void** comm) {
    IB_REQUIRE(comm && id128 && world >= 1 && rank >= 0 && rank < world && timeout_ms > 0,
               "bad communicator arguments");
    *comm = nullptr;
    Nccl* nc;
    int r = nccl_load(&nc);
    if (r) return r;
    IB_CUDA_CHECK(cudaSetDevice(device));
    ncclUniqueId id;
    memcpy(id.internal, id128, NCCL_UNIQUE_ID_BYTES);
    Comm* c = new Comm();
    c->rank = rank;
    c->world = world;
    c->device = device;
    c->timeout_ms = timeout_ms;
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    r = nccl_settle(nc, c, nc->init_rank_config(&c->nc, world, id, rank, &cfg), "ncclCommInitRankConfig");
    if (r) {
        delete c;
        return r;
    }
    *comm = c;
    return IB_OK;
}

extern "C" int ib_comm_init(int rank, int world, const uint8_t* id128, int device, void** comm) {
    return ib_comm_init_timeout(rank, world, id128, device, IB_COMM_DEFAULT_TIMEOUT_MS, comm);
}

extern "C" int ib_comm_allreduce_f32(void* comm, float* dev_buf, int64_t n, void* stream) {
    IB_REQUIRE(comm && dev_buf && n >= 0, "bad allreduce arguments");
    return comm_allreduce_sum_f32((Comm*)comm, dev_buf, (size_t)n, as_stream(stream));
}

extern "C" int ib_comm_abort(void* comm) {
    if (!comm) return IB_OK;
    Comm* c = (Comm*)comm;
    Nccl* nc;
    if (nccl_load(&nc) == IB_OK) comm_abort(nc, c);
    return IB_OK;
}

extern "C" int ib_comm_free(void* comm) {
    if (!comm) return IB_OK;
    Comm* c = (Comm*)comm;
    Nccl* nc;
    if (nccl_load(&nc) == IB_OK && c->nc) {
        // a communicator whose last call is still in progress cannot be destroyed
        // cleanly: abort it instead
        ncclResult_t st = ncclSuccess;
        if (nc->get_async_error(c->nc, &st) == ncclSuccess && st == ncclSuccess)
            nc->destroy(c->nc);
        else
            nc->abort(c->nc);
    }
    delete c;
    return IB_OK;
}

extern "C" int ib_comm_failed(void* comm, int* failed) {
    IB_REQUIRE(comm && failed, "null pointer argument");
    *failed = ((Comm*)comm)->failed ? 1 : 0;
    return IB_OK;
}

// Stand-in IPC layer for ib_peer_setup_check: a rank's "handle" is its rank number; the
// step `fail_step` (1 = export, 2 = map) fails on rank `fail_rank`; mappings are counted.
namespace {
struct FakeIpc {
    int rank, fail_rank, fail_step, opened, closed;
};
int fake_handle(void* ctx, void*, uint8_t* out, size_t bytes, std::string* err) {
    FakeIpc* f = (FakeIpc*)ctx;
    memset(out, 0, bytes);
    memcpy(out, &f->rank, 4);
    if (f->rank == f->fail_rank && f->fail_step == 1) {
        *err = "injected export failure";
        return 1;
    }
    return 0;
}
int fake_open(void* ctx, int peer, const uint8_t* handle, size_t, void** ptr, std::string* err) {
    FakeIpc* f = (FakeIpc*)ctx;
    int who = -1;
    memcpy(&who, handle, 4);
    if ((f->rank == f->fail_rank && f->fail_step == 2) || who != peer) {
        *err = who != peer ? "handle from the wrong rank" : "injected map failure";
        return 1;
    }
    ++f->opened;
    *ptr = (void*)(uintptr_t)(0x1000 + 16 * peer);
    return 0;
}
void fake_close(void* ctx, void*) { ++((FakeIpc*)ctx)->closed; }
struct HostGather {
    ib_gather_fn fn;
    void* ctx;
};
int host_gather(void* ctx, const uint8_t* mine, uint8_t* all, size_t bytes) {
    HostGather* g = (HostGather*)ctx;
    if (g->fn(g->ctx, mine, all, bytes) != 0) {
        set_error("peer set-up: the host all-gather failed");
        return IB_ERR_COMM;
    }
    return IB_OK;
}
}  // namespace

extern "C" int ib_peer_setup_check(int rank, int world, int local_status, int fail_rank,
                                   int fail_step, ib_gather_fn gather, void* gather_ctx,
                                   int* opened, int* closed) {
    IB_REQUIRE(gather && opened && closed && world >= 2 && world <= 64 && rank >= 0 &&
                   rank < world,
               "bad peer set-up check arguments");
    FakeIpc f{rank, fail_rank, fail_step, 0, 0};
    HostGather hg{gather, gather_ctx};
    const PeerIpc ipc{&f, fake_handle, fake_open, fake_close};
    const PeerGather pg{&hg, host_gather};
    std::vector<void*> peers(world, nullptr);
    if (local_status) set_error("injected local failure before the peer set-up");
    int dummy = 0;
    const int r = peer_setup(rank, world, &dummy, local_status, ipc, pg, peers.data());
    *opened = f.opened;
    *closed = f.closed;
    return r;
}

extern "C" int ib_tp_shard(int type, const void* host_src, int64_t rows, int64_t cols, int axis,
                           int rank, int world, void* host_dst) {
    IB_REQUIRE(host_src && host_dst && rows > 0 && cols > 0, "bad shard arguments");
    IB_REQUIRE(world >= 1 && rank >= 0 && rank < world && (axis == 0 || axis == 1),
               "bad shard rank, world or axis");
    const int64_t be = block_elems(type);
    IB_REQUIRE(be > 0 && cols % be == 0, "unsupported type or cols not whole blocks");
    const int64_t nb = cols / be, bb = block_bytes(type), row_bytes = nb * bb;
    const uint8_t* s = (const uint8_t*)host_src;
    uint8_t* d = (uint8_t*)host_dst;
    if (axis == 0) {
        IB_REQUIRE(rows % world == 0, "rows not divisible by the TP size");
        const int64_t r0 = rows / world * rank;
        memcpy(d, s + r0 * row_bytes, (size_t)(rows / world * row_bytes));
        return IB_OK;
    }
    IB_REQUIRE(nb % world == 0, "blocks per row not divisible by the TP size");
    const int64_t nbl = nb / world, shard = nbl * bb;
    for (int64_t r = 0; r < rows; ++r)
        memcpy(d + r * shard, s + r * row_bytes + rank * shard, (size_t)shard);
    return IB_OK;
}
