// Tensor-parallel plumbing: an NCCL communicator (libnccl.so.2 is opened at run time,
// so the library loads on machines without NCCL and only the TP entry points need it)
// and the host-side sharding of packed GGUF tensors.  The reference runs on one GPU;
// the partitioning follows the Megatron split of a Llama layer: q/k/v and gate/up rows
// by head / FFN column, o_proj and down input columns on block boundaries, the output
// head by vocabulary rows.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <mutex>
#include <string>
#include <vector>

#include "comm.cuh"
#include "common.cuh"

namespace ib {

namespace {

struct Nccl {
    void* so = nullptr;
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) init_rank = nullptr;
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
        n.init_rank = (decltype(n.init_rank))dlsym(n.so, "ncclCommInitRank");
        n.all_reduce = (decltype(n.all_reduce))dlsym(n.so, "ncclAllReduce");
        n.all_gather = (decltype(n.all_gather))dlsym(n.so, "ncclAllGather");
        n.destroy = (decltype(n.destroy))dlsym(n.so, "ncclCommDestroy");
        n.error_string = (decltype(n.error_string))dlsym(n.so, "ncclGetErrorString");
        if (!n.get_unique_id || !n.init_rank || !n.all_reduce || !n.all_gather || !n.destroy ||
            !n.error_string)
            err = "NCCL: libnccl.so.2 lacks an expected symbol";
    });
    if (!err.empty()) {
        set_error(err);
        return IB_ERR_COMM;
    }
    *out = &n;
    return IB_OK;
}

int nccl_check(Nccl* n, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return IB_OK;
    set_error(std::string("NCCL: ") + what + " failed: " + n->error_string(r));
    return IB_ERR_COMM;
}

}  // namespace

struct Comm {
    ncclComm_t nc = nullptr;
    int rank = 0, world = 1, device = 0;
};

int comm_rank(const Comm* c) { return c ? c->rank : 0; }
int comm_world(const Comm* c) { return c ? c->world : 1; }

int comm_allreduce_sum_f32(Comm* c, float* buf, size_t n, cudaStream_t st) {
    if (!c || c->world == 1 || n == 0) return IB_OK;
    Nccl* nc;
    int r = nccl_load(&nc);
    if (r) return r;
    return nccl_check(nc, nc->all_reduce(buf, buf, n, ncclFloat32, ncclSum, c->nc, st),
                      "ncclAllReduce");
}

int comm_allreduce_max_u64(Comm* c, unsigned long long* buf, size_t n, cudaStream_t st) {
    if (!c || c->world == 1 || n == 0) return IB_OK;
    Nccl* nc;
    int r = nccl_load(&nc);
    if (r) return r;
    return nccl_check(nc, nc->all_reduce(buf, buf, n, ncclUint64, ncclMax, c->nc, st),
                      "ncclAllReduce");
}

int comm_peer_alloc(Comm* c, size_t bytes, void** local, void** peers) {
    IB_REQUIRE(c && local && peers && bytes > 0, "bad peer allocation arguments");
    const int W = c->world;
    *local = nullptr;
    for (int q = 0; q < W; ++q) peers[q] = nullptr;
    IB_CUDA_CHECK(cudaMalloc(local, bytes));
    // a failed step below releases what was allocated before it
    auto fail = [&](cudaError_t e, const char* what, uint8_t* scratch) {
        set_error(std::string("peer memory: ") + what + " failed: " + cudaGetErrorString(e));
        if (scratch) cudaFree(scratch);
        cudaFree(*local);
        *local = nullptr;
        return IB_ERR_CUDA;
    };
    cudaError_t ce = cudaMemset(*local, 0, bytes);
    if (ce != cudaSuccess) return fail(ce, "cudaMemset", nullptr);
    if (W == 1) {
        peers[0] = *local;
        return IB_OK;
    }
    cudaIpcMemHandle_t mine;
    if ((ce = cudaIpcGetMemHandle(&mine, *local)) != cudaSuccess)
        return fail(ce, "cudaIpcGetMemHandle", nullptr);
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    uint8_t* dev = nullptr;
    if ((ce = cudaMalloc(&dev, hb * (W + 1))) != cudaSuccess) return fail(ce, "cudaMalloc", nullptr);
    cudaStream_t st;
    if ((ce = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking)) != cudaSuccess)
        return fail(ce, "cudaStreamCreateWithFlags", dev);
    std::vector<cudaIpcMemHandle_t> all(W);
    int r = IB_OK;
    Nccl* nc = nullptr;
    if ((r = nccl_load(&nc)) == IB_OK) {
        cudaMemcpyAsync(dev + hb * W, &mine, hb, cudaMemcpyHostToDevice, st);
        r = nccl_check(nc, nc->all_gather(dev + hb * W, dev, hb, ncclUint8, c->nc, st),
                       "ncclAllGather");
        if (r == IB_OK) cudaMemcpyAsync(all.data(), dev, hb * W, cudaMemcpyDeviceToHost, st);
        if (r == IB_OK && cudaStreamSynchronize(st) != cudaSuccess) {
            set_error("peer memory: handle exchange failed");
            r = IB_ERR_CUDA;
        }
    }
    cudaStreamDestroy(st);
    cudaFree(dev);
    for (int q = 0; q < W && r == IB_OK; ++q) {
        if (q == c->rank) {
            peers[q] = *local;
            continue;
        }
        const cudaError_t e = cudaIpcOpenMemHandle(&peers[q], all[q], cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            set_error(std::string("peer memory: cannot map rank ") + std::to_string(q) +
                      "'s buffer: " + cudaGetErrorString(e));
            peers[q] = nullptr;
            r = IB_ERR_CUDA;
        }
    }
    if (r != IB_OK) {
        comm_peer_free(W, *local, peers);
        *local = nullptr;
    }
    return r;
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
    int r = nccl_load(&nc);
    if (r) return r;
    return nccl_check(nc, nc->all_gather(send, recv, n_per_rank, ncclFloat32, c->nc, st),
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
    if ((r = nccl_check(nc, nc->get_unique_id(&id), "ncclGetUniqueId"))) return r;
    memcpy(id128, id.internal, NCCL_UNIQUE_ID_BYTES);
    return IB_OK;
}

extern "C" int ib_comm_init(int rank, int world, const uint8_t* id128, int device, void** comm) {
    IB_REQUIRE(comm && id128 && world >= 1 && rank >= 0 && rank < world, "bad communicator arguments");
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
    if ((r = nccl_check(nc, nc->init_rank(&c->nc, world, id, rank), "ncclCommInitRank"))) {
        delete c;
        return r;
    }
    *comm = c;
    return IB_OK;
}

extern "C" int ib_comm_allreduce_f32(void* comm, float* dev_buf, int64_t n, void* stream) {
    IB_REQUIRE(comm && dev_buf && n >= 0, "bad allreduce arguments");
    return comm_allreduce_sum_f32((Comm*)comm, dev_buf, (size_t)n, as_stream(stream));
}

extern "C" int ib_comm_free(void* comm) {
    if (!comm) return IB_OK;
    Comm* c = (Comm*)comm;
    Nccl* nc;
    if (nccl_load(&nc) == IB_OK && c->nc) nc->destroy(c->nc);
    delete c;
    return IB_OK;
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
