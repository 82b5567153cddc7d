// Tensor-parallel communicator (comm.cpp): NCCL opened at run time.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "ib_cuda.h"

namespace ib {

struct Comm;

int comm_rank(const Comm* c);
int comm_world(const Comm* c);
// In place; no-ops for a null communicator or a world of one.
int comm_allreduce_sum_f32(Comm* c, float* buf, size_t n, cudaStream_t st);
int comm_allreduce_max_u64(Comm* c, unsigned long long* buf, size_t n, cudaStream_t st);
// recv[r * n_per_rank ...] <- rank r's send.
int comm_allgather_f32(Comm* c, const float* send, float* recv, size_t n_per_rank,
                       cudaStream_t st);

// Peer memory: every rank allocates `bytes` (zeroed) of device memory and maps every
// other rank's allocation into its address space (CUDA IPC handles exchanged over the
// communicator; NVLink peer access).  peers[q] = rank q's allocation as seen here
// (peers[rank] = *local).  Collective: every rank calls it with the same size, and with
// local_status = the result of its own set-up so far; a rank whose status is not IB_OK
// still joins the exchange, and then every rank fails (each with a message naming the
// rank that failed; the failing rank keeps its own message).
int comm_peer_alloc(Comm* c, size_t bytes, int local_status, void** local, void** peers);

// The peer set-up protocol over replaceable layers (CUDA IPC and an NCCL all-gather in
// comm_peer_alloc; stand-ins in ib_peer_setup_check).  Layer functions return 0 on
// success; the failure text goes to *err.
constexpr size_t kPeerHandleBytes = 64;
struct PeerIpc {
    void* ctx;
    int (*handle)(void* ctx, void* local, uint8_t* out, size_t bytes, std::string* err);
    int (*open)(void* ctx, int peer, const uint8_t* handle, size_t bytes, void** ptr,
                std::string* err);
    void (*close)(void* ctx, void* ptr);
};
struct PeerGather {  // all[r * bytes ...] <- rank r's `bytes`; IB_OK or an IB_ERR_* code
    void* ctx;
    int (*all)(void* ctx, const uint8_t* mine, uint8_t* all, size_t bytes);
};
int peer_setup(int rank, int world, void* local, int local_status, const PeerIpc& ipc,
               const PeerGather& gather, void** peers);
// Unmaps the peers' allocations and frees this rank's (peers as filled above, world
// entries; the communicator itself is not needed).
void comm_peer_free(int world, void* local, void** peers);

}  // namespace ib
