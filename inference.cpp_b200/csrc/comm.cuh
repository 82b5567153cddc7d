// Tensor-parallel communicator (comm.cpp): NCCL opened at run time.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

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
// (peers[rank] = *local).  Collective: every rank calls it with the same size.
int comm_peer_alloc(Comm* c, size_t bytes, void** local, void** peers);
// Unmaps the peers' allocations and frees this rank's (peers as filled above, world
// entries; the communicator itself is not needed).
void comm_peer_free(int world, void* local, void** peers);

}  // namespace ib
