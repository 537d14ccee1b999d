// The ranks' communicator of a sharded search (comm.cu): NCCL, loaded at run time, for the per-layer reductions, and
// CUDA IPC for mapping the ranks' receive buffers into each other's address space.

#pragma once

#include "common.cuh"

#include <cuda_runtime.h>

#include <vector>

namespace b2
{
/// A device buffer of every rank, mapped into every other rank (CUDA IPC): ptr[r] is rank r's buffer.
struct PeerBuffer
{
    DeviceBuffer local;              // this rank's (cudaMalloc: IPC needs it)
    std::vector<void*> ptr;          // [world]
    DeviceBuffer table;              // the ptr array on the device
    size_t bytes = 0;
    ~PeerBuffer();
    void close();
};
}  // namespace b2

struct b2_comm
{
    int device = 0;
    b2::u32 rank = 0;
    b2::u32 world = 1;
    void* nccl = nullptr;       // ncclComm_t
    double timeout_s = 600.0;   // a wait on the ranks' collectives longer than this aborts the communicator
    bool aborted = false;
    // the sharded search's receive buffers (one search at a time per communicator); kept between searches so that
    // their IPC mappings are made once, not per search
    b2::PeerBuffer exchange;
    // per rank one 256-byte block in its own memory, mapped by all: word 0 is the fill cursor of its receive buffer,
    // advanced by the senders' atomics (zeroed before the mappings are shared)
    b2::PeerBuffer cursors;
};

namespace b2
{
enum class CommType
{
    U8,
    U32,
    U64
};
enum class CommOp
{
    Sum,
    Min,
    Max
};

void comm_allreduce(b2_comm* c, const void* send, void* recv, size_t count, CommType t, CommOp op, cudaStream_t s);
void comm_allgather(b2_comm* c, const void* send, void* recv, size_t count, CommType t, cudaStream_t s);
void comm_group_begin();
void comm_group_end();
/// Waits for the stream, polling the communicator's asynchronous error; past the communicator's timeout (a rank that
/// stopped taking part) the communicator is aborted and an error thrown, so that no rank waits for good.
void comm_sync(b2_comm* c, cudaStream_t s);

/// Collective: every rank reallocates its buffer to `bytes` (zeroed if `zero`, before any rank can reach it) and maps
/// the others'.
void peer_buffer_exchange(b2_comm* c, PeerBuffer& b, size_t bytes, cudaStream_t s, bool zero = false);
}  // namespace b2
