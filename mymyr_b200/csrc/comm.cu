// Communicators of sharded searches: NCCL loaded at run time (libnccl.so.2; the copy a process already loaded, such as
// PyTorch's, is reused), collectives on the caller's stream, a bounded wait that turns a rank that stopped taking part
// into an error, and CUDA IPC buffers mapped by every rank. No counterpart in the reference (it has no multi-GPU layer).

#include "comm.hpp"

#include <nccl.h>

#include <dlfcn.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

namespace b2
{
namespace
{
struct Nccl
{
    void* so = nullptr;
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) init_rank = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclCommAbort) abort = nullptr;
    decltype(&ncclCommGetAsyncError) async_error = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};

template<class F>
void sym(void* so, F& f, const char* name)
{
    f = reinterpret_cast<F>(dlsym(so, name));
    if (!f)
        throw Error(B2_CUDA_ERROR, std::string("mymyr_b200: libnccl.so.2 lacks ") + name);
}

const Nccl& nccl()
{
    static std::once_flag once;
    static Nccl n;
    static std::string failure;
    std::call_once(once, [] {
        void* so = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!so)
            so = dlopen("libnccl.so.2", RTLD_NOW);
        if (!so)
        {
            failure = "mymyr_b200: NCCL (libnccl.so.2) is not available for a multi-GPU search";
            return;
        }
        try
        {
            sym(so, n.get_unique_id, "ncclGetUniqueId");
            sym(so, n.init_rank, "ncclCommInitRank");
            sym(so, n.destroy, "ncclCommDestroy");
            sym(so, n.abort, "ncclCommAbort");
            sym(so, n.async_error, "ncclCommGetAsyncError");
            sym(so, n.all_reduce, "ncclAllReduce");
            sym(so, n.all_gather, "ncclAllGather");
            sym(so, n.group_start, "ncclGroupStart");
            sym(so, n.group_end, "ncclGroupEnd");
            sym(so, n.error_string, "ncclGetErrorString");
            n.so = so;
        }
        catch (const std::exception& e)
        {
            failure = e.what();
        }
    });
    if (!n.so)
        throw Error(B2_CUDA_ERROR, failure);
    return n;
}

void check(ncclResult_t r, const char* what)
{
    if (r != ncclSuccess)
        throw Error(B2_CUDA_ERROR, std::string(what) + ": " + nccl().error_string(r));
}

ncclComm_t handle(b2_comm* c)
{
    if (!c || !c->nccl)
        throw std::invalid_argument("mymyr_b200: no communicator");
    if (c->aborted)
        throw Error(B2_CUDA_ERROR, "mymyr_b200: the communicator was aborted after an earlier failure");
    return static_cast<ncclComm_t>(c->nccl);
}

ncclDataType_t type_of(CommType t)
{
    switch (t)
    {
        case CommType::U8: return ncclUint8;
        case CommType::U32: return ncclUint32;
        default: return ncclUint64;
    }
}

ncclRedOp_t op_of(CommOp o)
{
    switch (o)
    {
        case CommOp::Sum: return ncclSum;
        case CommOp::Min: return ncclMin;
        default: return ncclMax;
    }
}
}  // namespace

void comm_allreduce(b2_comm* c, const void* send, void* recv, size_t count, CommType t, CommOp op, cudaStream_t s)
{
    check(nccl().all_reduce(send, recv, count, type_of(t), op_of(op), handle(c), s), "ncclAllReduce");
}

void comm_allgather(b2_comm* c, const void* send, void* recv, size_t count, CommType t, cudaStream_t s)
{
    check(nccl().all_gather(send, recv, count, type_of(t), handle(c), s), "ncclAllGather");
}

void comm_group_begin() { check(nccl().group_start(), "ncclGroupStart"); }
void comm_group_end() { check(nccl().group_end(), "ncclGroupEnd"); }

void comm_sync(b2_comm* c, cudaStream_t s)
{
    const auto t0 = std::chrono::steady_clock::now();
    auto next_check = t0;
    for (;;)
    {
        const cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess)
            return;
        if (e != cudaErrorNotReady)
            B2_CUDA(e);
        const auto now = std::chrono::steady_clock::now();
        if (now < next_check)
        {
            // per-layer waits are short: poll; a wait past 50 ms (a slow peer) polls more gently
            if (now - t0 > std::chrono::milliseconds(50))
                std::this_thread::sleep_for(std::chrono::microseconds(20));
            continue;
        }
        next_check = now + std::chrono::milliseconds(5);
        ncclComm_t h = handle(c);
        ncclResult_t ae = ncclSuccess;
        check(nccl().async_error(h, &ae), "ncclCommGetAsyncError");
        const bool late = std::chrono::duration<double>(now - t0).count() > c->timeout_s;
        if ((ae != ncclSuccess && ae != ncclInProgress) || late)
        {
            // aborting ends the communicator's kernels that wait for the missing ranks; the stream then drains
            nccl().abort(h);
            c->nccl = nullptr;
            c->aborted = true;
            cudaStreamSynchronize(s);
            throw Error(B2_CUDA_ERROR, late ? "mymyr_b200: a collective of the search did not complete within the "
                                              "communicator's timeout (a rank stopped taking part); communicator aborted"
                                            : std::string("mymyr_b200: NCCL reported ") + nccl().error_string(ae));
        }
    }
}

PeerBuffer::~PeerBuffer() { close(); }

void PeerBuffer::close()
{
    for (void*& p : ptr)
        if (p && p != local.p)
            cudaIpcCloseMemHandle(p);
    ptr.clear();
    local.reset();
    table.reset();
    bytes = 0;
}

void peer_buffer_exchange(b2_comm* c, PeerBuffer& b, size_t bytes, cudaStream_t s, bool zero)
{
    const u32 world = c->world, me = c->rank;
    comm_sync(c, s);
    DeviceBuffer scratch;
    const size_t hs = sizeof(cudaIpcMemHandle_t);
    scratch.alloc(hs * (world + 1) + 16);
    // every rank unmaps the others' old buffers before any rank frees its own
    for (u32 r = 0; r < b.ptr.size(); ++r)
        if (r != me && b.ptr[r])
            B2_CUDA(cudaIpcCloseMemHandle(b.ptr[r]));
    b.ptr.assign(world, nullptr);
    u32* word = reinterpret_cast<u32*>(scratch.as<char>() + hs * (world + 1));
    B2_CUDA(cudaMemsetAsync(word, 0, 4, s));
    comm_allreduce(c, word, word, 1, CommType::U32, CommOp::Sum, s);
    comm_sync(c, s);
    b.local.alloc(bytes);
    if (zero)
        B2_CUDA(cudaMemset(b.local.p, 0, bytes));  // complete before the handle allgather below
    cudaIpcMemHandle_t h;
    B2_CUDA(cudaIpcGetMemHandle(&h, b.local.p));
    B2_CUDA(cudaMemcpyAsync(scratch.p, &h, hs, cudaMemcpyHostToDevice, s));
    comm_allgather(c, scratch.p, scratch.as<char>() + hs, hs, CommType::U8, s);
    std::vector<cudaIpcMemHandle_t> all(world);
    B2_CUDA(cudaMemcpyAsync(all.data(), scratch.as<char>() + hs, hs * world, cudaMemcpyDeviceToHost, s));
    comm_sync(c, s);
    for (u32 r = 0; r < world; ++r)
        if (r == me)
            b.ptr[r] = b.local.p;
        else
            B2_CUDA(cudaIpcOpenMemHandle(&b.ptr[r], all[r], cudaIpcMemLazyEnablePeerAccess));
    b.table.alloc(world * sizeof(void*));
    B2_CUDA(cudaMemcpy(b.table.p, b.ptr.data(), world * sizeof(void*), cudaMemcpyHostToDevice));
    b.bytes = bytes;
}
}  // namespace b2

using namespace b2;

extern "C" {

b2_status b2_comm_id_new(b2_comm_id* out)
{
    return guarded([&] {
        if (!out)
            throw std::invalid_argument("b2_comm_id_new: null argument");
        static_assert(sizeof(ncclUniqueId) == sizeof(b2_comm_id), "ncclUniqueId size");
        ncclUniqueId id;
        check(nccl().get_unique_id(&id), "ncclGetUniqueId");
        std::memcpy(out, &id, sizeof id);
    });
}

b2_status b2_comm_create(b2_ctx* ctx, const b2_comm_id* id, uint32_t rank, uint32_t world, b2_comm** out)
{
    return guarded([&] {
        if (!ctx || !id || !out)
            throw std::invalid_argument("b2_comm_create: null argument");
        if (world < 1 || world > dev::kMaxWorld || rank >= world)
            throw std::invalid_argument("b2_comm_create: rank " + std::to_string(rank) + " of " + std::to_string(world) +
                                        " (1 to " + std::to_string(dev::kMaxWorld) + " ranks)");
        B2_CUDA(cudaSetDevice(ctx->device));
        ncclUniqueId uid;
        std::memcpy(&uid, id, sizeof uid);
        ncclComm_t h = nullptr;
        check(nccl().init_rank(&h, static_cast<int>(world), uid, static_cast<int>(rank)), "ncclCommInitRank");
        auto c = std::make_unique<b2_comm>();
        c->device = ctx->device;
        c->rank = rank;
        c->world = world;
        c->nccl = h;
        *out = c.release();
    });
}

b2_status b2_comm_set_timeout(b2_comm* comm, double seconds)
{
    return guarded([&] {
        if (!comm || !(seconds > 0))
            throw std::invalid_argument("b2_comm_set_timeout: a communicator and a positive time");
        comm->timeout_s = seconds;
    });
}

void b2_comm_destroy(b2_comm* comm)
{
    if (!comm)
        return;
    cudaSetDevice(comm->device);
    comm->exchange.close();
    comm->cursors.close();
    if (comm->nccl)
        nccl().destroy(static_cast<ncclComm_t>(comm->nccl));
    delete comm;
}

}  // extern "C"
