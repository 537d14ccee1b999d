// Internal plumbing shared by the C-ABI translation units: the opaque handle types, error capture (no exception
// crosses the C ABI), the device upload of a compiled task, and the dispatch over the kernels' compile-time shapes
// (object-bitset words OW and state-row width class WR).

#pragma once

#include "device.cuh"
#include "jit.hpp"
#include "mymyr_b200.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

namespace b2
{
/// A failure carrying its C-ABI status.
struct Error : std::runtime_error
{
    b2_status status;
    Error(b2_status s, const std::string& m) : std::runtime_error(m), status(s) {}
};

void set_last_error(const std::string& m);

#define B2_CUDA(call)                                                                                              \
    do                                                                                                             \
    {                                                                                                              \
        const cudaError_t e_ = (call);                                                                             \
        if (e_ != cudaSuccess)                                                                                     \
            throw ::b2::Error(B2_CUDA_ERROR, std::string(#call) + ": " + cudaGetErrorString(e_));                \
    } while (0)

/// Runs f, converting exceptions into a status and the thread's last error.
template<class F>
b2_status guarded(F&& f)
{
    try
    {
        f();
        return B2_OK;
    }
    catch (const Error& e)
    {
        set_last_error(e.what());
        return e.status;
    }
    catch (const std::invalid_argument& e)
    {
        set_last_error(e.what());
        return B2_INVALID_ARGUMENT;
    }
    catch (const std::length_error& e)
    {
        set_last_error(e.what());
        return B2_CAPACITY;
    }
    catch (const std::bad_alloc&)
    {
        set_last_error("out of host memory");
        return B2_CAPACITY;
    }
    catch (const std::exception& e)
    {
        set_last_error(e.what());
        return B2_INVALID_ARGUMENT;
    }
    catch (...)
    {
        set_last_error("unknown error");
        return B2_INVALID_ARGUMENT;
    }
}

/// Sticky device status bits (written by kernels with atomicOr, read by the host).
enum : u32
{
    kStatusProbeLimit = 1u,      // a hash-set insert ran past its probe bound (table full)
    kStatusEffectOverflow = 2u,  // an action with more than 16 adds or deletes
    kStatusCapacity = 4u,        // a write past a buffer's capacity was dropped
};

/// A device allocation owned by the library. Plain buffers use cudaMalloc; stream-ordered ones (a stream given to
/// alloc/grow) come from the device's memory pool, which the context keeps from releasing memory between calls, so a
/// search that allocates and frees gigabytes does not pay for page mapping every time.
struct DeviceBuffer
{
    void* p = nullptr;
    size_t bytes = 0;
    cudaStream_t stream = nullptr;
    bool pooled = false;
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer() { reset(); }
    void reset()
    {
        if (p)
        {
            if (pooled)
                cudaFreeAsync(p, stream);
            else
                cudaFree(p);
        }
        p = nullptr;
        bytes = 0;
    }
    void alloc(size_t n)
    {
        reset();
        pooled = false;
        if (n)
            B2_CUDA(cudaMalloc(&p, n));
        bytes = n;
    }
    /// Stream-ordered allocation from the device's pool (contents undefined).
    void alloc(size_t n, cudaStream_t s)
    {
        reset();
        stream = s;
        pooled = true;
        if (n)
            B2_CUDA(cudaMallocAsync(&p, n, s));
        bytes = n;
    }
    /// Grows to at least n bytes (stream-ordered), keeping the first `keep` bytes.
    void grow(size_t n, size_t keep, cudaStream_t s)
    {
        if (n <= bytes)
            return;
        void* q = nullptr;
        B2_CUDA(cudaMallocAsync(&q, n, s));
        if (p && keep)
            B2_CUDA(cudaMemcpyAsync(q, p, keep, cudaMemcpyDeviceToDevice, s));
        reset();
        stream = s;
        pooled = true;
        p = q;
        bytes = n;
    }
    template<class T>
    T* as() const
    {
        return static_cast<T*>(p);
    }
    /// Exchanges two buffers' allocations.
    void swap(DeviceBuffer& o) noexcept
    {
        std::swap(p, o.p);
        std::swap(bytes, o.bytes);
        std::swap(stream, o.stream);
        std::swap(pooled, o.pooled);
    }
};
}  // namespace b2

namespace b2
{
/// Small pinned host blocks (a search's status mirror), kept for reuse: page-locking memory per search would cost
/// more than the search's own host work, and freeing pinned memory synchronizes the device.
struct PinnedPool
{
    static constexpr size_t kBlock = 512;
    std::mutex mu;
    std::vector<void*> blocks;
    void* take()
    {
        {
            std::lock_guard lock(mu);
            if (!blocks.empty())
            {
                void* p = blocks.back();
                blocks.pop_back();
                return p;
            }
        }
        void* p = nullptr;
        B2_CUDA(cudaMallocHost(&p, kBlock));
        return p;
    }
    void give(void* p)
    {
        if (!p)
            return;
        std::lock_guard lock(mu);
        blocks.push_back(p);
    }
    ~PinnedPool()
    {
        for (void* p : blocks)
            cudaFreeHost(p);
    }
};
}  // namespace b2

struct b2_ctx
{
    int device = 0;
    cudaDeviceProp prop{};
    int sms = 0;
    b2::DeviceBuffer scratch;  // per-call scratch of the stream-ordered calls (grown as needed)
    b2::PinnedPool pinned;     // status mirrors of searches on this device
    // the device buffers and layer-loop graph of a finished one-GPU BrFS, kept for the next search on this context
    // (brfs.cu: one search holds them at a time)
    std::mutex brfs_mu;
    bool brfs_cache_busy = false;
    std::shared_ptr<void> brfs_cache;
    // b2_expand_noalloc: the device address of its scratch array on this device, and a pinned word pair for its
    // results (both set up by b2_ctx_create, so that the call itself allocates nothing)
    void* noalloc_scratch = nullptr;
    void* noalloc_host = nullptr;
};

namespace b2
{
/// Sets up b2_expand_noalloc on the context's device (current): loads the module that holds its scratch array and the
/// kernels it launches, and records the array's device address in ctx.noalloc_scratch (expand.cu).
void noalloc_prepare(b2_ctx& ctx);
}  // namespace b2

struct b2_task
{
    b2_ctx* ctx = nullptr;
    b2::TaskSpec spec;
    b2::Layout layout;
    std::vector<b2::StaticRel> statics;
    b2::Program prog;
    b2::DeviceBuffer blob;
    b2::DevTask dev{};
    bool witness_refused = false;  // some schema cannot keep canonical order under witness pruning
    std::shared_ptr<b2::JitModule> jit;  // the compiled kernels (null: the interpreted ones)
};

namespace b2
{
/// Row-width class of a task: rows of up to WR words live in registers; 0 reads them from global memory.
inline int width_class(u32 W) { return W <= 1 ? 1 : W <= 2 ? 2 : W <= 4 ? 4 : W <= 8 ? 8 : 0; }

/// Calls f.template operator()<OW, WR>() for the task's shapes.
template<class F>
void dispatch_shapes(u32 ow, u32 words, F&& f)
{
    const int wr = width_class(words);
#define B2_WR(OWV)                                                                                                 \
    switch (wr)                                                                                                    \
    {                                                                                                              \
        case 1: f.template operator()<OWV, 1>(); break;                                                            \
        case 2: f.template operator()<OWV, 2>(); break;                                                            \
        case 4: f.template operator()<OWV, 4>(); break;                                                            \
        case 8: f.template operator()<OWV, 8>(); break;                                                            \
        default: f.template operator()<OWV, 0>(); break;                                                           \
    }
    switch (ow)
    {
        case 1: B2_WR(1) break;
        case 2: B2_WR(2) break;
        case 3: B2_WR(3) break;
        case 4: B2_WR(4) break;
        default: throw Error(B2_UNSUPPORTED, "object bitsets wider than 4 words");
    }
#undef B2_WR
}

/// The parent-row accessor of a kernel with width class WR (0: global memory).
template<int WR>
struct RowOf
{
    using type = RegRow<WR>;
};
template<>
struct RowOf<0>
{
    using type = GlobalRow;
};

template<int WR>
__device__ __forceinline__ typename RowOf<WR>::type load_row(const u64* p, u32 W)
{
    if constexpr (WR == 0)
        return GlobalRow{p, W};
    else
    {
        RegRow<WR> r;
#pragma unroll
        for (int k = 0; k < WR; ++k)
            r.w[k] = static_cast<u32>(k) < W ? p[k] : 0;
        return r;
    }
}

/// The successor of a parent accessor under collected effects, as a word accessor (computed on the fly).
template<class St>
struct SuccRow
{
    const St& parent;
    const Effects& e;
    __device__ __forceinline__ u64 word(u32 i) const { return succ_word(parent, e, i); }
};

inline unsigned grid_for(u64 n, unsigned block, unsigned cap = 1u << 20)
{
    const u64 g = (n + block - 1) / block;
    return static_cast<unsigned>(g < 1 ? 1 : (g > cap ? cap : g));
}

void check_status_word(const u32* dev_status, cudaStream_t s, const char* what);

/// Waits for the stream by polling it (the per-layer waits of a search are short; a blocking wait's wake-up latency
/// would dominate them).
inline void stream_wait(cudaStream_t s)
{
    for (;;)
    {
        const cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess)
            return;
        if (e != cudaErrorNotReady)
            B2_CUDA(e);
    }
}

/// stream_wait for release paths (no exception; an error ends the wait).
inline void stream_drain(cudaStream_t s)
{
    while (cudaStreamQuery(s) == cudaErrorNotReady)
    {
    }
}
}  // namespace b2
