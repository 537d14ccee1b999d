// Internal: the BrFS search object (brfs.cu, one GPU; dbrfs.cu, sharded over ranks) and the kernels both use.

#pragma once

#include "comm.hpp"
#include "scan.cuh"

#include <vector>

namespace b2
{
namespace
{
using dev::insert;
using dev::kEmpty;
using dev::LayerMisc;
using dev::DevLayerState;
using dev::Store;

template<int OW, int WR>
__global__ void __launch_bounds__(128) k_count(DevTask T, u32 pi, const u64* __restrict__ rows, u32 W,
                                               const u32* __restrict__ frontier, u64 E_in, u32* __restrict__ counts,
                                               LayerMisc* misc, const u64* E_dev = nullptr)
{
    const u64 E = E_dev ? *E_dev : E_in;  // a non-null E_dev: the parents are a count still on the device
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < E; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 g = frontier[i];
        const auto st = load_row<WR>(rows + g * W, W);
        if (goal_holds(T, st))
        {
            atomicAdd(&misc->goals, 1u);
            atomicMin(&misc->first_goal, static_cast<u32>(i));
        }
        u32 c = 0;
        u32 bind[kMaxLevels] = {};
        for (u32 s = 0; s < T.nschemas; ++s)
            enumerate<OW>(T, T.schemas[s].prog[pi], st, bind, [&](const u32*) {
                ++c;
                return true;
            });
        counts[i] = c;
    }
}

/// Interpreted matcher: calls f(successor accessor, hash) for the successor of `st` under schema sc's binding b.
template<int WR, class Row, class F>
__device__ __forceinline__ void with_successor_interp(const DevTask& T, const DSchema& sc, const Row& st, const u32* b,
                                                      u32 W, F&& f)
{
    if constexpr (WR > 0)
    {
        RegRow<WR> nx = st;
        for (u32 q = sc.del_begin; q < sc.del_end; ++q)
        {
            const u64 key = pattern_key(T, T.lits[q], b);
            if (key < T.fluent_count)
                nx.clear(static_cast<u32>(key));
        }
        for (u32 q = sc.add_begin; q < sc.add_end; ++q)
            nx.set(static_cast<u32>(pattern_key(T, T.lits[q], b)));
        f(nx, hash_words([&](u32 q) { return nx.word(q); }, W));
    }
    else
    {
        Effects e;
        collect_effects(T, sc, b, e);
        const SuccRow<Row> nx{st, e};
        f(nx, hash_words([&](u32 q) { return nx.word(q); }, W));
    }
}

/// Interpreted matcher: the records of the local parents' successors (the compiled twin is b2j_dbrfs_expand).
template<int OW, int WR>
__global__ void __launch_bounds__(128) k_dexpand(DevTask T, dev::DExpandArgs a)
{
    __shared__ u32 hist[dev::kMaxWorld];
    for (u32 d = threadIdx.x; d < a.world; d += blockDim.x)
        hist[d] = 0;
    __syncthreads();
    const u32 W = a.W;
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < a.E; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 id = a.frontier_id[i];
        if (id >= a.limit)
            continue;
        const auto st = load_row<WR>(a.rows + static_cast<u64>(a.frontier[i]) * W, W);
        const u64 c0 = a.gbase ? a.gbase[id - a.layer_begin] : id << 32;
        u64* out = a.staging + (a.local_base[i] - a.stage_base) * (W + 2);
        u32 k = 0;
        u32 bind[kMaxLevels] = {};
        for (u32 s = 0; s < T.nschemas; ++s)
        {
            const DSchema& sc = T.schemas[s];
            enumerate<OW>(T, sc.prog[a.pi], st, bind, [&](const u32* b) {
                with_successor_interp<WR>(T, sc, st, b, W, [&](const auto& nx, u64 h) {
                    u64* r = out + static_cast<u64>(k) * (W + 2);
                    for (u32 q = 0; q < W; ++q)
                        r[q] = nx.word(q);
                    r[W] = h;
                    r[W + 1] = c0 + k;
                    atomicAdd(&hist[dev::owner_of(h, a.world)], 1u);
                });
                ++k;
                return true;
            });
        }
    }
    __syncthreads();
    for (u32 d = threadIdx.x; d < a.world; d += blockDim.x)
        if (hist[d])
            atomicAdd(reinterpret_cast<unsigned long long*>(a.hist + d), static_cast<unsigned long long>(hist[d]));
}

/// Interpreted matcher, sharded count pass: k_count plus the successors per owner rank (the compiled twin is
/// b2j_dbrfs_count).
template<int OW, int WR>
__global__ void __launch_bounds__(128) k_dcount(DevTask T, u32 pi, const u64* __restrict__ rows, u32 W,
                                                const u32* __restrict__ frontier, u64 E_in, const u64* E_dev,
                                                u32* __restrict__ counts, LayerMisc* misc, u64* hist_out, u32 world)
{
    __shared__ u32 hist[dev::kMaxWorld];
    for (u32 d = threadIdx.x; d < world; d += blockDim.x)
        hist[d] = 0;
    __syncthreads();
    const u64 E = E_dev ? *E_dev : E_in;
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < E; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const auto st = load_row<WR>(rows + static_cast<u64>(frontier[i]) * W, W);
        if (goal_holds(T, st))
        {
            atomicAdd(&misc->goals, 1u);
            atomicMin(&misc->first_goal, static_cast<u32>(i));
        }
        u32 k = 0;
        u32 bind[kMaxLevels] = {};
        for (u32 s = 0; s < T.nschemas; ++s)
        {
            const DSchema& sc = T.schemas[s];
            enumerate<OW>(T, sc.prog[pi], st, bind, [&](const u32* b) {
                with_successor_interp<WR>(T, sc, st, b, W,
                                          [&](const auto&, u64 h) { atomicAdd(&hist[dev::owner_of(h, world)], 1u); });
                ++k;
                return true;
            });
        }
        counts[i] = k;
    }
    __syncthreads();
    for (u32 d = threadIdx.x; d < world; d += blockDim.x)
        if (hist[d])
            atomicAdd(reinterpret_cast<unsigned long long*>(hist_out + d), static_cast<unsigned long long>(hist[d]));
}

constexpr unsigned kPushThreads = 256;
constexpr u32 kPushSmemWords = 5120;  // 40 KB of staged records per block (with the static arrays, under 48 KB)

/// The exchange: each block loads a tile of staged records, orders it by owner rank in shared memory, reserves each
/// owner's run in this rank's region of that owner's receive buffer, and writes the runs with consecutive threads on
/// consecutive words (coalesced stores over NVLink for the other ranks). This rank's region of owner d starts after
/// the records of ranks < this one for d (M[s][d]: records of rank s for owner d, all-gathered).
///
/// `cap`: records each owner's receive buffer holds. A record that would land past it is dropped and sets *overflow, so
/// that a sizing error fails the layer instead of writing past another GPU's allocation.
__global__ void __launch_bounds__(kPushThreads) k_push(const u64* __restrict__ staging, const u64* __restrict__ M,
                                                       u64* const* __restrict__ peers, unsigned long long* cursor,
                                                       u32 me, u32 world, u32 RW, u32 tile, u64 cap, u32* overflow)
{
    extern __shared__ u64 sm[];
    __shared__ u32 cnt[dev::kMaxWorld], start[dev::kMaxWorld];
    __shared__ u64 off[dev::kMaxWorld], base[dev::kMaxWorld];
    __shared__ unsigned short order[kPushThreads];
    __shared__ u8 dst[kPushThreads];
    u64 n = 0;
    for (u32 d = 0; d < world; ++d)
        n += M[me * world + d];
    for (u32 d = threadIdx.x; d < world; d += blockDim.x)
    {
        u64 o = 0;
        for (u32 s = 0; s < me; ++s)
            o += M[s * world + d];
        off[d] = o;
    }
    for (u64 t0 = blockIdx.x * static_cast<u64>(tile); t0 < n; t0 += static_cast<u64>(gridDim.x) * tile)
    {
        const u32 m = static_cast<u32>(n - t0 < tile ? n - t0 : tile);
        for (u32 d = threadIdx.x; d < world; d += blockDim.x)
            cnt[d] = 0;
        const u64* src = staging + t0 * RW;
        for (u32 q = threadIdx.x; q < m * RW; q += blockDim.x)
            sm[q] = src[q];
        __syncthreads();
        u32 d = 0, p = 0;
        if (threadIdx.x < m)
        {
            d = dev::owner_of(sm[threadIdx.x * RW + RW - 2], world);
            p = atomicAdd(&cnt[d], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0)
        {
            u32 acc = 0;
            for (u32 x = 0; x < world; ++x)
            {
                start[x] = acc;
                acc += cnt[x];
            }
        }
        for (u32 x = threadIdx.x; x < world; x += blockDim.x)
            base[x] = cnt[x] ? atomicAdd(cursor + x, static_cast<unsigned long long>(cnt[x])) : 0;
        __syncthreads();
        if (threadIdx.x < m)
        {
            order[start[d] + p] = static_cast<unsigned short>(threadIdx.x);
            dst[threadIdx.x] = static_cast<u8>(d);
        }
        __syncthreads();
        for (u32 q = threadIdx.x; q < m * RW; q += blockDim.x)
        {
            const u32 sp = q / RW, w = q - sp * RW;
            const u32 rec = order[sp], dd = dst[rec];
            const u64 slot = off[dd] + base[dd] + (sp - start[dd]);
            if (slot < cap)
                peers[dd][slot * RW + w] = sm[rec * RW + w];
            else if (w == 0)
                atomicOr(overflow, 1u);
        }
        __syncthreads();
    }
    // the records are visible to every rank before this kernel completes; the ranks' next collective orders them
    // before the owners' inserts
    __threadfence_system();
}

/// The exchange without a prior all-gather of the per-owner counts: like k_push, but each block reserves each owner's
/// run by an atomic on that owner's fill cursor (in the owner's memory, over NVLink for the other ranks), so the
/// records of all senders interleave in the owner's buffer in an order of no meaning (the records carry their keys).
/// The staged records are the first sum(hist) of the staging area. `cap` and `overflow` as for k_push.
__global__ void __launch_bounds__(kPushThreads) k_push_reserve(const u64* __restrict__ staging,
                                                               const u64* __restrict__ hist, u64* const* __restrict__ peers,
                                                               u64* const* __restrict__ cursors,
                                                               unsigned long long* sent_self, u32 me, u32 world, u32 RW,
                                                               u32 tile, u64 cap, u32* overflow)
{
    extern __shared__ u64 sm[];
    __shared__ u32 cnt[dev::kMaxWorld], start[dev::kMaxWorld];
    __shared__ u64 base[dev::kMaxWorld];
    __shared__ unsigned short order[kPushThreads];
    __shared__ u8 dst[kPushThreads];
    u64 n = 0;
    for (u32 d = 0; d < world; ++d)
        n += hist[d];
    for (u64 t0 = blockIdx.x * static_cast<u64>(tile); t0 < n; t0 += static_cast<u64>(gridDim.x) * tile)
    {
        const u32 m = static_cast<u32>(n - t0 < tile ? n - t0 : tile);
        for (u32 d = threadIdx.x; d < world; d += blockDim.x)
            cnt[d] = 0;
        const u64* src = staging + t0 * RW;
        for (u32 q = threadIdx.x; q < m * RW; q += blockDim.x)
            sm[q] = src[q];
        __syncthreads();
        u32 d = 0, p = 0;
        if (threadIdx.x < m)
        {
            d = dev::owner_of(sm[threadIdx.x * RW + RW - 2], world);
            p = atomicAdd(&cnt[d], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0)
        {
            u32 acc = 0;
            for (u32 x = 0; x < world; ++x)
            {
                start[x] = acc;
                acc += cnt[x];
            }
        }
        for (u32 x = threadIdx.x; x < world; x += blockDim.x)
            base[x] = cnt[x] ? atomicAdd_system(reinterpret_cast<unsigned long long*>(cursors[x]),
                                                static_cast<unsigned long long>(cnt[x]))
                             : 0;
        if (threadIdx.x == 0 && cnt[me])
            atomicAdd(sent_self, static_cast<unsigned long long>(cnt[me]));
        __syncthreads();
        if (threadIdx.x < m)
        {
            order[start[d] + p] = static_cast<unsigned short>(threadIdx.x);
            dst[threadIdx.x] = static_cast<u8>(d);
        }
        __syncthreads();
        for (u32 q = threadIdx.x; q < m * RW; q += blockDim.x)
        {
            const u32 sp = q / RW, w = q - sp * RW;
            const u32 rec = order[sp], dd = dst[rec];
            const u64 slot = base[dd] + (sp - start[dd]);
            if (slot < cap)
                peers[dd][slot * RW + w] = sm[rec * RW + w];
            else if (w == 0)
                atomicOr(overflow, 1u);
        }
        __syncthreads();
    }
    // the records are visible to every rank before this kernel completes; the ranks' next collective orders them
    // before the owners' inserts
    __threadfence_system();
}

/// Reinserts the states `state_g[0, n)` (arena indices) into an empty table.
__global__ void k_rehash(u64* __restrict__ table, u64 mask, u32 max_probe, const u32* __restrict__ state_g, u64 n,
                         const u64* __restrict__ hash, u32* status)
{
    for (u64 id = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; id < n; id += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 g = state_g[id];
        const u64 h = hash[g];
        const u64 mine = (h & 0xFFFFFFFF00000000ull) | g;
        u64 j = h & mask;
        u32 probe = 0;
        for (; probe < max_probe; ++probe, j = (j + 1) & mask)
            if (atomicCAS(reinterpret_cast<unsigned long long*>(table + j), kEmpty, mine) == kEmpty)
                break;
        if (probe == max_probe)
            atomicOr(status, kStatusProbeLimit);
    }
}

struct CountIn
{
    const u32* c;
    __device__ __forceinline__ u32 operator()(u64 i) const { return c[i]; }
};
struct BaseOut
{
    u64* base;
    __device__ __forceinline__ void operator()(u64 i, u64 e, u32) const { base[i] = e; }
};

inline u32 max_probe(u64 slots) { return static_cast<u32>(std::min<u64>(slots, u64{1} << 20)); }
}  // namespace

struct ShardState;
}  // namespace b2

struct b2_brfs
{
    b2_task* task = nullptr;
    b2_brfs_options opt{};
    cudaStream_t stream = nullptr;
    b2::u32 W = 1;
    // per candidate
    b2::DeviceBuffer rows, hash, par, kid;
    b2::u64 cap_cand = 0;
    // per state
    b2::DeviceBuffer state_g;
    b2::u64 cap_states = 0;
    // hash set
    b2::DeviceBuffer table;
    b2::u64 table_slots = 0;
    b2::u32 rehashes = 0;
    // per layer scratch
    b2::DeviceBuffer counts, cand_base, flags, deferred, sums, misc;
    b2::u64 cap_layer = 0, cap_flags = 0;
    b2::dev::LayerMisc* misc_host = nullptr;  // pinned mirror of `misc` (two counter slots)
    unsigned slot = 0;                         // the current layer's counter slot
    // results
    std::vector<b2::u64> layer_begin;  // id of each layer's first state (+ the end)
    b2::u64 n_states = 0;
    b2::u64 launches = 0;
    double wait_s = 0;  // host time spent waiting for the device's layer results (this search)
    // the device-driven layer loop: its state, its per-layer log, the stream its body is captured on, the
    // instantiated graph and what it was captured over
    b2::DeviceBuffer dstate, dlog;
    cudaStream_t capture = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    std::vector<b2::u64> graph_key;
    bool from_cache = false;  // the buffers (and graph) came from the context's cache and go back to it
    bool ran_one_gpu = false; // the one-GPU buffers were used (a one-GPU search, or a sharded search's small layers)
    bool ran = false;
    bool own_stream = false;
    // sharded search (options.comm set)
    b2_comm* comm = nullptr;
    b2::ShardState* shard = nullptr;
};

namespace b2
{
/// The sharded search (dbrfs.cu): run, the rank's states, release.
void shard_run(b2_brfs& B, b2_brfs_result& R);
/// The one-GPU search of B up to the first layer whose frontier holds at least prefix_states states (brfs.cu): true
/// when it stopped there, false when the search ended before (R is then its whole result).
bool run_prefix(b2_brfs& B, b2_brfs_result& R, u64 prefix_states);
u64 shard_local_count(const b2_brfs& B);
void shard_local(b2_brfs& B, u64 first, u64 count, u64* ids, u64* rows, u32 words, u64* hashes, u32* parent,
                 u32* index);
void shard_free(b2_brfs& B);
}  // namespace b2
