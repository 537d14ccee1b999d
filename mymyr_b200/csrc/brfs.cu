// Layer-synchronous device BrFS (cuda::DeviceBrfs / mymyr::brfs with deterministic ids,
// include/mymyr/cuda/brfs.hpp:96-123, include/mymyr/search/brfs.hpp:140; loop semantics of run_flat,
// src/mymyr/search/brfs.cpp:273-404).
//
// Data layout in HBM. Every successor ever generated has a global candidate index g: a layer's candidates are
// numbered in canonical order (parent id, successor index) after the previous layers'. Per candidate (written only
// when it takes a hash-set slot): its row rows[g * W .. +W), its hash, its parent's index in its layer and its
// successor index. Per state id: state_g[id], the candidate that discovered it; a layer's frontier is the id range
// [begin, end) of state_g. The hash set is open addressing over u64 slots (hash >> 32) << 32 | g, linear probing
// from hash & mask; EMPTY is all ones.
//
// Deterministic ids without a sort: within a slot's lifetime every value refers to the same state, so an equal
// successor replaces a larger candidate index with atomicMin (the tag sits above g, equal tags compare by g). The
// smallest g of a state, its first discovery in canonical order, always ends up in the slot, and a state found in an
// earlier layer keeps its smaller g. A candidate that took a slot marks itself `claimed`; one that displaces a
// larger candidate of the layer marks that one `lost`. New states are the claimed, not lost candidates; an exclusive
// scan over the layer's candidates in order gives their ids, in the order of the reference's (parent id, successor
// index) discoverer keys (src/mymyr/search/brfs.cpp:1657-1778).
//
// Per layer: k_count (goal test + successor counts per parent) -> scan (candidate offsets) -> host reads the layer's
// candidate count -> k_expand (regenerate, hash, optimistic insert) -> k_resolve (deferred inserts) -> scan of winners
// (ids) -> host reads the new-state count.

#include "brfs.cuh"

#include <chrono>

namespace b2
{
namespace
{
/// Phase B: the deferred inserts, resumed at their slots. Every row they can meet was written by the expansion
/// kernel (or an earlier one), so the comparisons need no ordering within this kernel. Among equal candidates of the
/// layer the smallest g takes the slot by atomicMin (the tag sits above g); a displaced one is marked lost.
__global__ void k_resolve(Store S, const DevLayerState* dyn = nullptr)
{
    if (dyn)
        S.layer_cand_begin = dyn->cand_next;
    const u32 n = *S.ndeferred;
    for (u32 q = blockIdx.x * blockDim.x + threadIdx.x; q < n; q += gridDim.x * blockDim.x)
    {
        const u64 d = S.deferred[q];
        const u64 g = d & 0xFFFFFFFFull;
        const u64 h = S.hash[g];
        const u64 mine = (h & 0xFFFFFFFF00000000ull) | g;
        const u64* row = S.rows + g * S.W;
        u64 j = d >> 32;
        bool done = false;
        for (u32 probe = 0; probe < S.max_probe && !done; ++probe, j = (j + 1) & S.mask)
        {
            u64 cur = __ldcg(S.table + j);
            if (cur == kEmpty)
            {
                const u64 prev = atomicCAS(reinterpret_cast<unsigned long long*>(S.table + j), kEmpty, mine);
                if (prev == kEmpty)
                {
                    S.claimed[g - S.layer_cand_begin] = 1;
                    done = true;
                    break;
                }
                cur = prev;
            }
            if ((cur >> 32) != (mine >> 32))
                continue;
            const u64 og = cur & 0xFFFFFFFFull;
            const u64* r = S.rows + og * S.W;
            bool eq = true;
            for (u32 w = 0; w < S.W && eq; ++w)
                eq = __ldcg(r + w) == __ldcg(row + w);
            if (!eq)
                continue;
            done = true;
            if (og < g)
                break;  // an earlier discovery of the same state
            const u64 prev = atomicMin(reinterpret_cast<unsigned long long*>(S.table + j), mine);
            if (prev > mine)
            {
                S.claimed[g - S.layer_cand_begin] = 1;
                S.lost[(prev & 0xFFFFFFFFull) - S.layer_cand_begin] = 1;
            }
        }
        if (!done)
            atomicOr(S.status, kStatusProbeLimit);
    }
}

template<int OW, int WR>
__global__ void __launch_bounds__(128) k_expand(DevTask T, u32 pi, const u32* __restrict__ frontier, u64 E,
                                                const u64* __restrict__ cand_base, Store S)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < E; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 pg = frontier[i];
        const auto st = load_row<WR>(S.rows + pg * S.W, S.W);
        const u64 g0 = S.layer_cand_begin + cand_base[i];
        u32 k = 0;
        u32 bind[kMaxLevels] = {};
        for (u32 s = 0; s < T.nschemas; ++s)
        {
            const DSchema& sc = T.schemas[s];
            enumerate<OW>(T, sc.prog[pi], st, bind, [&](const u32* b) {
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
                    const u64 h = hash_words([&](u32 q) { return nx.word(q); }, S.W);
                    insert(S, nx, h, g0 + k, static_cast<u32>(i), k);
                }
                else
                {
                    Effects e;
                    collect_effects(T, sc, b, e);
                    const SuccRow<decltype(st)> nx{st, e};
                    const u64 h = hash_words([&](u32 q) { return nx.word(q); }, S.W);
                    insert(S, nx, h, g0 + k, static_cast<u32>(i), k);
                }
                ++k;
                return true;
            });
        }
    }
}

/// Goal states among the parents frontier[0, n) (a layer cut short by max_states).
__global__ void k_count_goals(DevTask T, const u64* __restrict__ rows, u32 W, const u32* __restrict__ frontier, u64 n,
                              u32* out)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < n; i += static_cast<u64>(gridDim.x) * blockDim.x)
        if (goal_holds(T, GlobalRow{rows + static_cast<u64>(frontier[i]) * W, W}))
            atomicAdd(out, 1u);
}

/// Resets a layer's counters (its slot of the two that alternate between layers).
__global__ void k_layer_init(LayerMisc* m) { *m = LayerMisc{0, 0, 0, 0, 0xFFFFFFFFu, 0, 0}; }

__global__ void k_seed_root(Store S, u32* state_g)
{
    const GlobalRow r{S.rows, S.W};
    const u64 h = hash_words([&](u32 q) { return r.word(q); }, S.W);
    S.hash[0] = h;
    S.par[0] = 0xFFFFFFFFu;
    S.kid[0] = 0;
    state_g[0] = 0;
    u64 j = h & S.mask;
    for (u32 probe = 0; probe < S.max_probe && S.table[j] != kEmpty; ++probe)
        j = (j + 1) & S.mask;
    if (S.table[j] == kEmpty)
        S.table[j] = (h & 0xFFFFFFFF00000000ull);
    else
        atomicOr(S.status, kStatusProbeLimit);
}

struct WinIn
{
    const u8* claimed;
    const u8* lost;
    __device__ __forceinline__ u32 operator()(u64 c) const { return claimed[c] & (lost[c] ^ 1u); }
};
struct WinOut
{
    u32* state_g;  // + id of the layer's first new state
    u64 cand_begin;
    __device__ __forceinline__ void operator()(u64 c, u64 rank, u32 v) const
    {
        if (v)
            state_g[rank] = static_cast<u32>(cand_begin + c);
    }
};

/// WinOut of the device-driven loop: the layer's first new state id and first candidate come from the device state.
struct WinOutDyn
{
    u32* state_g;
    const DevLayerState* d;
    __device__ __forceinline__ void operator()(u64 c, u64 rank, u32 v) const
    {
        if (v)
            state_g[d->n_states + rank] = static_cast<u32>(d->cand_next + c);
    }
};

// ------------------------------------------------------------------------------------------------ device-driven loop
// One iteration of a CUDA graph's while node per layer: k_g_begin, the count pass and its offsets scan, k_g_mid,
// k_g_clear, the expansion, the resolve pass, the winners scan, k_g_end (which sets the loop's condition). A layer that
// does not fit the buffers the graph was built over is left untouched (overflow) for the host loop.

/// The loop's initial state.
__global__ void k_g_init(DevLayerState* d, DevLayerState v) { *d = v; }

/// Layer start: the end conditions, the layer's parents, its counters.
__global__ void k_g_begin(DevLayerState* d)
{
    d->E = d->E_exp = d->G = 0;
    if (d->done || d->overflow)
        return;
    const u64 E = d->layer_end - d->layer_begin;
    if (E == 0)
    {
        d->exhausted = 1;
        d->done = 1;
        return;
    }
    if (d->layers == d->max_depth)
    {
        d->done = 1;
        return;
    }
    if (E > d->cap_layer || d->layers >= d->log_cap)
    {
        d->overflow = 1;
        return;
    }
    d->misc = LayerMisc{0, 0, 0, 0, 0xFFFFFFFFu, d->misc.status, 0};
    d->E = E;
}

/// After the count pass: the layer's candidates (up to the first goal parent when stopping at a goal), the check that
/// the buffers hold them, the goal bookkeeping.
__global__ void k_g_mid(DevLayerState* d, const u64* __restrict__ cand_base)
{
    if (d->E == 0)
        return;
    const u64 E = d->E;
    u64 E_exp = E, G = d->misc.total_cand;
    const u32 goals = d->misc.goals, first = d->misc.first_goal;
    const bool stop = goals && d->stop_at_goal;
    if (stop)
    {
        E_exp = first;
        if (E_exp < E)
            G = cand_base[E_exp];
    }
    const u64 room = (u64{1} << 32) - 1;
    if (G > d->cap_flags || d->cand_next + G > d->cap_cand || d->n_states + G > d->cap_states ||
        (d->n_states + G) * 4 > d->table_slots * 3 || G >= room - d->cand_next)
    {
        d->overflow = 1;  // nothing of this layer is kept: the host grows the buffers and runs it again
        d->E = 0;
        return;
    }
    if (goals && !d->solved)
    {
        d->solved = 1;
        d->goal_id = d->layer_begin + first;
    }
    d->goals += d->stop_at_goal ? (goals ? 1 : 0) : goals;
    d->stop = stop ? 1 : 0;
    d->E_exp = E_exp;
    d->G = G;
}

/// The layer's claimed and lost flags.
__global__ void k_g_clear(const DevLayerState* d, u8* __restrict__ claimed, u8* __restrict__ lost)
{
    const u64 G = d->G;
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < G; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        claimed[i] = 0;
        lost[i] = 0;
    }
}

/// After the winners scan: the layer's counts into the log, the next layer, the loop's condition.
__global__ void k_g_end(DevLayerState* d, cudaGraphConditionalHandle loop)
{
    if (d->E)
    {
        const u64 N = d->misc.total_new;
        u64* l = d->log + 3 * static_cast<u64>(d->layers);
        l[0] = d->E_exp;
        l[1] = d->G;
        l[2] = N;
        d->expanded += d->E_exp;
        d->generated += d->G;
        d->cand_next += d->G;
        d->n_states += N;
        d->layer_begin = d->layer_end;
        d->layer_end = d->n_states;
        d->layers += 1;
        if (d->stop || d->misc.status)
            d->done = 1;
        else if (d->stop_frontier && d->layer_end - d->layer_begin >= d->stop_frontier && d->layers < d->max_depth)
            d->done = d->cut = 1;
    }
    cudaGraphSetConditional(loop, d->done || d->overflow ? 0u : 1u);
}

__global__ void k_fingerprint(const u32* __restrict__ state_g, u64 first_id, u64 n, const u64* __restrict__ rows,
                              u32 W, u64* acc)
{
    u64 x = 0;
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < n; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 g = state_g[first_id + i];
        const GlobalRow r{rows + g * W, W};
        x ^= fingerprint_term(first_id + i, canonical_hash(r, W));
    }
    for (int o = 16; o > 0; o >>= 1)
        x ^= __shfl_xor_sync(0xFFFFFFFFu, x, o);
    if ((threadIdx.x & 31) == 0 && x)
        atomicXor(reinterpret_cast<unsigned long long*>(acc), x);
}

__global__ void k_gather_rows(const u32* __restrict__ state_g, u64 first, u64 n, const u64* __restrict__ rows, u32 W,
                              u64* __restrict__ out, u32 out_words)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < n; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 g = state_g[first + i];
        for (u32 w = 0; w < out_words; ++w)
            out[i * out_words + w] = w < W ? rows[g * W + w] : 0;
    }
}

__global__ void k_gather_hash(const u32* __restrict__ state_g, u64 first, u64 n, const u64* __restrict__ hash,
                              u64* __restrict__ out)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < n; i += static_cast<u64>(gridDim.x) * blockDim.x)
        out[i] = hash[state_g[first + i]];
}

__global__ void k_gather_nodes(const u32* __restrict__ state_g, u64 first, u64 n, const u32* __restrict__ par,
                               const u32* __restrict__ kid, const u64* __restrict__ layer_begin, u32 nlayers,
                               u32* __restrict__ out_parent, u32* __restrict__ out_index)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < n; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 id = first + i;
        const u64 g = state_g[id];
        if (id == 0)
        {
            out_parent[i] = 0xFFFFFFFFu;
            out_index[i] = 0;
            continue;
        }
        // layer L of id: layer_begin[L] <= id < layer_begin[L + 1]; its parents are in layer L - 1
        u32 lo = 0, hi = nlayers;
        while (hi - lo > 1)
        {
            const u32 mid = (lo + hi) / 2;
            if (layer_begin[mid] <= id)
                lo = mid;
            else
                hi = mid;
        }
        out_parent[i] = static_cast<u32>(layer_begin[lo - 1] + par[g]);
        out_index[i] = kid[g];
    }
}
}  // namespace
}  // namespace b2

using namespace b2;

namespace
{
/// Layer counters: two slots, so that the next layer's count can run before the host reads this layer's.
LayerMisc* misc_at(b2_brfs& B, unsigned slot) { return B.misc.as<LayerMisc>() + slot; }

void ensure_cand(b2_brfs& B, u64 need, u64 used)
{
    if (need <= B.cap_cand)
        return;
    const u64 cap = std::max<u64>(need, B.cap_cand + B.cap_cand / 2);
    B.rows.grow(cap * B.W * 8, used * B.W * 8, B.stream);
    B.hash.grow(cap * 8, used * 8, B.stream);
    B.par.grow(cap * 4, used * 4, B.stream);
    B.kid.grow(cap * 4, used * 4, B.stream);
    B.cap_cand = cap;
}

void ensure_states(b2_brfs& B, u64 need)
{
    if (need <= B.cap_states)
        return;
    const u64 cap = std::max<u64>(need, B.cap_states + B.cap_states / 2);
    B.state_g.grow(cap * 4, B.n_states * 4, B.stream);
    B.cap_states = cap;
}

void ensure_layer(b2_brfs& B, u64 E, u64 G)
{
    if (E > B.cap_layer)
    {
        const u64 cap = std::max<u64>(E, B.cap_layer * 2);
        B.counts.alloc(cap * 4, B.stream);
        B.cand_base.alloc((cap + 1) * 8, B.stream);
        B.sums.alloc(std::max(scan_scratch_bytes(cap), B.sums.bytes), B.stream);
        B.cap_layer = cap;
    }
    if (G > B.cap_flags)
    {
        const u64 cap = std::max<u64>(G, B.cap_flags * 2);
        B.flags.alloc(cap * 2 + 16, B.stream);
        B.deferred.alloc(cap * sizeof(u64), B.stream);
        if (B.sums.bytes < scan_scratch_bytes(cap))
            B.sums.alloc(scan_scratch_bytes(cap), B.stream);
        B.cap_flags = cap;
    }
}

/// Grows the hash set so that `states` entries keep it at most half full, and reinserts the stored states.
void ensure_table(b2_brfs& B, u64 states)
{
    // `states` is an upper bound (stored states + this layer's candidates): grow past 3/4 of it, to 1/2 load
    if (states * 4 <= B.table_slots * 3)
        return;
    u64 slots = B.table_slots ? B.table_slots : 1024;
    while (states * 2 > slots)
        slots *= 2;
    B.table.alloc(slots * 8, B.stream);
    B.table_slots = slots;
    B2_CUDA(cudaMemsetAsync(B.table.p, 0xFF, slots * 8, B.stream));
    if (B.n_states)
    {
        LayerMisc* misc = misc_at(B, B.slot);
        k_rehash<<<grid_for(B.n_states, 256), 256, 0, B.stream>>>(B.table.as<u64>(), slots - 1, max_probe(slots),
                                                                    B.state_g.as<u32>(), B.n_states, B.hash.as<u64>(),
                                                                    &misc->status);
        B2_CUDA(cudaGetLastError());
        ++B.rehashes;
        ++B.launches;
    }
}

Store make_store(b2_brfs& B, u64 layer_cand_begin)
{
    Store S;
    S.rows = B.rows.as<u64>();
    S.hash = B.hash.as<u64>();
    S.par = B.par.as<u32>();
    S.kid = B.kid.as<u32>();
    S.table = B.table.as<u64>();
    S.mask = B.table_slots - 1;
    S.W = B.W;
    S.max_probe = max_probe(B.table_slots);
    S.claimed = B.flags.as<u8>();
    S.lost = B.flags.as<u8>() + B.cap_flags;
    S.layer_cand_begin = layer_cand_begin;
    S.status = &misc_at(B, B.slot)->status;
    S.deferred = B.deferred.as<u64>();
    S.ndeferred = &misc_at(B, B.slot)->ndeferred;
    return S;
}

/// Waits for the stream and reads both counter slots: returns the current layer's, the other one into *other.
LayerMisc read_misc(b2_brfs& B, LayerMisc* other = nullptr)
{
    B2_CUDA(cudaMemcpyAsync(B.misc_host, B.misc.p, 2 * sizeof(LayerMisc), cudaMemcpyDeviceToHost, B.stream));
    const auto t0 = std::chrono::steady_clock::now();
    stream_wait(B.stream);
    B.wait_s += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    for (int k = 0; k < 2; ++k)
    {
        const u32 st = B.misc_host[k].status;
        if (st & kStatusProbeLimit)
            throw Error(B2_DEVICE_FAULT, "b2_brfs: a hash-set probe ran past its bound");
        if (st & kStatusScanStall)
            throw Error(B2_DEVICE_FAULT, "b2_brfs: a prefix scan gave up waiting for a tile");
        if (st)
            throw Error(B2_DEVICE_FAULT, "b2_brfs: device status " + std::to_string(st));
    }
    if (other)
        *other = B.misc_host[B.slot ^ 1];
    return B.misc_host[B.slot];
}

/// A finished one-GPU search's device buffers and layer-loop graph, kept in its context for the next search there
/// (b2_ctx::brfs_cache): repeated searches skip the allocations and the graph's capture and instantiation.
struct BrfsCache
{
    DeviceBuffer rows, hash, par, kid, state_g, table, counts, cand_base, flags, deferred, sums, dstate, dlog;
    u64 cap_cand = 0, cap_states = 0, table_slots = 0, cap_layer = 0, cap_flags = 0;
    u32 W = 0;
    cudaGraphExec_t graph_exec = nullptr;
    std::vector<u64> graph_key;
    ~BrfsCache()
    {
        if (graph_exec)
            cudaGraphExecDestroy(graph_exec);
    }
};

void exchange(b2_brfs& B, BrfsCache& C)
{
    DeviceBuffer* mine[] = {&B.rows,   &B.hash,      &B.par,   &B.kid,      &B.state_g, &B.table, &B.counts,
                            &B.cand_base, &B.flags, &B.deferred, &B.sums, &B.dstate, &B.dlog};
    DeviceBuffer* kept[] = {&C.rows,   &C.hash,      &C.par,   &C.kid,      &C.state_g, &C.table, &C.counts,
                            &C.cand_base, &C.flags, &C.deferred, &C.sums, &C.dstate, &C.dlog};
    for (size_t i = 0; i < std::size(mine); ++i)
        mine[i]->swap(*kept[i]);
    std::swap(B.cap_cand, C.cap_cand);
    std::swap(B.cap_states, C.cap_states);
    std::swap(B.table_slots, C.table_slots);
    std::swap(B.cap_layer, C.cap_layer);
    std::swap(B.cap_flags, C.cap_flags);
    std::swap(B.graph_exec, C.graph_exec);
    std::swap(B.graph_key, C.graph_key);
}

/// At the start of a one-GPU search: the context's kept buffers, if no other search holds them and they were sized for
/// rows of this width.
void cache_take(b2_brfs& B)
{
    b2_ctx* ctx = B.task->ctx;
    std::lock_guard lock(ctx->brfs_mu);
    if (ctx->brfs_cache_busy || !ctx->brfs_cache)
        return;
    auto* C = static_cast<BrfsCache*>(ctx->brfs_cache.get());
    if (C->W != B.W || !C->rows.p)
        return;
    exchange(B, *C);
    ctx->brfs_cache_busy = true;
    B.from_cache = true;
    // a buffer regrown during the search is freed in this search's stream order
    for (DeviceBuffer* b : {&B.rows, &B.hash, &B.par, &B.kid, &B.state_g, &B.table, &B.counts, &B.cand_base, &B.flags,
                            &B.deferred, &B.sums, &B.dstate, &B.dlog})
        b->stream = B.stream;
}

/// When a one-GPU search is released (its stream drained): its buffers and graph go back to the context if they came
/// from it, or replace the kept ones if no search holds those and they are not larger. What the search ends up holding
/// is freed by the caller.
void cache_give(b2_brfs& B)
{
    b2_ctx* ctx = B.task->ctx;
    std::lock_guard lock(ctx->brfs_mu);
    if (!ctx->brfs_cache)
        ctx->brfs_cache = std::shared_ptr<void>(new BrfsCache, [](void* p) { delete static_cast<BrfsCache*>(p); });
    auto* C = static_cast<BrfsCache*>(ctx->brfs_cache.get());
    if (B.from_cache)
    {
        exchange(B, *C);
        ctx->brfs_cache_busy = false;
        B.from_cache = false;
    }
    else if (!ctx->brfs_cache_busy && B.rows.p && B.cap_cand >= C->cap_cand)
        exchange(B, *C);
    else
        return;
    C->W = B.W;
    // kept buffers are freed (if ever) on no particular stream: the search's stream may be gone by then
    for (DeviceBuffer* b : {&C->rows, &C->hash, &C->par, &C->kid, &C->state_g, &C->table, &C->counts, &C->cand_base,
                            &C->flags, &C->deferred, &C->sums, &C->dstate, &C->dlog})
        b->stream = nullptr;
}

/// Layers the device-driven loop can log.
constexpr u32 kDeviceLogLayers = 4096;

/// The layer loop as one CUDA graph launch: a while node whose body is one layer (k_g_begin, count, offsets scan,
/// k_g_mid, k_g_clear, expansion, resolve, winners scan, k_g_end), over the buffers as they are now. Runs until the search
/// ends or a layer does not fit the buffers (DevLayerState::overflow: that layer is left to the host); returns the
/// final device state (its log copied into `log`).
void build_device_layers(b2_brfs& B, const std::vector<u64>& key, DevLayerState* d, u32 pi, unsigned sms);

DevLayerState run_device_layers(b2_brfs& B, const DevLayerState& init, std::vector<u64>& log)
{
    const Program& P = B.task->prog;
    const u32 pi = B.opt.witness_pruning ? 0 : 1;
    const unsigned sms = static_cast<unsigned>(B.task->ctx->sms);
    cudaStream_t s = B.stream;
    if (!B.dstate.p)
        B.dstate.alloc(sizeof(DevLayerState), s);
    if (!B.dlog.p)
        B.dlog.alloc(kDeviceLogLayers * 3 * sizeof(u64), s);
    DevLayerState* d = B.dstate.as<DevLayerState>();
    DevLayerState* host = reinterpret_cast<DevLayerState*>(reinterpret_cast<char*>(B.misc_host) + 128);
    static_assert(128 + sizeof(DevLayerState) <= PinnedPool::kBlock);
    DevLayerState v = init;
    v.log = B.dlog.as<u64>();
    v.log_cap = kDeviceLogLayers;
    v.cap_layer = B.cap_layer;
    v.cap_flags = B.cap_flags;
    v.cap_cand = B.cap_cand;
    v.cap_states = B.cap_states;
    v.table_slots = B.table_slots;
    k_g_init<<<1, 1, 0, s>>>(d, v);
    B2_CUDA(cudaGetLastError());
    ++B.launches;

    // the graph captures the buffers, the capacities the scans are sized for, the hash set's size and the kernels: an
    // earlier search's graph over the same ones is launched again as it is
    const std::vector<u64> key = {reinterpret_cast<u64>(B.rows.p),      reinterpret_cast<u64>(B.hash.p),
                                  reinterpret_cast<u64>(B.par.p),       reinterpret_cast<u64>(B.kid.p),
                                  reinterpret_cast<u64>(B.state_g.p),   reinterpret_cast<u64>(B.table.p),
                                  reinterpret_cast<u64>(B.counts.p),    reinterpret_cast<u64>(B.cand_base.p),
                                  reinterpret_cast<u64>(B.flags.p),     reinterpret_cast<u64>(B.deferred.p),
                                  reinterpret_cast<u64>(B.sums.p),      reinterpret_cast<u64>(d),
                                  B.cap_layer,                          B.cap_flags,
                                  B.table_slots,                        B.W,
                                  pi,                                   reinterpret_cast<u64>(B.task->jit->get(kJitBrfsCount, pi)),
                                  reinterpret_cast<u64>(B.task->jit->get(kJitBrfsExpand, pi)), sms};
    if (!B.graph_exec || B.graph_key != key)
        build_device_layers(B, key, d, pi, sms);
    B2_CUDA(cudaGraphLaunch(B.graph_exec, s));
    B.launches += 1;
    B2_CUDA(cudaMemcpyAsync(host, d, sizeof(DevLayerState), cudaMemcpyDeviceToHost, s));
    const auto t0 = std::chrono::steady_clock::now();
    stream_wait(s);
    B.wait_s += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    const DevLayerState r = *host;
    B.launches += static_cast<u64>(r.layers + (r.stop ? 0 : 1)) * 13;  // thirteen kernels per iteration
    log.assign(static_cast<size_t>(r.layers) * 3, 0);
    if (r.layers)
    {
        B2_CUDA(cudaMemcpyAsync(log.data(), B.dlog.p, log.size() * sizeof(u64), cudaMemcpyDeviceToHost, s));
        stream_wait(s);
    }
    (void)P;
    return r;
}

/// Captures and instantiates the device layer loop over the search's current buffers (into B.graph_exec).
void build_device_layers(b2_brfs& B, const std::vector<u64>& key, DevLayerState* d, u32 pi, unsigned sms)
{
    if (B.graph_exec)
    {
        cudaGraphExecDestroy(B.graph_exec);
        B.graph_exec = nullptr;
    }
    if (!B.capture)
        B2_CUDA(cudaStreamCreateWithFlags(&B.capture, cudaStreamNonBlocking));
    cudaGraph_t graph = nullptr;
    struct GraphGuard
    {
        cudaGraph_t& g;
        ~GraphGuard()
        {
            if (g)
                cudaGraphDestroy(g);
        }
    } guard{graph};
    B2_CUDA(cudaGraphCreate(&graph, 0));
    cudaGraphConditionalHandle loop;
    B2_CUDA(cudaGraphConditionalHandleCreate(&loop, graph, 1, cudaGraphCondAssignDefault));
    cudaGraphNodeParams cp{};
    cp.type = cudaGraphNodeTypeConditional;
    cp.conditional.handle = loop;
    cp.conditional.type = cudaGraphCondTypeWhile;
    cp.conditional.size = 1;
    cudaGraphNode_t node;
    B2_CUDA(cudaGraphAddNode(&node, graph, nullptr, 0, &cp));
    cudaGraph_t body = cp.conditional.phGraph_out[0];

    cudaStream_t c = B.capture;
    (void)scan_blocks(1);  // the SM count is read outside the capture
    B2_CUDA(cudaStreamBeginCaptureToGraph(c, body, nullptr, nullptr, 0, cudaStreamCaptureModeThreadLocal));
    Store S = make_store(B, 0);
    S.status = &d->misc.status;
    S.ndeferred = &d->misc.ndeferred;
    k_g_begin<<<1, 1, 0, c>>>(d);
    {
        dev::BrfsArgs a{};
        a.frontier = B.state_g.as<u32>();
        a.counts = B.counts.as<u32>();
        a.misc = &d->misc;
        a.S = S;
        a.pi = pi;
        a.dyn = d;
        jit_launch(B.task->jit->get(kJitBrfsCount, pi), sms * 16, 128, &a, c);
    }
    device_scan_dev(CountIn{B.counts.as<u32>()}, BaseOut{B.cand_base.as<u64>()}, &d->E, B.cap_layer,
                    &d->misc.total_cand, B.sums.as<u64>(), c, &d->misc.status);
    k_g_mid<<<1, 1, 0, c>>>(d, B.cand_base.as<u64>());
    k_g_clear<<<sms * 4, 256, 0, c>>>(d, S.claimed, S.lost);
    {
        dev::BrfsArgs a{};
        a.frontier = B.state_g.as<u32>();
        a.cand_base = B.cand_base.as<u64>();
        a.misc = &d->misc;
        a.S = S;
        a.pi = pi;
        a.dyn = d;
        jit_launch(B.task->jit->get(kJitBrfsExpand, pi), sms * dev::kBrfsExpandBlocksPerSm, 128, &a, c);
    }
    k_resolve<<<sms * 8, 256, 0, c>>>(S, d);
    device_scan_dev(WinIn{S.claimed, S.lost}, WinOutDyn{B.state_g.as<u32>(), d}, &d->G, B.cap_flags,
                    &d->misc.total_new, B.sums.as<u64>(), c, &d->misc.status);
    k_g_end<<<1, 1, 0, c>>>(d, loop);
    B2_CUDA(cudaGetLastError());
    cudaGraph_t captured = nullptr;
    B2_CUDA(cudaStreamEndCapture(c, &captured));
    B2_CUDA(cudaGraphInstantiate(&B.graph_exec, graph, 0));
    B.graph_key = key;
}

/// The one-GPU search. With prefix_states, it stops after the first layer whose new states number at least
/// prefix_states, before expanding them, and returns true (the search goes on elsewhere: a sharded search takes over
/// from there). Otherwise, and when it ends before that layer, it returns false.
bool run_search(b2_brfs& B, b2_brfs_result& R, u64 prefix_states = 0)
{
    const auto t0 = std::chrono::steady_clock::now();
    const Program& P = B.task->prog;
    const DevTask& T = B.task->dev;
    const b2_brfs_options& o = B.opt;
    const u32 pi = o.witness_pruning ? 0 : 1;
    const u32 W = B.W;
    cudaStream_t s = B.stream;
    cudaEvent_t ev[5];
    for (auto& e : ev)
        B2_CUDA(cudaEventCreate(&e));
    struct EvGuard
    {
        cudaEvent_t* e;
        ~EvGuard()
        {
            for (int i = 0; i < 5; ++i)
                cudaEventDestroy(e[i]);
        }
    } guard{ev};

    R.states = 1;
    R.words = W;
    if (o.stop_at_goal && P.goal_unsat)
    {
        R.status = B2_SEARCH_UNSOLVABLE;
        B.n_states = 1;
        return false;
    }
    bool cut = false;
    // root
    cache_take(B);
    if (B.table_slots)  // kept from an earlier search: emptied (a table grown below is emptied on allocation)
        B2_CUDA(cudaMemsetAsync(B.table.p, 0xFF, B.table_slots * 8, s));
    const u64 expect = std::max<u64>(o.expected_states, 1024);
    ensure_cand(B, expect * 2, 0);
    ensure_states(B, expect);
    if (o.expected_states)
        ensure_layer(B, expect / 2, expect);  // a layer holds at most the states, and about twice as many candidates
    B.misc.alloc(2 * sizeof(LayerMisc), s);
    static_assert(2 * sizeof(LayerMisc) <= PinnedPool::kBlock);
    if (!B.misc_host)
        B.misc_host = static_cast<LayerMisc*>(B.task->ctx->pinned.take());
    B2_CUDA(cudaMemsetAsync(B.misc.p, 0, 2 * sizeof(LayerMisc), s));
    B.slot = 0;
    B.wait_s = 0;
    ensure_table(B, expect);
    B2_CUDA(cudaMemcpyAsync(B.rows.p, P.initial.data(), W * 8, cudaMemcpyHostToDevice, s));
    k_seed_root<<<1, 1, 0, s>>>(make_store(B, 0), B.state_g.as<u32>());
    B2_CUDA(cudaGetLastError());
    ++B.launches;
    B.n_states = 1;
    u64 cand_next = 1;  // candidate 0 is the root
    u64 layer_begin = 0, layer_end = 1;
    B.layer_begin.assign(1, 0);
    u32 layers = 0;
    bool exhausted = false, solved = false, full = false;
    u64 expanded = 0, generated = 0, goals = 0, goal_id = 0, fingerprint = 0;
    double count_ms = 0, gen_ms = 0, dedup_ms = 0;
    std::vector<std::array<u64, 3>> counts;
    // The count pass of a layer: successors per parent, their offsets and total, goals among the parents, into the
    // counter slot `misc`. The parents are E, or, when E_dev is non-null, a count still on the device that is at most
    // E_max (the next layer's, launched before the host has read it).
    const auto launch_count = [&](const u32* frontier, u64 E, const u64* E_dev, u64 E_max, LayerMisc* misc,
                                  u64 cand_begin) {
        const unsigned grid = grid_for(E_max, 128, static_cast<unsigned>(B.task->ctx->sms) * 64);
        k_layer_init<<<1, 1, 0, s>>>(misc);
        if (o.timings)
            B2_CUDA(cudaEventRecord(ev[0], s));
        if (B.task->jit)
        {
            dev::BrfsArgs a{};
            a.frontier = frontier;
            a.E = E;
            a.E_dev = E_dev;
            a.counts = B.counts.as<u32>();
            a.misc = misc;
            a.S = make_store(B, cand_begin);
            a.pi = pi;
            jit_launch(B.task->jit->get(kJitBrfsCount, pi), grid, 128, &a, s);
        }
        else
            dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                k_count<OW, WR><<<grid, 128, 0, s>>>(T, pi, B.rows.as<u64>(), W, frontier, E, B.counts.as<u32>(), misc,
                                                     E_dev);
            });
        if (E_dev)
            device_scan_dev(CountIn{B.counts.as<u32>()}, BaseOut{B.cand_base.as<u64>()}, E_dev, E_max,
                            &misc->total_cand, B.sums.as<u64>(), s, &misc->status);
        else
            device_scan(CountIn{B.counts.as<u32>()}, BaseOut{B.cand_base.as<u64>()}, E, &misc->total_cand,
                        B.sums.as<u64>(), s, &misc->status);
        B2_CUDA(cudaGetLastError());
        B.launches += 5;
        if (o.timings)
            B2_CUDA(cudaEventRecord(ev[1], s));
    };
    bool counted = false;  // this layer's count already ran (launched with the previous layer), its counters in `next`
    LayerMisc next{};
    bool finished = false;
    // With the buffers presized (expected_states), no per-layer events and no max_states cut, the layers run as one
    // graph launch on the device; a layer that outgrows the buffers continues in the host loop below.
    if (B.task->jit && !o.timings && o.max_states == ~u64{0} && o.expected_states > 0)
    {
        DevLayerState init{};
        init.layer_begin = 0;
        init.layer_end = 1;
        init.n_states = 1;
        init.cand_next = 1;
        init.max_depth = o.max_depth;
        init.stop_at_goal = o.stop_at_goal ? 1 : 0;
        init.stop_frontier = prefix_states;
        std::vector<u64> log;
        const DevLayerState r = run_device_layers(B, init, log);
        if (r.misc.status & kStatusProbeLimit)
            throw Error(B2_DEVICE_FAULT, "b2_brfs: a hash-set probe ran past its bound");
        if (r.misc.status & kStatusScanStall)
            throw Error(B2_DEVICE_FAULT, "b2_brfs: a prefix scan gave up waiting for a tile");
        if (r.misc.status)
            throw Error(B2_DEVICE_FAULT, "b2_brfs: device status " + std::to_string(r.misc.status));
        u64 end = 1;
        for (u32 k = 0; k < r.layers; ++k)
        {
            counts.push_back({log[3 * k], log[3 * k + 1], log[3 * k + 2]});
            B.layer_begin.push_back(end);
            end += log[3 * k + 2];
        }
        layers = r.layers;
        expanded = r.expanded;
        generated = r.generated;
        goals = r.goals;
        solved = r.solved != 0;
        goal_id = r.goal_id;
        exhausted = r.exhausted != 0;
        cand_next = r.cand_next;
        B.n_states = r.n_states;
        layer_begin = r.layer_begin;
        layer_end = r.layer_end;
        finished = r.done != 0;
        cut = r.cut != 0;
    }
    while (!finished)
    {
        const u64 E = layer_end - layer_begin;
        if (E == 0)
        {
            exhausted = true;
            break;
        }
        if (layers == o.max_depth)
            break;
        if (B.n_states >= o.max_states)
        {
            full = true;  // the store is full before the layer (max_states <= 1)
            break;
        }
        ++layers;
        LayerMisc* misc = misc_at(B, B.slot);
        LayerMisc m;
        if (counted)
            m = next;
        else
        {
            ensure_layer(B, E, 0);
            launch_count(B.state_g.as<u32>() + layer_begin, E, nullptr, E, misc, cand_next);
            m = read_misc(B);
        }
        counted = false;
        if (o.timings)
        {
            float a = 0;
            B2_CUDA(cudaEventElapsedTime(&a, ev[0], ev[1]));
            count_ms += a;
        }
        u64 E_exp = E, G = m.total_cand;
        bool stop = false;
        const u32 layer_goals = m.goals, first_goal = m.first_goal;
        if (layer_goals && o.stop_at_goal)
        {
            E_exp = first_goal;
            if (E_exp < E)
                B2_CUDA(cudaMemcpyAsync(&G, B.cand_base.as<u64>() + E_exp, 8, cudaMemcpyDeviceToHost, s));
            stream_wait(s);
            stop = true;
        }
        if (G >= (u64{1} << 32) - 1 - cand_next)
            throw Error(B2_CAPACITY, "b2_brfs: more than 2^32 - 2 candidates");
        ensure_layer(B, E, G);
        ensure_cand(B, cand_next + G, cand_next);
        ensure_states(B, B.n_states + G);
        ensure_table(B, B.n_states + G);
        u64 N = 0;
        if (E_exp > 0 && G > 0)
        {
            B2_CUDA(cudaMemsetAsync(B.flags.p, 0, G, s));
            B2_CUDA(cudaMemsetAsync(B.flags.as<u8>() + B.cap_flags, 0, G, s));
            if (o.timings)
                B2_CUDA(cudaEventRecord(ev[2], s));
            const Store S = make_store(B, cand_next);
            const u32* frontier = B.state_g.as<u32>() + layer_begin;
            const unsigned grid_e = grid_for(E_exp, 128, static_cast<unsigned>(B.task->ctx->sms) * 64);
            if (B.task->jit)
            {
                dev::BrfsArgs a{};
                a.frontier = frontier;
                a.E = E_exp;
                a.cand_base = B.cand_base.as<u64>();
                a.misc = misc;
                a.S = S;
                a.pi = pi;
                jit_launch(B.task->jit->get(kJitBrfsExpand, pi), grid_e, 128, &a, s);
            }
            else
                dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                    k_expand<OW, WR><<<grid_e, 128, 0, s>>>(T, pi, frontier, E_exp, B.cand_base.as<u64>(), S);
                });
            k_resolve<<<static_cast<unsigned>(B.task->ctx->sms) * 8, 256, 0, s>>>(S);
            B2_CUDA(cudaGetLastError());
            ++B.launches;
            if (o.timings)
                B2_CUDA(cudaEventRecord(ev[3], s));
            device_scan(WinIn{S.claimed, S.lost}, WinOut{B.state_g.as<u32>() + B.n_states, cand_next}, G,
                        &misc->total_new, B.sums.as<u64>(), s, &misc->status);
            B.launches += 4;
            if (o.timings)
                B2_CUDA(cudaEventRecord(ev[4], s));
            // The next layer's count, launched now over this layer's new states (at most G, their number still on
            // the device), so that one wait returns both. Skipped where this layer may be the last: a goal stop, the
            // depth bound, or a store that this layer can fill (max_states stops inside the layer).
            if (!stop && layers < o.max_depth && B.n_states + G < o.max_states)
            {
                ensure_layer(B, G, 0);
                launch_count(B.state_g.as<u32>() + B.n_states, 0, &misc->total_new, G, misc_at(B, B.slot ^ 1),
                             cand_next + G);
                counted = true;
            }
            m = read_misc(B, &next);
            N = m.total_new;
            if (o.timings)
            {
                float b = 0, c = 0;
                B2_CUDA(cudaEventElapsedTime(&b, ev[2], ev[3]));
                B2_CUDA(cudaEventElapsedTime(&c, ev[3], ev[4]));
                gen_ms += b;
                dedup_ms += c;
            }
        }
        // the goal parents reached: under stop_at_goal the first one (expansion stops there), else all of them
        u64 goals_layer = o.stop_at_goal ? (layer_goals ? 1 : 0) : layer_goals;
        bool goal_reached = layer_goals > 0;
        if (B.n_states + N >= o.max_states && N > 0)
        {
            // max_states: the search stops right after storing state max_states - 1 (inside its parent's expansion,
            // as run_flat does, src/mymyr/search/brfs.cpp:301-384): the layer's parents up to that parent are
            // expanded, its successors up to that candidate generated
            const u64 last = o.max_states - 1;
            u32 gstar = 0, pstar = 0;
            B2_CUDA(cudaMemcpyAsync(&gstar, B.state_g.as<u32>() + last, 4, cudaMemcpyDeviceToHost, s));
            stream_wait(s);
            B2_CUDA(cudaMemcpyAsync(&pstar, B.par.as<u32>() + gstar, 4, cudaMemcpyDeviceToHost, s));
            stream_wait(s);
            N = o.max_states - B.n_states;
            E_exp = static_cast<u64>(pstar) + 1;
            G = gstar - cand_next + 1;
            full = stop = true;
            if (o.stop_at_goal)
            {
                goals_layer = 0;  // the layer's first goal parent lies after the cut (E_exp was at most it)
                goal_reached = false;
            }
            else
            {
                B2_CUDA(cudaMemsetAsync(&misc->goals, 0, 4, s));
                k_count_goals<<<grid_for(E_exp, 256), 256, 0, s>>>(T, B.rows.as<u64>(), W,
                                                                     B.state_g.as<u32>() + layer_begin, E_exp,
                                                                     &misc->goals);
                B2_CUDA(cudaGetLastError());
                ++B.launches;
                goals_layer = read_misc(B).goals;
                goal_reached = layer_goals > 0 && first_goal <= pstar;
            }
        }
        if (goal_reached && !solved)
        {
            solved = true;
            goal_id = layer_begin + first_goal;
        }
        goals += goals_layer;
        expanded += E_exp;
        generated += G;
        counts.push_back({E_exp, G, N});
        cand_next += G;
        B.n_states += N;
        layer_begin = layer_end;
        layer_end = B.n_states;
        B.layer_begin.push_back(layer_begin);
        if (stop)
            break;
        if (prefix_states && layer_end - layer_begin >= prefix_states && layers < o.max_depth)
        {
            cut = true;  // the next layer is large enough to shard
            break;
        }
        if (counted)
            B.slot ^= 1;
    }
    stream_wait(s);  // a next layer's count launched before the cut has finished with the buffers
    B.layer_begin.push_back(B.n_states);
    if (o.fingerprint)
    {
        u64* acc = &misc_at(B, B.slot)->fingerprint;
        B2_CUDA(cudaMemsetAsync(acc, 0, 8, s));
        k_fingerprint<<<grid_for(B.n_states, 256, static_cast<unsigned>(B.task->ctx->sms) * 8), 256, 0, s>>>(
            B.state_g.as<u32>(), 0, B.n_states, B.rows.as<u64>(), W, acc);
        B2_CUDA(cudaGetLastError());
        ++B.launches;
        fingerprint = read_misc(B).fingerprint;
    }
    stream_wait(s);
    R.states = B.n_states;
    R.expanded = expanded;
    R.generated = generated;
    R.num_goal_states = goals;
    R.layers = layers;
    R.exhausted = exhausted ? 1 : 0;
    R.solved = solved ? 1 : 0;
    R.goal_id = solved ? goal_id : 0;
    R.fingerprint = fingerprint;
    R.count_ms = count_ms;
    R.gen_ms = gen_ms;
    R.dedup_ms = dedup_ms;
    R.wait_ms = B.wait_s * 1000;
    R.kernel_launches = B.launches;
    R.status = solved ? B2_SEARCH_SOLVED
                      : full ? B2_SEARCH_OUT_OF_STATES
                             : (exhausted || layers >= o.max_depth ? B2_SEARCH_EXHAUSTED : B2_SEARCH_OUT_OF_STATES);
    R.rehashes = B.rehashes;
    u32 lg = 0;
    while ((u64{1} << lg) < B.table_slots)
        ++lg;
    R.table_log2 = lg;
    if (R.layer_counts)
        for (u32 i = 0; i < counts.size() && i < R.layer_capacity; ++i)
            for (int k = 0; k < 3; ++k)
                R.layer_counts[3 * i + k] = counts[i][k];
    R.search_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    return cut;
}
}  // namespace

bool b2::run_prefix(b2_brfs& B, b2_brfs_result& R, u64 prefix_states)
{
    B.ran_one_gpu = true;  // its buffers (and any layer-loop graph) go to the context's cache for the next search
    return run_search(B, R, prefix_states);
}

extern "C" {

void b2_brfs_options_default(b2_brfs_options* o)
{
    if (!o)
        return;
    *o = b2_brfs_options{};
    o->witness_pruning = 1;
    o->stop_at_goal = 1;
    o->fingerprint = 0;
    o->max_depth = 0xFFFFFFFFu;
    o->max_states = ~uint64_t{0};
    o->expected_states = 0;
    o->timings = 0;
    o->world_rank = 0;
    o->world_size = 1;
}

b2_status b2_brfs_create(b2_task* task, const b2_brfs_options* options, b2_brfs** out)
{
    return guarded([&] {
        if (!task || !options || !out)
            throw std::invalid_argument("b2_brfs_create: null argument");
        if (!task->ctx)
            throw std::invalid_argument("a host-only task (created without a context) cannot run on the device");
        if (options->comm)
        {
            if (options->comm->device != task->ctx->device)
                throw std::invalid_argument("b2_brfs_create: the communicator belongs to another device");
            if ((options->world_size != 1 || options->world_rank != 0) &&
                (options->world_size != static_cast<int32_t>(options->comm->world) ||
                 options->world_rank != static_cast<int32_t>(options->comm->rank)))
                throw std::invalid_argument("b2_brfs_create: world_rank/world_size differ from the communicator's");
        }
        else if (options->world_size != 1 || options->world_rank != 0)
            throw std::invalid_argument("b2_brfs_create: world_size > 1 needs a communicator (options.comm)");
        if (options->witness_pruning && task->witness_refused)
            throw Error(B2_UNSUPPORTED, "witness pruning with a witness parameter before an effect parameter");
        B2_CUDA(cudaSetDevice(task->ctx->device));
        auto b = std::make_unique<b2_brfs>();
        b->task = task;
        b->opt = *options;
        b->W = task->prog.words;
        b->comm = options->comm;
        if (options->stream)
            b->stream = static_cast<cudaStream_t>(options->stream);
        else
        {
            B2_CUDA(cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking));
            b->own_stream = true;
        }
        *out = b.release();
    });
}

b2_status b2_brfs_run(b2_brfs* search, b2_brfs_result* result)
{
    return guarded([&] {
        if (!search || !result)
            throw std::invalid_argument("b2_brfs_run: null argument");
        if (search->ran)
            throw std::invalid_argument("b2_brfs_run: the search ran already");
        search->ran = true;
        B2_CUDA(cudaSetDevice(search->task->ctx->device));
        uint64_t* lc = result->layer_counts;
        const uint32_t cap = result->layer_capacity;
        *result = b2_brfs_result{};
        result->layer_counts = lc;
        result->layer_capacity = cap;
        if (search->comm)
            shard_run(*search, *result);
        else
        {
            run_search(*search, *result);
            result->local_states = search->n_states;
        }
    });
}

b2_status b2_brfs_states(b2_brfs* B, uint64_t first, uint64_t count, uint64_t* rows, uint32_t words)
{
    return guarded([&] {
        if (B && B->comm)
            throw std::invalid_argument("b2_brfs_states: a sharded search's states are read per rank (b2_brfs_local)");
        if (!B || (count && !rows) || !B->ran)
            throw std::invalid_argument("b2_brfs_states: bad argument");
        if (first + count > B->n_states || words < B->W)
            throw std::invalid_argument("b2_brfs_states: range or width out of bounds");
        if (!count)
            return;
        DeviceBuffer tmp;
        tmp.alloc(count * words * 8);
        k_gather_rows<<<grid_for(count, 256), 256, 0, B->stream>>>(B->state_g.as<u32>(), first, count, B->rows.as<u64>(),
                                                                   B->W, tmp.as<u64>(), words);
        B2_CUDA(cudaGetLastError());
        B2_CUDA(cudaMemcpyAsync(rows, tmp.p, count * words * 8, cudaMemcpyDeviceToHost, B->stream));
        B2_CUDA(cudaStreamSynchronize(B->stream));
    });
}

b2_status b2_brfs_state_hashes(b2_brfs* B, uint64_t first, uint64_t count, uint64_t* hashes)
{
    return guarded([&] {
        if (B && B->comm)
            throw std::invalid_argument("b2_brfs_state_hashes: a sharded search's states are read per rank (b2_brfs_local)");
        if (!B || (count && !hashes) || !B->ran || first + count > B->n_states)
            throw std::invalid_argument("b2_brfs_state_hashes: bad argument");
        if (!count)
            return;
        DeviceBuffer tmp;
        tmp.alloc(count * 8);
        k_gather_hash<<<grid_for(count, 256), 256, 0, B->stream>>>(B->state_g.as<u32>(), first, count,
                                                                   B->hash.as<u64>(), tmp.as<u64>());
        B2_CUDA(cudaGetLastError());
        B2_CUDA(cudaMemcpyAsync(hashes, tmp.p, count * 8, cudaMemcpyDeviceToHost, B->stream));
        B2_CUDA(cudaStreamSynchronize(B->stream));
    });
}

b2_status b2_brfs_nodes(b2_brfs* B, uint64_t first, uint64_t count, uint32_t* parent, uint32_t* index)
{
    return guarded([&] {
        if (B && B->comm)
            throw std::invalid_argument("b2_brfs_nodes: a sharded search's states are read per rank (b2_brfs_local)");
        if (!B || (count && (!parent || !index)) || !B->ran || first + count > B->n_states)
            throw std::invalid_argument("b2_brfs_nodes: bad argument");
        if (!count)
            return;
        DeviceBuffer tmp, lb;
        tmp.alloc(count * 8);
        lb.alloc(B->layer_begin.size() * 8);
        B2_CUDA(cudaMemcpyAsync(lb.p, B->layer_begin.data(), B->layer_begin.size() * 8, cudaMemcpyHostToDevice, B->stream));
        u32* tp = tmp.as<u32>();
        k_gather_nodes<<<grid_for(count, 256), 256, 0, B->stream>>>(B->state_g.as<u32>(), first, count, B->par.as<u32>(),
                                                                    B->kid.as<u32>(), lb.as<u64>(),
                                                                    static_cast<u32>(B->layer_begin.size()), tp, tp + count);
        B2_CUDA(cudaGetLastError());
        B2_CUDA(cudaMemcpyAsync(parent, tp, count * 4, cudaMemcpyDeviceToHost, B->stream));
        B2_CUDA(cudaMemcpyAsync(index, tp + count, count * 4, cudaMemcpyDeviceToHost, B->stream));
        B2_CUDA(cudaStreamSynchronize(B->stream));
    });
}

static void rethrow(b2_status st)
{
    if (st == B2_OK)
        return;
    char msg[1024];
    b2_last_error(msg, sizeof msg);
    throw Error(st, msg);
}

b2_status b2_brfs_local_count(b2_brfs* B, uint64_t* count)
{
    return guarded([&] {
        if (!B || !count || !B->ran)
            throw std::invalid_argument("b2_brfs_local_count: bad argument");
        *count = B->comm ? shard_local_count(*B) : B->n_states;
    });
}

b2_status b2_brfs_local(b2_brfs* B, uint64_t first, uint64_t count, uint64_t* ids, uint64_t* rows, uint32_t words,
                        uint64_t* hashes, uint32_t* parent, uint32_t* index)
{
    return guarded([&] {
        if (!B || !B->ran)
            throw std::invalid_argument("b2_brfs_local: bad argument");
        B2_CUDA(cudaSetDevice(B->task->ctx->device));
        if (B->comm)
        {
            shard_local(*B, first, count, ids, rows, words, hashes, parent, index);
            return;
        }
        if (first + count > B->n_states || (rows && words < B->W))
            throw std::invalid_argument("b2_brfs_local: range or width out of bounds");
        if (ids)
            for (uint64_t i = 0; i < count; ++i)
                ids[i] = first + i;
        if (rows)
            rethrow(b2_brfs_states(B, first, count, rows, words));
        if (hashes)
            rethrow(b2_brfs_state_hashes(B, first, count, hashes));
        if (parent || index)
        {
            std::vector<uint32_t> p(parent ? 0 : count), k(index ? 0 : count);
            rethrow(b2_brfs_nodes(B, first, count, parent ? parent : p.data(), index ? index : k.data()));
        }
    });
}

void b2_brfs_destroy(b2_brfs* search)
{
    if (!search)
        return;
    cudaSetDevice(search->task->ctx->device);
    // the buffers are freed in stream order (after the search's last kernel), with no wait here
    if (search->shard)
        shard_free(*search);
    if (search->stream)
    {
        if (search->ran && (!search->shard || search->ran_one_gpu))
        {
            // an idle search's buffers (and layer-loop graph) are kept by the context for its next search
            stream_drain(search->stream);
            cache_give(*search);
        }
        if (search->graph_exec)
            cudaGraphExecDestroy(search->graph_exec);
        for (DeviceBuffer* b : {&search->rows, &search->hash, &search->par, &search->kid, &search->state_g,
                                &search->table, &search->counts, &search->cand_base, &search->flags, &search->deferred,
                                &search->sums, &search->misc, &search->dstate, &search->dlog})
            b->reset();
        // the status mirror goes back to the context's pool once no copy into it can be pending
        stream_drain(search->stream);
        if (search->own_stream)
            cudaStreamDestroy(search->stream);
    }
    if (search->capture)
        cudaStreamDestroy(search->capture);
    search->task->ctx->pinned.give(search->misc_host);
    delete search;
}

}  // extern "C"
