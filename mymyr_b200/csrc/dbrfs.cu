// The BrFS sharded over the ranks of a communicator (one GPU per rank), with the ids, layer counts and fingerprint of
// the one-GPU search (brfs.cu) and of the reference's run_flat with deterministic ids
// (src/mymyr/search/brfs.cpp:273-404, discoverer order :1657-1778). The reference has no multi-GPU search; this is the
// hash-owner partition of its visited set.
//
// Ownership. State s lives on rank owner(hash::state(s)) (the hash's high 32 bits scaled to the ranks): its row, hash
// and node record sit in that rank's arena, its slot in that rank's hash set, and that rank expands it.
//
// Per layer (parents: the layer's states, ids [layer_begin, layer_end), each on its owner):
//   1. count: each rank counts the successors of its parents (and tests the goal); the counts are scattered to a
//      layer-wide array by parent id and summed over ranks (NCCL all-reduce), whose exclusive scan gives every
//      successor its candidate index c in canonical order (parent id, successor index) over the whole layer;
//   2. expand: each rank regenerates its parents' successors into a staging area as records [row | hash | c] and
//      counts them per owner; the ranks all-gather the per-owner counts, so every rank knows where its records go in
//      every owner's receive buffer;
//   3. push: one kernel writes the records straight into the owners' receive buffers in peer memory (NVLink stores
//      through CUDA IPC mappings; no library copy), then a one-word all-reduce orders the exchange before the inserts;
//   4. insert: each owner inserts its received records into its hash set: a record that takes an empty slot is a new
//      state; an equal record of the same layer keeps the smallest c at that slot's entry (atomicMin), an equal state
//      of an earlier layer drops it. The smallest c of a state is its first discovery in canonical order;
//   5. ids: each owner flags its new states' c in a layer-wide byte array; the all-reduced flags' exclusive scan gives
//      every new state its id (the one-GPU id), and the scan of the rank's own flags gives its local order, so each
//      rank keeps its states in id order. The node record (parent id, successor index) comes from c by a binary search
//      of the layer's candidate offsets.
// Every decision the host takes (stop, capacities, buffer growth) uses values that all ranks share, so the ranks take
// the same collective steps in the same order.

#include "brfs.cuh"

#include <array>
#include <chrono>
#include <cstring>

namespace b2
{
namespace
{
using dev::DExpandArgs;
using dev::DistMisc;
using dev::kMaxWorld;
using dev::owner_of;

__global__ void k_dseed(u64* __restrict__ rows, u64* __restrict__ hash, u32 W, u64* table, u64 mask, u32 max_probe,
                        u32 me, u32 world, u32* state_lc, u32* state_id, u32* state_par, u32* state_kid, DistMisc* misc)
{
    const GlobalRow r{rows, W};
    const u64 h = hash_words([&](u32 q) { return r.word(q); }, W);
    hash[0] = h;
    if (owner_of(h, world) != me)
    {
        misc->new_packed = 1;
        return;
    }
    u64 j = h & mask;
    for (u32 probe = 0; probe < max_probe && table[j] != kEmpty; ++probe)
        j = (j + 1) & mask;
    if (table[j] == kEmpty)
        table[j] = h & 0xFFFFFFFF00000000ull;  // arena index 0
    else
        atomicOr(&misc->lm.status, kStatusProbeLimit);
    state_lc[0] = 0;
    state_id[0] = 0;
    state_par[0] = 0xFFFFFFFFu;
    state_kid[0] = 0;
    misc->new_packed = 1 | (u64{1} << 32);
}

/// The local successor counts into the layer-wide array (by parent id), and the rank's goal count and first goal id.
__global__ void k_dscatter(const u32* __restrict__ counts, const u32* __restrict__ ids, u64 E, u64 layer_begin,
                           u32* __restrict__ cg, u64 n_layer, DistMisc* misc)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < E; i += static_cast<u64>(gridDim.x) * blockDim.x)
        cg[ids[i] - layer_begin] = counts[i];
    if (blockIdx.x == 0 && threadIdx.x == 0)
    {
        cg[n_layer] = misc->lm.goals;
        misc->goal_id = misc->lm.first_goal != 0xFFFFFFFFu ? ids[misc->lm.first_goal] : ~u64{0};
    }
}

/// The owner's inserts of its received records (all of them in memory before this kernel, so rows are compared in
/// place with no ordering within the kernel). Table entries are (hash >> 32) << 32 | arena index; the arena index of
/// received record r is cand_begin + r, and its row stays in the receive buffer during the layer.
__global__ void k_dinsert(const u64* __restrict__ recv, const u64* __restrict__ M, u32 me, u32 world,
                          u64* __restrict__ rows, u64* __restrict__ hash, u64* table, u64 mask, u32 max_probe,
                          u64 cand_begin, u32 W, u32* gmin, u8* __restrict__ claimed, DistMisc* misc)
{
    u64 n = 0;
    for (u32 s = 0; s < world; ++s)
        n += M[s * world + me];
    if (blockIdx.x == 0 && threadIdx.x == 0)
    {
        misc->recv = n;
        misc->lm.ndeferred = static_cast<u32>(n - M[me * world + me]);  // received from other ranks
    }
    const u32 RW = W + 2;
    for (u64 r = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; r < n; r += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64* rec = recv + r * RW;
        const u64 h = rec[W];
        const u32 c = static_cast<u32>(rec[W + 1]);
        const u64 lc = cand_begin + r;
        const u64 mine = (h & 0xFFFFFFFF00000000ull) | lc;
        u64 j = h & mask;
        bool done = false;
        for (u32 probe = 0; probe < max_probe; ++probe, j = (j + 1) & mask)
        {
            u64 cur = __ldcg(table + j);
            if (cur == kEmpty)
            {
                const u64 prev = atomicCAS(reinterpret_cast<unsigned long long*>(table + j), kEmpty, mine);
                if (prev == kEmpty)
                {
                    u64* dst = rows + lc * W;
                    for (u32 q = 0; q < W; ++q)
                        dst[q] = rec[q];
                    hash[lc] = h;
                    claimed[r] = 1;
                    atomicMin(gmin + r, c);
                    done = true;
                    break;
                }
                cur = prev;
            }
            if ((cur >> 32) != (mine >> 32))
                continue;
            const u64 o = cur & 0xFFFFFFFFull;
            const bool this_layer = o >= cand_begin;
            const u64* orow = this_layer ? recv + (o - cand_begin) * RW : rows + o * W;
            bool eq = true;
            for (u32 q = 0; q < W && eq; ++q)
                eq = orow[q] == rec[q];
            if (!eq)
                continue;
            if (this_layer)
                atomicMin(gmin + (o - cand_begin), c);
            done = true;
            break;
        }
        if (!done)
            atomicOr(&misc->lm.status, kStatusProbeLimit);
    }
}

/// Flags the candidate index of each new state of this rank (its smallest discovery) and remembers its arena index.
__global__ void k_dmark(const u64* __restrict__ M, u32 me, u32 world, const u8* __restrict__ claimed,
                        const u32* __restrict__ gmin, u64 cand_begin, u8* __restrict__ fm, u32* __restrict__ mark)
{
    u64 n = 0;
    for (u32 s = 0; s < world; ++s)
        n += M[s * world + me];
    for (u64 r = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; r < n; r += static_cast<u64>(gridDim.x) * blockDim.x)
        if (claimed[r])
        {
            const u32 c = gmin[r];
            fm[c] = 1;
            mark[c] = static_cast<u32>(cand_begin + r);
        }
}

/// Packed flags of candidate c: new state of any rank (low half) | new state of this rank (high half).
struct PackIn
{
    const u8* f;
    const u8* fm;
    __device__ __forceinline__ u64 operator()(u64 c) const { return f[c] | (static_cast<u64>(fm[c]) << 32); }
};
struct PackOut
{
    const u32* mark;
    const u64* gbase;  // candidate offsets of the layer's expanded parents
    u64 parents;
    u64 layer_begin, layer_end, n_local;
    u32* state_lc;
    u32* state_id;
    u32* state_par;
    u32* state_kid;
    __device__ __forceinline__ void operator()(u64 c, u64 e, u64 v) const
    {
        if (!(v >> 32))
            return;
        const u64 lp = n_local + (e >> 32);
        state_lc[lp] = mark[c];
        state_id[lp] = static_cast<u32>(layer_end + (e & 0xFFFFFFFFull));
        // the parent: the last p with gbase[p] <= c (it has successors, since c < gbase[p + 1])
        u64 lo = 0, hi = parents;
        while (hi - lo > 1)
        {
            const u64 mid = (lo + hi) / 2;
            if (gbase[mid] <= c)
                lo = mid;
            else
                hi = mid;
        }
        state_par[lp] = static_cast<u32>(layer_begin + lo);
        state_kid[lp] = static_cast<u32>(c - gbase[lo]);
    }
};

__global__ void k_dfingerprint(const u32* __restrict__ state_lc, const u32* __restrict__ state_id, u64 n,
                               const u64* __restrict__ rows, u32 W, u64* acc)
{
    u64 x = 0;
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < n; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const GlobalRow r{rows + static_cast<u64>(state_lc[i]) * W, W};
        x ^= fingerprint_term(state_id[i], canonical_hash(r, W));
    }
    for (int o = 16; o > 0; o >>= 1)
        x ^= __shfl_xor_sync(0xFFFFFFFFu, x, o);
    if ((threadIdx.x & 31) == 0 && x)
        atomicXor(reinterpret_cast<unsigned long long*>(acc), x);
}

/// Local states [first, first + n): ids, rows (out_words each), hashes, node records (NULL outputs skipped).
__global__ void k_dgather(const u32* __restrict__ state_lc, const u32* __restrict__ state_id,
                          const u32* __restrict__ state_par, const u32* __restrict__ state_kid, u64 first, u64 n,
                          const u64* __restrict__ rows, const u64* __restrict__ hash, u32 W, u64* ids, u64* out_rows,
                          u32 out_words, u64* hashes, u32* parent, u32* index)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < n; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 s = first + i;
        const u64 lc = state_lc[s];
        if (ids)
            ids[i] = state_id[s];
        if (out_rows)
            for (u32 w = 0; w < out_words; ++w)
                out_rows[i * out_words + w] = w < W ? rows[lc * W + w] : 0;
        if (hashes)
            hashes[i] = hash[lc];
        if (parent)
            parent[i] = state_par[s];
        if (index)
            index[i] = state_kid[s];
    }
}
}  // namespace

/// A rank's part of a sharded search.
struct ShardState
{
    u32 rank = 0, world = 1;
    // per local candidate (arena): rows and hashes of the received records that took a slot
    DeviceBuffer rows, hash;
    u64 cap_cand = 0, cand_next = 0;
    // per local state, in id order: arena index, id, parent id, successor index
    DeviceBuffer state_lc, state_id, state_par, state_kid;
    u64 cap_states = 0, n_local = 0;
    DeviceBuffer table;
    u64 table_slots = 0;
    u32 rehashes = 0;
    // per local parent of the layer
    DeviceBuffer counts, local_base;
    u64 cap_local = 0;
    // per parent of the layer (all ranks)
    DeviceBuffer cg, gbase;
    u64 cap_layer = 0;
    // staged records
    DeviceBuffer staging;
    u64 cap_staging = 0;
    // per candidate of the layer (all ranks): flags, the all-reduced flags, arena index; per received record: its
    // state's smallest candidate index, whether it took a slot
    DeviceBuffer fm, f, mark, gmin, claimed;
    u64 cap_g = 0;
    DeviceBuffer small;  // hist[world] | M[world, world] | cursor[world] | fingerprints[world]
    DeviceBuffer misc, sums;
    DistMisc* misc_host = nullptr;
    std::vector<u64> layer_begin;
    u64 n_total = 0;
    u64 exchanged = 0;  // records received from other ranks
    u64* hist() { return small.as<u64>(); }
    u64* matrix() { return small.as<u64>() + world; }
    u64* cursor() { return small.as<u64>() + world + world * world; }
    u64* prints() { return small.as<u64>() + 2 * world + world * world; }
};

namespace
{
u64 grown(u64 need, u64 cap) { return std::max<u64>(need, cap + cap / 2); }

void ensure_scan(ShardState& S, u64 n, cudaStream_t s)
{
    if (S.sums.bytes < scan_scratch_bytes(n))
        S.sums.alloc(scan_scratch_bytes(grown(n, 0)), s);
}

void ensure_cand(ShardState& S, u32 W, u64 need, cudaStream_t s)
{
    if (need <= S.cap_cand)
        return;
    const u64 cap = grown(need, S.cap_cand);
    S.rows.grow(cap * W * 8, S.cand_next * W * 8, s);
    S.hash.grow(cap * 8, S.cand_next * 8, s);
    S.cap_cand = cap;
}

void ensure_states(ShardState& S, u64 need, cudaStream_t s)
{
    if (need <= S.cap_states)
        return;
    const u64 cap = grown(need, S.cap_states);
    for (DeviceBuffer* b : {&S.state_lc, &S.state_id, &S.state_par, &S.state_kid})
        b->grow(cap * 4, S.n_local * 4, s);
    S.cap_states = cap;
}

void ensure_local(ShardState& S, u64 E, cudaStream_t s)
{
    if (E > S.cap_local)
    {
        const u64 cap = grown(E, S.cap_local);
        S.counts.alloc(cap * 4, s);
        S.local_base.alloc((cap + 1) * 8, s);
        S.cap_local = cap;
    }
    ensure_scan(S, E, s);
}

void ensure_layer(ShardState& S, u64 n, cudaStream_t s)
{
    if (n > S.cap_layer)
    {
        const u64 cap = grown(n, S.cap_layer);
        S.cg.alloc((cap + 1) * 4, s);
        S.gbase.alloc((cap + 1) * 8, s);
        S.cap_layer = cap;
    }
    ensure_scan(S, n, s);
}

void ensure_g(ShardState& S, u64 G, cudaStream_t s)
{
    if (G > S.cap_g)
    {
        const u64 cap = grown(G, S.cap_g);
        S.fm.alloc(cap, s);
        S.f.alloc(cap, s);
        S.mark.alloc(cap * 4, s);
        S.gmin.alloc(cap * 4, s);
        S.claimed.alloc(cap, s);
        S.cap_g = cap;
    }
    ensure_scan(S, G, s);
}

/// Collective (every rank passes the same G and W): the communicator's receive buffers hold G records.
void ensure_recv(b2_comm* comm, u32 W, u64 G, cudaStream_t s)
{
    const u64 need = G * (W + 2) * 8;
    if (need <= comm->exchange.bytes)
        return;
    peer_buffer_exchange(comm, comm->exchange, std::max<u64>(grown(need, comm->exchange.bytes), u64{1} << 20), s);
}

void ensure_table(ShardState& S, u64 bound, DistMisc* misc, cudaStream_t s, u64& launches)
{
    if (bound * 4 <= S.table_slots * 3)
        return;
    u64 slots = S.table_slots ? S.table_slots : 1024;
    while (bound * 2 > slots)
        slots *= 2;
    S.table.alloc(slots * 8, s);
    S.table_slots = slots;
    B2_CUDA(cudaMemsetAsync(S.table.p, 0xFF, slots * 8, s));
    if (S.n_local)
    {
        k_rehash<<<grid_for(S.n_local, 256), 256, 0, s>>>(S.table.as<u64>(), slots - 1, max_probe(slots),
                                                            S.state_lc.as<u32>(), S.n_local, S.hash.as<u64>(),
                                                            &misc->lm.status);
        B2_CUDA(cudaGetLastError());
        ++S.rehashes;
        ++launches;
    }
}

const DistMisc& read_misc(ShardState& S, b2_comm* comm, cudaStream_t s)
{
    B2_CUDA(cudaMemcpyAsync(S.misc_host, S.misc.p, sizeof(DistMisc), cudaMemcpyDeviceToHost, s));
    comm_sync(comm, s);
    const DistMisc& m = *S.misc_host;
    if (m.lm.status & kStatusProbeLimit)
        throw Error(B2_DEVICE_FAULT, "b2_brfs: a hash-set probe ran past its bound");
    if (m.lm.status)
        throw Error(B2_DEVICE_FAULT, "b2_brfs: device status " + std::to_string(m.lm.status));
    return m;
}
}  // namespace

void shard_run(b2_brfs& B, b2_brfs_result& R)
{
    const auto t0 = std::chrono::steady_clock::now();
    if (!B.shard)
        B.shard = new ShardState;
    ShardState& S = *B.shard;
    b2_comm* comm = B.comm;
    S.rank = comm->rank;
    S.world = comm->world;
    const u32 me = S.rank, world = S.world;
    const Program& P = B.task->prog;
    const DevTask& T = B.task->dev;
    const b2_brfs_options& o = B.opt;
    const u32 pi = o.witness_pruning ? 0 : 1;
    const u32 W = B.W, RW = W + 2;
    const unsigned sms = static_cast<unsigned>(B.task->ctx->sms);
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
    const u64 expect = std::max<u64>(o.expected_states / world + o.expected_states / (4 * world), 1024);
    ensure_cand(S, W, expect * 2, s);
    ensure_states(S, expect, s);
    S.misc.alloc(sizeof(DistMisc), s);
    static_assert(sizeof(DistMisc) <= PinnedPool::kBlock);
    if (!S.misc_host)
        S.misc_host = static_cast<DistMisc*>(B.task->ctx->pinned.take());
    S.small.alloc((3 * world + world * world) * 8, s);
    B2_CUDA(cudaMemsetAsync(S.misc.p, 0, sizeof(DistMisc), s));
    DistMisc* misc = S.misc.as<DistMisc>();
    ensure_table(S, expect, misc, s, B.launches);
    // the root: arena index 0 on every rank, stored by its owner
    B2_CUDA(cudaMemcpyAsync(S.rows.p, P.initial.data(), W * 8, cudaMemcpyHostToDevice, s));
    k_dseed<<<1, 1, 0, s>>>(S.rows.as<u64>(), S.hash.as<u64>(), W, S.table.as<u64>(), S.table_slots - 1,
                            max_probe(S.table_slots), me, world, S.state_lc.as<u32>(), S.state_id.as<u32>(),
                            S.state_par.as<u32>(), S.state_kid.as<u32>(), misc);
    B2_CUDA(cudaGetLastError());
    ++B.launches;
    S.n_local = read_misc(S, comm, s).new_packed >> 32;
    S.cand_next = 1;
    S.n_total = 1;
    B.n_states = 1;
    if (o.stop_at_goal && P.goal_unsat)
    {
        R.status = B2_SEARCH_UNSOLVABLE;
        S.layer_begin = {0, 1};
        return;
    }
    u64 layer_begin = 0, layer_end = 1, lb_local = 0, le_local = S.n_local;
    S.layer_begin.assign(1, 0);
    u32 layers = 0;
    bool exhausted = false, solved = false;
    u64 expanded = 0, generated = 0, goals = 0, goal_id = 0;
    double count_ms = 0, gen_ms = 0, dedup_ms = 0;
    std::vector<std::array<u64, 3>> counts;
    for (;;)
    {
        const u64 E = layer_end - layer_begin, El = le_local - lb_local;
        if (E == 0)
        {
            exhausted = true;
            break;
        }
        if (layers == o.max_depth)
            break;
        ++layers;
        ensure_local(S, El, s);
        ensure_layer(S, E, s);
        *S.misc_host = DistMisc{};
        S.misc_host->lm.first_goal = 0xFFFFFFFFu;
        B2_CUDA(cudaMemcpyAsync(misc, S.misc_host, sizeof(DistMisc), cudaMemcpyHostToDevice, s));
        B2_CUDA(cudaMemsetAsync(S.cg.p, 0, (E + 1) * 4, s));
        const u32* frontier = S.state_lc.as<u32>() + lb_local;
        const u32* frontier_id = S.state_id.as<u32>() + lb_local;
        if (o.timings)
            B2_CUDA(cudaEventRecord(ev[0], s));
        if (El)
        {
            const unsigned grid = grid_for(El, 128, sms * 64);
            if (B.task->jit)
            {
                dev::BrfsArgs a{};
                a.frontier = frontier;
                a.E = El;
                a.counts = S.counts.as<u32>();
                a.misc = &misc->lm;
                a.S.rows = S.rows.as<u64>();
                a.S.W = W;
                a.pi = pi;
                jit_launch(B.task->jit->brfs_count[pi], grid, 128, &a, s);
            }
            else
                dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                    k_count<OW, WR><<<grid, 128, 0, s>>>(T, pi, S.rows.as<u64>(), W, frontier, El,
                                                         S.counts.as<u32>(), &misc->lm);
                });
            ++B.launches;
        }
        k_dscatter<<<grid_for(El, 256, sms * 8), 256, 0, s>>>(S.counts.as<u32>(), frontier_id, El, layer_begin,
                                                              S.cg.as<u32>(), E, misc);
        B2_CUDA(cudaGetLastError());
        comm_group_begin();
        comm_allreduce(comm, S.cg.p, S.cg.p, E + 1, CommType::U32, CommOp::Sum, s);
        comm_allreduce(comm, &misc->goal_id, &misc->goal_id, 1, CommType::U64, CommOp::Min, s);
        comm_group_end();
        B2_CUDA(cudaMemcpyAsync(&misc->goals_all, S.cg.as<u32>() + E, 4, cudaMemcpyDeviceToDevice, s));
        device_scan(CountIn{S.cg.as<u32>()}, BaseOut{S.gbase.as<u64>()}, E, &misc->lm.total_cand, S.sums.as<u64>(), s);
        device_scan(CountIn{S.counts.as<u32>()}, BaseOut{S.local_base.as<u64>()}, El, &misc->total_local,
                    S.sums.as<u64>(), s);
        B.launches += 7;
        if (o.timings)
            B2_CUDA(cudaEventRecord(ev[1], s));
        const DistMisc m1 = read_misc(S, comm, s);
        u64 limit = layer_end, G = m1.lm.total_cand;
        bool stop = false;
        if (m1.goals_all)
        {
            if (!solved)
            {
                solved = true;
                goal_id = m1.goal_id;
            }
            if (o.stop_at_goal)
            {
                limit = m1.goal_id;
                if (limit < layer_end)
                {
                    B2_CUDA(cudaMemcpyAsync(&G, S.gbase.as<u64>() + (limit - layer_begin), 8, cudaMemcpyDeviceToHost, s));
                    comm_sync(comm, s);
                }
                goals += 1;
                stop = true;
            }
            else
                goals += m1.goals_all;
        }
        const u64 E_exp = limit - layer_begin;
        if (S.n_total + G >= (u64{1} << 32) - 1 || S.cand_next + G >= (u64{1} << 32) - 1)
            throw Error(B2_CAPACITY, "b2_brfs: more than 2^32 - 2 states or candidates on a rank");
        u64 N = 0, N_local = 0;
        if (E_exp > 0 && G > 0)
        {
            ensure_g(S, G, s);
            ensure_recv(comm, W, G, s);
            if (S.cap_staging < m1.total_local)
            {
                S.cap_staging = grown(m1.total_local, S.cap_staging);
                S.staging.alloc(S.cap_staging * RW * 8, s);
            }
            ensure_cand(S, W, S.cand_next + G, s);
            ensure_states(S, S.n_local + G, s);
            ensure_table(S, S.n_local + G, misc, s, B.launches);
            B2_CUDA(cudaMemsetAsync(S.small.p, 0, (3 * world + world * world) * 8, s));
            B2_CUDA(cudaMemsetAsync(S.fm.p, 0, G, s));
            B2_CUDA(cudaMemsetAsync(S.claimed.p, 0, G, s));
            B2_CUDA(cudaMemsetAsync(S.gmin.p, 0xFF, G * 4, s));
            if (o.timings)
                B2_CUDA(cudaEventRecord(ev[2], s));
            // the state arrays may have moved (ensure_states)
            frontier = S.state_lc.as<u32>() + lb_local;
            frontier_id = S.state_id.as<u32>() + lb_local;
            if (El)
            {
                DExpandArgs a{};
                a.rows = S.rows.as<u64>();
                a.frontier = frontier;
                a.frontier_id = frontier_id;
                a.E = El;
                a.layer_begin = layer_begin;
                a.limit = limit;
                a.gbase = S.gbase.as<u64>();
                a.local_base = S.local_base.as<u64>();
                a.staging = S.staging.as<u64>();
                a.hist = S.hist();
                a.world = world;
                a.W = W;
                a.pi = pi;
                const unsigned grid = grid_for(El, 128, sms * 64);
                if (B.task->jit)
                    jit_launch(B.task->jit->dbrfs_expand[pi], grid, 128, &a, s);
                else
                    dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                        k_dexpand<OW, WR><<<grid, 128, 0, s>>>(T, a);
                    });
                ++B.launches;
            }
            comm_allgather(comm, S.hist(), S.matrix(), world, CommType::U64, s);
            const u32 tile = std::min<u32>(kPushThreads, kPushSmemWords / RW);
            k_push<<<grid_for(m1.total_local, tile, sms * 8), kPushThreads, tile * RW * 8, s>>>(
                S.staging.as<u64>(), S.matrix(), reinterpret_cast<u64* const*>(comm->exchange.table.p),
                reinterpret_cast<unsigned long long*>(S.cursor()), me, world, RW, tile);
            B2_CUDA(cudaGetLastError());
            comm_allreduce(comm, &misc->barrier, &misc->barrier, 1, CommType::U32, CommOp::Sum, s);
            k_dinsert<<<sms * 8, 256, 0, s>>>(static_cast<const u64*>(comm->exchange.local.p), S.matrix(), me, world,
                                              S.rows.as<u64>(), S.hash.as<u64>(), S.table.as<u64>(), S.table_slots - 1,
                                              max_probe(S.table_slots), S.cand_next, W, S.gmin.as<u32>(),
                                              S.claimed.as<u8>(), misc);
            B2_CUDA(cudaGetLastError());
            if (o.timings)
                B2_CUDA(cudaEventRecord(ev[3], s));
            k_dmark<<<sms * 8, 256, 0, s>>>(S.matrix(), me, world, S.claimed.as<u8>(), S.gmin.as<u32>(), S.cand_next,
                                            S.fm.as<u8>(), S.mark.as<u32>());
            B2_CUDA(cudaGetLastError());
            comm_allreduce(comm, S.fm.p, S.f.p, G, CommType::U8, CommOp::Sum, s);
            PackOut out{S.mark.as<u32>(), S.gbase.as<u64>(), E_exp, layer_begin, layer_end, S.n_local,
                        S.state_lc.as<u32>(), S.state_id.as<u32>(), S.state_par.as<u32>(), S.state_kid.as<u32>()};
            device_scan(PackIn{S.f.as<u8>(), S.fm.as<u8>()}, out, G, &misc->new_packed, S.sums.as<u64>(), s);
            B.launches += 6;
            if (o.timings)
                B2_CUDA(cudaEventRecord(ev[4], s));
            const DistMisc& m3 = read_misc(S, comm, s);
            N = m3.new_packed & 0xFFFFFFFFull;
            N_local = m3.new_packed >> 32;
            S.cand_next += m3.recv;
            S.exchanged += m3.lm.ndeferred;
            if (o.timings)
            {
                float a = 0, b = 0, c = 0;
                B2_CUDA(cudaEventElapsedTime(&a, ev[0], ev[1]));
                B2_CUDA(cudaEventElapsedTime(&b, ev[2], ev[3]));
                B2_CUDA(cudaEventElapsedTime(&c, ev[3], ev[4]));
                count_ms += a;
                gen_ms += b;
                dedup_ms += c;
            }
        }
        expanded += E_exp;
        generated += G;
        counts.push_back({E_exp, G, N});
        S.n_local += N_local;
        S.n_total += N;
        lb_local = le_local;
        le_local = S.n_local;
        layer_begin = layer_end;
        layer_end = S.n_total;
        S.layer_begin.push_back(layer_begin);
        if (stop)
            break;
    }
    S.layer_begin.push_back(S.n_total);
    B.n_states = S.n_total;
    u64 fingerprint = 0;
    if (o.fingerprint)
    {
        B2_CUDA(cudaMemsetAsync(&misc->fingerprint, 0, 8, s));
        k_dfingerprint<<<grid_for(S.n_local, 256, sms * 8), 256, 0, s>>>(S.state_lc.as<u32>(), S.state_id.as<u32>(),
                                                                         S.n_local, S.rows.as<u64>(), W,
                                                                         &misc->fingerprint);
        B2_CUDA(cudaGetLastError());
        comm_allgather(comm, &misc->fingerprint, S.prints(), 1, CommType::U64, s);
        std::vector<u64> prints(world);
        B2_CUDA(cudaMemcpyAsync(prints.data(), S.prints(), world * 8, cudaMemcpyDeviceToHost, s));
        comm_sync(comm, s);
        ++B.launches;
        for (u64 x : prints)
            fingerprint ^= x;
    }
    comm_sync(comm, s);
    R.states = S.n_total;
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
    R.kernel_launches = B.launches;
    R.status = solved ? B2_SEARCH_SOLVED
                      : (exhausted || layers >= o.max_depth ? B2_SEARCH_EXHAUSTED : B2_SEARCH_OUT_OF_STATES);
    R.rehashes = S.rehashes;
    R.exchanged = S.exchanged;
    R.local_states = S.n_local;
    u32 lg = 0;
    while ((u64{1} << lg) < S.table_slots)
        ++lg;
    R.table_log2 = lg;
    if (R.layer_counts)
        for (u32 i = 0; i < counts.size() && i < R.layer_capacity; ++i)
            for (int k = 0; k < 3; ++k)
                R.layer_counts[3 * i + k] = counts[i][k];
    R.search_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

u64 shard_local_count(const b2_brfs& B) { return B.shard ? B.shard->n_local : 0; }

void shard_local(b2_brfs& B, u64 first, u64 count, u64* ids, u64* rows, u32 words, u64* hashes, u32* parent,
                 u32* index)
{
    ShardState& S = *B.shard;
    if (first + count > S.n_local || (rows && words < B.W))
        throw std::invalid_argument("b2_brfs_local: range or width out of bounds");
    if (!count)
        return;
    const u64 per = (ids ? 8 : 0) + (rows ? 8ull * words : 0) + (hashes ? 8 : 0) + (parent ? 4 : 0) + (index ? 4 : 0);
    DeviceBuffer tmp;
    tmp.alloc(count * per + 64);
    char* p = tmp.as<char>();
    auto take = [&](u64 bytes) {
        char* q = p;
        p += bytes;
        return q;
    };
    u64* d_ids = ids ? reinterpret_cast<u64*>(take(count * 8)) : nullptr;
    u64* d_rows = rows ? reinterpret_cast<u64*>(take(count * 8ull * words)) : nullptr;
    u64* d_hash = hashes ? reinterpret_cast<u64*>(take(count * 8)) : nullptr;
    u32* d_par = parent ? reinterpret_cast<u32*>(take(count * 4)) : nullptr;
    u32* d_kid = index ? reinterpret_cast<u32*>(take(count * 4)) : nullptr;
    k_dgather<<<grid_for(count, 256), 256, 0, B.stream>>>(S.state_lc.as<u32>(), S.state_id.as<u32>(),
                                                          S.state_par.as<u32>(), S.state_kid.as<u32>(), first, count,
                                                          S.rows.as<u64>(), S.hash.as<u64>(), B.W, d_ids, d_rows, words,
                                                          d_hash, d_par, d_kid);
    B2_CUDA(cudaGetLastError());
    if (ids)
        B2_CUDA(cudaMemcpyAsync(ids, d_ids, count * 8, cudaMemcpyDeviceToHost, B.stream));
    if (rows)
        B2_CUDA(cudaMemcpyAsync(rows, d_rows, count * 8ull * words, cudaMemcpyDeviceToHost, B.stream));
    if (hashes)
        B2_CUDA(cudaMemcpyAsync(hashes, d_hash, count * 8, cudaMemcpyDeviceToHost, B.stream));
    if (parent)
        B2_CUDA(cudaMemcpyAsync(parent, d_par, count * 4, cudaMemcpyDeviceToHost, B.stream));
    if (index)
        B2_CUDA(cudaMemcpyAsync(index, d_kid, count * 4, cudaMemcpyDeviceToHost, B.stream));
    B2_CUDA(cudaStreamSynchronize(B.stream));
}

void shard_free(b2_brfs& B)
{
    if (!B.shard)
        return;
    ShardState& S = *B.shard;
    for (DeviceBuffer* b : {&S.rows, &S.hash, &S.state_lc, &S.state_id, &S.state_par, &S.state_kid, &S.table,
                            &S.counts, &S.local_base, &S.cg, &S.gbase, &S.staging, &S.fm, &S.f, &S.mark, &S.gmin,
                            &S.claimed, &S.small, &S.misc, &S.sums})
        b->reset();
    B.task->ctx->pinned.give(S.misc_host);
    delete B.shard;
    B.shard = nullptr;
}
}  // namespace b2
