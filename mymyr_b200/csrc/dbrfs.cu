// The BrFS sharded over the ranks of a communicator (one GPU per rank), with the ids, layer counts and fingerprint of
// the one-GPU search (brfs.cu) and of the reference's run_flat with deterministic ids
// (src/mymyr/search/brfs.cpp:273-404, discoverer order :1657-1778). The reference has no multi-GPU search; this is the
// hash-owner partition of its visited set.
//
// Ownership. State s lives on rank owner(hash::state(s)) (the hash's high 32 bits scaled to the ranks): its row, hash
// and node record sit in that rank's arena, its slot in that rank's hash set, and that rank expands it.
//
// Per layer (parents: the layer's states, ids [layer_begin, layer_end), each on its owner):
//   1. count: each rank counts the successors of its parents (and tests the goal); the counts go into a layer-wide
//      array of byte lanes by parent id (each lane written by the parent's owner alone; word lanes for the rest of the
//      search once a parent has more than 255 successors) and are summed over ranks (NCCL all-reduce), whose
//      exclusive scan gives every parent the candidate index of its first successor in canonical order;
//   2. expand: each rank regenerates its parents' successors into a staging area as records [row | hash | key], key =
//      parent id << 32 | successor index (the canonical order);
//   3. push: one kernel writes the records straight into the owners' receive buffers in peer memory (NVLink stores
//      through CUDA IPC mappings; no library copy), each block reserving its run in an owner's buffer by an atomic on
//      that owner's fill cursor; then a one-word all-reduce orders the exchange before the inserts;
//   4. insert: each owner inserts its received records into its hash set: a record that takes an empty slot is a new
//      state; an equal record of the same layer keeps the smallest key at that slot's entry (atomicMin), an equal
//      state of an earlier layer drops it. The smallest key of a state is its first discovery in canonical order;
//   5. ids: each owner sets the bit of its new states' candidate index c (the parent's offset + successor index) in a
//      layer-wide bitmap; the all-reduced bitmap's exclusive popcount scan gives every new state its id (the one-GPU
//      id), and the scan of the rank's own bits its local order, so each rank keeps its states in id order. The node
//      record (parent id, successor index) is the key.
// Every decision the host takes (stop, capacities, buffer growth) uses values that all ranks share, so the ranks take
// the same collective steps in the same order. The next layer's count (step 1) is launched right after step 5, over
// parents whose number is still on the device, so that one wait per layer returns both: the counters alternate
// between two slots.

#include "brfs.cuh"

#include <array>
#include <chrono>
#include <cstddef>
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

/// The states a rank owns among those of a one-GPU search that every rank ran alone (the replicated small layers):
/// scanned over the state ids, in id order, so that local index l of the rank's states is the exclusive count of
/// owned ids before it.
struct OwnIn
{
    const u32* state_g;  // id -> candidate index of the one-GPU store
    const u64* hash;     // per candidate
    u32 me, world;
    __device__ __forceinline__ u32 operator()(u64 id) const { return owner_of(hash[state_g[id]], world) == me ? 1u : 0u; }
};
/// Copies an owned state into the rank's arena and state lists (arena index = local index) and records the local
/// index of the frontier's first id.
struct OwnOut
{
    const u32* state_g;
    const u64* rows;  // one-GPU rows, hashes and node records (parent index in its layer, successor index)
    const u64* hash;
    const u32* par;
    const u32* kid;
    const u64* layer_begin;  // the one-GPU search's layer starts, nlayers of them
    u32 nlayers;
    u32 W;
    u64 frontier_begin;  // id of the frontier's first state
    u64* rows_out;
    u64* hash_out;
    u32* state_lc;
    u32* state_id;
    u32* state_par;
    u32* state_kid;
    u64* frontier_local;  // out: the local index of the frontier's first state
    __device__ __forceinline__ void operator()(u64 id, u64 l, u32 own) const
    {
        if (id == frontier_begin)
            *frontier_local = l;
        if (!own)
            return;
        const u64 g = state_g[id];
        for (u32 q = 0; q < W; ++q)
            rows_out[l * W + q] = rows[g * W + q];
        hash_out[l] = hash[g];
        state_lc[l] = static_cast<u32>(l);
        state_id[l] = static_cast<u32>(id);
        state_kid[l] = id == 0 ? 0u : kid[g];
        if (id == 0)
        {
            state_par[l] = 0xFFFFFFFFu;
            return;
        }
        u32 lo = 0, hi = nlayers;  // layer L of id: layer_begin[L] <= id < layer_begin[L + 1]
        while (hi - lo > 1)
        {
            const u32 mid = (lo + hi) / 2;
            if (layer_begin[mid] <= id)
                lo = mid;
            else
                hi = mid;
        }
        state_par[l] = static_cast<u32>(layer_begin[lo - 1] + par[g]);
    }
};

/// The local successor counts into the layer-wide lane array (by parent id: bytes for lane 1, words for lane 4), then
/// after the lanes: the rank's goal parents, its parents whose count does not fit a byte lane (saturated, counted), and
/// its row of the per-owner successor counts M[rank][owner]; and the rank's first goal id. A parent's lane and a rank's
/// row are written by one rank alone, so the all-reduce sums without carries.
__global__ void k_dscatter(const u32* __restrict__ counts, const u32* __restrict__ ids, u64 E_in, const u64* E_dev,
                           u64 layer_begin, u32* __restrict__ cg, u64 lane_words, u32 lane, const u64* __restrict__ hist,
                           u32 me, u32 world, DistMisc* misc)
{
    const u64 E = E_dev ? *E_dev : E_in;  // the local parents (a count still on the device when E_dev is set)
    u32* tail = cg + lane_words;  // [goals, overflow, M[world][world]]
    if (blockIdx.x == 0)
        for (u32 d = threadIdx.x; d < world; d += blockDim.x)
            tail[2 + me * world + d] = static_cast<u32>(hist[d]);
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < E; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 j = ids[i] - layer_begin;
        const u32 c = counts[i];
        if (lane == 4)
            cg[j] = c;
        else
        {
            if (c > 0xFFu)
                atomicAdd(tail + 1, 1u);
            reinterpret_cast<u8*>(cg)[j] = static_cast<u8>(c > 0xFFu ? 0xFFu : c);
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0)
    {
        tail[0] = misc->lm.goals;
        misc->goal_id = misc->lm.first_goal != 0xFFFFFFFFu ? ids[misc->lm.first_goal] : ~u64{0};
    }
}

/// From the summed tail: the layer's goal parents and overflowing parents over all ranks, the successors this rank
/// owns and the most any rank owns.
__global__ void k_dtail(const u32* __restrict__ tail, u32 me, u32 world, DistMisc* misc)
{
    if (threadIdx.x != 0)
        return;
    misc->goals_all = tail[0];
    misc->overflow_all = tail[1];
    u64 most = 0;
    for (u32 d = 0; d < world; ++d)
    {
        u64 n = 0;
        for (u32 s = 0; s < world; ++s)
            n += tail[2 + s * world + d];
        if (d == me)
            misc->recv_me = n;
        most = n > most ? n : most;
    }
    misc->recv_max = most;
}

/// The count of parent i from the summed lanes.
struct LaneIn
{
    const u32* cg;
    u32 lane;
    __device__ __forceinline__ u32 operator()(u64 i) const
    {
        return lane == 4 ? cg[i] : static_cast<u32>(reinterpret_cast<const u8*>(cg)[i]);
    }
};

/// The owner's inserts of its received records (all of them in memory before this kernel, so rows are compared in
/// place with no ordering within the kernel). Table entries are (hash >> 32) << 32 | arena index; the arena index of
/// received record r is cand_begin + r, and its row stays in the receive buffer during the layer. gmin[r] ends as the
/// smallest key of record r's state if r took a slot, and stays all ones otherwise. The received records are the
/// first *fill of the buffer (its cursor, advanced by all senders).
__global__ void k_dinsert(const u64* __restrict__ recv, const u64* fill, u64* __restrict__ rows, u64* __restrict__ hash,
                          u64* table, u64 mask, u32 max_probe, u64 cand_begin, u32 W, unsigned long long* gmin,
                          DistMisc* misc, u64 cap)
{
    // the fill cursor counts every reservation, also those a sender dropped past the buffer (its overflow flag fails
    // the layer on every rank): only the records that fit are read
    const u64 n = min(*fill, cap);
    if (blockIdx.x == 0 && threadIdx.x == 0)
    {
        misc->recv = n;
        misc->lm.ndeferred = static_cast<u32>(n - misc->sent_self);  // received from other ranks
    }
    const u32 RW = W + 2;
    for (u64 r = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; r < n; r += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64* rec = recv + r * RW;
        const u64 h = rec[W];
        const u64 key = rec[W + 1];
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
                    atomicMin(gmin + r, static_cast<unsigned long long>(key));
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
                atomicMin(gmin + (o - cand_begin), static_cast<unsigned long long>(key));
            done = true;
            break;
        }
        if (!done)
            atomicOr(&misc->lm.status, kStatusProbeLimit);
    }
}

/// Sets the bit of the candidate index c of each new state of this rank (its first discovery: parent offset +
/// successor index) and remembers c. Resets the receive buffer's fill cursor (no sender advances it before the next
/// layer's collectives, which follow this kernel on this rank).
__global__ void k_dmark(const DistMisc* misc, u64* fill, const u64* __restrict__ gmin, const u64* __restrict__ gbase,
                        u64 layer_begin, u32* __restrict__ fm, u32* __restrict__ cw)
{
    const u64 n = misc->recv;
    if (blockIdx.x == 0 && threadIdx.x == 0)
        *fill = 0;
    for (u64 r = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; r < n; r += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 key = gmin[r];
        if (key == ~u64{0})
            continue;
        const u64 c = gbase[(key >> 32) - layer_begin] + (key & 0xFFFFFFFFull);
        atomicOr(fm + (c >> 5), 1u << (c & 31));
        cw[r] = static_cast<u32>(c);
    }
}

/// Per bitmap word: new states of any rank (low half) | new states of this rank (high half).
struct WordIn
{
    const u32* f;
    const u32* fm;
    __device__ __forceinline__ u64 operator()(u64 w) const
    {
        return static_cast<u64>(__popc(f[w])) | (static_cast<u64>(__popc(fm[w])) << 32);
    }
};
struct WordOut
{
    u64* wpre;
    __device__ __forceinline__ void operator()(u64 w, u64 e, u64) const { wpre[w] = e; }
};

/// Each new state of this rank: its id (layer_end + the new states of all ranks before its candidate index), its place
/// in the rank's id-ordered lists (after the rank's states before it), its arena index and node record (the key).
/// Resets gmin to all ones for the next layer, and unpacks the layer's new-state counts for the next layer's count.
__global__ void k_dassign(DistMisc* misc, u64* __restrict__ gmin, const u32* __restrict__ cw, const u32* __restrict__ f,
                          const u32* __restrict__ fm, const u64* __restrict__ wpre, u64 layer_end, u64 n_local,
                          u64 cand_begin, u32* __restrict__ state_lc, u32* __restrict__ state_id,
                          u32* __restrict__ state_par, u32* __restrict__ state_kid)
{
    const u64 n = misc->recv;
    if (blockIdx.x == 0 && threadIdx.x == 0)
    {
        misc->next_all = misc->new_packed & 0xFFFFFFFFull;
        misc->next_local = misc->new_packed >> 32;
    }
    for (u64 r = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; r < n; r += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 key = gmin[r];
        if (key == ~u64{0})
            continue;
        gmin[r] = ~u64{0};
        const u32 c = cw[r];
        const u32 w = c >> 5, below = (1u << (c & 31)) - 1u;
        const u64 e = wpre[w];
        const u64 lp = n_local + (e >> 32) + __popc(fm[w] & below);
        state_lc[lp] = static_cast<u32>(cand_begin + r);
        state_id[lp] = static_cast<u32>(layer_end + (e & 0xFFFFFFFFull) + __popc(f[w] & below));
        state_par[lp] = static_cast<u32>(key >> 32);
        state_kid[lp] = static_cast<u32>(key);
    }
}

/// max_states: among this rank's new states of the layer (ids ascending), the ones below max_states (kept), and the key
/// of state `last` (max_states - 1) if this rank holds it.
__global__ void k_dcut(const u32* __restrict__ ids, const u32* __restrict__ par, const u32* __restrict__ kid, u64 n,
                       u64 last, DistMisc* misc)
{
    if (threadIdx.x != 0)
        return;
    u64 lo = 0, hi = n;  // the first id above last
    while (lo < hi)
    {
        const u64 mid = (lo + hi) / 2;
        if (ids[mid] <= last)
            lo = mid + 1;
        else
            hi = mid;
    }
    misc->kept = lo;
    misc->cut = lo > 0 && ids[lo - 1] == last ? 1 + ((static_cast<u64>(par[lo - 1]) << 32) | kid[lo - 1]) : 0;
}

/// max_states: goal states among this rank's parents with an id up to `last_parent` (the parents expanded before the
/// cut).
__global__ void k_dcut_goals(DevTask T, const u64* __restrict__ rows, u32 W, const u32* __restrict__ lc,
                             const u32* __restrict__ ids, u64 n, u64 last_parent, u32* out)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < n; i += static_cast<u64>(gridDim.x) * blockDim.x)
        if (ids[i] <= last_parent && goal_holds(T, GlobalRow{rows + static_cast<u64>(lc[i]) * W, W}))
            atomicAdd(out, 1u);
}

/// Resets a layer's counter slot.
__global__ void k_dmisc_init(DistMisc* m)
{
    *m = DistMisc{};
    m->lm.first_goal = 0xFFFFFFFFu;
}

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
    // per candidate of the layer (all ranks), one bit each: this rank's new states, all ranks' (all-reduced); per
    // bitmap word: the exclusive prefix of both; per received record: its state's smallest key (all ones unless the
    // record took a slot: kept all ones between layers), its candidate index
    DeviceBuffer fm, f, wpre, gmin, cw;
    u64 cap_g = 0, cap_recv = 0;
    bool gmin_clean = false;  // gmin all ones (false after an interrupted layer)
    u32 lane = 1;             // bytes per count lane (1, or 4 once a parent had more than 255 successors)
    // per-owner successor counts in the count pass (hashing every successor there), which size each rank's buffers to
    // its own share; with two ranks the bound by the layer's candidates is at most twice that, and cheaper
    bool owner_counts = false;
    DeviceBuffer small;  // hist[world] | fingerprints[world]
    DeviceBuffer misc, sums;  // misc: two counter slots, alternating between layers
    DistMisc* misc_host = nullptr;  // pinned mirror of both slots
    unsigned slot = 0;              // the current layer's slot
    double wait_s = 0;              // host time spent waiting for the layers' results (this search)
    std::vector<u64> layer_begin;
    u64 n_total = 0;
    u64 exchanged = 0;  // records received from other ranks
    u64* hist() { return small.as<u64>(); }
    u64* prints() { return small.as<u64>() + world; }
    DistMisc* misc_at(unsigned k) { return misc.as<DistMisc>() + k; }
};

namespace
{
u64 grown(u64 need, u64 cap) { return std::max<u64>(need, cap + cap / 2); }

/// The frontier from which a sharded search exchanges (b2_brfs_options::shard_from_states 0): below it a sharded
/// layer's fixed cost (its collectives, one host wait, some twenty launches) exceeds what splitting its work saves.
constexpr u64 kShardFromStates = u64{1} << 20;

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
        S.cg.alloc((cap + 2 + kMaxWorld * kMaxWorld) * 4, s);  // word lanes, goals, overflow, per-owner counts
        S.gbase.alloc((cap + 1) * 8, s);
        S.cap_layer = cap;
    }
    ensure_scan(S, n, s);
}

/// The layer's candidate bitmaps (G candidates over all ranks) and the per-received-record arrays (recv records).
void ensure_g(ShardState& S, u64 G, u64 recv, cudaStream_t s)
{
    if (G > S.cap_g)
    {
        const u64 cap = grown(G, S.cap_g);
        const u64 nw = (cap + 31) / 32;
        S.fm.alloc(nw * 4, s);
        S.f.alloc(nw * 4, s);
        S.wpre.alloc(nw * 8, s);
        S.cap_g = cap;
    }
    if (recv > S.cap_recv)
    {
        const u64 cap = grown(recv, S.cap_recv);
        S.gmin.alloc(cap * 8, s);
        S.cw.alloc(cap * 4, s);
        S.cap_recv = cap;
        S.gmin_clean = false;
    }
    if (!S.gmin_clean)
    {
        B2_CUDA(cudaMemsetAsync(S.gmin.p, 0xFF, S.cap_recv * 8, s));
        S.gmin_clean = true;
    }
    ensure_scan(S, (G + 31) / 32, s);
}

/// Collective (every rank passes the same G and W): the communicator's receive buffers hold G records, and their
/// fill cursors are mapped.
void ensure_recv(b2_comm* comm, u32 W, u64 G, cudaStream_t s)
{
    if (!comm->cursors.bytes)
        peer_buffer_exchange(comm, comm->cursors, 256, s, true);
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

/// Waits for the stream and reads both counter slots: returns the current layer's, the other one into *other.
DistMisc read_misc(ShardState& S, b2_comm* comm, cudaStream_t s, DistMisc* other = nullptr)
{
    B2_CUDA(cudaMemcpyAsync(S.misc_host, S.misc.p, 2 * sizeof(DistMisc), cudaMemcpyDeviceToHost, s));
    const auto t0 = std::chrono::steady_clock::now();
    comm_sync(comm, s);
    S.wait_s += std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    for (int k = 0; k < 2; ++k)
    {
        const u32 st = S.misc_host[k].lm.status;
        if (st & kStatusProbeLimit)
            throw Error(B2_DEVICE_FAULT, "b2_brfs: a hash-set probe ran past its bound");
        if (st & kStatusScanStall)
            throw Error(B2_DEVICE_FAULT, "b2_brfs: a prefix scan gave up waiting for a tile");
        if (st)
            throw Error(B2_DEVICE_FAULT, "b2_brfs: device status " + std::to_string(st));
    }
    if (other)
        *other = S.misc_host[S.slot ^ 1];
    return S.misc_host[S.slot];
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
    cudaEvent_t ev[7];
    for (auto& e : ev)
        B2_CUDA(cudaEventCreate(&e));
    struct EvGuard
    {
        cudaEvent_t* e;
        ~EvGuard()
        {
            for (int i = 0; i < 7; ++i)
                cudaEventDestroy(e[i]);
        }
    } guard{ev};

    R.states = 1;
    R.words = W;
    const u64 expect = std::max<u64>(o.expected_states / world + o.expected_states / (4 * world), 1024);
    ensure_cand(S, W, expect * 2, s);
    ensure_states(S, expect, s);
    S.misc.alloc(2 * sizeof(DistMisc), s);
    static_assert(2 * sizeof(DistMisc) <= PinnedPool::kBlock);
    if (!S.misc_host)
        S.misc_host = static_cast<DistMisc*>(B.task->ctx->pinned.take());
    S.small.alloc(2 * world * 8, s);
    B2_CUDA(cudaMemsetAsync(S.misc.p, 0, 2 * sizeof(DistMisc), s));
    S.slot = 0;
    S.wait_s = 0;
    if (comm->cursors.bytes)  // a search that ended early may have left it advanced; no rank pushes before the
        B2_CUDA(cudaMemsetAsync(comm->cursors.local.p, 0, 8, s));  // first layer's collectives
    ensure_table(S, expect, S.misc_at(0), s, B.launches);
    u64 layer_begin = 0, layer_end = 1, lb_local = 0, le_local = 0;
    u32 layers = 0;
    bool exhausted = false, solved = false, full = false;
    bool finished = false;  // the replicated layers ended the search
    u64 expanded = 0, generated = 0, goals = 0, goal_id = 0;
    double count_ms = 0, gen_ms = 0, dedup_ms = 0, exchange_ms = 0;
    std::vector<std::array<u64, 3>> counts;
    const u64 shard_from = o.shard_from_states ? o.shard_from_states : kShardFromStates;
    if (shard_from > 1)
    {
        // The small layers: every rank runs the same one-GPU search alone, with no exchange and no collective (its
        // per-layer cost is far below a sharded layer's), up to the first frontier of shard_from states. Each rank
        // then keeps the states it owns, in id order, with their node records, and the sharded loop goes on from
        // that frontier. The ids, counts and fingerprint are the one-GPU search's either way.
        const b2_brfs_options saved = B.opt;
        // the host loop, its buffers grown as the layers need (the device-driven loop would instantiate its graph for
        // the prefix's buffers once per process and keep it in the context's cache)
        B.opt.expected_states = 0;
        B.opt.fingerprint = 0;
        B.opt.timings = 0;
        std::vector<u64> plc(3 * 4096);
        b2_brfs_result PR{};
        PR.layer_counts = plc.data();
        PR.layer_capacity = 4096;
        bool cut = false;
        try
        {
            cut = run_prefix(B, PR, shard_from);
        }
        catch (...)
        {
            B.opt = saved;
            throw;
        }
        B.opt = saved;
        if (PR.status == B2_SEARCH_UNSOLVABLE)
        {
            R.status = B2_SEARCH_UNSOLVABLE;
            S.layer_begin = {0, 1};
            B.n_states = 1;
            S.n_total = 1;
            return;
        }
        const u64 n = B.n_states;
        const std::vector<u64> lbv = B.layer_begin;  // [0, the layers' starts..., n]
        const u64 frontier_begin = lbv.size() >= 2 ? lbv[lbv.size() - 2] : 0;
        ensure_cand(S, W, n, s);
        ensure_states(S, n, s);
        ensure_scan(S, n, s);
        DeviceBuffer lbd;
        lbd.alloc(lbv.size() * 8);
        B2_CUDA(cudaMemcpyAsync(lbd.p, lbv.data(), lbv.size() * 8, cudaMemcpyHostToDevice, s));
        DistMisc* m0 = S.misc_at(0);
        device_scan(OwnIn{B.state_g.as<u32>(), B.hash.as<u64>(), me, world},
                    OwnOut{B.state_g.as<u32>(), B.rows.as<u64>(), B.hash.as<u64>(), B.par.as<u32>(), B.kid.as<u32>(),
                           lbd.as<u64>(), static_cast<u32>(lbv.size()), W, frontier_begin, S.rows.as<u64>(),
                           S.hash.as<u64>(), S.state_lc.as<u32>(), S.state_id.as<u32>(), S.state_par.as<u32>(),
                           S.state_kid.as<u32>(), &m0->kept},
                    n, &m0->total_local, S.sums.as<u64>(), s, &m0->lm.status);
        B.launches += 3;
        const DistMisc mp = read_misc(S, comm, s);
        // the rank's states into its hash set (sized first, while it holds none)
        ensure_table(S, std::max<u64>(expect, mp.total_local), m0, s, B.launches);
        S.n_local = mp.total_local;
        S.cand_next = S.n_local;
        if (S.n_local)
        {
            k_rehash<<<grid_for(S.n_local, 256), 256, 0, s>>>(S.table.as<u64>(), S.table_slots - 1,
                                                                max_probe(S.table_slots), S.state_lc.as<u32>(),
                                                                S.n_local, S.hash.as<u64>(), &m0->lm.status);
            B2_CUDA(cudaGetLastError());
            ++B.launches;
        }
        read_misc(S, comm, s);  // the status of the inserts
        S.n_total = n;
        S.layer_begin.assign(lbv.begin(), lbv.end() - 1);
        layers = PR.layers;
        expanded = PR.expanded;
        generated = PR.generated;
        goals = PR.num_goal_states;
        solved = PR.solved != 0;
        goal_id = PR.goal_id;
        for (u32 i = 0; i < PR.layers && i < PR.layer_capacity; ++i)
            counts.push_back({plc[3 * i], plc[3 * i + 1], plc[3 * i + 2]});
        layer_begin = frontier_begin;
        layer_end = n;
        lb_local = cut ? mp.kept : S.n_local;
        le_local = S.n_local;
        if (!cut)
        {
            finished = true;
            exhausted = PR.exhausted != 0;
            full = PR.status == B2_SEARCH_OUT_OF_STATES && !solved;
        }
        B2_CUDA(cudaMemsetAsync(S.misc.p, 0, 2 * sizeof(DistMisc), s));
    }
    else
    {
        // the root: arena index 0 on every rank, stored by its owner
        B2_CUDA(cudaMemcpyAsync(S.rows.p, P.initial.data(), W * 8, cudaMemcpyHostToDevice, s));
        k_dseed<<<1, 1, 0, s>>>(S.rows.as<u64>(), S.hash.as<u64>(), W, S.table.as<u64>(), S.table_slots - 1,
                                max_probe(S.table_slots), me, world, S.state_lc.as<u32>(), S.state_id.as<u32>(),
                                S.state_par.as<u32>(), S.state_kid.as<u32>(), S.misc_at(0));
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
        le_local = S.n_local;
        S.layer_begin.assign(1, 0);
    }
    S.lane = 1;
    S.owner_counts = world > 2;
    u64* fill = nullptr;  // this rank's receive-buffer cursor (mapped on the first exchange)
    // The count pass of a layer into counter slot `misc`: the local parents' successor counts and goals, their local
    // offsets (staging), and the layer's counts by parent id summed over the ranks and their offsets. The local
    // parents are El (host) or *El_dev and the layer's parents E or *E_dev (counts still on the device, launched with
    // the previous layer), at most El_max and E_max.
    const auto launch_count = [&](DistMisc* misc, u64 lb, u64 layer_first, u64 El, const u64* El_dev, u64 El_max,
                                  u64 E, const u64* E_dev, u64 E_max) {
        const u32* frontier = S.state_lc.as<u32>() + lb;
        const u32* frontier_id = S.state_id.as<u32>() + lb;
        k_dmisc_init<<<1, 1, 0, s>>>(misc);
        B2_CUDA(cudaMemsetAsync(S.hist(), 0, world * 8, s));
        if (o.timings)
            B2_CUDA(cudaEventRecord(ev[0], s));
        if (El_max)
        {
            const unsigned grid = grid_for(El_max, 128, sms * 64);
            if (B.task->jit)
            {
                dev::BrfsArgs a{};
                a.frontier = frontier;
                a.E = El;
                a.E_dev = El_dev;
                a.counts = S.counts.as<u32>();
                a.misc = &misc->lm;
                a.S.rows = S.rows.as<u64>();
                a.S.W = W;
                a.pi = pi;
                a.hist = S.hist();
                a.world = world;
                jit_launch(S.owner_counts ? B.task->jit->get(kJitDbrfsCount, pi) : B.task->jit->get(kJitBrfsCount, pi), grid, 128,
                           &a, s);
            }
            else if (S.owner_counts)
                dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                    k_dcount<OW, WR><<<grid, 128, 0, s>>>(T, pi, S.rows.as<u64>(), W, frontier, El, El_dev,
                                                          S.counts.as<u32>(), &misc->lm, S.hist(), world);
                });
            else
                dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                    k_count<OW, WR><<<grid, 128, 0, s>>>(T, pi, S.rows.as<u64>(), W, frontier, El,
                                                         S.counts.as<u32>(), &misc->lm, El_dev);
                });
            ++B.launches;
        }
        const u64 lane_words = S.lane == 4 ? E_max : (E_max + 3) / 4;
        const u64 tail_words = 2 + u64{world} * world;
        B2_CUDA(cudaMemsetAsync(S.cg.p, 0, (lane_words + tail_words) * 4, s));
        k_dscatter<<<grid_for(El_max, 256, sms * 8), 256, 0, s>>>(S.counts.as<u32>(), frontier_id, El, El_dev,
                                                                  layer_first, S.cg.as<u32>(), lane_words, S.lane,
                                                                  S.hist(), me, world, misc);
        B2_CUDA(cudaGetLastError());
        comm_group_begin();
        comm_allreduce(comm, S.cg.p, S.cg.p, lane_words + tail_words, CommType::U32, CommOp::Sum, s);
        comm_allreduce(comm, &misc->goal_id, &misc->goal_id, 1, CommType::U64, CommOp::Min, s);
        comm_group_end();
        k_dtail<<<1, 32, 0, s>>>(S.cg.as<u32>() + lane_words, me, world, misc);
        B2_CUDA(cudaGetLastError());
        if (E_dev)
        {
            device_scan_dev(LaneIn{S.cg.as<u32>(), S.lane}, BaseOut{S.gbase.as<u64>()}, E_dev, E_max,
                            &misc->lm.total_cand, S.sums.as<u64>(), s, &misc->lm.status);
            device_scan_dev(CountIn{S.counts.as<u32>()}, BaseOut{S.local_base.as<u64>()}, El_dev, El_max,
                            &misc->total_local, S.sums.as<u64>(), s, &misc->lm.status);
        }
        else
        {
            device_scan(LaneIn{S.cg.as<u32>(), S.lane}, BaseOut{S.gbase.as<u64>()}, E, &misc->lm.total_cand,
                        S.sums.as<u64>(), s, &misc->lm.status);
            device_scan(CountIn{S.counts.as<u32>()}, BaseOut{S.local_base.as<u64>()}, El, &misc->total_local,
                        S.sums.as<u64>(), s, &misc->lm.status);
        }
        B.launches += 9;
        if (o.timings)
            B2_CUDA(cudaEventRecord(ev[1], s));
    };
    bool counted = false;  // this layer's count ran with the previous layer; its counters are in `next`
    DistMisc next{};
    while (!finished)
    {
        const u64 E = layer_end - layer_begin, El = le_local - lb_local;
        if (E == 0)
        {
            exhausted = true;
            break;
        }
        if (layers == o.max_depth)
            break;
        if (S.n_total >= o.max_states)
        {
            full = true;  // the store is full before the layer (max_states <= 1)
            break;
        }
        ++layers;
        DistMisc* misc = S.misc_at(S.slot);
        DistMisc m1;
        if (counted)
            m1 = next;
        else
        {
            ensure_local(S, El, s);
            ensure_layer(S, E, s);
            launch_count(misc, lb_local, layer_begin, El, nullptr, El, E, nullptr, E);
            m1 = read_misc(S, comm, s);
        }
        counted = false;
        if (m1.overflow_all)
        {
            // a parent has more than 255 successors: word lanes from here on (every rank sees the same sum); the
            // count pass again, over the known parents
            S.lane = 4;
            ensure_local(S, El, s);
            ensure_layer(S, E, s);
            launch_count(misc, lb_local, layer_begin, El, nullptr, El, E, nullptr, E);
            m1 = read_misc(S, comm, s);
        }
        if (o.timings)
        {
            float a = 0;
            B2_CUDA(cudaEventElapsedTime(&a, ev[0], ev[1]));
            count_ms += a;
        }
        u64 limit = layer_end, G = m1.lm.total_cand;
        bool stop = false;
        const u32 layer_goals = m1.goals_all;
        if (layer_goals && o.stop_at_goal)
        {
            limit = m1.goal_id;
            if (limit < layer_end)
            {
                B2_CUDA(cudaMemcpyAsync(&G, S.gbase.as<u64>() + (limit - layer_begin), 8, cudaMemcpyDeviceToHost, s));
                comm_sync(comm, s);
            }
            stop = true;
        }
        u64 E_exp = limit - layer_begin;
        if (S.n_total + G >= (u64{1} << 32) - 1 || S.cand_next + G >= (u64{1} << 32) - 1)
            throw Error(B2_CAPACITY, "b2_brfs: more than 2^32 - 2 states or candidates on a rank");
        u64 N = 0, N_local = 0;
        if (E_exp > 0 && G > 0)
        {
            // this rank receives recv_me records (no rank more than recv_max): the per-owner counts of the count pass;
            // without them, at most the layer's G
            const u64 recv = S.owner_counts ? m1.recv_me : G;
            ensure_g(S, G, recv, s);
            ensure_recv(comm, W, S.owner_counts ? m1.recv_max : G, s);
            fill = static_cast<u64*>(comm->cursors.local.p);
            // records a receive buffer holds (the same on every rank), at most options.max_exchange_records: the push
            // kernels drop a record past it and flag the layer, which then fails on every rank with B2_CAPACITY
            u64 recv_cap = comm->exchange.bytes / (RW * 8);
            if (o.max_exchange_records)
                recv_cap = std::min<u64>(recv_cap, o.max_exchange_records);
            if (!B.task->jit && S.cap_staging < m1.total_local)
            {
                S.cap_staging = grown(m1.total_local, S.cap_staging);
                S.staging.alloc(S.cap_staging * RW * 8, s);
            }
            ensure_cand(S, W, S.cand_next + recv, s);
            ensure_states(S, S.n_local + recv, s);
            ensure_table(S, S.n_local + recv, misc, s, B.launches);
            const u64 nw = (G + 31) / 32;
            B2_CUDA(cudaMemsetAsync(S.small.p, 0, world * 8, s));
            B2_CUDA(cudaMemsetAsync(S.fm.p, 0, nw * 4, s));
            if (o.timings)
                B2_CUDA(cudaEventRecord(ev[2], s));
            // the compiled matcher pushes its records to their owners as it generates them; the interpreted one
            // stages them and pushes them after
            const bool fused = B.task->jit != nullptr;
            if (El)
            {
                // the state arrays may have moved (ensure_states)
                DExpandArgs a{};
                a.rows = S.rows.as<u64>();
                a.frontier = S.state_lc.as<u32>() + lb_local;
                a.frontier_id = S.state_id.as<u32>() + lb_local;
                a.E = El;
                a.layer_begin = layer_begin;
                a.limit = limit;
                a.gbase = nullptr;  // keys id << 32 | successor index
                a.local_base = S.local_base.as<u64>();
                a.staging = S.staging.as<u64>();
                a.hist = S.hist();
                a.world = world;
                a.W = W;
                a.pi = pi;
                a.me = me;
                a.peers = reinterpret_cast<u64* const*>(comm->exchange.table.p);
                a.cursors = reinterpret_cast<u64* const*>(comm->cursors.table.p);
                a.sent_self = reinterpret_cast<unsigned long long*>(&misc->sent_self);
                a.recv_cap = recv_cap;
                a.overflow = &misc->barrier;
                const unsigned grid = grid_for(El, 128, sms * 64);
                if (fused)
                    jit_launch(B.task->jit->get(kJitDbrfsPush, pi), grid, 128, &a, s);
                else
                    dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                        k_dexpand<OW, WR><<<grid, 128, 0, s>>>(T, a);
                    });
                ++B.launches;
            }
            if (o.timings)
                B2_CUDA(cudaEventRecord(ev[5], s));
            if (!fused)
            {
                const u32 tile = std::min<u32>(kPushThreads, kPushSmemWords / RW);
                k_push_reserve<<<grid_for(m1.total_local, tile, sms * 8), kPushThreads, tile * RW * 8, s>>>(
                    S.staging.as<u64>(), S.hist(), reinterpret_cast<u64* const*>(comm->exchange.table.p),
                    reinterpret_cast<u64* const*>(comm->cursors.table.p),
                    reinterpret_cast<unsigned long long*>(&misc->sent_self), me, world, RW, tile, recv_cap,
                    &misc->barrier);
                B2_CUDA(cudaGetLastError());
                ++B.launches;
            }
            // orders the pushes before the inserts; its sum is the number of ranks that dropped a record
            comm_allreduce(comm, &misc->barrier, &misc->barrier, 1, CommType::U32, CommOp::Sum, s);
            if (o.timings)
                B2_CUDA(cudaEventRecord(ev[6], s));
            S.gmin_clean = false;
            k_dinsert<<<sms * 8, 256, 0, s>>>(static_cast<const u64*>(comm->exchange.local.p), fill, S.rows.as<u64>(),
                                              S.hash.as<u64>(), S.table.as<u64>(), S.table_slots - 1,
                                              max_probe(S.table_slots), S.cand_next, W,
                                              S.gmin.as<unsigned long long>(), misc, std::min(recv_cap, S.cap_recv));
            B2_CUDA(cudaGetLastError());
            if (o.timings)
                B2_CUDA(cudaEventRecord(ev[3], s));
            k_dmark<<<sms * 8, 256, 0, s>>>(misc, fill, S.gmin.as<u64>(), S.gbase.as<u64>(), layer_begin,
                                            S.fm.as<u32>(), S.cw.as<u32>());
            B2_CUDA(cudaGetLastError());
            comm_allreduce(comm, S.fm.p, S.f.p, nw, CommType::U32, CommOp::Sum, s);
            device_scan(WordIn{S.f.as<u32>(), S.fm.as<u32>()}, WordOut{S.wpre.as<u64>()}, nw, &misc->new_packed,
                        S.sums.as<u64>(), s, &misc->lm.status);
            k_dassign<<<sms * 8, 256, 0, s>>>(misc, S.gmin.as<u64>(), S.cw.as<u32>(), S.f.as<u32>(), S.fm.as<u32>(),
                                              S.wpre.as<u64>(), layer_end, S.n_local, S.cand_next,
                                              S.state_lc.as<u32>(), S.state_id.as<u32>(), S.state_par.as<u32>(),
                                              S.state_kid.as<u32>());
            B2_CUDA(cudaGetLastError());
            S.gmin_clean = true;
            B.launches += 6;
            if (o.timings)
                B2_CUDA(cudaEventRecord(ev[4], s));
            // the next layer's count, over this layer's new states (at most G on all ranks together), so that one
            // wait returns both; skipped where this layer may be the last (a goal stop, the depth bound, or a store
            // that this layer can fill)
            if (!stop && layers < o.max_depth && S.n_total + G < o.max_states)
            {
                ensure_local(S, recv, s);
                ensure_layer(S, G, s);
                launch_count(S.misc_at(S.slot ^ 1), S.n_local, layer_end, 0, &misc->next_local, recv, 0,
                             &misc->next_all, G);
                counted = true;
            }
            const DistMisc m3 = read_misc(S, comm, s, &next);
            if (m3.barrier)  // the same sum on every rank: all of them fail here
                throw Error(B2_CAPACITY, "b2_brfs: a layer's successor records did not fit a rank's receive buffer (" +
                                             std::to_string(recv_cap) + " records); " + std::to_string(m3.barrier) +
                                             " rank(s) dropped records");
            N = m3.new_packed & 0xFFFFFFFFull;
            N_local = m3.new_packed >> 32;
            S.cand_next += m3.recv;
            S.exchanged += m3.lm.ndeferred;
            if (o.timings)
            {
                float b = 0, c = 0, x = 0;
                B2_CUDA(cudaEventElapsedTime(&b, ev[2], ev[3]));
                B2_CUDA(cudaEventElapsedTime(&c, ev[3], ev[4]));
                B2_CUDA(cudaEventElapsedTime(&x, ev[5], ev[6]));
                gen_ms += b;
                dedup_ms += c;
                exchange_ms += x;
            }
        }
        // the goal parents reached: under stop_at_goal the first one (expansion stops there), else all of them
        u64 goals_layer = o.stop_at_goal ? (layer_goals ? 1 : 0) : layer_goals;
        bool goal_reached = layer_goals > 0;
        if (S.n_total + N >= o.max_states && N > 0)
        {
            // max_states: the search stops right after storing state max_states - 1, inside its parent's expansion
            // (run_flat, src/mymyr/search/brfs.cpp:301-384): the parents up to that parent are expanded, its
            // successors up to that one generated, the states after it dropped (each rank keeps a prefix of its
            // id-ordered new states)
            const u64 last = o.max_states - 1;
            k_dcut<<<1, 32, 0, s>>>(S.state_id.as<u32>() + S.n_local, S.state_par.as<u32>() + S.n_local,
                                    S.state_kid.as<u32>() + S.n_local, N_local, last, misc);
            B2_CUDA(cudaGetLastError());
            comm_allreduce(comm, &misc->cut, &misc->cut, 1, CommType::U64, CommOp::Max, s);
            ++B.launches;
            const DistMisc mc = read_misc(S, comm, s);
            if (!mc.cut)
                throw Error(B2_DEVICE_FAULT, "b2_brfs: no rank holds the state at max_states");
            const u64 pstar = (mc.cut - 1) >> 32, kstar = (mc.cut - 1) & 0xFFFFFFFFull;
            u64 first = 0;
            B2_CUDA(cudaMemcpyAsync(&first, S.gbase.as<u64>() + (pstar - layer_begin), 8, cudaMemcpyDeviceToHost, s));
            comm_sync(comm, s);
            E_exp = pstar - layer_begin + 1;
            G = first + kstar + 1;
            N = o.max_states - S.n_total;
            N_local = mc.kept;
            full = stop = true;
            if (o.stop_at_goal)
            {
                goals_layer = 0;  // the layer's first goal parent lies after the cut (the expansion stopped before it)
                goal_reached = false;
            }
            else
            {
                B2_CUDA(cudaMemsetAsync(&misc->lm.goals, 0, 4, s));
                if (El)
                    k_dcut_goals<<<grid_for(El, 256, sms * 8), 256, 0, s>>>(
                        T, S.rows.as<u64>(), W, S.state_lc.as<u32>() + lb_local, S.state_id.as<u32>() + lb_local, El,
                        pstar, &misc->lm.goals);
                B2_CUDA(cudaGetLastError());
                comm_allreduce(comm, &misc->lm.goals, &misc->lm.goals, 1, CommType::U32, CommOp::Sum, s);
                ++B.launches;
                goals_layer = read_misc(S, comm, s).lm.goals;
                goal_reached = layer_goals > 0 && m1.goal_id <= pstar;
            }
        }
        if (goal_reached && !solved)
        {
            solved = true;
            goal_id = m1.goal_id;
        }
        goals += goals_layer;
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
        if (counted)
            S.slot ^= 1;
    }
    S.layer_begin.push_back(S.n_total);
    B.n_states = S.n_total;
    u64 fingerprint = 0;
    DistMisc* misc = S.misc_at(S.slot);
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
    R.exchange_ms = exchange_ms;
    R.wait_ms = S.wait_s * 1000;
    R.kernel_launches = B.launches;
    R.status = solved ? B2_SEARCH_SOLVED
                      : full ? B2_SEARCH_OUT_OF_STATES
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
                            &S.counts, &S.local_base, &S.cg, &S.gbase, &S.staging, &S.fm, &S.f, &S.wpre, &S.gmin,
                            &S.cw, &S.small, &S.misc, &S.sums})
        b->reset();
    B.task->ctx->pinned.give(S.misc_host);
    delete B.shard;
    B.shard = nullptr;
}
}  // namespace b2
