// A* with h^max on the device (search::astar_eager with heuristics::Kind::Max and unit costs,
// src/mymyr/search/astar.cpp:67-256 and include/mymyr/search/best_first.hpp:9-15 of maichmueller/mymyr), and the
// batched h^max evaluation it uses (heuristics::RelaxationHeuristic, src/mymyr/heuristics/heuristics.cpp:185-420;
// cuda::DeviceHeuristic::evaluate, include/mymyr/cuda/heuristics.hpp:115).
//
// h^max. With unit costs, h^max(s) is the index of the first layer of the relaxed planning graph from s that holds
// every goal atom: layer 0 = the atoms of s, layer k + 1 = layer k plus the adds of every operator whose
// preconditions are in layer k (the least fixpoint of cost(p) = 0 for p in s, min over achievers of 1 + max over
// their preconditions, which the reference computes by a generalized Dijkstra). One warp per state keeps the layer's
// atom bitset in shared memory and sweeps the grounded operators (relax.cpp) lane by lane; a layer that adds nothing
// ends the state as a dead end (+inf).
//
// A*. h^max is consistent, so the states leave the open list in f order with their final g, and a bucket of equal f
// can be expanded as a batch: each wave expands the current frontier (all open states of the current f) into staged
// records [row | hash | c] (c: the successor's index in the wave, in canonical order), inserts them into the hash set
// in one kernel (all staged rows are in memory, so the insert is single-phase), gives the new states compact ids by a
// scan, goal-tests and evaluates them, and pushes every state whose g was set or lowered: into the next wave if its f
// equals the current f, else into the open list of later f. When the current f reaches the g of the best goal found,
// that g is the optimal cost (a goal is recognized when generated and returned when it is the minimum f, as in the
// reference). Open entries of states lowered later are stale and skipped (f != g + h).
//
// A state's best path is one u64, key = g << 48 | parent << 16 | successor index: atomicMin on it keeps the smallest
// g and, among equal g, the smallest (parent, successor index), so the plan is deterministic and needs no parent
// arrays. A table slot holds (hash >> 32) << 32 | id, id a state or, during a wave's insert, 2^31 | r for the wave's
// record r that claimed the slot (rewritten to the new state's id by the id scan).

#include "brfs.cuh"
#include "comm.hpp"
#include "relax.hpp"

#include <array>
#include <chrono>
#include <cstddef>
#include <stdexcept>

namespace b2
{
namespace
{
constexpr u32 kDeadEnd = 0xFFFFFFFFu;
constexpr u8 kClosed = 1, kGoal = 2, kDead = 4;

struct HmaxArgs
{
    const u32* pre_begin;
    const u32* pre;
    const u32* add_begin;
    const u32* add;
    const u32* goal;
    u32 ops, ngoal, W, unreachable;
    // optional goal test of the evaluated states (A*): goal masks and the flags to mark
    const u64* goal_pos;
    const u64* goal_neg;
    u8* flags;
    // the triggered evaluation: the operators that need each proposition (CSR over the props), the goal propositions
    // as a bitset
    const u32* need_begin;
    const u32* need;
    const u32* goal_bits;
    u32 props;
};

__device__ __forceinline__ bool sbit(const u64* b, u32 s) { return (b[s >> 6] >> (s & 63)) & 1; }

/// h^max of states: state i is row rows + node(i) * stride, node(i) = nodes[i] (or i), for i < n (*n_dev if given).
/// Warp per state; shared memory: two W-word bitsets per warp.
__global__ void k_hmax(HmaxArgs H, const u64* __restrict__ rows, u64 stride, const u32* __restrict__ nodes,
                       const u64* n_dev, u64 n_host, u32* __restrict__ out, u32 out_by_node)
{
    extern __shared__ u64 sm[];
    const u32 lane = threadIdx.x & 31, wib = threadIdx.x >> 5, wpb = blockDim.x >> 5;
    u64* cur = sm + static_cast<u64>(wib) * 2 * H.W;
    u64* nxt = cur + H.W;
    const u64 n = n_dev ? *n_dev : n_host;
    for (u64 i = static_cast<u64>(blockIdx.x) * wpb + wib; i < n; i += static_cast<u64>(gridDim.x) * wpb)
    {
        const u64 node = nodes ? nodes[i] : i;
        const u64* row = rows + node * stride;
        bool gpos = true, gneg = true;
        for (u32 w = lane; w < H.W; w += 32)
        {
            const u64 x = row[w];
            cur[w] = x;
            nxt[w] = x;
            if (H.flags)
            {
                gpos = gpos && (x & H.goal_pos[w]) == H.goal_pos[w];
                gneg = gneg && (x & H.goal_neg[w]) == 0;
            }
        }
        __syncwarp();
        if (H.flags && __all_sync(0xFFFFFFFFu, gpos && gneg) && lane == 0)
            H.flags[node] |= kGoal;
        auto goal_reached = [&]() {
            bool ok = true;
            for (u32 q = lane; q < H.ngoal; q += 32)
                ok = ok && sbit(cur, H.goal[q]);
            return __all_sync(0xFFFFFFFFu, ok);
        };
        u32 h = 0;
        if (H.unreachable)
            h = kDeadEnd;
        else if (!goal_reached())
        {
            for (u32 layer = 1;; ++layer)
            {
                bool changed = false;
                for (u32 o = lane; o < H.ops; o += 32)
                {
                    bool app = true;
                    for (u32 q = H.pre_begin[o], e = H.pre_begin[o + 1]; q < e && app; ++q)
                        app = sbit(cur, H.pre[q]);
                    if (!app)
                        continue;
                    for (u32 q = H.add_begin[o], e = H.add_begin[o + 1]; q < e; ++q)
                    {
                        const u32 s = H.add[q];
                        if (!sbit(cur, s))
                        {
                            changed = true;
                            if (!sbit(nxt, s))
                                atomicOr(reinterpret_cast<unsigned long long*>(nxt + (s >> 6)), 1ull << (s & 63));
                        }
                    }
                }
                changed = __any_sync(0xFFFFFFFFu, changed);
                __syncwarp();
                if (!changed)
                {
                    h = kDeadEnd;
                    break;
                }
                for (u32 w = lane; w < H.W; w += 32)
                    cur[w] = nxt[w];
                __syncwarp();
                if (goal_reached())
                {
                    h = layer;
                    break;
                }
            }
        }
        if (lane == 0)
            out[out_by_node ? node : i] = h;
        __syncwarp();
    }
}

/// h^max by operator triggering (unit costs): the same layers as k_hmax, without sweeping every operator per layer.
/// Warp per state; per warp in shared memory: the reached propositions (W words), each operator's count of
/// preconditions not reached yet (ops words), and the propositions in the order they are reached (props words, a
/// queue whose layers follow one another). Layer 0 is the state; an operator whose count is 0 adds its propositions to
/// the next layer; every proposition first reached in layer L lowers the counts of the operators that need it, and an
/// operator that reaches 0 then adds its propositions to layer L + 1. h is the layer in which the last goal proposition
/// is reached, a dead end (kDeadEnd) when a layer adds nothing before.
__global__ void k_hmax_trig(HmaxArgs H, const u64* __restrict__ rows, u64 stride, const u32* __restrict__ nodes,
                            const u64* n_dev, u64 n_host, u32* __restrict__ out, u32 out_by_node)
{
    extern __shared__ u64 sm[];
    const u32 lane = threadIdx.x & 31, wib = threadIdx.x >> 5, wpb = blockDim.x >> 5;
    const u64 per_warp = H.W + (static_cast<u64>(H.ops) + H.props + 4 + 1) / 2;  // u64 words
    u64* reached = sm + wib * per_warp;
    u32* unsat = reinterpret_cast<u32*>(reached + H.W);
    u32* queue = unsat + H.ops;
    u32* ctl = queue + H.props;  // [0] queue tail, [1] goal propositions left
    const u64 n = n_dev ? *n_dev : n_host;
    for (u64 i = static_cast<u64>(blockIdx.x) * wpb + wib; i < n; i += static_cast<u64>(gridDim.x) * wpb)
    {
        const u64 node = nodes ? nodes[i] : i;
        const u64* row = rows + node * stride;
        bool gpos = true, gneg = true;
        for (u32 w = lane; w < H.W; w += 32)
        {
            const u64 x = row[w];
            reached[w] = x;
            if (H.flags)
            {
                gpos = gpos && (x & H.goal_pos[w]) == H.goal_pos[w];
                gneg = gneg && (x & H.goal_neg[w]) == 0;
            }
        }
        if (lane == 0)
            ctl[0] = 0;
        __syncwarp();
        if (H.flags && __all_sync(0xFFFFFFFFu, gpos && gneg) && lane == 0)
            H.flags[node] |= kGoal;
        // goal propositions not true in the state
        u32 left = 0;
        for (u32 q = lane; q < H.ngoal; q += 32)
            left += sbit(reached, H.goal[q]) ? 0u : 1u;
        for (int o = 16; o > 0; o >>= 1)
            left += __shfl_xor_sync(0xFFFFFFFFu, left, o);
        u32 h = 0;
        if (H.unreachable)
            h = kDeadEnd;
        else if (left)
        {
            if (lane == 0)
                ctl[1] = left;
            // layer 0: every operator's unreached preconditions; those with none add layer 1
            for (u32 o = lane; o < H.ops; o += 32)
            {
                u32 c = 0;
                for (u32 q = H.pre_begin[o], e = H.pre_begin[o + 1]; q < e; ++q)
                    c += sbit(reached, H.pre[q]) ? 0u : 1u;
                unsat[o] = c;
            }
            __syncwarp();
            // an operator that fires adds its propositions not reached yet to the queue (the next layer)
            const auto fire = [&](u32 o) {
                for (u32 q = H.add_begin[o], e = H.add_begin[o + 1]; q < e; ++q)
                {
                    const u32 p = H.add[q];
                    const unsigned long long bit = 1ull << (p & 63);
                    if (reached[p >> 6] & bit)
                        continue;
                    const unsigned long long was = atomicOr(reinterpret_cast<unsigned long long*>(reached + (p >> 6)), bit);
                    if (was & bit)
                        continue;
                    queue[atomicAdd(&ctl[0], 1u)] = p;
                    if ((H.goal_bits[p >> 5] >> (p & 31)) & 1u)
                        atomicSub(&ctl[1], 1u);
                }
            };
            for (u32 o = lane; o < H.ops; o += 32)
                if (unsat[o] == 0)
                    fire(o);
            __syncwarp();
            u32 head = 0;
            for (u32 layer = 1;; ++layer)
            {
                const u32 tail = ctl[0];
                if (ctl[1] == 0)
                {
                    h = layer;  // the last goal proposition was reached in this layer
                    break;
                }
                if (tail == head)
                {
                    h = kDeadEnd;  // the layer added nothing
                    break;
                }
                __syncwarp();
                // the layer's propositions lower the counts of the operators that need them; those reaching 0 add
                // the next layer
                for (u32 k = head + lane; k < tail; k += 32)
                {
                    const u32 p = queue[k];
                    for (u32 q = H.need_begin[p], e = H.need_begin[p + 1]; q < e; ++q)
                    {
                        const u32 o = H.need[q];
                        if (atomicSub(&unsat[o], 1u) == 1u)
                            fire(o);
                    }
                }
                head = tail;
                __syncwarp();
            }
        }
        if (lane == 0)
            out[out_by_node ? node : i] = h;
        __syncwarp();
    }
}

/// Per-wave counters of the A* (device side, mirrored to pinned host memory). The first block (up to nnext) restarts
/// with every chunk of a wave, nnext with every wave; the rest persists.
struct AstarMisc
{
    LayerMisc lm;   // count pass: total candidates of the wave, status
    u32 ntouched;   // states whose g was set or lowered by the chunk
    u32 ndead;      // dead ends among the chunk's new states
    u64 nfresh;     // new states of the chunk (the id scan's total)
    u32 nnext;      // states of the next wave (f = current f)
    u32 pad;
    u64 nopen;      // open entries of later f
    u64 best_goal;  // (g << 32 | state) of the best goal found (~0: none)
    u64 fmin;       // smallest f of a valid open entry (bucket switch)
    u64 nkeep;      // open entries kept by the extraction
    u64 nfront;     // states extracted into the frontier
    // sharded search: this rank's values and their reductions over the ranks
    u64 gsum;       // the wave's successors (SUM)
    u64 nnext_all;  // the next wave's states (SUM)
    u64 goal_all;   // the best goal over the ranks, (g << 32 | rank << 27 | state) (MIN)
    u64 stats[5];   // expanded, generated, states, evaluations, dead ends (SUM, at the end)
};

/// Chunks of a wave whose candidates exceed `chunk`: chunk k starts at the first frontier state whose first
/// successor's index is in [k * chunk, (k + 1) * chunk) (bounds[k] = that state, ~0 if none).
__global__ void k_chunk_bounds(const u64* __restrict__ cand_base, u64 nF, u64 chunk, u64* bounds)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < nF; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 k = cand_base[i] / chunk;
        if (i == 0 || cand_base[i - 1] / chunk != k)
            bounds[k] = i;
    }
}

constexpr u32 kWaveBit = 0x80000000u;
constexpr u64 kNoParent = 0xFFFFFFFFull;

__device__ __forceinline__ u32 key_g(u64 key) { return static_cast<u32>(key >> 48); }

struct InsertArgs
{
    const u64* staging;  // records [row | hash | key]
    u64 G;
    u32 W;
    u32 wave;          // the chunk's stamp (unique per chunk): a state is listed touched once per chunk
    const u64* rows;   // states
    u64* best;         // per state
    const u8* flags;   // per state
    u32* stamp;        // per state
    u64* table;
    u64 mask;
    u32 max_probe;
    u32 pad;
    u64* best_rec;     // per record: the key of a record that claimed a slot
    u64* slot_of;      // per record: its slot
    u8* claimed;       // per record
    u32* touched;
    AstarMisc* misc;
};

__global__ void k_astar_insert(InsertArgs a)
{
    const u32 W = a.W, RW = W + 2;
    for (u64 r = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; r < a.G; r += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64* rec = a.staging + r * RW;
        const u64 h = rec[W], key = rec[W + 1];  // key = (g << 48 | parent << 16 | successor index), made by staging
        const u32 gnew = key_g(key);
        const u64 tag = h & 0xFFFFFFFF00000000ull;
        u64 j = h & a.mask;
        bool done = false;
        for (u32 probe = 0; probe < a.max_probe; ++probe, j = (j + 1) & a.mask)
        {
            u64 cur = __ldcg(a.table + j);
            if (cur == kEmpty)
            {
                const u64 prev = atomicCAS(reinterpret_cast<unsigned long long*>(a.table + j), kEmpty,
                                           tag | kWaveBit | r);
                if (prev == kEmpty)
                {
                    a.claimed[r] = 1;
                    a.slot_of[r] = j;
                    atomicMin(reinterpret_cast<unsigned long long*>(a.best_rec + r), key);
                    done = true;
                    break;
                }
                cur = prev;
            }
            if ((cur & 0xFFFFFFFF00000000ull) != tag)
                continue;
            const u32 holder = static_cast<u32>(cur);
            const bool wave = holder & kWaveBit;
            const u64 o = holder & ~kWaveBit;
            const u64* orow = wave ? a.staging + o * RW : a.rows + o * W;
            bool eq = true;
            for (u32 q = 0; q < W && eq; ++q)
                eq = orow[q] == rec[q];
            if (!eq)
                continue;
            done = true;
            if (wave)
                atomicMin(reinterpret_cast<unsigned long long*>(a.best_rec + o), key);
            else if (!(a.flags[o] & (kClosed | kDead)))  // closed states have their final g (h^max is consistent)
            {
                const u64 old = atomicMin(reinterpret_cast<unsigned long long*>(a.best + o), key);
                if (key_g(old) > gnew && atomicExch(a.stamp + o, a.wave) != a.wave)
                    a.touched[atomicAdd(&a.misc->ntouched, 1u)] = static_cast<u32>(o);
            }
            break;
        }
        if (!done)
            atomicOr(&a.misc->lm.status, kStatusProbeLimit);
    }
}

/// The id scan's input: whether record r claimed a slot.
struct ClaimIn
{
    const u8* claimed;
    __device__ __forceinline__ u32 operator()(u64 r) const { return claimed[r]; }
};

/// The id scan's output: record r that claimed a slot becomes state n_states + its rank; its row, hash and key move to
/// the state arrays, its slot is rewritten to the state's id, and the state is listed fresh and touched.
struct ClaimOut
{
    const u64* staging;
    u32 W;
    u32 wave;
    u64 n_states;
    const u64* best_rec;
    const u64* slot_of;
    u64* table;
    u64* rows;
    u64* hash;
    u64* best;
    u8* flags;
    u32* stamp;
    u32* fresh;
    u32* touched;
    AstarMisc* misc;
    __device__ __forceinline__ void operator()(u64 r, u64 rank, u32 v) const
    {
        if (!v)
            return;
        const u64 s = n_states + rank;
        const u64* rec = staging + r * (W + 2);
        for (u32 q = 0; q < W; ++q)
            rows[s * W + q] = rec[q];
        const u64 h = rec[W];
        hash[s] = h;
        best[s] = best_rec[r];
        flags[s] = 0;
        stamp[s] = wave;
        table[slot_of[r]] = (h & 0xFFFFFFFF00000000ull) | s;
        fresh[rank] = static_cast<u32>(s);
        touched[atomicAdd(&misc->ntouched, 1u)] = static_cast<u32>(s);
    }
};

/// Pushes the states whose g was set or lowered this wave: dead ends are marked, goals recorded, the others go to
/// the next wave (f = fcur; closed now, as they will be expanded) or to the open list of later f.
__global__ void k_astar_push(const u32* __restrict__ touched, AstarMisc* misc, const u64* __restrict__ best,
                             const u32* __restrict__ h, u8* flags, u32 fcur, u32* next, u64* open)
{
    const u32 n = misc->ntouched;
    for (u32 t = blockIdx.x * blockDim.x + threadIdx.x; t < n; t += gridDim.x * blockDim.x)
    {
        const u32 o = touched[t];
        const u32 hv = h[o];
        if (hv == kDeadEnd)
        {
            flags[o] |= kDead;
            atomicAdd(&misc->ndead, 1u);
            continue;
        }
        const u64 g = key_g(best[o]);
        if (flags[o] & kGoal)
            atomicMin(reinterpret_cast<unsigned long long*>(&misc->best_goal), (g << 32) | o);
        const u64 f = g + hv;
        if (f == fcur)
        {
            flags[o] |= kClosed;
            next[atomicAdd(&misc->nnext, 1u)] = o;
        }
        else
            open[atomicAdd(reinterpret_cast<unsigned long long*>(&misc->nopen), 1ull)] = (f << 32) | o;
    }
}

__device__ __forceinline__ bool open_valid(u64 e, const u64* best, const u32* h, const u8* flags)
{
    const u32 o = static_cast<u32>(e);
    return !(flags[o] & (kClosed | kDead)) && (e >> 32) == static_cast<u64>(key_g(best[o])) + h[o];
}

__global__ void k_astar_fmin(const u64* __restrict__ open, u64 n, const u64* __restrict__ best,
                             const u32* __restrict__ h, const u8* __restrict__ flags, AstarMisc* misc)
{
    u64 m = ~u64{0};
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < n; i += static_cast<u64>(gridDim.x) * blockDim.x)
        if (open_valid(open[i], best, h, flags))
            m = min(m, open[i] >> 32);
    for (int s = 16; s > 0; s >>= 1)
        m = min(m, __shfl_xor_sync(0xFFFFFFFFu, m, s));
    if ((threadIdx.x & 31) == 0 && m != ~u64{0})
        atomicMin(reinterpret_cast<unsigned long long*>(&misc->fmin), m);
}

/// The open entries of f = fmin become the frontier (closed now); the other valid ones are kept.
__global__ void k_astar_extract(const u64* __restrict__ open, u64 n, const u64* __restrict__ best,
                                const u32* __restrict__ h, u8* flags, u64 fmin, u32* front, u64* keep,
                                AstarMisc* misc)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < n; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 e = open[i];
        if (!open_valid(e, best, h, flags))
            continue;
        if ((e >> 32) == fmin)
        {
            const u32 o = static_cast<u32>(e);
            flags[o] |= kClosed;
            front[atomicAdd(reinterpret_cast<unsigned long long*>(&misc->nfront), 1ull)] = o;
        }
        else
            keep[atomicAdd(reinterpret_cast<unsigned long long*>(&misc->nkeep), 1ull)] = e;
    }
}

__global__ void k_astar_seed(u64* rows, u64* hash, u32 W, u64* best, u8* flags, u64* table, u64 mask, u32 max_probe,
                             AstarMisc* misc)
{
    const GlobalRow r{rows, W};
    const u64 h = hash_words([&](u32 q) { return r.word(q); }, W);
    hash[0] = h;
    best[0] = kNoParent << 16;  // g 0, no parent
    flags[0] = kClosed;
    u64 j = h & mask;
    for (u32 probe = 0; probe < max_probe && table[j] != kEmpty; ++probe)
        j = (j + 1) & mask;
    if (table[j] == kEmpty)
        table[j] = h & 0xFFFFFFFF00000000ull;
    else
        atomicOr(&misc->lm.status, kStatusProbeLimit);
}

/// The path from the root to state `goal` by the states' keys: (parent state, successor index) per step, goal first.
__global__ void k_astar_path(const u64* best, u32 goal, u32 cap, u32* out_parent, u32* out_index, u32* len)
{
    u32 s = goal, n = 0;
    while (s != 0 && n < cap)
    {
        const u64 key = best[s];
        const u32 p = static_cast<u32>((key >> 16) & 0xFFFFFFFFull);
        out_parent[n] = p;
        out_index[n] = static_cast<u32>(key & 0xFFFF);
        s = p;
        ++n;
    }
    *len = s == 0 ? n : 0xFFFFFFFFu;
}

/// Moves every entry of an old table (tag | state) into a new one, probing from the state's full hash.
__global__ void k_rehash_entries(const u64* __restrict__ old, u64 old_slots, u64* table, u64 mask, u32 max_probe,
                                 const u64* __restrict__ hash, u32* status)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < old_slots; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 e = old[i];
        if (e == kEmpty)
            continue;
        u64 j = hash[e & 0xFFFFFFFFull] & mask;
        u32 probe = 0;
        for (; probe < max_probe; ++probe, j = (j + 1) & mask)
            if (atomicCAS(reinterpret_cast<unsigned long long*>(table + j), kEmpty, e) == kEmpty)
                break;
        if (probe == max_probe)
            atomicOr(status, kStatusProbeLimit);
    }
}

/// The key base of each frontier state: ((g + 1) << 48) | (parent id << 16), parent id = rank << kRankShift | state;
/// the staging kernel adds the successor index (its records carry their key).
constexpr u32 kRankShift = 27;  // a sharded search's local states stay below 2^27
__global__ void k_key_base(const u32* __restrict__ frontier, u64 nF, const u64* __restrict__ best,
                           const u32* __restrict__ counts, u64 rank_bits, u64* __restrict__ keys, AstarMisc* misc)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < nF; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 s = frontier[i];
        const u64 g = key_g(best[s]) + 1;
        if (g > 0xFFFF || counts[i] > 0x10000u)
            atomicOr(&misc->lm.status, kStatusCapacity);  // a path of 2^16 steps or a state with 2^16 successors
        keys[i] = (g << 48) | ((rank_bits | s) << 16);
    }
}

/// Sharded search: this rank's best goal and next-wave size into the fields the ranks reduce (goal ids global).
__global__ void k_astar_globalize(AstarMisc* misc, u64 rank_bits)
{
    const u64 b = misc->best_goal;  // this rank's, with a local state id
    if (b != ~u64{0})
    {
        const u64 g = (b & 0xFFFFFFFF00000000ull) | rank_bits | (b & 0xFFFFFFFFull);
        if (g < misc->goal_all)
            misc->goal_all = g;
    }
    misc->nnext_all = misc->nnext;
}

__global__ void k_iota(u32* p, u64 n)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < n; i += static_cast<u64>(gridDim.x) * blockDim.x)
        p[i] = static_cast<u32>(i);
}
}  // namespace
}  // namespace b2

using namespace b2;

namespace b2
{
constexpr int kAstarBuffers = 27, kAstarCaps = 6;
/// An A* search's device buffers, kept by a shared heuristic between the searches that use it (one at a time): a
/// search grows its buffers to its waves, and the next search reuses them instead of allocating gigabytes again.
struct AstarCache
{
    DeviceBuffer bufs[kAstarBuffers];
    u64 caps[kAstarCaps] = {};
    bool busy = false;
};
}  // namespace b2

struct b2_heuristic
{
    b2_task* task = nullptr;
    Relaxation R;
    DeviceBuffer blob;  // u32: pre_begin | pre | add_begin | add | goal
    DeviceBuffer goal_masks;  // u64: goal_pos | goal_neg
    HmaxArgs args{};
    AstarCache cache;
};

namespace
{
b2_heuristic* make_heuristic(b2_task* task)
{
    auto H = std::make_unique<b2_heuristic>();
    H->task = task;
    try
    {
        H->R = ground_relaxation(task->spec, task->layout, task->statics, task->prog);
    }
    catch (const std::domain_error& e)
    {
        throw Error(B2_UNSUPPORTED, std::string("b2_heuristic: ") + e.what());
    }
    const Relaxation& R = H->R;
    if (task->ctx)
    {
        B2_CUDA(cudaSetDevice(task->ctx->device));
        std::vector<u32> blob;
        auto put = [&](const std::vector<u32>& v) {
            const u64 at = blob.size();
            blob.insert(blob.end(), v.begin(), v.end());
            blob.push_back(0);  // no empty array
            return at;
        };
        // the operators that need each proposition (the precondition CSR inverted), and the goal propositions as
        // a bitset, for the triggered evaluation
        std::vector<u32> need_begin(R.props + 1, 0), need;
        for (u32 q = 0; q < R.pre.size(); ++q)
            ++need_begin[R.pre[q] + 1];
        for (u32 p = 0; p < R.props; ++p)
            need_begin[p + 1] += need_begin[p];
        need.assign(R.pre.size(), 0);
        {
            std::vector<u32> fill(need_begin.begin(), need_begin.end() - 1);
            for (u32 o = 0; o < R.ops(); ++o)
                for (u32 q = R.pre_begin[o]; q < R.pre_begin[o + 1]; ++q)
                    need[fill[R.pre[q]]++] = o;
        }
        std::vector<u32> goal_bits((R.props + 31) / 32 + 1, 0);
        for (u32 g : R.goal)
            goal_bits[g >> 5] |= 1u << (g & 31);
        const u64 o0 = put(R.pre_begin), o1 = put(R.pre), o2 = put(R.add_begin), o3 = put(R.add), o4 = put(R.goal);
        const u64 o5 = put(need_begin), o6 = put(need), o7 = put(goal_bits);
        H->blob.alloc(blob.size() * 4);
        B2_CUDA(cudaMemcpy(H->blob.p, blob.data(), blob.size() * 4, cudaMemcpyHostToDevice));
        const u32* b = H->blob.as<u32>();
        const u32 W = task->prog.words;
        std::vector<u64> masks(task->prog.goal_pos);
        masks.insert(masks.end(), task->prog.goal_neg.begin(), task->prog.goal_neg.end());
        H->goal_masks.alloc(masks.size() * 8);
        B2_CUDA(cudaMemcpy(H->goal_masks.p, masks.data(), masks.size() * 8, cudaMemcpyHostToDevice));
        H->args = HmaxArgs{b + o0, b + o1, b + o2, b + o3, b + o4, R.ops(), static_cast<u32>(R.goal.size()), W,
                           R.goal_unreachable || task->prog.goal_unsat ? 1u : 0u, H->goal_masks.as<u64>(),
                           H->goal_masks.as<u64>() + W, nullptr, b + o5, b + o6, b + o7, R.props};
    }
    return H.release();
}

constexpr unsigned kHmaxThreads = 128;

void launch_hmax(const b2_heuristic& H, const u64* rows, u64 stride, const u32* nodes, const u64* n_dev, u64 n_bound,
                 u32* out, bool by_node, u8* flags, int sms, cudaStream_t s)
{
    HmaxArgs a = H.args;
    a.flags = flags;
    // the triggered evaluation where its per-warp tables (reached props, operator counts, queue) fit shared memory
    const size_t trig_warp = (a.W + (static_cast<size_t>(a.ops) + a.props + 4 + 1) / 2) * 8;
    if (a.props >= a.W * 64 - 63 && trig_warp * (kHmaxThreads / 32) <= 160 * 1024)
    {
        const size_t smem = trig_warp * (kHmaxThreads / 32);
        if (smem > 48 * 1024)
            B2_CUDA(cudaFuncSetAttribute(k_hmax_trig, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)));
        const unsigned grid = grid_for(n_bound, kHmaxThreads / 32, static_cast<unsigned>(sms) * 32);
        k_hmax_trig<<<grid, kHmaxThreads, smem, s>>>(a, rows, stride, nodes, n_dev, n_bound, out, by_node ? 1 : 0);
        B2_CUDA(cudaGetLastError());
        return;
    }
    const unsigned warps = kHmaxThreads / 32;
    const size_t smem = static_cast<size_t>(warps) * 2 * a.W * 8;
    if (smem > 200 * 1024)
        throw Error(B2_UNSUPPORTED, "b2_heuristic: state rows too wide for the h^max kernel's shared memory");
    if (smem > 48 * 1024)
        B2_CUDA(cudaFuncSetAttribute(k_hmax, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    const unsigned grid = grid_for(n_bound, warps, static_cast<unsigned>(sms) * 32);
    k_hmax<<<grid, kHmaxThreads, smem, s>>>(a, rows, stride, nodes, n_dev, n_bound, out, by_node ? 1 : 0);
    B2_CUDA(cudaGetLastError());
}
}  // namespace

// ------------------------------------------------------------------------------------------------ A* search object
struct b2_astar
{
    b2_task* task = nullptr;
    b2_heuristic* H = nullptr;
    bool own_h = false;
    b2_astar_options opt{};
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    u32 W = 1;
    // per state
    DeviceBuffer rows, hash, best, hval, flags, stamp;
    u64 cap_states = 0, n_states = 0;
    DeviceBuffer table;
    u64 table_slots = 0;
    // per wave: frontier-sized and candidate-sized scratch
    DeviceBuffer counts, cand_base, keyb, iota, sums;
    u64 cap_front = 0, cap_iota = 0;
    DeviceBuffer staging, best_rec, slot_of, claimed, touched, fresh;
    u64 cap_wave = 0;
    DeviceBuffer bounds;  // chunk starts of a large wave
    DeviceBuffer front, next;  // state lists (swapped between waves)
    DeviceBuffer open, keep;   // open entries (f << 32 | state)
    u64 cap_open = 0;
    DeviceBuffer misc;
    AstarMisc* misc_host = nullptr;
    DeviceBuffer hist;  // the staging kernel's per-owner counter (one rank)
    u64 launches = 0;
    bool ran = false;
    u32 goal_state = 0;
    bool solved = false;
    u64 cost = 0;
    b2_comm* comm = nullptr;  // sharded search
    DeviceBuffer hist_m;      // sharded: per-owner counts and their all-gather [world + world * world]
    DeviceBuffer sstage;      // sharded: this rank's staged records before the push
    bool borrowed = false;    // the buffers came from the shared heuristic's cache and go back to it

    std::array<DeviceBuffer*, kAstarBuffers> buffers()
    {
        return {&rows, &hash, &best, &hval, &flags, &stamp, &table, &counts, &cand_base, &keyb, &iota, &sums,
                &staging, &best_rec, &slot_of, &claimed, &touched, &fresh, &bounds, &front, &next, &open, &keep,
                &misc, &hist, &hist_m, &sstage};
    }
    std::array<u64*, kAstarCaps> caps() { return {&cap_states, &table_slots, &cap_front, &cap_iota, &cap_wave, &cap_open}; }
};

namespace
{
u64 grow_to(u64 need, u64 cap) { return std::max<u64>(need, cap * 2); }

void ensure_states(b2_astar& A, u64 need)
{
    if (need <= A.cap_states)
        return;
    const u64 cap = grow_to(need, A.cap_states);
    const u64 used = A.n_states;
    cudaStream_t s = A.stream;
    A.rows.grow(cap * A.W * 8, used * A.W * 8, s);
    A.hash.grow(cap * 8, used * 8, s);
    A.best.grow(cap * 8, used * 8, s);
    A.hval.grow(cap * 4, used * 4, s);
    A.flags.grow(cap, used, s);
    A.stamp.grow(cap * 4, used * 4, s);
    A.cap_states = cap;
}

void rehash(b2_astar& A, u64 slots)
{
    // the table's entries (tag | state) move into a table of `slots` slots, probing from each state's full hash
    DeviceBuffer old;
    old.swap(A.table);
    const u64 old_slots = A.table_slots;
    A.table.alloc(slots * 8, A.stream);
    B2_CUDA(cudaMemsetAsync(A.table.p, 0xFF, slots * 8, A.stream));
    A.table_slots = slots;
    if (old_slots)
    {
        auto* misc = A.misc.as<AstarMisc>();
        k_rehash_entries<<<grid_for(old_slots, 256), 256, 0, A.stream>>>(old.as<u64>(), old_slots, A.table.as<u64>(),
                                                                          slots - 1, max_probe(slots), A.hash.as<u64>(),
                                                                          &misc->lm.status);
        B2_CUDA(cudaGetLastError());
        ++A.launches;
    }
}

void ensure_table(b2_astar& A, u64 bound)
{
    if (bound * 4 <= A.table_slots * 3)
        return;
    u64 slots = A.table_slots ? A.table_slots : 1024;
    while (bound * 2 > slots)
        slots *= 2;
    rehash(A, slots);
}

void ensure_front(b2_astar& A, u64 nF)
{
    cudaStream_t s = A.stream;
    if (nF > A.cap_front)
    {
        const u64 cap = grow_to(nF, A.cap_front);
        A.counts.alloc(cap * 4, s);
        A.cand_base.alloc((cap + 1) * 8, s);
        A.keyb.alloc(cap * 8, s);
        A.cap_front = cap;
    }
    if (nF > A.cap_iota)
    {
        const u64 cap = grow_to(nF, A.cap_iota);
        A.iota.alloc(cap * 4, s);
        k_iota<<<grid_for(cap, 256), 256, 0, s>>>(A.iota.as<u32>(), cap);
        B2_CUDA(cudaGetLastError());
        ++A.launches;
        A.cap_iota = cap;
    }
    if (A.front.bytes < nF * 4)
        A.front.grow(grow_to(nF, A.front.bytes / 4) * 4, A.front.bytes, s);
}

/// Scratch of a wave of G candidates, and room for G more open entries and next-wave states.
void ensure_wave(b2_astar& A, u64 G, u64 nopen)
{
    cudaStream_t s = A.stream;
    if (G > A.cap_wave)
    {
        const u64 cap = grow_to(G, A.cap_wave);
        A.staging.alloc(cap * (A.W + 2) * 8, s);
        A.best_rec.alloc(cap * 8, s);
        A.slot_of.alloc(cap * 8, s);
        A.claimed.alloc(cap, s);
        A.touched.alloc(cap * 4, s);
        A.fresh.alloc(cap * 4, s);
        A.cap_wave = cap;
    }
    (void)0;
    if (A.sums.bytes < scan_scratch_bytes(std::max(G, A.cap_front)))
        A.sums.alloc(scan_scratch_bytes(grow_to(std::max(G, A.cap_front), 0)), s);
    if (nopen + G > A.cap_open)
    {
        const u64 cap = grow_to(nopen + G, A.cap_open);
        A.open.grow(cap * 8, nopen * 8, s);
        A.keep.alloc(cap * 8, s);
        A.cap_open = cap;
    }
}

u32 dev_owner(u64 h, u32 world) { return static_cast<u32>(((h >> 32) * world) >> 32); }

const AstarMisc& read_misc(b2_astar& A);

/// read_misc for a sharded search: the wait polls the communicator (a rank that stopped taking part fails it).
const AstarMisc& read_misc_sync(b2_astar& A)
{
    B2_CUDA(cudaMemcpyAsync(A.misc_host, A.misc.p, sizeof(AstarMisc), cudaMemcpyDeviceToHost, A.stream));
    comm_sync(A.comm, A.stream);
    if (A.misc_host->lm.status & kStatusProbeLimit)
        throw Error(B2_DEVICE_FAULT, "b2_astar: a hash-set probe ran past its bound");
    if (A.misc_host->lm.status & kStatusCapacity)
        throw Error(B2_CAPACITY, "b2_astar: a state with 2^16 successors or a path of 2^16 steps");
    if (A.misc_host->lm.status)
        throw Error(B2_DEVICE_FAULT, "b2_astar: device status " + std::to_string(A.misc_host->lm.status));
    return *A.misc_host;
}

const AstarMisc& read_misc(b2_astar& A)
{
    B2_CUDA(cudaMemcpyAsync(A.misc_host, A.misc.p, sizeof(AstarMisc), cudaMemcpyDeviceToHost, A.stream));
    stream_wait(A.stream);
    if (A.misc_host->lm.status & kStatusProbeLimit)
        throw Error(B2_DEVICE_FAULT, "b2_astar: a hash-set probe ran past its bound");
    if (A.misc_host->lm.status & kStatusCapacity)
        throw Error(B2_CAPACITY, "b2_astar: a state with 2^16 successors or a path of 2^16 steps");
    if (A.misc_host->lm.status)
        throw Error(B2_DEVICE_FAULT, "b2_astar: device status " + std::to_string(A.misc_host->lm.status));
    return *A.misc_host;
}

void run_astar(b2_astar& A, b2_astar_result& R)
{
    const auto t0 = std::chrono::steady_clock::now();
    b2_task* task = A.task;
    const Program& P = task->prog;
    const DevTask& T = task->dev;
    const u32 pi = A.opt.witness_pruning ? 0 : 1;
    const u32 W = A.W;
    const unsigned sms = static_cast<unsigned>(task->ctx->sms);
    cudaStream_t s = A.stream;
    cudaEvent_t ev[6];
    for (auto& e : ev)
        B2_CUDA(cudaEventCreate(&e));
    struct EvGuard
    {
        cudaEvent_t* e;
        ~EvGuard()
        {
            for (int i = 0; i < 6; ++i)
                cudaEventDestroy(e[i]);
        }
    } guard{ev};
    R.relaxed_ops = A.H->R.ops();
    R.relaxed_atoms = A.H->R.reached;
    if (P.goal_unsat)
    {
        R.status = B2_SEARCH_UNSOLVABLE;
        return;
    }
    const u64 expect = std::max<u64>(A.opt.expected_states, 4096);
    const u64 chunk = A.opt.chunk_candidates ? std::max<u64>(A.opt.chunk_candidates, u64{1} << 16) : u64{1} << 26;
    if (A.table_slots)  // reused buffers: an empty table
        B2_CUDA(cudaMemsetAsync(A.table.p, 0xFF, A.table_slots * 8, s));
    ensure_states(A, expect);
    A.misc.alloc(sizeof(AstarMisc), s);
    static_assert(sizeof(AstarMisc) <= PinnedPool::kBlock);
    A.misc_host = static_cast<AstarMisc*>(task->ctx->pinned.take());
    *A.misc_host = AstarMisc{};
    A.misc_host->best_goal = ~u64{0};
    B2_CUDA(cudaMemcpyAsync(A.misc.p, A.misc_host, sizeof(AstarMisc), cudaMemcpyHostToDevice, s));
    ensure_table(A, expect);
    AstarMisc* misc = A.misc.as<AstarMisc>();
    B2_CUDA(cudaMemcpyAsync(A.rows.p, P.initial.data(), W * 8, cudaMemcpyHostToDevice, s));
    k_astar_seed<<<1, 1, 0, s>>>(A.rows.as<u64>(), A.hash.as<u64>(), W, A.best.as<u64>(), A.flags.as<u8>(),
                                 A.table.as<u64>(), A.table_slots - 1, max_probe(A.table_slots), misc);
    B2_CUDA(cudaGetLastError());
    ++A.launches;
    A.n_states = 1;
    ensure_front(A, std::max<u64>(expect / 8, 1024));
    ensure_wave(A, std::min(std::max<u64>(expect / 2, 1024), chunk), 0);
    B2_CUDA(cudaMemsetAsync(A.front.p, 0, 4, s));  // the frontier: the root (state 0)
    launch_hmax(*A.H, A.rows.as<u64>(), W, A.front.as<u32>(), nullptr, 1, A.hval.as<u32>(), true, A.flags.as<u8>(),
                static_cast<int>(sms), s);
    ++A.launches;
    u32 h0 = 0;
    u8 f0 = 0;
    B2_CUDA(cudaMemcpyAsync(&h0, A.hval.p, 4, cudaMemcpyDeviceToHost, s));
    B2_CUDA(cudaMemcpyAsync(&f0, A.flags.p, 1, cudaMemcpyDeviceToHost, s));
    stream_wait(s);
    R.evaluations = 1;
    R.initial_h = h0 == kDeadEnd ? -1.0 : static_cast<double>(h0);
    const bool dead_start = h0 == kDeadEnd && !(f0 & kGoal);
    if (f0 & kGoal)
    {
        A.solved = true;
        A.cost = 0;
        A.goal_state = 0;
    }
    else if (dead_start)
        R.dead_ends = 1;
    u64 fcur = h0, nF = 1, nopen = 0, expanded = 0, generated = 0, fresh_total = 0, dead = 0;
    u32 wave = 0, f_layers = 1, stamp = 0;
    double count_ms = 0, expand_ms = 0, insert_ms = 0, eval_ms = 0;
    bool exhausted = false;
    while (!A.solved && !dead_start)
    {
        if (A.opt.max_expansions && expanded >= A.opt.max_expansions)
            break;
        ++wave;
        ensure_front(A, nF);
        // per-wave counters (the open-list count and the best goal persist)
        B2_CUDA(cudaMemsetAsync(misc, 0, offsetof(AstarMisc, nopen), s));
        const unsigned grid = grid_for(nF, 128, sms * 64);
        if (A.opt.timings)
            B2_CUDA(cudaEventRecord(ev[0], s));
        if (task->jit)
        {
            dev::BrfsArgs a{};
            a.frontier = A.front.as<u32>();
            a.E = nF;
            a.counts = A.counts.as<u32>();
            a.misc = &misc->lm;
            a.S.rows = A.rows.as<u64>();
            a.S.W = W;
            a.pi = pi;
            jit_launch(task->jit->get(kJitBrfsCount, pi), grid, 128, &a, s);
        }
        else
            dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                k_count<OW, WR><<<grid, 128, 0, s>>>(T, pi, A.rows.as<u64>(), W, A.front.as<u32>(), nF,
                                                     A.counts.as<u32>(), &misc->lm);
            });
        if (A.sums.bytes < scan_scratch_bytes(nF))
            A.sums.alloc(scan_scratch_bytes(grow_to(nF, 0)), s);
        device_scan(CountIn{A.counts.as<u32>()}, BaseOut{A.cand_base.as<u64>()}, nF, &misc->lm.total_cand,
                    A.sums.as<u64>(), s, &misc->lm.status);
        A.launches += 4;
        if (A.opt.timings)
            B2_CUDA(cudaEventRecord(ev[1], s));
        k_key_base<<<grid_for(nF, 256, sms * 16), 256, 0, s>>>(A.front.as<u32>(), nF, A.best.as<u64>(),
                                                                A.counts.as<u32>(), 0, A.keyb.as<u64>(), misc);
        B2_CUDA(cudaGetLastError());
        ++A.launches;
        const u64 G = read_misc(A).lm.total_cand;
        // the wave's chunks: [first state, end state, first candidate, end candidate)
        std::vector<std::array<u64, 4>> chunks;
        if (G > 0 && G <= chunk)
            chunks.push_back({0, nF, 0, G});
        else if (G > 0)
        {
            const u64 nk = (G + chunk - 1) / chunk;
            A.bounds.alloc(nk * 8, s);
            B2_CUDA(cudaMemsetAsync(A.bounds.p, 0xFF, nk * 8, s));
            k_chunk_bounds<<<grid_for(nF, 256, sms * 16), 256, 0, s>>>(A.cand_base.as<u64>(), nF, chunk,
                                                                        A.bounds.as<u64>());
            B2_CUDA(cudaGetLastError());
            ++A.launches;
            std::vector<u64> starts(nk);
            B2_CUDA(cudaMemcpyAsync(starts.data(), A.bounds.p, nk * 8, cudaMemcpyDeviceToHost, s));
            stream_wait(s);
            std::vector<u64> first;  // the chunks' first states (ids without one merge into the previous chunk)
            for (u64 k = 0; k < nk; ++k)
                if (starts[k] != ~u64{0})
                    first.push_back(starts[k]);
            std::vector<u64> cb(first.size());
            for (u64 k = 0; k < first.size(); ++k)
                B2_CUDA(cudaMemcpyAsync(&cb[k], A.cand_base.as<u64>() + first[k], 8, cudaMemcpyDeviceToHost, s));
            stream_wait(s);
            for (u64 k = 0; k < first.size(); ++k)
                chunks.push_back({first[k], k + 1 < first.size() ? first[k + 1] : nF, cb[k],
                                  k + 1 < first.size() ? cb[k + 1] : G});
        }
        u64 nnext = 0;
        for (u64 ci = 0; ci < chunks.size(); ++ci)
        {
            ++stamp;  // a state lowered again by a later chunk of the wave must be pushed again
            const u64 i0 = chunks[ci][0], i1 = chunks[ci][1], c0 = chunks[ci][2], Gc = chunks[ci][3] - c0;
            if (Gc == 0)
                continue;
            if (A.n_states + Gc >= kWaveBit)
                throw Error(B2_CAPACITY, "b2_astar: more than 2^31 states");
            ensure_wave(A, Gc, nopen);
            if (A.next.bytes < (nnext + Gc) * 4)
                A.next.grow(grow_to(nnext + Gc, A.next.bytes / 4) * 4, nnext * 4, s);
            ensure_states(A, A.n_states + Gc);
            ensure_table(A, A.n_states + Gc);
            if (ci > 0)
                B2_CUDA(cudaMemsetAsync(misc, 0, offsetof(AstarMisc, nnext), s));
            B2_CUDA(cudaMemsetAsync(A.best_rec.p, 0xFF, Gc * 8, s));
            B2_CUDA(cudaMemsetAsync(A.claimed.p, 0, Gc, s));
            if (A.opt.timings)
                B2_CUDA(cudaEventRecord(ev[2], s));
            const unsigned gridc = grid_for(i1 - i0, 128, sms * 64);
            dev::DExpandArgs a{};
            a.rows = A.rows.as<u64>();
            a.frontier = A.front.as<u32>() + i0;
            a.frontier_id = A.iota.as<u32>();
            a.E = i1 - i0;
            a.layer_begin = 0;
            a.limit = ~u64{0};
            a.gbase = A.keyb.as<u64>() + i0;  // the records' last word: key base + successor index
            a.local_base = A.cand_base.as<u64>() + i0;
            a.stage_base = c0;
            a.staging = A.staging.as<u64>();
            a.hist = A.hist.as<u64>();
            a.world = 1;
            a.W = W;
            a.pi = pi;
            if (task->jit)
                jit_launch(task->jit->get(kJitDbrfsExpand, pi), gridc, 128, &a, s);
            else
                dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() { k_dexpand<OW, WR><<<gridc, 128, 0, s>>>(T, a); });
            InsertArgs in{};
            in.staging = A.staging.as<u64>();
            in.G = Gc;
            in.W = W;
            in.wave = stamp;
            in.rows = A.rows.as<u64>();
            in.best = A.best.as<u64>();
            in.flags = A.flags.as<u8>();
            in.stamp = A.stamp.as<u32>();
            in.table = A.table.as<u64>();
            in.mask = A.table_slots - 1;
            in.max_probe = max_probe(A.table_slots);
            in.best_rec = A.best_rec.as<u64>();
            in.slot_of = A.slot_of.as<u64>();
            in.claimed = A.claimed.as<u8>();
            in.touched = A.touched.as<u32>();
            in.misc = misc;
            k_astar_insert<<<grid_for(Gc, 256, sms * 16), 256, 0, s>>>(in);
            B2_CUDA(cudaGetLastError());
            ClaimOut co{A.staging.as<u64>(), W, stamp, A.n_states, A.best_rec.as<u64>(), A.slot_of.as<u64>(),
                        A.table.as<u64>(), A.rows.as<u64>(), A.hash.as<u64>(), A.best.as<u64>(), A.flags.as<u8>(),
                        A.stamp.as<u32>(), A.fresh.as<u32>(), A.touched.as<u32>(), misc};
            device_scan(ClaimIn{A.claimed.as<u8>()}, co, Gc, &misc->nfresh, A.sums.as<u64>(), s, &misc->lm.status);
            if (A.opt.timings)
                B2_CUDA(cudaEventRecord(ev[3], s));
            launch_hmax(*A.H, A.rows.as<u64>(), W, A.fresh.as<u32>(), &misc->nfresh, Gc, A.hval.as<u32>(), true,
                        A.flags.as<u8>(), static_cast<int>(sms), s);
            if (A.opt.timings)
                B2_CUDA(cudaEventRecord(ev[4], s));
            k_astar_push<<<grid_for(Gc, 256, sms * 16), 256, 0, s>>>(A.touched.as<u32>(), misc, A.best.as<u64>(),
                                                                       A.hval.as<u32>(), A.flags.as<u8>(),
                                                                       static_cast<u32>(fcur), A.next.as<u32>(),
                                                                       A.open.as<u64>());
            B2_CUDA(cudaGetLastError());
            A.launches += 7;
            if (A.opt.timings)
                B2_CUDA(cudaEventRecord(ev[5], s));
            const AstarMisc mc = read_misc(A);
            if (A.opt.timings)
            {
                float x = 0, y = 0, z = 0;
                B2_CUDA(cudaEventElapsedTime(&x, ev[2], ev[3]));
                B2_CUDA(cudaEventElapsedTime(&y, ev[3], ev[4]));
                B2_CUDA(cudaEventElapsedTime(&z, ev[4], ev[5]));
                expand_ms += x;  // staging + insert + ids
                eval_ms += y;
                insert_ms += z;  // push
            }
            fresh_total += mc.nfresh;
            dead += mc.ndead;
            A.n_states += mc.nfresh;
            nopen = mc.nopen;
            nnext = mc.nnext;
        }
        if (A.opt.timings)
        {
            float x = 0;
            B2_CUDA(cudaEventElapsedTime(&x, ev[0], ev[1]));
            count_ms += x;
        }
        const AstarMisc m = *A.misc_host;  // as of the last chunk (or the count pass of a wave without successors)
        expanded += nF;
        generated += G;
        if (m.best_goal != ~u64{0} && (m.best_goal >> 32) <= fcur)
        {
            A.solved = true;
            A.cost = m.best_goal >> 32;
            A.goal_state = static_cast<u32>(m.best_goal);
            break;
        }
        if (nnext > 0)
        {
            A.front.swap(A.next);
            nF = nnext;
            continue;
        }
        // the current f is done: the smallest f of the open list is next
        if (nopen == 0)
        {
            exhausted = true;
            break;
        }
        B2_CUDA(cudaMemsetAsync(&misc->fmin, 0xFF, 8, s));
        k_astar_fmin<<<grid_for(nopen, 256, sms * 16), 256, 0, s>>>(A.open.as<u64>(), nopen, A.best.as<u64>(),
                                                                      A.hval.as<u32>(), A.flags.as<u8>(), misc);
        B2_CUDA(cudaGetLastError());
        ++A.launches;
        const u64 fmin = read_misc(A).fmin;
        if (fmin == ~u64{0})
        {
            exhausted = true;
            break;
        }
        if (m.best_goal != ~u64{0} && (m.best_goal >> 32) <= fmin)
        {
            A.solved = true;
            A.cost = m.best_goal >> 32;
            A.goal_state = static_cast<u32>(m.best_goal);
            break;
        }
        fcur = fmin;
        ++f_layers;
        ensure_front(A, nopen);
        B2_CUDA(cudaMemsetAsync(&misc->nkeep, 0, 16, s));
        k_astar_extract<<<grid_for(nopen, 256, sms * 16), 256, 0, s>>>(A.open.as<u64>(), nopen, A.best.as<u64>(),
                                                                         A.hval.as<u32>(), A.flags.as<u8>(), fmin,
                                                                         A.front.as<u32>(), A.keep.as<u64>(), misc);
        B2_CUDA(cudaGetLastError());
        ++A.launches;
        const AstarMisc m4 = read_misc(A);
        A.open.swap(A.keep);
        nopen = m4.nkeep;
        nF = m4.nfront;
        A.misc_host->nopen = nopen;
        B2_CUDA(cudaMemcpyAsync(&misc->nopen, &A.misc_host->nopen, 8, cudaMemcpyHostToDevice, s));
        if (nF == 0)
        {
            exhausted = true;
            break;
        }
    }
    stream_wait(s);
    R.status = A.solved ? B2_SEARCH_SOLVED
                        : dead_start ? B2_SEARCH_UNSOLVABLE : exhausted ? B2_SEARCH_EXHAUSTED : B2_SEARCH_OUT_OF_STATES;
    R.cost = A.solved ? static_cast<double>(A.cost) : 0.0;
    R.expanded = expanded;
    R.generated = generated;
    R.states = A.n_states;
    R.evaluations += fresh_total;
    R.dead_ends += dead;
    R.waves = wave;
    R.f_layers = f_layers;
    R.plan_length = A.solved ? static_cast<u32>(A.cost) : 0;
    R.count_ms = count_ms;
    R.expand_ms = expand_ms;
    R.insert_ms = insert_ms;
    R.eval_ms = eval_ms;
    R.kernel_launches = A.launches;
    R.search_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

/// A* sharded over the communicator's ranks by state-hash owner (HDA*-style, with the batched f layers of run_astar):
/// every wave, each rank expands its part of the frontier into records [row | hash | key] (the key's parent is the
/// global id rank << 27 | state), the records go to their owners through the peer-memory push of the sharded BrFS,
/// and each owner inserts, evaluates and pushes its own. The ranks agree on every decision through reductions: the
/// wave's successors, the next wave's size and the best goal (g << 32 | global id) after each wave, the smallest f of
/// the open lists at a bucket switch.
void run_astar_sharded(b2_astar& A, b2_astar_result& R)
{
    const auto t0 = std::chrono::steady_clock::now();
    b2_task* task = A.task;
    b2_comm* comm = A.comm;
    const u32 me = comm->rank, world = comm->world;
    const Program& P = task->prog;
    const DevTask& T = task->dev;
    const u32 pi = A.opt.witness_pruning ? 0 : 1;
    const u32 W = A.W, RW = W + 2;
    const unsigned sms = static_cast<unsigned>(task->ctx->sms);
    cudaStream_t s = A.stream;
    R.relaxed_ops = A.H->R.ops();
    R.relaxed_atoms = A.H->R.reached;
    if (P.goal_unsat)
    {
        R.status = B2_SEARCH_UNSOLVABLE;
        return;
    }
    const u64 expect = std::max<u64>(A.opt.expected_states / world, 4096);
    if (A.table_slots)  // reused buffers: an empty table
        B2_CUDA(cudaMemsetAsync(A.table.p, 0xFF, A.table_slots * 8, s));
    ensure_states(A, expect);
    A.misc.alloc(sizeof(AstarMisc), s);
    A.misc_host = static_cast<AstarMisc*>(task->ctx->pinned.take());
    *A.misc_host = AstarMisc{};
    A.misc_host->best_goal = ~u64{0};
    A.misc_host->goal_all = ~u64{0};
    B2_CUDA(cudaMemcpyAsync(A.misc.p, A.misc_host, sizeof(AstarMisc), cudaMemcpyHostToDevice, s));
    ensure_table(A, expect);
    AstarMisc* misc = A.misc.as<AstarMisc>();
    A.hist_m.alloc((world + world * world) * 8, s);
    u64* hist = A.hist_m.as<u64>();
    u64* M = hist + world;
    // the root: state 0 on every rank (row and hash), stored and expanded by its owner
    B2_CUDA(cudaMemcpyAsync(A.rows.p, P.initial.data(), W * 8, cudaMemcpyHostToDevice, s));
    k_astar_seed<<<1, 1, 0, s>>>(A.rows.as<u64>(), A.hash.as<u64>(), W, A.best.as<u64>(), A.flags.as<u8>(),
                                 A.table.as<u64>(), A.table_slots - 1, max_probe(A.table_slots), misc);
    B2_CUDA(cudaGetLastError());
    ++A.launches;
    u64 root_hash = 0;
    B2_CUDA(cudaMemcpyAsync(&root_hash, A.hash.p, 8, cudaMemcpyDeviceToHost, s));
    ensure_front(A, 1024);
    ensure_wave(A, 1024, 0);
    B2_CUDA(cudaMemsetAsync(A.front.p, 0, 4, s));
    launch_hmax(*A.H, A.rows.as<u64>(), W, A.front.as<u32>(), nullptr, 1, A.hval.as<u32>(), true, A.flags.as<u8>(),
                static_cast<int>(sms), s);
    ++A.launches;
    u32 h0 = 0;
    u8 f0 = 0;
    B2_CUDA(cudaMemcpyAsync(&h0, A.hval.p, 4, cudaMemcpyDeviceToHost, s));
    B2_CUDA(cudaMemcpyAsync(&f0, A.flags.p, 1, cudaMemcpyDeviceToHost, s));
    comm_sync(comm, s);
    // the root's table entry and state stay only on its owner (the others keep row 0 as scratch)
    const bool own_root = dev_owner(root_hash, world) == me;
    if (!own_root)
    {
        B2_CUDA(cudaMemsetAsync(A.table.p, 0xFF, A.table_slots * 8, s));
        A.n_states = 0;
    }
    else
        A.n_states = 1;
    R.evaluations = 1;
    R.initial_h = h0 == kDeadEnd ? -1.0 : static_cast<double>(h0);
    const bool dead_start = h0 == kDeadEnd && !(f0 & kGoal);
    if (f0 & kGoal)
    {
        A.solved = true;
        A.cost = 0;
    }
    else if (dead_start)
        R.dead_ends = 1;
    u64 fcur = h0, nF = own_root ? 1 : 0, nopen = 0, nnext_all = 1;
    u64 expanded = 0, generated = 0, fresh_total = 0, dead = 0;
    u32 wave = 0, f_layers = 1, stamp = 0;
    bool exhausted = false;
    if (A.n_states >= (u64{1} << kRankShift))
        throw Error(B2_CAPACITY, "b2_astar: a rank of a sharded search holds at most 2^27 states");
    while (!A.solved && !dead_start)
    {
        if (A.opt.max_expansions && expanded * world >= A.opt.max_expansions)
            break;
        ++wave;
        ++stamp;
        ensure_front(A, nF);
        B2_CUDA(cudaMemsetAsync(misc, 0, offsetof(AstarMisc, nopen), s));
        if (nF)
        {
            const unsigned grid = grid_for(nF, 128, sms * 64);
            if (task->jit)
            {
                dev::BrfsArgs a{};
                a.frontier = A.front.as<u32>();
                a.E = nF;
                a.counts = A.counts.as<u32>();
                a.misc = &misc->lm;
                a.S.rows = A.rows.as<u64>();
                a.S.W = W;
                a.pi = pi;
                jit_launch(task->jit->get(kJitBrfsCount, pi), grid, 128, &a, s);
            }
            else
                dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                    k_count<OW, WR><<<grid, 128, 0, s>>>(T, pi, A.rows.as<u64>(), W, A.front.as<u32>(), nF,
                                                         A.counts.as<u32>(), &misc->lm);
                });
            ++A.launches;
        }
        if (A.sums.bytes < scan_scratch_bytes(nF))
            A.sums.alloc(scan_scratch_bytes(grow_to(nF, 0)), s);
        device_scan(CountIn{A.counts.as<u32>()}, BaseOut{A.cand_base.as<u64>()}, nF, &misc->lm.total_cand,
                    A.sums.as<u64>(), s, &misc->lm.status);
        if (nF)
            k_key_base<<<grid_for(nF, 256, sms * 16), 256, 0, s>>>(A.front.as<u32>(), nF, A.best.as<u64>(),
                                                                    A.counts.as<u32>(), u64{me} << kRankShift,
                                                                    A.keyb.as<u64>(), misc);
        B2_CUDA(cudaMemcpyAsync(&misc->gsum, &misc->lm.total_cand, 8, cudaMemcpyDeviceToDevice, s));
        comm_allreduce(comm, &misc->gsum, &misc->gsum, 1, CommType::U64, CommOp::Sum, s);
        A.launches += 4;
        const AstarMisc m1 = read_misc_sync(A);
        const u64 Gl = m1.lm.total_cand, Gt = m1.gsum;
        if (Gt > 0)
        {
            // stage this rank's successors by owner, then learn every rank's counts (the receive sizes)
            if (A.sstage.bytes < Gl * RW * 8)
                A.sstage.alloc(grow_to(Gl, A.sstage.bytes / (RW * 8)) * RW * 8, s);
            B2_CUDA(cudaMemsetAsync(hist, 0, world * 8, s));
            if (nF && Gl)
            {
                dev::DExpandArgs a{};
                a.rows = A.rows.as<u64>();
                a.frontier = A.front.as<u32>();
                a.frontier_id = A.iota.as<u32>();
                a.E = nF;
                a.layer_begin = 0;
                a.limit = ~u64{0};
                a.gbase = A.keyb.as<u64>();
                a.local_base = A.cand_base.as<u64>();
                a.stage_base = 0;
                a.staging = A.sstage.as<u64>();
                a.hist = hist;
                a.world = world;
                a.W = W;
                a.pi = pi;
                const unsigned grid = grid_for(nF, 128, sms * 64);
                if (task->jit)
                    jit_launch(task->jit->get(kJitDbrfsExpand, pi), grid, 128, &a, s);
                else
                    dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() { k_dexpand<OW, WR><<<grid, 128, 0, s>>>(T, a); });
                ++A.launches;
            }
            comm_allgather(comm, hist, M, world, CommType::U64, s);
            std::vector<u64> Mh(static_cast<std::size_t>(world) * world);
            B2_CUDA(cudaMemcpyAsync(Mh.data(), M, Mh.size() * 8, cudaMemcpyDeviceToHost, s));
            comm_sync(comm, s);
            u64 recv = 0, most = 0;
            for (u32 d = 0; d < world; ++d)
            {
                u64 col = 0;
                for (u32 r = 0; r < world; ++r)
                    col += Mh[static_cast<std::size_t>(r) * world + d];
                most = std::max(most, col);
                if (d == me)
                    recv = col;
            }
            // the same decision on every rank: receive buffers for the largest owner's records
            const u64 need = most * RW * 8;
            if (need > comm->exchange.bytes)
                peer_buffer_exchange(comm, comm->exchange, std::max<u64>(grow_to(need, comm->exchange.bytes / 2),
                                                                         u64{1} << 20), s);
            if (A.n_states + recv >= (u64{1} << kRankShift))
                throw Error(B2_CAPACITY, "b2_astar: a rank of a sharded search holds at most 2^27 states");
            ensure_wave(A, std::max<u64>(recv, 1), nopen);
            if (A.next.bytes < (recv + 1) * 4)
                A.next.alloc(grow_to(recv + 1, 0) * 4, s);
            ensure_states(A, A.n_states + recv);
            ensure_table(A, A.n_states + recv);
            B2_CUDA(cudaMemsetAsync(misc, 0, offsetof(AstarMisc, nnext), s));  // the count pass's status was read
            const u32 tile = std::min<u32>(kPushThreads, kPushSmemWords / RW);
            u64* cursor = hist;  // the counts were gathered: reuse as this rank's per-owner cursors
            B2_CUDA(cudaMemsetAsync(cursor, 0, world * 8, s));
            // a record past a receive buffer is dropped and flags the wave (the all-reduce below orders the pushes
            // before the inserts and sums the flags: every rank then fails the search with B2_CAPACITY)
            k_push<<<grid_for(Gl, tile, sms * 8), kPushThreads, tile * RW * 8, s>>>(
                A.sstage.as<u64>(), M, reinterpret_cast<u64* const*>(comm->exchange.table.p),
                reinterpret_cast<unsigned long long*>(cursor), me, world, RW, tile, comm->exchange.bytes / (RW * 8),
                &misc->lm.ndeferred);
            B2_CUDA(cudaGetLastError());
            comm_allreduce(comm, &misc->lm.ndeferred, &misc->lm.ndeferred, 1, CommType::U32, CommOp::Sum, s);
            A.launches += 1;
            if (recv)
            {
                const u64* in_rec = static_cast<const u64*>(comm->exchange.local.p);
                B2_CUDA(cudaMemsetAsync(A.best_rec.p, 0xFF, recv * 8, s));
                B2_CUDA(cudaMemsetAsync(A.claimed.p, 0, recv, s));
                InsertArgs in{};
                in.staging = in_rec;
                in.G = recv;
                in.W = W;
                in.wave = stamp;
                in.rows = A.rows.as<u64>();
                in.best = A.best.as<u64>();
                in.flags = A.flags.as<u8>();
                in.stamp = A.stamp.as<u32>();
                in.table = A.table.as<u64>();
                in.mask = A.table_slots - 1;
                in.max_probe = max_probe(A.table_slots);
                in.best_rec = A.best_rec.as<u64>();
                in.slot_of = A.slot_of.as<u64>();
                in.claimed = A.claimed.as<u8>();
                in.touched = A.touched.as<u32>();
                in.misc = misc;
                k_astar_insert<<<grid_for(recv, 256, sms * 16), 256, 0, s>>>(in);
                B2_CUDA(cudaGetLastError());
                ClaimOut co{in_rec, W, stamp, A.n_states, A.best_rec.as<u64>(), A.slot_of.as<u64>(),
                            A.table.as<u64>(), A.rows.as<u64>(), A.hash.as<u64>(), A.best.as<u64>(), A.flags.as<u8>(),
                            A.stamp.as<u32>(), A.fresh.as<u32>(), A.touched.as<u32>(), misc};
                device_scan(ClaimIn{A.claimed.as<u8>()}, co, recv, &misc->nfresh, A.sums.as<u64>(), s,
                            &misc->lm.status);
                launch_hmax(*A.H, A.rows.as<u64>(), W, A.fresh.as<u32>(), &misc->nfresh, recv, A.hval.as<u32>(), true,
                            A.flags.as<u8>(), static_cast<int>(sms), s);
                k_astar_push<<<grid_for(recv, 256, sms * 16), 256, 0, s>>>(A.touched.as<u32>(), misc, A.best.as<u64>(),
                                                                            A.hval.as<u32>(), A.flags.as<u8>(),
                                                                            static_cast<u32>(fcur), A.next.as<u32>(),
                                                                            A.open.as<u64>());
                B2_CUDA(cudaGetLastError());
                A.launches += 6;
            }
        }
        // the ranks' next waves and best goal (global ids: rank << 27 | state)
        B2_CUDA(cudaMemsetAsync(&misc->nnext_all, 0, 8, s));
        k_astar_globalize<<<1, 1, 0, s>>>(misc, u64{me} << kRankShift);
        comm_group_begin();
        comm_allreduce(comm, &misc->nnext_all, &misc->nnext_all, 1, CommType::U64, CommOp::Sum, s);
        comm_allreduce(comm, &misc->goal_all, &misc->goal_all, 1, CommType::U64, CommOp::Min, s);
        comm_group_end();
        const AstarMisc m = read_misc_sync(A);
        if (m.lm.ndeferred)
            throw Error(B2_CAPACITY, "b2_astar: a wave's successor records did not fit a rank's receive buffer");
        expanded += nF;
        generated += Gl;
        fresh_total += m.nfresh;
        dead += m.ndead;
        A.n_states += m.nfresh;
        nopen = m.nopen;
        nnext_all = m.nnext_all;
        if (m.goal_all != ~u64{0} && (m.goal_all >> 32) <= fcur)
        {
            A.solved = true;
            A.cost = m.goal_all >> 32;
            break;
        }
        if (nnext_all > 0)
        {
            A.front.swap(A.next);
            nF = m.nnext;
            continue;
        }
        // the current f is done everywhere: the smallest f of the ranks' open lists is next
        B2_CUDA(cudaMemsetAsync(&misc->fmin, 0xFF, 8, s));
        if (nopen)
            k_astar_fmin<<<grid_for(nopen, 256, sms * 16), 256, 0, s>>>(A.open.as<u64>(), nopen, A.best.as<u64>(),
                                                                          A.hval.as<u32>(), A.flags.as<u8>(), misc);
        comm_allreduce(comm, &misc->fmin, &misc->fmin, 1, CommType::U64, CommOp::Min, s);
        ++A.launches;
        const u64 fmin = read_misc_sync(A).fmin;
        if (fmin == ~u64{0})
        {
            exhausted = true;
            break;
        }
        if (m.goal_all != ~u64{0} && (m.goal_all >> 32) <= fmin)
        {
            A.solved = true;
            A.cost = m.goal_all >> 32;
            break;
        }
        fcur = fmin;
        ++f_layers;
        ensure_front(A, nopen);
        B2_CUDA(cudaMemsetAsync(&misc->nkeep, 0, 16, s));
        if (nopen)
        {
            k_astar_extract<<<grid_for(nopen, 256, sms * 16), 256, 0, s>>>(A.open.as<u64>(), nopen, A.best.as<u64>(),
                                                                             A.hval.as<u32>(), A.flags.as<u8>(), fmin,
                                                                             A.front.as<u32>(), A.keep.as<u64>(), misc);
            B2_CUDA(cudaGetLastError());
            ++A.launches;
        }
        const AstarMisc m4 = read_misc_sync(A);
        if (nopen)
            A.open.swap(A.keep);
        nopen = m4.nkeep;
        nF = m4.nfront;
        A.misc_host->nopen = nopen;
        B2_CUDA(cudaMemcpyAsync(&misc->nopen, &A.misc_host->nopen, 8, cudaMemcpyHostToDevice, s));
    }
    // the search's counters over all ranks
    A.misc_host->stats[0] = expanded;
    A.misc_host->stats[1] = generated;
    A.misc_host->stats[2] = A.n_states;
    A.misc_host->stats[3] = fresh_total;
    A.misc_host->stats[4] = dead;
    B2_CUDA(cudaMemcpyAsync(misc->stats, A.misc_host->stats, 5 * 8, cudaMemcpyHostToDevice, s));
    comm_allreduce(comm, misc->stats, misc->stats, 5, CommType::U64, CommOp::Sum, s);
    const AstarMisc mt = read_misc_sync(A);
    R.status = A.solved ? B2_SEARCH_SOLVED
                        : dead_start ? B2_SEARCH_UNSOLVABLE : exhausted ? B2_SEARCH_EXHAUSTED : B2_SEARCH_OUT_OF_STATES;
    R.cost = A.solved ? static_cast<double>(A.cost) : 0.0;
    R.expanded = mt.stats[0];
    R.generated = mt.stats[1];
    R.states = mt.stats[2];
    R.evaluations += mt.stats[3];
    R.dead_ends += mt.stats[4];
    R.waves = wave;
    R.f_layers = f_layers;
    R.plan_length = A.solved ? static_cast<u32>(A.cost) : 0;
    R.kernel_launches = A.launches;
    R.search_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

}  // namespace

extern "C" {

b2_status b2_heuristic_create(b2_task* task, int32_t kind, b2_heuristic** out)
{
    return guarded([&] {
        if (!task || !out)
            throw std::invalid_argument("b2_heuristic_create: null argument");
        if (kind != B2_HEURISTIC_MAX)
            throw Error(B2_UNSUPPORTED, "b2_heuristic_create: the device evaluates h^max only");
        *out = make_heuristic(task);
    });
}

b2_status b2_heuristic_info_get(const b2_heuristic* h, b2_heuristic_info* out)
{
    return guarded([&] {
        if (!h || !out)
            throw std::invalid_argument("b2_heuristic_info_get: null argument");
        out->props = h->R.props;
        out->ops = h->R.ops();
        out->reached_atoms = h->R.reached;
        out->ground_actions = h->R.ground_actions;
        out->goal_atoms = static_cast<uint32_t>(h->R.goal.size());
        out->goal_unreachable = h->R.goal_unreachable ? 1 : 0;
    });
}

b2_status b2_heuristic_evaluate(b2_heuristic* h, const uint64_t* rows, uint64_t stride, uint32_t words, uint64_t n,
                                uint32_t* out, void* stream)
{
    return guarded([&] {
        if (!h || (n && (!rows || !out)))
            throw std::invalid_argument("b2_heuristic_evaluate: null argument");
        if (!h->task->ctx)
            throw std::invalid_argument("a host-only task (created without a context) cannot run on the device");
        if (words != h->task->prog.words || stride < words)
            throw std::invalid_argument("b2_heuristic_evaluate: rows must have the task's " +
                                        std::to_string(h->task->prog.words) + " words (stride >= words)");
        if (!n)
            return;
        B2_CUDA(cudaSetDevice(h->task->ctx->device));
        launch_hmax(*h, rows, stride, nullptr, nullptr, n, out, false, nullptr, h->task->ctx->sms,
                    static_cast<cudaStream_t>(stream));
    });
}

void b2_heuristic_destroy(b2_heuristic* h)
{
    if (h && h->task && h->task->ctx)
        cudaSetDevice(h->task->ctx->device);  // the cached search buffers are this device's
    delete h;
}

void b2_astar_options_default(b2_astar_options* o)
{
    if (!o)
        return;
    *o = b2_astar_options{};
}

b2_status b2_astar_create(b2_task* task, const b2_astar_options* options, b2_astar** out)
{
    return guarded([&] {
        if (!task || !options || !out)
            throw std::invalid_argument("b2_astar_create: null argument");
        if (!task->ctx)
            throw std::invalid_argument("a host-only task (created without a context) cannot run on the device");
        if (options->witness_pruning && task->witness_refused)
            throw Error(B2_UNSUPPORTED, "witness pruning with a witness parameter before an effect parameter");
        B2_CUDA(cudaSetDevice(task->ctx->device));
        auto A = std::make_unique<b2_astar>();
        A->task = task;
        A->opt = *options;
        A->W = task->prog.words;
        if (options->heuristic)
        {
            if (options->heuristic->task != task)
                throw std::invalid_argument("b2_astar_create: the heuristic belongs to another task");
            A->H = options->heuristic;
        }
        else
        {
            A->H = make_heuristic(task);
            A->own_h = true;
        }
        if (options->stream)
            A->stream = static_cast<cudaStream_t>(options->stream);
        else
        {
            B2_CUDA(cudaStreamCreateWithFlags(&A->stream, cudaStreamNonBlocking));
            A->own_stream = true;
        }
        if (options->heuristic && !options->heuristic->cache.busy)
        {
            // reuse the buffers the heuristic's previous search left (their contents are stale: the search clears
            // what it reads)
            AstarCache& c = options->heuristic->cache;
            auto bufs = A->buffers();
            auto caps = A->caps();
            for (int i = 0; i < kAstarBuffers; ++i)
                bufs[i]->swap(c.bufs[i]);
            for (int i = 0; i < kAstarCaps; ++i)
                *caps[i] = c.caps[i];
            c.busy = true;
            A->borrowed = true;
        }
        if (A->hist.bytes < 64)
            A->hist.alloc(64, A->stream);
        if (options->comm)
        {
            if (options->comm->device != task->ctx->device)
                throw std::invalid_argument("b2_astar_create: the communicator belongs to another device");
            A->comm = options->comm;
        }
        *out = A.release();
    });
}

b2_status b2_astar_run(b2_astar* A, b2_astar_result* result)
{
    return guarded([&] {
        if (!A || !result)
            throw std::invalid_argument("b2_astar_run: null argument");
        if (A->ran)
            throw std::invalid_argument("b2_astar_run: the search ran already");
        A->ran = true;
        B2_CUDA(cudaSetDevice(A->task->ctx->device));
        *result = b2_astar_result{};
        if (A->comm)
            run_astar_sharded(*A, *result);
        else
            run_astar(*A, *result);
    });
}

b2_status b2_astar_plan(b2_astar* A, uint32_t* parent, uint32_t* index, uint32_t cap, uint32_t* len)
{
    return guarded([&] {
        if (!A || !len || !A->ran)
            throw std::invalid_argument("b2_astar_plan: bad argument");
        if (!A->solved)
            throw std::invalid_argument("b2_astar_plan: the search found no plan");
        if (A->comm)
            throw Error(B2_UNSUPPORTED, "b2_astar_plan: a sharded search keeps no plan");
        const u32 n = static_cast<u32>(A->cost);
        *len = n;
        if (cap < n || !n)
            return;
        if (!parent || !index)
            throw std::invalid_argument("b2_astar_plan: null output");
        B2_CUDA(cudaSetDevice(A->task->ctx->device));
        DeviceBuffer tmp;
        tmp.alloc((2 * static_cast<u64>(n) + 1) * 4);
        u32* tp = tmp.as<u32>();
        k_astar_path<<<1, 1, 0, A->stream>>>(A->best.as<u64>(), A->goal_state, n, tp, tp + n, tp + 2 * n);
        B2_CUDA(cudaGetLastError());
        std::vector<u32> host(2 * static_cast<u64>(n) + 1);
        B2_CUDA(cudaMemcpyAsync(host.data(), tp, host.size() * 4, cudaMemcpyDeviceToHost, A->stream));
        B2_CUDA(cudaStreamSynchronize(A->stream));
        if (host[2 * n] != n)
            throw Error(B2_DEVICE_FAULT, "b2_astar_plan: the parent chain does not reach the root in cost steps");
        for (u32 i = 0; i < n; ++i)  // root first
        {
            parent[i] = host[n - 1 - i];
            index[i] = host[n + n - 1 - i];
        }
    });
}

void b2_astar_destroy(b2_astar* A)
{
    if (!A)
        return;
    cudaSetDevice(A->task->ctx->device);
    if (A->borrowed)
    {
        // the buffers go back to the heuristic's cache, usable from any stream once this search's work is done
        // (a later release frees them on the default stream)
        if (A->stream)
            stream_drain(A->stream);
        AstarCache& c = A->H->cache;
        auto bufs = A->buffers();
        auto caps = A->caps();
        for (int i = 0; i < kAstarBuffers; ++i)
        {
            bufs[i]->stream = nullptr;
            bufs[i]->swap(c.bufs[i]);
        }
        for (int i = 0; i < kAstarCaps; ++i)
            c.caps[i] = *caps[i];
        c.busy = false;
    }
    for (DeviceBuffer* b : A->buffers())
        b->reset();
    if (A->stream)
    {
        stream_drain(A->stream);
        if (A->own_stream)
            cudaStreamDestroy(A->stream);
    }
    A->task->ctx->pinned.give(A->misc_host);
    if (A->own_h)
        delete A->H;
    delete A;
}

}  // extern "C"
