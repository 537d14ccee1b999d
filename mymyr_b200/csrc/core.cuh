// Device primitives shared by the nvcc-compiled kernels and the per-task kernels compiled at run time (NVRTC): scalar
// types, the reference's state hash and Philox RNG (bit-exact restatements), register rows, bit extraction, the
// hash-set insert protocol of the BrFS, and the kernel argument blocks. Self-contained: no standard headers, so that
// NVRTC compiles it as is.

#pragma once

#if defined(__CUDACC_RTC__)
typedef unsigned char u8_t;
typedef unsigned int u32_t;
typedef unsigned long long u64_t;
typedef int i32_t;
typedef long long i64_t;
#else
#include <cstdint>
typedef std::uint8_t u8_t;
typedef std::uint32_t u32_t;
typedef std::uint64_t u64_t;
typedef std::int32_t i32_t;
typedef std::int64_t i64_t;
#endif

namespace b2
{
namespace dev
{
using u8 = u8_t;
using u32 = u32_t;
using u64 = u64_t;
using i32 = i32_t;
using i64 = i64_t;

#define B2_DI __device__ __forceinline__

// ------------------------------------------------------------------------------------------------ hash
// hash::mix64 / mulfold / words / state_words (include/mymyr/core/hash.hpp:12-55 of maichmueller/mymyr).
constexpr u64 kHashSeed = 0x2d358dccaa6c78a5ULL;
constexpr u64 kHashP1 = 0x8bb84b93962eacc9ULL;
constexpr u64 kHashP2 = 0x4b33a62ed433d4a3ULL;

B2_DI u64 mix64(u64 x)
{
    x ^= x >> 30;
    x *= 0xbf58476d1ce4e5b9ULL;
    x ^= x >> 27;
    x *= 0x94d049bb133111ebULL;
    x ^= x >> 31;
    return x;
}

B2_DI u64 mulfold(u64 a, u64 b) { return (a * b) ^ __umul64hi(a, b); }

/// hash::words over all n words w(0..n-1), untrimmed; `seed` as hash::words takes it.
template<class Get>
B2_DI u64 hash_span(Get&& w, u32 n, u64 seed = kHashSeed)
{
    u64 h = seed ^ (static_cast<u64>(n) * kHashP1);
    u32 i = 0;
    for (; i + 1 < n; i += 2)
        h = mulfold(h ^ w(i) ^ kHashP1, w(i + 1) ^ kHashP2);
    if (i < n)
        h = mulfold(h ^ w(i) ^ kHashP1, kHashP2);
    return mix64(h);
}

/// hash::state_words over words w(0..W-1) of a zero-padded row (trailing zero words ignored); a row with numeric
/// words passes their hash_span as the seed (hash::state).
template<class Get>
B2_DI u64 hash_words(Get&& w, u32 W, u64 seed = kHashSeed)
{
    u32 n = W;
    while (n > 0 && w(n - 1) == 0)
        --n;
    return hash_span(w, n, seed);
}

/// hash_words for a compile-time width NW (every loop unrolled, so register rows are indexed by constants); the
/// trimmed length stays a run-time value: pair i is folded iff i + 1 < n, the odd tail iff i == n - 1.
template<int NW, class Get>
B2_DI u64 hash_words_fixed(Get&& w)
{
    u32 n = 0;
#pragma unroll
    for (int i = 0; i < NW; ++i)
        n = w(i) != 0 ? static_cast<u32>(i + 1) : n;
    u64 h = kHashSeed ^ (static_cast<u64>(n) * kHashP1);
#pragma unroll
    for (int i = 0; i < NW; i += 2)
    {
        const u64 a = w(i), b = i + 1 < NW ? w(i + 1) : 0;
        if (static_cast<u32>(i) + 1 < n)
            h = mulfold(h ^ a ^ kHashP1, b ^ kHashP2);
        else if (static_cast<u32>(i) < n)
            h = mulfold(h ^ a ^ kHashP1, kHashP2);
    }
    return mix64(h);
}

/// brfs_fingerprint_term (src/mymyr/search/brfs.cpp:34-37).
B2_DI u64 fingerprint_term(u64 id, u64 canonical) { return mix64(id * 0x9E3779B97F4A7C15ULL ^ canonical); }

// ------------------------------------------------------------------------------------------------ static key sets
/// The empty slot of a static predicate's key set (no packed key of an arity below 8 has its top byte set).
constexpr u64 kNoStaticKey = ~u64{0};

/// Home slot of a packed static key in a key set of mask + 1 slots.
B2_DI u64 static_key_slot(u64 key, u64 mask) { return mix64(key ^ 0x6a09e667f3bcc909ULL) & mask; }

/// Membership of a packed key in a static key set: linear probing from its home slot, at most `probes` slots (the
/// longest run any stored key needed when the set was built).
B2_DI bool static_member(const u64* table, u64 mask, u32 probes, u64 key)
{
    u64 j = static_key_slot(key, mask);
    for (u32 i = 0; i < probes; ++i, j = (j + 1) & mask)
    {
        const u64 x = table[j];
        if (x == key)
            return true;
        if (x == kNoStaticKey)
            return false;
    }
    return false;
}

// ------------------------------------------------------------------------------------------------ Philox
// rl::rng (include/mymyr/rl/rng.hpp:45-84): Philox-4x32-10 of (seed; draw lo, draw hi, env, purpose).
B2_DI u64 philox_bits64(u64 seed, u64 env, u64 draw, u32 purpose)
{
    u32 c0 = static_cast<u32>(draw), c1 = static_cast<u32>(draw >> 32), c2 = static_cast<u32>(env), c3 = purpose;
    u32 k0 = static_cast<u32>(seed), k1 = static_cast<u32>(seed >> 32);
#pragma unroll
    for (int r = 0; r < 10; ++r)
    {
        const u32 hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
        const u32 hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
        const u32 n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0;
        c1 = lo1;
        c2 = n2;
        c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return static_cast<u64>(c0) | (static_cast<u64>(c1) << 32);
}

/// The position of the r-th set bit (0-based, from the lowest) of x; x has more than r set bits.
B2_DI u32 nth_bit64(u64 x, u32 r)
{
    const u32 lo = static_cast<u32>(x), k = static_cast<u32>(__popc(lo));
    return r < k ? __fns(lo, 0u, static_cast<int>(r + 1)) : 32u + __fns(static_cast<u32>(x >> 32), 0u, static_cast<int>(r - k + 1));
}

/// high64(x * n) (rng::below).
B2_DI u32 below(u64 x, u32 n)
{
    const u64 hi = (x >> 32) * n, lo = (x & 0xFFFFFFFFull) * n;
    return static_cast<u32>((hi + (lo >> 32)) >> 32);
}

// ------------------------------------------------------------------------------------------------ sorted bindings
/// Emits the bindings that raw(f) enumerates (f(const u32* b) for each, `arity` parameters, objects below 256) in
/// canonical order, the order the reference emits a matcher's bindings in when the matcher does not bind in index
/// order (it buffers them, packs them into keys and sorts them): the keys (8 bits per parameter, the first highest) of
/// up to 16 bindings are buffered and sorted; more are emitted by selection passes, each of which enumerates again and
/// emits the smallest key above the last one. emit returning false stops (and returns false).
template<class Raw, class Emit>
B2_DI bool emit_sorted(u32 arity, Raw&& raw, Emit&& emit)
{
    constexpr u32 kBuf = 16;
    u64 buf[kBuf];
    u32 n = 0;
    bool over = false;
    raw([&](const u32* b) {
        u64 k = 0;
        for (u32 v = 0; v < arity; ++v)
            k = (k << 8) | b[v];
        if (n < kBuf)
            buf[n++] = k;
        else
            over = true;
        return true;
    });
    u32 b[8];
    const auto unpack = [&](u64 k) {
        for (u32 v = arity; v-- > 0;)
        {
            b[v] = static_cast<u32>(k & 0xFFu);
            k >>= 8;
        }
    };
    if (!over)
    {
        for (u32 i = 1; i < n; ++i)
        {
            const u64 x = buf[i];
            u32 j = i;
            while (j > 0 && buf[j - 1] > x)
            {
                buf[j] = buf[j - 1];
                --j;
            }
            buf[j] = x;
        }
        for (u32 i = 0; i < n; ++i)
        {
            unpack(buf[i]);
            if (!emit(static_cast<const u32*>(b)))
                return false;
        }
        return true;
    }
    u64 last = 0;
    bool first = true;
    for (;;)
    {
        u64 best = ~u64{0};
        bool any = false;
        raw([&](const u32* x) {
            u64 k = 0;
            for (u32 v = 0; v < arity; ++v)
                k = (k << 8) | x[v];
            if ((first || k > last) && k <= best)
            {
                best = k;
                any = true;
            }
            return true;
        });
        if (!any)
            return true;
        unpack(best);
        if (!emit(static_cast<const u32*>(b)))
            return false;
        last = best;
        first = false;
    }
}

// ------------------------------------------------------------------------------------------------ rows
/// A state row of up to WR words in registers; word(i) for i >= WR reads zero.
template<int WR>
struct RegRow
{
    u64 w[WR];
    B2_DI u64 word(u32 i) const
    {
        u64 r = 0;
#pragma unroll
        for (int k = 0; k < WR; ++k)
            r = (static_cast<u32>(k) == i) ? w[k] : r;
        return r;
    }
    B2_DI void set(u32 bit)
    {
#pragma unroll
        for (int k = 0; k < WR; ++k)
            w[k] |= (static_cast<u32>(k) == (bit >> 6)) ? (u64{1} << (bit & 63)) : 0;
    }
    B2_DI void clear(u32 bit)
    {
#pragma unroll
        for (int k = 0; k < WR; ++k)
            w[k] &= (static_cast<u32>(k) == (bit >> 6)) ? ~(u64{1} << (bit & 63)) : ~u64{0};
    }
};

/// A state row read from global memory (rows wider than the register classes).
struct GlobalRow
{
    const u64* p;
    u32 W;
    B2_DI u64 word(u32 i) const { return i < W ? __ldg(p + i) : 0; }
};

template<int WR>
B2_DI RegRow<WR> load_reg_row(const u64* p, u32 W)
{
    RegRow<WR> r;
#pragma unroll
    for (int k = 0; k < WR; ++k)
        r.w[k] = static_cast<u32>(k) < W ? p[k] : 0;
    return r;
}

template<class St>
B2_DI bool bit_of(const St& st, u64 bit)
{
    return (st.word(static_cast<u32>(bit >> 6)) >> (bit & 63)) & 1;
}

/// 64 bits of the row from bit `pos` (bits past the row read as zero).
template<class St>
B2_DI u64 extract64(const St& st, u64 pos)
{
    const u32 w = static_cast<u32>(pos >> 6), sh = static_cast<u32>(pos & 63);
    const u64 lo = st.word(w) >> sh;
    return sh ? lo | (st.word(w + 1) << (64 - sh)) : lo;
}

/// The successor word i of a parent under delete-then-add effect slots.
template<class St>
B2_DI u64 succ_word(const St& st, const u32* del, u32 nd, const u32* add, u32 na, u32 i)
{
    u64 w = st.word(i);
    for (u32 j = 0; j < nd; ++j)
        if ((del[j] >> 6) == i)
            w &= ~(u64{1} << (del[j] & 63));
    for (u32 j = 0; j < na; ++j)
        if ((add[j] >> 6) == i)
            w |= u64{1} << (add[j] & 63);
    return w;
}

/// canonical_hash of a dense-slot state (src/mymyr/task/task.cpp:387-403).
template<class St>
B2_DI u64 canonical_hash(const St& st, u32 W)
{
    u64 x = 0;
    for (u32 i = 0; i < W; ++i)
    {
        u64 w = st.word(i);
        while (w)
        {
            const u32 b = __ffsll(static_cast<long long>(w)) - 1;
            w &= w - 1;
            x ^= mix64(static_cast<u64>(i) * 64 + b + 0x1234567ULL);
        }
    }
    return x;
}

// ------------------------------------------------------------------------------------------------ status words
constexpr u32 kStatusProbeLimit = 1u;
constexpr u32 kStatusEffectOverflow = 2u;
constexpr u32 kStatusCapacity = 4u;
constexpr u32 kStatusTaskId = 8u;  // an env's next_task_ids named a task it does not have

/// Resident blocks per SM of the compiled BrFS expansion (its launch bound, and the device-driven loop's grid).
constexpr u32 kBrfsExpandBlocksPerSm = 8;

// ------------------------------------------------------------------------------------------------ BrFS hash set
constexpr u64 kEmpty = ~u64{0};

/// The device side of a BrFS layer: per-candidate arenas (row, hash, parent index, successor index), the
/// open-addressing set of u64 slots (hash >> 32) << 32 | g, and the layer's claim/loss flags and deferred inserts.
struct Store
{
    u64* rows;
    u64* hash;
    u32* par;
    u32* kid;
    u64* table;
    u64 mask;
    u32 W;
    u32 max_probe;
    u8* claimed;  // per candidate of the layer
    u8* lost;
    u64 layer_cand_begin;
    u32* status;
    u64* deferred;  // (slot << 32 | candidate g) of inserts left to the resolve pass
    u32* ndeferred;
};

/// Phase A of an insert, with no fence and no acquire: other threads read this candidate's row only in the resolve
/// pass (a later kernel), so plain stores suffice. A slot holding a state of an earlier layer is compared in place
/// (its row was written by an earlier kernel); an empty slot is claimed by CAS; a slot holding a candidate of this
/// layer with the same tag defers the insert (row, hash and node record written first) to the resolve pass.
/// Calls f(q) for q < NW (unrolled) or, with NW == 0, for q < W.
template<int NW, class F>
B2_DI void for_words(u32 W, F&& f)
{
    if constexpr (NW > 0)
    {
#pragma unroll
        for (int q = 0; q < NW; ++q)
            f(static_cast<u32>(q));
    }
    else
        for (u32 q = 0; q < W; ++q)
            f(q);
}

template<int NW, class Row>
B2_DI void write_candidate(const Store& S, const Row& s, u64 h, u64 g, u32 i, u32 k)
{
    u64* r = S.rows + g * S.W;
    for_words<NW>(S.W, [&](u32 q) { r[q] = s.word(q); });
    S.hash[g] = h;
    S.par[g] = i;
    S.kid[g] = k;
}

/// NW: the row width when it is a compile-time constant (0: S.W at run time).
template<int NW = 0, class Row>
B2_DI void insert(const Store& S, const Row& s, u64 h, u64 g, u32 i, u32 k)
{
    const u64 mine = (h & 0xFFFFFFFF00000000ull) | g;
    u64 j = h & S.mask;
    for (u32 probe = 0; probe < S.max_probe; ++probe, j = (j + 1) & S.mask)
    {
        u64 cur = __ldcg(S.table + j);
        if (cur == kEmpty)
        {
            const u64 prev = atomicCAS(reinterpret_cast<unsigned long long*>(S.table + j), kEmpty, mine);
            if (prev == kEmpty)
            {
                write_candidate<NW>(S, s, h, g, i, k);
                S.claimed[g - S.layer_cand_begin] = 1;
                return;
            }
            cur = prev;
        }
        if ((cur >> 32) != (mine >> 32))
            continue;
        const u64 og = cur & 0xFFFFFFFFull;
        if (og >= S.layer_cand_begin)
        {
            write_candidate<NW>(S, s, h, g, i, k);
            const u32 q = atomicAdd(S.ndeferred, 1u);
            S.deferred[q] = (j << 32) | g;
            return;
        }
        const u64* r = S.rows + og * S.W;
        bool eq = true;
        for_words<NW>(S.W, [&](u32 q) { eq = eq && __ldcg(r + q) == s.word(q); });
        if (eq)
            return;  // a state of an earlier layer
    }
    atomicOr(S.status, kStatusProbeLimit);
}

/// insert() for up to NB candidates of one lane at once (n valid), with their probes interleaved so that their memory
/// accesses overlap: candidate e has hash h[e], candidate index g[e], parent index i[e], successor index k[e] and row
/// words rw(e, q). Same protocol and outcomes as insert(), step by step: read the slot; claim an empty one by CAS;
/// compare a state of an earlier layer in place; defer a tag match with a candidate of this layer.
template<int NB, int NW, class RowWord>
B2_DI void insert_batch(const Store& S, u32 n, const u64* h, const u64* g, const u32* i, const u32* k, RowWord&& rw)
{
    u64 j[NB], mine[NB], og[NB];
    u32 ph[NB], probes[NB];  // ph: 0 done, 1 read the slot at j, 2 claim it by CAS, 3 compare the row of og
#pragma unroll
    for (int e = 0; e < NB; ++e)
    {
        ph[e] = static_cast<u32>(e) < n ? 1u : 0u;
        mine[e] = (h[e] & 0xFFFFFFFF00000000ull) | g[e];
        j[e] = h[e] & S.mask;
        og[e] = 0;
        probes[e] = 0;
    }
    for (;;)
    {
        u32 any = 0;
#pragma unroll
        for (int e = 0; e < NB; ++e)
            any |= ph[e];
        if (!any)
            break;
        u64 cur[NB];
        bool eq[NB];
#pragma unroll
        for (int e = 0; e < NB; ++e)
        {
            cur[e] = 0;
            eq[e] = false;
            if (ph[e] == 1)
                cur[e] = __ldcg(S.table + j[e]);
            else if (ph[e] == 2)
                cur[e] = atomicCAS(reinterpret_cast<unsigned long long*>(S.table + j[e]), kEmpty, mine[e]);
            else if (ph[e] == 3)
            {
                const u64* r = S.rows + og[e] * S.W;
                bool same = true;
                for_words<NW>(S.W, [&](u32 q) { same = same && __ldcg(r + q) == rw(e, q); });
                eq[e] = same;
            }
        }
#pragma unroll
        for (int e = 0; e < NB; ++e)
        {
            if (ph[e] == 3)
            {
                if (eq[e])
                    ph[e] = 0;  // a state of an earlier layer
                else
                {
                    j[e] = (j[e] + 1) & S.mask;
                    ph[e] = ++probes[e] < S.max_probe ? 1u : 4u;
                }
                continue;
            }
            if (ph[e] != 1 && ph[e] != 2)
                continue;
            if (cur[e] == kEmpty)
            {
                if (ph[e] == 2)
                {
                    const u64 ge = g[e];
                    u64* r = S.rows + ge * S.W;
                    for_words<NW>(S.W, [&](u32 q) { r[q] = rw(e, q); });
                    S.hash[ge] = h[e];
                    S.par[ge] = i[e];
                    S.kid[ge] = k[e];
                    S.claimed[ge - S.layer_cand_begin] = 1;
                    ph[e] = 0;
                }
                else
                    ph[e] = 2;
                continue;
            }
            if ((cur[e] >> 32) != (mine[e] >> 32))
            {
                j[e] = (j[e] + 1) & S.mask;
                ph[e] = ++probes[e] < S.max_probe ? 1u : 4u;
                continue;
            }
            og[e] = cur[e] & 0xFFFFFFFFull;
            if (og[e] >= S.layer_cand_begin)
            {
                // a candidate of this layer with the same tag: this one's record, then the resolve pass
                const u64 ge = g[e];
                u64* r = S.rows + ge * S.W;
                for_words<NW>(S.W, [&](u32 q) { r[q] = rw(e, q); });
                S.hash[ge] = h[e];
                S.par[ge] = i[e];
                S.kid[ge] = k[e];
                const u32 qd = atomicAdd(S.ndeferred, 1u);
                S.deferred[qd] = (j[e] << 32) | ge;
                ph[e] = 0;
            }
            else
                ph[e] = 3;
        }
#pragma unroll
        for (int e = 0; e < NB; ++e)
            if (ph[e] == 4)
            {
                atomicOr(S.status, kStatusProbeLimit);
                ph[e] = 0;
            }
    }
}

// ------------------------------------------------------------------------------------------------ kernel arguments
struct LayerMisc
{
    u64 total_cand;  // candidates of the layer (scan total)
    u64 total_new;   // new states of the layer (scan total)
    u64 fingerprint;
    u32 goals;       // goal states among the layer's parents
    u32 first_goal;  // smallest parent index that is a goal (0xFFFFFFFF: none)
    u32 status;
    u32 ndeferred;   // inserts left to the resolve pass
};

/// The state of a BrFS whose layer loop runs on the device (a CUDA graph's while node): the layer's sizes live here,
/// the kernels of the loop read them, and a few one-thread kernels advance them.
struct DevLayerState
{
    u64 layer_begin, layer_end;  // ids of the current layer's states
    u64 n_states, cand_next;     // stored states, candidates so far
    u64 E, E_exp, G;             // the layer's parents, parents expanded, candidates (0 when the layer is skipped)
    u64 expanded, generated, goals, goal_id;
    u64 cap_layer, cap_flags, cap_cand, cap_states, table_slots;  // the buffers the loop was built over
    u64* log;                    // [log_cap, 3] per layer: expanded, generated, new
    u32 log_cap;
    u32 layers, max_depth, stop_at_goal;
    u32 done;                    // the search is over (exhausted, depth bound, goal stop)
    u32 overflow;                // a buffer is too small for the current layer: left to the host, nothing of it done
    u32 exhausted, solved, stop, cut;  // cut: ended at stop_frontier, the search goes on elsewhere
    u64 stop_frontier;           // 0, or end the loop after the first layer with at least this many new states
    LayerMisc misc;              // the current layer's counters
};

/// Arguments of the BrFS count / expand kernels.
struct BrfsArgs
{
    const u32* frontier;  // candidate index of each parent
    u64 E;                // parents
    u32* counts;          // [E] successor counts (count pass)
    const u64* cand_base; // [E] candidate offsets (expand pass)
    LayerMisc* misc;
    Store S;
    u32 pi;               // 0: witness pruning, 1: off
    const u64* E_dev;     // count pass: when non-null, the parents are *E_dev (a count still on the device), not E
    u64* hist;            // sharded count pass: successors per owner rank (added to)
    u32 world;            // sharded count pass: ranks
    const DevLayerState* dyn;  // device-driven loop: frontier = frontier + layer_begin, the parents E (count) or E_exp
                               // (expand) and the layer's first candidate come from here
};

// ------------------------------------------------------------------------------------------------ sharded BrFS
constexpr u32 kMaxWorld = 64;

/// The owner rank of a state hash among `world` ranks: the high 32 bits of the hash, scaled to [0, world).
B2_DI u32 owner_of(u64 h, u32 world) { return static_cast<u32>(((h >> 32) * world) >> 32); }

/// Per-layer values of a sharded search (device side, mirrored to pinned host memory).
struct DistMisc
{
    LayerMisc lm;     // count pass over the local parents: goals, first local goal, status
    u64 total_local;  // local candidates of the layer (scan of the local counts)
    u64 goal_id;      // smallest goal id among the layer's parents (this rank's, then the MIN over ranks)
    u64 new_packed;   // new states of the layer: all ranks | this rank's << 32
    u64 recv;         // candidates this rank received
    u64 fingerprint;
    u64 sent_self;    // records this rank pushed to itself (the rest of those received came over NVLink)
    u64 recv_me;      // successors of the layer owned by this rank (from the all-reduced per-owner counts)
    u64 recv_max;     // the most successors of the layer any rank owns
    u64 cut;          // max_states: 1 + the key (parent id << 32 | successor index) of the last state kept (MAX)
    u64 kept;         // max_states: this rank's new states of the layer with an id below max_states
    u64 next_all;     // new states of the layer over all ranks (the next layer's parents), unpacked on the device
    u64 next_local;   // new states of the layer on this rank (its next local parents)
    u32 goals_all;    // goal parents of the layer over all ranks
    u32 overflow_all; // parents over all ranks whose successor count did not fit the count lanes
    u32 barrier;      // reduced by all ranks between the exchange and the inserts
    u32 pad;
};

/// Arguments of the sharded expansion: each local parent's successors are staged as records [row | hash | key], key =
/// the parent's key base + successor index. With gbase null the key base is id << 32, so that keys order successors in
/// canonical order (parent id, successor index) over all ranks.
struct DExpandArgs
{
    const u64* rows;         // the rank's arena rows (parents)
    const u32* frontier;     // arena index of each local parent (local parents are in id order)
    const u32* frontier_id;  // id of each local parent
    u64 E;                   // local parents
    u64 layer_begin;         // id of the layer's first state
    u64 limit;               // expand the parents with id < limit
    const u64* gbase;        // [layer states] key base of each parent of the layer, or null (id << 32)
    const u64* local_base;   // [E] staging record of each local parent's first successor (minus stage_base)
    u64 stage_base;          // subtracted from local_base (a chunk of a larger batch stages from 0)
    u64* staging;            // [local candidates, W + 2]
    u64* hist;               // [world] staged records per owner rank
    u32 world;
    u32 W;
    u32 pi;                  // 0: witness pruning, 1: off
    u32 me;                  // fused push (b2j_dbrfs_push): this rank
    u64* const* peers;       // fused push: each rank's receive buffer (peer memory)
    u64* const* cursors;     // fused push: each rank's fill cursor (peer memory)
    unsigned long long* sent_self;  // fused push: records pushed to this rank
    u64 recv_cap;            // fused push: records each rank's receive buffer holds; a record past it is dropped
    u32* overflow;           // fused push: set to 1 when a record was dropped (reduced over the ranks by the host)
};

/// Arguments of the env kernels (b2_env_batch and b2_step_out, flattened).
struct EnvArgs
{
    u64* states;
    u64 rows;
    u32 words;
    u32 label_width;
    i32* steps;
    u64* draws;
    u8* at_goal;
    u32* counts;
    u64 first_env;
    float* reward;
    u8* terminated;
    u8* truncated;
    i32* count;
    u64* final_states;
    i32* schema;
    i32* binding;
    u8* invalid;
    u8* goal;
    const i64* actions;
    const u64* init;       // the initial row
    const u32* init_info;  // goal, total, per-schema counts of the initial state
    u32* status;
    u64 seed;
    u32 max_steps;
    float step_reward, goal_reward, dead_end_reward;
    u32 dead_end_none, dead_end_terminal, autoreset, pi;
};

/// Arguments of the batched-expand kernels.
struct ExpandArgs
{
    const u64* states;
    u64 rows;
    u32 W;
    u32 pi;
    u32* counts;          // [rows * schemas]
    const u64* seg_off;   // [rows * schemas]
    u64 capacity;
    u32 out_words;
    u32 label_width;
    u64* succ;
    i32* parent;
    i32* schema;
    i32* binding;
    u64* succ_hash;
    u32* status;
    const u64* total;     // the call's successors (device), for the hash pass
    u32 hash_pass;        // successor hashes and rows by a separate pass over the written records
};
}  // namespace dev
}  // namespace b2
