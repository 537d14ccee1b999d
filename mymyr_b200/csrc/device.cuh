// Device-side core of the path: the task view the kernels read, the reference's state hash and Philox RNG
// (bit-exact restatements), and the lifted matcher.
//
// The matcher enumerates the applicable bindings of one schema in one state in canonical order (parameters in
// index order, each level's candidates ascending): a depth-first search over object bitsets of OW words where a
// level's candidates are the static domain AND the runs of fluent relations selected by earlier parameters AND
// static row tables; literals of arity >= 3 are checked when their last parameter is bound. Witness-only parameters
// (witness pruning) are bound last and only the first completion is emitted. Rows never leave registers: a run of a
// fluent relation is extracted from the state words directly (no per-state view table).

#pragma once

#include "core.cuh"
#include "task.hpp"

#include <cstdint>
#include <cuda_runtime.h>

namespace b2
{
#define B2_HD __host__ __device__ __forceinline__

// Hash, Philox, rows and bit extraction come from core.cuh (shared with the run-time compiled kernels).
using dev::below;
using dev::bit_of;
using dev::canonical_hash;
using dev::extract64;
using dev::fingerprint_term;
using dev::GlobalRow;
using dev::hash_words;
using dev::mix64;
using dev::philox_bits64;
using dev::RegRow;
using dev::static_member;

template<class St>
__device__ __forceinline__ bool test_bit(const St& st, u64 bit)
{
    return bit_of(st, bit);
}

// ------------------------------------------------------------------------------------------------ task view
/// Device pointers into the uploaded program (one blob), plus scalars. Passed to kernels by value.
struct DevTask
{
    u32 n, ow, words, nschemas, label_width, goal_unsat;
    u64 fluent_count;
    const u64* pool;
    const DLit* lits;
    const DVar* vars;
    const DFilter* filters;
    const DLevel* levels;
    const u32* checks;
    const DSchema* schemas;
    const u32* domain;
    const u32* pos_dom_begin;
    const u64* srel_table;   // per predicate: pool offset of its static key set
    const u64* srel_mask;
    const u64* srel_probes;
    const u64* goal_pos;
    const u64* goal_neg;
};

// ------------------------------------------------------------------------------------------------ matcher
template<int OW>
struct ObjSet
{
    u64 w[OW];
};

template<int OW>
__device__ __forceinline__ void or_shifted(ObjSet<OW>& s, u64 bits, u32 at)
{
    const u32 wi = at >> 6, sh = at & 63;
#pragma unroll
    for (int k = 0; k < OW; ++k)
    {
        if (static_cast<u32>(k) == wi)
            s.w[k] |= bits << sh;
        if (sh && static_cast<u32>(k) == wi + 1)
            s.w[k] |= bits >> (64 - sh);
    }
}

template<int OW>
__device__ __forceinline__ void set_obj(ObjSet<OW>& s, u32 o)
{
#pragma unroll
    for (int k = 0; k < OW; ++k)
        if (static_cast<u32>(k) == (o >> 6))
            s.w[k] |= u64{1} << (o & 63);
}

/// The objects of a fluent relation run: object of rank r is in the set iff bit start + r * step is set.
template<int OW, class St>
__device__ __forceinline__ ObjSet<OW> run_objects(const DevTask& T, const St& st, const DFilter& f, u64 start)
{
    ObjSet<OW> out;
#pragma unroll
    for (int k = 0; k < OW; ++k)
        out.w[k] = 0;
    if (start >= T.fluent_count)
        return out;  // the bound object lies outside the position's domain: the relation holds for nothing
    const u32* dom = T.domain + T.pos_dom_begin[f.map_pos];
    if (f.step == 1)
    {
        for (u32 r0 = 0; r0 < f.count; r0 += 64)
        {
            const u32 len = f.count - r0 < 64 ? f.count - r0 : 64;
            u64 bits = extract64(st, start + r0);
            if (len < 64)
                bits &= (u64{1} << len) - 1;
            if (f.map_lo != kNone)
                or_shifted(out, bits, f.map_lo + r0);
            else
                while (bits)
                {
                    const u32 r = __ffsll(static_cast<long long>(bits)) - 1;
                    bits &= bits - 1;
                    set_obj(out, dom[r0 + r]);
                }
        }
    }
    else
    {
        for (u32 r = 0; r < f.count; ++r)
            if (test_bit(st, start + static_cast<u64>(r) * f.step))
                set_obj(out, f.map_lo != kNone ? f.map_lo + r : dom[r]);
    }
    return out;
}

/// key of a pattern under the binding.
__device__ __forceinline__ u64 pattern_key(const DevTask& T, const DLit& l, const u32* bind)
{
    u64 k = l.base;
    for (u32 i = 0; i < l.nvars; ++i)
    {
        const DVar v = T.vars[l.var_begin + i];
        k += T.pool[v.rs + bind[v.param]];
    }
    return k;
}

template<class St>
__device__ __forceinline__ bool literal_holds(const DevTask& T, const St& st, const DLit& l, const u32* bind)
{
    const u64 k = pattern_key(T, l, bind);
    bool t;
    if (l.fluent)
        t = k < T.fluent_count && test_bit(st, k);
    else
        t = static_member(T.pool + T.srel_table[l.pred], T.srel_mask[l.pred],
                          static_cast<u32>(T.srel_probes[l.pred]), k);
    return t != (l.neg != 0);
}

template<class St>
__device__ __forceinline__ bool goal_holds(const DevTask& T, const St& st)
{
    if (T.goal_unsat)
        return false;
    for (u32 i = 0; i < T.words; ++i)
    {
        const u64 s = st.word(i), p = T.goal_pos[i], q = T.goal_neg[i];
        if ((s & p) != p || (s & q) != 0)
            return false;
    }
    return true;
}

template<int OW, class St>
__device__ __forceinline__ bool level_candidates(const DevTask& T, const St& st, const DLevel& lv, const u32* bind,
                                                 ObjSet<OW>& c)
{
    u64 any = 0;
#pragma unroll
    for (int k = 0; k < OW; ++k)
        c.w[k] = T.pool[lv.dom0 + k];
    for (u32 fi = lv.filt_begin; fi < lv.filt_end; ++fi)
    {
        const DFilter f = T.filters[fi];
        ObjSet<OW> s;
        if (f.kind == kFiltRun)
        {
            const u64 start = f.base + (f.src != kNone ? T.pool[f.src_rs + bind[f.src]] : 0);
            s = run_objects<OW>(T, st, f, start);
        }
        else
        {
            const u64* row = T.pool + f.base + static_cast<u64>(bind[f.src]) * OW;
#pragma unroll
            for (int k = 0; k < OW; ++k)
                s.w[k] = row[k];
        }
#pragma unroll
        for (int k = 0; k < OW; ++k)
            c.w[k] &= f.neg ? ~s.w[k] : s.w[k];
    }
#pragma unroll
    for (int k = 0; k < OW; ++k)
        any |= c.w[k];
    return any != 0;
}

constexpr int kMaxLevels = 8;

/// Calls emit(bind) for every applicable binding of program `pg` in state `st`, in the program's binding order. emit
/// returns false to stop; the function then returns false.
template<int OW, class St, class Emit>
__device__ bool enumerate_raw(const DevTask& T, const DProgram& pg, const St& st, u32* bind, Emit&& emit)
{
    if (pg.never)
        return true;
    for (u32 c = pg.pre_begin; c < pg.pre_end; ++c)
        if (!literal_holds(T, st, T.lits[T.checks[c]], bind))
            return true;
    if (pg.nlevels == 0)
        return emit(bind);
    ObjSet<OW> cand[kMaxLevels];
    const DLevel* lv = T.levels + pg.level_begin;
    if (!level_candidates<OW>(T, st, lv[0], bind, cand[0]))
        return true;
    int d = 0;
    while (d >= 0)
    {
        // next candidate at level d
        int k = 0;
#pragma unroll
        for (int q = OW - 1; q >= 0; --q)
            if (cand[d].w[q])
                k = q;
        u64 word = cand[d].w[k];
        if (!word)
        {
            --d;
            continue;
        }
        const u32 o = static_cast<u32>(k) * 64 + (__ffsll(static_cast<long long>(word)) - 1);
#pragma unroll
        for (int q = 0; q < OW; ++q)
            if (q == k)
                cand[d].w[q] = word & (word - 1);
        const DLevel L = lv[d];
        bind[L.param] = o;
        bool ok = true;
        for (u32 c = L.chk_begin; c < L.chk_end && ok; ++c)
            ok = literal_holds(T, st, T.lits[T.checks[c]], bind);
        if (!ok)
            continue;
        if (static_cast<u32>(d) + 1 == pg.nlevels)
        {
            if (!emit(bind))
                return false;
            if (pg.first_exist < pg.nlevels)
            {
                // witness found: back to the last effect-relevant level
                d = static_cast<int>(pg.first_exist) - 1;
            }
            continue;
        }
        if (level_candidates<OW>(T, st, lv[d + 1], bind, cand[d + 1]))
            ++d;
    }
    return true;
}

/// enumerate_raw() in canonical order: a program whose bindings do not come out in it (pg.sorted) has them buffered
/// and sorted (emit_sorted).
template<int OW, class St, class Emit>
__device__ bool enumerate(const DevTask& T, const DProgram& pg, const St& st, u32* bind, Emit&& emit)
{
    if (!pg.sorted)
        return enumerate_raw<OW>(T, pg, st, bind, emit);
    return dev::emit_sorted(
        pg.nparams, [&](auto&& f) { return enumerate_raw<OW>(T, pg, st, bind, f); },
        [&](const u32* b) {
            for (u32 v = 0; v < pg.nparams; ++v)
                bind[v] = b[v];
            return emit(static_cast<const u32*>(bind));
        });
}

/// The slots an action deletes and adds (dense: slot = canonical id). Deletes outside the layout are dropped.
struct Effects
{
    u32 n_del, n_add;
    u32 del[16];
    u32 add[16];
};

__device__ __forceinline__ void collect_effects(const DevTask& T, const DSchema& S, const u32* bind, Effects& e)
{
    e.n_del = 0;
    e.n_add = 0;
    for (u32 i = S.del_begin; i < S.del_end && e.n_del < 16; ++i)
    {
        const u64 k = pattern_key(T, T.lits[i], bind);
        if (k < T.fluent_count)
            e.del[e.n_del++] = static_cast<u32>(k);
    }
    for (u32 i = S.add_begin; i < S.add_end && e.n_add < 16; ++i)
        e.add[e.n_add++] = static_cast<u32>(pattern_key(T, T.lits[i], bind));
}

/// Word i of the successor (delete, then add).
template<class St>
__device__ __forceinline__ u64 succ_word(const St& st, const Effects& e, u32 i)
{
    u64 w = st.word(i);
    for (u32 j = 0; j < e.n_del; ++j)
        if ((e.del[j] >> 6) == i)
            w &= ~(u64{1} << (e.del[j] & 63));
    for (u32 j = 0; j < e.n_add; ++j)
        if ((e.add[j] >> 6) == i)
            w |= u64{1} << (e.add[j] & 63);
    return w;
}

}  // namespace b2
