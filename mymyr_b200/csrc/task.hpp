// Host-side task model of the device path: the normalized lifted STRIPS task (TaskSpec), its typed-dense canonical
// atom layout (Layout), and the flat device program the kernels read (DevTask and the pools it points into).
//
// The layout restates the reference's canonical-id rule so that slots, rows and hashes are bit-identical to
// maichmueller/mymyr's Task under TaskOptions::Atoms::Dense:
//   cid(p, a_0..a_k-1) = offset[p] + sum_i rank_i(a_i) * stride_i     (include/mymyr/task/atom_index.hpp:9-16)
// with position domains from the add effects' static parameter domains plus the initial atoms
// (src/mymyr/task/compile.cpp:1103-1180). The matcher program is this library's own design: parameters are bound in
// index order (the canonical binding order), so bindings come out in canonical order with no per-segment sort.

#pragma once

#include <cstdint>
#include <string>
#include <algorithm>
#include <vector>

namespace b2
{
using u8 = std::uint8_t;
using u32 = std::uint32_t;
using u64 = std::uint64_t;
using i32 = std::int32_t;
using i64 = std::int64_t;

enum : u8
{
    kStatic = 0,
    kFluent = 1,
    kDerived = 2,
};

struct Lit
{
    u32 pred = 0;
    bool pos = true;
    std::vector<i32> terms;  // >= 0 parameter, < 0 object -(o+1)
};

struct Schema
{
    std::string name;
    u32 arity = 0;
    std::vector<Lit> pre;
    std::vector<Lit> eff;
};

struct TaskSpec
{
    u32 n = 0;  // objects
    std::vector<u8> kind;
    std::vector<u32> arity;
    std::vector<std::string> pred_names;
    std::vector<std::vector<u32>> static_init;  // [pred, args...]
    std::vector<std::vector<u32>> fluent_init;
    std::vector<Lit> goal;  // ground
    std::vector<Schema> schemas;
    std::string unsupported;  // non-empty: a feature the device path does not run
};

/// Contribution of an object outside a position's domain (as in the reference: any sum containing it is >= total).
constexpr u64 kOutside = u64{1} << 40;
/// The same for static relations.
constexpr u64 kStaticOutside = u64{1} << 56;
constexpr u32 kNone = 0xFFFFFFFFu;

struct Layout
{
    u64 fluent_count = 0;
    std::vector<u64> offset;      // per predicate (~0 for static)
    std::vector<u64> size;        // per predicate
    std::vector<u32> pos_begin;   // per predicate: first position
    std::vector<u64> stride;      // per position
    std::vector<u32> dsize;       // per position
    std::vector<u32> dom_begin;   // per position, into domain
    std::vector<u32> domain;      // objects of each position, ascending
    std::vector<u64> rs;          // per position: n entries, rank * stride or kOutside
};

/// A static predicate's ground atoms as packed keys: argument i of an atom is its object in bits 8i..8i+7 (objects
/// are below 256, arities below 8), so a literal's key is its constants' part plus one shifted object per bound
/// parameter, the same additive form as a fluent literal's slot. `keys` holds them sorted (host lookups);
/// `table` is the open-addressed set the kernels probe (2^k slots, kEmptyStaticSlot empty, linear probing from
/// static_key_home), and no stored key sits more than `probes` - 1 slots past its home.
struct StaticRel
{
    u32 arity = 0;
    std::vector<u64> keys;
    std::vector<u64> table;
    u32 probes = 0;
    bool holds(u64 key) const { return std::binary_search(keys.begin(), keys.end(), key); }
};

/// The contribution of object o at argument position i to a static atom's packed key.
inline u64 static_arg_key(u32 i, u32 o) { return static_cast<u64>(o) << (8 * i); }

/// The empty slot of a static key set (a packed key of an arity below 8 never has its top byte set).
constexpr u64 kEmptyStaticSlot = ~u64{0};

/// Home slot of a packed static key in a key set of mask + 1 slots: the splitmix64 finalizer of the key xor a fixed
/// constant. The kernels' static_key_slot (core.cuh) computes the same.
inline u64 static_key_home(u64 key, u64 mask)
{
    u64 x = key ^ 0x6a09e667f3bcc909ULL;
    x ^= x >> 30;
    x *= 0xbf58476d1ce4e5b9ULL;
    x ^= x >> 27;
    x *= 0x94d049bb133111ebULL;
    x ^= x >> 31;
    return x & mask;
}

// ------------------------------------------------------------------------------------------------ device program

enum : u32
{
    kFiltRun = 0,   // fluent relation run: bits start + r * step, r < count, object of rank r in map_pos's domain
    kFiltSRow = 1,  // static binary row table: row(bind[src]) of OW words at u64 pool offset `base`
};

struct DFilter
{
    u32 kind = kFiltRun;
    u32 neg = 0;
    u32 src = kNone;     // parameter whose value selects the run / row (kNone: fixed start)
    u32 map_pos = 0;     // position whose domain maps ranks to objects (run)
    u64 base = 0;        // run: fixed part of the start bit; srow: word offset of the row table
    u64 src_rs = 0;      // run: u64 pool offset of the source position's rs table (start += rs[bind[src]])
    u64 step = 1;        // run: bit distance between consecutive ranks
    u32 count = 0;       // run: ranks
    u32 map_lo = kNone;  // run: the domain is the contiguous object range [map_lo, map_lo + count) (kNone: not)
};

struct DLit  // a literal check or an effect pattern: key = base + sum_v rs[bind[param_v]]
{
    u32 fluent = 1;
    u32 neg = 0;
    u32 pred = 0;
    u32 nvars = 0;
    u64 base = 0;
    u32 var_begin = 0;  // into vars
    u32 pad = 0;
};

struct DVar
{
    u32 param = 0;
    u32 pad = 0;
    u64 rs = 0;  // u64 pool offset of the rs table (n entries)
};

struct DLevel
{
    u32 param = 0;
    u32 filt_begin = 0, filt_end = 0;  // into filters
    u32 chk_begin = 0, chk_end = 0;    // into checks (indices into lits)
    u32 pad = 0;
    u64 dom0 = 0;                      // u64 pool offset of the static domain (OW words)
};

struct DProgram
{
    u32 nlevels = 0;
    u32 first_exist = 0;      // levels >= first_exist bind witness-only parameters (witness pruning)
    u32 level_begin = 0;      // into levels
    u32 pre_begin = 0, pre_end = 0;  // ground fluent checks (into checks)
    u32 never = 0;            // statically inapplicable
    u32 sorted = 0;           // the bindings do not come out in canonical order (witness pruning with a witness-only
                              // parameter before an effect parameter): they are buffered and emitted sorted
    u32 nparams = 0;          // the schema's parameters (the sorted bindings' keys)
};

struct DSchema
{
    u32 arity = 0;
    u32 add_begin = 0, add_end = 0;  // into lits
    u32 del_begin = 0, del_end = 0;
    u32 fast_on = 0;   // the compiled matcher binds in `fast`'s order and sorts (see below)
    DProgram prog[2];  // [0] witness pruning on, [1] off
    /// Every parameter in a selectivity order (most constrained first, from static estimates), for the compiled
    /// matcher: its bindings are buffered and sorted into canonical order before they are emitted. Used when the
    /// estimated search is at most half of index order's, and for witness pruning only when the schema has no
    /// witness-only parameter. The interpreted matcher always binds in index order.
    DProgram fast;
};

/// Everything the kernels read, as host vectors (uploaded into one device blob) plus scalar facts.
struct Program
{
    u32 n = 0, ow = 1, words = 1, nschemas = 0, label_width = 0;
    u64 fluent_count = 0;
    u32 goal_unsat = 0;
    std::vector<u64> pool;        // dom0 bitsets, static row tables, static relation bits, rs tables
    std::vector<DLit> lits;
    std::vector<DVar> vars;
    std::vector<DFilter> filters;
    std::vector<DLevel> levels;
    std::vector<u32> checks;
    std::vector<DSchema> schemas;
    std::vector<u32> domain;      // the layout's domains (rank -> object)
    std::vector<u32> pos_dom_begin;
    std::vector<u64> srel_table;  // per predicate: u64 pool offset of its static key set (StaticRel::table)
    std::vector<u64> srel_mask;   // per predicate: slots of the key set - 1
    std::vector<u64> srel_probes; // per predicate: probes that find any stored key (StaticRel::probes)
    std::vector<u64> goal_pos, goal_neg;  // [words] goal masks
    std::vector<u64> initial;     // [words]
    std::vector<std::vector<u32>> slot_atoms;  // per slot: [pred, args...]
};

/// Parses the reference's task text format. Throws std::runtime_error on malformed input.
TaskSpec read_task_text(const std::string& text);
/// Compiles the task (throws std::invalid_argument for unsupported features).
void compile_task(const TaskSpec& spec, Layout& layout, std::vector<StaticRel>& statics, Program& prog);

/// Words per object bitset over n objects.
inline u32 object_words(u32 n) { return n <= 64 ? 1u : (n + 63) / 64; }
inline u32 words_for(u64 bits) { return static_cast<u32>((bits + 63) >> 6); }
}  // namespace b2
