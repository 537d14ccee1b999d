// Task text reader and task compiler of the device path (host code).
//
// read_task_text: the reference's normalized text format (src/mymyr/formalism/text_format.cpp:16-190 reads it;
// this is an independent reader of the same format). Sections O P SI FI G A, optional trailing X / C / EG.
//
// compile_task:
//   1. static relations and unary static bitsets (ranks in object order; compile.cpp:102-190 of the reference);
//   2. per schema parameter its static domain dom0: all objects restricted by static unary literals, static binary
//      literals with a constant, and projections of static positive k-ary literals (compile.cpp:808-906);
//   3. the typed-dense canonical layout: position domains = dom0 of the add effects' parameters, the effects'
//      constants and the initial atoms; fluent predicates in id order; strides from the last position
//      (compile.cpp:1103-1180);
//   4. the device matcher program of each schema (this library's design): parameters bound in index order, each
//      level's candidates = dom0 & per-state runs of fluent relations & static rows, literals of arity >= 3 checked
//      at the level of their last parameter. Under witness pruning the witness-only parameters are bound last, in the
//      order the reference's fixed-order matcher gives them (compile.cpp:908-937), so that the first witness found
//      is the reference's.

#include "task.hpp"

#include <algorithm>
#include <array>
#include <bit>
#include <map>
#include <set>
#include <sstream>
#include <stdexcept>
#include <tuple>

namespace b2
{
namespace
{
[[noreturn]] void parse_fail(const std::string& m) { throw std::runtime_error("task text: " + m); }

class Reader
{
public:
    explicit Reader(const std::string& text) : in(text) {}

    TaskSpec read()
    {
        TaskSpec t;
        expect("O");
        t.n = u();
        expect("P");
        const u32 np = u();
        for (u32 i = 0; i < np; ++i)
        {
            const std::string k = word();
            u8 kind = kStatic;
            if (k == "S")
                kind = kStatic;
            else if (k == "F")
                kind = kFluent;
            else if (k == "D" || k == "C" || k == "P")
                kind = kDerived;
            else
                parse_fail("bad predicate kind " + k);
            t.kind.push_back(kind);
            t.arity.push_back(u());
            t.pred_names.push_back(word());
            if (kind == kDerived)
                note(t, "derived predicates");
        }
        std::string tag = word();
        if (tag == "N")
            parse_fail("numeric tasks are not supported by this reader");
        if (tag != "SI")
            parse_fail("expected SI, got " + tag);
        atoms(t, t.static_init);
        expect("FI");
        atoms(t, t.fluent_init);
        expect("G");
        const u32 ng = u();
        for (u32 i = 0; i < ng; ++i)
        {
            Lit l;
            l.pred = pred(t);
            l.pos = u() != 0;
            for (u32 j = 0; j < t.arity[l.pred]; ++j)
                l.terms.push_back(-static_cast<i32>(object(t)) - 1);
            t.goal.push_back(std::move(l));
        }
        expect("A");
        const u32 ns = u();
        for (u32 s = 0; s < ns; ++s)
        {
            Schema sc;
            sc.name = word();
            sc.arity = u();
            sc.pre = literals(t, "L", sc.arity);
            expect("E");
            const u32 ne = u();
            for (u32 e = 0; e < ne; ++e)
            {
                const u32 extra = u();
                std::vector<Lit> cond = literals(t, "L", sc.arity + extra);
                std::vector<Lit> effs = literals(t, "F", sc.arity + extra);
                if (extra || !cond.empty())
                {
                    note(t, "conditional effects");
                    continue;
                }
                for (Lit& l : effs)
                    sc.eff.push_back(std::move(l));
            }
            t.schemas.push_back(std::move(sc));
        }
        // optional trailing sections
        while (in >> tag)
        {
            if (tag == "X")
            {
                const u32 nx = u();
                if (nx)
                    note(t, "axioms");
                for (u32 i = 0; i < nx; ++i)
                {
                    const u32 p = pred(t);
                    const u32 arity = u();
                    expect("H");
                    for (u32 j = 0; j < t.arity[p]; ++j)
                        i32v();
                    literals(t, "L", arity);
                }
            }
            else if (tag == "C")
            {
                const u32 k = u();
                if (k)
                    note(t, "collapsed parameters");
                for (u32 i = 0; i < k; ++i)
                {
                    u();
                    u();
                    u();
                    i32v();
                }
            }
            else if (tag == "EG")
            {
                u();
                const u32 k = u();
                for (u32 i = 0; i < k; ++i)
                {
                    const u32 p = pred(t);
                    u();
                    for (u32 j = 0; j < t.arity[p]; ++j)
                        object(t);
                }
            }
            else
                parse_fail("unexpected section " + tag);
        }
        return t;
    }

private:
    static void note(TaskSpec& t, const char* what)
    {
        if (t.unsupported.empty())
            t.unsupported = what;
    }
    std::string word()
    {
        std::string w;
        if (!(in >> w))
            parse_fail("unexpected end of input");
        return w;
    }
    void expect(const char* s)
    {
        const std::string w = word();
        if (w != s)
            parse_fail(std::string("expected ") + s + ", got '" + w + "'");
    }
    u32 u()
    {
        const std::string w = word();
        if (w.empty() || w.size() > 10 || w.find_first_not_of("0123456789") != std::string::npos)
            parse_fail("expected unsigned integer, got '" + w + "'");
        const unsigned long long v = std::stoull(w);
        if (v > 0xFFFFFFFFull)
            parse_fail("integer out of range '" + w + "'");
        return static_cast<u32>(v);
    }
    i32 i32v()
    {
        const std::string w = word();
        std::size_t used = 0;
        long long v = 0;
        try
        {
            v = std::stoll(w, &used);
        }
        catch (...)
        {
            parse_fail("expected integer, got '" + w + "'");
        }
        if (used != w.size() || v < INT32_MIN || v > INT32_MAX)
            parse_fail("expected integer, got '" + w + "'");
        return static_cast<i32>(v);
    }
    u32 pred(const TaskSpec& t)
    {
        const u32 p = u();
        if (p >= t.kind.size())
            parse_fail("predicate id out of range");
        return p;
    }
    u32 object(const TaskSpec& t)
    {
        const u32 o = u();
        if (o >= t.n)
            parse_fail("object id out of range");
        return o;
    }
    void atoms(const TaskSpec& t, std::vector<std::vector<u32>>& out)
    {
        const u32 k = u();
        for (u32 i = 0; i < k; ++i)
        {
            std::vector<u32> rec{pred(t)};
            for (u32 j = 0; j < t.arity[rec[0]]; ++j)
                rec.push_back(object(t));
            out.push_back(std::move(rec));
        }
    }
    std::vector<Lit> literals(const TaskSpec& t, const char* tag, u32 params)
    {
        expect(tag);
        const u32 k = u();
        std::vector<Lit> ls;
        for (u32 i = 0; i < k; ++i)
        {
            Lit l;
            l.pred = pred(t);
            l.pos = u() != 0;
            for (u32 j = 0; j < t.arity[l.pred]; ++j)
            {
                const i32 x = i32v();
                if (x >= 0 && static_cast<u32>(x) >= params)
                    parse_fail("parameter index out of range");
                if (x < 0 && static_cast<u32>(-(static_cast<long long>(x) + 1)) >= t.n)
                    parse_fail("object term out of range");
                l.terms.push_back(x);
            }
            ls.push_back(std::move(l));
        }
        return ls;
    }

    std::istringstream in;
};

inline u32 obj_of(i32 term) { return static_cast<u32>(-(static_cast<long long>(term) + 1)); }

/// a * b, or kSizeCap once the product passes it (key spaces that large are refused where they arise).
constexpr u64 kSizeCap = u64{1} << 62;
u64 capped_product(u64 a, u64 b)
{
    u64 r = 0;
    return __builtin_mul_overflow(a, b, &r) || r > kSizeCap ? kSizeCap : r;
}

/// The parameters a literal mentions, in the order of their first occurrence (schemas have at most 8).
std::vector<u32> params_of(const std::vector<i32>& terms)
{
    std::vector<u32> out;
    u32 seen = 0;
    for (i32 x : terms)
        if (x >= 0 && !((seen >> x) & 1u))
        {
            seen |= 1u << x;
            out.push_back(static_cast<u32>(x));
        }
    return out;
}

struct Compiler
{
    const TaskSpec& T;
    Layout& L;
    std::vector<StaticRel>& S;
    Program& P;
    u32 n = 0, OW = 1;
    std::vector<std::vector<const std::vector<u32>*>> sfacts;  // per static predicate: its atoms (task order)
    std::vector<std::vector<u64>> sunary;                      // per static unary predicate: its object set
    std::vector<std::array<u64, 2>> sadj;                      // per static binary predicate: adjacency tables
    std::vector<std::vector<std::vector<u64>>> dom0;           // per schema, per parameter: OW words
    std::vector<u64> layout_rs_off;                            // per position: pool offset of rs
    std::vector<u64> static_rs_off;                            // per static predicate: pool offset of its
                                                               // per-argument key contributions (arity x n)

    Compiler(const TaskSpec& t, Layout& l, std::vector<StaticRel>& s, Program& p) : T(t), L(l), S(s), P(p) {}

    static void set_bit(u64* w, u64 b) { w[b >> 6] |= u64{1} << (b & 63); }
    static bool test_bit(const u64* w, u64 b) { return (w[b >> 6] >> (b & 63)) & 1; }

    void run()
    {
        if (!T.unsupported.empty())
            throw std::invalid_argument("mymyr_b200: the device path does not support " + T.unsupported);
        n = T.n;
        if (n == 0)
            throw std::invalid_argument("mymyr_b200: a task without objects");
        OW = object_words(n);
        if (OW > 4)
            throw std::invalid_argument("mymyr_b200: more than 256 objects are not supported by the device kernels");
        for (const Schema& s : T.schemas)
            if (s.arity > 8)
                throw std::invalid_argument("mymyr_b200: schema " + s.name + " has more than 8 parameters");
        index_statics();
        domains();
        layout();
        program();
    }

    // ---------------------------------------------------------------------------------------------- statics
    /// Indexes every static predicate's atoms (StaticRel): packed keys, sorted, and the open-addressed key set the
    /// kernels probe (at most half full); unary predicates also as object sets.
    void index_statics()
    {
        const u32 m = static_cast<u32>(T.kind.size());
        sfacts.assign(m, {});
        sunary.assign(m, {});
        sadj.assign(m, {kNoTable, kNoTable});
        S.assign(m, {});
        for (const auto& a : T.static_init)
        {
            if (T.kind[a[0]] != kStatic)
                throw std::invalid_argument("mymyr_b200: a static initial atom over a non-static predicate");
            sfacts[a[0]].push_back(&a);
        }
        for (u32 p = 0; p < m; ++p)
        {
            if (T.kind[p] != kStatic)
                continue;
            StaticRel& R = S[p];
            R.arity = T.arity[p];
            if (R.arity >= 8)
                throw std::invalid_argument("mymyr_b200: static predicate " + T.pred_names[p] +
                                            " has 8 or more arguments");
            R.keys.reserve(sfacts[p].size());
            for (const auto* a : sfacts[p])
                R.keys.push_back(fact_key(*a));
            std::sort(R.keys.begin(), R.keys.end());
            R.keys.erase(std::unique(R.keys.begin(), R.keys.end()), R.keys.end());
            u64 slots = 8;
            while (slots < 2 * R.keys.size())
                slots <<= 1;
            R.table.assign(slots, kEmptyStaticSlot);
            R.probes = 1;
            for (const u64 k : R.keys)
            {
                u64 j = static_key_home(k, slots - 1);
                u32 run = 1;
                for (; R.table[j] != kEmptyStaticSlot; j = (j + 1) & (slots - 1))
                    ++run;
                R.table[j] = k;
                R.probes = std::max(R.probes, run);
            }
            if (R.arity == 1)
            {
                sunary[p].assign(OW, 0);
                for (const auto* a : sfacts[p])
                    set_bit(sunary[p].data(), (*a)[1]);
            }
        }
    }

    static constexpr u64 kNoTable = ~u64{0};

    /// The packed key of a static atom record [pred, args...].
    static u64 fact_key(const std::vector<u32>& a)
    {
        u64 k = 0;
        for (u32 i = 1; i < a.size(); ++i)
            k += static_arg_key(i - 1, a[i]);
        return k;
    }

    /// Whether a ground static literal's atom is a static fact.
    bool static_fact(const Lit& l) const
    {
        u64 k = 0;
        for (u32 i = 0; i < l.terms.size(); ++i)
            k += static_arg_key(i, obj_of(l.terms[i]));
        return S[l.pred].holds(k);
    }

    /// The adjacency table of static binary predicate `pred` selected by argument `by` (0 or 1): n object sets of OW
    /// words in the pool, set o holding the objects o is related to at the other argument. Built on first use.
    u64 adjacency(u32 pred, u32 by)
    {
        u64& off = sadj[pred][by];
        if (off != kNoTable)
            return off;
        off = P.pool.size();
        P.pool.resize(off + static_cast<std::size_t>(n) * OW, 0);
        for (const auto* a : sfacts[pred])
        {
            const u32 sel = (*a)[1 + by], other = (*a)[2 - by];
            set_bit(P.pool.data() + off + static_cast<std::size_t>(sel) * OW, other);
        }
        return off;
    }

    // ---------------------------------------------------------------------------------------------- dom0
    void domains()
    {
        dom0.assign(T.schemas.size(), {});
        for (std::size_t s = 0; s < T.schemas.size(); ++s)
        {
            const Schema& sc = T.schemas[s];
            auto& D = dom0[s];
            D.assign(sc.arity, std::vector<u64>(OW, 0));
            for (auto& d : D)
                for (u32 o = 0; o < n; ++o)
                    set_bit(d.data(), o);
            auto and_words = [&](u32 v, const u64* w, bool neg) {
                for (u32 i = 0; i < OW; ++i)
                    D[v][i] &= neg ? ~w[i] : w[i];
            };
            for (const Lit& l : sc.pre)
            {
                const bool fluent = T.kind[l.pred] != kStatic;
                const auto vars = params_of(l.terms);
                if (vars.empty() || fluent)
                    continue;
                const u32 ar = T.arity[l.pred];
                if (ar == 1)
                {
                    and_words(vars[0], sunary[l.pred].data(), !l.pos);
                    continue;
                }
                if (ar == 2 && l.terms[0] != l.terms[1])
                {
                    const bool f0 = l.terms[0] >= 0, f1 = l.terms[1] >= 0;
                    if (f0 && f1)
                        continue;
                    const u32 fpos = f0 ? 0 : 1, opos = 1 - fpos;
                    const u32 v = static_cast<u32>(l.terms[fpos]);
                    const u64 off = adjacency(l.pred, opos);
                    and_words(v, P.pool.data() + off + static_cast<std::size_t>(obj_of(l.terms[opos])) * OW, !l.pos);
                    continue;
                }
                if (l.pos && ar >= 3)
                    for (u32 i = 0; i < ar; ++i)
                        if (l.terms[i] >= 0)
                        {
                            std::vector<u64> proj(OW, 0);
                            for (const auto* a : sfacts[l.pred])
                            {
                                bool ok = true;
                                for (u32 j = 0; j < ar && ok; ++j)
                                    if (l.terms[j] < 0 && (*a)[1 + j] != obj_of(l.terms[j]))
                                        ok = false;
                                if (ok)
                                    set_bit(proj.data(), (*a)[1 + i]);
                            }
                            and_words(static_cast<u32>(l.terms[i]), proj.data(), false);
                        }
            }
        }
    }

    // ---------------------------------------------------------------------------------------------- layout
    void layout()
    {
        const u32 m = static_cast<u32>(T.kind.size());
        std::vector<std::vector<std::vector<u64>>> bits(m);
        for (u32 p = 0; p < m; ++p)
            if (T.kind[p] == kFluent)
                bits[p].assign(T.arity[p], std::vector<u64>(OW, 0));
        for (std::size_t s = 0; s < T.schemas.size(); ++s)
            for (const Lit& l : T.schemas[s].eff)
            {
                if (!l.pos)
                    continue;
                if (T.kind[l.pred] != kFluent)
                    throw std::invalid_argument("mymyr_b200: an effect on a non-fluent predicate");
                for (u32 i = 0; i < l.terms.size(); ++i)
                {
                    const i32 t = l.terms[i];
                    if (t < 0)
                        set_bit(bits[l.pred][i].data(), obj_of(t));
                    else
                        for (u32 w = 0; w < OW; ++w)
                            bits[l.pred][i][w] |= dom0[s][t][w];
                }
            }
        for (const auto& a : T.fluent_init)
        {
            if (T.kind[a[0]] != kFluent)
                throw std::invalid_argument("mymyr_b200: a fluent initial atom over a non-fluent predicate");
            for (u32 i = 0; i < T.arity[a[0]]; ++i)
                set_bit(bits[a[0]][i].data(), a[1 + i]);
        }
        L.offset.assign(m, ~u64{0});
        L.size.assign(m, 0);
        L.pos_begin.assign(m, 0);
        u32 positions = 0;
        for (u32 p = 0; p < m; ++p)
            if (T.kind[p] == kFluent)
            {
                L.pos_begin[p] = positions;
                positions += T.arity[p];
            }
        L.rs.assign(static_cast<std::size_t>(positions) * n, kOutside);
        L.stride.assign(positions, 0);
        L.dsize.assign(positions, 0);
        L.dom_begin.assign(positions, 0);
        u64 running = 0;
        for (u32 p = 0; p < m; ++p)
        {
            if (T.kind[p] != kFluent)
                continue;
            const u32 ar = T.arity[p];
            u64 size = 1;
            for (u32 i = 0; i < ar; ++i)
            {
                const u32 pos = L.pos_begin[p] + i;
                L.dom_begin[pos] = static_cast<u32>(L.domain.size());
                for (u32 o = 0; o < n; ++o)
                    if (test_bit(bits[p][i].data(), o))
                        L.domain.push_back(o);
                L.dsize[pos] = static_cast<u32>(L.domain.size() - L.dom_begin[pos]);
                size = capped_product(size, L.dsize[pos]);
            }
            u64 st = 1;
            for (u32 i = ar; i-- > 0;)
            {
                const u32 pos = L.pos_begin[p] + i;
                L.stride[pos] = st;
                for (u32 r = 0; r < L.dsize[pos]; ++r)
                    L.rs[static_cast<std::size_t>(pos) * n + L.domain[L.dom_begin[pos] + r]] = r * st;
                st = capped_product(st, std::max<u32>(1, L.dsize[pos]));
            }
            L.size[p] = size;
            L.offset[p] = running;
            running = std::min<u64>(running + size, u64{1} << 62);
        }
        L.fluent_count = running;
        if (L.fluent_count > (u64{1} << 24))
            throw std::invalid_argument("mymyr_b200: more than 2^24 fluent atoms (rows of more than 262144 words)");
    }

    u64 cid(u32 p, const u32* args) const
    {
        u64 c = L.offset[p];
        for (u32 i = 0; i < T.arity[p]; ++i)
            c += L.rs[static_cast<std::size_t>(L.pos_begin[p] + i) * n + args[i]];
        return c;
    }

    // ---------------------------------------------------------------------------------------------- program
    /// A literal as key pattern (check or effect).
    u32 pattern(const Lit& l)
    {
        DLit d;
        d.fluent = T.kind[l.pred] == kFluent ? 1 : 0;
        d.neg = l.pos ? 0 : 1;
        d.pred = l.pred;
        d.var_begin = static_cast<u32>(P.vars.size());
        if (d.fluent)
        {
            d.base = L.offset[l.pred];
            for (u32 i = 0; i < l.terms.size(); ++i)
            {
                const u32 pos = L.pos_begin[l.pred] + i;
                if (l.terms[i] < 0)
                    d.base += L.rs[static_cast<std::size_t>(pos) * n + obj_of(l.terms[i])];
                else
                    P.vars.push_back({static_cast<u32>(l.terms[i]), 0, layout_rs_off[pos]});
            }
        }
        else
        {
            for (u32 i = 0; i < l.terms.size(); ++i)
            {
                if (l.terms[i] < 0)
                    d.base += static_arg_key(i, obj_of(l.terms[i]));
                else
                    P.vars.push_back({static_cast<u32>(l.terms[i]), 0, static_rs_off[l.pred] + static_cast<u64>(i) * n});
            }
        }
        d.nvars = static_cast<u32>(P.vars.size()) - d.var_begin;
        P.lits.push_back(d);
        return static_cast<u32>(P.lits.size() - 1);
    }

    /// The reference's order of the witness-only parameters of a fixed-order matcher (compile.cpp:908-937): with
    /// every effect-relevant parameter placed, repeatedly take the one with most binary links to placed parameters,
    /// then most per-state unary constraints, then fewest static candidates; ties to the lowest index.
    std::vector<u32> witness_order(std::size_t s, const std::vector<u8>& relevant)
    {
        const Schema& sc = T.schemas[s];
        struct Bin
        {
            u32 a, b;
        };
        std::vector<Bin> bins;
        std::vector<u32> unary(sc.arity, 0);
        for (const Lit& l : sc.pre)
        {
            const bool fluent = T.kind[l.pred] != kStatic;
            const auto vars = params_of(l.terms);
            if (vars.empty())
                continue;
            const u32 ar = T.arity[l.pred];
            if (ar == 1)
            {
                if (fluent)
                    ++unary[vars[0]];
                continue;
            }
            if (ar == 2 && l.terms[0] != l.terms[1])
            {
                const bool f0 = l.terms[0] >= 0, f1 = l.terms[1] >= 0;
                if (f0 && f1)
                    bins.push_back({static_cast<u32>(l.terms[0]), static_cast<u32>(l.terms[1])});
                else if (fluent)
                    ++unary[static_cast<u32>(l.terms[f0 ? 0 : 1])];
                continue;
            }
            if (!fluent && l.pos && ar >= 3)
                for (u32 i = 0; i < ar; ++i)
                    for (u32 j = 0; j < ar; ++j)
                        if (i != j && l.terms[j] >= 0 && l.terms[i] >= 0 && l.terms[i] != l.terms[j] && i < j)
                            bins.push_back({static_cast<u32>(l.terms[i]), static_cast<u32>(l.terms[j])});
        }
        std::vector<bool> placed(sc.arity, false);
        for (u32 v = 0; v < sc.arity; ++v)
            placed[v] = relevant[v] != 0;
        std::vector<u32> order;
        for (;;)
        {
            long best = -1, best_score = 0;
            for (u32 v = 0; v < sc.arity; ++v)
            {
                if (placed[v])
                    continue;
                long links = 0;
                for (const Bin& b : bins)
                    if ((b.a == v && placed[b.b]) || (b.b == v && placed[b.a]))
                        ++links;
                long pc = 0;
                for (u32 w = 0; w < OW; ++w)
                    pc += std::popcount(dom0[s][v][w]);
                const long score = links * 1000000 + static_cast<long>(unary[v]) * 10000 - pc;
                if (best < 0 || score > best_score)
                    best = v, best_score = score;
            }
            if (best < 0)
                break;
            placed[best] = true;
            order.push_back(static_cast<u32>(best));
        }
        return order;
    }

    /// Estimated candidates of parameter v once the parameters in `placed` are bound: its static domain, narrowed by
    /// every positive precondition literal of arity 1 or 2 whose other parameters are placed: the literal's atoms
    /// (fluent: in the initial state; static: all) over the values of its bound positions.
    double candidates(std::size_t s, u32 v, const std::vector<bool>& placed, const std::vector<u64>& init_count,
                      const std::vector<std::vector<u32>>& static_pos_values) const
    {
        const Schema& sc = T.schemas[s];
        double e = 0;
        for (u32 w = 0; w < OW; ++w)
            e += std::popcount(dom0[s][v][w]);
        for (const Lit& l : sc.pre)
        {
            const u32 ar = T.arity[l.pred];
            if (!l.pos || ar == 0 || ar > 2 || T.kind[l.pred] == kDerived)
                continue;
            bool has_v = false, others_placed = true;
            for (i32 t : l.terms)
                if (t >= 0)
                {
                    if (static_cast<u32>(t) == v)
                        has_v = true;
                    else if (!placed[t])
                        others_placed = false;
                }
            if (!has_v || !others_placed)
                continue;
            const bool fluent = T.kind[l.pred] == kFluent;
            double atoms = fluent ? static_cast<double>(init_count[l.pred]) : static_cast<double>(sfacts[l.pred].size());
            double values = 1;
            for (u32 i = 0; i < ar; ++i)
                if (l.terms[i] < 0 || static_cast<u32>(l.terms[i]) != v)
                    values *= std::max<double>(1, fluent ? L.dsize[L.pos_begin[l.pred] + i]
                                                         : static_pos_values[l.pred][i]);
            e = std::min(e, std::max(atoms / values, 0.5));
        }
        return e;
    }

    /// A selectivity order for schema s (greedy: the parameter with the fewest estimated candidates next) and the
    /// estimated nodes of its search and of index order's.
    std::vector<u32> selective_order(std::size_t s, double& cost_sel, double& cost_idx) const
    {
        const Schema& sc = T.schemas[s];
        std::vector<u64> init_count(T.kind.size(), 0);
        for (const auto& a : T.fluent_init)
            ++init_count[a[0]];
        std::vector<std::vector<u32>> spv(T.kind.size());
        for (std::size_t p = 0; p < T.kind.size(); ++p)
        {
            if (T.kind[p] != kStatic)
                continue;
            spv[p].assign(T.arity[p], 0);
            for (u32 i = 0; i < T.arity[p]; ++i)
            {
                std::vector<u8> seen(n, 0);
                for (const auto* a : sfacts[p])
                    if (!seen[(*a)[1 + i]]++)
                        ++spv[p][i];
            }
        }
        auto cost = [&](const std::vector<u32>& order) {
            std::vector<bool> placed(sc.arity, false);
            double nodes = 1, total = 0;
            for (u32 v : order)
            {
                nodes *= candidates(s, v, placed, init_count, spv);
                total += nodes;
                placed[v] = true;
            }
            return total;
        };
        std::vector<u32> order, idx(sc.arity);
        std::vector<bool> placed(sc.arity, false);
        for (u32 d = 0; d < sc.arity; ++d)
        {
            idx[d] = d;
            u32 best = kNone;
            double best_e = 0;
            for (u32 v = 0; v < sc.arity; ++v)
            {
                if (placed[v])
                    continue;
                const double e = candidates(s, v, placed, init_count, spv);
                if (best == kNone || e < best_e)
                    best = v, best_e = e;
            }
            placed[best] = true;
            order.push_back(best);
        }
        cost_sel = cost(order);
        cost_idx = cost(idx);
        return order;
    }

    DProgram matcher(std::size_t s, const std::vector<u32>& order, u32 first_exist)
    {
        const Schema& sc = T.schemas[s];
        DProgram pg;
        pg.nlevels = static_cast<u32>(order.size());
        pg.first_exist = first_exist;
        pg.nparams = static_cast<u32>(T.schemas[s].arity);
        pg.level_begin = static_cast<u32>(P.levels.size());
        std::vector<i32> level_of(sc.arity, -1);
        for (u32 d = 0; d < order.size(); ++d)
            level_of[order[d]] = static_cast<i32>(d);
        std::vector<std::vector<DFilter>> filt(order.size());
        std::vector<std::vector<u32>> chk(order.size());
        std::vector<u32> pre;
        // a level's candidates: the parameter's static domain, less the objects that have no slot at some position of
        // a positive fluent precondition (such an atom is never true); the layout still follows the static domains
        std::vector<std::vector<u64>> cand = dom0[s];
        for (const Lit& l : sc.pre)
        {
            if (!l.pos || T.kind[l.pred] != kFluent)
                continue;
            const u32 P0 = L.pos_begin[l.pred];
            for (u32 i = 0; i < l.terms.size(); ++i)
            {
                if (l.terms[i] < 0)
                    continue;
                std::vector<u64>& c = cand[static_cast<u32>(l.terms[i])];
                for (u32 o = 0; o < n; ++o)
                    if (L.rs[static_cast<std::size_t>(P0 + i) * n + o] == kOutside)
                        c[o >> 6] &= ~(u64{1} << (o & 63));
            }
        }
        for (u32 v = 0; v < sc.arity; ++v)
        {
            bool any = false;
            for (u32 w = 0; w < OW; ++w)
                any |= cand[v][w] != 0;
            if (!any)
                pg.never = 1;
        }
        for (const Lit& l : sc.pre)
        {
            const bool fluent = T.kind[l.pred] == kFluent;
            const u32 ar = T.arity[l.pred];
            const auto vars = params_of(l.terms);
            if (vars.empty())
            {
                if (!fluent)
                {
                    if (static_fact(l) != l.pos)
                        pg.never = 1;
                }
                else
                    pre.push_back(pattern(l));
                continue;
            }
            if (ar == 1)
            {
                if (!fluent)
                    continue;  // folded into dom0
                const u32 pos = L.pos_begin[l.pred];
                DFilter f;
                f.kind = kFiltRun;
                f.neg = l.pos ? 0 : 1;
                f.base = L.offset[l.pred];
                f.step = 1;
                f.count = L.dsize[pos];
                f.map_pos = pos;
                filt[level_of[vars[0]]].push_back(f);
                continue;
            }
            if (ar == 2 && l.terms[0] != l.terms[1])
            {
                const bool f0 = l.terms[0] >= 0, f1 = l.terms[1] >= 0;
                if (f0 && f1)
                {
                    const u32 a = static_cast<u32>(l.terms[0]), b = static_cast<u32>(l.terms[1]);
                    const bool a_first = level_of[a] < level_of[b];
                    const u32 later = a_first ? b : a, earlier = a_first ? a : b;
                    const u32 lpos = a_first ? 1 : 0, epos = 1 - lpos;
                    DFilter f;
                    f.neg = l.pos ? 0 : 1;
                    f.src = earlier;
                    if (fluent)
                    {
                        f.kind = kFiltRun;
                        const u32 P0 = L.pos_begin[l.pred];
                        f.base = L.offset[l.pred];
                        f.src_rs = layout_rs_off[P0 + epos];
                        f.step = L.stride[P0 + lpos];
                        f.count = L.dsize[P0 + lpos];
                        f.map_pos = P0 + lpos;
                    }
                    else
                    {
                        f.kind = kFiltSRow;
                        f.base = adjacency(l.pred, epos);
                    }
                    filt[level_of[later]].push_back(f);
                    continue;
                }
                if (!fluent)
                    continue;  // static with a constant: folded into dom0
                const u32 fpos = f0 ? 0 : 1, opos = 1 - fpos;
                const u32 v = static_cast<u32>(l.terms[fpos]);
                const u32 P0 = L.pos_begin[l.pred];
                DFilter f;
                f.kind = kFiltRun;
                f.neg = l.pos ? 0 : 1;
                f.base = L.offset[l.pred] + L.rs[static_cast<std::size_t>(P0 + opos) * n + obj_of(l.terms[opos])];
                f.step = L.stride[P0 + fpos];
                f.count = L.dsize[P0 + fpos];
                f.map_pos = P0 + fpos;
                filt[level_of[v]].push_back(f);
                continue;
            }
            // arity >= 3 or a repeated parameter: checked at the level of the last parameter bound
            i32 last = -1;
            for (u32 v : vars)
                last = std::max(last, level_of[v]);
            chk[last].push_back(pattern(l));
        }
        for (u32 d = 0; d < order.size(); ++d)
        {
            DLevel lv;
            lv.param = order[d];
            lv.filt_begin = static_cast<u32>(P.filters.size());
            for (DFilter f : filt[d])
            {
                if (f.kind == kFiltRun)
                {
                    const u32 b = L.dom_begin[f.map_pos];
                    bool contiguous = f.count > 0;
                    for (u32 r = 1; r < f.count && contiguous; ++r)
                        contiguous = L.domain[b + r] == L.domain[b] + r;
                    f.map_lo = contiguous ? L.domain[b] : kNone;
                }
                P.filters.push_back(f);
            }
            lv.filt_end = static_cast<u32>(P.filters.size());
            lv.chk_begin = static_cast<u32>(P.checks.size());
            P.checks.insert(P.checks.end(), chk[d].begin(), chk[d].end());
            lv.chk_end = static_cast<u32>(P.checks.size());
            lv.dom0 = P.pool.size();
            P.pool.insert(P.pool.end(), cand[order[d]].begin(), cand[order[d]].end());
            P.levels.push_back(lv);
        }
        pg.pre_begin = static_cast<u32>(P.checks.size());
        P.checks.insert(P.checks.end(), pre.begin(), pre.end());
        pg.pre_end = static_cast<u32>(P.checks.size());
        return pg;
    }

    void program()
    {
        const u32 m = static_cast<u32>(T.kind.size());
        P.n = n;
        P.ow = OW;
        P.fluent_count = L.fluent_count;
        P.words = std::max<u32>(1, words_for(L.fluent_count));
        P.nschemas = static_cast<u32>(T.schemas.size());
        // rs tables into the pool
        layout_rs_off.assign(L.stride.size(), 0);
        for (std::size_t pos = 0; pos < L.stride.size(); ++pos)
        {
            layout_rs_off[pos] = P.pool.size();
            P.pool.insert(P.pool.end(), L.rs.begin() + pos * n, L.rs.begin() + (pos + 1) * n);
        }
        static_rs_off.assign(m, 0);
        P.srel_table.assign(m, 0);
        P.srel_mask.assign(m, 0);
        P.srel_probes.assign(m, 0);
        for (u32 p = 0; p < m; ++p)
            if (T.kind[p] == kStatic)
            {
                // per argument position: the key contribution of each object (the kernels add one per bound
                // parameter), then the key set
                static_rs_off[p] = P.pool.size();
                for (u32 i = 0; i < T.arity[p]; ++i)
                    for (u32 o = 0; o < n; ++o)
                        P.pool.push_back(static_arg_key(i, o));
                P.srel_table[p] = P.pool.size();
                P.pool.insert(P.pool.end(), S[p].table.begin(), S[p].table.end());
                P.srel_mask[p] = S[p].table.size() - 1;
                P.srel_probes[p] = S[p].probes;
            }
        P.domain = L.domain;
        P.pos_dom_begin = L.dom_begin;
        for (std::size_t s = 0; s < T.schemas.size(); ++s)
        {
            const Schema& sc = T.schemas[s];
            P.label_width = std::max(P.label_width, sc.arity);
            DSchema ds;
            ds.arity = sc.arity;
            std::vector<u8> relevant(sc.arity, 0);
            for (const Lit& l : sc.eff)
                for (i32 x : l.terms)
                    if (x >= 0)
                        relevant[x] = 1;
            // witness pruning off: every parameter in index order
            std::vector<u32> all(sc.arity);
            for (u32 v = 0; v < sc.arity; ++v)
                all[v] = v;
            ds.prog[1] = matcher(s, all, sc.arity);
            // witness pruning on: relevant parameters in index order, then the witness-only ones in the reference's
            // order for them; every assignment of the relevant parameters keeps the first witness found
            std::vector<u32> order;
            for (u32 v = 0; v < sc.arity; ++v)
                if (relevant[v])
                    order.push_back(v);
            const u32 first_exist = static_cast<u32>(order.size());
            // the bindings come out in canonical order when every witness parameter follows every relevant one (they
            // then differ in their relevant parameters, which decide the order alone); otherwise the matchers buffer
            // and sort them, as the reference does for a matcher that does not bind in index order
            // (successor/successors.hpp:147-248)
            const u32 last_relevant = order.empty() ? 0 : order.back();
            bool in_order = true;
            for (u32 v : witness_order(s, relevant))
            {
                if (!order.empty() && v < last_relevant)
                    in_order = false;
                order.push_back(v);
            }
            ds.prog[0] = matcher(s, order, first_exist);
            ds.prog[0].sorted = in_order ? 0 : 1;
            // the compiled matcher's selectivity order: keys of 8 bits per parameter (at most 256 objects, 8
            // parameters) sort into canonical order
            double cost_sel = 0, cost_idx = 0;
            const std::vector<u32> sel = selective_order(s, cost_sel, cost_idx);
            if (sc.arity >= 2 && n <= 256 && sel != all && cost_sel * 2 <= cost_idx && !ds.prog[1].never)
            {
                ds.fast = matcher(s, sel, sc.arity);
                ds.fast_on = 1;
            }
            ds.add_begin = static_cast<u32>(P.lits.size());
            for (const Lit& l : sc.eff)
                if (l.pos)
                    pattern(l);
            ds.add_end = static_cast<u32>(P.lits.size());
            ds.del_begin = ds.add_end;
            for (const Lit& l : sc.eff)
                if (!l.pos)
                    pattern(l);
            ds.del_end = static_cast<u32>(P.lits.size());
            P.schemas.push_back(ds);
        }
        // goal masks and the initial row
        P.goal_pos.assign(P.words, 0);
        P.goal_neg.assign(P.words, 0);
        for (const Lit& l : T.goal)
        {
            if (T.kind[l.pred] == kStatic)
            {
                if (static_fact(l) != l.pos)
                    P.goal_unsat = 1;
                continue;
            }
            if (T.kind[l.pred] != kFluent)
                throw std::invalid_argument("mymyr_b200: a derived goal literal");
            std::vector<u32> args;
            for (i32 x : l.terms)
                args.push_back(obj_of(x));
            const u64 c = cid(l.pred, args.data());
            if (c >= L.fluent_count)
            {
                if (l.pos)
                    P.goal_unsat = 1;
                continue;
            }
            set_bit(l.pos ? P.goal_pos.data() : P.goal_neg.data(), c);
        }
        for (u32 w = 0; w < P.words; ++w)
            if (P.goal_pos[w] & P.goal_neg[w])
                P.goal_unsat = 1;
        P.initial.assign(P.words, 0);
        for (const auto& a : T.fluent_init)
        {
            const u64 c = cid(a[0], a.data() + 1);
            if (c >= L.fluent_count)
                throw std::logic_error("mymyr_b200: an initial atom outside the canonical space");
            set_bit(P.initial.data(), c);
        }
        // slot records (decode of every canonical id)
        P.slot_atoms.assign(L.fluent_count, {});
        for (u32 p = 0; p < m; ++p)
        {
            if (T.kind[p] != kFluent)
                continue;
            const u32 ar = T.arity[p];
            for (u64 r = 0; r < L.size[p]; ++r)
            {
                std::vector<u32> rec{p};
                u64 rem = r;
                for (u32 i = 0; i < ar; ++i)
                {
                    const u32 pos = L.pos_begin[p] + i;
                    const u64 q = rem / L.stride[pos];
                    rem -= q * L.stride[pos];
                    rec.push_back(L.domain[L.dom_begin[pos] + q]);
                }
                P.slot_atoms[L.offset[p] + r] = std::move(rec);
            }
        }
    }
};
}  // namespace

TaskSpec read_task_text(const std::string& text) { return Reader(text).read(); }

void compile_task(const TaskSpec& spec, Layout& layout, std::vector<StaticRel>& statics, Program& prog)
{
    Compiler(spec, layout, statics, prog).run();
}
}  // namespace b2
