// Grounding of the delete relaxation (the reference's RelaxedTask::build, include/mymyr/heuristics/relaxed_task.hpp:1-22
// and src/mymyr/heuristics/relaxed_task.cpp of maichmueller/mymyr), for tasks whose preconditions and goal are
// positive (the device h^max has no "atom false" propositions):
//   1. exploration: from the initial state's atoms, every schema binding whose static literals hold (both polarities)
//      and whose positive fluent preconditions are reached adds its add effects; rounds repeat until no atom is new;
//   2. operators: the bindings applicable in the final reached set, with their positive fluent preconditions and their
//      add effects (deletes dropped). Operators that add nothing outside their own preconditions are dropped: they
//      never lower a cost (drive l -> l, say).
// Bindings are enumerated by a depth-first search over the parameters' static domains (the compiler's dom0), each
// literal checked at the depth of its last parameter.

#include "relax.hpp"

#include <algorithm>
#include <stdexcept>

namespace b2
{
namespace
{
struct Grounder
{
    const TaskSpec& T;
    const Layout& L;
    const std::vector<StaticRel>& S;
    const Program& P;
    u32 n;
    u64 max_bindings;
    u64 bindings = 0;

    struct CLit
    {
        u32 pred;
        bool pos;
        bool fluent;
        std::vector<i32> terms;
        i32 last;  // the literal's last parameter (-1: ground)
    };
    struct CSchema
    {
        u32 arity = 0;
        bool never = false;
        std::vector<std::vector<u32>> dom;  // per parameter: objects
        std::vector<CLit> pre;
        std::vector<CLit> add;
    };
    std::vector<CSchema> cs;

    static bool test(const std::vector<u64>& bits, u64 b) { return (bits[b >> 6] >> (b & 63)) & 1; }

    u32 object(i32 term, const u32* bind) const { return term >= 0 ? bind[term] : static_cast<u32>(-(term + 1)); }

    /// Slot of a fluent atom (kNone: outside the layout, never true).
    u64 slot(const CLit& l, const u32* bind) const
    {
        u64 c = L.offset[l.pred];
        for (u32 i = 0; i < l.terms.size(); ++i)
            c += L.rs[static_cast<std::size_t>(L.pos_begin[l.pred] + i) * n + object(l.terms[i], bind)];
        return c < L.fluent_count ? c : kNone;
    }

    bool static_holds(const CLit& l, const u32* bind) const
    {
        u64 k = 0;
        for (u32 i = 0; i < l.terms.size(); ++i)
            k += static_arg_key(i, object(l.terms[i], bind));
        return S[l.pred].holds(k);
    }

    bool holds(const CLit& l, const u32* bind, const std::vector<u64>& reached) const
    {
        if (!l.fluent)
            return static_holds(l, bind) == l.pos;
        const u64 s = slot(l, bind);
        return s != kNone && test(reached, s);  // positive fluent literal (negative ones are refused)
    }

    void prepare()
    {
        cs.resize(T.schemas.size());
        for (u32 si = 0; si < T.schemas.size(); ++si)
        {
            const Schema& sc = T.schemas[si];
            CSchema& c = cs[si];
            c.arity = sc.arity;
            const DProgram& pg = P.schemas[si].prog[1];
            c.never = pg.never != 0;
            c.dom.assign(sc.arity, {});
            for (u32 d = 0; d < pg.nlevels; ++d)
            {
                const DLevel& lv = P.levels[pg.level_begin + d];
                for (u32 o = 0; o < n; ++o)
                    if ((P.pool[lv.dom0 + (o >> 6)] >> (o & 63)) & 1)
                        c.dom[lv.param].push_back(o);
            }
            auto make = [&](const Lit& l) {
                CLit x{l.pred, l.pos, T.kind[l.pred] != kStatic, l.terms, -1};
                for (i32 t : l.terms)
                    x.last = std::max(x.last, t);
                return x;
            };
            for (const Lit& l : sc.pre)
            {
                if (T.kind[l.pred] == kFluent && !l.pos)
                    throw std::domain_error("the device h^max grounds positive preconditions only (schema " + sc.name +
                                            " has a negative one)");
                if (T.kind[l.pred] == kDerived)
                    throw std::domain_error("the device h^max does not ground derived predicates");
                c.pre.push_back(make(l));
            }
            for (const Lit& l : sc.eff)
                if (l.pos && T.kind[l.pred] == kFluent)
                    c.add.push_back(make(l));
        }
    }

    /// Calls emit(bind) for every binding of schema s applicable in the relaxed state `reached`.
    template<class F>
    void enumerate(u32 s, const std::vector<u64>& reached, F&& emit)
    {
        const CSchema& c = cs[s];
        if (c.never)
            return;
        u32 bind[16] = {};
        for (const CLit& l : c.pre)
            if (l.last < 0 && !holds(l, bind, reached))
                return;
        auto rec = [&](auto&& self, u32 d) -> void {
            if (d == c.arity)
            {
                if (++bindings > max_bindings)
                    throw std::length_error("the relaxation's exploration enumerates more than the binding budget");
                emit(static_cast<const u32*>(bind));
                return;
            }
            for (u32 o : c.dom[d])
            {
                bind[d] = o;
                bool ok = true;
                for (const CLit& l : c.pre)
                    if (l.last == static_cast<i32>(d) && !holds(l, bind, reached))
                    {
                        ok = false;
                        break;
                    }
                if (ok)
                    self(self, d + 1);
            }
        };
        rec(rec, 0);
    }
};
}  // namespace

Relaxation ground_relaxation(const TaskSpec& spec, const Layout& layout, const std::vector<StaticRel>& statics,
                             const Program& prog, u64 max_ops, u64 max_bindings)
{
    Grounder G{spec, layout, statics, prog, spec.n, max_bindings};
    G.prepare();
    Relaxation R;
    R.props = static_cast<u32>(layout.fluent_count);
    std::vector<u64> reached(std::max<u64>(1, (layout.fluent_count + 63) / 64), 0);
    const u32 W = prog.words;
    for (u32 w = 0; w < W && w < reached.size(); ++w)
        reached[w] = prog.initial[w];
    // exploration rounds: the reached set grows until a round adds nothing
    for (;;)
    {
        ++R.rounds;
        std::vector<u64> next = reached;
        for (u32 s = 0; s < G.cs.size(); ++s)
            G.enumerate(s, reached, [&](const u32* b) {
                for (const auto& a : G.cs[s].add)
                    if (const u64 sl = G.slot(a, b); sl != kNone)
                        next[sl >> 6] |= u64{1} << (sl & 63);
            });
        if (next == reached)
            break;
        reached.swap(next);
    }
    for (u64 w : reached)
        R.reached += static_cast<u64>(__builtin_popcountll(w));
    // operators: the bindings applicable in the fixpoint
    R.pre_begin.push_back(0);
    R.add_begin.push_back(0);
    std::vector<u32> pre, add;
    for (u32 s = 0; s < G.cs.size(); ++s)
        G.enumerate(s, reached, [&](const u32* b) {
            ++R.ground_actions;
            pre.clear();
            add.clear();
            for (const auto& l : G.cs[s].pre)
                if (l.fluent)
                    if (const u64 sl = G.slot(l, b); sl != kNone)
                        pre.push_back(static_cast<u32>(sl));
            for (const auto& a : G.cs[s].add)
                if (const u64 sl = G.slot(a, b); sl != kNone)
                    add.push_back(static_cast<u32>(sl));
            std::sort(pre.begin(), pre.end());
            pre.erase(std::unique(pre.begin(), pre.end()), pre.end());
            std::sort(add.begin(), add.end());
            add.erase(std::unique(add.begin(), add.end()), add.end());
            bool adds_new = false;
            for (u32 a : add)
                adds_new = adds_new || !std::binary_search(pre.begin(), pre.end(), a);
            if (!adds_new)
                return;
            if (R.pre_begin.size() > max_ops)
                throw std::length_error("the relaxation has more operators than the budget");
            R.pre.insert(R.pre.end(), pre.begin(), pre.end());
            R.add.insert(R.add.end(), add.begin(), add.end());
            R.pre_begin.push_back(static_cast<u32>(R.pre.size()));
            R.add_begin.push_back(static_cast<u32>(R.add.size()));
        });
    R.bindings = G.bindings;
    for (const Lit& l : spec.goal)
    {
        if (spec.kind[l.pred] == kStatic)
            continue;  // a false static goal makes the task unsolvable (Program::goal_unsat)
        if (!l.pos || spec.kind[l.pred] != kFluent)
            throw std::domain_error("the device h^max takes positive fluent goals only");
        Grounder::CLit c{l.pred, true, true, l.terms, -1};
        const u64 sl = G.slot(c, nullptr);
        if (sl == kNone || !((reached[sl >> 6] >> (sl & 63)) & 1))
            R.goal_unreachable = true;
        else
            R.goal.push_back(static_cast<u32>(sl));
    }
    return R;
}
}  // namespace b2
