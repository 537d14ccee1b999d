// Per-task matcher code generation (host). Translates the compiled matcher program (task.hpp: levels, filters,
// checks, effect patterns) into CUDA source for the run-time compiled kernels (jit_kernels.cuh): one nested loop per
// binding level, every layout constant folded in (position offsets, strides, contiguous domains, static domains),
// bindings and candidate sets in registers. The generated matcher enumerates exactly what the interpreted one does
// (device.cuh: enumerate), in the same order; only the execution differs.
//
// Generated interface (namespace b2::gen):
//   constexpr u32 NS, W, WR, OW, NLW;  constexpr u64 F;  __device__ const u64 POOL[];  __device__ const u32 DOM[];
//   template<int S, int PI> struct Run  { template<class St, class E> static bool go(const St&, E& emit); };
//   template<int S> struct Eff          { static constexpr int ND, NA; static void keys(const u32* b, ...); };
//   template<class St> bool goal(const St&);   template<class F> void for_each_schema(F&&);
//   template<class F> void with_schema(u32 s, F&&);   __device__ const u32 ARITY[NS];

#include "task.hpp"

#include <sstream>
#include <stdexcept>
#include <string>

namespace b2
{
namespace
{
std::string hex(u64 v)
{
    std::ostringstream o;
    o << "0x" << std::hex << v << "ull";
    return o.str();
}

struct Gen
{
    const Program& P;
    std::ostringstream o;
    u32 OW;

    explicit Gen(const Program& p) : P(p), OW(p.ow) {}

    /// An rs table (n entries at pool offset `off`) as an expression of the object `b`: affine over a contiguous
    /// object range when it is one, else a POOL lookup.
    std::string rs_expr(u64 off, const std::string& b, u64 outside) const
    {
        const u32 n = P.n;
        i64 lo = -1, hi = -1;
        for (u32 x = 0; x < n; ++x)
            if (P.pool[off + x] != outside)
            {
                if (lo < 0)
                    lo = x;
                hi = x + 1;
            }
        if (lo < 0)
            return hex(outside);
        bool affine = true;
        const u64 stride = hi - lo > 1 ? P.pool[off + lo + 1] - P.pool[off + lo] : 1;
        for (i64 x = lo; x < hi && affine; ++x)
            affine = P.pool[off + x] == static_cast<u64>(x - lo) * stride;
        if (!affine)
            return "POOL[" + std::to_string(off) + "ull + " + b + "]";
        std::ostringstream e;
        e << "((" << b << " - " << lo << "u) < " << (hi - lo) << "u ? static_cast<u64>(" << b << " - " << lo << "u) * "
          << stride << "ull : " << hex(outside) << ")";
        return e.str();
    }

    std::string key_expr(const DLit& l) const
    {
        std::ostringstream e;
        e << "(" << hex(l.base);
        const u64 outside = l.fluent ? kOutside : kStaticOutside;
        for (u32 i = 0; i < l.nvars; ++i)
        {
            const DVar& v = P.vars[l.var_begin + i];
            e << " + " << rs_expr(v.rs, "b[" + std::to_string(v.param) + "]", outside);
        }
        e << ")";
        return e.str();
    }

    /// Truth of a literal (check) as a boolean expression.
    std::string holds_expr(const DLit& l) const
    {
        std::ostringstream e;
        const std::string k = key_expr(l);
        if (l.fluent)
            e << "([&] { const u64 k_ = " << k << "; return k_ < F && bit_of(st, k_); }())";
        else
            e << "static_member(POOL + " << P.srel_table[l.pred] << "ull, " << P.srel_mask[l.pred] << "ull, "
              << P.srel_probes[l.pred] << "u, " << k << ")";
        return l.neg ? "(!" + e.str() + ")" : e.str();
    }

    void filter(const DFilter& f, u32 d)
    {
        const std::string c = "c" + std::to_string(d) + "_";
        o << "    {\n";
        if (f.kind == kFiltSRow)
        {
            o << "      const u64* row_ = POOL + " << f.base << "ull + static_cast<u64>(b[" << f.src << "]) * " << OW
              << "u;\n";
            for (u32 k = 0; k < OW; ++k)
                o << "      " << c << k << " &= " << (f.neg ? "~" : "") << "row_[" << k << "];\n";
            o << "    }\n";
            return;
        }
        for (u32 k = 0; k < OW; ++k)
            o << "      u64 x" << k << " = 0;\n";
        std::string start = hex(f.base);
        if (f.src != kNone)
            start = "(" + hex(f.base) + " + " + rs_expr(f.src_rs, "b[" + std::to_string(f.src) + "]", kOutside) + ")";
        o << "      const u64 s_ = " << start << ";\n";
        o << "      if (s_ < F) {\n";
        auto set_runtime = [&](const std::string& obj) {
            for (u32 k = 0; k < OW; ++k)
                o << "          x" << k << " |= ((" << obj << ") >> 6) == " << k << "u ? (1ull << ((" << obj
                  << ") & 63)) : 0ull;\n";
        };
        if (f.step == 1)
        {
            for (u32 r0 = 0; r0 < f.count; r0 += 64)
            {
                const u32 len = f.count - r0 < 64 ? f.count - r0 : 64;
                o << "        {\n          u64 bits_ = extract64(st, s_ + " << r0 << "u)";
                if (len < 64)
                    o << " & " << hex((u64{1} << len) - 1);
                o << ";\n";
                if (f.map_lo != kNone)
                {
                    const u32 at = f.map_lo + r0, wi = at >> 6, sh = at & 63;
                    if (wi < OW)
                        o << "          x" << wi << " |= bits_ << " << sh << ";\n";
                    if (sh && wi + 1 < OW)
                        o << "          x" << wi + 1 << " |= bits_ >> " << 64 - sh << ";\n";
                }
                else
                {
                    o << "          while (bits_) { const u32 r_ = __ffsll(static_cast<long long>(bits_)) - 1; bits_ &= bits_ - 1;\n"
                      << "            const u32 ob_ = DOM[" << P.pos_dom_begin[f.map_pos] + r0 << "u + r_];\n";
                    set_runtime("ob_");
                    o << "          }\n";
                }
                o << "        }\n";
            }
        }
        else if (f.step <= 32 && 64 % f.step == 0)
        {
            // a strided run word by word: the run's bits in a word are those congruent to s_ modulo the step
            u64 rep = 0;
            for (u32 b = 0; b < 64; b += static_cast<u32>(f.step))
                rep |= u64{1} << b;
            const u64 span = static_cast<u64>(f.count - 1) * f.step;
            o << "        const u64 e_ = s_ + " << span << "ull;\n"
              << "        const u64 rep_ = " << hex(rep) << " << (s_ % " << f.step << "u);\n";
            auto body = [&](const std::string& w, const std::string& wv) {
                o << "          u64 m_ = " << wv << " & rep_;\n"
                  << "          if ((s_ >> 6) == " << w << ") m_ &= ~0ull << (s_ & 63);\n"
                  << "          if ((e_ >> 6) == " << w << ") m_ &= (e_ & 63) == 63 ? ~0ull : ((2ull << (e_ & 63)) - 1);\n"
                  << "          while (m_) { const u32 bt_ = __ffsll(static_cast<long long>(m_)) - 1; m_ &= m_ - 1;\n"
                  << "            const u32 r_ = static_cast<u32>((64ull * " << w << " + bt_ - s_) / " << f.step
                  << "u);\n";
                if (f.map_lo != kNone)
                    o << "            const u32 ob_ = " << f.map_lo << "u + r_;\n";
                else
                    o << "            const u32 ob_ = DOM[" << P.pos_dom_begin[f.map_pos] << "u + r_];\n";
                set_runtime("ob_");
                o << "          }\n";
            };
            if (P.words <= 8)
                for (u32 w = 0; w < P.words; ++w)
                {
                    const std::string ws = std::to_string(w) + "u";
                    o << "        if ((s_ >> 6) <= " << ws << " && (e_ >> 6) >= " << ws << ") {\n";
                    body(ws, "st.word(" + ws + ")");
                    o << "        }\n";
                }
            else
            {
                o << "        for (u32 w_ = static_cast<u32>(s_ >> 6); w_ <= static_cast<u32>(e_ >> 6) && w_ < "
                  << P.words << "u; ++w_) {\n";
                body("w_", "st.word(w_)");
                o << "        }\n";
            }
        }
        else
        {
            o << "        for (u32 r_ = 0; r_ < " << f.count << "u; ++r_)\n"
              << "          if (bit_of(st, s_ + static_cast<u64>(r_) * " << f.step << "ull)) {\n";
            if (f.map_lo != kNone)
                o << "            const u32 ob_ = " << f.map_lo << "u + r_;\n";
            else
                o << "            const u32 ob_ = DOM[" << P.pos_dom_begin[f.map_pos] << "u + r_];\n";
            set_runtime("ob_");
            o << "          }\n";
        }
        o << "      }\n";
        for (u32 k = 0; k < OW; ++k)
            o << "      " << c << k << " &= " << (f.neg ? "~" : "") << "x" << k << ";\n";
        o << "    }\n";
    }

    /// Leaf of a buffered (selectivity-ordered) matcher: the binding's canonical key (8 bits per parameter, the first
    /// parameter highest) into the buffer; a full buffer hands the state to the index-order matcher.
    std::string canon;  // the index-order matcher of the schema being generated, for the fallback
    u32 buffer_arity = 0;

    /// Counting matchers (Count<S, PI>): the leaf adds its candidates instead of emitting them. Selecting matchers
    /// (Select<S, PI>): the leaf skips r_ bindings, by popcount where it can, and emits the next one.
    bool counting = false;
    bool selecting = false;

    void level(const DProgram& pg, u32 d, u32 arity)
    {
        const DLevel& L = P.levels[pg.level_begin + d];
        const std::string D = std::to_string(d);
        o << "  {\n";
        for (u32 k = 0; k < OW; ++k)
            o << "    u64 c" << D << "_" << k << " = " << hex(P.pool[L.dom0 + k]) << ";\n";
        for (u32 fi = L.filt_begin; fi < L.filt_end; ++fi)
            filter(P.filters[fi], d);
        if (counting && d + 1 == pg.nlevels && L.chk_begin == L.chk_end && d <= pg.first_exist)
        {
            // a leaf without checks: every candidate is a binding (an effect level), or the level's first candidate
            // is the binding's witness (the one witness level)
            o << "    n_ += ";
            if (d < pg.first_exist)
                for (u32 k = 0; k < OW; ++k)
                    o << (k ? " + " : "") << "static_cast<u32>(__popcll(c" << D << "_" << k << "))";
            else
            {
                o << "((";
                for (u32 k = 0; k < OW; ++k)
                    o << (k ? " | " : "") << "c" << D << "_" << k;
                o << ") != 0ull ? 1u : 0u)";
            }
            o << ";\n  }\n";
            return;
        }
        if (selecting && d + 1 == pg.nlevels && L.chk_begin == L.chk_end && d <= pg.first_exist)
        {
            const std::string bp = "b[" + std::to_string(L.param) + "]";
            if (d < pg.first_exist)
                for (u32 k = 0; k < OW; ++k)
                {
                    const std::string c = "c" + D + "_" + std::to_string(k);
                    o << "    { const u32 p_ = static_cast<u32>(__popcll(" << c << "));\n"
                      << "      if (sel_ < p_) { " << bp << " = " << 64 * k << "u + nth_bit64(" << c
                      << ", static_cast<u32>(sel_)); emit(static_cast<const u32*>(b)); return true; }\n"
                      << "      sel_ -= p_; }\n";
                }
            else
            {
                o << "    {\n";
                for (u32 k = 0; k < OW; ++k)
                {
                    const std::string c = "c" + D + "_" + std::to_string(k);
                    o << "      " << (k ? "else if (" : "if (") << c << ") { if (sel_ == 0) { " << bp << " = " << 64 * k
                      << "u + (__ffsll(static_cast<long long>(" << c
                      << ")) - 1); emit(static_cast<const u32*>(b)); return true; } --sel_; }\n";
                }
                o << "    }\n";
            }
            o << "  }\n";
            return;
        }
        // one loop per level over the candidates in ascending object order (lowest word first)
        o << "    for (;;) {\n      u32 o" << D << ";\n";
        for (u32 k = 0; k < OW; ++k)
        {
            const std::string c = "c" + D + "_" + std::to_string(k);
            o << "      " << (k ? "else if (" : "if (") << c << ") { o" << D << " = " << 64 * k
              << "u + (__ffsll(static_cast<long long>(" << c << ")) - 1); " << c << " &= " << c << " - 1; }\n";
        }
        o << "      else break;\n";
        o << "      b[" << L.param << "] = o" << D << ";\n";
        for (u32 c = L.chk_begin; c < L.chk_end; ++c)
            o << "      if (!" << holds_expr(P.lits[P.checks[c]]) << ") continue;\n";
        if (d + 1 == pg.nlevels && buffer_arity)
        {
            o << "      {\n        u64 key_ = 0;\n";
            for (u32 v = 0; v < buffer_arity; ++v)
                o << "        key_ |= static_cast<u64>(b[" << v << "]) << " << 8 * (buffer_arity - 1 - v) << ";\n";
            o << "        if (nb_ == 16u) return " << canon << "::go(st, emit);\n"
              << "        buf_[nb_++] = key_;\n      }\n";
        }
        else if (d + 1 == pg.nlevels)
        {
            o << (counting    ? "      ++n_;\n"
                  : selecting ? "      if (sel_ == 0) { emit(static_cast<const u32*>(b)); return true; }\n      --sel_;\n"
                              : "      if (!emit(static_cast<const u32*>(b))) return false;\n");
            if (pg.first_exist < pg.nlevels)
            {
                if (pg.first_exist == 0)
                    o << (counting ? "      return n_;\n" : selecting ? "      return false;\n" : "      return true;\n");
                else
                    o << "      goto next_" << pg.first_exist - 1 << ";\n";
            }
        }
        else
            level(pg, d + 1, arity);
        o << "      next_" << D << ":;\n";
        o << "    }\n  }\n";
    }

    /// One matcher struct `name` over program pg: index order emits as it goes; a buffered one (buffer_arity set)
    /// collects up to 16 bindings, sorts their keys and emits them in canonical order.
    void run_struct(const std::string& name, const DSchema& S, const DProgram& pg)
    {
        o << "template<> struct " << name << " {\n"
          << "template<class St, class E> B2_DI static bool go(const St& st, E&& emit) {\n"
          << "  (void)st;\n  u32 b[" << (S.arity ? S.arity : 1) << "] = {};\n";
        if (pg.never)
        {
            o << "  return true;\n}\n};\n";
            return;
        }
        if (buffer_arity)
            o << "  u64 buf_[16];\n  u32 nb_ = 0;\n";
        for (u32 c = pg.pre_begin; c < pg.pre_end; ++c)
            o << "  if (!" << holds_expr(P.lits[P.checks[c]]) << ") return true;\n";
        if (pg.nlevels == 0)
            o << "  return emit(static_cast<const u32*>(b));\n";
        else
        {
            // a witness exit jumps to the end of the last effect-relevant level's loop body
            level(pg, 0, S.arity);
            if (buffer_arity)
            {
                o << "  for (u32 i_ = 1; i_ < nb_; ++i_) {\n"
                  << "    const u64 x_ = buf_[i_];\n    u32 j_ = i_;\n"
                  << "    while (j_ > 0 && buf_[j_ - 1] > x_) { buf_[j_] = buf_[j_ - 1]; --j_; }\n"
                  << "    buf_[j_] = x_;\n  }\n"
                  << "  for (u32 i_ = 0; i_ < nb_; ++i_) {\n    const u64 k_ = buf_[i_];\n";
                for (u32 v = 0; v < buffer_arity; ++v)
                    o << "    b[" << v << "] = static_cast<u32>((k_ >> " << 8 * (buffer_arity - 1 - v) << ") & 0xffu);\n";
                o << "    if (!emit(static_cast<const u32*>(b))) return false;\n  }\n";
            }
            o << "  return true;\n";
        }
        o << "}\n};\n";
    }

    /// Count<s, pi>: the number of bindings Run<s, pi> emits, by the same levels without emitting (the order does not
    /// matter, so a schema with a selectivity order counts in it); a leaf level without checks adds its candidates
    /// by popcount.
    void count(u32 s, u32 pi)
    {
        const DSchema& S = P.schemas[s];
        const DProgram& pg = S.prog[pi];
        o << "template<> struct Count<" << s << ", " << pi << "> {\n"
          << "template<class St> B2_DI static u32 go(const St& st) {\n  (void)st;\n";
        if (pg.never)
        {
            o << "  return 0u;\n}\n};\n";
            return;
        }
        const bool fast = S.fast_on && pg.first_exist == pg.nlevels && pg.nlevels == S.arity && !pg.sorted;
        const DProgram& cp = fast ? S.fast : pg;
        o << "  u32 b[" << (S.arity ? S.arity : 1) << "] = {};\n  (void)b;\n  u32 n_ = 0;\n";
        for (u32 c = cp.pre_begin; c < cp.pre_end; ++c)
            o << "  if (!" << holds_expr(P.lits[P.checks[c]]) << ") return 0u;\n";
        if (cp.nlevels == 0)
            o << "  return 1u;\n";
        else
        {
            counting = true;
            level(cp, 0, S.arity);
            counting = false;
            o << "  return n_;\n";
        }
        o << "}\n};\n";
    }

    /// Select<s, pi>: emits the r-th binding (0-based) of Run<s, pi>'s canonical order and returns true, or returns
    /// false when there are at most r. It walks the index-order program (the canonical order without buffering);
    /// a leaf level without checks skips whole candidate sets by popcount. Programs whose bindings are emitted
    /// sorted select through Run.
    void select(u32 s, u32 pi)
    {
        const DSchema& S = P.schemas[s];
        const DProgram& pg = S.prog[pi];
        o << "template<> struct Select<" << s << ", " << pi << "> {\n"
          << "template<class St, class E> B2_DI static bool go(const St& st, u64 sel_, E&& emit) {\n  (void)st;\n";
        if (pg.never)
        {
            o << "  (void)sel_; (void)emit;\n  return false;\n}\n};\n";
            return;
        }
        if (pg.sorted)
        {
            o << "  bool found_ = false;\n"
              << "  Run<" << s << ", " << pi << ">::go(st, [&](const u32* b) {\n"
              << "    if (sel_-- != 0) return true;\n    emit(b);\n    found_ = true;\n    return false;\n  });\n"
              << "  return found_;\n}\n};\n";
            return;
        }
        o << "  u32 b[" << (S.arity ? S.arity : 1) << "] = {};\n";
        for (u32 c = pg.pre_begin; c < pg.pre_end; ++c)
            o << "  if (!" << holds_expr(P.lits[P.checks[c]]) << ") return false;\n";
        if (pg.nlevels == 0)
            o << "  if (sel_ != 0) return false;\n  emit(static_cast<const u32*>(b));\n  return true;\n";
        else
        {
            selecting = true;
            level(pg, 0, S.arity);
            selecting = false;
            o << "  return false;\n";
        }
        o << "}\n};\n";
    }

    void run(u32 s, u32 pi)
    {
        const DSchema& S = P.schemas[s];
        const DProgram& pg = S.prog[pi];
        const std::string name = "Run<" + std::to_string(s) + ", " + std::to_string(pi) + ">";
        if (pg.sorted && !pg.never)
        {
            // bindings that do not come out in canonical order: the matcher as it binds (RunRaw), emitted sorted
            const std::string raw = "RunRaw<" + std::to_string(s) + ", " + std::to_string(pi) + ">";
            run_struct(raw, S, pg);
            o << "template<> struct " << name << " {\n"
              << "template<class St, class E> B2_DI static bool go(const St& st, E&& emit) {\n"
              << "  return emit_sorted(" << S.arity << "u, [&](auto&& f_) { return " << raw
              << "::go(st, f_); }, emit);\n}\n};\n";
            return;
        }
        // the selectivity order applies when the program binds every parameter (witness pruning without
        // witness-only parameters binds them all too)
        const bool fast = S.fast_on && !pg.never && pg.first_exist == pg.nlevels && pg.nlevels == S.arity;
        if (!fast)
        {
            run_struct(name, S, pg);
            return;
        }
        canon = "RunCanon<" + std::to_string(s) + ", " + std::to_string(pi) + ">";
        run_struct(canon, S, pg);
        buffer_arity = S.arity;
        run_struct(name, S, S.fast);
        buffer_arity = 0;
    }

    std::string source()
    {
        o << "// generated by mymyr_b200 codegen\n#include \"b2_core.cuh\"\n"
          << "namespace b2 { namespace gen {\nusing namespace b2::dev;\n";
        const int wr = P.words <= 1 ? 1 : P.words <= 2 ? 2 : P.words <= 4 ? 4 : P.words <= 8 ? 8 : 0;
        o << "constexpr u32 NS = " << P.nschemas << "u, W = " << P.words << "u, OW = " << OW << "u, NLW = "
          << (P.label_width ? P.label_width : 1) << "u;\nconstexpr int WR = " << wr << ";\nconstexpr u64 F = "
          << P.fluent_count << "ull;\n";
        o << "__device__ const u64 POOL[" << (P.pool.empty() ? 1 : P.pool.size()) << "] = {";
        for (std::size_t i = 0; i < P.pool.size(); ++i)
            o << (i ? "," : "") << (i % 8 == 0 ? "\n" : "") << hex(P.pool[i]);
        if (P.pool.empty())
            o << "0";
        o << "};\n__device__ const u32 DOM[" << (P.domain.empty() ? 1 : P.domain.size()) << "] = {";
        for (std::size_t i = 0; i < P.domain.size(); ++i)
            o << (i ? "," : "") << (i % 16 == 0 ? "\n" : "") << P.domain[i];
        if (P.domain.empty())
            o << "0";
        o << "};\n__device__ const u32 ARITY[" << (P.nschemas ? P.nschemas : 1) << "] = {";
        for (u32 s = 0; s < P.nschemas; ++s)
            o << (s ? "," : "") << P.schemas[s].arity;
        if (!P.nschemas)
            o << "0";
        o << "};\n";
        // goal
        o << "template<class St> B2_DI bool goal(const St& st) {\n  (void)st;\n";
        if (P.goal_unsat)
            o << "  return false;\n";
        else
        {
            for (u32 w = 0; w < P.words; ++w)
                if (P.goal_pos[w] || P.goal_neg[w])
                    o << "  { const u64 x_ = st.word(" << w << "u); if ((x_ & " << hex(P.goal_pos[w]) << ") != "
                      << hex(P.goal_pos[w]) << " || (x_ & " << hex(P.goal_neg[w]) << ") != 0) return false; }\n";
            o << "  return true;\n";
        }
        o << "}\n";
        o << "template<int S, int PI> struct Run;\ntemplate<int S, int PI> struct RunCanon;\n"
          << "template<int S, int PI> struct RunRaw;\n"
          << "template<int S, int PI> struct Count;\n"
          << "template<int S, int PI> struct Select;\n"
          << "template<int S> struct Eff;\n";
        for (u32 s = 0; s < P.nschemas; ++s)
        {
            for (u32 pi = 0; pi < 2; ++pi)
            {
                const DProgram& pg = P.schemas[s].prog[pi];
                if (pi == 0 && pg.never == 0xFFFFFFFFu)
                {
                    o << "template<> struct Run<" << s << ", 0> { template<class St, class E> B2_DI static bool go("
                      << "const St&, E&&) { return true; } };\n"
                      << "template<> struct Count<" << s << ", 0> { template<class St> B2_DI static u32 go("
                      << "const St&) { return 0u; } };\n"
                      << "template<> struct Select<" << s << ", 0> { template<class St, class E> B2_DI static bool "
                      << "go(const St&, u64, E&&) { return false; } };\n";
                    continue;
                }
                run(s, pi);
                count(s, pi);
                select(s, pi);
            }
            const DSchema& S = P.schemas[s];
            o << "template<> struct Eff<" << s << "> {\n  static constexpr int ND = " << (S.del_end - S.del_begin)
              << ", NA = " << (S.add_end - S.add_begin) << ";\n"
              << "  B2_DI static void keys(const u32* b, u32* del, u32& nd, u32* add, u32& na) {\n"
              << "    (void)b; (void)del; (void)add; nd = 0; na = 0;\n";
            for (u32 i = S.del_begin; i < S.del_end; ++i)
                o << "    { const u64 k_ = " << key_expr(P.lits[i]) << "; if (k_ < F) del[nd++] = static_cast<u32>(k_); }\n";
            for (u32 i = S.add_begin; i < S.add_end; ++i)
                o << "    { const u64 k_ = " << key_expr(P.lits[i]) << "; if (k_ < F) add[na++] = static_cast<u32>(k_); }\n";
            o << "  }\n};\n";
        }
        o << "template<class Fn> B2_DI void for_each_schema(Fn&& f) {\n  (void)f;\n";
        for (u32 s = 0; s < P.nschemas; ++s)
            o << "  f.template operator()<" << s << ">();\n";
        o << "}\ntemplate<class Fn> B2_DI void with_schema(u32 s, Fn&& f) {\n  (void)f;\n  switch (s) {\n";
        for (u32 s = 0; s < P.nschemas; ++s)
            o << "    case " << s << ": f.template operator()<" << s << ">(); break;\n";
        o << "    default: break;\n  }\n}\n";
        o << "}}  // namespace b2::gen\n#include \"b2_jit_kernels.cuh\"\n";
        return o.str();
    }
};
}  // namespace

std::string generate_matcher_source(const Program& prog) { return Gen(prog).source(); }
}  // namespace b2
