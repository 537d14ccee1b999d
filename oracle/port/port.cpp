// Test infrastructure, not product code: a CPU restatement of the reference planner's hot path (maichmueller/mymyr),
// written independently of both the reference's code and this repository's device library, as the checker of last
// resort. Small and slow on purpose: bindings are enumerated exhaustively in parameter order over each parameter's
// static domain (the reference's own test oracle works the same way, tests/cpp/support/suite.hpp:76-), and every
// literal is tested directly. Pinned by tests/test_port.py against the reference's golden BrFS counts
// (tests/cpp/support/suite.hpp:31-54) and against the compiled reference (oracle/_ref).
//
// What it restates (reference file:line):
//   text format reader            src/mymyr/formalism/text_format.cpp:16-190
//   static parameter domains      src/mymyr/task/compile.cpp:808-906 (static unary, static binary with a constant,
//                                 projections of static positive k-ary literals)
//   dense canonical layout        src/mymyr/task/compile.cpp:1103-1180, include/mymyr/task/atom_index.hpp:9-16
//   witness-only parameter order  src/mymyr/task/compile.cpp:908-937
//   canonical successor order     include/mymyr/successor/successors.hpp:147-248
//   delete-then-add               include/mymyr/successor/successors.hpp:423-452
//   state hash                    include/mymyr/core/hash.hpp:12-60
//   BrFS loop and fingerprint     src/mymyr/search/brfs.cpp:34-37, 273-404
//   canonical state hash          src/mymyr/task/task.cpp:387-403
//   Philox draws                  include/mymyr/rl/rng.hpp:45-84
//   env step                      src/mymyr/rl/env.cpp:351-520
// Only STRIPS tasks with unconditional effects (what the device path runs).

#include <algorithm>
#include <array>
#include <cstdint>
#include <memory>
#include <cstring>
#include <map>
#include <set>
#include <sstream>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace
{
using u32 = uint32_t;
using u64 = uint64_t;
using i32 = int32_t;

thread_local std::string g_err;

struct L
{
    u32 p;
    bool pos;
    std::vector<i32> t;
};
struct S
{
    u32 arity;
    std::vector<L> pre, eff;
};

struct PortTask
{
    u32 n = 0;
    std::vector<char> kind;  // 'S' static, 'F' fluent
    std::vector<u32> ar;
    std::set<std::vector<u32>> statics;  // [pred, args...]
    std::vector<std::vector<u32>> init;
    std::vector<L> goal;
    std::vector<S> schemas;
    // layout
    std::vector<u64> off;                        // per pred
    std::vector<std::vector<std::vector<u32>>> dom;  // per pred, per position: objects ascending
    std::vector<std::vector<u64>> stride;
    u64 F = 0;  // fluent atoms
    u32 W = 1;
    std::vector<std::vector<std::vector<char>>> pdom;  // per schema, per parameter: static domain (n flags)
    std::vector<std::vector<u32>> order;               // per schema: witness-on binding order
    std::vector<u32> nrel;                             // per schema: relevant parameters
};

std::vector<std::string> toks(const std::string& text)
{
    std::istringstream in(text);
    std::vector<std::string> v;
    std::string w;
    while (in >> w)
        v.push_back(w);
    return v;
}

struct Parse
{
    std::vector<std::string> v;
    size_t i = 0;
    std::string w()
    {
        if (i >= v.size())
            throw std::runtime_error("port: end of input");
        return v[i++];
    }
    long long num() { return std::stoll(w()); }
    void expect(const char* s)
    {
        if (w() != s)
            throw std::runtime_error(std::string("port: expected ") + s);
    }
};

u64 cid(const PortTask& T, u32 p, const u32* a, bool* inside)
{
    u64 c = T.off[p];
    for (u32 i = 0; i < T.ar[p]; ++i)
    {
        const auto& d = T.dom[p][i];
        const auto it = std::lower_bound(d.begin(), d.end(), a[i]);
        if (it == d.end() || *it != a[i])
        {
            *inside = false;
            return 0;
        }
        c += static_cast<u64>(it - d.begin()) * T.stride[p][i];
    }
    *inside = true;
    return c;
}

bool test(const u64* s, u64 b) { return (s[b >> 6] >> (b & 63)) & 1; }

/// Truth of a literal under a binding (objects for terms < 0).
bool holds(const PortTask& T, const L& l, const u32* bind, const u64* s)
{
    std::vector<u32> a(l.t.size());
    for (size_t i = 0; i < l.t.size(); ++i)
        a[i] = l.t[i] >= 0 ? bind[l.t[i]] : static_cast<u32>(-(l.t[i] + 1));
    bool t;
    if (T.kind[l.p] == 'S')
    {
        std::vector<u32> key{l.p};
        key.insert(key.end(), a.begin(), a.end());
        t = T.statics.count(key) != 0;
    }
    else
    {
        bool inside = false;
        const u64 c = cid(T, l.p, a.data(), &inside);
        t = inside && test(s, c);
    }
    return t == l.pos;
}

PortTask* open_text(const std::string& text)
{
    auto T = std::make_unique<PortTask>();
    Parse P{toks(text)};
    P.expect("O");
    T->n = static_cast<u32>(P.num());
    P.expect("P");
    const u32 np = static_cast<u32>(P.num());
    for (u32 i = 0; i < np; ++i)
    {
        const std::string k = P.w();
        if (k != "S" && k != "F")
            throw std::runtime_error("port: only static and fluent predicates");
        T->kind.push_back(k[0]);
        T->ar.push_back(static_cast<u32>(P.num()));
        P.w();
    }
    P.expect("SI");
    for (long long k = P.num(); k-- > 0;)
    {
        std::vector<u32> a{static_cast<u32>(P.num())};
        for (u32 j = 0; j < T->ar[a[0]]; ++j)
            a.push_back(static_cast<u32>(P.num()));
        T->statics.insert(a);
    }
    P.expect("FI");
    for (long long k = P.num(); k-- > 0;)
    {
        std::vector<u32> a{static_cast<u32>(P.num())};
        for (u32 j = 0; j < T->ar[a[0]]; ++j)
            a.push_back(static_cast<u32>(P.num()));
        T->init.push_back(a);
    }
    P.expect("G");
    for (long long k = P.num(); k-- > 0;)
    {
        L l;
        l.p = static_cast<u32>(P.num());
        l.pos = P.num() != 0;
        for (u32 j = 0; j < T->ar[l.p]; ++j)
            l.t.push_back(-static_cast<i32>(P.num()) - 1);
        T->goal.push_back(l);
    }
    auto lits = [&](const char* tag) {
        P.expect(tag);
        std::vector<L> out;
        for (long long k = P.num(); k-- > 0;)
        {
            L l;
            l.p = static_cast<u32>(P.num());
            l.pos = P.num() != 0;
            for (u32 j = 0; j < T->ar[l.p]; ++j)
                l.t.push_back(static_cast<i32>(P.num()));
            out.push_back(l);
        }
        return out;
    };
    P.expect("A");
    for (long long k = P.num(); k-- > 0;)
    {
        S s;
        P.w();
        s.arity = static_cast<u32>(P.num());
        s.pre = lits("L");
        P.expect("E");
        for (long long e = P.num(); e-- > 0;)
        {
            if (P.num() != 0)
                throw std::runtime_error("port: conditional effects");
            if (!lits("L").empty())
                throw std::runtime_error("port: conditional effects");
            for (L& l : lits("F"))
                s.eff.push_back(l);
        }
        T->schemas.push_back(s);
    }
    if (P.i != P.v.size())
        throw std::runtime_error("port: trailing sections");
    const u32 n = T->n;
    // static parameter domains
    for (const S& s : T->schemas)
    {
        std::vector<std::vector<char>> D(s.arity, std::vector<char>(n, 1));
        for (const L& l : s.pre)
        {
            if (T->kind[l.p] != 'S')
                continue;
            std::vector<i32> ps;
            for (i32 x : l.t)
                if (x >= 0 && std::find(ps.begin(), ps.end(), x) == ps.end())
                    ps.push_back(x);
            if (ps.empty())
                continue;
            const u32 a = T->ar[l.p];
            auto restrict_to = [&](u32 v, const std::vector<char>& allowed) {
                for (u32 o = 0; o < n; ++o)
                    D[v][o] = D[v][o] && allowed[o];
            };
            if (a == 1 || (a == 2 && l.t[0] != l.t[1] && (l.t[0] < 0 || l.t[1] < 0)))
            {
                // one parameter, the other position (if any) a constant: the objects making the literal true
                const u32 fpos = l.t[0] >= 0 ? 0 : 1;
                std::vector<char> ok(n, 0);
                for (u32 o = 0; o < n; ++o)
                {
                    std::vector<u32> key{l.p};
                    for (u32 j = 0; j < a; ++j)
                        key.push_back(j == fpos ? o : static_cast<u32>(-(l.t[j] + 1)));
                    ok[o] = (T->statics.count(key) != 0) == l.pos;
                }
                restrict_to(static_cast<u32>(l.t[fpos]), ok);
            }
            else if (l.pos && a >= 3)
                for (u32 i = 0; i < a; ++i)
                    if (l.t[i] >= 0)
                    {
                        std::vector<char> ok(n, 0);
                        for (const auto& key : T->statics)
                        {
                            if (key[0] != l.p)
                                continue;
                            bool match = true;
                            for (u32 j = 0; j < a && match; ++j)
                                if (l.t[j] < 0 && key[1 + j] != static_cast<u32>(-(l.t[j] + 1)))
                                    match = false;
                            if (match)
                                ok[key[1 + i]] = 1;
                        }
                        restrict_to(static_cast<u32>(l.t[i]), ok);
                    }
        }
        T->pdom.push_back(D);
    }
    // dense layout: position domains from the add effects and the initial atoms
    const u32 m = static_cast<u32>(T->kind.size());
    std::vector<std::vector<std::set<u32>>> pos(m);
    for (u32 p = 0; p < m; ++p)
        pos[p].resize(T->ar[p]);
    for (size_t si = 0; si < T->schemas.size(); ++si)
        for (const L& l : T->schemas[si].eff)
            if (l.pos)
                for (size_t i = 0; i < l.t.size(); ++i)
                {
                    if (l.t[i] < 0)
                        pos[l.p][i].insert(static_cast<u32>(-(l.t[i] + 1)));
                    else
                        for (u32 o = 0; o < n; ++o)
                            if (T->pdom[si][l.t[i]][o])
                                pos[l.p][i].insert(o);
                }
    for (const auto& a : T->init)
        for (u32 i = 0; i < T->ar[a[0]]; ++i)
            pos[a[0]][i].insert(a[1 + i]);
    T->off.assign(m, 0);
    T->dom.resize(m);
    T->stride.resize(m);
    u64 run = 0;
    for (u32 p = 0; p < m; ++p)
    {
        if (T->kind[p] != 'F')
            continue;
        u64 size = 1;
        for (u32 i = 0; i < T->ar[p]; ++i)
        {
            T->dom[p].emplace_back(pos[p][i].begin(), pos[p][i].end());
            size *= T->dom[p][i].size();
        }
        T->stride[p].assign(T->ar[p], 1);
        for (u32 i = T->ar[p]; i-- > 1;)
            T->stride[p][i - 1] = T->stride[p][i] * std::max<u64>(1, T->dom[p][i].size());
        T->off[p] = run;
        run += size;
    }
    T->F = run;
    T->W = std::max<u32>(1, static_cast<u32>((run + 63) / 64));
    // witness order (fixed-order matcher): relevant parameters, then witness-only ones by the reference's greedy score
    for (size_t si = 0; si < T->schemas.size(); ++si)
    {
        const S& s = T->schemas[si];
        std::vector<char> rel(s.arity, 0);
        for (const L& l : s.eff)
            for (i32 x : l.t)
                if (x >= 0)
                    rel[x] = 1;
        std::vector<std::pair<u32, u32>> bins;
        std::vector<long> unary(s.arity, 0);
        for (const L& l : s.pre)
        {
            const bool fl = T->kind[l.p] == 'F';
            const u32 a = T->ar[l.p];
            bool any = false;
            for (i32 x : l.t)
                any |= x >= 0;
            if (!any)
                continue;
            if (a == 1)
                unary[l.t[0]] += fl;
            else if (a == 2 && l.t[0] != l.t[1])
            {
                if (l.t[0] >= 0 && l.t[1] >= 0)
                    bins.emplace_back(l.t[0], l.t[1]);
                else if (fl)
                    ++unary[l.t[0] >= 0 ? l.t[0] : l.t[1]];
            }
            else if (!fl && l.pos && a >= 3)
                for (u32 i = 0; i < a; ++i)
                    for (u32 j = i + 1; j < a; ++j)
                        if (l.t[i] >= 0 && l.t[j] >= 0 && l.t[i] != l.t[j])
                            bins.emplace_back(l.t[i], l.t[j]);
        }
        std::vector<u32> order;
        std::vector<char> placed(s.arity, 0);
        for (u32 v = 0; v < s.arity; ++v)
            if (rel[v])
            {
                order.push_back(v);
                placed[v] = 1;
            }
        T->nrel.push_back(static_cast<u32>(order.size()));
        for (;;)
        {
            long best = -1, bs = 0;
            for (u32 v = 0; v < s.arity; ++v)
            {
                if (placed[v])
                    continue;
                long links = 0;
                for (auto [a, b] : bins)
                    links += (a == v && placed[b]) || (b == v && placed[a]);
                long pc = 0;
                for (u32 o = 0; o < n; ++o)
                    pc += T->pdom[si][v][o];
                const long sc = links * 1000000 + unary[v] * 10000 - pc;
                if (best < 0 || sc > bs)
                    best = v, bs = sc;
            }
            if (best < 0)
                break;
            placed[best] = 1;
            order.push_back(static_cast<u32>(best));
        }
        T->order.push_back(order);
    }
    return T.release();
}

struct Succ
{
    u32 schema;
    std::vector<u32> bind;
    std::vector<u64> row;
};

/// Successors of state s in canonical order (exhaustive enumeration, then sorted by binding).
std::vector<Succ> successors(const PortTask& T, const u64* s, bool witness)
{
    std::vector<Succ> out;
    for (u32 si = 0; si < T.schemas.size(); ++si)
    {
        const S& sc = T.schemas[si];
        const u32 k = sc.arity;
        std::vector<std::vector<u32>> cand(k);
        bool empty = false;
        for (u32 v = 0; v < k; ++v)
        {
            for (u32 o = 0; o < T.n; ++o)
                if (T.pdom[si][v][o])
                    cand[v].push_back(o);
            empty |= cand[v].empty();
        }
        // ground preconditions first
        bool ok = true;
        std::vector<u32> b(k, 0);
        for (const L& l : sc.pre)
        {
            bool any = false;
            for (i32 x : l.t)
                any |= x >= 0;
            if (!any)
                ok = ok && holds(T, l, b.data(), s);
        }
        if (!ok || empty)
            continue;
        std::vector<u32> ord(k);
        for (u32 v = 0; v < k; ++v)
            ord[v] = witness ? T.order[si][v] : v;
        const u32 nrel = witness ? T.nrel[si] : k;
        // each literal is tested at the depth (in `ord`) where its last parameter is bound
        std::vector<std::vector<const L*>> at(k + 1);
        for (const L& l : sc.pre)
        {
            u32 last = 0;
            for (i32 x : l.t)
                if (x >= 0)
                    last = std::max<u32>(last, 1 + static_cast<u32>(std::find(ord.begin(), ord.end(), x) - ord.begin()));
            at[last].push_back(&l);
        }
        std::vector<std::vector<u32>> found;
        // depth-first over `ord` with ascending candidates: lexicographic in `ord`, so the first completion of each
        // relevant prefix is the first witness the reference's fixed-order search finds
        auto dfs = [&](auto&& self, u32 d) -> bool {
            if (d == k)
            {
                found.push_back(b);
                return true;
            }
            const u32 v = ord[d];
            for (u32 o : cand[v])
            {
                b[v] = o;
                bool ok = true;
                for (const L* l : at[d + 1])
                    if (!holds(T, *l, b.data(), s))
                    {
                        ok = false;
                        break;
                    }
                if (!ok)
                    continue;
                if (self(self, d + 1) && d + 1 > nrel)
                    return true;  // inside the witness part: one completion is enough
            }
            return false;
        };
        if (k == 0)
            found.push_back({});
        else
            dfs(dfs, 0);
        std::sort(found.begin(), found.end());
        for (const auto& bb : found)
        {
            Succ x;
            x.schema = si;
            x.bind = bb;
            x.row.assign(s, s + T.W);
            for (int pass = 0; pass < 2; ++pass)
                for (const L& l : sc.eff)
                {
                    if (l.pos != (pass == 1))
                        continue;
                    std::vector<u32> a;
                    for (i32 t : l.t)
                        a.push_back(t >= 0 ? bb[t] : static_cast<u32>(-(t + 1)));
                    bool inside = false;
                    const u64 c = cid(T, l.p, a.data(), &inside);
                    if (!inside)
                        continue;
                    if (l.pos)
                        x.row[c >> 6] |= u64{1} << (c & 63);
                    else
                        x.row[c >> 6] &= ~(u64{1} << (c & 63));
                }
            out.push_back(std::move(x));
        }
    }
    return out;
}

u64 mix(u64 x)
{
    x ^= x >> 30;
    x *= 0xbf58476d1ce4e5b9ULL;
    x ^= x >> 27;
    x *= 0x94d049bb133111ebULL;
    x ^= x >> 31;
    return x;
}

u64 fold(u64 a, u64 b)
{
    const unsigned __int128 r = static_cast<unsigned __int128>(a) * b;
    return static_cast<u64>(r) ^ static_cast<u64>(r >> 64);
}

u64 hash_row(const u64* w, u32 W)
{
    u32 n = W;
    while (n && !w[n - 1])
        --n;
    u64 h = 0x2d358dccaa6c78a5ULL ^ (static_cast<u64>(n) * 0x8bb84b93962eacc9ULL);
    u32 i = 0;
    for (; i + 1 < n; i += 2)
        h = fold(h ^ w[i] ^ 0x8bb84b93962eacc9ULL, w[i + 1] ^ 0x4b33a62ed433d4a3ULL);
    if (i < n)
        h = fold(h ^ w[i] ^ 0x8bb84b93962eacc9ULL, 0x4b33a62ed433d4a3ULL);
    return mix(h);
}

bool goal(const PortTask& T, const u64* s)
{
    std::vector<u32> none;
    for (const L& l : T.goal)
        if (!holds(T, l, none.data(), s))
            return false;
    return true;
}

struct RowKey
{
    std::vector<u64> w;
    bool operator==(const RowKey& o) const { return w == o.w; }
};
struct RowHash
{
    size_t operator()(const RowKey& k) const { return hash_row(k.w.data(), static_cast<u32>(k.w.size())); }
};

u64 philox_bits(u64 seed, u64 env, u64 draw)
{
    u32 c[4] = {static_cast<u32>(draw), static_cast<u32>(draw >> 32), static_cast<u32>(env), 0};
    u32 k0 = static_cast<u32>(seed), k1 = static_cast<u32>(seed >> 32);
    for (int r = 0; r < 10; ++r)
    {
        const u64 p0 = static_cast<u64>(0xD2511F53u) * c[0], p1 = static_cast<u64>(0xCD9E8D57u) * c[2];
        const u32 n0 = static_cast<u32>(p1 >> 32) ^ c[1] ^ k0, n1 = static_cast<u32>(p1);
        const u32 n2 = static_cast<u32>(p0 >> 32) ^ c[3] ^ k1, n3 = static_cast<u32>(p0);
        c[0] = n0, c[1] = n1, c[2] = n2, c[3] = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return static_cast<u64>(c[0]) | (static_cast<u64>(c[1]) << 32);
}

u32 below(u64 x, u32 n)
{
    const u64 hi = (x >> 32) * n, lo = (x & 0xFFFFFFFFull) * n;
    return static_cast<u32>((hi + (lo >> 32)) >> 32);
}

template<class F>
int64_t guard(F&& f)
{
    try
    {
        return f();
    }
    catch (const std::exception& e)
    {
        g_err = e.what();
        return -1;
    }
}
}  // namespace

extern "C" {

const char* port_last_error() { return g_err.c_str(); }

void* port_task_open(const char* text)
{
    try
    {
        return open_text(text);
    }
    catch (const std::exception& e)
    {
        g_err = e.what();
        return nullptr;
    }
}

void port_task_close(void* t) { delete static_cast<PortTask*>(t); }

/// out: words, fluent atoms.
void port_task_info(void* t, uint64_t* out)
{
    const PortTask& T = *static_cast<PortTask*>(t);
    out[0] = T.W;
    out[1] = T.F;
}

int64_t port_initial_state(void* t, uint64_t* row)
{
    return guard([&] {
        const PortTask& T = *static_cast<PortTask*>(t);
        std::memset(row, 0, T.W * 8);
        for (const auto& a : T.init)
        {
            bool inside = false;
            const u64 c = cid(T, a[0], a.data() + 1, &inside);
            row[c >> 6] |= u64{1} << (c & 63);
        }
        return int64_t{0};
    });
}

uint64_t port_hash(const uint64_t* row, uint32_t words) { return hash_row(row, words); }

uint64_t port_philox_bits64(uint64_t seed, uint64_t env, uint64_t draw) { return philox_bits(seed, env, draw); }

/// The BrFS loop of run_flat: expands states of depth < max_depth in id order; every successor in canonical order is
/// inserted (first discovery keeps its id). layer_counts[3 * cap]; out: states, expanded, generated, goal states,
/// layers, fingerprint (xor of mix64(id * golden ^ canonical hash)). rows: the states in id order (or null).
int64_t port_brfs(void* t, uint32_t max_depth, int witness, uint64_t* out, uint64_t* layer_counts, uint32_t cap,
                  uint64_t* rows, uint64_t row_cap)
{
    return guard([&]() -> int64_t {
        const PortTask& T = *static_cast<PortTask*>(t);
        const u32 W = T.W;
        std::vector<std::vector<u64>> states;
        std::unordered_map<RowKey, u64, RowHash> ids;
        std::vector<u64> s0(W);
        port_initial_state(t, s0.data());
        states.push_back(s0);
        ids.emplace(RowKey{s0}, 0);
        u64 expanded = 0, generated = 0, goals = 0;
        u32 layers = 0;
        u64 begin = 0, end = 1;
        std::vector<std::array<u64, 3>> lc;
        while (begin < end && layers < max_depth)
        {
            ++layers;
            u64 e = 0, g = 0;
            const u64 before = states.size();
            for (u64 id = begin; id < end; ++id)
            {
                const std::vector<u64> cur = states[id];
                goals += goal(T, cur.data());
                ++e;
                for (Succ& x : successors(T, cur.data(), witness != 0))
                {
                    ++g;
                    if (ids.emplace(RowKey{x.row}, states.size()).second)
                        states.push_back(x.row);
                }
            }
            expanded += e;
            generated += g;
            lc.push_back({e, g, states.size() - before});
            begin = end;
            end = states.size();
        }
        u64 fp = 0;
        for (u64 id = 0; id < states.size(); ++id)
        {
            u64 x = 0;
            for (u32 w = 0; w < W; ++w)
                for (u64 v = states[id][w]; v; v &= v - 1)
                    x ^= mix(static_cast<u64>(w) * 64 + __builtin_ctzll(v) + 0x1234567ULL);
            fp ^= mix(id * 0x9E3779B97F4A7C15ULL ^ x);
        }
        out[0] = states.size();
        out[1] = expanded;
        out[2] = generated;
        out[3] = goals;
        out[4] = layers;
        out[5] = fp;
        for (u32 i = 0; i < lc.size() && i < cap; ++i)
            for (int k = 0; k < 3; ++k)
                layer_counts[3 * i + k] = lc[i][k];
        if (rows)
            for (u64 id = 0; id < states.size() && id < row_cap; ++id)
                std::memcpy(rows + id * W, states[id].data(), W * 8);
        return static_cast<int64_t>(lc.size());
    });
}

/// Successors of n states [n, W]: offsets[n + 1]; per successor schema, binding [label_width], hash. Returns the
/// count (capacity bounds the written rows).
int64_t port_expand(void* t, const uint64_t* states, uint64_t n, int witness, int32_t* offsets, int32_t* schema,
                    int32_t* binding, uint32_t label_width, uint64_t* succ_hash, uint64_t capacity)
{
    return guard([&]() -> int64_t {
        const PortTask& T = *static_cast<PortTask*>(t);
        u64 m = 0;
        for (u64 i = 0; i < n; ++i)
        {
            offsets[i] = static_cast<int32_t>(m);
            for (const Succ& x : successors(T, states + i * T.W, witness != 0))
            {
                if (m < capacity)
                {
                    schema[m] = static_cast<int32_t>(x.schema);
                    for (u32 k = 0; k < label_width; ++k)
                        binding[m * label_width + k] = k < x.bind.size() ? static_cast<int32_t>(x.bind[k]) : -1;
                    succ_hash[m] = hash_row(x.row.data(), T.W);
                }
                ++m;
            }
        }
        offsets[n] = static_cast<int32_t>(m);
        return static_cast<int64_t>(m);
    });
}

/// `steps` random-policy steps of `rows` environments from the initial state (EnvConfig defaults: witness pruning
/// off, goal reward 1, dead ends terminal, SAME_STEP autoreset, no truncation), env ids first_env + row.
/// Writes the final states [rows, W], draws and the sum of rewards per row.
int64_t port_env_run(void* t, uint64_t rows, uint32_t steps, uint64_t seed, uint64_t first_env, uint64_t* states,
                     float* reward_sum)
{
    return guard([&]() -> int64_t {
        const PortTask& T = *static_cast<PortTask*>(t);
        const u32 W = T.W;
        std::vector<u64> s0(W);
        port_initial_state(t, s0.data());
        const bool g0 = goal(T, s0.data());
        for (u64 r = 0; r < rows; ++r)
        {
            std::vector<u64> s = s0;
            bool at_goal = g0;
            float sum = 0;
            for (u32 step = 0; step < steps; ++step)
            {
                std::vector<Succ> xs = at_goal ? std::vector<Succ>{} : successors(T, s.data(), false);
                const u64 draw = step;
                bool moved = false, g = at_goal;
                u32 c2 = 0;
                if (!at_goal && !xs.empty())
                {
                    const u32 a = below(philox_bits(seed, first_env + r, draw), static_cast<u32>(xs.size()));
                    s = xs[a].row;
                    moved = true;
                    g = goal(T, s.data());
                    c2 = static_cast<u32>(successors(T, s.data(), false).size());
                }
                const bool stuck = !at_goal && xs.empty();
                const bool dead = !g && ((moved && c2 == 0) || stuck);
                const bool term = g || dead;
                const bool absorbed = at_goal || (stuck && dead);
                sum += absorbed ? 0.0f : (g ? 1.0f : 0.0f);
                if (term)
                {
                    s = s0;
                    at_goal = g0;
                }
                else
                    at_goal = g;
            }
            std::memcpy(states + r * W, s.data(), W * 8);
            reward_sum[r] = sum;
        }
        return int64_t{0};
    });
}

}  // extern "C"
