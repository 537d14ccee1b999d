// Test infrastructure, not product code: a C API over the reference planner's public C++ API (maichmueller/mymyr,
// compiled from its own sources by oracle/Makefile), loaded by tests/ through ctypes as the parity oracle and by
// bench.py's reference arm as the timed CPU baseline. Every entry point calls the reference's own code path:
//   ref_brfs           mymyr::brfs                              include/mymyr/search/brfs.hpp:140
//   ref_brfs_states    the single-threaded BrFS loop of run_flat over the reference's Successors and
//                      FlatStateStore (src/mymyr/search/brfs.cpp:273-404), to read the stored rows in id order
//   ref_expand         mymyr::rl::expand (+ its ThreadPool variant) include/mymyr/rl/expand.hpp:137-147
//   ref_env_*          mymyr::rl::HostEnv reset/step             include/mymyr/rl/env.hpp:214-260
//   ref_pool_bench     mymyr::rl::CpuEnvPool step               include/mymyr/rl/pool.hpp:114-172
//   ref_astar          mymyr::search::astar_eager (h^max)       include/mymyr/search/best_first.hpp:191
//   ref_hmax           heuristics::make_heuristic(Kind::Max)    include/mymyr/heuristics/heuristic.hpp:259
//   ref_brfs_limited   mymyr::brfs with max_states               include/mymyr/search/brfs.hpp:79
//   ref_ground_stats   heuristics::ground (GroundingStats)      include/mymyr/heuristics/heuristic.hpp:165
//   ref_hash_state     mymyr::hash::state                       include/mymyr/core/hash.hpp:58
//   ref_hash_state_numeric  the same with numeric words          include/mymyr/core/hash.hpp:55-60
//   ref_philox_bits64  mymyr::rl::rng::bits64                   include/mymyr/rl/rng.hpp:68
// Errors are caught here and reported as a negative return code plus ref_last_error().

#include "mymyr/core/hash.hpp"
#include "mymyr/core/thread_pool.hpp"
#include "mymyr/heuristics/heuristic.hpp"
#include "mymyr/heuristics/relaxed_task.hpp"
#include "mymyr/rl/env.hpp"
#include "mymyr/rl/expand.hpp"
#include "mymyr/rl/pool.hpp"
#include "mymyr/rl/rng.hpp"
#include "mymyr/rl/task_table.hpp"
#include "mymyr/search/best_first.hpp"
#include "mymyr/search/brfs.hpp"
#include "mymyr/state/flat_store.hpp"
#include "mymyr/successor/successors.hpp"
#include "mymyr/task/task.hpp"
#include "mymyr/task/workspace.hpp"

#include <chrono>
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

using namespace mymyr;

namespace
{
thread_local std::string g_error;

template<class F>
int64_t guarded(F&& f)
{
    try
    {
        return f();
    }
    catch (const std::exception& e)
    {
        g_error = e.what();
        return -1;
    }
    catch (...)
    {
        g_error = "unknown exception";
        return -1;
    }
}

struct TaskHandle
{
    TaskPtr task;
};

const Task& T(void* h) { return *static_cast<TaskHandle*>(h)->task; }

double now_s()
{
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_error.c_str(); }

/// atoms: 0 auto, 1 reachable, 2 dense. matching: 0 auto, 1 fixed order, 2 forward checking.
void* ref_task_open(const char* path, int atoms, int matching)
{
    try
    {
        TaskOptions o;
        o.atoms = atoms == 1 ? TaskOptions::Atoms::Reachable : atoms == 2 ? TaskOptions::Atoms::Dense : TaskOptions::Atoms::Auto;
        o.matching = matching == 1   ? TaskOptions::Matching::FixedOrder
                     : matching == 2 ? TaskOptions::Matching::ForwardChecking
                                     : TaskOptions::Matching::Auto;
        return new TaskHandle{Task::from_text_file(path, o)};
    }
    catch (const std::exception& e)
    {
        g_error = e.what();
        return nullptr;
    }
}

void ref_task_close(void* h) { delete static_cast<TaskHandle*>(h); }

/// out[0..7]: words, fluent slots, schemas, objects, max schema arity, atom mode (0 reachable, 1 dense, 2 lazy),
/// dense fluent atoms, max label width.
int64_t ref_task_info(void* h, uint64_t* out)
{
    return guarded([&] {
        const Task& t = T(h);
        u32 max_arity = 0;
        for (u32 s = 0; s < t.num_schemas(); ++s)
            max_arity = std::max(max_arity, t.compiled().schemas[s].arity);
        out[0] = t.words();
        out[1] = t.atoms().fluent_slots();
        out[2] = t.num_schemas();
        out[3] = t.num_objects();
        out[4] = max_arity;
        out[5] = static_cast<uint64_t>(t.info().atom_mode);
        out[6] = t.info().dense_fluent;
        out[7] = rl::max_label_width(t);
        return int64_t{0};
    });
}

/// The initial state, zero-padded to `words` words.
int64_t ref_initial_state(void* h, uint64_t* out, uint32_t words)
{
    return guarded([&] {
        const State s = T(h).initial_state();
        if (s.size_words() > words)
            throw std::invalid_argument("ref_initial_state: row too narrow");
        std::memset(out, 0, words * sizeof(uint64_t));
        std::memcpy(out, s.data(), s.size_words() * sizeof(uint64_t));
        return int64_t{0};
    });
}

int64_t ref_is_goal(void* h, const uint64_t* row, uint32_t words)
{
    return guarded([&] { return int64_t{T(h).is_goal(StateView{row, bits::trimmed_size(row, words)})}; });
}

uint64_t ref_hash_state(const uint64_t* row, uint32_t words) { return hash::state(row, words, nullptr, 0); }
/// hash::state of a row [words - nnum atom words | nnum numeric words].
uint64_t ref_hash_state_numeric(const uint64_t* row, uint32_t words, uint32_t nnum)
{
    return hash::state(row, words - nnum, row + (words - nnum), nnum);
}

uint64_t ref_canonical_hash(void* h, const uint64_t* row, uint32_t words)
{
    return T(h).canonical_hash(StateView{row, bits::trimmed_size(row, words)});
}

uint64_t ref_fingerprint_term(uint64_t id, uint64_t canonical) { return brfs_fingerprint_term(id, canonical); }

uint64_t ref_philox_bits64(uint64_t seed, uint64_t env, uint64_t draw, uint32_t purpose)
{
    return rl::rng::bits64(seed, env, draw, purpose);
}

void ref_philox_block(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0, uint32_t k1, uint32_t* out)
{
    const rl::rng::Block4 b = rl::rng::philox4x32_10(rl::rng::Block4{{c0, c1, c2, c3}}, k0, k1);
    for (int i = 0; i < 4; ++i)
        out[i] = b.v[i];
}

/// mymyr::brfs. out[0..9]: states, expanded, generated, num_goal_states, layers, exhausted, solved, fingerprint,
/// plan length, status. layer_counts[3 * layer_cap]: {expanded, generated, new} per layer. seconds: search_s.
int64_t ref_brfs(void* h, uint32_t threads, uint32_t max_depth, int stop_at_goal, int witness, int fingerprint,
                 uint64_t* out, double* seconds, uint64_t* layer_counts, uint32_t layer_cap, int store)
{
    return guarded([&] {
        BrfsOptions o;
        o.threads = threads;
        o.max_depth = max_depth;
        o.stop_at_goal = stop_at_goal != 0;
        o.witness_pruning = witness != 0;
        o.fingerprint = fingerprint != 0;
        o.layer_stats = true;
        o.store = store == 1 ? BrfsOptions::Store::Flat : store == 4 ? BrfsOptions::Store::Concurrent : BrfsOptions::Store::Auto;
        const BrfsResult r = brfs(T(h), o);
        out[0] = r.states;
        out[1] = r.expanded;
        out[2] = r.generated;
        out[3] = r.num_goal_states;
        out[4] = r.layers;
        out[5] = r.exhausted;
        out[6] = r.solved;
        out[7] = r.fingerprint;
        out[8] = r.plan.size();
        out[9] = static_cast<uint64_t>(r.status);
        *seconds = r.search_s;
        for (uint32_t i = 0; i < r.layer_counts.size() && i < layer_cap; ++i)
            for (int k = 0; k < 3; ++k)
                layer_counts[3 * i + k] = r.layer_counts[i][k];
        return static_cast<int64_t>(r.layer_counts.size());
    });
}

/// mymyr::brfs single-threaded (flat store) with a state budget: out as ref_brfs (status: SearchStatus).
int64_t ref_brfs_limited(void* h, uint64_t max_states, uint32_t max_depth, int stop_at_goal, int witness,
                         int fingerprint, uint64_t* out, uint64_t* layer_counts, uint32_t layer_cap)
{
    return guarded([&] {
        BrfsOptions o;
        o.threads = 1;
        o.max_states = max_states;
        o.max_depth = max_depth;
        o.stop_at_goal = stop_at_goal != 0;
        o.witness_pruning = witness != 0;
        o.fingerprint = fingerprint != 0;
        o.layer_stats = true;
        o.store = BrfsOptions::Store::Flat;
        const BrfsResult r = brfs(T(h), o);
        out[0] = r.states;
        out[1] = r.expanded;
        out[2] = r.generated;
        out[3] = r.num_goal_states;
        out[4] = r.layers;
        out[5] = r.exhausted;
        out[6] = r.solved;
        out[7] = r.fingerprint;
        out[8] = r.plan.size();
        out[9] = static_cast<uint64_t>(r.status);
        for (uint32_t i = 0; i < r.layer_counts.size() && i < layer_cap; ++i)
            for (int k = 0; k < 3; ++k)
                layer_counts[3 * i + k] = r.layer_counts[i][k];
        return static_cast<int64_t>(r.layer_counts.size());
    });
}

/// The states the single-threaded BrFS stores, in id order (the loop of run_flat, brfs.cpp:273-404, without
/// observers, budgets or goal stops: every state of depth < max_depth is expanded). rows[cap_rows, words];
/// parent[i], succ_index[i]: the node record of state i (the root's parent is 0xFFFFFFFF). Returns the number of
/// states, or -2 if cap_rows is too small.
int64_t ref_brfs_states(void* h, uint32_t max_depth, int witness, uint64_t* rows, uint64_t cap_rows, uint32_t words,
                        uint32_t* parent, uint32_t* succ_index)
{
    return guarded([&]() -> int64_t {
        const Task& task = T(h);
        const WorkspaceLease ws = task.workspace();
        Successors& succ = ws->successors();
        FlatStateStore store(std::max<u32>(1, task.words()), 16, 0);
        const State s0 = task.initial_state();
        store.insert(s0.view());
        std::vector<u32> par{~u32{0}}, idx{0};
        std::vector<u64> cur, next;
        u32 layers = 0, layer_end = 0;
        for (u32 pos = 0; pos < store.size(); ++pos)
        {
            if (pos == layer_end)
            {
                if (layers == max_depth)
                    break;
                ++layers;
                layer_end = store.size();
            }
            const u32 W = store.stride();
            const u64* rec = store.words(StateId{pos});
            cur.assign(rec, rec + W);
            const u32 n = bits::trimmed_size(cur.data(), W);
            succ.prepare(StateView{cur.data(), n});
            u32 k = 0;
            succ.generate<false>(
                [&](u32, const ObjectId*, const Delta& d) -> bool {
                    const u32 nn = apply_delta(cur.data(), n, d, next);
                    const auto [child, fresh] = store.insert(next.data(), nn);
                    if (fresh)
                    {
                        par.push_back(pos);
                        idx.push_back(k);
                    }
                    ++k;
                    return true;
                },
                witness != 0, true);
        }
        if (store.size() > cap_rows)
            return -2;
        if (store.stride() > words)
            throw std::invalid_argument("ref_brfs_states: rows too narrow");
        for (u32 i = 0; i < store.size(); ++i)
        {
            uint64_t* r = rows + static_cast<uint64_t>(i) * words;
            std::memset(r, 0, words * sizeof(uint64_t));
            std::memcpy(r, store.words(StateId{i}), store.stride() * sizeof(uint64_t));
            if (parent)
                parent[i] = par[i];
            if (succ_index)
                succ_index[i] = idx[i];
        }
        return static_cast<int64_t>(store.size());
    });
}

/// mymyr::rl::expand over a single task. threads > 1: the ThreadPool variant. Null outputs are not written.
/// Returns the successor count (generated); capacity bounds the written rows. seconds: wall time of the call.
int64_t ref_expand(void* h, const uint64_t* states, uint64_t n, uint32_t words, int witness, int canonical,
                   uint32_t threads, int32_t* offsets, int32_t* parent, int32_t* schema, int32_t* binding,
                   uint32_t label_width, uint64_t* succ_hash, uint64_t* succ, uint64_t capacity, double* seconds)
{
    return guarded([&] {
        const Task& task = T(h);
        rl::StateBatchView in{states, n, words, 0, 0};
        rl::Expansion out;
        out.capacity = capacity;
        out.words = words;
        out.label_width = label_width;
        out.succ = succ;
        out.parent = parent;
        out.schema = schema;
        out.binding = binding;
        out.offsets = offsets;
        out.succ_hash = succ_hash;
        rl::ExpandOptions opt;
        opt.witness_pruning = witness != 0;
        opt.canonical_order = canonical != 0;
        const double t0 = now_s();
        if (threads > 1)
        {
            ThreadPool pool(threads);
            rl::ExpandScratch scratch;
            const double t1 = now_s();
            rl::expand(task, in, nullptr, out, opt, pool, scratch);
            *seconds = now_s() - t1;
        }
        else
        {
            rl::expand(task, in, nullptr, out, opt);
            *seconds = now_s() - t0;
        }
        return static_cast<int64_t>(out.generated);
    });
}

// ------------------------------------------------------------------------------------------------ host env

struct EnvHandle
{
    std::unique_ptr<rl::HostEnv> env;
    std::unique_ptr<ThreadPool> pool;
};

/// A HostEnv over the one-instance table of the task, with EnvConfig{seed, max_steps, rewards, dead ends,
/// autoreset, witness pruning off, canonical order on}.
void* ref_env_create(void* h, uint64_t seed, uint32_t max_steps, float step_reward, float goal_reward,
                     float dead_end_reward, int dead_end_none, int dead_end_terminal, int autoreset, uint32_t threads)
{
    try
    {
        rl::EnvConfig c;
        c.seed = seed;
        c.max_steps = max_steps;
        c.step_reward = step_reward;
        c.goal_reward = goal_reward;
        c.dead_end_reward = dead_end_reward;
        c.dead_end = dead_end_none ? rl::DeadEnd::None : rl::DeadEnd::NoSuccessors;
        c.dead_end_terminal = dead_end_terminal != 0;
        c.autoreset = autoreset != 0;
        auto* e = new EnvHandle;
        e->env = std::make_unique<rl::HostEnv>(rl::TaskTable::single(static_cast<TaskHandle*>(h)->task), c);
        if (threads > 1)
            e->pool = std::make_unique<ThreadPool>(threads);
        return e;
    }
    catch (const std::exception& e)
    {
        g_error = e.what();
        return nullptr;
    }
}

void ref_env_destroy(void* e) { delete static_cast<EnvHandle*>(e); }

/// HostEnv::reset of every row: states[rows, words], steps, draws kept, at_goal, count.
int64_t ref_env_reset(void* eh, uint64_t* states, uint64_t rows, uint32_t words, int32_t* steps, uint64_t* draws,
                      uint8_t* at_goal, int32_t* count)
{
    return guarded([&] {
        rl::EnvBatch b;
        b.states = states;
        b.rows = rows;
        b.words = words;
        b.steps = steps;
        b.draws = draws;
        b.at_goal = at_goal;
        static_cast<EnvHandle*>(eh)->env->reset(b, nullptr, count);
        return int64_t{0};
    });
}

/// HostEnv::step of every row under the random policy (actions null) or the given int64 actions.
int64_t ref_env_step(void* eh, uint64_t* states, uint64_t rows, uint32_t words, int32_t* steps, uint64_t* draws,
                     uint8_t* at_goal, uint64_t first_env, const int64_t* actions, float* reward, uint8_t* terminated,
                     uint8_t* truncated, int32_t* count, uint64_t* final_states, int32_t* schema, int32_t* binding,
                     uint32_t label_width, uint8_t* invalid, uint8_t* goal, double* seconds)
{
    return guarded([&] {
        EnvHandle* e = static_cast<EnvHandle*>(eh);
        rl::EnvBatch b;
        b.states = states;
        b.rows = rows;
        b.words = words;
        b.steps = steps;
        b.draws = draws;
        b.at_goal = at_goal;
        b.first_env = first_env;
        rl::StepOutputs o;
        o.reward = reward;
        o.terminated = terminated;
        o.truncated = truncated;
        o.count = count;
        o.final_states = final_states;
        o.schema = schema;
        o.binding = binding;
        o.label_width = label_width;
        o.invalid = invalid;
        o.goal = goal;
        rl::Actions a;
        a.v64 = actions;
        const double t0 = now_s();
        e->env->step(b, o, a, nullptr, e->pool.get());
        if (seconds)
            *seconds = now_s() - t0;
        return int64_t{0};
    });
}

/// CpuEnvPool(table, EnvConfig{seed}, num_envs, {threads}) stepping every env `steps` times under the random policy.
/// Returns 0; seconds: the wall time of the steps (construction and reset excluded). out_hash: xor of
/// hash::state over the final states (a cheap whole-batch digest).
int64_t ref_pool_bench(void* h, uint32_t num_envs, uint32_t steps, uint32_t threads, uint64_t seed, double* seconds,
                       uint64_t* out_hash)
{
    return guarded([&] {
        rl::EnvConfig c;
        c.seed = seed;
        rl::PoolOptions po;
        po.threads = threads;
        rl::CpuEnvPool pool(rl::TaskTable::single(static_cast<TaskHandle*>(h)->task), c, num_envs, po);
        pool.reset(nullptr, 0, nullptr);
        rl::PoolBatch last;
        const double t0 = now_s();
        for (uint32_t s = 0; s < steps; ++s)
        {
            last = pool.step(nullptr, 0, rl::Actions{}, nullptr);
            if (s + 1 < steps)
                pool.recycle(std::move(last));
        }
        *seconds = now_s() - t0;
        uint64_t x = 0;
        for (uint64_t i = 0; i < last.rows; ++i)
            x ^= hash::state(last.states.data() + i * last.row_words(), last.words, nullptr, 0);
        *out_hash = x;
        return int64_t{0};
    });
}

/// search::astar_eager with h^max, unit costs. out[0..4]: solved, cost, plan length, expanded, generated.
int64_t ref_astar(void* h, double* out, double* seconds)
{
    return guarded([&] {
        search::BestFirstOptions o;
        o.heuristic.kind = heuristics::Kind::Max;
        o.heuristic.costs = heuristics::Costs::Unit;
        const double t0 = now_s();
        const search::BestFirstResult r = search::astar_eager(T(h), o);
        *seconds = now_s() - t0;
        out[0] = r.status == search::SearchStatus::Solved ? 1 : 0;
        out[1] = r.cost;
        out[2] = static_cast<double>(r.plan.size());
        out[3] = static_cast<double>(r.stats.expanded);
        out[4] = static_cast<double>(r.stats.generated);
        return int64_t{0};
    });
}

/// h^max (unit costs, grounded evaluation) of n rows of `words` words; +inf marks a dead end.
int64_t ref_hmax(void* h, const uint64_t* rows, uint64_t n, uint32_t words, double* out)
{
    return guarded([&] {
        heuristics::Options o;
        o.kind = heuristics::Kind::Max;
        o.costs = heuristics::Costs::Unit;
        o.evaluation = heuristics::Evaluation::Grounded;
        auto H = heuristics::make_heuristic(T(h), o);
        for (uint64_t i = 0; i < n; ++i)
        {
            const uint64_t* r = rows + i * words;
            out[i] = H->evaluate(StateView{r, bits::trimmed_size(r, words)});
        }
        return int64_t{0};
    });
}

/// The grounding's statistics: reached atoms, ground actions, operators, propositions, rounds.
int64_t ref_ground_stats(void* h, uint64_t* out)
{
    return guarded([&] {
        heuristics::GroundingStats st;
        auto R = heuristics::ground(T(h), heuristics::GroundingBudget{}, &st);
        if (!R)
            return int64_t{-3};
        out[0] = st.reached_atoms;
        out[1] = st.ground_actions;
        out[2] = st.operators;
        out[3] = st.propositions;
        out[4] = st.rounds;
        return int64_t{0};
    });
}

}  // extern "C"
