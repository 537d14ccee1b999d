// mymyr_b200_shim.hpp: the reference-side binding of the device path, a header a maintainer of maichmueller/mymyr adds
// to the reference (it includes the reference's own headers and compiles only against them). It is the C++ shim of
// INTEGRATION.md as source:
//
//   describe(task.data())   formalism::TaskData (include/mymyr/formalism/task_data.hpp:240-336) -> b2_task_desc
//   check(status)           b2_status -> the reference's exceptions (std::invalid_argument, std::length_error,
//                           std::runtime_error for a device failure)
//   Device                  one b2_ctx per device, kept for the process: repeated searches reuse its pools and the
//                           BrFS layer-loop graph (a context per call would throw them away)
//   brfs(task, options)     mymyr::brfs (include/mymyr/search/brfs.hpp:140) on the device: same signature, same
//                           BrfsResult fields for the options the device path takes (states, expanded, generated,
//                           num_goal_states, layers, layer_counts, exhausted, solved, status, fingerprint, words,
//                           fluent_slots); it refuses the others with std::invalid_argument, as the reference
//                           refuses options a store does not take. The plan and goal state are left empty.
//   dense_initial(task)     the task's initial state in the dense slot order the device path uses, through the
//                           reference's own Task::translate (include/mymyr/task/task.hpp:191) for Auto and Reachable
//                           slots.
//
// The device path numbers atom slots densely (slot = canonical id, TaskOptions::Atoms::Dense). Counts, the fingerprint
// (over canonical ids) and node records do not depend on the slot order; exported rows do, and dense_initial shows the
// translation.

#pragma once

#include "mymyr/formalism/task_data.hpp"
#include "mymyr/search/brfs.hpp"
#include "mymyr/task/task.hpp"
#include "mymyr_b200.h"

#include <cstdint>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

namespace mymyr::b2shim
{
/// A b2_task_desc with the pools it points into.
struct Desc
{
    std::vector<uint8_t> kind;
    std::vector<uint32_t> arity;
    std::vector<int32_t> terms;
    std::vector<b2_literal> lits;
    std::vector<b2_schema_desc> schemas;
    std::vector<uint32_t> static_init, fluent_init;
    b2_task_desc d{};
    Desc() = default;
    Desc(const Desc&) = delete;  // d points into the pools
    Desc& operator=(const Desc&) = delete;
};

inline uint32_t add_literal(Desc& D, const formalism::TaskData& t, const formalism::Literal& l)
{
    const auto ts = t.terms_of(l);
    D.lits.push_back({l.pred.v, l.positive ? 1u : 0u, static_cast<uint32_t>(D.terms.size()),
                      static_cast<uint32_t>(ts.size())});
    D.terms.insert(D.terms.end(), ts.begin(), ts.end());
    return static_cast<uint32_t>(D.lits.size() - 1);
}

/// The task's fields the device path reads, as flat pools. Features it does not run (axioms and derived predicates,
/// numeric fluents, conditional or quantified effects, collapsed parameters) set d.unsupported, which b2_task_create
/// refuses with B2_UNSUPPORTED.
inline std::unique_ptr<Desc> describe(const formalism::TaskData& t)
{
    auto D = std::make_unique<Desc>();
    for (const auto& p : t.predicates)
    {
        D->kind.push_back(p.kind == formalism::PredKind::Static  ? B2_PRED_STATIC
                          : p.kind == formalism::PredKind::Fluent ? B2_PRED_FLUENT
                                                                  : B2_PRED_DERIVED);
        D->arity.push_back(p.arity);
    }
    const auto atoms = [&](const std::vector<formalism::GroundAtom>& v, std::vector<uint32_t>& out) {
        for (const auto& a : v)
        {
            out.push_back(a.pred.v);
            for (const auto o : t.objects_of(a))
                out.push_back(o.v);
        }
    };
    atoms(t.static_init, D->static_init);
    atoms(t.fluent_init, D->fluent_init);
    D->d.goal_begin = static_cast<uint32_t>(D->lits.size());
    for (const auto& l : t.literals_of(t.goal))
        add_literal(*D, t, l);
    D->d.goal_count = static_cast<uint32_t>(D->lits.size()) - D->d.goal_begin;
    if (t.goal.constraints.count)
        D->d.unsupported = 1;
    for (const auto& s : t.schemas)
    {
        b2_schema_desc sd{s.arity(), static_cast<uint32_t>(D->lits.size()), 0, 0, 0, nullptr};
        for (const auto& l : t.literals_of(s.precondition))
        {
            add_literal(*D, t, l);
            ++sd.pre_count;
        }
        if (s.precondition.constraints.count)
            D->d.unsupported = 1;
        sd.eff_begin = static_cast<uint32_t>(D->lits.size());
        for (const auto& ce : t.effects_of(s))
        {
            if (ce.extra_params.count || ce.condition.literals.count || ce.condition.constraints.count ||
                ce.numeric_effects.count)
                D->d.unsupported = 1;  // conditional, quantified or numeric effects
            for (const auto& l : formalism::TaskData::slice(t.literals, ce.effects))
            {
                add_literal(*D, t, l);
                ++sd.eff_count;
            }
        }
        D->schemas.push_back(sd);
    }
    if (!t.axioms.empty() || t.has_numerics() || t.unused_parameters_collapsed)
        D->d.unsupported = 1;
    D->d.num_objects = t.num_objects();
    D->d.num_predicates = static_cast<uint32_t>(D->kind.size());
    D->d.pred_kind = D->kind.data();
    D->d.pred_arity = D->arity.data();
    D->d.terms = D->terms.data();
    D->d.num_terms = static_cast<uint32_t>(D->terms.size());
    D->d.literals = D->lits.data();
    D->d.num_literals = static_cast<uint32_t>(D->lits.size());
    D->d.schemas = D->schemas.data();
    D->d.num_schemas = static_cast<uint32_t>(D->schemas.size());
    D->d.static_init = D->static_init.data();
    D->d.static_init_words = D->static_init.size();
    D->d.fluent_init = D->fluent_init.data();
    D->d.fluent_init_words = D->fluent_init.size();
    return D;
}

/// A b2_status as the reference's exceptions.
inline void check(b2_status s)
{
    if (s == B2_OK)
        return;
    char msg[2048];
    b2_last_error(msg, sizeof msg);
    if (s == B2_INVALID_ARGUMENT || s == B2_UNSUPPORTED || s == B2_PARSE_ERROR)
        throw std::invalid_argument(msg);
    if (s == B2_CAPACITY)
        throw std::length_error(msg);
    throw std::runtime_error(std::string("mymyr_b200 device failure: ") + msg);
}

/// The process's context on a device, created once and kept (its pools and the BrFS layer-loop graph serve every
/// later search on the device).
inline b2_ctx* device(int index = 0)
{
    static std::mutex mu;
    static std::vector<b2_ctx*> ctx;
    std::lock_guard lock(mu);
    if (index < 0)
        throw std::invalid_argument("b2shim::device: negative device index");
    if (ctx.size() <= static_cast<std::size_t>(index))
        ctx.resize(static_cast<std::size_t>(index) + 1, nullptr);
    if (!ctx[static_cast<std::size_t>(index)])
        check(b2_ctx_create(index, &ctx[static_cast<std::size_t>(index)]));
    return ctx[static_cast<std::size_t>(index)];
}

/// A device task (owned; destroyed with the object).
struct DeviceTask
{
    b2_task* t = nullptr;
    DeviceTask(b2_ctx* ctx, const formalism::TaskData& data)
    {
        const auto D = describe(data);
        check(b2_task_create(ctx, &D->d, &t));
    }
    ~DeviceTask() { b2_task_destroy(t); }
    DeviceTask(const DeviceTask&) = delete;
    DeviceTask& operator=(const DeviceTask&) = delete;
};

/// mymyr::brfs on the device (the options and result of include/mymyr/search/brfs.hpp:62-140).
inline BrfsResult brfs(const Task& task, const BrfsOptions& o = {}, int device_index = 0)
{
    if (o.start || !o.blocked_states.empty() || o.max_expanded != ~u64{0} || !o.canonical_order ||
        !o.deterministic_ids || o.goal.kind != search::GoalSpec::Kind::Task)
        throw std::invalid_argument("b2shim::brfs: an option the device BrFS does not take (start, blocked_states, "
                                    "max_expanded, canonical_order=false, deterministic_ids=false, a custom goal)");
    DeviceTask dt(device(device_index), task.data());
    b2_brfs_options bo;
    b2_brfs_options_default(&bo);
    bo.witness_pruning = o.witness_pruning ? 1 : 0;
    bo.stop_at_goal = o.stop_at_goal ? 1 : 0;
    bo.fingerprint = o.fingerprint ? 1 : 0;
    bo.max_depth = o.max_depth;
    bo.max_states = o.max_states;
    std::vector<uint64_t> lc(3 * 4096);
    b2_brfs_result r{};
    r.layer_counts = lc.data();
    r.layer_capacity = 4096;
    b2_brfs* s = nullptr;
    check(b2_brfs_create(dt.t, &bo, &s));
    struct Release
    {
        b2_brfs* s;
        ~Release() { b2_brfs_destroy(s); }
    } release{s};
    check(b2_brfs_run(s, &r));
    BrfsResult out;
    out.states = r.states;
    out.expanded = r.expanded;
    out.generated = r.generated;
    out.num_goal_states = r.num_goal_states;
    out.layers = r.layers;
    out.exhausted = r.exhausted != 0;
    out.solved = r.solved != 0;
    out.fingerprint = r.fingerprint;
    out.search_s = r.search_s;
    out.words = task.words();
    out.fluent_slots = task.atoms().fluent_slots();
    out.store = "device";
    out.status = r.status == B2_SEARCH_SOLVED         ? search::SearchStatus::Solved
                 : r.status == B2_SEARCH_EXHAUSTED    ? search::SearchStatus::Exhausted
                 : r.status == B2_SEARCH_UNSOLVABLE   ? search::SearchStatus::Unsolvable
                                                      : search::SearchStatus::OutOfStates;
    if (o.layer_stats)
        for (uint32_t i = 0; i < r.layers && i < 4096; ++i)
            out.layer_counts.push_back({lc[3 * i], lc[3 * i + 1], lc[3 * i + 2]});
    return out;
}

/// The task's initial state in dense slot order (the rows of the device path): the reference's own Task::translate
/// into the task's dense twin when the task's slots are not dense already.
inline State dense_initial(const Task& task)
{
    const auto dense = task.frozen(TaskOptions::Atoms::Dense);
    return task.translate(task.initial_state(), *dense);
}
}  // namespace mymyr::b2shim
