// The grounded delete relaxation behind h^max (relax.cpp): the reference's RelaxedTask
// (include/mymyr/heuristics/relaxed_task.hpp:1-22 of maichmueller/mymyr) for STRIPS tasks with positive preconditions.

#pragma once

#include "task.hpp"

#include <string>
#include <vector>

namespace b2
{
struct Relaxation
{
    u32 props = 0;  // the task's fluent slots (a proposition per slot: the atom is true)
    // operators as CSR: precondition and add slots of operator o in [pre_begin[o], pre_begin[o + 1]) and
    // [add_begin[o], add_begin[o + 1])
    std::vector<u32> pre_begin, pre, add_begin, add;
    std::vector<u32> goal;          // goal slots
    bool goal_unreachable = false;  // a goal atom the relaxation never reaches: every state is a dead end
    u64 reached = 0;                // atoms of the delete-free fixpoint from the initial state
    u64 ground_actions = 0;
    u64 bindings = 0;               // enumerated by the exploration rounds
    u32 rounds = 0;
    u32 ops() const { return pre_begin.empty() ? 0u : static_cast<u32>(pre_begin.size() - 1); }
};

/// Grounds the delete relaxation of a compiled task from its initial state (throws Error(B2_UNSUPPORTED) for
/// negative fluent preconditions or goals, B2_CAPACITY beyond max_ops operators or max_bindings bindings).
Relaxation ground_relaxation(const TaskSpec& spec, const Layout& layout, const std::vector<StaticRel>& statics,
                             const Program& prog, u64 max_ops = 5'000'000, u64 max_bindings = 100'000'000);
}  // namespace b2
