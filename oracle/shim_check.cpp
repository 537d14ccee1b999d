// Test driver of include/mymyr_b200_shim.hpp (test infrastructure, loaded only by tests/): the reference-side shim
// compiled against the reference's own headers and core, next to the reference's own results.
//
//   shim_check_layout   describe(task.data()) -> b2_task_create (host only): words, fluent slots and initial row equal
//                       the reference's dense twin of the task (dense_initial: Task::translate for Auto slots)
//   shim_check_brfs     b2shim::brfs (the device) and mymyr::brfs (the reference CPU) on the same Task: states,
//                       expanded, generated, goal states, layers, per-layer counts, fingerprint, status

#include "mymyr/formalism/text_format.hpp"
#include "mymyr_b200_shim.hpp"

#include <cstring>
#include <sstream>

using namespace mymyr;

namespace
{
std::shared_ptr<const Task> make_task(const char* text, int atoms)
{
    std::istringstream in(text);
    TaskOptions o;
    o.atoms = atoms == 1 ? TaskOptions::Atoms::Reachable : atoms == 2 ? TaskOptions::Atoms::Dense : TaskOptions::Atoms::Auto;
    return Task::create(formalism::read_task_text(in), o);
}

int fail(char* msg, size_t cap, const std::string& m)
{
    if (msg && cap)
    {
        std::strncpy(msg, m.c_str(), cap - 1);
        msg[cap - 1] = 0;
    }
    return 1;
}
}  // namespace

extern "C" {

/// 0: the host-only device task of describe(task.data()) has the dense twin's words, slots and initial row; 1 with a
/// message otherwise; -1 on an exception.
int shim_check_layout(const char* text, int atoms, char* msg, size_t cap)
{
    try
    {
        const auto task = make_task(text, atoms);
        const auto desc = b2shim::describe(task->data());
        b2_task* t = nullptr;
        b2shim::check(b2_task_create(nullptr, &desc->d, &t));
        b2_task_info info{};
        b2shim::check(b2_task_info_get(t, &info));
        const auto dense = task->frozen(TaskOptions::Atoms::Dense);
        const State init = b2shim::dense_initial(*task);
        std::vector<uint64_t> row(info.words);
        b2shim::check(b2_task_initial_state(t, row.data(), info.words));
        b2_task_destroy(t);
        if (info.words != dense->words() || info.fluent_slots != dense->atoms().fluent_slots())
            return fail(msg, cap, "words or slots differ from the dense twin");
        const StateView v = init.view();
        for (uint32_t w = 0; w < info.words; ++w)
            if (row[w] != (w < v.nw ? v.w[w] : 0))
                return fail(msg, cap, "initial row differs at word " + std::to_string(w));
        return 0;
    }
    catch (const std::exception& e)
    {
        return fail(msg, cap, e.what()) * -1;
    }
}

/// out[0..7] the device's, out[8..15] the reference's: states, expanded, generated, goal states, layers, fingerprint,
/// solved, status. 0 when they and the per-layer counts agree, 1 otherwise, -1 on an exception.
int shim_check_brfs(const char* text, int atoms, uint32_t max_depth, int witness, int stop_at_goal, uint64_t* out,
                    char* msg, size_t cap)
{
    try
    {
        const auto task = make_task(text, atoms);
        BrfsOptions o;
        o.max_depth = max_depth;
        o.witness_pruning = witness != 0;
        o.stop_at_goal = stop_at_goal != 0;
        o.fingerprint = true;
        o.layer_stats = true;
        const BrfsResult dev = b2shim::brfs(*task, o);
        o.store = BrfsOptions::Store::Flat;
        const BrfsResult ref = brfs(*task, o);
        const BrfsResult* rs[2] = {&dev, &ref};
        for (int k = 0; k < 2; ++k)
        {
            const BrfsResult& r = *rs[k];
            uint64_t* x = out + 8 * k;
            x[0] = r.states;
            x[1] = r.expanded;
            x[2] = r.generated;
            x[3] = r.num_goal_states;
            x[4] = r.layers;
            x[5] = r.fingerprint;
            x[6] = r.solved ? 1 : 0;
            x[7] = static_cast<uint64_t>(r.status);
        }
        if (dev.layer_counts != ref.layer_counts)
            return fail(msg, cap, "per-layer counts differ");
        for (int i = 0; i < 8; ++i)
            if (out[i] != out[8 + i])
                return fail(msg, cap, "result field " + std::to_string(i) + " differs");
        return 0;
    }
    catch (const std::exception& e)
    {
        return fail(msg, cap, e.what()) * -1;
    }
}
}
