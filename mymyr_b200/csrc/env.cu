// Batched environment step (rl::HostEnv::step_row_impl, src/mymyr/rl/env.cpp:351-520; device twin cuda::DeviceEnv,
// include/mymyr/cuda/env.hpp:125-198), Index action space, one task, random policy or given actions.
//
// One fused kernel, one thread per environment. The batch keeps per-schema successor counts of each row's current
// state (b2_env_batch.counts, written by reset and step), so a step needs no full enumeration of the current state:
//   1. choose: c = sum of the cached counts; the index a = below(philox(seed; draw, env, k_successor), c) or the
//      given action; the draw counter advances every step;
//   2. move: the schema whose cached-count prefix holds a, then the (a - prefix)-th binding of that schema in
//      canonical order (early exit), then delete-then-add;
//   3. goal test, one full count of the successor's per-schema counts (the count cache of the next step);
//   4. rewards, termination, truncation; SAME_STEP autoreset into the initial state (its counts precomputed).

#include "common.cuh"

namespace b2
{
namespace
{
struct EnvInit
{
    u32 goal;
    u32 total;
    u32 counts[1];  // [nschemas]
};

template<int OW, int WR>
__global__ void k_env_init(DevTask T, const u64* __restrict__ init, u32 W, u32 pi, u32* __restrict__ out)
{
    const auto st = load_row<WR>(init, W);
    u32 total = 0;
    u32 bind[kMaxLevels] = {};
    for (u32 s = 0; s < T.nschemas; ++s)
    {
        u32 c = 0;
        enumerate<OW>(T, T.schemas[s].prog[pi], st, bind, [&](const u32*) {
            ++c;
            return true;
        });
        out[2 + s] = c;
        total += c;
    }
    out[0] = goal_holds(T, st) ? 1 : 0;
    out[1] = total;
}

/// next_task_ids of a one-task env: every id must name its one instance (0); another id is reported by
/// b2_env_check_errors, and the row keeps its instance (cuda::DeviceEnv::step, include/mymyr/cuda/env.hpp:180-184).
__global__ void k_check_task_ids(const i32* __restrict__ ids, u64 rows, u32* status)
{
    bool bad = false;
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < rows; i += static_cast<u64>(gridDim.x) * blockDim.x)
        bad |= ids[i] != 0;
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0)
        atomicOr(status, dev::kStatusTaskId);
}

struct EnvParams
{
    u64 seed;
    u32 max_steps;
    float step_reward, goal_reward, dead_end_reward;
    u32 dead_end_none, dead_end_terminal, autoreset, pi;
};

template<int OW, int WR>
__global__ void __launch_bounds__(128) k_env_step(DevTask T, EnvParams p, b2_env_batch b, b2_step_out o,
                                                  const i64* __restrict__ actions, const u64* __restrict__ init,
                                                  const u32* __restrict__ init_info, u32* __restrict__ status)
{
    const u32 W = b.words, S = T.nschemas;
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < b.rows; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        u64* row = b.states + i * W;
        u32* cache = b.counts + i * S;
        const auto st = load_row<WR>(row, W);
        const bool already_goal = b.at_goal[i] != 0;
        u32 c = 0;
        for (u32 s = 0; s < S; ++s)
            c += cache[s];
        // 2. the choice
        enum : u32
        {
            kOk,
            kGoal,
            kStuck,
            kInvalid
        };
        u32 stt = already_goal ? kGoal : kOk;
        u64 a = 0;
        if (!already_goal && c == 0)
            stt = kStuck;
        else if (!already_goal && actions)
        {
            const i64 x = actions[i];
            if (x < 0 || static_cast<u64>(x) >= c)
                stt = kInvalid;
            else
                a = static_cast<u64>(x);
        }
        else if (!already_goal)
            a = below(philox_bits64(p.seed, b.first_env + i, b.draws[i], 0u), c);
        b.draws[i] += 1;
        // the move
        u32 bind[kMaxLevels] = {};
        u32 schema = 0;
        Effects e;
        e.n_add = e.n_del = 0;
        if (stt == kOk)
        {
            u64 r = a;
            while (schema < S && r >= cache[schema])
                r -= cache[schema++];
            const DSchema& sc = T.schemas[schema];
            u64 seen = 0;
            const bool exhausted = enumerate<OW>(T, sc.prog[p.pi], st, bind, [&](const u32*) { return seen++ != r; });
            if (exhausted)
            {
                // the cached counts disagree with the state: report it and do not move
                atomicOr(status, kStatusCapacity);
                stt = kStuck;
            }
            else
                collect_effects(T, sc, bind, e);
            if (o.schema)
                o.schema[i] = static_cast<i32>(schema);
            if (o.binding)
                for (u32 k = 0; k < o.label_width; ++k)
                    o.binding[i * o.label_width + k] = k < sc.arity ? static_cast<i32>(bind[k]) : -1;
        }
        else
        {
            if (o.schema)
                o.schema[i] = -1;
            if (o.binding)
                for (u32 k = 0; k < o.label_width; ++k)
                    o.binding[i * o.label_width + k] = -1;
        }
        if (o.invalid)
            o.invalid[i] = stt == kInvalid ? 1 : 0;
        // 3. the reached state's goal test and successor counts
        bool g = already_goal;
        u32 c2 = c;
        u32 newc[16];
        const bool cache_new = stt == kOk;
        if (stt == kOk)
        {
            auto nx = load_row<WR>(row, W);  // overwritten below with the successor words
            if constexpr (WR > 0)
            {
#pragma unroll
                for (int q = 0; q < WR; ++q)
                    nx.w[q] = succ_word(st, e, q);
            }
            else
            {
                for (u32 q = 0; q < W; ++q)
                    row[q] = succ_word(st, e, q);  // wide rows: the successor is written in place first
                nx = GlobalRow{row, W};
            }
            g = goal_holds(T, nx);
            c2 = 0;
            for (u32 s = 0; s < S; ++s)
            {
                u32 cs = 0;
                enumerate<OW>(T, T.schemas[s].prog[p.pi], nx, bind, [&](const u32*) {
                    ++cs;
                    return true;
                });
                if (s < 16)
                    newc[s] = cs;
                else
                    cache[s] = cs;  // beyond the register copy (only written when the row moves)
                c2 += cs;
            }
            if constexpr (WR > 0)
            {
                if (o.final_states)
                    for (u32 q = 0; q < W; ++q)
                        o.final_states[i * W + q] = nx.word(q);
#pragma unroll
                for (int q = 0; q < WR; ++q)
                    if (static_cast<u32>(q) < W)
                        row[q] = nx.w[q];  // provisional: an autoreset overwrites it
            }
            else if (o.final_states)
                for (u32 q = 0; q < W; ++q)
                    o.final_states[i * W + q] = row[q];
        }
        else if (o.final_states)
            for (u32 q = 0; q < W; ++q)
                o.final_states[i * W + q] = st.word(q);
        // 4. rewards, termination, truncation
        const bool dead = !p.dead_end_none && !g && ((stt == kOk && c2 == 0) || stt == kStuck);
        const bool term = g || (dead && p.dead_end_terminal);
        const bool absorbed = already_goal || (stt == kStuck && dead && p.dead_end_terminal);
        const i32 t2 = b.steps ? b.steps[i] + (absorbed ? 0 : 1) : 0;
        const bool trunc = !term && p.max_steps && t2 >= static_cast<i32>(p.max_steps);
        if (o.reward)
            o.reward[i] = absorbed ? 0.0f
                                   : p.step_reward + (g ? p.goal_reward : 0.0f) + (dead ? p.dead_end_reward : 0.0f);
        if (o.terminated)
            o.terminated[i] = term ? 1 : 0;
        if (o.truncated)
            o.truncated[i] = trunc ? 1 : 0;
        if (o.goal)
            o.goal[i] = g ? 1 : 0;
        // 5. the move, or the autoreset
        if (p.autoreset && (term || trunc))
        {
            for (u32 q = 0; q < W; ++q)
                row[q] = init[q];
            if (b.steps)
                b.steps[i] = 0;
            for (u32 s = 0; s < S; ++s)
                cache[s] = init_info[2 + s];
            b.at_goal[i] = static_cast<u8>(init_info[0]);
            if (o.count)
                o.count[i] = static_cast<i32>(init_info[1]);
            continue;
        }
        b.at_goal[i] = g ? 1 : 0;
        if (cache_new)
            for (u32 s = 0; s < S && s < 16; ++s)
                cache[s] = newc[s];
        if (b.steps)
            b.steps[i] = t2;
        if (o.count)
            o.count[i] = static_cast<i32>(c2);
    }
}

__global__ void k_env_reset(u64 rows, u32 W, u32 S, b2_env_batch b, const u8* __restrict__ mask, i32* __restrict__ count,
                            const u64* __restrict__ init, const u32* __restrict__ init_info)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < rows; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        if (mask && !mask[i])
            continue;
        for (u32 q = 0; q < W; ++q)
            b.states[i * W + q] = init[q];
        if (b.steps)
            b.steps[i] = 0;
        for (u32 s = 0; s < S; ++s)
            b.counts[i * S + s] = init_info[2 + s];
        b.at_goal[i] = static_cast<u8>(init_info[0]);
        if (count)
            count[i] = static_cast<i32>(init_info[1]);
    }
}
}  // namespace
}  // namespace b2

using namespace b2;

struct b2_env
{
    b2_task* task = nullptr;
    b2_env_config cfg{};
    DeviceBuffer init;       // [W] initial row
    DeviceBuffer init_info;  // goal, total, counts per schema
    DeviceBuffer status;     // sticky status word (kStatus*)
};

extern "C" {

void b2_env_config_default(b2_env_config* c)
{
    if (!c)
        return;
    *c = b2_env_config{};
    c->goal_reward = 1.0f;
    c->dead_end_terminal = 1;
    c->autoreset = 1;
}

b2_status b2_env_create(b2_task* task, const b2_env_config* config, b2_env** out)
{
    return guarded([&] {
        if (!task || !config || !out)
            throw std::invalid_argument("b2_env_create: null argument");
        if (!task->ctx)
            throw std::invalid_argument("a host-only task (created without a context) cannot run on the device");
        if (config->witness_pruning && task->witness_refused)
            throw Error(B2_UNSUPPORTED, "witness pruning with a witness parameter before an effect parameter");
        B2_CUDA(cudaSetDevice(task->ctx->device));
        auto e = std::make_unique<b2_env>();
        e->task = task;
        e->cfg = *config;
        const Program& P = task->prog;
        e->init.alloc(P.words * 8);
        B2_CUDA(cudaMemcpy(e->init.p, P.initial.data(), P.words * 8, cudaMemcpyHostToDevice));
        e->init_info.alloc((2 + P.nschemas) * 4);
        e->status.alloc(4);
        B2_CUDA(cudaMemset(e->status.p, 0, 4));
        const u32 pi = config->witness_pruning ? 0 : 1;
        if (task->jit)
        {
            dev::EnvArgs a{};
            a.init = e->init.as<u64>();
            a.status = e->init_info.as<u32>();  // the init kernel writes goal, total and per-schema counts here
            jit_launch(task->jit->get(kJitEnvInit, pi), 1, 1, &a, nullptr);
        }
        else
            dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                k_env_init<OW, WR><<<1, 1>>>(task->dev, e->init.as<u64>(), P.words, pi, e->init_info.as<u32>());
            });
        B2_CUDA(cudaGetLastError());
        B2_CUDA(cudaDeviceSynchronize());
        *out = e.release();
    });
}

static void check_batch(const b2_env* env, const b2_env_batch* b)
{
    if (!b || (b->rows && (!b->states || !b->at_goal || !b->counts)))
        throw std::invalid_argument("b2_env: the batch needs states, at_goal and counts");
    if (b->words != env->task->prog.words)
        throw std::invalid_argument("b2_env: rows of " + std::to_string(b->words) + " words; the task has " +
                                    std::to_string(env->task->prog.words));
    if (b->rows > static_cast<u64>(INT32_MAX))
        throw std::invalid_argument("b2_env: more than 2^31 - 1 environments in one batch");
}

b2_status b2_env_reset(b2_env* env, const b2_env_batch* batch, const uint8_t* mask, int32_t* count, void* stream)
{
    return guarded([&] {
        if (!env)
            throw std::invalid_argument("b2_env_reset: null env");
        check_batch(env, batch);
        if (!batch->rows)
            return;
        const Program& P = env->task->prog;
        B2_CUDA(cudaSetDevice(env->task->ctx->device));
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        k_env_reset<<<grid_for(batch->rows, 256), 256, 0, s>>>(batch->rows, P.words, P.nschemas, *batch, mask,
                                                                     count, env->init.as<u64>(),
                                                                     env->init_info.as<u32>());
        B2_CUDA(cudaGetLastError());
    });
}

b2_status b2_env_step(b2_env* env, const b2_env_batch* batch, const b2_step_out* out, const int64_t* actions,
                      void* stream)
{
    return b2_env_step_ex(env, batch, out, actions, nullptr, stream);
}

b2_status b2_env_step_ex(b2_env* env, const b2_env_batch* batch, const b2_step_out* out, const int64_t* actions,
                         const int32_t* next_task_ids, void* stream)
{
    return guarded([&] {
        if (!env || !out)
            throw std::invalid_argument("b2_env_step: null argument");
        check_batch(env, batch);
        if (!actions && batch->rows && !batch->draws)
            throw std::invalid_argument("b2_env_step: the random policy needs the draw counters");
        if (env->cfg.max_steps && batch->rows && !batch->steps)
            throw std::invalid_argument("b2_env_step: truncation (max_steps) needs the step counters");
        const Program& P = env->task->prog;
        if (out->binding && out->label_width < P.label_width)
            throw std::invalid_argument("b2_env_step: label width below the largest schema arity");
        if (!batch->rows)
            return;
        B2_CUDA(cudaSetDevice(env->task->ctx->device));
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (next_task_ids)
            k_check_task_ids<<<grid_for(batch->rows, 256, static_cast<unsigned>(env->task->ctx->sms) * 8), 256, 0, s>>>(
                next_task_ids, batch->rows, env->status.as<u32>());
        EnvParams p;
        p.seed = env->cfg.seed;
        p.max_steps = env->cfg.max_steps;
        p.step_reward = env->cfg.step_reward;
        p.goal_reward = env->cfg.goal_reward;
        p.dead_end_reward = env->cfg.dead_end_reward;
        p.dead_end_none = env->cfg.dead_end_none ? 1 : 0;
        p.dead_end_terminal = env->cfg.dead_end_terminal ? 1 : 0;
        p.autoreset = env->cfg.autoreset ? 1 : 0;
        p.pi = env->cfg.witness_pruning ? 0 : 1;
        const unsigned grid = grid_for(batch->rows, 128, static_cast<unsigned>(env->task->ctx->sms) * 64);
        if (env->task->jit)
        {
            dev::EnvArgs a{};
            a.states = batch->states;
            a.rows = batch->rows;
            a.words = batch->words;
            a.label_width = out->label_width;
            a.steps = batch->steps;
            a.draws = batch->draws;
            a.at_goal = batch->at_goal;
            a.counts = batch->counts;
            a.first_env = batch->first_env;
            a.reward = out->reward;
            a.terminated = out->terminated;
            a.truncated = out->truncated;
            a.count = out->count;
            a.final_states = out->final_states;
            a.schema = out->schema;
            a.binding = out->binding;
            a.invalid = out->invalid;
            a.goal = out->goal;
            a.actions = actions;
            a.init = env->init.as<u64>();
            a.init_info = env->init_info.as<u32>();
            a.status = env->status.as<u32>();
            a.seed = p.seed;
            a.max_steps = p.max_steps;
            a.step_reward = p.step_reward;
            a.goal_reward = p.goal_reward;
            a.dead_end_reward = p.dead_end_reward;
            a.dead_end_none = p.dead_end_none;
            a.dead_end_terminal = p.dead_end_terminal;
            a.autoreset = p.autoreset;
            a.pi = p.pi;
            jit_launch(env->task->jit->get(kJitEnvStep, p.pi), grid, 128, &a, s);
        }
        else
            dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                k_env_step<OW, WR><<<grid, 128, 0, s>>>(env->task->dev, p, *batch, *out, actions, env->init.as<u64>(),
                                                        env->init_info.as<u32>(), env->status.as<u32>());
            });
        B2_CUDA(cudaGetLastError());
    });
}

b2_status b2_env_check_errors(b2_env* env)
{
    return guarded([&] {
        if (!env)
            throw std::invalid_argument("b2_env_check_errors: null env");
        B2_CUDA(cudaGetLastError());
        B2_CUDA(cudaSetDevice(env->task->ctx->device));
        B2_CUDA(cudaDeviceSynchronize());
        u32 st = 0;
        B2_CUDA(cudaMemcpy(&st, env->status.p, 4, cudaMemcpyDeviceToHost));
        if (st)
            B2_CUDA(cudaMemset(env->status.p, 0, 4));  // reported once; later steps flag anew
        if (st & ~dev::kStatusTaskId)
            throw Error(B2_DEVICE_FAULT, "b2_env: the per-schema count cache disagreed with a state (status " +
                                             std::to_string(st) + "); refresh the batch with b2_env_reset");
        if (st & dev::kStatusTaskId)
            throw std::invalid_argument("b2_env: a next_task_ids entry outside the env's tasks (a one-task env "
                                        "takes id 0 only); the rows kept their task");
    });
}

void b2_env_destroy(b2_env* env) { delete env; }

}  // extern "C"
