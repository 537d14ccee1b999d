// The kernels of the device path over a generated matcher (namespace b2::gen, see codegen.cpp), compiled at run time
// by NVRTC for sm_100a together with the task's matcher: the BrFS count and expand passes, the env step, and the
// batched expand. Their logic is the one of the nvcc-compiled kernels (brfs.cu, env.cu, expand.cu); only the matcher
// calls differ.

#pragma once

namespace b2
{
namespace gen
{
using namespace b2::dev;

template<int N>
struct RowSel
{
    using type = RegRow<N>;
    B2_DI static type load(const u64* p) { return load_reg_row<N>(p, W); }
};
template<>
struct RowSel<0>
{
    using type = GlobalRow;
    B2_DI static type load(const u64* p) { return GlobalRow{p, W}; }
};
using Row = typename RowSel<WR>::type;

/// The successor of `st` under the effect keys, as a word accessor (wide rows).
struct SuccView
{
    const Row& st;
    const u32* del;
    u32 nd;
    const u32* add;
    u32 na;
    B2_DI u64 word(u32 i) const { return succ_word(st, del, nd, add, na, i); }
};

/// Calls f(successor accessor, hash) for the successor of `st` under schema S's binding b.
template<int S, class F>
B2_DI void with_successor(const Row& st, const u32* b, F&& f)
{
    u32 del[Eff<S>::ND ? Eff<S>::ND : 1], add[Eff<S>::NA ? Eff<S>::NA : 1];
    u32 nd = 0, na = 0;
    Eff<S>::keys(b, del, nd, add, na);
    if constexpr (WR > 0)
    {
        Row nx = st;
#pragma unroll
        for (int j = 0; j < Eff<S>::ND; ++j)
            if (static_cast<u32>(j) < nd)
                nx.clear(del[j]);
#pragma unroll
        for (int j = 0; j < Eff<S>::NA; ++j)
            if (static_cast<u32>(j) < na)
                nx.set(add[j]);
        const u64 h = hash_words_fixed<W>([&](u32 q) { return nx.word(q); });
        f(nx, h);
    }
    else
    {
        const SuccView nx{st, del, nd, add, na};
        const u64 h = hash_words([&](u32 q) { return nx.word(q); }, W);
        f(nx, h);
    }
}

template<int PI>
B2_DI u32 count_all(const Row& st)
{
    u32 c = 0;
    for_each_schema([&]<int S>() { c += Count<S, PI>::go(st); });
    return c;
}

// ------------------------------------------------------------------------------------------------ BrFS
template<int PI>
B2_DI void brfs_count(const BrfsArgs& a)
{
    const u64 E = a.dyn ? a.dyn->E : a.E_dev ? *a.E_dev : a.E;
    const u32* frontier = a.dyn ? a.frontier + a.dyn->layer_begin : a.frontier;
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < E; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 g = frontier[i];
        const Row st = RowSel<WR>::load(a.S.rows + g * W);
        if (goal(st))
        {
            atomicAdd(&a.misc->goals, 1u);
            atomicMin(&a.misc->first_goal, static_cast<u32>(i));
        }
        a.counts[i] = count_all<PI>(st);
    }
}

/// The sharded count pass: brfs_count, plus the successors per owner rank (hashed here, so that every rank learns how
/// many records it will receive before any is pushed).
template<int PI>
B2_DI void dbrfs_count(const BrfsArgs& a)
{
    __shared__ u32 hist[kMaxWorld];
    for (u32 d = threadIdx.x; d < a.world; d += blockDim.x)
        hist[d] = 0;
    __syncthreads();
    const u64 E = a.E_dev ? *a.E_dev : a.E;
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < E; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 g = a.frontier[i];
        const Row st = RowSel<WR>::load(a.S.rows + g * W);
        if (goal(st))
        {
            atomicAdd(&a.misc->goals, 1u);
            atomicMin(&a.misc->first_goal, static_cast<u32>(i));
        }
        u32 k = 0;
        for_each_schema([&]<int S>() {
            Run<S, PI>::go(st, [&](const u32* b) {
                with_successor<S>(st, b, [&](const auto&, u64 h) {
                    // one shared atomic per owner among the lanes emitting together
                    const u32 d = owner_of(h, a.world);
                    const u32 peers = __match_any_sync(__activemask(), d);
                    if ((threadIdx.x & 31) == static_cast<u32>(__ffs(peers) - 1))
                        atomicAdd(&hist[d], static_cast<u32>(__popc(peers)));
                });
                ++k;
                return true;
            });
        });
        a.counts[i] = k;
    }
    __syncthreads();
    for (u32 d = threadIdx.x; d < a.world; d += blockDim.x)
        if (hist[d])
            atomicAdd(reinterpret_cast<unsigned long long*>(a.hist + d), static_cast<unsigned long long>(hist[d]));
}

/// A successor waiting in a warp's queue for its insert.
struct QEntry
{
    u64 w[W];
    u64 h;
    u64 g;
    u32 i, k;
};
/// Queue entries per warp: about 21 KB per 128-thread block (kBrfsExpandBlocksPerSm blocks per SM).
constexpr u32 kQueue = W <= 4 ? 96u : W <= 6 ? 80u : 64u;
/// Queued successors a lane inserts at once (their probes interleaved).
constexpr int kInsertBatch = 4;

/// The expansion with warp-cooperative inserts (rows in registers): each lane runs its parent's matcher and queues
/// every successor (row, hash, candidate index) in shared memory; after the round all 32 lanes insert the queued
/// successors together, so the insert runs on full warps instead of the few lanes whose matcher emitted. A successor
/// that finds the queue full is inserted in place. Same inserts, same protocol: only which thread issues them changes.
template<int PI>
B2_DI void brfs_expand_queued(const BrfsArgs& a)
{
    // the layer's parameters: from the arguments, or from the device state of a device-driven loop
    Store St = a.S;
    u64 E = a.E;
    const u32* frontier = a.frontier;
    if (a.dyn)
    {
        St.layer_cand_begin = a.dyn->cand_next;
        E = a.dyn->E_exp;
        frontier += a.dyn->layer_begin;
    }
    __shared__ QEntry q[4][kQueue];  // blockDim.x = 128: four warps
    __shared__ u32 qn[4];
    const u32 wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0)
        qn[wid] = 0;
    __syncwarp();
    const u64 stride = static_cast<u64>(gridDim.x) * blockDim.x;
    for (u64 base = blockIdx.x * static_cast<u64>(blockDim.x) + wid * 32; base < E; base += stride)
    {
        const u64 i = base + lane;
        if (i < E)
        {
            const u64 pg = frontier[i];
            const Row st = RowSel<WR>::load(St.rows + pg * W);
            const u64 g0 = St.layer_cand_begin + a.cand_base[i];
            u32 k = 0;
            for_each_schema([&]<int S>() {
                Run<S, PI>::go(st, [&](const u32* b) {
                    with_successor<S>(st, b, [&](const auto& nx, u64 h) {
                        const u32 s = atomicAdd(&qn[wid], 1u);
                        if (s < kQueue)
                        {
                            QEntry& e = q[wid][s];
#pragma unroll
                            for (u32 x = 0; x < W; ++x)
                                e.w[x] = nx.word(x);
                            e.h = h;
                            e.g = g0 + k;
                            e.i = static_cast<u32>(i);
                            e.k = k;
                        }
                        else
                            insert<static_cast<int>(W)>(St, nx, h, g0 + k, static_cast<u32>(i), k);
                    });
                    ++k;
                    return true;
                });
            });
        }
        __syncwarp();
        const u32 n = min(qn[wid], kQueue);
        // the queued successors, kInsertBatch per lane at a time with their probes interleaved
        for (u32 s0 = lane; s0 < n; s0 += 32 * kInsertBatch)
        {
            u64 h[kInsertBatch], g[kInsertBatch];
            u32 ii[kInsertBatch], kk[kInsertBatch], idx[kInsertBatch];
            u32 m = 0;
#pragma unroll
            for (int e = 0; e < kInsertBatch; ++e)
            {
                const u32 sx = s0 + 32 * static_cast<u32>(e);
                idx[e] = sx < n ? sx : s0;
                const QEntry& x = q[wid][idx[e]];
                h[e] = x.h;
                g[e] = x.g;
                ii[e] = x.i;
                kk[e] = x.k;
                if (sx < n)
                    m = static_cast<u32>(e) + 1;
            }
            insert_batch<kInsertBatch, static_cast<int>(W)>(St, m, h, g, ii, kk,
                                                              [&](int e, u32 w) { return q[wid][idx[e]].w[w]; });
        }
        __syncwarp();
        if (lane == 0)
            qn[wid] = 0;
        __syncwarp();
    }
}

template<int PI>
B2_DI void brfs_expand(const BrfsArgs& a)
{
    // the layer's parameters: from the arguments, or from the device state of a device-driven loop
    Store St = a.S;
    u64 E = a.E;
    const u32* frontier = a.frontier;
    if (a.dyn)
    {
        St.layer_cand_begin = a.dyn->cand_next;
        E = a.dyn->E_exp;
        frontier += a.dyn->layer_begin;
    }
    if constexpr (WR > 0)
    {
        brfs_expand_queued<PI>(a);
        return;
    }
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < E; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 pg = frontier[i];
        const Row st = RowSel<WR>::load(St.rows + pg * W);
        const u64 g0 = St.layer_cand_begin + a.cand_base[i];
        u32 k = 0;
        for_each_schema([&]<int S>() {
            Run<S, PI>::go(st, [&](const u32* b) {
                with_successor<S>(st, b, [&](const auto& nx, u64 h) {
                    insert<(WR > 0 ? static_cast<int>(W) : 0)>(St, nx, h, g0 + k, static_cast<u32>(i), k);
                });
                ++k;
                return true;
            });
        });
    }
}

/// Sharded BrFS: stages every successor of the local parents with id < limit as [row | hash | c] and counts the
/// records per owner rank (block-local counts, then one atomic per block and rank).
template<int PI>
B2_DI void dbrfs_expand(const DExpandArgs& a)
{
    __shared__ u32 hist[kMaxWorld];
    for (u32 d = threadIdx.x; d < a.world; d += blockDim.x)
        hist[d] = 0;
    __syncthreads();
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < a.E; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 id = a.frontier_id[i];
        if (id >= a.limit)
            continue;
        const Row st = RowSel<WR>::load(a.rows + static_cast<u64>(a.frontier[i]) * W);
        const u64 c0 = a.gbase ? a.gbase[id - a.layer_begin] : id << 32;
        u64* out = a.staging + (a.local_base[i] - a.stage_base) * (W + 2);
        u32 k = 0;
        for_each_schema([&]<int S>() {
            Run<S, PI>::go(st, [&](const u32* b) {
                with_successor<S>(st, b, [&](const auto& nx, u64 h) {
                    u64* r = out + static_cast<u64>(k) * (W + 2);
#pragma unroll
                    for (u32 q = 0; q < W; ++q)
                        r[q] = nx.word(q);
                    r[W] = h;
                    r[W + 1] = c0 + k;
                    atomicAdd(&hist[owner_of(h, a.world)], 1u);
                });
                ++k;
                return true;
            });
        });
    }
    __syncthreads();
    for (u32 d = threadIdx.x; d < a.world; d += blockDim.x)
        if (hist[d])
            atomicAdd(reinterpret_cast<unsigned long long*>(a.hist + d), static_cast<unsigned long long>(hist[d]));
}

/// Words of an exchange record [row | hash | key], and records per warp queue of the fused expansion + push (at most
/// 1024 words a warp: about 32 KB of queue per 128-thread block).
constexpr u32 kRW = W + 2;
constexpr u32 kPushQ = 1024u / kRW < 128u ? 1024u / kRW : 128u;

/// The sharded expansion fused with the exchange: each lane runs its parent's matcher and queues every successor's
/// record [row | hash | parent id << 32 | successor index] in its warp's shared-memory queue; after the round the warp
/// orders the queue by owner rank, reserves each owner's run by one atomic on that owner's fill cursor (in the owner's
/// memory, over NVLink for the other ranks), and writes the runs with consecutive lanes on consecutive words
/// (coalesced NVLink stores). A record that finds the queue full reserves its own slot. No staging area: the records
/// cross NVLink while the matchers run.
template<int PI>
B2_DI void dbrfs_expand_push(const DExpandArgs& a)
{
    __shared__ u64 q[4][kPushQ * kRW];  // blockDim.x = 128: four warps
    __shared__ u32 qn[4];
    __shared__ u32 cnt[4][kMaxWorld], start[4][kMaxWorld];
    __shared__ u64 base[4][kMaxWorld];
    __shared__ unsigned short order[4][kPushQ], pos[4][kPushQ];
    __shared__ u8 dst[4][kPushQ];
    const u32 wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    u64* Q = q[wid];
    if (lane == 0)
        qn[wid] = 0;
    __syncwarp();
    const u64 stride = static_cast<u64>(gridDim.x) * blockDim.x;
    for (u64 first = blockIdx.x * static_cast<u64>(blockDim.x) + wid * 32; first < a.E; first += stride)
    {
        const u64 i = first + lane;
        const u64 id = i < a.E ? a.frontier_id[i] : a.limit;
        if (id < a.limit)
        {
            const Row st = RowSel<WR>::load(a.rows + static_cast<u64>(a.frontier[i]) * W);
            const u64 key0 = id << 32;
            u32 k = 0;
            for_each_schema([&]<int S>() {
                Run<S, PI>::go(st, [&](const u32* b) {
                    with_successor<S>(st, b, [&](const auto& nx, u64 h) {
                        const u32 s = atomicAdd(&qn[wid], 1u);
                        u64* r = nullptr;
                        if (s < kPushQ)
                            r = Q + s * kRW;
                        else
                        {
                            const u32 d = owner_of(h, a.world);
                            const u64 slot = atomicAdd_system(reinterpret_cast<unsigned long long*>(a.cursors[d]), 1ull);
                            if (d == a.me)
                                atomicAdd(a.sent_self, 1ull);
                            if (slot < a.recv_cap)
                                r = a.peers[d] + slot * kRW;
                            else
                                atomicOr(a.overflow, 1u);  // past the owner's buffer: dropped, the layer fails
                        }
                        if (r)
                        {
#pragma unroll
                            for (u32 x = 0; x < W; ++x)
                                r[x] = nx.word(x);
                            r[W] = h;
                            r[W + 1] = key0 + k;
                        }
                    });
                    ++k;
                    return true;
                });
            });
        }
        __syncwarp();
        const u32 n = min(qn[wid], kPushQ);
        if (n)
        {
            for (u32 d = lane; d < a.world; d += 32)
                cnt[wid][d] = 0;
            __syncwarp();
            for (u32 s = lane; s < n; s += 32)
            {
                const u32 d = owner_of(Q[s * kRW + W], a.world);
                dst[wid][s] = static_cast<u8>(d);
                pos[wid][s] = static_cast<unsigned short>(atomicAdd(&cnt[wid][d], 1u));
            }
            __syncwarp();
            if (lane == 0)
            {
                u32 acc = 0;
                for (u32 d = 0; d < a.world; ++d)
                {
                    start[wid][d] = acc;
                    acc += cnt[wid][d];
                }
                if (cnt[wid][a.me])
                    atomicAdd(a.sent_self, static_cast<unsigned long long>(cnt[wid][a.me]));
            }
            for (u32 d = lane; d < a.world; d += 32)
                base[wid][d] = cnt[wid][d] ? atomicAdd_system(reinterpret_cast<unsigned long long*>(a.cursors[d]),
                                                              static_cast<unsigned long long>(cnt[wid][d]))
                                           : 0;
            __syncwarp();
            for (u32 s = lane; s < n; s += 32)
                order[wid][start[wid][dst[wid][s]] + pos[wid][s]] = static_cast<unsigned short>(s);
            __syncwarp();
            for (u32 x = lane; x < n * kRW; x += 32)
            {
                const u32 sp = x / kRW, w = x - sp * kRW;
                const u32 s = order[wid][sp], d = dst[wid][s];
                const u64 slot = base[wid][d] + (sp - start[wid][d]);
                if (slot < a.recv_cap)
                    a.peers[d][slot * kRW + w] = Q[s * kRW + w];
                else if (w == 0)
                    atomicOr(a.overflow, 1u);  // past the owner's buffer: dropped, the layer fails
            }
            __syncwarp();
            if (lane == 0)
                qn[wid] = 0;
            __syncwarp();
        }
    }
    // the records are visible to every rank before this kernel completes; the ranks' next collective orders them
    // before the owners' inserts
    __threadfence_system();
}

// ------------------------------------------------------------------------------------------------ env
template<int PI>
B2_DI void env_init(const EnvArgs& a)
{
    const Row st = RowSel<WR>::load(a.init);
    u32* out = a.status;  // [2 + NS]: goal, total, per-schema counts
    u32 total = 0;
    for_each_schema([&]<int S>() {
        const u32 c = Count<S, PI>::go(st);
        out[2 + S] = c;
        total += c;
    });
    out[0] = goal(st) ? 1 : 0;
    out[1] = total;
}

template<int PI>
B2_DI void env_step(const EnvArgs& a)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < a.rows; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        u64* row = a.states + i * W;
        u32* cache = a.counts + i * NS;
        const Row st = RowSel<WR>::load(row);
        const bool already_goal = a.at_goal[i] != 0;
        u32 c = 0;
        for (u32 s = 0; s < NS; ++s)
            c += cache[s];
        enum : u32
        {
            kOk,
            kGoal,
            kStuck,
            kInvalid
        };
        u32 stt = already_goal ? kGoal : kOk;
        u64 act = 0;
        if (!already_goal && c == 0)
            stt = kStuck;
        else if (!already_goal && a.actions)
        {
            const i64 x = a.actions[i];
            if (x < 0 || static_cast<u64>(x) >= c)
                stt = kInvalid;
            else
                act = static_cast<u64>(x);
        }
        else if (!already_goal)
            act = below(philox_bits64(a.seed, a.first_env + i, a.draws[i], 0u), c);
        a.draws[i] += 1;
        u32 schema = 0;
        u64 r = act;
        if (stt == kOk)
            while (schema < NS && r >= cache[schema])
                r -= cache[schema++];
        bool g = already_goal;
        u32 c2 = c;
        bool moved = false;
        u32 newc[NS ? NS : 1];
        if (stt == kOk)
        {
            bool found = false;
            with_schema(schema, [&]<int S>() {
                found = Select<S, PI>::go(st, r, [&](const u32* b) {
                    if (a.schema)
                        a.schema[i] = static_cast<i32>(S);
                    if (a.binding)
                        for (u32 k = 0; k < a.label_width; ++k)
                            a.binding[i * a.label_width + k] = k < ARITY[S] ? static_cast<i32>(b[k]) : -1;
                    with_successor<S>(st, b, [&](const auto& nx, u64) {
                        for (u32 q = 0; q < W; ++q)
                        {
                            const u64 x = nx.word(q);
                            if (a.final_states)
                                a.final_states[i * W + q] = x;
                            row[q] = x;  // provisional: an autoreset overwrites it (wide rows: reads stay ahead)
                        }
                    });
                });
            });
            if (!found)
            {
                atomicOr(a.status, kStatusCapacity);  // the count cache disagreed with the state
                stt = kStuck;
            }
            else
            {
                moved = true;
                const Row nx = RowSel<WR>::load(row);
                g = goal(nx);
                c2 = 0;
                for_each_schema([&]<int S>() {
                    const u32 cs = Count<S, PI>::go(nx);
                    newc[S] = cs;
                    c2 += cs;
                });
            }
        }
        if (stt != kOk)
        {
            if (a.schema)
                a.schema[i] = -1;
            if (a.binding)
                for (u32 k = 0; k < a.label_width; ++k)
                    a.binding[i * a.label_width + k] = -1;
            if (a.final_states)
                for (u32 q = 0; q < W; ++q)
                    a.final_states[i * W + q] = st.word(q);
        }
        if (a.invalid)
            a.invalid[i] = stt == kInvalid ? 1 : 0;
        const bool dead = !a.dead_end_none && !g && ((moved && c2 == 0) || stt == kStuck);
        const bool term = g || (dead && a.dead_end_terminal);
        const bool absorbed = already_goal || (stt == kStuck && dead && a.dead_end_terminal);
        const i32 t2 = a.steps ? a.steps[i] + (absorbed ? 0 : 1) : 0;
        const bool trunc = !term && a.max_steps && t2 >= static_cast<i32>(a.max_steps);
        if (a.reward)
            a.reward[i] = absorbed ? 0.0f : a.step_reward + (g ? a.goal_reward : 0.0f) + (dead ? a.dead_end_reward : 0.0f);
        if (a.terminated)
            a.terminated[i] = term ? 1 : 0;
        if (a.truncated)
            a.truncated[i] = trunc ? 1 : 0;
        if (a.goal)
            a.goal[i] = g ? 1 : 0;
        if (a.autoreset && (term || trunc))
        {
            for (u32 q = 0; q < W; ++q)
                row[q] = a.init[q];
            if (a.steps)
                a.steps[i] = 0;
            for (u32 s = 0; s < NS; ++s)
                cache[s] = a.init_info[2 + s];
            a.at_goal[i] = static_cast<u8>(a.init_info[0]);
            if (a.count)
                a.count[i] = static_cast<i32>(a.init_info[1]);
            continue;
        }
        a.at_goal[i] = g ? 1 : 0;
        if (moved)
            for (u32 s = 0; s < NS; ++s)
                cache[s] = newc[s];
        if (a.steps)
            a.steps[i] = t2;
        if (a.count)
            a.count[i] = static_cast<i32>(c2);
    }
}

// ------------------------------------------------------------------------------------------------ batched expand
// One thread per state, all schemas in order: the lanes of a warp run the same schema's matcher on 32 states at once
// (a thread per (state, schema) segment made every warp step through all schemas' code, a divergence of NS ways).
template<int PI>
B2_DI void expand_count(const ExpandArgs& a)
{
    for (u64 r = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; r < a.rows; r += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const Row st = RowSel<WR>::load(a.states + r * W);
        u32* out = a.counts + r * NS;
        for_each_schema([&]<int S>() { out[S] = Count<S, PI>::go(st); });
    }
}

template<int PI>
B2_DI void expand_write(const ExpandArgs& a)
{
    for (u64 r = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; r < a.rows; r += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const Row st = RowSel<WR>::load(a.states + r * W);
        for_each_schema([&]<int S>() {
            u64 idx = a.seg_off[r * NS + S];
            Run<S, PI>::go(st, [&](const u32* b) {
                if (idx < a.capacity)
                {
                    if (a.parent)
                        a.parent[idx] = static_cast<i32>(r);
                    if (a.schema)
                        a.schema[idx] = static_cast<i32>(S);
                    if (a.binding)
                        for (u32 k = 0; k < a.label_width; ++k)
                            a.binding[idx * a.label_width + k] = k < ARITY[S] ? static_cast<i32>(b[k]) : -1;
                    if (!a.hash_pass && (a.succ_hash || a.succ))
                        with_successor<S>(st, b, [&](const auto& nx, u64 h) {
                            if (a.succ_hash)
                                a.succ_hash[idx] = h;
                            if (a.succ)
                                for (u32 w = 0; w < a.out_words; ++w)
                                    a.succ[idx * a.out_words + w] = w < W ? nx.word(w) : 0;
                        });
                }
                ++idx;
                return true;
            });
        });
    }
}

/// The successors' hashes and rows from the written records (parent, schema, binding), one thread per successor:
/// the lanes of a warp hash 32 successors at once (in the writing pass only the few lanes whose matcher found a
/// binding would hash, one successor at a time), and consecutive successors share their parent's row.
template<int PI>
B2_DI void expand_hash(const ExpandArgs& a)
{
    const u64 m = *a.total < a.capacity ? *a.total : a.capacity;
    for (u64 idx = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; idx < m; idx += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 r = static_cast<u64>(a.parent[idx]);
        const u32 s = static_cast<u32>(a.schema[idx]);
        u32 b[NLW];
        for (u32 k = 0; k < NLW; ++k)
            b[k] = k < a.label_width ? static_cast<u32>(a.binding[idx * a.label_width + k]) : 0u;
        const Row st = RowSel<WR>::load(a.states + r * W);
        with_schema(s, [&]<int S>() {
            with_successor<S>(st, b, [&](const auto& nx, u64 h) {
                if (a.succ_hash)
                    a.succ_hash[idx] = h;
                if (a.succ)
                    for (u32 w = 0; w < a.out_words; ++w)
                        a.succ[idx * a.out_words + w] = w < W ? nx.word(w) : 0;
            });
        });
    }
}
}  // namespace gen
}  // namespace b2

#if defined(B2J_ALL) || defined(B2J_K0)
// Each pair is compiled alone (-DB2J_K<index of the pair in JitKernel>, jit.cu) or all together (-DB2J_ALL).
extern "C" __global__ void __launch_bounds__(128) b2j_brfs_count_w(b2::dev::BrfsArgs a) { b2::gen::brfs_count<0>(a); }
extern "C" __global__ void __launch_bounds__(128) b2j_brfs_count_nw(b2::dev::BrfsArgs a) { b2::gen::brfs_count<1>(a); }
#endif
#if defined(B2J_ALL) || defined(B2J_K1)
extern "C" __global__ void __launch_bounds__(128, b2::dev::kBrfsExpandBlocksPerSm) b2j_brfs_expand_w(b2::dev::BrfsArgs a) { b2::gen::brfs_expand<0>(a); }
extern "C" __global__ void __launch_bounds__(128, b2::dev::kBrfsExpandBlocksPerSm) b2j_brfs_expand_nw(b2::dev::BrfsArgs a) { b2::gen::brfs_expand<1>(a); }
#endif
#if defined(B2J_ALL) || defined(B2J_K2)
extern "C" __global__ void __launch_bounds__(128) b2j_dbrfs_expand_w(b2::dev::DExpandArgs a) { b2::gen::dbrfs_expand<0>(a); }
extern "C" __global__ void __launch_bounds__(128) b2j_dbrfs_expand_nw(b2::dev::DExpandArgs a) { b2::gen::dbrfs_expand<1>(a); }
#endif
#if defined(B2J_ALL) || defined(B2J_K3)
extern "C" __global__ void __launch_bounds__(128) b2j_dbrfs_count_w(b2::dev::BrfsArgs a) { b2::gen::dbrfs_count<0>(a); }
extern "C" __global__ void __launch_bounds__(128) b2j_dbrfs_count_nw(b2::dev::BrfsArgs a) { b2::gen::dbrfs_count<1>(a); }
#endif
#if defined(B2J_ALL) || defined(B2J_K4)
extern "C" __global__ void __launch_bounds__(128) b2j_dbrfs_push_w(b2::dev::DExpandArgs a) { b2::gen::dbrfs_expand_push<0>(a); }
extern "C" __global__ void __launch_bounds__(128) b2j_dbrfs_push_nw(b2::dev::DExpandArgs a) { b2::gen::dbrfs_expand_push<1>(a); }
#endif
#if defined(B2J_ALL) || defined(B2J_K5)
extern "C" __global__ void b2j_env_init_w(b2::dev::EnvArgs a) { b2::gen::env_init<0>(a); }
extern "C" __global__ void b2j_env_init_nw(b2::dev::EnvArgs a) { b2::gen::env_init<1>(a); }
#endif
#if defined(B2J_ALL) || defined(B2J_K6)
extern "C" __global__ void __launch_bounds__(128) b2j_env_step_w(b2::dev::EnvArgs a) { b2::gen::env_step<0>(a); }
extern "C" __global__ void __launch_bounds__(128) b2j_env_step_nw(b2::dev::EnvArgs a) { b2::gen::env_step<1>(a); }
#endif
#if defined(B2J_ALL) || defined(B2J_K7)
extern "C" __global__ void __launch_bounds__(128) b2j_expand_count_w(b2::dev::ExpandArgs a) { b2::gen::expand_count<0>(a); }
extern "C" __global__ void __launch_bounds__(128) b2j_expand_count_nw(b2::dev::ExpandArgs a) { b2::gen::expand_count<1>(a); }
#endif
#if defined(B2J_ALL) || defined(B2J_K8)
extern "C" __global__ void __launch_bounds__(128) b2j_expand_write_w(b2::dev::ExpandArgs a) { b2::gen::expand_write<0>(a); }
extern "C" __global__ void __launch_bounds__(128) b2j_expand_write_nw(b2::dev::ExpandArgs a) { b2::gen::expand_write<1>(a); }
#endif
#if defined(B2J_ALL) || defined(B2J_K9)
extern "C" __global__ void __launch_bounds__(128) b2j_expand_hash_w(b2::dev::ExpandArgs a) { b2::gen::expand_hash<0>(a); }
extern "C" __global__ void __launch_bounds__(128) b2j_expand_hash_nw(b2::dev::ExpandArgs a) { b2::gen::expand_hash<1>(a); }
#endif
