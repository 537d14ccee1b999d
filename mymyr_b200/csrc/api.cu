// C ABI: errors, contexts, task descriptions and upload, row hashing.

#include "common.cuh"
#include "scan.cuh"
#include "jit.hpp"

#include <atomic>
#include <cstring>
#include <mutex>

namespace b2
{
namespace
{
thread_local std::string g_last_error;

/// A library-owned b2_task_desc with the pools it points into (b2_task_desc_read_text).
struct DescHolder
{
    b2_task_desc d{};
    std::vector<uint8_t> kind;
    std::vector<uint32_t> arity;
    std::vector<int32_t> terms;
    std::vector<b2_literal> literals;
    std::vector<b2_schema_desc> schemas;
    std::vector<std::string> names;
    std::vector<uint32_t> static_init, fluent_init;
};

u32 add_literal(DescHolder& h, const Lit& l)
{
    b2_literal x{};
    x.pred = l.pred;
    x.positive = l.pos ? 1 : 0;
    x.term_begin = static_cast<u32>(h.terms.size());
    x.term_count = static_cast<u32>(l.terms.size());
    h.terms.insert(h.terms.end(), l.terms.begin(), l.terms.end());
    h.literals.push_back(x);
    return static_cast<u32>(h.literals.size() - 1);
}

DescHolder* to_desc(const TaskSpec& t)
{
    auto h = std::make_unique<DescHolder>();
    h->kind = t.kind;
    h->arity = t.arity;
    for (const auto& a : t.static_init)
        h->static_init.insert(h->static_init.end(), a.begin(), a.end());
    for (const auto& a : t.fluent_init)
        h->fluent_init.insert(h->fluent_init.end(), a.begin(), a.end());
    const u32 gb = static_cast<u32>(h->literals.size());
    for (const Lit& l : t.goal)
        add_literal(*h, l);
    h->d.goal_begin = gb;
    h->d.goal_count = static_cast<u32>(t.goal.size());
    h->names.reserve(t.schemas.size());
    for (const Schema& s : t.schemas)
    {
        b2_schema_desc sd{};
        sd.arity = s.arity;
        sd.pre_begin = static_cast<u32>(h->literals.size());
        for (const Lit& l : s.pre)
            add_literal(*h, l);
        sd.pre_count = static_cast<u32>(s.pre.size());
        sd.eff_begin = static_cast<u32>(h->literals.size());
        for (const Lit& l : s.eff)
            add_literal(*h, l);
        sd.eff_count = static_cast<u32>(s.eff.size());
        h->names.push_back(s.name);
        h->schemas.push_back(sd);
    }
    for (std::size_t i = 0; i < h->schemas.size(); ++i)
        h->schemas[i].name = h->names[i].c_str();
    h->d.num_objects = t.n;
    h->d.num_predicates = static_cast<u32>(t.kind.size());
    h->d.pred_kind = h->kind.data();
    h->d.pred_arity = h->arity.data();
    h->d.terms = h->terms.data();
    h->d.num_terms = static_cast<u32>(h->terms.size());
    h->d.literals = h->literals.data();
    h->d.num_literals = static_cast<u32>(h->literals.size());
    h->d.schemas = h->schemas.data();
    h->d.num_schemas = static_cast<u32>(h->schemas.size());
    h->d.static_init = h->static_init.data();
    h->d.static_init_words = h->static_init.size();
    h->d.fluent_init = h->fluent_init.data();
    h->d.fluent_init_words = h->fluent_init.size();
    h->d.unsupported = t.unsupported.empty() ? 0 : 1;
    return h.release();
}

TaskSpec from_desc(const b2_task_desc& d)
{
    if (d.unsupported)
        throw Error(B2_UNSUPPORTED, "the task description has features the device path does not run");
    if (!d.pred_kind || !d.pred_arity || (d.num_literals && !d.literals) || (d.num_terms && !d.terms) ||
        (d.num_schemas && !d.schemas))
        throw std::invalid_argument("b2_task_create: null pools");
    TaskSpec t;
    t.n = d.num_objects;
    t.kind.assign(d.pred_kind, d.pred_kind + d.num_predicates);
    t.arity.assign(d.pred_arity, d.pred_arity + d.num_predicates);
    for (u32 p = 0; p < d.num_predicates; ++p)
    {
        t.pred_names.push_back("p" + std::to_string(p));
        if (t.kind[p] == kDerived)
            throw Error(B2_UNSUPPORTED, "derived predicates are not supported by the device path");
        if (t.kind[p] > kDerived)
            throw std::invalid_argument("b2_task_create: bad predicate kind");
    }
    auto lit = [&](u32 i, u32 params, bool ground) {
        if (i >= d.num_literals)
            throw std::invalid_argument("b2_task_create: literal index out of range");
        const b2_literal& x = d.literals[i];
        if (x.pred >= d.num_predicates || x.term_count != t.arity[x.pred] ||
            static_cast<u64>(x.term_begin) + x.term_count > d.num_terms)
            throw std::invalid_argument("b2_task_create: malformed literal");
        Lit l;
        l.pred = x.pred;
        l.pos = x.positive != 0;
        for (u32 j = 0; j < x.term_count; ++j)
        {
            const i32 term = d.terms[x.term_begin + j];
            if (term >= 0 && (ground || static_cast<u32>(term) >= params))
                throw std::invalid_argument("b2_task_create: parameter term out of range");
            if (term < 0 && static_cast<u32>(-(static_cast<long long>(term) + 1)) >= d.num_objects)
                throw std::invalid_argument("b2_task_create: object term out of range");
            l.terms.push_back(term);
        }
        return l;
    };
    auto atoms = [&](const uint32_t* w, u64 n, std::vector<std::vector<u32>>& out) {
        for (u64 i = 0; i < n;)
        {
            const u32 p = w[i];
            if (p >= d.num_predicates || i + 1 + t.arity[p] > n)
                throw std::invalid_argument("b2_task_create: malformed atom records");
            std::vector<u32> rec(w + i, w + i + 1 + t.arity[p]);
            for (u32 j = 1; j < rec.size(); ++j)
                if (rec[j] >= d.num_objects)
                    throw std::invalid_argument("b2_task_create: atom object out of range");
            out.push_back(std::move(rec));
            i += 1 + t.arity[p];
        }
    };
    atoms(d.static_init, d.static_init_words, t.static_init);
    atoms(d.fluent_init, d.fluent_init_words, t.fluent_init);
    for (u32 i = 0; i < d.goal_count; ++i)
        t.goal.push_back(lit(d.goal_begin + i, 0, true));
    for (u32 s = 0; s < d.num_schemas; ++s)
    {
        const b2_schema_desc& sd = d.schemas[s];
        Schema sc;
        sc.name = sd.name ? sd.name : "s" + std::to_string(s);
        sc.arity = sd.arity;
        for (u32 i = 0; i < sd.pre_count; ++i)
            sc.pre.push_back(lit(sd.pre_begin + i, sd.arity, false));
        for (u32 i = 0; i < sd.eff_count; ++i)
            sc.eff.push_back(lit(sd.eff_begin + i, sd.arity, false));
        t.schemas.push_back(std::move(sc));
    }
    return t;
}

/// Copies every program pool into one device blob and fills the pointer view.
void upload(b2_task& t)
{
    const Program& P = t.prog;
    std::vector<char> host;
    auto put = [&](const void* src, size_t bytes) -> size_t {
        const size_t at = (host.size() + 255) & ~size_t{255};
        host.resize(at + bytes + 8);
        if (bytes)
            std::memcpy(host.data() + at, src, bytes);
        return at;
    };
    const size_t o_pool = put(P.pool.data(), P.pool.size() * 8);
    const size_t o_lits = put(P.lits.data(), P.lits.size() * sizeof(DLit));
    const size_t o_vars = put(P.vars.data(), P.vars.size() * sizeof(DVar));
    const size_t o_filt = put(P.filters.data(), P.filters.size() * sizeof(DFilter));
    const size_t o_lev = put(P.levels.data(), P.levels.size() * sizeof(DLevel));
    const size_t o_chk = put(P.checks.data(), P.checks.size() * 4);
    const size_t o_sch = put(P.schemas.data(), P.schemas.size() * sizeof(DSchema));
    const size_t o_dom = put(P.domain.data(), P.domain.size() * 4);
    const size_t o_pdb = put(P.pos_dom_begin.data(), P.pos_dom_begin.size() * 4);
    const size_t o_srt = put(P.srel_table.data(), P.srel_table.size() * 8);
    const size_t o_srm = put(P.srel_mask.data(), P.srel_mask.size() * 8);
    const size_t o_srp = put(P.srel_probes.data(), P.srel_probes.size() * 8);
    const size_t o_gp = put(P.goal_pos.data(), P.goal_pos.size() * 8);
    const size_t o_gn = put(P.goal_neg.data(), P.goal_neg.size() * 8);
    t.blob.alloc(host.size());
    B2_CUDA(cudaMemcpy(t.blob.p, host.data(), host.size(), cudaMemcpyHostToDevice));
    char* b = t.blob.as<char>();
    DevTask& D = t.dev;
    D.n = P.n;
    D.ow = P.ow;
    D.words = P.words;
    D.nschemas = P.nschemas;
    D.label_width = P.label_width;
    D.goal_unsat = P.goal_unsat;
    D.fluent_count = P.fluent_count;
    D.pool = reinterpret_cast<const u64*>(b + o_pool);
    D.lits = reinterpret_cast<const DLit*>(b + o_lits);
    D.vars = reinterpret_cast<const DVar*>(b + o_vars);
    D.filters = reinterpret_cast<const DFilter*>(b + o_filt);
    D.levels = reinterpret_cast<const DLevel*>(b + o_lev);
    D.checks = reinterpret_cast<const u32*>(b + o_chk);
    D.schemas = reinterpret_cast<const DSchema*>(b + o_sch);
    D.domain = reinterpret_cast<const u32*>(b + o_dom);
    D.pos_dom_begin = reinterpret_cast<const u32*>(b + o_pdb);
    D.srel_table = reinterpret_cast<const u64*>(b + o_srt);
    D.srel_mask = reinterpret_cast<const u64*>(b + o_srm);
    D.srel_probes = reinterpret_cast<const u64*>(b + o_srp);
    D.goal_pos = reinterpret_cast<const u64*>(b + o_gp);
    D.goal_neg = reinterpret_cast<const u64*>(b + o_gn);
}

/// hash::state of rows [atom words | nnum numeric words] (W words in all): the trimmed atom words, seeded by the
/// numeric words' hash when there are any.
__global__ void k_hash_rows(const u64* __restrict__ rows, u64 n, u32 W, u32 nnum, u64* __restrict__ out)
{
    for (u64 i = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; i < n; i += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64* r = rows + i * W;
        const u32 na = W - nnum;
        const u64 seed = nnum ? dev::hash_span([&](u32 k) { return __ldg(r + na + k); }, nnum) : dev::kHashSeed;
        out[i] = hash_words([&](u32 k) { return __ldg(r + k); }, na, seed);
    }
}
}  // namespace

void set_last_error(const std::string& m) { g_last_error = m; }

void check_status_word(const u32* dev_status, cudaStream_t s, const char* what)
{
    u32 st = 0;
    B2_CUDA(cudaMemcpyAsync(&st, dev_status, 4, cudaMemcpyDeviceToHost, s));
    B2_CUDA(cudaStreamSynchronize(s));
    if (st & kStatusProbeLimit)
        throw Error(B2_DEVICE_FAULT, std::string(what) + ": a hash-set probe ran past its bound");
    if (st & kStatusEffectOverflow)
        throw Error(B2_UNSUPPORTED, std::string(what) + ": an action with more than 16 adds or deletes");
    if (st)
        throw Error(B2_DEVICE_FAULT, std::string(what) + ": device status " + std::to_string(st));
}
}  // namespace b2

using namespace b2;

extern "C" {

size_t b2_last_error(char* buf, size_t cap)
{
    const std::string& e = g_last_error;
    if (buf && cap)
    {
        const size_t n = e.size() < cap - 1 ? e.size() : cap - 1;
        std::memcpy(buf, e.data(), n);
        buf[n] = 0;
    }
    return e.size();
}

const char* b2_version(void) { return "mymyr_b200 0.1 (sm_100a)"; }

b2_status b2_ctx_create(int device, b2_ctx** out)
{
    return guarded([&] {
        if (!out)
            throw std::invalid_argument("b2_ctx_create: null output");
        int count = 0;
        B2_CUDA(cudaGetDeviceCount(&count));
        if (device < 0 || device >= count)
            throw std::invalid_argument("b2_ctx_create: no device " + std::to_string(device));
        auto c = std::make_unique<b2_ctx>();
        c->device = device;
        B2_CUDA(cudaSetDevice(device));
        B2_CUDA(cudaGetDeviceProperties(&c->prop, device));
        if (c->prop.major < 10)
            throw Error(B2_UNSUPPORTED, "mymyr_b200 is built for sm_100a (B200); device " + std::to_string(device) +
                                            " is sm_" + std::to_string(c->prop.major * 10 + c->prop.minor));
        c->sms = c->prop.multiProcessorCount;
        // keep the device pool's memory between stream-ordered frees (searches allocate and free gigabytes)
        cudaMemPool_t pool;
        B2_CUDA(cudaDeviceGetDefaultMemPool(&pool, device));
        uint64_t keep = ~uint64_t{0};
        B2_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
        noalloc_prepare(*c);
        c->noalloc_host = c->pinned.take();
        *out = c.release();
    });
}

void b2_ctx_destroy(b2_ctx* ctx)
{
    if (!ctx)
        return;
    cudaSetDevice(ctx->device);  // the kept buffers are freed on this device
    ctx->pinned.give(ctx->noalloc_host);  // freed with the pool
    ctx->noalloc_host = nullptr;
    delete ctx;
}

b2_status b2_task_desc_read_text(const char* text, size_t len, b2_task_desc** out)
{
    const b2_status s = guarded([&] {
        if (!text || !out)
            throw std::invalid_argument("b2_task_desc_read_text: null argument");
        *out = &to_desc(read_task_text(std::string(text, len)))->d;
    });
    if (s == B2_INVALID_ARGUMENT && g_last_error.rfind("task text:", 0) == 0)
        return B2_PARSE_ERROR;
    return s;
}

void b2_task_desc_free(b2_task_desc* desc) { delete reinterpret_cast<DescHolder*>(desc); }

b2_status b2_task_create(b2_ctx* ctx, const b2_task_desc* desc, b2_task** out)
{
    return b2_task_create_ex(ctx, desc, nullptr, out);
}

b2_status b2_task_create_ex(b2_ctx* ctx, const b2_task_desc* desc, const b2_task_options* options, b2_task** out)
{
    return guarded([&] {
        if (!desc || !out)
            throw std::invalid_argument("b2_task_create: null argument");
        const int32_t matcher = options ? options->matcher : B2_MATCHER_AUTO;
        if (matcher < B2_MATCHER_AUTO || matcher > B2_MATCHER_COMPILED)
            throw std::invalid_argument("b2_task_create: bad matcher option");
        if (ctx)
            B2_CUDA(cudaSetDevice(ctx->device));
        auto t = std::make_unique<b2_task>();
        t->ctx = ctx;
        t->spec = from_desc(*desc);
        try
        {
            compile_task(t->spec, t->layout, t->statics, t->prog);
        }
        catch (const std::invalid_argument& e)
        {
            throw Error(B2_UNSUPPORTED, e.what());
        }
        for (const DSchema& s : t->prog.schemas)
            if (s.prog[0].never == 0xFFFFFFFFu)
                t->witness_refused = true;
        for (const DSchema& s : t->prog.schemas)
            if (s.add_end - s.add_begin > 16 || s.del_end - s.del_begin > 16)
                throw Error(B2_UNSUPPORTED, "an action schema with more than 16 add or delete effects");
        if (ctx)
        {
            upload(*t);  // a host-only task (ctx NULL) is compiled but cannot run kernels
            if (matcher != B2_MATCHER_INTERPRETED)
                t->jit = jit_module(ctx->device, t->prog);
        }
        *out = t.release();
    });
}

b2_status b2_task_compile(const b2_task* task, char* src, size_t src_cap, size_t* src_len)
{
    return guarded([&] {
        if (!task)
            throw std::invalid_argument("b2_task_compile: null task");
        const std::string text = generate_matcher_source(task->prog);
        jit_cubin(task->prog);
        if (src && src_cap)
        {
            const size_t n = text.size() < src_cap - 1 ? text.size() : src_cap - 1;
            std::memcpy(src, text.data(), n);
            src[n] = 0;
        }
        if (src_len)
            *src_len = text.size();
    });
}

void b2_task_destroy(b2_task* task) { delete task; }

b2_status b2_task_info_get(const b2_task* task, b2_task_info* out)
{
    return guarded([&] {
        if (!task || !out)
            throw std::invalid_argument("b2_task_info_get: null argument");
        out->words = task->prog.words;
        out->fluent_slots = static_cast<uint32_t>(task->prog.fluent_count);
        out->num_schemas = task->prog.nschemas;
        out->num_objects = task->prog.n;
        out->label_width = task->prog.label_width;
        out->object_words = task->prog.ow;
    });
}

b2_status b2_task_initial_state(const b2_task* task, uint64_t* row, uint32_t words)
{
    return guarded([&] {
        if (!task || !row)
            throw std::invalid_argument("b2_task_initial_state: null argument");
        if (words < task->prog.words)
            throw std::invalid_argument("b2_task_initial_state: row narrower than the task's words");
        std::memset(row, 0, words * sizeof(uint64_t));
        std::memcpy(row, task->prog.initial.data(), task->prog.words * sizeof(uint64_t));
    });
}

b2_status b2_task_slot_atom(const b2_task* task, uint32_t slot, uint32_t* pred_args, uint32_t cap)
{
    return guarded([&] {
        if (!task || !pred_args)
            throw std::invalid_argument("b2_task_slot_atom: null argument");
        if (slot >= task->prog.slot_atoms.size())
            throw std::invalid_argument("b2_task_slot_atom: slot out of range");
        const auto& rec = task->prog.slot_atoms[slot];
        if (rec.size() > cap)
            throw std::length_error("b2_task_slot_atom: buffer too small");
        std::memcpy(pred_args, rec.data(), rec.size() * 4);
    });
}

b2_status b2_hash_rows_numeric(b2_ctx* ctx, const uint64_t* rows, uint64_t n, uint32_t words, uint32_t numeric_words,
                               uint64_t* out, void* stream)
{
    return guarded([&] {
        if (!ctx || (n && (!rows || !out)) || words == 0)
            throw std::invalid_argument("b2_hash_rows: bad argument");
        if (numeric_words > words)
            throw std::invalid_argument("b2_hash_rows: numeric_words exceeds the row width");
        if (!n)
            return;
        B2_CUDA(cudaSetDevice(ctx->device));
        const unsigned grid = grid_for(n, 256, static_cast<unsigned>(ctx->sms) * 16);
        k_hash_rows<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(rows, n, words, numeric_words, out);
        B2_CUDA(cudaGetLastError());
    });
}

b2_status b2_hash_rows(b2_ctx* ctx, const uint64_t* rows, uint64_t n, uint32_t words, uint64_t* out, void* stream)
{
    return b2_hash_rows_numeric(ctx, rows, n, words, 0, out, stream);
}

}  // extern "C"

namespace b2
{
unsigned scan_blocks(u64 nb)
{
    // SM count of the calling thread's current device, read once per device
    static std::atomic<int> sms[64];
    int dev = 0;
    B2_CUDA(cudaGetDevice(&dev));
    int n = dev < 64 ? sms[dev].load(std::memory_order_relaxed) : 0;
    if (n == 0)
    {
        B2_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
        if (dev < 64)
            sms[dev].store(n, std::memory_order_relaxed);
    }
    const u64 cap = static_cast<u64>(n) * 8;
    return static_cast<unsigned>(nb < cap ? nb : cap);
}
}  // namespace b2

namespace b2
{
__global__ void __launch_bounds__(1024) k_scan_sums(u64* __restrict__ sums, u64 n_in, const u64* n_dev,
                                                    u64* __restrict__ total)
{
    using Scan = cub::BlockScan<u64, 1024>;
    __shared__ typename Scan::TempStorage tmp;
    __shared__ u64 carry;
    const u64 n = scan_count(n_in, n_dev);
    const u64 nb = (n + kScanTile - 1) / kScanTile;
    if (threadIdx.x == 0)
        carry = 0;
    __syncthreads();
    for (u64 base = 0; base < nb; base += 1024)
    {
        const u64 i = base + threadIdx.x;
        const u64 v = i < nb ? sums[i] : 0;
        u64 e, agg;
        Scan(tmp).ExclusiveSum(v, e, agg);
        const u64 c = carry;
        if (i < nb)
            sums[i] = c + e;
        __syncthreads();
        if (threadIdx.x == 0)
            carry = c + agg;
        __syncthreads();
    }
    if (threadIdx.x == 0)
        *total = carry;
}
}  // namespace b2
