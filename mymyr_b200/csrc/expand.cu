// Batched expand (rl::expand, include/mymyr/rl/expand.hpp:137-147, on the device): the successors of a batch of
// states as CSR in canonical order. One thread per (state, schema) segment: a count pass, a scan of the segment
// counts (segment order = (state, schema) = canonical order), and a write pass that regenerates each segment at its
// offset and writes labels, successor hashes (hash::state of the successor, bit-exact) and, optionally, rows.

#include "scan.cuh"

#include <mutex>

namespace b2
{
namespace
{
struct SegCountIn
{
    const u32* c;
    __device__ __forceinline__ u32 operator()(u64 i) const { return c[i]; }
};
struct SegCountOut
{
    u64* off;
    __device__ __forceinline__ void operator()(u64 i, u64 e, u32) const { off[i] = e; }
};

template<int OW, int WR>
__global__ void __launch_bounds__(128) k_expand_count(DevTask T, const u64* __restrict__ states, u64 rows, u32 W,
                                                      u32 pi, u32* __restrict__ counts)
{
    const u64 nseg = rows * T.nschemas;
    for (u64 q = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; q < nseg; q += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 r = q / T.nschemas;
        const u32 s = static_cast<u32>(q - r * T.nschemas);
        const auto st = load_row<WR>(states + r * W, W);
        u32 bind[kMaxLevels] = {};
        u32 c = 0;
        enumerate<OW>(T, T.schemas[s].prog[pi], st, bind, [&](const u32*) {
            ++c;
            return true;
        });
        counts[q] = c;
    }
}

template<int OW, int WR>
__global__ void __launch_bounds__(128) k_expand_write(DevTask T, const u64* __restrict__ states, u64 rows, u32 W,
                                                      u32 pi, const u64* __restrict__ seg_off, b2_expansion out,
                                                      u32* __restrict__ status)
{
    const u64 nseg = rows * T.nschemas;
    for (u64 q = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; q < nseg; q += static_cast<u64>(gridDim.x) * blockDim.x)
    {
        const u64 r = q / T.nschemas;
        const u32 s = static_cast<u32>(q - r * T.nschemas);
        const auto st = load_row<WR>(states + r * W, W);
        const DSchema S = T.schemas[s];
        u32 bind[kMaxLevels] = {};
        u64 idx = seg_off[q];
        enumerate<OW>(T, S.prog[pi], st, bind, [&](const u32* b) {
            if (idx < out.capacity)
            {
                if (out.parent)
                    out.parent[idx] = static_cast<i32>(r);
                if (out.schema)
                    out.schema[idx] = static_cast<i32>(s);
                if (out.binding)
                    for (u32 k = 0; k < out.label_width; ++k)
                        out.binding[idx * out.label_width + k] = k < S.arity ? static_cast<i32>(b[k]) : -1;
                if (out.succ_hash || out.succ)
                {
                    Effects e;
                    collect_effects(T, S, b, e);
                    const SuccRow<decltype(st)> sr{st, e};
                    if (out.succ_hash)
                        out.succ_hash[idx] = hash_words([&](u32 i) { return sr.word(i); }, W);
                    if (out.succ)
                        for (u32 i = 0; i < out.words; ++i)
                            out.succ[idx * out.words + i] = i < W ? sr.word(i) : 0;
                }
            }
            ++idx;
            return true;
        });
    }
}

__global__ void k_offsets(const u64* __restrict__ seg_off, u64 rows, u32 nschemas, const u64* __restrict__ total,
                          i32* __restrict__ offsets)
{
    for (u64 r = blockIdx.x * static_cast<u64>(blockDim.x) + threadIdx.x; r <= rows; r += static_cast<u64>(gridDim.x) * blockDim.x)
        offsets[r] = nschemas == 0 ? 0 : static_cast<i32>(r < rows ? seg_off[r * nschemas] : *total);
}
}  // namespace
}  // namespace b2

using namespace b2;

extern "C" b2_status b2_expand(b2_task* task, const uint64_t* states, uint64_t rows, uint32_t words, int witness_pruning,
                               b2_expansion* out, void* stream)
{
    return guarded([&] {
        if (!task || !out || (rows && !states))
            throw std::invalid_argument("b2_expand: null argument");
        if (!task->ctx)
            throw std::invalid_argument("a host-only task (created without a context) cannot run on the device");
        const Program& P = task->prog;
        if (words != P.words)
            throw std::invalid_argument("b2_expand: rows of " + std::to_string(words) + " words; the task has " +
                                        std::to_string(P.words));
        if (out->binding && out->label_width < P.label_width)
            throw std::invalid_argument("b2_expand: label width below the largest schema arity");
        if (out->succ && out->words < P.words)
            throw std::invalid_argument("b2_expand: successor rows narrower than the task's words");
        if (rows > (u64{1} << 31) - 1)
            throw std::invalid_argument("b2_expand: more than 2^31 - 1 states");
        if (witness_pruning && task->witness_refused)
            throw Error(B2_UNSUPPORTED, "witness pruning with a witness parameter before an effect parameter");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        b2_ctx* ctx = task->ctx;
        B2_CUDA(cudaSetDevice(ctx->device));
        const u64 nseg = rows * P.nschemas;
        // scratch: counts [nseg] u32, offsets [nseg] u64, total u64, scan sums
        const size_t b_counts = ((nseg * 4 + 255) / 256) * 256, b_off = ((nseg * 8 + 255) / 256) * 256;
        const size_t need = b_counts + b_off + 256 + scan_scratch_bytes(nseg) + 256;
        if (ctx->scratch.bytes < need)
        {
            B2_CUDA(cudaStreamSynchronize(s));
            ctx->scratch.alloc(need);
        }
        char* base = ctx->scratch.as<char>();
        u32* counts = reinterpret_cast<u32*>(base);
        u64* seg_off = reinterpret_cast<u64*>(base + b_counts);
        u64* total = reinterpret_cast<u64*>(base + b_counts + b_off);
        u64* sums = reinterpret_cast<u64*>(base + b_counts + b_off + 256);
        u32* status = reinterpret_cast<u32*>(base + b_counts + b_off + 8);
        B2_CUDA(cudaMemsetAsync(status, 0, 4, s));
        const u32 pi = witness_pruning ? 0 : 1;
        const unsigned grid = grid_for(nseg, 128, static_cast<unsigned>(ctx->sms) * 64);
        const unsigned grid_rows = grid_for(rows, 128, static_cast<unsigned>(ctx->sms) * 64);  // compiled: a thread per state
        dev::ExpandArgs a{};
        a.states = states;
        a.rows = rows;
        a.W = words;
        a.pi = pi;
        a.counts = counts;
        a.seg_off = seg_off;
        a.capacity = out->capacity;
        a.out_words = out->words;
        a.label_width = out->label_width;
        a.succ = out->succ;
        a.parent = out->parent;
        a.schema = out->schema;
        a.binding = out->binding;
        a.succ_hash = out->succ_hash;
        a.status = status;
        a.total = total;
        // the compiled path hashes the successors in a pass of its own when the records it reads are written
        a.hash_pass = task->jit && (out->succ_hash || out->succ) && out->parent && out->schema && out->binding ? 1 : 0;
        if (nseg && task->jit)
            jit_launch(task->jit->get(kJitExpandCount, pi), grid_rows, 128, &a, s);
        else if (nseg)
            dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                k_expand_count<OW, WR><<<grid, 128, 0, s>>>(task->dev, states, rows, words, pi, counts);
            });
        device_scan(SegCountIn{counts}, SegCountOut{seg_off}, nseg, total, sums, s, status);
        if (nseg && task->jit)
            jit_launch(task->jit->get(kJitExpandWrite, pi), grid_rows, 128, &a, s);
        if (nseg && a.hash_pass)
            jit_launch(task->jit->get(kJitExpandHash, pi), static_cast<unsigned>(ctx->sms) * 16, 128, &a, s);
        else if (nseg)
            dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                k_expand_write<OW, WR><<<grid, 128, 0, s>>>(task->dev, states, rows, words, pi, seg_off, *out, status);
            });
        if (out->offsets)
            k_offsets<<<grid_for(rows + 1, 256), 256, 0, s>>>(seg_off, rows, P.nschemas, total, out->offsets);
        B2_CUDA(cudaGetLastError());
        u64 gen = 0;
        B2_CUDA(cudaMemcpyAsync(&gen, total, 8, cudaMemcpyDeviceToHost, s));
        B2_CUDA(cudaStreamSynchronize(s));
        out->generated = gen;
        check_status_word(status, s, "b2_expand");
        if (gen > out->capacity && (out->succ || out->parent || out->schema || out->binding || out->succ_hash))
            throw Error(B2_CAPACITY, "b2_expand: " + std::to_string(gen) + " successors exceed the capacity of " +
                                         std::to_string(out->capacity));
        if (gen > (u64{1} << 31) - 1)
            throw Error(B2_CAPACITY, "b2_expand: more than 2^31 - 1 successors");
    });
}

// ------------------------------------------------------------------------------------------------ b2_expand_noalloc
// The batched expand without any allocation, for callers that cannot allocate device memory while they run: a
// process that reserves the GPU's memory up front through its own allocator (a training or serving framework's caching
// allocator, or a fixed per-process budget) and forbids other allocations, or a latency-bound caller for which the
// device-wide synchronization of cudaMalloc/cudaFree is unacceptable. Its scratch (per-segment counts and offsets, the
// scan's block sums, the total and a status word) lives in a file-scope __device__ array of kNoAllocScratchBytes
// that every GPU loading this library holds until the process exits.
//
// Everything that needs memory is set up before the first call: b2_ctx_create (noalloc_prepare) loads this file's
// module on the device, which places the array in device memory, loads the kernels the call launches and records the
// array's device address (cudaGetSymbolAddress, with the device current: the array's host-side name is not a device
// address); it also takes the pinned word pair the call reads its results into. The task's compiled kernels are loaded
// by b2_task_create.

namespace b2
{
namespace
{
/// Segments ((state, schema) pairs) a b2_expand_noalloc call may have.
constexpr u64 kNoAllocMaxSegments = u64{1} << 18;
constexpr size_t kNoAllocCounts = kNoAllocMaxSegments * 4;
constexpr size_t kNoAllocOffsets = kNoAllocMaxSegments * 8;
constexpr size_t kNoAllocSums = scan_scratch_bytes(kNoAllocMaxSegments);
constexpr size_t kNoAllocScratchBytes = kNoAllocCounts + kNoAllocOffsets + 256 + kNoAllocSums;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

/// One b2_expand_noalloc call at a time in this process: the calls share the scratch array (and each context's pinned
/// result words), and each returns only after its stream has finished, so taking turns keeps them from overlapping.
std::mutex g_noalloc_mu;

template<class K>
void load_kernel(K* k)
{
    cudaFuncAttributes attr{};
    B2_CUDA(cudaFuncGetAttributes(&attr, reinterpret_cast<const void*>(k)));
}
}  // namespace

void noalloc_prepare(b2_ctx& ctx)
{
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
        throw Error(B2_CUDA_ERROR, std::string("b2_expand_noalloc set-up: cudaGetSymbolAddress: ") +
                                       cudaGetErrorString(e));
    ctx.noalloc_scratch = p;
    // the kernels of the call, loaded now (lazy module loading would otherwise load them at its first launch)
    load_kernel(k_offsets);
    load_kernel(k_tile_reduce<SegCountIn>);
    load_kernel(k_scan_sums);
    load_kernel(k_tile_apply<SegCountIn, SegCountOut>);
    for (u32 ow = 1; ow <= 4; ++ow)
        for (u32 words : {1u, 2u, 4u, 8u, 9u})
            dispatch_shapes(ow, words, [&]<int OW, int WR>() {
                load_kernel(k_expand_count<OW, WR>);
                load_kernel(k_expand_write<OW, WR>);
            });
}
}  // namespace b2

extern "C" b2_status b2_expand_noalloc(b2_task* task, const uint64_t* states, uint64_t rows, uint32_t words,
                                       int witness_pruning, b2_expansion* out, void* stream)
{
    return guarded([&] {
        if (!task || !out || (rows && !states))
            throw std::invalid_argument("b2_expand_noalloc: null argument");
        if (!task->ctx)
            throw std::invalid_argument("a host-only task (created without a context) cannot run on the device");
        const Program& P = task->prog;
        if (words != P.words)
            throw std::invalid_argument("b2_expand_noalloc: rows of " + std::to_string(words) + " words; the task has " +
                                        std::to_string(P.words));
        if (out->binding && out->label_width < P.label_width)
            throw std::invalid_argument("b2_expand_noalloc: label width below the largest schema arity");
        if (out->succ && out->words < P.words)
            throw std::invalid_argument("b2_expand_noalloc: successor rows narrower than the task's words");
        if (rows > (u64{1} << 31) - 1)
            throw std::invalid_argument("b2_expand_noalloc: more than 2^31 - 1 states");
        if (witness_pruning && task->witness_refused)
            throw Error(B2_UNSUPPORTED, "witness pruning with a witness parameter before an effect parameter");
        const u64 nseg = rows * P.nschemas;
        if (P.nschemas && rows > kNoAllocMaxSegments / P.nschemas)
            throw Error(B2_CAPACITY, "b2_expand_noalloc: " + std::to_string(rows) + " states x " +
                                         std::to_string(P.nschemas) + " schemas exceed its fixed scratch of " +
                                         std::to_string(kNoAllocMaxSegments) +
                                         " (state, schema) segments; use b2_expand or smaller batches");
        b2_ctx* ctx = task->ctx;
        if (!ctx->noalloc_scratch || !ctx->noalloc_host)
            throw Error(B2_CUDA_ERROR, "b2_expand_noalloc: the context was not set up for it");
        std::lock_guard lock(g_noalloc_mu);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        B2_CUDA(cudaSetDevice(ctx->device));
        char* base = static_cast<char*>(ctx->noalloc_scratch);
        u32* counts = reinterpret_cast<u32*>(base);
        u64* seg_off = reinterpret_cast<u64*>(base + kNoAllocCounts);
        u64* total = reinterpret_cast<u64*>(base + kNoAllocCounts + kNoAllocOffsets);
        u32* status = reinterpret_cast<u32*>(base + kNoAllocCounts + kNoAllocOffsets + 8);
        u64* sums = reinterpret_cast<u64*>(base + kNoAllocCounts + kNoAllocOffsets + 256);
        // the array keeps the last call's contents: the status word and the total start at zero
        B2_CUDA(cudaMemsetAsync(total, 0, 16, s));
        const u32 pi = witness_pruning ? 0 : 1;
        const unsigned grid = grid_for(nseg, 128, static_cast<unsigned>(ctx->sms) * 64);
        const unsigned grid_rows = grid_for(rows, 128, static_cast<unsigned>(ctx->sms) * 64);  // compiled: a thread per state
        dev::ExpandArgs a{};
        a.states = states;
        a.rows = rows;
        a.W = words;
        a.pi = pi;
        a.counts = counts;
        a.seg_off = seg_off;
        a.capacity = out->capacity;
        a.out_words = out->words;
        a.label_width = out->label_width;
        a.succ = out->succ;
        a.parent = out->parent;
        a.schema = out->schema;
        a.binding = out->binding;
        a.succ_hash = out->succ_hash;
        a.status = status;
        a.total = total;
        // the compiled path hashes the successors in a pass of its own when the records it reads are written
        a.hash_pass = task->jit && (out->succ_hash || out->succ) && out->parent && out->schema && out->binding ? 1 : 0;
        if (nseg && task->jit)
            jit_launch(task->jit->get(kJitExpandCount, pi), grid_rows, 128, &a, s);
        else if (nseg)
            dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                k_expand_count<OW, WR><<<grid, 128, 0, s>>>(task->dev, states, rows, words, pi, counts);
            });
        if (nseg)
            device_scan(SegCountIn{counts}, SegCountOut{seg_off}, nseg, total, sums, s, status);
        if (nseg && task->jit)
            jit_launch(task->jit->get(kJitExpandWrite, pi), grid_rows, 128, &a, s);
        if (nseg && a.hash_pass)
            jit_launch(task->jit->get(kJitExpandHash, pi), static_cast<unsigned>(ctx->sms) * 16, 128, &a, s);
        else if (nseg)
            dispatch_shapes(P.ow, P.words, [&]<int OW, int WR>() {
                k_expand_write<OW, WR><<<grid, 128, 0, s>>>(task->dev, states, rows, words, pi, seg_off, *out, status);
            });
        if (out->offsets)
            k_offsets<<<grid_for(rows + 1, 256), 256, 0, s>>>(seg_off, rows, P.nschemas, total, out->offsets);
        B2_CUDA(cudaGetLastError());
        // total (u64) and status (u32) sit next to each other: one copy into the context's pinned words
        u64* host = static_cast<u64*>(ctx->noalloc_host);
        B2_CUDA(cudaMemcpyAsync(host, total, 16, cudaMemcpyDeviceToHost, s));
        B2_CUDA(cudaStreamSynchronize(s));
        const u64 gen = host[0];
        const u32 st = static_cast<u32>(host[1]);
        out->generated = gen;
        if (st)
            throw Error(B2_DEVICE_FAULT, "b2_expand_noalloc: device status " + std::to_string(st));
        if (gen > out->capacity && (out->succ || out->parent || out->schema || out->binding || out->succ_hash))
            throw Error(B2_CAPACITY, "b2_expand_noalloc: " + std::to_string(gen) +
                                         " successors exceed the capacity of " + std::to_string(out->capacity));
        if (gen > (u64{1} << 31) - 1)
            throw Error(B2_CAPACITY, "b2_expand_noalloc: more than 2^31 - 1 successors");
    });
}
