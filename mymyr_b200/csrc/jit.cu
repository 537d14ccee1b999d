// Run-time compilation of a task's kernels: the generated matcher (codegen.cpp) plus jit_kernels.cuh, compiled by
// NVRTC (loaded with dlopen on first use) to sm_100a cubins, loaded with the runtime's library API
// (cudaLibraryLoadData) and launched with cudaLaunchKernel. Every kernel pair (witness pruning on, off) is its own
// compile unit, compiled when first used: a task with a large matcher pays only for the kernels its calls launch.
// Cubins are cached per process by (source digest, kernel), modules per (device, digest): tasks with the same
// compiled program share them. Compiling needs no GPU.

#include "common.cuh"
#include "jit.hpp"

#include <nvrtc.h>

#include <dlfcn.h>

#include <map>
#include <mutex>

extern "C" const char b2_jit_core_source[];
extern "C" const char b2_jit_kernels_source[];

namespace b2
{
namespace
{
std::mutex g_mu;
std::map<std::pair<u64, u32>, std::shared_ptr<std::vector<char>>> g_cubins;  // (digest, kernel) -> cubin
std::map<std::pair<int, u64>, std::shared_ptr<JitModule>> g_modules;  // (device, digest) -> module

u64 digest(const std::string& s)
{
    u64 h = 0xcbf29ce484222325ull;  // FNV-1a, then the splitmix finalizer
    for (unsigned char c : s)
        h = (h ^ c) * 0x100000001b3ull;
    h ^= h >> 30;
    h *= 0xbf58476d1ce4e5b9ULL;
    h ^= h >> 27;
    return h ^ (static_cast<u64>(s.size()) << 1);
}

/// NVRTC, loaded on first use (the library itself does not link it, so it loads where NVRTC is absent).
struct Nvrtc
{
    decltype(&::nvrtcCreateProgram) create = nullptr;
    decltype(&::nvrtcCompileProgram) compile = nullptr;
    decltype(&::nvrtcGetProgramLogSize) log_size = nullptr;
    decltype(&::nvrtcGetProgramLog) log = nullptr;
    decltype(&::nvrtcGetCUBINSize) cubin_size = nullptr;
    decltype(&::nvrtcGetCUBIN) cubin = nullptr;
    decltype(&::nvrtcDestroyProgram) destroy = nullptr;
    decltype(&::nvrtcGetErrorString) error = nullptr;
};

const Nvrtc& nvrtc()
{
    static Nvrtc api = [] {
        Nvrtc a;
        void* h = nullptr;
        for (const char* name : {"libnvrtc.so.12", "/usr/local/cuda/lib64/libnvrtc.so.12", "libnvrtc.so"})
            if ((h = dlopen(name, RTLD_NOW | RTLD_LOCAL)))
                break;
        if (!h)
            return a;
        a.create = reinterpret_cast<decltype(a.create)>(dlsym(h, "nvrtcCreateProgram"));
        a.compile = reinterpret_cast<decltype(a.compile)>(dlsym(h, "nvrtcCompileProgram"));
        a.log_size = reinterpret_cast<decltype(a.log_size)>(dlsym(h, "nvrtcGetProgramLogSize"));
        a.log = reinterpret_cast<decltype(a.log)>(dlsym(h, "nvrtcGetProgramLog"));
        a.cubin_size = reinterpret_cast<decltype(a.cubin_size)>(dlsym(h, "nvrtcGetCUBINSize"));
        a.cubin = reinterpret_cast<decltype(a.cubin)>(dlsym(h, "nvrtcGetCUBIN"));
        a.destroy = reinterpret_cast<decltype(a.destroy)>(dlsym(h, "nvrtcDestroyProgram"));
        a.error = reinterpret_cast<decltype(a.error)>(dlsym(h, "nvrtcGetErrorString"));
        return a;
    }();
    if (!api.create || !api.compile || !api.cubin || !api.error)
        throw Error(B2_CUDA_ERROR, "mymyr_b200: NVRTC (libnvrtc.so.12) is not available to compile the task's kernels");
    return api;
}

#define B2_NVRTC(call)                                                                                             \
    do                                                                                                             \
    {                                                                                                              \
        const nvrtcResult r_ = (call);                                                                             \
        if (r_ != NVRTC_SUCCESS)                                                                                   \
            throw Error(B2_CUDA_ERROR, std::string(#call) + ": " + N.error(r_));                                  \
    } while (0)

/// Compiles the kernel pair `which` of the source (kJitKernels: all of them).
std::shared_ptr<std::vector<char>> compile(const std::string& src, u32 which, std::string& log)
{
    const Nvrtc& N = nvrtc();
    nvrtcProgram prog;
    const char* headers[] = {b2_jit_core_source, b2_jit_kernels_source};
    const char* names[] = {"b2_core.cuh", "b2_jit_kernels.cuh"};
    B2_NVRTC(N.create(&prog, src.c_str(), "b2_task.cu", 2, headers, names));
    const std::string select = which == kJitKernels ? "-DB2J_ALL" : "-DB2J_K" + std::to_string(which);
    const char* opts[] = {"-arch=sm_100a", "-std=c++20", "-lineinfo", "-DNDEBUG", "-default-device", select.c_str()};
    const nvrtcResult rc = N.compile(prog, 6, opts);
    size_t n = 0;
    N.log_size(prog, &n);
    log.assign(n, '\0');
    if (n)
        N.log(prog, log.data());
    if (rc != NVRTC_SUCCESS)
    {
        N.destroy(&prog);
        throw Error(B2_CUDA_ERROR, std::string("mymyr_b200: compiling the task's kernels failed: ") + N.error(rc) +
                                       "\n" + log.substr(0, 4000));
    }
    size_t bytes = 0;
    B2_NVRTC(N.cubin_size(prog, &bytes));
    auto cubin = std::make_shared<std::vector<char>>(bytes);
    B2_NVRTC(N.cubin(prog, cubin->data()));
    N.destroy(&prog);
    return cubin;
}

cudaKernel_t kernel(cudaLibrary_t lib, const char* name)
{
    cudaKernel_t k = nullptr;
    B2_CUDA(cudaLibraryGetKernel(&k, lib, name));
    return k;
}

constexpr const char* kKernelNames[kJitKernels] = {"brfs_count", "brfs_expand", "dbrfs_expand", "dbrfs_count",
                                                   "dbrfs_push", "env_init",    "env_step",     "expand_count",
                                                   "expand_write", "expand_hash"};

/// The cubin of kernel pair `which` (kJitKernels: all) of a source, compiled once per process.
std::shared_ptr<std::vector<char>> cubin_of(const std::string& src, u64 key, u32 which, std::string* log_out)
{
    {
        std::lock_guard lock(g_mu);
        if (auto it = g_cubins.find({key, which}); it != g_cubins.end())
            return it->second;
    }
    std::string log;
    auto cubin = compile(src, which, log);
    if (log_out)
        *log_out = log;
    std::lock_guard lock(g_mu);
    return g_cubins.emplace(std::make_pair(key, which), cubin).first->second;
}
}  // namespace

JitModule::~JitModule()
{
    for (cudaLibrary_t l : lib)
        if (l)
            cudaLibraryUnload(l);
}

cudaKernel_t JitModule::get(JitKernel which, u32 pi)
{
    std::lock_guard lock(mu);
    if (!lib[which])
    {
        const auto cubin = cubin_of(source, digest, which, &log);
        B2_CUDA(cudaLibraryLoadData(&lib[which], cubin->data(), nullptr, nullptr, 0, nullptr, nullptr, 0));
        const std::string name = std::string("b2j_") + kKernelNames[which];
        k[which][0] = kernel(lib[which], (name + "_w").c_str());
        k[which][1] = kernel(lib[which], (name + "_nw").c_str());
    }
    return k[which][pi];
}

std::shared_ptr<std::vector<char>> jit_cubin(const Program& prog, u64* key_out, std::string* log_out)
{
    const std::string src = generate_matcher_source(prog);
    const u64 key = digest(src);
    if (key_out)
        *key_out = key;
    return cubin_of(src, key, kJitKernels, log_out);
}

std::shared_ptr<JitModule> jit_module(int device, const Program& prog)
{
    std::string src = generate_matcher_source(prog);
    const u64 key = digest(src);
    {
        std::lock_guard lock(g_mu);
        if (auto it = g_modules.find({device, key}); it != g_modules.end())
            return it->second;
    }
    auto m = std::make_shared<JitModule>();
    m->device = device;
    m->digest = key;
    m->source = std::move(src);
    // the batched expand's kernels are compiled and loaded on the device now, not at their first launch, so that
    // b2_expand_noalloc's calls load nothing
    for (JitKernel which : {kJitExpandCount, kJitExpandWrite, kJitExpandHash})
        for (u32 pi = 0; pi < 2; ++pi)
        {
            cudaFuncAttributes attr{};
            B2_CUDA(cudaFuncGetAttributes(&attr, reinterpret_cast<const void*>(m->get(which, pi))));
        }
    std::lock_guard lock(g_mu);
    return g_modules.emplace(std::make_pair(device, key), m).first->second;
}

void jit_launch(cudaKernel_t k, unsigned grid, unsigned block, void* arg, cudaStream_t s)
{
    void* args[] = {arg};
    B2_CUDA(cudaLaunchKernel(reinterpret_cast<const void*>(k), dim3(grid), dim3(block), args, 0, s));
}
}  // namespace b2
