// A task's run-time compiled kernels (jit.cu).

#pragma once

#include "task.hpp"

#include <cuda_runtime.h>

#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace b2
{
/// The kernels of a task's compiled module. Each pair (witness pruning on, off) is its own compile unit, compiled
/// on first use, so that a task pays only for the kernels its calls launch.
enum JitKernel : u32
{
    kJitBrfsCount,
    kJitBrfsExpand,
    kJitDbrfsExpand,
    kJitDbrfsCount,
    kJitDbrfsPush,
    kJitEnvInit,
    kJitEnvStep,
    kJitExpandCount,
    kJitExpandWrite,
    kJitExpandHash,
    kJitKernels
};

struct JitModule
{
    int device = 0;
    u64 digest = 0;  // of the generated source
    std::string source;
    std::string log;
    std::mutex mu;
    cudaLibrary_t lib[kJitKernels]{};
    cudaKernel_t k[kJitKernels][2]{};  // [kernel][0]: witness pruning on, [1]: off
    /// The kernel (compiled for sm_100a and loaded with its twin on first use; the device must be current).
    cudaKernel_t get(JitKernel which, u32 pi);
    JitModule() = default;
    JitModule(const JitModule&) = delete;
    JitModule& operator=(const JitModule&) = delete;
    ~JitModule();
};

/// The CUDA source of a task's matcher (codegen.cpp).
std::string generate_matcher_source(const Program& prog);

/// The sm_100a cubin of all of `prog`'s kernels (compiled once per process and program; needs no GPU).
std::shared_ptr<std::vector<char>> jit_cubin(const Program& prog, u64* key = nullptr, std::string* log = nullptr);

/// The compiled module of `prog` on `device` (one per process, program and device). The batched expand's kernels are
/// compiled and loaded here; the others when first used.
std::shared_ptr<JitModule> jit_module(int device, const Program& prog);

/// Launches a module kernel whose only parameter is the struct at `arg`.
void jit_launch(cudaKernel_t k, unsigned grid, unsigned block, void* arg, cudaStream_t s);
}  // namespace b2
