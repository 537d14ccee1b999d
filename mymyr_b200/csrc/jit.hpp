// A task's run-time compiled kernels (jit.cu).

#pragma once

#include "task.hpp"

#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

namespace b2
{
struct JitModule
{
    cudaLibrary_t lib = nullptr;
    u64 digest = 0;
    std::string log;
    // [0]: witness pruning on, [1]: off
    cudaKernel_t brfs_count[2]{}, brfs_expand[2]{}, dbrfs_expand[2]{}, dbrfs_push[2]{}, dbrfs_count[2]{}, env_init[2]{}, env_step[2]{}, expand_count[2]{}, expand_write[2]{};
    JitModule() = default;
    JitModule(const JitModule&) = delete;
    JitModule& operator=(const JitModule&) = delete;
    ~JitModule();
};

/// The CUDA source of a task's matcher (codegen.cpp).
std::string generate_matcher_source(const Program& prog);

/// The sm_100a cubin of `prog`'s kernels (compiled once per process and program; needs no GPU).
std::shared_ptr<std::vector<char>> jit_cubin(const Program& prog, u64* key = nullptr, std::string* log = nullptr);

/// The compiled module of `prog` on `device` (compiled once per process and program, loaded once per device).
std::shared_ptr<JitModule> jit_module(int device, const Program& prog);

/// Launches a module kernel whose only parameter is the struct at `arg`.
void jit_launch(cudaKernel_t k, unsigned grid, unsigned block, void* arg, cudaStream_t s);
}  // namespace b2
