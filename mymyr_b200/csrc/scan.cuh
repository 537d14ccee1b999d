// Device-wide exclusive scan, generic over an input functor (the u32 or u64 value of element i) and an output functor
// (called with i, its exclusive prefix and its value). Prefixes are u64. Used for candidate offsets (successor counts
// per parent), CSR offsets and the ranks of new states.
//
// Three launches: tile sums, a one-block scan of the tile sums, and the tiles' own scans with their offsets. Each pass
// reads the input once at full bandwidth and no block waits on another. The element count may be a value still on
// the device (a count the host has not read, at most a capacity the launch is sized for): the tile passes run
// grid-stride loops of at most eight blocks per SM over the tiles the count covers, so a scan sized for a capacity costs
// little when the count is small.

#pragma once

#include "common.cuh"

#include <algorithm>

#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>

namespace b2
{
constexpr int kScanBlock = 256;
constexpr int kScanItems = 8;
constexpr u64 kScanTile = static_cast<u64>(kScanBlock) * kScanItems;
/// Status bit of a scan that failed (reserved: no block of this scan waits on another).
constexpr u32 kStatusScanStall = 8u;

__device__ __forceinline__ u64 scan_count(u64 n_in, const u64* n_dev) { return n_dev ? *n_dev : n_in; }

template<class In>
__global__ void __launch_bounds__(kScanBlock) k_tile_reduce(In in, u64 n_in, const u64* n_dev, u64* __restrict__ sums)
{
    using Reduce = cub::BlockReduce<u64, kScanBlock>;
    __shared__ typename Reduce::TempStorage tmp;
    const u64 n = scan_count(n_in, n_dev);
    const u64 nb = (n + kScanTile - 1) / kScanTile;
    for (u64 t = blockIdx.x; t < nb; t += gridDim.x)
    {
        const u64 base = t * kScanTile;
        u64 s = 0;
#pragma unroll
        for (int k = 0; k < kScanItems; ++k)
        {
            const u64 i = base + static_cast<u64>(threadIdx.x) * kScanItems + k;
            if (i < n)
                s += in(i);
        }
        const u64 total = Reduce(tmp).Sum(s);
        if (threadIdx.x == 0)
            sums[t] = total;
        __syncthreads();  // the reduce storage is reused by the next tile
    }
}

/// In-place exclusive scan of the tile sums by one block; the grand total goes to *total.
__global__ void __launch_bounds__(1024) k_scan_sums(u64* __restrict__ sums, u64 n_in, const u64* n_dev,
                                                    u64* __restrict__ total);

template<class In, class Out>
__global__ void __launch_bounds__(kScanBlock) k_tile_apply(In in, u64 n_in, const u64* n_dev,
                                                           const u64* __restrict__ offs, Out out)
{
    using Scan = cub::BlockScan<u64, kScanBlock>;
    __shared__ typename Scan::TempStorage tmp;
    using V = decltype(in(u64{0}));
    const u64 n = scan_count(n_in, n_dev);
    const u64 nb = (n + kScanTile - 1) / kScanTile;
    for (u64 t = blockIdx.x; t < nb; t += gridDim.x)
    {
        const u64 base = t * kScanTile;
        V v[kScanItems];
        u64 e[kScanItems];
#pragma unroll
        for (int k = 0; k < kScanItems; ++k)
        {
            const u64 i = base + static_cast<u64>(threadIdx.x) * kScanItems + k;
            v[k] = i < n ? in(i) : 0;
            e[k] = v[k];
        }
        Scan(tmp).ExclusiveSum(e, e);
        const u64 off = offs[t];
#pragma unroll
        for (int k = 0; k < kScanItems; ++k)
        {
            const u64 i = base + static_cast<u64>(threadIdx.x) * kScanItems + k;
            if (i < n)
                out(i, off + e[k], v[k]);
        }
        __syncthreads();  // the scan storage is reused by the next tile
    }
}

/// Blocks of a tile pass: one per tile up to eight per SM (more tiles are taken in turn by the same blocks).
unsigned scan_blocks(u64 nb);

/// Scratch bytes a scan of up to n elements needs (the tile sums).
constexpr size_t scan_scratch_bytes(u64 n) { return ((n + kScanTile - 1) / kScanTile + 1) * sizeof(u64); }

/// Exclusive scan of in(i), i < n (or i < *n_dev, at most n, when n_dev is set); out(i, prefix, value) for each
/// element, the total into *total (device). `scratch` holds scan_scratch_bytes(n) bytes. `status` is the caller's
/// status word, for a scan that can fail; this one cannot.
template<class In, class Out>
void device_scan_impl(In in, Out out, u64 n, const u64* n_dev, u64* total, u64* scratch, cudaStream_t s, u32* status)
{
    (void)status;
    const u64 nb = std::max<u64>(1, (n + kScanTile - 1) / kScanTile);
    const unsigned grid = scan_blocks(nb);
    k_tile_reduce<<<grid, kScanBlock, 0, s>>>(in, n, n_dev, scratch);
    k_scan_sums<<<1, 1024, 0, s>>>(scratch, n, n_dev, total);
    k_tile_apply<<<grid, kScanBlock, 0, s>>>(in, n, n_dev, scratch, out);
    B2_CUDA(cudaGetLastError());
}

template<class In, class Out>
void device_scan(In in, Out out, u64 n, u64* total, u64* scratch, cudaStream_t s, u32* status = nullptr)
{
    device_scan_impl(in, out, n, nullptr, total, scratch, s, status);
}

/// device_scan over *n_dev elements, a count that only the device knows yet and that is at most n_max.
template<class In, class Out>
void device_scan_dev(In in, Out out, const u64* n_dev, u64 n_max, u64* total, u64* scratch, cudaStream_t s,
                     u32* status = nullptr)
{
    device_scan_impl(in, out, n_max, n_dev, total, scratch, s, status);
}
}  // namespace b2
