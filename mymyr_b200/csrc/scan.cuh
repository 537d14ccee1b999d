// Device-wide exclusive scan in three launches (tile sums, one-block scan of the sums, tile apply), generic over an
// input functor (the u32 or u64 value of element i) and an output functor (called with i, its exclusive prefix and its
// value). Prefixes are u64.
// Used for candidate offsets (successor counts per parent), CSR offsets and the ranks of new states.

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

template<class In>
__global__ void __launch_bounds__(kScanBlock) k_tile_reduce(In in, u64 n_in, const u64* n_dev, u64* __restrict__ sums)
{
    using Reduce = cub::BlockReduce<u64, kScanBlock>;
    __shared__ typename Reduce::TempStorage tmp;
    const u64 n = n_dev ? *n_dev : n_in;  // a count known only on the device: the tiles past it sum to zero
    const u64 base = blockIdx.x * kScanTile;
    u64 s = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k)
    {
        const u64 i = base + static_cast<u64>(threadIdx.x) * kScanItems + k;
        if (i < n)
            s += in(i);
    }
    const u64 t = Reduce(tmp).Sum(s);
    if (threadIdx.x == 0)
        sums[blockIdx.x] = t;
}

/// In-place exclusive scan of nb block sums by one block; the grand total goes to *total.
__global__ void __launch_bounds__(1024) k_scan_sums(u64* __restrict__ sums, u64 nb, u64* __restrict__ total);

template<class In, class Out>
__global__ void __launch_bounds__(kScanBlock) k_tile_apply(In in, u64 n_in, const u64* n_dev,
                                                           const u64* __restrict__ offs, Out out)
{
    using Scan = cub::BlockScan<u64, kScanBlock>;
    __shared__ typename Scan::TempStorage tmp;
    using V = decltype(in(u64{0}));
    const u64 n = n_dev ? *n_dev : n_in;
    const u64 base = blockIdx.x * kScanTile;
    if (base >= n)
        return;  // uniform over the block
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
    const u64 off = offs[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kScanItems; ++k)
    {
        const u64 i = base + static_cast<u64>(threadIdx.x) * kScanItems + k;
        if (i < n)
            out(i, off + e[k], v[k]);
    }
}

/// Scratch bytes a scan of n elements needs.
inline size_t scan_scratch_bytes(u64 n) { return ((n + kScanTile - 1) / kScanTile + 1) * sizeof(u64); }

/// Exclusive scan of in(i), i < n; out(i, prefix, value) for each element, the total into *total (device).
/// `scratch` holds scan_scratch_bytes(n) bytes.
template<class In, class Out>
void device_scan(In in, Out out, u64 n, u64* total, u64* scratch, cudaStream_t s)
{
    const u64 nb = (n + kScanTile - 1) / kScanTile;
    if (nb == 0)
    {
        B2_CUDA(cudaMemsetAsync(total, 0, sizeof(u64), s));
        return;
    }
    k_tile_reduce<<<static_cast<unsigned>(nb), kScanBlock, 0, s>>>(in, n, nullptr, scratch);
    k_scan_sums<<<1, 1024, 0, s>>>(scratch, nb, total);
    k_tile_apply<<<static_cast<unsigned>(nb), kScanBlock, 0, s>>>(in, n, nullptr, scratch, out);
    B2_CUDA(cudaGetLastError());
}

/// device_scan over *n_dev elements, a count that only the device knows yet and that is at most n_max: launched for
/// n_max elements, the tiles past the count add nothing and write nothing. `scratch` holds scan_scratch_bytes(n_max).
template<class In, class Out>
void device_scan_dev(In in, Out out, const u64* n_dev, u64 n_max, u64* total, u64* scratch, cudaStream_t s)
{
    const u64 nb = std::max<u64>(1, (n_max + kScanTile - 1) / kScanTile);
    k_tile_reduce<<<static_cast<unsigned>(nb), kScanBlock, 0, s>>>(in, n_max, n_dev, scratch);
    k_scan_sums<<<1, 1024, 0, s>>>(scratch, nb, total);
    k_tile_apply<<<static_cast<unsigned>(nb), kScanBlock, 0, s>>>(in, n_max, n_dev, scratch, out);
    B2_CUDA(cudaGetLastError());
}
}  // namespace b2
