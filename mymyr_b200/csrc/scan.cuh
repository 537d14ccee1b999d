// Device-wide exclusive scan in one pass (decoupled look-back, after Merrill and Garland, "Single-pass Parallel Prefix
// Scan with Decoupled Look-back", NVIDIA technical report NVR-2016-002), generic over an input functor (the u32 or u64
// value of element i) and an output functor (called with i, its exclusive prefix and its value). Prefixes are u64.
// Used for candidate offsets (successor counts per parent), CSR offsets and the ranks of new states.
//
// Each block takes the next tile by a ticket (so a block only ever waits on tiles that running blocks hold), scans it,
// publishes its aggregate, then its first warp walks back over the preceding tiles' published values, 32 at a time,
// until it meets an inclusive prefix; it publishes its own inclusive prefix, writes its outputs and takes the next
// ticket (a grid of at most eight blocks per SM, so that a scan sized for a capacity but run over a count still on the
// device costs little). The tile states live in the caller's scratch and are cleared before each scan (8 bytes per
// tile).

#pragma once

#include "common.cuh"

#include <algorithm>

#include <cub/block/block_scan.cuh>

namespace b2
{
constexpr int kScanBlock = 256;
constexpr int kScanItems = 8;
constexpr u64 kScanTile = static_cast<u64>(kScanBlock) * kScanItems;
/// Tile states: nothing published yet, aggregate published, inclusive prefix published.
constexpr u64 kTileNone = 0, kTileAggregate = 1, kTilePrefix = 2;
/// A look-back lane gives up waiting for a tile after this many polls (the wait always ends on a working device: a
/// tile's holder is running and never waits on later tiles).
constexpr u32 kScanSpinLimit = 1u << 22;
/// Status bit (the caller's status word) of a look-back that gave up.
constexpr u32 kStatusScanStall = 8u;

/// Scratch of a scan of nb tiles: ticket | (unused) | state[nb] | aggregate[nb] | inclusive[nb].
struct ScanTiles
{
    unsigned long long* ticket;
    u64* state;
    u64* aggregate;
    u64* inclusive;
};
__host__ __device__ inline ScanTiles scan_tiles(u64* scratch, u64 nb)
{
    return {reinterpret_cast<unsigned long long*>(scratch), scratch + 2, scratch + 2 + nb, scratch + 2 + 2 * nb};
}

__device__ __forceinline__ u64 load_volatile(const u64* p) { return *reinterpret_cast<const volatile u64*>(p); }
__device__ __forceinline__ void store_volatile(u64* p, u64 v) { *reinterpret_cast<volatile u64*>(p) = v; }

template<class In, class Out>
__global__ void __launch_bounds__(kScanBlock) k_scan(In in, u64 n_in, const u64* n_dev, Out out, u64* total,
                                                     u64* scratch, u64 nb_max, u32* status)
{
    using Scan = cub::BlockScan<u64, kScanBlock>;
    using V = decltype(in(u64{0}));
    __shared__ typename Scan::TempStorage tmp;
    __shared__ u64 sh_tile, sh_prefix;
    const ScanTiles T = scan_tiles(scratch, nb_max);
    const u64 n = n_dev ? *n_dev : n_in;  // a count known only on the device: up to nb_max tiles
    const u64 nb = (n + kScanTile - 1) / kScanTile;
    if (nb == 0)
    {
        if (blockIdx.x == 0 && threadIdx.x == 0)
            *total = 0;
        return;
    }
    // tiles by ticket, as many per block as the grid needs: a block waits only on tiles that running blocks hold
    for (;;)
    {
        if (threadIdx.x == 0)
            sh_tile = atomicAdd(T.ticket, 1ull);
        __syncthreads();
        const u64 tile = sh_tile;
        if (tile >= nb)
            break;
        const u64 base = tile * kScanTile;
        V v[kScanItems];
        u64 e[kScanItems];
#pragma unroll
        for (int k = 0; k < kScanItems; ++k)
        {
            const u64 i = base + static_cast<u64>(threadIdx.x) * kScanItems + k;
            v[k] = i < n ? in(i) : 0;
            e[k] = v[k];
        }
        u64 agg = 0;
        Scan(tmp).ExclusiveSum(e, e, agg);
        if (threadIdx.x < 32)
        {
            const u32 lane = threadIdx.x;
            if (tile == 0)
            {
                if (lane == 0)
                {
                    T.inclusive[0] = agg;
                    __threadfence();
                    store_volatile(T.state, kTilePrefix);
                    sh_prefix = 0;
                }
            }
            else
            {
                if (lane == 0)
                {
                    T.aggregate[tile] = agg;
                    __threadfence();
                    store_volatile(T.state + tile, kTileAggregate);
                }
                u64 prefix = 0;
                long long hi = static_cast<long long>(tile) - 1;
                for (;;)
                {
                    const long long t = hi - static_cast<long long>(lane);
                    u64 st = kTilePrefix, val = 0;
                    if (t >= 0)
                    {
                        st = load_volatile(T.state + t);
                        u32 spins = 0;
                        while (st == kTileNone)
                        {
                            if (++spins > kScanSpinLimit)
                            {
                                if (status)
                                    atomicOr(status, kStatusScanStall);
                                st = kTilePrefix;  // give up: the caller sees the status and discards the scan
                                break;
                            }
                            if (spins > 32)
                                __nanosleep(128);
                            st = load_volatile(T.state + t);
                        }
                        __threadfence();
                        val = st == kTilePrefix ? load_volatile(T.inclusive + t) : load_volatile(T.aggregate + t);
                    }
                    const u32 pmask = __ballot_sync(0xFFFFFFFFu, st == kTilePrefix);
                    const u32 upto = pmask ? static_cast<u32>(__ffs(pmask) - 1) : 31u;  // the nearest inclusive prefix
                    u64 c = lane <= upto ? val : 0;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1)
                        c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
                    prefix += c;
                    if (pmask)
                        break;
                    hi -= 32;
                }
                if (lane == 0)
                {
                    T.inclusive[tile] = prefix + agg;
                    __threadfence();
                    store_volatile(T.state + tile, kTilePrefix);
                    sh_prefix = prefix;
                }
            }
        }
        __syncthreads();
        const u64 off = sh_prefix;
#pragma unroll
        for (int k = 0; k < kScanItems; ++k)
        {
            const u64 i = base + static_cast<u64>(threadIdx.x) * kScanItems + k;
            if (i < n)
                out(i, off + e[k], v[k]);
        }
        if (tile == nb - 1 && threadIdx.x == 0)
            *total = off + agg;
        __syncthreads();  // the shared tile, prefix and scan storage are reused by the next tile
    }
}

/// Clears a scan's ticket and tile states (a kernel rather than a memset, so that a captured scan is kernels only).
__global__ void k_scan_clear(u64* __restrict__ scratch, u64 words);

/// Blocks of a scan: one per tile up to eight per SM (more tiles are taken in turn by the same blocks).
unsigned scan_blocks(u64 nb);

/// Scratch bytes a scan of n elements needs.
constexpr size_t scan_scratch_bytes(u64 n)
{
    const u64 nb = n > kScanTile ? (n + kScanTile - 1) / kScanTile : 1;
    return (2 + 3 * nb) * sizeof(u64);
}

/// Exclusive scan of in(i), i < n (or i < *n_dev, at most n, when n_dev is set); out(i, prefix, value) for each
/// element, the total into *total (device). `scratch` holds scan_scratch_bytes(n) bytes; a look-back that gives up
/// sets kStatusScanStall in *status (if given).
template<class In, class Out>
void device_scan_impl(In in, Out out, u64 n, const u64* n_dev, u64* total, u64* scratch, cudaStream_t s, u32* status)
{
    const u64 nb = std::max<u64>(1, (n + kScanTile - 1) / kScanTile);
    k_scan_clear<<<scan_blocks((2 + nb + 255) / 256), 256, 0, s>>>(scratch, 2 + nb);  // ticket and tile states
    k_scan<<<scan_blocks(nb), kScanBlock, 0, s>>>(in, n, n_dev, out, total, scratch, nb, status);
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
