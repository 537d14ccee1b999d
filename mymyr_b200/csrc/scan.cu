#include "scan.cuh"

namespace b2
{
__global__ void __launch_bounds__(1024) k_scan_sums(u64* __restrict__ sums, u64 nb, u64* __restrict__ total)
{
    using Scan = cub::BlockScan<u64, 1024>;
    __shared__ typename Scan::TempStorage tmp;
    __shared__ u64 carry;
    if (threadIdx.x == 0)
        carry = 0;
    __syncthreads();
    for (u64 base = 0; base < nb; base += 1024)
    {
        const u64 i = base + threadIdx.x;
        u64 v = i < nb ? sums[i] : 0;
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
