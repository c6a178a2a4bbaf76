// topk.cuh - top-32 of packed keys by warp bitonic sorts and a merge tree (sm_100a).
#pragma once

#include "common.cuh"

namespace lsa {

// Descending bitonic sort of 32 keys, one per lane, by shuffles only.
__device__ __forceinline__ int64_t warp_sort32_desc(int64_t x, int lane) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            int64_t y = __shfl_xor_sync(0xFFFFFFFFu, x, j);
            bool lower = (lane & j) == 0, desc = (lane & k) == 0;
            x = (lower == desc) ? (x > y ? x : y) : (x < y ? x : y);
        }
    }
    return x;
}

// Sorts a bitonic 32-sequence descending (half-cleaners of strides 16 .. 1).
__device__ __forceinline__ int64_t warp_clean32_desc(int64_t x, int lane) {
#pragma unroll
    for (int j = 16; j > 0; j >>= 1) {
        int64_t y = __shfl_xor_sync(0xFFFFFFFFu, x, j);
        x = (lane & j) == 0 ? (x > y ? x : y) : (x < y ? x : y);
    }
    return x;
}

// The 32 greatest of keys[0, n) (EMPTY-padded), sorted descending, into out[0, 32).
// Every warp folds its 32-key chunks into one sorted list (merging two sorted lists A, B
// keeps max(A[i], B[31 - i]), a bitonic sequence holding their top 32), then a merge
// tree over the warps' lists through shared memory. lists: blockDim.x int64.
__device__ __forceinline__ void block_top32_desc(const int64_t* keys, int n, int64_t* lists, int64_t* out) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int64_t x = warp * 32 + lane < n ? keys[warp * 32 + lane] : kEmpty;
    x = warp_sort32_desc(x, lane);
    for (int c = warp + nw; c * 32 < n; c += nw) {
        int64_t y = c * 32 + lane < n ? keys[c * 32 + lane] : kEmpty;
        y = warp_sort32_desc(y, lane);
        y = __shfl_sync(0xFFFFFFFFu, y, 31 - lane);
        x = warp_clean32_desc(x > y ? x : y, lane);
    }
    lists[warp * 32 + lane] = x;
    __syncthreads();
    for (int step = 1; step < nw; step <<= 1) {
        if ((warp % (2 * step)) == 0 && warp + step < nw) {
            int64_t y = lists[(warp + step) * 32 + 31 - lane];
            x = warp_clean32_desc(x > y ? x : y, lane);
            lists[warp * 32 + lane] = x;
        }
        __syncthreads();
    }
    if (warp == 0) out[lane] = x;
    __syncthreads();
}

}  // namespace lsa
