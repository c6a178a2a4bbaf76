// topk.cuh - top-k of packed keys by warp bitonic sorts and merge trees (sm_100a).
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

// ------------------------------------------------------------------ top-K lists in a warp

// A warp list of K = 32 * KW keys: key i lives in register i / 32 of lane i % 32.
// Descending bitonic sort: strides >= 32 compare registers of the same lane, smaller
// strides exchange by shuffles.
template <int KW>
__device__ __forceinline__ void warp_sort_desc(int64_t (&x)[KW], int lane) {
    constexpr int K = 32 * KW;
#pragma unroll
    for (int k = 2; k <= K; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j >= 32) {
                const int wj = j >> 5;
#pragma unroll
                for (int w = 0; w < KW; ++w) {
                    if ((w & wj) == 0) {
                        const bool desc = ((w * 32) & k) == 0;
                        const int64_t a = x[w], b = x[w | wj];
                        const bool swap = desc ? (a < b) : (a > b);
                        x[w] = swap ? b : a;
                        x[w | wj] = swap ? a : b;
                    }
                }
            } else {
#pragma unroll
                for (int w = 0; w < KW; ++w) {
                    const int64_t y = __shfl_xor_sync(0xFFFFFFFFu, x[w], j);
                    const bool lower = (lane & j) == 0, desc = ((w * 32 + lane) & k) == 0;
                    x[w] = (lower == desc) ? (x[w] > y ? x[w] : y) : (x[w] < y ? x[w] : y);
                }
            }
        }
    }
}

// Sorts a bitonic warp list descending (half-cleaners of strides K/2 .. 1).
template <int KW>
__device__ __forceinline__ void warp_clean_desc(int64_t (&x)[KW], int lane) {
    constexpr int K = 32 * KW;
#pragma unroll
    for (int j = K >> 1; j > 0; j >>= 1) {
        if (j >= 32) {
            const int wj = j >> 5;
#pragma unroll
            for (int w = 0; w < KW; ++w) {
                if ((w & wj) == 0) {
                    const int64_t a = x[w], b = x[w | wj];
                    x[w] = a > b ? a : b;
                    x[w | wj] = a > b ? b : a;
                }
            }
        } else {
#pragma unroll
            for (int w = 0; w < KW; ++w) {
                const int64_t y = __shfl_xor_sync(0xFFFFFFFFu, x[w], j);
                x[w] = (lane & j) == 0 ? (x[w] > y ? x[w] : y) : (x[w] < y ? x[w] : y);
            }
        }
    }
}

// x <- the top K of two sorted warp lists x and y: max(x[i], y[K - 1 - i]) is bitonic and
// holds exactly their K greatest keys; the cleaner sorts it.
template <int KW>
__device__ __forceinline__ void warp_merge_desc(int64_t (&x)[KW], const int64_t (&y)[KW], int lane) {
#pragma unroll
    for (int w = 0; w < KW; ++w) {
        const int64_t r = __shfl_sync(0xFFFFFFFFu, y[KW - 1 - w], 31 - lane);
        x[w] = x[w] > r ? x[w] : r;
    }
    warp_clean_desc<KW>(x, lane);
}

// The K = 32 * KW greatest of key(0 .. n) (EMPTY past n), sorted descending, into out[0, K),
// by NW warps (warp in [0, NW)) that share the barrier `sync` (n the same in every warp).
// Every warp whose first K-key chunk holds keys folds its chunks into one sorted list (the
// next chunk's loads in flight while the current one sorts); the merge tree then runs over
// those warps' lists only - the other warps' lists would be all EMPTY, and merging one in
// changes nothing - so few keys take few merge levels and the idle warps take no issue
// slots from the sorting ones. lists: NW * K int64 of shared memory.
template <int KW, int NW, typename Loader, typename Sync>
__device__ __forceinline__ void group_topk_desc(const Loader& key, int n, int64_t* lists, int64_t* out, int warp,
                                                int lane, Sync sync) {
    constexpr int K = 32 * KW;
    const int nl = n <= 0 ? 0 : ((n + K - 1) / K < NW ? (n + K - 1) / K : NW);  // warps holding keys
    int64_t x[KW], nx[KW];
#pragma unroll
    for (int w = 0; w < KW; ++w) x[w] = kEmpty;
    auto load = [&](int chunk, int64_t (&y)[KW]) {
#pragma unroll
        for (int w = 0; w < KW; ++w) {
            const int i = chunk * K + w * 32 + lane;
            y[w] = i < n ? key(i) : kEmpty;
        }
    };
    if (warp < nl) {
        load(warp, x);
        if ((warp + NW) * K < n) load(warp + NW, nx);
        warp_sort_desc<KW>(x, lane);
        for (int c = warp + NW; c * K < n; c += NW) {
            int64_t y[KW];
#pragma unroll
            for (int w = 0; w < KW; ++w) y[w] = nx[w];
            if ((c + NW) * K < n) load(c + NW, nx);
            warp_sort_desc<KW>(y, lane);
            warp_merge_desc<KW>(x, y, lane);
        }
#pragma unroll
        for (int w = 0; w < KW; ++w) lists[warp * K + w * 32 + lane] = x[w];
    }
    sync();
#pragma unroll 1
    for (int step = 1; step < nl; step <<= 1) {
        if ((warp % (2 * step)) == 0 && warp + step < nl) {
#pragma unroll
            for (int w = 0; w < KW; ++w) {
                const int64_t y = lists[(warp + step) * K + K - 1 - (w * 32 + lane)];
                x[w] = x[w] > y ? x[w] : y;
            }
            warp_clean_desc<KW>(x, lane);
#pragma unroll
            for (int w = 0; w < KW; ++w) lists[warp * K + w * 32 + lane] = x[w];
        }
        sync();
    }
    if (warp == 0) {
#pragma unroll
        for (int w = 0; w < KW; ++w) out[w * 32 + lane] = x[w];
    }
    sync();
}

}  // namespace lsa
