// common.cuh - shared device helpers for the LSA select + read kernels (sm_100a).
//
// Bit-exact arithmetic: every value that feeds a selection (scores, Gram entries, merge
// costs, sums, norms) is computed with explicit round-to-nearest intrinsics
// (__fadd_rn, __fmul_rn, __fmaf_rn, __fdiv_rn, __fsqrt_rn), which the compiler never
// contracts or reorders. The operation sequence is the canonical one the CPU checker
// defines:
//   cdot(x, y): chunk c of 8 consecutive elements belongs to lane c % 32; each lane runs an
//   fp32 fmaf chain over its chunks in increasing c; a butterfly (xor 16, 8, 4, 2, 1) adds
//   the 32 partials. Every lane ends with the same value (fp add is commutative).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lsa {

constexpr int64_t kEmpty = INT64_MIN;  // empty packed key: sorts after every real key

// kF32AsBF16: fp32 storage read as bf16 values (rounded to nearest even on load) - the
// selects' query code for "bf16 scoring of an fp32 index query" without a cast launch
enum Dtype : int { kF32 = 0, kF16 = 1, kBF16 = 2, kF32AsBF16 = 3 };

// ------------------------------------------------------------------ conversions

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Load 8 consecutive elements (16 B for 16-bit types, 32 B for fp32) as fp32.
template <typename T> __device__ __forceinline__ void load8(const T* p, float (&out)[8]);

template <> __device__ __forceinline__ void load8<float>(const float* p, float (&out)[8]) {
    float4 a = *reinterpret_cast<const float4*>(p);
    float4 b = *reinterpret_cast<const float4*>(p + 4);
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
}

// An fp32 element that reads as its bf16 rounding (dtype code kF32AsBF16).
struct F32AsBF16 {
    float v;
};
template <> __device__ __forceinline__ void load8<F32AsBF16>(const F32AsBF16* p, float (&out)[8]) {
    load8<float>(reinterpret_cast<const float*>(p), out);
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = __bfloat162float(__float2bfloat16_rn(out[e]));
}

// A query read as its index-space row, built inside the select: the storage is the raw
// query [R, Hq, D] of T, and index element (h, e) is the fp32 mean of q[h G + g][e] over the
// G query heads of KV head h (added in head order from 0, then divided by G: the regroup's
// arithmetic), read as its bf16 rounding when RB (bf16 scoring).
template <typename T, bool RB> struct GroupMean {
    T v;
};
template <typename T> struct GroupMeanOf {
    static constexpr bool value = false;
};
template <typename T, bool RB> struct GroupMeanOf<GroupMean<T, RB>> {
    static constexpr bool value = true;
    static constexpr bool round_bf16 = RB;
    using raw = T;
};
struct QGroup {
    int G, D;  // query heads per KV head, head dim (GroupMean queries only)
};

template <> __device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&out)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        out[2 * i] = __uint_as_float(w[i] << 16);
        out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

template <> __device__ __forceinline__ void load8<__half>(const __half* p, float (&out)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f = __half22float2(h[i]);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}

// ------------------------------------------------------------------ keys

// Order-preserving fp32 -> int32: -NaN < -inf < ... < -0 < +0 < ... < +inf < +NaN.
__device__ __forceinline__ int32_t ordered_bits(float f) {
    int32_t b = __float_as_int(f);
    return b >= 0 ? b : (b ^ 0x7FFFFFFF);
}

// key = ordered_bits(score) << 32 | (0x7FFFFFFF - column)
__device__ __forceinline__ int64_t pack_key(float score, int32_t column) {
    uint64_t hi = (uint64_t)(uint32_t)ordered_bits(score) << 32;
    uint64_t lo = (uint64_t)(uint32_t)(0x7FFFFFFF - column);
    return (int64_t)(hi | lo);
}

__device__ __forceinline__ int32_t key_bucket(int64_t key) {
    return key == kEmpty ? -1 : (int32_t)(0x7FFFFFFF - (int32_t)((uint64_t)key & 0xFFFFFFFFull));
}

// ------------------------------------------------------------------ canonical dot

// Butterfly sum of one fp32 partial per lane; all 32 lanes return the same value.
__device__ __forceinline__ float butterfly_sum(float p) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) p = __fadd_rn(p, __shfl_xor_sync(0xFFFFFFFFu, p, off));
    return p;
}

// Lane partial of cdot(x, y) where x is held in registers (this lane's chunks, in
// increasing chunk order, 8 floats each) and y is read from memory.
template <typename T, int CHUNKS>
__device__ __forceinline__ float lane_partial_regs(const float (&x)[CHUNKS][8], const T* y, int lane, int nchunks) {
    float p = 0.0f;
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
        int c = lane + 32 * j;
        if (c < nchunks) {
            float yv[8];
            load8<T>(y + (size_t)c * 8, yv);
#pragma unroll
            for (int e = 0; e < 8; ++e) p = __fmaf_rn(x[j][e], yv[e], p);
        }
    }
    return p;
}

// Canonical cdot of two vectors in memory, computed by one full warp.
template <typename TX, typename TY>
__device__ __forceinline__ float warp_cdot(const TX* x, const TY* y, int d, int lane) {
    float p = 0.0f;
    int nchunks = d >> 3;
    for (int c = lane; c < nchunks; c += 32) {
        float xv[8], yv[8];
        load8<TX>(x + (size_t)c * 8, xv);
        load8<TY>(y + (size_t)c * 8, yv);
#pragma unroll
        for (int e = 0; e < 8; ++e) p = __fmaf_rn(xv[e], yv[e], p);
    }
    return butterfly_sum(p);
}

// ------------------------------------------------------------------ block sort

// In-place bitonic sort of n (power of two) int64 keys in shared memory, descending.
// All threads of the block must call it.
__device__ __forceinline__ void bitonic_sort_desc(int64_t* s, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                int ixj = i ^ j;
                if (ixj > i) {
                    int64_t a = s[i], b = s[ixj];
                    bool desc = (i & k) == 0;
                    if (desc ? (a < b) : (a > b)) {
                        s[i] = b;
                        s[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
}

__host__ __device__ __forceinline__ int next_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

// Exclusive scan of one int per thread over a group of NT threads (tid in [0, NT), NT a
// multiple of 32, at most 1024) that share the barrier `sync`. Returns the exclusive prefix;
// *total receives the group sum. Uses 33 ints of smem.
template <int NT, typename Sync>
__device__ __forceinline__ int group_exclusive_scan(int v, int* smem, int* total, int tid, Sync sync) {
    constexpr int NWARPS = NT / 32;
    const int lane = tid & 31, warp = tid >> 5;
    int x = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        int y = __shfl_up_sync(0xFFFFFFFFu, x, off);
        if (lane >= off) x += y;
    }
    if (lane == 31) smem[warp] = x;
    sync();
    if (warp == 0) {
        int w = lane < NWARPS ? smem[lane] : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            int y = __shfl_up_sync(0xFFFFFFFFu, w, off);
            if (lane >= off) w += y;
        }
        if (lane < NWARPS) smem[lane] = w;  // inclusive prefix of warp sums
        if (lane == NWARPS - 1) smem[32] = w;
    }
    sync();
    int before = warp > 0 ? smem[warp - 1] : 0;
    int res = before + x - v;
    *total = smem[32];
    sync();
    return res;
}

// Block-wide exclusive scan of one int per thread (blockDim.x <= 1024, multiple of 32).
// Returns the exclusive prefix; *total receives the block sum. Uses 33 ints of smem.
__device__ __forceinline__ int block_exclusive_scan(int v, int* smem, int* total) {
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    int x = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        int y = __shfl_up_sync(0xFFFFFFFFu, x, off);
        if (lane >= off) x += y;
    }
    if (lane == 31) smem[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nwarps ? smem[lane] : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            int y = __shfl_up_sync(0xFFFFFFFFu, w, off);
            if (lane >= off) w += y;
        }
        if (lane < nwarps) smem[lane] = w;  // inclusive prefix of warp sums
        if (lane == nwarps - 1) smem[32] = w;
    }
    __syncthreads();
    int before = warp > 0 ? smem[warp - 1] : 0;
    int res = before + x - v;
    *total = smem[32];
    __syncthreads();
    return res;
}

// ------------------------------------------------------------------ timing / status

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}


// ------------------------------------------------------------------ mbarriers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: true when the phase completed, false after limit_ns (default 2 s).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > limit_ns) return false;
    }
    return true;
}

}  // namespace lsa

// Host-side status codes shared by every entry point.
#define LSA_OK 0
#define LSA_ERR_ARG (-1)
#define LSA_ERR_CUDA (-2)
#define LSA_ERR_TIMEOUT (-3)
#define LSA_ERR_SHORT (-4)
#define LSA_ERR_SIZE (-5)

#define LSA_LAUNCH_CHECK()                                    \
    do {                                                      \
        cudaError_t _e = cudaGetLastError();                  \
        if (_e != cudaSuccess) return LSA_ERR_CUDA;           \
    } while (0)
