// decode.cu - the fused decode step: selection and sparse read in ONE launch (sm_100a).
//
// For a few query rows of one sequence (decode), flat_select + lsa_read (the reference's
// pipeline.py:248-316 then read_kernel_tiled.py:41-89) as one cooperative grid:
//   A  every warp of the grid scores visible buckets (canonical cdot of the bf16 index query
//      with the bf16 centroids), stores their packed keys and prefetches their member rows
//      into L2;
//   B  one grid barrier (bounded spin on an arrival count: all CTAs are co-resident by the
//      cooperative launch);
//   C  every reading CTA takes its row's top-32 keys itself (warp bitonic sorts + merge
//      tree), stages the picked buckets' members and builds the row's read list in shared
//      memory (the expansion walk: members with sink <= id < window_start in pick order,
//      first top_k, then the window, then the sinks) - redundantly, so no second barrier;
//   D  the CTA reads its split of the list for one KV head: the K and V rows go to shared
//      memory by 16-byte cp.async, two 64-key stages in flight, then 16 lanes per row
//      with an online softmax for the G query heads; the CTA merges its warps, and the
//      last CTA of the (row, KV head) merges the splits (atomic ticket).
// Results equal flat_select + lsa_read: the list is the same walk (bit-exact, written out
// when asked), the read the same math in another summation order.
#include <cooperative_groups.h>

#include "common.cuh"
#include "topk.cuh"
#include "umma.cuh"

namespace lsa {
namespace {

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecMaxRows = 4;
constexpr int kDecChunk = 64;  // K/V rows per shared-memory stage
constexpr uint64_t kDecWaitNs = 1000000000ull;

struct FusedDecodeArgs {
    const __nv_bfloat16* iq;  // [R, d] index queries (bf16)
    int64_t ldq;
    int d;
    const __nv_bfloat16* cent;  // [N, d]
    int64_t N;
    const int32_t* members;  // [N, cap]
    int cap;
    const int32_t* positions;  // [R]
    int64_t block, bpb;
    int top_p, window, sink, top_k, width;
    const void* q;  // [R, Hq, 128]
    const void* k;  // [Tk, Hkv, 128]
    const void* v;
    int64_t Tk;
    int R, Hq, Hkv, splits, span;
    float scale_log2;
    void* out;          // [R, Hq, 128]
    int32_t* lists;     // [R, width] or null
    int32_t* lengths;   // [R] or null
    int64_t* keys;      // [R, N] scratch
    float* part_o;      // [R * Hkv, splits, G, 128]
    float* part_ml;     // [R * Hkv, splits, G, 2]
    uint32_t* bar;      // [0] arrivals, [1] departures (zero at rest)
    int32_t* tickets;   // [R * Hkv]
    int32_t* status;
};

// All CTAs of the (co-resident) grid meet; false after ~1 s (status set). bar[0] counts
// arrivals, bar[1] departures; every CTA counts its departure - also one whose wait
// expired - and the last to leave resets both, so the words are back at zero once every
// CTA has passed (other kernels share the counter buffer, and the next launch must not
// find a stale arrival count).
__device__ bool grid_barrier(uint32_t* bar, int32_t* status) {
    __shared__ int ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        ok = 1;
        __threadfence();
        atomicAdd(bar, 1u);
        volatile uint32_t* arrived = bar;
        const uint64_t t0 = global_ns();
        while (*arrived < gridDim.x) {
            if (global_ns() - t0 > kDecWaitNs) {
                atomicExch(status, LSA_ERR_TIMEOUT);
                ok = 0;
                break;
            }
        }
        // departures reach gridDim.x only after every CTA has arrived: the reset cannot
        // race a late arrival
        if (atomicAdd(bar + 1, 1u) == gridDim.x - 1) {
            atomicExch(bar, 0u);
            atomicExch(bar + 1, 0u);
        }
        __threadfence();
    }
    __syncthreads();
    return ok != 0;
}

template <typename T, int G>
__global__ void __launch_bounds__(kDecThreads) fused_decode_kernel(const FusedDecodeArgs a) {
    extern __shared__ __align__(16) unsigned char dsm[];
    __shared__ int64_t tl[kDecThreads];  // top-32 merge lists
    __shared__ int64_t picks[32];
    __shared__ int pick_kept[32], pick_off[32];
    __shared__ int list_len;
    __shared__ int is_last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    // ------------------------------------------------------------------ A: scoring
    {
        const int nchunks = a.d >> 3;
        const int64_t gw = (int64_t)blockIdx.x * kDecWarps + warp, nwarps = (int64_t)gridDim.x * kDecWarps;
        for (int64_t w = gw; w < (int64_t)a.R * a.N; w += nwarps) {
            const int r = (int)(w / a.N);
            const int64_t n = w % a.N;
            const int64_t vis = (int64_t)a.positions[r] / a.block * a.bpb;
            if (n >= vis) continue;
            const int lines = (a.cap * 4 + 127) / 128;
            if (lane < lines) asm volatile("prefetch.global.L2 [%0];" ::"l"(a.members + n * a.cap + lane * 32));
            float p = 0.0f;
            for (int c = lane; c < nchunks; c += 32) {  // canonical cdot: lane c % 32, chunks in order
                float xv[8], yv[8];
                load8<__nv_bfloat16>(a.iq + r * a.ldq + (int64_t)c * 8, xv);
                load8<__nv_bfloat16>(a.cent + n * a.d + (int64_t)c * 8, yv);
#pragma unroll
                for (int e = 0; e < 8; ++e) p = __fmaf_rn(xv[e], yv[e], p);
            }
            p = butterfly_sum(p);
            if (lane == 0) a.keys[(int64_t)r * a.N + n] = pack_key(p, (int32_t)n);
        }
    }
    if (!grid_barrier(a.bar, a.status)) return;

    const int units = a.R * a.Hkv * a.splits;
    const int u = blockIdx.x;
    if (u >= units) return;
    const int r = u / (a.Hkv * a.splits), h = (u / a.splits) % a.Hkv, split = u % a.splits;
    const int64_t pos = a.positions[r];

    // ------------------------------------------------------------------ C: top-32 + list
    // shared memory: [keys N x 8 | members 32 x cap x 4 | list width x 4 | K/V 2 stages];
    // the CTA merge reuses it from the start once the read is done
    int64_t* skeys = reinterpret_cast<int64_t*>(dsm);
    int32_t* mem = reinterpret_cast<int32_t*>(dsm + ((a.N * 8 + 15) / 16) * 16);
    int32_t* list = mem + 32 * a.cap;
    T* kvs = reinterpret_cast<T*>(dsm + (((a.N * 8 + 15) / 16) * 16 + (int64_t)(32 * a.cap + a.width) * 4 + 15) / 16 *
                                            16);  // [2][kDecChunk][2][128]
    {
        const int64_t vis = pos / a.block * a.bpb;
        const int count = (int)(vis < a.N ? (vis < 0 ? 0 : vis) : a.N);
        for (int i = threadIdx.x; i < count; i += kDecThreads) skeys[i] = __ldcg(a.keys + (int64_t)r * a.N + i);
        __syncthreads();
        block_top32_desc(skeys, count, tl, picks);
        const int kp = (int)min((int64_t)a.top_p, a.N);
        // picks past the live keys are EMPTY and sort last: the valid picks are a prefix
        int kv = 0;
        for (int p = 0; p < kp; ++p) kv += key_bucket(picks[p]) >= 0;
        // stage the picked buckets' member rows with 16-byte copies, all in flight at once
        const int q4 = a.cap / 4;
        for (int i = threadIdx.x; i < kv * q4; i += kDecThreads) {
            const int p = i / q4, c4 = i % q4;
            cp_async16(smem_u32(mem + p * a.cap + c4 * 4), a.members + (int64_t)key_bucket(picks[p]) * a.cap + c4 * 4,
                       16u);
        }
        cp_async_wait_all();
        __syncthreads();
        int64_t ws = pos + 1 - a.window;
        if (ws < 0) ws = 0;
        // kept members per pick (sink <= id < ws), then their offsets by a warp scan
        for (int p = warp; p < 32; p += kDecWarps) {
            int c = 0;
            if (p < kv) {
                for (int s0 = 0; s0 < a.cap; s0 += 32) {
                    const int slot = s0 + lane;
                    const int id = slot < a.cap ? mem[p * a.cap + slot] : -1;
                    c += __popc(__ballot_sync(0xFFFFFFFFu, id >= a.sink && (int64_t)id < ws));
                }
            }
            if (lane == 0) pick_kept[p] = c;
        }
        __syncthreads();
        if (warp == 0) {
            int c = pick_kept[lane], incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
                if (lane >= o) incl += y;
            }
            pick_off[lane] = incl - c;
            if (lane == 31) list_len = incl < a.top_k ? incl : a.top_k;
        }
        __syncthreads();
        const int nk = list_len;
        for (int p = warp; p < kv; p += kDecWarps) {
            int base = pick_off[p];
            for (int s0 = 0; s0 < a.cap && base < nk; s0 += 32) {
                const int slot = s0 + lane;
                const int id = slot < a.cap ? mem[p * a.cap + slot] : -1;
                const bool keep = id >= a.sink && (int64_t)id < ws;
                const uint32_t bal = __ballot_sync(0xFFFFFFFFu, keep);
                const int at = base + __popc(bal & ((1u << lane) - 1u));
                if (keep && at < nk) list[at] = id;
                base += __popc(bal);
            }
        }
        const int nwin = (int)(pos - ws + 1 > 0 ? pos - ws + 1 : 0);
        const int nsink = (int)(a.sink < ws ? a.sink : ws);
        for (int i = threadIdx.x; i < a.width - nk; i += kDecThreads) {
            int v = -1;
            if (i < nwin) v = (int)(ws + i);
            else if (i < nwin + nsink) v = i - nwin;
            list[nk + i] = v;
        }
        __syncthreads();
        if (threadIdx.x == 0) list_len = nk + nwin + nsink;
        __syncthreads();
        if (a.lists && h == 0 && split == 0) {
            for (int i = threadIdx.x; i < a.width; i += kDecThreads) a.lists[(int64_t)r * a.width + i] = list[i];
            if (threadIdx.x == 0) a.lengths[r] = list_len;
        }
    }

    // ------------------------------------------------------------------ D: split read
    const int len = list_len;
    const int lo = split * a.span, hi = min(lo + a.span, len);
    const int nch = hi > lo ? (hi - lo + kDecChunk - 1) / kDecChunk : 0;
    const T* kb = static_cast<const T*>(a.k) + (int64_t)h * 128;
    const T* vb = static_cast<const T*>(a.v) + (int64_t)h * 128;
    const int64_t rs = (int64_t)a.Hkv * 128;
    // stage chunk c of the split's K and V rows into buffer c & 1 (16-byte copies, zero-fill
    // for skipped ids); rows [kk][kv][128]
    auto stage = [&](int c) {
        T* dst = kvs + (c & 1) * kDecChunk * 2 * 128;
        for (int t = threadIdx.x; t < kDecChunk * 2 * 16; t += kDecThreads) {
            const int kk = t >> 5, kvsel = (t >> 4) & 1, c16 = t & 15;
            const int j = lo + c * kDecChunk + kk;
            const int id = j < hi ? list[j] : -1;
            const bool ok = id >= 0 && id < a.Tk;
            const T* src = (kvsel ? vb : kb) + (int64_t)(ok ? id : 0) * rs + c16 * 8;
            cp_async16(smem_u32(dst + (kk * 2 + kvsel) * 128 + c16 * 8), src, ok ? 16u : 0u);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    if (nch > 0) stage(0);
    if (nch > 1) stage(1);
    const int sub = lane >> 4, dl = (lane & 15) * 8;  // half-warp = one key row, 8 dims per lane
    const T* qp = static_cast<const T*>(a.q) + ((int64_t)r * a.Hq + h * G) * 128 + dl;
    float qv[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g) load8<T>(qp + g * 128, qv[g]);
    float m[G], l[G], o[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[g][e] = 0.0f;
    }
    for (int c = 0; c < nch; ++c) {
        if (c + 1 < nch)
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        else
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();
        const T* buf = kvs + (c & 1) * kDecChunk * 2 * 128;
        // the loop bound is warp-uniform (the shuffles below need all 32 lanes)
#pragma unroll 2
        for (int i = 0; i < kDecChunk / (2 * kDecWarps); ++i) {
            const int kk = i * 2 * kDecWarps + warp * 2 + sub;
            const int j = lo + c * kDecChunk + kk;
            const int id = j < hi ? list[j] : -1;
            const bool live = id >= 0 && id < a.Tk;
            float kx[8], vx[8];
            load8<T>(buf + (kk * 2) * 128 + dl, kx);
            load8<T>(buf + (kk * 2 + 1) * 128 + dl, vx);
            float s[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float acc = 0.0f;
#pragma unroll
                for (int e = 0; e < 8; ++e) acc = fmaf(qv[g][e], kx[e], acc);
                acc += __shfl_xor_sync(0xFFFFFFFFu, acc, 8);
                acc += __shfl_xor_sync(0xFFFFFFFFu, acc, 4);
                acc += __shfl_xor_sync(0xFFFFFFFFu, acc, 2);
                acc += __shfl_xor_sync(0xFFFFFFFFu, acc, 1);
                s[g] = acc * a.scale_log2;
            }
            if (live) {  // uniform within the half-warp
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float mn = fmaxf(m[g], s[g]);
                    const float corr = exp2f(m[g] - mn);  // m = -inf first: 0
                    const float pw = exp2f(s[g] - mn);
                    l[g] = l[g] * corr + pw;
#pragma unroll
                    for (int e = 0; e < 8; ++e) o[g][e] = fmaf(pw, vx[e], o[g][e] * corr);
                    m[g] = mn;
                }
            }
        }
        __syncthreads();  // buffer c & 1 is free again
        if (c + 2 < nch) stage(c + 2);
    }
    // merge the 16 half-warp states of the CTA through shared memory
    float* red_o = reinterpret_cast<float*>(dsm);                        // [16][G][128]
    float* red_ml = red_o + 16 * G * 128;                                // [16][G][2]
    __syncthreads();  // the list region is free again
    const int hw = warp * 2 + sub;
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int e = 0; e < 8; ++e) red_o[(hw * G + g) * 128 + dl + e] = o[g][e];
        if ((lane & 15) == 0) {
            red_ml[(hw * G + g) * 2] = m[g];
            red_ml[(hw * G + g) * 2 + 1] = l[g];
        }
    }
    __syncthreads();
    const int rh = r * a.Hkv + h;
    for (int oi = threadIdx.x; oi < G * 128; oi += kDecThreads) {
        const int g = oi / 128, e = oi % 128;
        float M = -INFINITY;
        for (int t = 0; t < 16; ++t) M = fmaxf(M, red_ml[(t * G + g) * 2]);
        float L = 0.0f, O = 0.0f;
        if (M != -INFINITY) {
            for (int t = 0; t < 16; ++t) {
                const float f = exp2f(red_ml[(t * G + g) * 2] - M);
                L += red_ml[(t * G + g) * 2 + 1] * f;
                O += red_o[(t * G + g) * 128 + e] * f;
            }
        }
        if (a.splits == 1) {
            static_cast<T*>(a.out)[((int64_t)r * a.Hq + h * G + g) * 128 + e] = from_f32<T>(L > 0.0f ? O / L : 0.0f);
        } else {
            const int64_t pi = ((int64_t)rh * a.splits + split) * G + g;
            a.part_o[pi * 128 + e] = O;
            if (e == 0) {
                a.part_ml[pi * 2] = M;
                a.part_ml[pi * 2 + 1] = L;
            }
        }
    }
    if (a.splits == 1) return;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int t = atomicAdd(a.tickets + rh, 1);
        is_last = t == a.splits - 1;
        if (is_last) a.tickets[rh] = 0;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    for (int oi = threadIdx.x; oi < G * 128; oi += kDecThreads) {
        const int g = oi / 128, e = oi % 128;
        float M = -INFINITY;
        for (int sp = 0; sp < a.splits; ++sp)
            M = fmaxf(M, __ldcg(a.part_ml + (((int64_t)rh * a.splits + sp) * G + g) * 2));
        float L = 0.0f, O = 0.0f;
        if (M != -INFINITY) {
            for (int sp = 0; sp < a.splits; ++sp) {
                const int64_t pi = ((int64_t)rh * a.splits + sp) * G + g;
                const float f = exp2f(__ldcg(a.part_ml + pi * 2) - M);
                L += __ldcg(a.part_ml + pi * 2 + 1) * f;
                O += __ldcg(a.part_o + pi * 128 + e) * f;
            }
        }
        static_cast<T*>(a.out)[((int64_t)r * a.Hq + h * G + g) * 128 + e] = from_f32<T>(L > 0.0f ? O / L : 0.0f);
    }
}

struct DecodePlan {
    int grid, splits, span, smem;
    int64_t keys_bytes, part_o_bytes, part_ml_bytes, scratch_bytes, counters;
};

int64_t r256(int64_t x) { return (x + 255) / 256 * 256; }

template <typename T, int G>
int occupancy_blocks(int smem) {
    int per_sm = 0;
    if (smem > 40 * 1024 && cudaFuncSetAttribute(fused_decode_kernel<T, G>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fused_decode_kernel<T, G>, kDecThreads, smem) !=
        cudaSuccess)
        return 0;
    return per_sm;
}

DecodePlan plan_decode(int64_t R, int64_t Hkv, int64_t G, int64_t N, int64_t cap, int64_t width, int sms,
                       int per_sm) {
    DecodePlan p;
    const int64_t list_smem = ((N * 8 + 15) / 16) * 16 + ((32 * cap + width) * 4 + 15) / 16 * 16 +
                              2 * kDecChunk * 2 * 128 * 2;
    const int64_t red_smem = 16 * G * 128 * 4 + 16 * G * 2 * 4;
    p.smem = (int)(list_smem > red_smem ? list_smem : red_smem);
    const int64_t resident = (int64_t)sms * (per_sm > 0 ? per_sm : 1);
    int64_t splits = resident / (R * Hkv);
    if (splits < 1) splits = 1;
    if (splits > 64) splits = 64;
    p.splits = (int)splits;
    p.span = (int)((width + splits - 1) / splits);
    int64_t units = R * Hkv * splits;
    p.grid = (int)(units < resident ? resident : units);
    if (p.grid > resident) p.grid = (int)resident;
    p.keys_bytes = r256(R * N * 8);
    p.part_o_bytes = r256(R * Hkv * splits * G * 128 * 4);
    p.part_ml_bytes = r256(R * Hkv * splits * G * 2 * 4);
    p.scratch_bytes = p.keys_bytes + p.part_o_bytes + p.part_ml_bytes;
    p.counters = 2 + R * Hkv + 1;  // barrier (arrivals, departures), tickets, status
    return p;
}

int sm_count() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

}  // namespace
}  // namespace lsa

using namespace lsa;

extern "C" {

int lsa_decode_fused_plan(int64_t R, int64_t Hq, int64_t Hkv, int64_t N, int64_t cap, int64_t width,
                          int64_t* scratch_bytes, int64_t* n_counters) {
    if (R <= 0 || R > kDecMaxRows || Hkv <= 0 || Hq % Hkv || N < 0 || cap <= 0) return LSA_ERR_ARG;
    const int64_t G = Hq / Hkv;
    if (G != 4 && G != 8) return LSA_ERR_ARG;
    DecodePlan p = plan_decode(R, Hkv, G, N, cap, width, sm_count(), 1);
    if (scratch_bytes) *scratch_bytes = p.scratch_bytes;
    if (n_counters) *n_counters = p.counters;
    return LSA_OK;
}

int lsa_decode_fused(const void* index_queries, int64_t R, int64_t ldq, const void* centroids, int64_t N, int64_t d,
                     const int32_t* members, int64_t cap, const int32_t* positions, int64_t block, int64_t bpb,
                     int64_t top_p, int64_t window, int64_t sink, int64_t top_k, const void* q, const void* k,
                     const void* v, int dtype, int64_t Tk, int64_t Hq, int64_t Hkv, int64_t D, float scale, void* out,
                     int32_t* lists, int32_t* lengths, void* scratch, int64_t scratch_bytes, int32_t* counters,
                     int64_t n_counters, cudaStream_t stream) {
    if (R <= 0 || R > kDecMaxRows || D != 128 || Hkv <= 0 || Hq % Hkv || d <= 0 || d % 8 || ldq < d) return LSA_ERR_ARG;
    if (top_p <= 0 || top_p > 32 || cap <= 0 || cap % 4 || block <= 0 || top_k < 0 || window < 0 || sink < 0)
        return LSA_ERR_ARG;
    if (((uintptr_t)members & 15) != 0) return LSA_ERR_ARG;
    if ((lists == nullptr) != (lengths == nullptr) || Tk > INT32_MAX) return LSA_ERR_ARG;
    if (dtype != kBF16 && dtype != kF16) return LSA_ERR_ARG;
    auto al16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
    if (!al16(index_queries) || !al16(centroids) || !al16(q) || !al16(k) || !al16(v) || !al16(out) ||
        !al16(scratch))
        return LSA_ERR_ARG;
    const int64_t G = Hq / Hkv;
    if (G != 4 && G != 8) return LSA_ERR_ARG;
    const int64_t width = top_k + window + sink;
    const int sms = sm_count();
    DecodePlan p0 = plan_decode(R, Hkv, G, N, cap, width, sms, 1);
    int per_sm = 0;
#define LSA_DEC_OCC(TT, GG) per_sm = occupancy_blocks<TT, GG>(p0.smem)
    if (dtype == kBF16) {
        if (G == 4) LSA_DEC_OCC(__nv_bfloat16, 4); else LSA_DEC_OCC(__nv_bfloat16, 8);
    } else {
        if (G == 4) LSA_DEC_OCC(__half, 4); else LSA_DEC_OCC(__half, 8);
    }
#undef LSA_DEC_OCC
    if (per_sm <= 0) return LSA_ERR_ARG;  // the list / merge buffers do not fit one CTA
    // the plan sized from one CTA per SM is the scratch the caller allocated
    DecodePlan p = p0;
    if (scratch_bytes < p.scratch_bytes || n_counters < p.counters || counters == nullptr) return LSA_ERR_ARG;
    char* w = (char*)scratch;
    FusedDecodeArgs a;
    a.iq = (const __nv_bfloat16*)index_queries;
    a.ldq = ldq;
    a.d = (int)d;
    a.cent = (const __nv_bfloat16*)centroids;
    a.N = N;
    a.members = members;
    a.cap = (int)cap;
    a.positions = positions;
    a.block = block;
    a.bpb = bpb;
    a.top_p = (int)top_p;
    a.window = (int)window;
    a.sink = (int)sink;
    a.top_k = (int)top_k;
    a.width = (int)width;
    a.q = q;
    a.k = k;
    a.v = v;
    a.Tk = Tk;
    a.R = (int)R;
    a.Hq = (int)Hq;
    a.Hkv = (int)Hkv;
    a.splits = p.splits;
    a.span = p.span;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.out = out;
    a.lists = lists;
    a.lengths = lengths;
    a.keys = (int64_t*)w;
    a.part_o = (float*)(w + p.keys_bytes);
    a.part_ml = (float*)(w + p.keys_bytes + p.part_o_bytes);
    a.bar = (uint32_t*)counters;
    a.tickets = counters + 2;
    a.status = counters + 2 + R * Hkv;
    void* args[] = {&a};
    cudaError_t e;
#define LSA_DEC_LAUNCH(TT, GG)                                                                                \
    do {                                                                                                    \
        auto kern = fused_decode_kernel<TT, GG>;                                                            \
        if (p.smem > 40 * 1024 &&                                                                           \
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem) != cudaSuccess) \
            return LSA_ERR_CUDA;                                                                            \
        e = cudaLaunchCooperativeKernel((const void*)kern, dim3(p.grid), dim3(kDecThreads), args, p.smem,   \
                                        stream);                                                            \
    } while (0)
    if (dtype == kBF16) {
        if (G == 4) LSA_DEC_LAUNCH(__nv_bfloat16, 4); else LSA_DEC_LAUNCH(__nv_bfloat16, 8);
    } else {
        if (G == 4) LSA_DEC_LAUNCH(__half, 4); else LSA_DEC_LAUNCH(__half, 8);
    }
#undef LSA_DEC_LAUNCH
    if (e != cudaSuccess) {
        cudaGetLastError();
        return LSA_ERR_CUDA;
    }
    return LSA_OK;
}

}  // extern "C"
