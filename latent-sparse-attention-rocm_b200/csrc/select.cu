// select.cu - bucket scoring, packed-key top-k and the rank-order expansion (sm_100a).
//
// Reference (AIwork4me/latent-sparse-attention-rocm, paths inside that project):
//   scores            src/lsa_rocm_lab/port/pipeline.py:217-232 (_production_scores)
//   listing + top-k   pipeline.py:189-214, 248-271; select_fused.py:52-137
//   expansion walk    select_fused.py:140-280 (upstream _expand_in_order semantics)
//
// Three arms, byte-identical by construction (LSA_SELECT_IMPL):
//   reference    : scores -> pack (listing) -> best-first top-k -> unpack -> expand
//   fused_unpack : scores -> pack -> best-first top-k -> expand reading the keys
//   fused        : ONE launch from index queries to read lists: the CTAs of a row's
//                  thread-block cluster score slices of the buckets into the leader CTA's
//                  shared memory, which orders the packed keys and walks the expansion
//                  (rows wider than one cluster: the last CTA by atomic ticket does it).
#include <cooperative_groups.h>

#include <type_traits>

#include "common.cuh"
#include "topk.cuh"
#include "umma.cuh"
#include "walk.cuh"

namespace cg = cooperative_groups;

namespace lsa {

constexpr int kSortCap = 8192;  // keys sorted in one shared-memory pass (64 KB)

// Programmatic dependent launch: a kernel launched with programmatic stream serialization
// may start while the previous kernel runs; griddepcontrol.wait blocks until that kernel
// has completed and its memory is visible, launch_dependents lets the next kernel start.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------ scoring

// scores[r, n] = cdot(q_r, c_n) for n < N. One warp per column; the query row's lane
// chunks stay in registers for all the CTA's columns.
template <typename TQ, typename TC, int CHUNKS>
__global__ void __launch_bounds__(256) scores_kernel(const TQ* __restrict__ q, int64_t ldq, const TC* __restrict__ c,
                                                     int64_t N, int d, float* __restrict__ out, int64_t ldo,
                                                     int cols_per_cta) {
    int r = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int nchunks = d >> 3;
    float x[CHUNKS][8];
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
        int ch = lane + 32 * j;
        if (ch < nchunks) load8<TQ>(q + r * ldq + (size_t)ch * 8, x[j]);
    }
    int64_t c0 = (int64_t)blockIdx.x * cols_per_cta;
    int64_t c1 = min(c0 + cols_per_cta, N);
    for (int64_t n = c0 + warp; n < c1; n += blockDim.x >> 5) {
        float p = lane_partial_regs<TC, CHUNKS>(x, c + n * d, lane, nchunks);
        p = butterfly_sum(p);
        if (lane == 0) out[r * ldo + n] = p;
    }
}

__global__ void visible_counts_kernel(const int32_t* positions, int64_t R, int64_t block, int64_t bpb, int64_t rows,
                                      int32_t* counts) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < R) {
        int64_t v = (int64_t)positions[i] / block * bpb;
        counts[i] = (int32_t)(v < rows ? v : rows);
    }
}

// Tile queries of the prefill arm: tq[t, j] = fp32 sum over the tile's rows, in row order,
// of the bf16-rounded index query element (one thread per column j).
template <typename T>
__global__ void tile_queries_kernel(const T* __restrict__ iq, int64_t R, int64_t ldq, int64_t d, int64_t tile,
                                    float* __restrict__ out) {
    int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t t = blockIdx.y;
    if (j >= d) return;
    int64_t r1 = min((t + 1) * tile, R);
    float acc = 0.0f;
#pragma unroll 16
    for (int64_t r = t * tile; r < r1; ++r)  // loads run ahead; the adds stay in row order
        acc = __fadd_rn(acc, __bfloat162float(__float2bfloat16_rn(to_f32(iq[r * ldq + j]))));
    out[t * d + j] = acc;
}

__global__ void pack_keys_kernel(const float* __restrict__ s, int64_t R, int64_t N, int64_t lds,
                                 const int32_t* __restrict__ lengths, int64_t* __restrict__ keys, int64_t ldk) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= R * N) return;
    int64_t r = i / N, n = i % N;
    keys[r * ldk + n] = n < lengths[r] ? pack_key(s[r * lds + n], (int32_t)n) : kEmpty;
}

__global__ void unpack_kernel(const int64_t* __restrict__ keys, int64_t n, int32_t* __restrict__ ids) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) ids[i] = key_bucket(keys[i]);
}

// ------------------------------------------------------------------ positional arm

// The positional decode arm's static picks: of a row's visible buckets v = min(rows,
// pos / block * bpb), the first `first`, the last `last`, and top_p - first - last strided
// ones in between (bucket first + floor(i * (v - first - last) / n_mid)), ascending and
// unique, -1 padded; v <= top_p: every visible bucket.
__global__ void positional_picks_kernel(const int32_t* __restrict__ positions, int64_t R, int64_t block, int64_t bpb,
                                        int64_t rows, int top_p, int first, int last, int32_t* __restrict__ picks) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= R) return;
    int64_t v = (int64_t)positions[r] / block * bpb;
    if (v > rows) v = rows;
    if (v < 0) v = 0;
    int32_t* out = picks + r * top_p;
    int n = 0;
    if (v <= top_p) {
        for (int64_t b = 0; b < v; ++b) out[n++] = (int32_t)b;
    } else {
        const int mid = top_p - first - last;
        const int64_t span = v - first - last;
        for (int i = 0; i < first; ++i) out[n++] = i;
        int64_t prev = first - 1;
        for (int i = 0; i < mid; ++i) {
            const int64_t b = first + (int64_t)i * span / mid;
            if (b > prev && b < v - last) {
                out[n++] = (int32_t)b;
                prev = b;
            }
        }
        for (int i = 0; i < last; ++i) out[n++] = (int32_t)(v - last + i);
    }
    for (; n < top_p; ++n) out[n] = -1;
}

// ------------------------------------------------------------------ top-k

// Loader interface: key(n) for n < N. Sorted top-k of N keys into out[0..k) (EMPTY past N).
// Shared: kSortCap int64. When N fits the buffer: one bitonic sort. Otherwise the running
// best k2 = next_pow2(k) keys are kept at the front and merged with successive chunks.
template <typename Loader>
__device__ void block_topk(const Loader& key, int N, int k, int64_t* sbuf, int64_t* out, int ldo_k) {
    int n2 = next_pow2(max(N, 1));
    if (n2 <= kSortCap) {
        for (int i = threadIdx.x; i < n2; i += blockDim.x) sbuf[i] = i < N ? key(i) : kEmpty;
        __syncthreads();
        bitonic_sort_desc(sbuf, n2);
        for (int i = threadIdx.x; i < ldo_k; i += blockDim.x) out[i] = i < k ? sbuf[i] : kEmpty;
        __syncthreads();
        return;
    }
    int k2 = next_pow2(k);
    int chunk = kSortCap - k2;
    for (int i = threadIdx.x; i < k2; i += blockDim.x) sbuf[i] = kEmpty;
    for (int start = 0; start < N; start += chunk) {
        __syncthreads();
        for (int i = threadIdx.x; i < chunk; i += blockDim.x) sbuf[k2 + i] = start + i < N ? key(start + i) : kEmpty;
        __syncthreads();
        bitonic_sort_desc(sbuf, kSortCap);
    }
    for (int i = threadIdx.x; i < ldo_k; i += blockDim.x) out[i] = i < k ? sbuf[i] : kEmpty;
    __syncthreads();
}

struct MaskedKeys {
    const int64_t* row;
    int count;  // slots at or past count read as EMPTY (upstream TopK.best()'s ~listed mask)
    __device__ int64_t operator()(int i) const { return i < count ? row[i] : kEmpty; }
};

struct PackedScores {
    const float* row;
    int live;
    __device__ int64_t operator()(int i) const { return i < live ? pack_key(row[i], i) : kEmpty; }
};

// best_first_keys (pipeline.py:189-214): masked, sorted descending, k = min(top_p, N).
__global__ void __launch_bounds__(1024) best_first_kernel(const int64_t* __restrict__ keys, int64_t N, int64_t ldk,
                                                          int k, const int32_t* __restrict__ counts,
                                                          int64_t* __restrict__ out, int64_t ldo) {
    extern __shared__ int64_t sbuf[];
    int r = blockIdx.x;
    int cnt = counts ? min((int64_t)counts[r], N) : (int)N;
    cnt = max(cnt, 0);
    MaskedKeys loader{keys + r * ldk, cnt};
    block_topk(loader, (int)N, k, sbuf, out + r * ldo, (int)ldo);
}

// select_topk_scores (select_fused.py:52-80): scores -> K2 greatest packed keys.
__global__ void __launch_bounds__(1024) select_topk_kernel(const float* __restrict__ s, int64_t N, int64_t lds,
                                                           const int32_t* __restrict__ lengths, int k,
                                                           int64_t* __restrict__ out, int64_t ldo) {
    extern __shared__ int64_t sbuf[];
    int r = blockIdx.x;
    int live = (int)min((int64_t)max(lengths[r], 0), N);
    PackedScores loader{s + r * lds, live};
    block_topk(loader, (int)N, k, sbuf, out + r * ldo, (int)ldo);
}

// ------------------------------------------------------------------ expansion

struct PickFromIds {
    const int32_t* row;
    __device__ int32_t operator()(int p) const { return row[p]; }
};
struct PickFromKeys {
    const int64_t* row;
    __device__ int32_t operator()(int p) const { return key_bucket(row[p]); }
};

// The rank-order walk of one row (select_fused.py:172-214) by the whole block:
// slots (pick, member) in walk order; keep ids with sink <= id < window_start; the first
// top_k kept, then the window [window_start, pos] and the sinks [0, min(sink, ws)).
template <typename Picks>
__device__ void expand_row(const Picks& pick_of, int P, const int32_t* __restrict__ members, int64_t member_rows,
                           int cap, int64_t pos, int window, int sink, int top_k, int32_t* __restrict__ out,
                           int width, int32_t* length_out, int* scan_smem) {
    int64_t ws = pos + 1 - window;
    if (ws < 0) ws = 0;
    constexpr int SPT = 4;
    int tile = blockDim.x * SPT;
    int total_slots = P * cap;
    int filled = 0;
    for (int t0 = 0; t0 < total_slots && filled < top_k; t0 += tile) {
        int ids[SPT];
        int cnt = 0;
#pragma unroll
        for (int e = 0; e < SPT; ++e) {
            int s = t0 + threadIdx.x * SPT + e;
            int id = -1;
            if (s < total_slots) {
                int p = s / cap, m = s - p * cap;
                int b = pick_of(p);
                if (b >= 0 && b < member_rows) {
                    int v = members[(int64_t)b * cap + m];
                    if (v >= sink && v < ws) id = v;
                }
            }
            ids[e] = id;
            cnt += id >= 0;
        }
        int total;
        int at = filled + block_exclusive_scan(cnt, scan_smem, &total);
#pragma unroll
        for (int e = 0; e < SPT; ++e) {
            if (ids[e] >= 0) {
                if (at < top_k) out[at] = ids[e];
                ++at;
            }
        }
        filled += total;
    }
    if (filled > top_k) filled = top_k;
    int nwin = (int)(pos - ws + 1);
    if (nwin < 0) nwin = 0;
    int nsink = (int)(sink < ws ? sink : ws);
    int length = filled + nwin + nsink;
    for (int i = threadIdx.x; i < width - filled; i += blockDim.x) {
        int j = filled + i, v = -1;
        if (i < nwin) v = (int)(ws + i);
        else if (i < nwin + nsink) v = i - nwin;
        out[j] = v;
    }
    if (threadIdx.x == 0) *length_out = length;
}

template <typename PickT>
__global__ void __launch_bounds__(512) expand_kernel(const PickT* __restrict__ picks, int P, int64_t ldp,
                                                     const int32_t* __restrict__ members, int64_t member_rows, int cap,
                                                     const int32_t* __restrict__ positions, int window, int sink,
                                                     int top_k, int32_t* __restrict__ lists,
                                                     int32_t* __restrict__ lengths) {
    __shared__ int scan_smem[33];
    pdl_wait();  // the picks are the previous kernel's output
    pdl_trigger();
    int r = blockIdx.x;
    int width = top_k + window + sink;
    if constexpr (sizeof(PickT) == 8) {
        PickFromKeys pk{reinterpret_cast<const int64_t*>(picks) + r * ldp};
        expand_row(pk, P, members, member_rows, cap, positions[r], window, sink, top_k, lists + (int64_t)r * width,
                   width, lengths + r, scan_smem);
    } else {
        PickFromIds pk{reinterpret_cast<const int32_t*>(picks) + r * ldp};
        expand_row(pk, P, members, member_rows, cap, positions[r], window, sink, top_k, lists + (int64_t)r * width,
                   width, lengths + r, scan_smem);
    }
}

// ------------------------------------------------------------------ fused select

struct SmemPicks {
    const int64_t* keys;
    __device__ int32_t operator()(int p) const { return key_bucket(keys[p]); }
};

struct GlobalKeysCg {
    const int64_t* row;
    int count;
    __device__ int64_t operator()(int i) const { return i < count ? __ldcg(row + i) : kEmpty; }
};

// Where a selection row stands. Token rows (tile == 0) use positions[r] for both the
// visible count and the walk. Tile rows (tile > 0, the prefill arm) are the query tiles
// [r * tile, (r + 1) * tile): the visible count is taken at the tile's first row and the
// walk runs at the virtual position block_start - 1 with window 0, so a tile's list holds
// the picked members of closed blocks and the sinks below the tile's open block.
// Ragged batches (one sequence per row, e.g. batched decode): row r's buckets are rows
// [table_off[r], table_off[r] + table_rows[r]) of concatenated centroid / member tables;
// null tables: every row reads the whole table.
struct RowPos {
    const int32_t* positions;
    int64_t tile, block;
    const int64_t* table_off;
    const int32_t* table_rows;
    __device__ __forceinline__ int64_t count_pos(int r) const { return tile ? r * tile : (int64_t)positions[r]; }
    __device__ __forceinline__ int64_t walk_pos(int r) const {
        return tile ? r * tile / block * block - 1 : (int64_t)positions[r];
    }
    __device__ __forceinline__ int64_t off(int r) const { return table_off ? table_off[r] : 0; }
    __device__ __forceinline__ int64_t rows(int r, int64_t N) const {
        return table_rows ? (int64_t)table_rows[r] : N;
    }
};

constexpr int kFusedThreads = 512;
constexpr int kDecodeMaxD = 2048;  // index dims the decode select stages for a built query
// the raw element type of a built query (GroupMean<T, RB> -> T; other query types: a stand-in)
template <typename TQ> struct QRawOf {
    using type = __nv_bfloat16;
};
template <typename T, bool RB> struct QRawOf<GroupMean<T, RB>> {
    using type = T;
};
constexpr int kMemberPrefetch = 8192;  // member slots staged in shared memory in one round trip
constexpr int kGatherMax = 8192;       // read-list slots the fused selects gather in shared memory

// Descending bitonic sort of one key per thread across the block (blockDim.x a power of
// two); returns the key of rank threadIdx.x. Strides below 32 exchange by warp shuffles,
// larger strides through shared memory (xchg: blockDim.x int64).
__device__ __forceinline__ int64_t block_bitonic_desc_regs(int64_t x, int64_t* xchg) {
    const int tid = threadIdx.x, n = blockDim.x;
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            int64_t y;
            if (j >= 32) {
                xchg[tid] = x;
                __syncthreads();
                y = xchg[tid ^ j];
                __syncthreads();
            } else {
                y = __shfl_xor_sync(0xFFFFFFFFu, x, j);
            }
            bool lower = (tid & j) == 0;
            bool desc = (tid & k) == 0;
            x = (lower == desc) ? (x > y ? x : y) : (x < y ? x : y);
        }
    }
    return x;
}

struct BlockSync {
    __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

// The walk of expand_row with every picked bucket's member row staged in shared memory
// first (one memory round trip), then expand_walk over all (pick, member) slots. A block of
// kFusedThreads threads. Requires P * cap <= kMemberPrefetch; mem (16-byte aligned) holds
// that many int32; gather (optional, top_k int32) collects the kept ids for one coalesced
// copy out.
__device__ void expand_row_prefetched(const int64_t* picks, int P, const int32_t* __restrict__ members,
                                      int64_t member_rows, int cap, int64_t pos, int window, int sink, int top_k,
                                      int32_t* __restrict__ out, int width, int32_t* length_out, int* scan_smem,
                                      int* mem, int* gather = nullptr) {
    const int total = P * cap;
    // addresses first, then every member load of this thread in flight together, then the
    // stores: one memory round trip for the whole staging
    constexpr int kMaxPer = kMemberPrefetch / kFusedThreads;
    const int32_t* src[kMaxPer];
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
        int s = threadIdx.x + i * kFusedThreads;
        src[i] = nullptr;
        if (s < total) {
            int p = s / cap, m = s - p * cap;
            int b = key_bucket(picks[p]);
            if (b >= 0 && b < member_rows) src[i] = members + (int64_t)b * cap + m;
        }
    }
    int vals[kMaxPer];
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) vals[i] = src[i] ? __ldg(src[i]) : -1;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
        int s = threadIdx.x + i * kFusedThreads;
        if (s < total) mem[s] = vals[i];
    }
    __syncthreads();
    expand_walk<kFusedThreads>(mem, total, pos, window, sink, top_k, out, width, length_out, scan_smem,
                               (int)threadIdx.x, BlockSync{}, gather);
}

// The same walk with every picked member row staged in shared memory first (16-byte
// cp.async pieces when cap % 4 == 0 and the table is 16-byte aligned, else plain loads):
// one memory round trip instead of two per 2048-slot tile, then expand_walk with its output
// gathered in shared memory. Dynamic smem: round4(P * cap) + top_k ints.
template <typename PickT>
__global__ void __launch_bounds__(512) expand_staged_kernel(const PickT* __restrict__ picks, int P, int64_t ldp,
                                                            const int32_t* __restrict__ members, int64_t member_rows,
                                                            int cap, const int32_t* __restrict__ positions, int window,
                                                            int sink, int top_k, int32_t* __restrict__ lists,
                                                            int32_t* __restrict__ lengths, int vec16) {
    extern __shared__ __align__(16) int esm[];
    __shared__ int scan_smem[33];
    pdl_wait();  // the picks are the previous kernel's output
    pdl_trigger();
    const int total = P * cap;
    int* mem = esm;
    int* gather = esm + ((total + 3) & ~3);
    const int r = blockIdx.x, tid = threadIdx.x;
    const PickT* prow = picks + (int64_t)r * ldp;
    auto bucket = [&](int p) -> int {
        if constexpr (sizeof(PickT) == 8) return key_bucket((int64_t)prow[p]);
        else return (int)prow[p];
    };
    if (vec16) {
        const int q4 = cap / 4;
        for (int i = tid; i < P * q4; i += blockDim.x) {
            const int pk = i / q4, piece = i - pk * q4;
            const int b = bucket(pk);
            int* dst = mem + pk * cap + piece * 4;
            if (b >= 0 && b < member_rows) cp_async16(smem_u32(dst), members + (int64_t)b * cap + piece * 4, 16);
            else *reinterpret_cast<int4*>(dst) = make_int4(-1, -1, -1, -1);
        }
        cp_async_wait_all();
    } else {
        for (int s = tid; s < total; s += blockDim.x) {
            const int pk = s / cap, m = s - pk * cap;
            const int b = bucket(pk);
            mem[s] = (b >= 0 && b < member_rows) ? members[(int64_t)b * cap + m] : -1;
        }
    }
    __syncthreads();
    const int width = top_k + window + sink;
    expand_walk<512>(mem, total, positions[r], window, sink, top_k, lists + (int64_t)r * width, width, lengths + r,
                     scan_smem, tid, BlockSync{}, gather);
}

// One launch from index queries to read lists. grid = (chunks, R), block = 512: every
// warp scores one visible column; the last CTA of a row (atomic ticket) orders the row's
// packed keys (register bitonic up to 512 keys) and walks the expansion.
// Scratch: keys [R, N] int64; counters: tickets [R] int32 (zero before the first launch; the
// last CTA of a row resets its ticket, so launches replay, e.g. from a CUDA graph).
// Launched with programmatic stream serialization: griddepcontrol.wait precedes every read.
template <typename TQ, typename TC, int CHUNKS>
__global__ void __launch_bounds__(kFusedThreads) select_fused_kernel(
    const TQ* __restrict__ q, int64_t ldq, const TC* __restrict__ c, int64_t N, int d,
    RowPos rp, int64_t block, int64_t bpb, int cols_per_cta, int top_p,
    const int32_t* __restrict__ members, int cap, int window, int sink, int top_k, int32_t* __restrict__ lists,
    int32_t* __restrict__ lengths, int64_t* __restrict__ ws_keys, int32_t* __restrict__ tickets) {
    extern __shared__ int64_t sbuf[];
    __shared__ int64_t slists[kFusedThreads];
    __shared__ int scan_smem[33];
    __shared__ int is_last;
    pdl_wait();
    pdl_trigger();
    int r = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t Nr = rp.rows(r, N);  // this row's bucket count (N: the key stride)
    const TC* cr = c + rp.off(r) * d;
    const int32_t* mr = members + rp.off(r) * cap;
    // score the grid's columns without waiting for the row's position: the last CTA masks
    // the columns past the row's visible count (the grid covers the widest row)
    int64_t c0 = (int64_t)blockIdx.x * cols_per_cta;
    int64_t c1 = min(c0 + cols_per_cta, Nr);
    if (c0 < c1) {
        int nchunks = d >> 3;
        float x[CHUNKS][8];
#pragma unroll
        for (int j = 0; j < CHUNKS; ++j) {
            int ch = lane + 32 * j;
            if (ch < nchunks) load8<TQ>(q + r * ldq + (size_t)ch * 8, x[j]);
        }
        // four columns per warp per pass, their centroid loads in flight together; each row
        // starts at its own column offset so concurrent rows do not all read the same lines
        const int nw = blockDim.x >> 5;
        const int64_t span = c1 - c0, rot = ((int64_t)r * 97) % span;
        for (int64_t i0 = warp; i0 < span; i0 += 4 * nw) {
            float part[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int64_t ii = i0 + (int64_t)i * nw;
                const int64_t n = c0 + (ii + rot < span ? ii + rot : ii + rot - span);
                part[i] = ii < span ? lane_partial_regs<TC, CHUNKS>(x, cr + n * d, lane, nchunks) : 0.0f;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int64_t ii = i0 + (int64_t)i * nw;
                const int64_t n = c0 + (ii + rot < span ? ii + rot : ii + rot - span);
                const float p = butterfly_sum(part[i]);
                if (ii < span && lane == 0) ws_keys[r * N + n] = pack_key(p, (int32_t)n);
            }
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = atomicAdd(tickets + r, 1);
        is_last = (t == (int)gridDim.x - 1);
        if (is_last) tickets[r] = 0;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    int64_t pos = rp.walk_pos(r);
    int64_t vis = rp.count_pos(r) / block * bpb;
    int count = (int)(vis < Nr ? vis : Nr);
    if (count < 0) count = 0;
    int k = (int)min((int64_t)top_p, Nr);
    GlobalKeysCg loader{ws_keys + r * N, count};
    int n2 = next_pow2(max(count, 1));
    int64_t* picks = sbuf;  // sorted keys live at the front of the buffer
    if (k <= 32 && count <= 4 * (int)blockDim.x) {
        // top-32: warp sorts + merge tree over the keys staged in shared memory
        for (int i = threadIdx.x; i < count; i += blockDim.x) sbuf[i] = loader(i);
        __syncthreads();
        block_top32_desc(sbuf, count, slists, slists);
        if ((int)threadIdx.x < 32) picks[threadIdx.x] = slists[threadIdx.x];
        __syncthreads();
    } else if (count <= (int)blockDim.x) {
        int64_t x = block_bitonic_desc_regs(loader((int)threadIdx.x), sbuf);
        __syncthreads();  // the exchange buffer becomes the picks
        if ((int)threadIdx.x < k) picks[threadIdx.x] = x;
        for (int i = blockDim.x + threadIdx.x; i < k; i += blockDim.x) picks[i] = kEmpty;
        __syncthreads();
    } else if (n2 <= kSortCap) {
        // every live key sits below n2; picks in [n2, k) stay EMPTY
        int fill = n2 > k ? n2 : k;
        for (int i = threadIdx.x; i < fill; i += blockDim.x) sbuf[i] = loader(i);
        __syncthreads();
        bitonic_sort_desc(sbuf, n2);
    } else {
        block_topk(loader, count, k, sbuf, sbuf, k);  // in-place: out aliases the buffer front
    }
    int width = top_k + window + sink;
    if (k * cap <= kMemberPrefetch) {
        int* mem = reinterpret_cast<int*>(sbuf + ((k + 1) & ~1));  // 16-byte aligned
        int* gather = top_k <= kGatherMax ? mem + (k * cap + 3) / 4 * 4 : nullptr;
        expand_row_prefetched(picks, k, mr, Nr, cap, pos, window, sink, top_k, lists + (int64_t)r * width, width,
                              lengths + r, scan_smem, mem, gather);
    } else {
        SmemPicks pk{picks};
        expand_row(pk, k, mr, Nr, cap, pos, window, sink, top_k, lists + (int64_t)r * width, width, lengths + r,
                   scan_smem);
    }
}

// ------------------------------------------------------------------ top-32 by warps

// ------------------------------------------------------------------ cluster select

constexpr int kMaxColsPerWarp = 4;  // cluster path: up to 16 CTAs x 16 warps x 4 columns

// One launch from index queries to read lists, one thread-block cluster per row: every
// CTA scores 16 * cpw columns and stores their packed keys straight into the shared
// memory of the cluster's rank-0 CTA (distributed shared memory: no global round trip,
// no fence, no ticket), prefetching the scored buckets' member rows into L2 on the way;
// after one cluster barrier the leader orders the keys (warp sorts + merge tree for
// top_p <= 32) and walks the expansion. grid = (cluster size, R); block = 512.
template <typename TQ, typename TC, int CHUNKS>
__global__ void __launch_bounds__(kFusedThreads) select_cluster_kernel(
    const TQ* __restrict__ q, int64_t ldq, const TC* __restrict__ c, int64_t N, int d,
    RowPos rp, int64_t block, int64_t bpb, int cpw, int top_p,
    const int32_t* __restrict__ members, int cap, int window, int sink, int top_k, int32_t* __restrict__ lists,
    int32_t* __restrict__ lengths) {
    extern __shared__ int64_t sbuf[];
    __shared__ int64_t slists[kFusedThreads];
    __shared__ int scan_smem[33];
    pdl_wait();
    pdl_trigger();
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int r = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int64_t Nr = rp.rows(r, N);  // this row's bucket count
    const TC* cr = c + rp.off(r) * d;
    const int32_t* mr = members + rp.off(r) * cap;
    const int cols_per_cta = nw * cpw;
    const int64_t c0 = (int64_t)rank * cols_per_cta;
    // column n's key lands at sbuf[n] of the cluster's rank-0 CTA: every CTA stores its keys
    // there through distributed shared memory before the one cluster barrier
    int64_t* lead_keys = cluster.map_shared_rank(sbuf, 0);
    {
        int nchunks = d >> 3;
        float x[CHUNKS][8];
#pragma unroll
        for (int j = 0; j < CHUNKS; ++j) {
            int ch = lane + 32 * j;
            if (ch < nchunks) load8<TQ>(q + r * ldq + (size_t)ch * 8, x[j]);
        }
        float part[kMaxColsPerWarp];
        const int lines = (cap * 4 + 127) / 128;  // 128-byte lines of one member row
#pragma unroll
        for (int i = 0; i < kMaxColsPerWarp; ++i) {  // every column's loads in flight together
            int64_t n = c0 + warp + nw * i;
            bool live = i < cpw && n < Nr;
            part[i] = live ? lane_partial_regs<TC, CHUNKS>(x, cr + n * d, lane, nchunks) : 0.0f;
            // the leader reads the picked buckets' member rows next: pull every scored
            // bucket's row into L2 now
            if (live && lane < lines)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(mr + n * cap + lane * 32));
        }
#pragma unroll
        for (int i = 0; i < kMaxColsPerWarp; ++i) {
            int64_t n = c0 + warp + nw * i;
            if (i < cpw && n < Nr) {
                float p = butterfly_sum(part[i]);
                if (lane == 0) lead_keys[n] = pack_key(p, (int32_t)n);
            }
        }
    }
    cluster.sync();  // every column's key is in the leader's shared memory
    if (rank != 0) return;
    const int k = (int)min((int64_t)top_p, Nr);
    const int64_t pos = rp.walk_pos(r);
    int64_t vis = rp.count_pos(r) / block * bpb;
    int count = (int)(vis < Nr ? vis : Nr);
    if (count < 0) count = 0;
    const int n2 = next_pow2(max(count, 1));
    for (int t = count + threadIdx.x; t < max(n2, k); t += blockDim.x) sbuf[t] = kEmpty;  // unseen columns
    __syncthreads();
    int64_t* picks = sbuf;
    if (k <= 32 && count <= (int)blockDim.x * 4) {
        block_top32_desc(sbuf, count, slists, slists);
        if ((int)threadIdx.x < 32) picks[threadIdx.x] = slists[threadIdx.x];  // k <= 32: EMPTY tail past k
        __syncthreads();
    } else {
        bitonic_sort_desc(sbuf, n2);
    }
    int width = top_k + window + sink;
    if (k * cap <= kMemberPrefetch) {
        int* mem = reinterpret_cast<int*>(sbuf + ((max(k, 32) + 1) & ~1));  // 16-byte aligned
        int* gather = top_k <= kGatherMax ? mem + (k * cap + 3) / 4 * 4 : nullptr;
        expand_row_prefetched(picks, k, mr, Nr, cap, pos, window, sink, top_k, lists + (int64_t)r * width, width,
                              lengths + r, scan_smem, mem, gather);
    } else {
        SmemPicks pk{picks};
        expand_row(pk, k, mr, Nr, cap, pos, window, sink, top_k, lists + (int64_t)r * width, width, lengths + r,
                   scan_smem);
    }
}

// ------------------------------------------------------------------ decode select (latency path)

// Rows of up to 16 x 16 x CPW visible buckets with top_p <= 32 (single-sequence decode):
// one cluster of <= 16 CTAs per row, laid out so the chain after the previous kernel is as
// short as it can be:
//   * before griddepcontrol.wait every warp pulls its columns' centroid rows and member rows
//     into L2 (prefetch only: the index is not produced by the kernel this one overlaps,
//     but a hint cannot read stale data either way), so the scoring loads after the wait
//     hit L2 instead of HBM;
//   * after the wait, each warp issues the query and all its columns' centroid loads before
//     the first FMA (canonical cdot: lane = chunk mod 32, fp32 fma chain in chunk order,
//     butterfly), masks columns past the row's visible count to EMPTY, and each CTA sorts
//     its own 16 CPW keys into one descending 32-list (warp bitonic sorts, in parallel
//     across the cluster) that it stores into the leader's shared memory (DSMEM);
//   * one cluster barrier (the other CTAs arrive and leave); the leader's warps merge the
//     sorted lists pairwise (max(A[i], B[31 - i]) is bitonic and holds the top 32; a
//     half-cleaner sorts it) in log2(cluster) levels;
//   * the walk: warp w takes picks w and w + 16, loads their member rows straight into
//     registers (32 slots per load, all loads in flight together), keeps ids in
//     [sink, window_start) by ballots, counts per pick; pick offsets are warp reductions
//     over the 32 counts; every kept id is stored at its offset (capped at top_k), then the
//     window, the sinks and the -1 tail.
// Identical output to select_cluster_kernel (same keys, same order, same walk).
constexpr int kDecodeSelThreads = 512;
constexpr int kDecodeSelWarps = kDecodeSelThreads / 32;
constexpr int kDecodeMaxCap = 128;  // member slots per bucket the walk holds in registers

template <typename TC>
struct RawChunk;  // 8 consecutive elements of a centroid (or query) row, as loaded
template <>
struct RawChunk<__nv_bfloat16> {
    uint4 v;
    __device__ __forceinline__ void load(const __nv_bfloat16* p) { v = __ldg(reinterpret_cast<const uint4*>(p)); }
    __device__ __forceinline__ void get(float (&out)[8]) const {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f = __bfloat1622float2(h[i]);
            out[2 * i] = f.x;
            out[2 * i + 1] = f.y;
        }
    }
};
template <>
struct RawChunk<__half> {
    uint4 v;
    __device__ __forceinline__ void load(const __half* p) { v = __ldg(reinterpret_cast<const uint4*>(p)); }
    __device__ __forceinline__ void get(float (&out)[8]) const {
        const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f = __half22float2(h[i]);
            out[2 * i] = f.x;
            out[2 * i + 1] = f.y;
        }
    }
};
template <>
struct RawChunk<float> {
    float4 a, b;
    __device__ __forceinline__ void load(const float* p) {
        a = __ldg(reinterpret_cast<const float4*>(p));
        b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    }
    __device__ __forceinline__ void get(float (&out)[8]) const {
        out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
        out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
    }
};

__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <typename TQ, typename TC, int CHUNKS, int CPW>
__global__ void __launch_bounds__(kDecodeSelThreads) select_decode_kernel(
    const TQ* __restrict__ q, int64_t ldq, const TC* __restrict__ c, int64_t N, int d, RowPos rp, int64_t block,
    int64_t bpb, int top_p, const int32_t* __restrict__ members, int cap, int window, int sink, int top_k,
    int32_t* __restrict__ lists, int32_t* __restrict__ lengths, QGroup qg) {
    static_assert(CPW == 1 || CPW == 2 || CPW == 4, "16, 32 or 64 columns per CTA");
    __shared__ int64_t lead[16 * 32];           // the cluster's sorted 32-lists (leader's copy is used)
    __shared__ int64_t local[16 * CPW];         // this CTA's keys, column order
    __shared__ int64_t half[32];                // CPW == 4: the second warp's sorted list
    __shared__ int pick_bucket[32], pick_count[32];
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank(), cs = (int)cluster.num_blocks();
    const int r = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t Nr = rp.rows(r, N);
    const int64_t c0 = (int64_t)rank * (kDecodeSelWarps * CPW);
    const int nchunks = d >> 3;
    const int mlines = (cap * 4 + 127) / 128;
    // first cluster phase: every CTA has started before any of them writes the leader's
    // shared memory (waited on just before that store)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    // One table (no per-row offsets, the decode rows): the index is read-only here, and the
    // kernels that write centroids or member rows (the builds, table copies) never trigger
    // their dependents early, so this grid starts only after they completed - the warp's
    // centroid chunks are loaded into registers before griddepcontrol.wait (overlapping the
    // previous kernel, in a decode step the previous layer's read) and its member rows pulled
    // into L2. Only the query, which the previous kernel may produce, is read after the wait.
    // (only where the chunks fit in 32 registers: wider tiles keep the loads after the wait,
    // where the compiler may interleave them with the FMAs instead of spilling)
    constexpr bool kEarlyFits = CPW * CHUNKS * sizeof(RawChunk<TC>) <= 128;
    const bool early = kEarlyFits && rp.table_off == nullptr;
    RawChunk<TC> raw[CPW][CHUNKS];
    if (early && Nr > 0) {
#pragma unroll
        for (int i = 0; i < CPW; ++i) {
            int64_t n = c0 + warp + kDecodeSelWarps * i;
            n = n < Nr ? n : Nr - 1;  // a valid row; masked below
#pragma unroll
            for (int j = 0; j < CHUNKS; ++j) {
                const int ch = min(lane + 32 * j, nchunks - 1);
                raw[i][j].load(c + n * d + (size_t)ch * 8);
            }
            if (n == c0 + warp + kDecodeSelWarps * i && lane < mlines)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(members + n * cap + lane * 32));
        }
    }
    pdl_wait();
    pdl_trigger();
    const TC* cr = c + rp.off(r) * d;
    const int32_t* mr = members + rp.off(r) * cap;
    int64_t vis = rp.count_pos(r) / block * bpb;
    const int64_t count = vis < 0 ? 0 : (vis < Nr ? vis : Nr);
    // ---- scores: every load of the warp in flight before the first FMA
    if (Nr > 0) {  // (block-uniform) loads are unconditional, at clamped valid addresses, so
                   // the compiler issues all of them before the first use
        float x[CHUNKS][8];
        // a built query: thread i (< d / 8) owns index chunk i; its query rows are requested
        // first, ahead of the centroid chunks (held raw, the first kGQ heads of the group)
        constexpr int kGQ = GroupMeanOf<TQ>::value ? (sizeof(typename QRawOf<TQ>::type) == 4 ? 4 : 8) : 1;
        RawChunk<typename QRawOf<TQ>::type> qraw[kGQ];
        const typename QRawOf<TQ>::type* qbase = nullptr;
        if constexpr (GroupMeanOf<TQ>::value) {
            const int i = min((int)threadIdx.x, nchunks - 1);
            const int j0 = i * 8, h = j0 / qg.D, e0 = j0 - h * qg.D;
            qbase = reinterpret_cast<const typename QRawOf<TQ>::type*>(q) + r * ldq + (int64_t)h * qg.G * qg.D + e0;
#pragma unroll
            for (int g = 0; g < kGQ; ++g) qraw[g].load(qbase + (int64_t)min(g, qg.G - 1) * qg.D);
        }
        if constexpr (!GroupMeanOf<TQ>::value) {
#pragma unroll
            for (int j = 0; j < CHUNKS; ++j) {
                const int ch = min(lane + 32 * j, nchunks - 1);
                load8<TQ>(q + r * ldq + (size_t)ch * 8, x[j]);
            }
        }
        if (!early) {
#pragma unroll
            for (int i = 0; i < CPW; ++i) {
                int64_t n = c0 + warp + kDecodeSelWarps * i;
                n = n < Nr ? n : Nr - 1;  // a valid row; masked below
#pragma unroll
                for (int j = 0; j < CHUNKS; ++j) {
                    const int ch = min(lane + 32 * j, nchunks - 1);
                    raw[i][j].load(cr + n * d + (size_t)ch * 8);
                }
            }
        }
        if constexpr (GroupMeanOf<TQ>::value) {
            // the index query from the raw query row (the centroid loads above are in flight):
            // thread i builds chunk i (8 elements of one KV head) in shared memory
            using TR = typename GroupMeanOf<TQ>::raw;
            __shared__ __align__(16) float qsm[kDecodeMaxD];
            if ((int)threadIdx.x < nchunks) {  // (kDecodeMaxD / 8 <= kDecodeSelThreads: one chunk a thread)
                float acc[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
#pragma unroll
                for (int g = 0; g < kGQ; ++g) {
                    if (g < qg.G) {
                        float v[8];
                        qraw[g].get(v);
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(acc[e], v[e]);
                    }
                }
                for (int g = kGQ; g < qg.G; ++g) {  // larger groups: the rest in order
                    float v[8];
                    load8<TR>(qbase + (int64_t)g * qg.D, v);
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[e] = __fadd_rn(acc[e], v[e]);
                }
                const int j0 = threadIdx.x * 8;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    float m = __fdiv_rn(acc[e], (float)qg.G);
                    if (GroupMeanOf<TQ>::round_bf16) m = __bfloat162float(__float2bfloat16_rn(m));
                    qsm[j0 + e] = m;
                }
            }
            __syncthreads();
#pragma unroll
            for (int j = 0; j < CHUNKS; ++j) {
                const int ch = min(lane + 32 * j, nchunks - 1);
                load8<float>(qsm + ch * 8, x[j]);
            }
        }
        float part[CPW];
#pragma unroll
        for (int i = 0; i < CPW; ++i) {
            float p = 0.0f;
#pragma unroll
            for (int j = 0; j < CHUNKS; ++j) {
                if (lane + 32 * j < nchunks) {
                    float y[8];
                    raw[i][j].get(y);
#pragma unroll
                    for (int e = 0; e < 8; ++e) p = __fmaf_rn(x[j][e], y[e], p);
                }
            }
            part[i] = p;
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
#pragma unroll
            for (int i = 0; i < CPW; ++i) part[i] = __fadd_rn(part[i], __shfl_xor_sync(0xFFFFFFFFu, part[i], off));
        }
        if (lane == 0) {
#pragma unroll
            for (int i = 0; i < CPW; ++i) {
                const int64_t n = c0 + warp + kDecodeSelWarps * i;
                local[warp + kDecodeSelWarps * i] = n < count ? pack_key(part[i], (int32_t)n) : kEmpty;
            }
        }
    } else if (lane == 0) {
#pragma unroll
        for (int i = 0; i < CPW; ++i) local[warp + kDecodeSelWarps * i] = kEmpty;
    }
    __syncthreads();
    // ---- this CTA's keys as one sorted 32-list in the leader's shared memory
    int64_t* lead0 = cluster.map_shared_rank(lead, 0);
    if (CPW == 4 && warp == 1) half[lane] = warp_sort32_desc(local[32 + lane], lane);
    if (CPW == 4) __syncthreads();
    cluster_wait_acquire();  // (first phase)
    if (warp == 0) {
        int64_t x = (CPW == 1 && lane >= 16) ? kEmpty : local[lane];
        x = warp_sort32_desc(x, lane);
        if (CPW == 4) {
            const int64_t y = half[31 - lane];
            x = warp_clean32_desc(x > y ? x : y, lane);
        }
        lead0[rank * 32 + lane] = x;
    }
    cluster_arrive_release();
    if (rank != 0) return;  // the leader alone reads the keys; nothing reads this CTA's memory
    cluster_wait_acquire();
    // ---- merge tree over the cs sorted lists (warp w holds list w)
    int64_t x = warp < cs ? lead[warp * 32 + lane] : kEmpty;
    for (int step = 1; step < cs; step <<= 1) {
        if ((warp % (2 * step)) == 0 && warp + step < cs) {
            const int64_t y = lead[(warp + step) * 32 + 31 - lane];
            x = warp_clean32_desc(x > y ? x : y, lane);
            lead[warp * 32 + lane] = x;
        }
        __syncthreads();
    }
    const int k = (int)min((int64_t)top_p, Nr);
    if (warp == 0) pick_bucket[lane] = lane < k ? key_bucket(x) : -1;
    __syncthreads();
    // ---- the walk over the picks' member rows
    const int64_t pos = rp.walk_pos(r);
    int64_t ws = pos + 1 - window;
    if (ws < 0) ws = 0;
    const int nch = (cap + 31) >> 5;
    constexpr int kMaxCh = kDecodeMaxCap / 32;
    int vals[2][kMaxCh];
    if (Nr > 0) {  // (block-uniform) unconditional loads at clamped valid addresses
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int b = pick_bucket[warp + kDecodeSelWarps * t];
            const int64_t row = b >= 0 ? b : 0;
#pragma unroll
            for (int ch = 0; ch < kMaxCh; ++ch) vals[t][ch] = __ldcg(mr + row * cap + min(ch * 32 + lane, cap - 1));
        }
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int b = pick_bucket[warp + kDecodeSelWarps * t];
#pragma unroll
            for (int ch = 0; ch < kMaxCh; ++ch)
                if (b < 0 || ch >= nch || ch * 32 + lane >= cap) vals[t][ch] = -1;
        }
    } else {
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int ch = 0; ch < kMaxCh; ++ch) vals[t][ch] = -1;
    }
    unsigned masks[2][kMaxCh];
    int cnt[2] = {0, 0};
#pragma unroll
    for (int t = 0; t < 2; ++t) {
#pragma unroll
        for (int ch = 0; ch < kMaxCh; ++ch) {
            const int v = vals[t][ch];
            const bool keep = v >= 0 && v >= sink && (int64_t)v < ws;
            masks[t][ch] = __ballot_sync(0xFFFFFFFFu, keep);
            cnt[t] += __popc(masks[t][ch]);
        }
    }
    if (lane == 0) {
        pick_count[warp] = cnt[0];
        pick_count[warp + kDecodeSelWarps] = cnt[1];
    }
    __syncthreads();
    const int mine = pick_count[lane];
    const int total = __reduce_add_sync(0xFFFFFFFFu, (unsigned)mine);
    const int filled = total < top_k ? total : top_k;
    const int width = top_k + window + sink;
    int32_t* out = lists + (int64_t)r * width;
    const unsigned lt = (1u << lane) - 1u;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        const int p = warp + kDecodeSelWarps * t;
        int at = (int)__reduce_add_sync(0xFFFFFFFFu, lane < p ? (unsigned)mine : 0u);
#pragma unroll
        for (int ch = 0; ch < kMaxCh; ++ch) {
            const int o = at + __popc(masks[t][ch] & lt);
            if (((masks[t][ch] >> lane) & 1u) && o < top_k) out[o] = vals[t][ch];
            at += __popc(masks[t][ch]);
        }
    }
    int nwin = (int)(pos - ws + 1);
    if (nwin < 0) nwin = 0;
    const int nsink = (int)(sink < ws ? sink : ws);
    for (int i = threadIdx.x; i < width - filled; i += kDecodeSelThreads) {
        int v = -1;
        if (i < nwin) v = (int)(ws + i);
        else if (i < nwin + nsink) v = i - nwin;
        out[filled + i] = v;
    }
    if (threadIdx.x == 0) lengths[r] = filled + nwin + nsink;
}

// ------------------------------------------------------------------ host helpers

// ------------------------------------------------------------------ streaming select

// Rows wider than one cluster (batched decode over long sequences, top_p <= 128) take two
// launches. (1) select_stream_kernel, a persistent grid, streams the centroid tables
// through shared memory with TMA bulk copies while scoring warps consume them, so HBM sees
// one continuous stream per SM:
//   * work items: item_cols (<= 128, a multiple of a stage's columns) visible columns of
//     one row - smaller items when the batch is small, so every CTA gets work; CTA b takes
//     items b, b + grid, ... in row order;
//   * one producer warp (lane 0) copies 32 KB stages (contiguous centroid rows) into a ring
//     of kStreamStages buffers (full/empty mbarriers, bounded waits) and posts each stage's
//     (row, first column, columns) beside it;
//   * kStreamWarps scoring warps score the staged columns (canonical cdot, the row's query
//     in registers) into packed keys in global scratch [R, N].
// (2) select_finish_kernel, one CTA per row (programmatic dependent launch): the row's top
// K = 32 KW keys by warp-list sorts and a merge tree, the picked member rows staged with
// cp.async, and the expansion walk with its output gathered in shared memory.
// Counters: counters[R] is the status word (LSA_ERR_TIMEOUT after an expired wait).
constexpr int kStreamWarps = 8;
constexpr int kStreamThreads = 32 * (kStreamWarps + 1);
constexpr int kStreamStages = 3;
constexpr int kStreamStageBytes = 32768;
constexpr int kStreamItemCols = 128;  // the largest work item (columns of one row)
constexpr int kStreamMaxRows = 256;
constexpr int kFinishMaxTopK = 16384;  // read-list slots gathered in shared memory

struct StreamStage {
    int row;  // < 0: no more items for this CTA
    int col0, ncols;
};

__device__ __forceinline__ int64_t stream_visible(const RowPos& rp, int r, int64_t N, int64_t block, int64_t bpb) {
    const int64_t Nr = rp.rows(r, N);
    int64_t cnt = rp.count_pos(r) / block * bpb;
    if (cnt > Nr) cnt = Nr;
    return cnt < 0 ? 0 : cnt;
}

template <typename TQ, int CHUNKS>
__global__ void __launch_bounds__(kStreamThreads, 2) select_stream_kernel(
    const TQ* __restrict__ q, int64_t ldq, const __nv_bfloat16* __restrict__ c, int64_t N, int d, RowPos rp,
    int64_t block, int64_t bpb, int R, int item_cols, int64_t* __restrict__ ws_keys, int32_t* __restrict__ status) {
    constexpr int NS = kStreamStages;
    extern __shared__ __align__(128) unsigned char stage_buf[];  // [NS][32 KB]
    __shared__ __align__(8) uint64_t full[NS], empty[NS];
    __shared__ StreamStage meta[NS];
    __shared__ int item_start[kStreamMaxRows + 1];
    __shared__ int row_count[kStreamMaxRows];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
#pragma unroll
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kStreamWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    pdl_wait();
    pdl_trigger();
    // visible columns of every row and the first item of every row (rows over the lanes)
    if (warp == 0) {
        constexpr int PER = kStreamMaxRows / 32;
        int n_items[PER];
        int mine = 0;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int r = lane * PER + i;
            n_items[i] = 0;
            if (r < R) {
                const int64_t cnt = stream_visible(rp, r, N, block, bpb);
                row_count[r] = (int)cnt;
                n_items[i] = (int)((cnt + item_cols - 1) / item_cols);
            }
            mine += n_items[i];
        }
        int incl = mine;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            int y = __shfl_up_sync(0xFFFFFFFFu, incl, off);
            if (lane >= off) incl += y;
        }
        int at = incl - mine;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int r = lane * PER + i;
            if (r < R) item_start[r] = at;
            at += n_items[i];
        }
        if (lane == 31) item_start[kStreamMaxRows] = incl;
    }
    __syncthreads();
    const int total_items = item_start[kStreamMaxRows];

    if (warp == kStreamWarps) {  // producer
        if (lane == 0) {
            const int cps = kStreamStageBytes / (d * 2);  // columns per stage
            int s = 0;
            bool ok = true;
            for (int it = blockIdx.x;; it += gridDim.x) {
                const bool stop = it >= total_items;
                int r = 0, col0 = 0, col1 = 0;
                if (!stop) {  // the last row whose first item is at or before it (empty rows share it)
                    int lo = 0, hi = R - 1;
                    while (lo < hi) {
                        int mid = (lo + hi + 1) >> 1;
                        if (item_start[mid] <= it) lo = mid;
                        else hi = mid - 1;
                    }
                    r = lo;
                    col0 = (it - item_start[r]) * item_cols;
                    col1 = min(col0 + item_cols, row_count[r]);
                }
                for (int c0 = col0;; c0 += cps) {  // a stop posts one stage with row -1
                    const int slot = s % NS;
                    if (!mbar_wait_bounded(&empty[slot], ((s / NS) & 1) ^ 1)) {
                        ok = false;
                        break;
                    }
                    const int n = stop ? 0 : min(cps, col1 - c0);
                    meta[slot] = StreamStage{stop ? -1 : r, c0, n};
                    if (n > 0) {
                        mbar_arrive_expect_tx(&full[slot], (uint32_t)(n * d * 2));
                        bulk_g2s(stage_buf + slot * kStreamStageBytes, c + (rp.off(r) + c0) * d, (uint32_t)(n * d * 2),
                                 &full[slot]);
                    } else {
                        mbar_arrive(&full[slot]);
                    }
                    ++s;
                    if (stop || c0 + cps >= col1) break;
                }
                if (stop || !ok) break;
            }
            if (!ok) {  // the scoring warps stopped consuming: wait (bounded) for copies in flight
                atomicExch(status, LSA_ERR_TIMEOUT);
                for (int s2 = max(0, s - NS); s2 < s; ++s2) mbar_wait_bounded(&full[s2 % NS], (s2 / NS) & 1);
            }
        }
        return;
    }

    // scoring warps
    const int nchunks = d >> 3;
    float x[CHUNKS][8];
    int cur = -1;
    for (int s = 0;; ++s) {
        const int slot = s % NS;
        if (!mbar_wait_bounded(&full[slot], (s / NS) & 1)) {
            if (lane == 0) atomicExch(status, LSA_ERR_TIMEOUT);
            break;  // every scoring warp waits on the same phase and leaves here too
        }
        const StreamStage m = meta[slot];
        if (m.row < 0) break;
        if (m.row != cur) {
            cur = m.row;
#pragma unroll
            for (int j = 0; j < CHUNKS; ++j) {
                const int ch = lane + 32 * j;
                if (ch < nchunks) load8<TQ>(q + cur * ldq + (size_t)ch * 8, x[j]);
            }
        }
        const __nv_bfloat16* sc = reinterpret_cast<const __nv_bfloat16*>(stage_buf + slot * kStreamStageBytes);
        for (int cc = warp; cc < m.ncols; cc += kStreamWarps) {
            const float p = butterfly_sum(lane_partial_regs<__nv_bfloat16, CHUNKS>(x, sc + (size_t)cc * d, lane, nchunks));
            if (lane == 0) ws_keys[(int64_t)cur * N + m.col0 + cc] = pack_key(p, m.col0 + cc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
}

template <int KW>
constexpr int finish_smem_bytes(int top_k) {
    return (kFusedThreads / 32 + 1) * 32 * KW * 8 + kMemberPrefetch * 4 + top_k * 4;
}

// One CTA per row after select_stream_kernel: top K of the row's visible keys, the picked
// member rows staged with 16-byte cp.async (cap % 4 == 0, 16-byte aligned members), the walk.
template <int KW>
__global__ void __launch_bounds__(kFusedThreads) select_finish_kernel(
    const int64_t* __restrict__ ws_keys, int64_t N, RowPos rp, int64_t block, int64_t bpb, int top_p,
    const int32_t* __restrict__ members, int cap, int window, int sink, int top_k, int32_t* __restrict__ lists,
    int32_t* __restrict__ lengths) {
    constexpr int K = 32 * KW, NW = kFusedThreads / 32;
    extern __shared__ __align__(128) unsigned char fsm[];
    int64_t* wlists = reinterpret_cast<int64_t*>(fsm);  // [NW][K]
    int64_t* picks = wlists + NW * K;                    // [K]
    int* mem = reinterpret_cast<int*>(picks + K);        // [kMemberPrefetch]
    int* ostage = mem + kMemberPrefetch;                 // [top_k]
    __shared__ int scan_smem[33];
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int count = (int)stream_visible(rp, r, N, block, bpb);
    const int64_t Nr = rp.rows(r, N);
    const int k = (int)min((int64_t)top_p, Nr);
    GlobalKeysCg loader{ws_keys + (int64_t)r * N, count};
    group_topk_desc<KW, NW>(loader, count, wlists, picks, warp, lane, BlockSync{});
    const int32_t* mr = members + rp.off(r) * cap;
    const int q4 = cap / 4;
    for (int i = tid; i < k * q4; i += kFusedThreads) {
        const int pk = i / q4, piece = i - pk * q4;
        const int b = key_bucket(picks[pk]);
        int* dst = mem + pk * cap + piece * 4;
        if (b >= 0 && b < Nr) cp_async16(smem_u32(dst), mr + (int64_t)b * cap + piece * 4, 16);
        else *reinterpret_cast<int4*>(dst) = make_int4(-1, -1, -1, -1);
    }
    cp_async_wait_all();
    __syncthreads();
    const int width = top_k + window + sink;
    expand_walk<kFusedThreads>(mem, k * cap, rp.walk_pos(r), window, sink, top_k, lists + (int64_t)r * width, width,
                               lengths + r, scan_smem, tid, BlockSync{}, ostage);
}

template <typename K>
static int set_smem(K kernel, int bytes) {
    // opt in above 40 KB of dynamic memory: the kernel's static shared memory counts toward
    // the 48 KB default too
    if (bytes > 40 * 1024) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess ||
            cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared) != cudaSuccess)
            return LSA_ERR_CUDA;
    }
    return LSA_OK;
}

static int sort_smem_bytes(int64_t N) {
    int n2 = next_pow2((int)(N > 0 ? N : 1));
    return (n2 <= kSortCap ? n2 : kSortCap) * 8;
}

template <typename TQ, typename TC>
static int launch_scores(const void* q, int64_t R, int64_t ldq, const void* c, int64_t N, int64_t d, float* out,
                         int64_t ldo, cudaStream_t st) {
    int chunks = (int)((d / 8 + 31) / 32);
    int cols = 64;
    dim3 grid((unsigned)((N + cols - 1) / cols), (unsigned)R);
    if (grid.x == 0 || R == 0) return LSA_OK;
    auto qq = (const TQ*)q;
    auto cc = (const TC*)c;
#define LSA_SC(CH) scores_kernel<TQ, TC, CH><<<grid, 256, 0, st>>>(qq, ldq, cc, N, (int)d, out, ldo, cols)
    if (chunks <= 1) LSA_SC(1);
    else if (chunks <= 2) LSA_SC(2);
    else if (chunks <= 4) LSA_SC(4);
    else if (chunks <= 8) LSA_SC(8);
    else return LSA_ERR_ARG;
#undef LSA_SC
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

}  // namespace lsa

using namespace lsa;

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// the expansion launch (defined with the other launchers below)
static int expand_launch(bool keys64, const void* picks, int64_t R, int64_t P, int64_t ldp, const int32_t* members,
                         int64_t member_rows, int64_t cap, const int32_t* positions, int64_t window, int64_t sink,
                         int64_t top_k, int32_t* lists, int32_t* lengths, cudaStream_t stream);

static int num_sms_select() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

extern "C" {

int lsa_bucket_scores(const void* queries, int q_dtype, int64_t R, int64_t ldq, const void* centroids, int c_dtype,
                      int64_t N, int64_t d, float* scores, int64_t lds, cudaStream_t stream) {
    if (d <= 0 || d % 8 || d > 2048 || R < 0 || N < 0 || ldq % 8) return LSA_ERR_ARG;
    if (!aligned16(queries) || !aligned16(centroids)) return LSA_ERR_ARG;
    if (q_dtype == kBF16 && c_dtype == kBF16)
        return launch_scores<__nv_bfloat16, __nv_bfloat16>(queries, R, ldq, centroids, N, d, scores, lds, stream);
    if (q_dtype == kF32 && c_dtype == kF32)
        return launch_scores<float, float>(queries, R, ldq, centroids, N, d, scores, lds, stream);
    if (q_dtype == kF32 && c_dtype == kBF16)
        return launch_scores<float, __nv_bfloat16>(queries, R, ldq, centroids, N, d, scores, lds, stream);
    return LSA_ERR_ARG;
}

int lsa_visible_counts(const int32_t* positions, int64_t R, int64_t block, int64_t bpb, int64_t rows, int32_t* counts,
                       cudaStream_t stream) {
    if (block <= 0 || bpb < 0) return LSA_ERR_ARG;
    if (R == 0) return LSA_OK;
    visible_counts_kernel<<<(unsigned)((R + 255) / 256), 256, 0, stream>>>(positions, R, block, bpb, rows, counts);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

int lsa_pack_keys(const float* scores, int64_t R, int64_t N, int64_t lds, const int32_t* lengths, int64_t* keys,
                  int64_t ldk, cudaStream_t stream) {
    if (R * N == 0) return LSA_OK;
    pack_keys_kernel<<<(unsigned)((R * N + 255) / 256), 256, 0, stream>>>(scores, R, N, lds, lengths, keys, ldk);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

int lsa_best_first_keys(const int64_t* keys, int64_t R, int64_t N, int64_t ldk, int64_t k, const int32_t* counts,
                        int64_t* out, int64_t ldo, cudaStream_t stream) {
    if (k < 0 || k > 4096 || ldo < k) return LSA_ERR_ARG;
    if (R == 0) return LSA_OK;
    int smem = sort_smem_bytes(N);
    if (set_smem(best_first_kernel, smem)) return LSA_ERR_CUDA;
    best_first_kernel<<<(unsigned)R, 1024, smem, stream>>>(keys, N, ldk, (int)k, counts, out, ldo);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

int lsa_unpack_ids(const int64_t* keys, int64_t n, int32_t* ids, cudaStream_t stream) {
    if (n == 0) return LSA_OK;
    unpack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(keys, n, ids);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

int lsa_select_topk_scores(const float* scores, int64_t R, int64_t N, int64_t lds, const int32_t* lengths,
                           int64_t top_p, int64_t* out, int64_t ldo, cudaStream_t stream) {
    int64_t k = top_p < N ? top_p : N;
    if (k < 0 || k > 4096 || ldo < k) return LSA_ERR_ARG;
    if (R == 0) return LSA_OK;
    int smem = sort_smem_bytes(N);
    if (set_smem(select_topk_kernel, smem)) return LSA_ERR_CUDA;
    select_topk_kernel<<<(unsigned)R, 1024, smem, stream>>>(scores, N, lds, lengths, (int)k, out, ldo);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

int lsa_expand_in_order(const int32_t* picked, int64_t R, int64_t P, int64_t ldp, const int32_t* members,
                        int64_t member_rows, int64_t cap, const int32_t* positions, int64_t window, int64_t sink,
                        int64_t top_k, int32_t* lists, int32_t* lengths, cudaStream_t stream) {
    if (cap <= 0 || window < 0 || sink < 0 || top_k < 0 || P < 0) return LSA_ERR_ARG;
    if (R == 0) return LSA_OK;
    return expand_launch(false, picked, R, P, ldp, members, member_rows, cap, positions, window, sink, top_k, lists,
                         lengths, stream);
}

int lsa_expand_from_keys(const int64_t* keys, int64_t R, int64_t P, int64_t ldk, const int32_t* members,
                         int64_t member_rows, int64_t cap, const int32_t* positions, int64_t window, int64_t sink,
                         int64_t top_k, int32_t* lists, int32_t* lengths, cudaStream_t stream) {
    if (cap <= 0 || window < 0 || sink < 0 || top_k < 0 || P < 0) return LSA_ERR_ARG;
    if (R == 0) return LSA_OK;
    return expand_launch(true, keys, R, P, ldk, members, member_rows, cap, positions, window, sink, top_k, lists,
                         lengths, stream);
}

// Scratch of lsa_select_fused: the packed keys [R, N] int64. Counters: one int32 ticket
// per row, zero before the call; the kernel leaves them zero.
int64_t lsa_select_fused_scratch(int64_t R, int64_t N) { return ((R * N * 8 + 255) / 256) * 256; }

}  // extern "C"

// The expansion launch: member rows staged in shared memory when they (and the gathered
// output) fit, else the tiled walk reading members from global memory.
static int expand_launch(bool keys64, const void* picks, int64_t R, int64_t P, int64_t ldp, const int32_t* members,
                         int64_t member_rows, int64_t cap, const int32_t* positions, int64_t window, int64_t sink,
                         int64_t top_k, int32_t* lists, int32_t* lengths, cudaStream_t stream) {
    // programmatic dependent launch: the kernels wait for the picks' producer before any read
    cudaLaunchAttribute pdl;
    pdl.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl.val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)R);
    lc.blockDim = dim3(512);
    lc.stream = stream;
    lc.attrs = &pdl;
    lc.numAttrs = 1;
    cudaError_t e;
    const int64_t staged = ((P * cap + 3) / 4 * 4 + top_k) * 4;
    if (staged <= 200 * 1024 && P * cap < (1 << 30)) {
        const int vec16 = cap % 4 == 0 && aligned16(members);
        lc.dynamicSmemBytes = (size_t)staged;
        if (keys64) {
            auto kern = expand_staged_kernel<int64_t>;
            if (set_smem(kern, (int)staged)) return LSA_ERR_CUDA;
            e = cudaLaunchKernelEx(&lc, kern, (const int64_t*)picks, (int)P, ldp, members, member_rows, (int)cap,
                                   positions, (int)window, (int)sink, (int)top_k, lists, lengths, vec16);
        } else {
            auto kern = expand_staged_kernel<int32_t>;
            if (set_smem(kern, (int)staged)) return LSA_ERR_CUDA;
            e = cudaLaunchKernelEx(&lc, kern, (const int32_t*)picks, (int)P, ldp, members, member_rows, (int)cap,
                                   positions, (int)window, (int)sink, (int)top_k, lists, lengths, vec16);
        }
    } else if (keys64) {
        e = cudaLaunchKernelEx(&lc, expand_kernel<int64_t>, (const int64_t*)picks, (int)P, ldp, members, member_rows,
                               (int)cap, positions, (int)window, (int)sink, (int)top_k, lists, lengths);
    } else {
        e = cudaLaunchKernelEx(&lc, expand_kernel<int32_t>, (const int32_t*)picks, (int)P, ldp, members, member_rows,
                               (int)cap, positions, (int)window, (int)sink, (int)top_k, lists, lengths);
    }
    if (e != cudaSuccess) return LSA_ERR_CUDA;
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

// The fused selection's launch for token rows and tile rows alike (RowPos).
static int select_fused_launch(const void* queries, int q_dtype, int64_t R, int64_t ldq, const void* centroids,
                               int c_dtype, int64_t N, int64_t d, RowPos positions, int64_t block, int64_t bpb,
                               const int32_t* members, int64_t cap, int64_t top_p, int64_t window, int64_t sink,
                               int64_t top_k, int32_t* lists, int32_t* lengths, void* scratch, int64_t scratch_bytes,
                               int32_t* counters, int64_t n_counters, int64_t max_position, cudaStream_t stream) {
    if (d <= 0 || d % 8 || d > 2048 || ldq % 8 || cap <= 0 || block <= 0) return LSA_ERR_ARG;
    if (!aligned16(queries) || !aligned16(centroids) || !aligned16(scratch)) return LSA_ERR_ARG;
    if (top_p > 4096 || scratch_bytes < lsa_select_fused_scratch(R, N) || n_counters < R) return LSA_ERR_ARG;
    if (R == 0) return LSA_OK;
    int64_t* ws_keys = (int64_t*)scratch;
    int32_t* tickets = counters;
    // columns any row can see: the grid covers the widest row (max_position < 0: all N)
    int64_t most = max_position < 0 ? N : (max_position / block * bpb < N ? max_position / block * bpb : N);
    // few rows (decode): one column per warp, the centroid read spread over many SMs;
    // many rows (prefill tiles): one CTA per row scores all its columns (no cross-CTA merge)
    const bool many_rows = R >= 256;
    int cols = 4 * (kFusedThreads / 32);  // four columns per warp, loads in flight together
    if (many_rows) cols = (int)(((most > 0 ? most : 1) + 15) / 16 * 16);
    int chunks_x = (int)((most + cols - 1) / cols);
    if (chunks_x < 1) chunks_x = 1;
    dim3 grid((unsigned)chunks_x, (unsigned)R);
    int64_t k = top_p < N ? top_p : N;
    int64_t staged = k * cap <= kMemberPrefetch ? k * cap : 0;
    if (staged && top_k <= kGatherMax) staged = (staged + 3) / 4 * 4 + top_k;  // + the gathered list
    int smem = sort_smem_bytes(most);
    if (smem < kFusedThreads * 8) smem = kFusedThreads * 8;
    if (smem < top_p * 8) smem = (int)(top_p * 8);
    if (smem < (k + 1) * 8 + staged * 4) smem = (int)((k + 1) * 8 + staged * 4);
    int ch = (int)((d / 8 + 31) / 32);
    cudaLaunchAttribute pdl;
    pdl.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl.val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = grid;
    lc.blockDim = dim3(kFusedThreads);
    lc.dynamicSmemBytes = smem;
    lc.stream = stream;
    lc.attrs = &pdl;
    lc.numAttrs = 1;
    // cluster path: the row's columns fit one cluster of <= 16 CTAs (16 warps x <= 4 columns)
    int cpw = (int)((most + 16 * 16 - 1) / (16 * 16));
    if (cpw < 1) cpw = 1;
    int cs = (int)((most + 16 * cpw - 1) / (16 * cpw));
    if (cs < 1) cs = 1;
    bool use_cluster = !many_rows && cpw <= kMaxColsPerWarp && cs <= 16;
    // rows wider than one cluster, or batches with enough columns to fill the GPU (measured:
    // 32 rows x 504 buckets, 20 us streamed vs 25 us in clusters): the streaming scorer +
    // per-row finish when their limits hold (bf16 centroids, top_p <= 128, staged members
    // fit, 16-byte member rows, a status word)
    const bool wide_batch = R * most >= 8192;
    if (!many_rows && (!use_cluster || wide_batch) && c_dtype == kBF16 &&
        (q_dtype == kBF16 || q_dtype == kF32 || q_dtype == kF32AsBF16) &&
        R <= kStreamMaxRows && top_p <= 128 && k * cap <= kMemberPrefetch && cap % 4 == 0 && aligned16(members) &&
        top_k <= kFinishMaxTopK && n_counters >= R + 1 && d * 2 <= kStreamStageBytes && N < (1ll << 30)) {
        // item size: up to 128 columns, smaller (whole stages) until the batch makes about two
        // items per CTA slot
        const int cps_host = (int)(kStreamStageBytes / (d * 2));
        const int64_t slots_host = 2 * (int64_t)num_sms_select();
        int64_t icols = R * most / (2 * slots_host);
        if (icols > kStreamItemCols) icols = kStreamItemCols;
        icols = icols / cps_host * cps_host;
        if (icols < cps_host) icols = cps_host;
        const int item_cols = (int)icols;
        int64_t items = R * ((most + item_cols - 1) / item_cols);
        if (items < 1) items = 1;
#define LSA_ST(TQ, CH)                                                                                              \
    do {                                                                                                            \
        auto kern = select_stream_kernel<TQ, CH>;                                                                   \
        constexpr int ssm = kStreamStages * kStreamStageBytes;                                                      \
        if (set_smem(kern, ssm)) return LSA_ERR_CUDA;                                                               \
        int per_sm = 0;                                                                                             \
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kStreamThreads, ssm) != cudaSuccess ||     \
            per_sm < 1)                                                                                             \
            return LSA_ERR_CUDA;                                                                                    \
        int64_t grid = (int64_t)per_sm * num_sms_select();                                                          \
        if (grid > items) grid = items;                                                                             \
        cudaLaunchConfig_t sc = {};                                                                                 \
        sc.gridDim = dim3((unsigned)grid);                                                                          \
        sc.blockDim = dim3(kStreamThreads);                                                                         \
        sc.dynamicSmemBytes = ssm;                                                                                  \
        sc.stream = stream;                                                                                         \
        sc.attrs = &pdl;                                                                                            \
        sc.numAttrs = 1;                                                                                            \
        if (cudaLaunchKernelEx(&sc, kern, (const TQ*)queries, ldq, (const __nv_bfloat16*)centroids, N, (int)d,     \
                               positions, block, bpb, (int)R, item_cols, ws_keys, counters + R) != cudaSuccess)     \
            return LSA_ERR_CUDA;                                                                                    \
    } while (0)
#define LSA_FIN(KW)                                                                                                 \
    do {                                                                                                            \
        auto fk = select_finish_kernel<KW>;                                                                         \
        const int fsm = finish_smem_bytes<KW>((int)top_k);                                                          \
        if (set_smem(fk, fsm)) return LSA_ERR_CUDA;                                                                 \
        cudaLaunchConfig_t fc = {};                                                                                 \
        fc.gridDim = dim3((unsigned)R);                                                                             \
        fc.blockDim = dim3(kFusedThreads);                                                                          \
        fc.dynamicSmemBytes = fsm;                                                                                  \
        fc.stream = stream;                                                                                         \
        fc.attrs = &pdl;                                                                                            \
        fc.numAttrs = 1;                                                                                            \
        if (cudaLaunchKernelEx(&fc, fk, (const int64_t*)ws_keys, N, positions, block, bpb, (int)top_p, members,     \
                               (int)cap, (int)window, (int)sink, (int)top_k, lists, lengths) != cudaSuccess)        \
            return LSA_ERR_CUDA;                                                                                    \
    } while (0)
        if (q_dtype == kBF16) {
            if (ch <= 1) LSA_ST(__nv_bfloat16, 1);
            else if (ch <= 2) LSA_ST(__nv_bfloat16, 2);
            else if (ch <= 4) LSA_ST(__nv_bfloat16, 4);
            else LSA_ST(__nv_bfloat16, 8);
        } else if (q_dtype == kF32AsBF16) {
            if (ch <= 1) LSA_ST(F32AsBF16, 1);
            else if (ch <= 2) LSA_ST(F32AsBF16, 2);
            else if (ch <= 4) LSA_ST(F32AsBF16, 4);
            else LSA_ST(F32AsBF16, 8);
        } else {
            if (ch <= 1) LSA_ST(float, 1);
            else if (ch <= 2) LSA_ST(float, 2);
            else if (ch <= 4) LSA_ST(float, 4);
            else LSA_ST(float, 8);
        }
        if (top_p <= 32) LSA_FIN(1);
        else if (top_p <= 64) LSA_FIN(2);
        else LSA_FIN(4);
#undef LSA_FIN
#undef LSA_ST
        LSA_LAUNCH_CHECK();
        return LSA_OK;
    }
    int csmem = sort_smem_bytes(most);
    if (csmem < ((k > 32 ? k : 32) + 1) * 8 + staged * 4) csmem = (int)(((k > 32 ? k : 32) + 1) * 8 + staged * 4);
    if (csmem < k * 8) csmem = (int)(k * 8);
    if (csmem < cs * 16 * cpw * 8) csmem = cs * 16 * cpw * 8;  // every scored column's key slot
    cudaLaunchAttribute cattrs[2];
    cattrs[0] = pdl;
    cattrs[1].id = cudaLaunchAttributeClusterDimension;
    // single-sequence decode rows (top_p <= 32): the latency path, one cluster per row
    const int dcpw = cpw <= 1 ? 1 : (cpw <= 2 ? 2 : 4);
    // (registers: the warp holds its columns' raw chunks, at most 8 x 16 bytes per lane)
    if (use_cluster && top_p <= 32 && cap <= kDecodeMaxCap && (d % 8) == 0 &&
        (c_dtype == kBF16 || c_dtype == kF32) && ch * dcpw * (c_dtype == kF32 ? 2 : 1) <= 8) {
        const int dcs = (int)((most + kDecodeSelWarps * dcpw - 1) / (kDecodeSelWarps * dcpw));
        cattrs[1].val.clusterDim.x = (unsigned)(dcs < 1 ? 1 : dcs);
        cattrs[1].val.clusterDim.y = 1;
        cattrs[1].val.clusterDim.z = 1;
        cudaLaunchConfig_t dc = {};
        dc.gridDim = dim3(cattrs[1].val.clusterDim.x, (unsigned)R);
        dc.blockDim = dim3(kDecodeSelThreads);
        dc.dynamicSmemBytes = 0;
        dc.stream = stream;
        dc.attrs = cattrs;
        dc.numAttrs = 2;
        int rc = LSA_ERR_ARG;
#define LSA_DS(TQ, TC, CH)                                                                                       \
    do {                                                                                                         \
        auto launch = [&](auto kern) -> int {                                                                    \
            if (dcs > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=      \
                               cudaSuccess)                                                                      \
                return LSA_ERR_CUDA;                                                                             \
            return cudaLaunchKernelEx(&dc, kern, (const TQ*)queries, ldq, (const TC*)centroids, N, (int)d,       \
                                      positions, block, bpb, (int)top_p, members, (int)cap, (int)window,         \
                                      (int)sink, (int)top_k, lists, lengths, QGroup{0, 0}) == cudaSuccess        \
                       ? LSA_OK                                                                                  \
                       : LSA_ERR_CUDA;                                                                           \
        };                                                                                                       \
        if (dcpw == 1) rc = launch(select_decode_kernel<TQ, TC, CH, 1>);                                         \
        else if (dcpw == 2) rc = launch(select_decode_kernel<TQ, TC, CH, 2>);                                    \
        else rc = launch(select_decode_kernel<TQ, TC, CH, 4>);                                                   \
    } while (0)
#define LSA_DS_CH(TQ, TC)                  \
    do {                                   \
        if (ch <= 1) LSA_DS(TQ, TC, 1);      \
        else if (ch <= 2) LSA_DS(TQ, TC, 2); \
        else if (ch <= 4) LSA_DS(TQ, TC, 4); \
        else LSA_DS(TQ, TC, 8);              \
    } while (0)
        if (q_dtype == kBF16 && c_dtype == kBF16) LSA_DS_CH(__nv_bfloat16, __nv_bfloat16);
        else if (q_dtype == kF32AsBF16 && c_dtype == kBF16) LSA_DS_CH(F32AsBF16, __nv_bfloat16);
        else if (q_dtype == kF32 && c_dtype == kF32) LSA_DS_CH(float, float);
        else if (q_dtype == kF32 && c_dtype == kBF16) LSA_DS_CH(float, __nv_bfloat16);
        else return LSA_ERR_ARG;
#undef LSA_DS_CH
#undef LSA_DS
        if (rc != LSA_OK) return rc;
        LSA_LAUNCH_CHECK();
        return LSA_OK;
    }
    cattrs[1].val.clusterDim.x = (unsigned)cs;
    cattrs[1].val.clusterDim.y = 1;
    cattrs[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t cc = {};
    cc.gridDim = dim3((unsigned)cs, (unsigned)R);
    cc.blockDim = dim3(kFusedThreads);
    cc.dynamicSmemBytes = csmem;
    cc.stream = stream;
    cc.attrs = cattrs;
    cc.numAttrs = 2;
#define LSA_FS(TQ, TC, CH)                                                                                       \
    do {                                                                                                         \
        bool launched = false;                                                                                   \
        if (use_cluster) {                                                                                       \
            auto ck = select_cluster_kernel<TQ, TC, CH>;                                                         \
            if (!set_smem(ck, csmem) &&                                                                          \
                (cs <= 8 || cudaFuncSetAttribute(ck, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==      \
                                cudaSuccess) &&                                                                  \
                cudaLaunchKernelEx(&cc, ck, (const TQ*)queries, ldq, (const TC*)centroids, N, (int)d, positions, \
                                   block, bpb, cpw, (int)top_p, members, (int)cap, (int)window, (int)sink,       \
                                   (int)top_k, lists, lengths) == cudaSuccess)                                   \
                launched = true;                                                                                 \
            else                                                                                                 \
                cudaGetLastError(); /* a refused cluster launch falls back to the ticket kernel */              \
        }                                                                                                        \
        if (!launched) {                                                                                         \
            auto kern = select_fused_kernel<TQ, TC, CH>;                                                         \
            if (set_smem(kern, smem)) return LSA_ERR_CUDA;                                                       \
            if (cudaLaunchKernelEx(&lc, kern, (const TQ*)queries, ldq, (const TC*)centroids, N, (int)d,          \
                                   positions, block, bpb, cols, (int)top_p, members, (int)cap, (int)window,      \
                                   (int)sink, (int)top_k, lists, lengths, ws_keys, tickets) != cudaSuccess)      \
                return LSA_ERR_CUDA;                                                                             \
        }                                                                                                        \
    } while (0)
#define LSA_FS_CH(TQ, TC)              \
    do {                               \
        if (ch <= 1) LSA_FS(TQ, TC, 1);  \
        else if (ch <= 2) LSA_FS(TQ, TC, 2); \
        else if (ch <= 4) LSA_FS(TQ, TC, 4); \
        else LSA_FS(TQ, TC, 8);          \
    } while (0)
    if (q_dtype == kBF16 && c_dtype == kBF16) LSA_FS_CH(__nv_bfloat16, __nv_bfloat16);
    else if (q_dtype == kF32AsBF16 && c_dtype == kBF16) LSA_FS_CH(F32AsBF16, __nv_bfloat16);
    else if (q_dtype == kF32 && c_dtype == kF32) LSA_FS_CH(float, float);
    else if (q_dtype == kF32 && c_dtype == kBF16) LSA_FS_CH(float, __nv_bfloat16);
    else return LSA_ERR_ARG;
#undef LSA_FS_CH
#undef LSA_FS
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

extern "C" {

int64_t lsa_select_batched_scratch(int64_t R, int64_t max_rows) { return lsa_select_fused_scratch(R, max_rows); }

int lsa_positional_picks(const int32_t* positions, int64_t R, int64_t block, int64_t bpb, int64_t rows, int64_t top_p,
                         int64_t first, int64_t last, int32_t* picks, cudaStream_t stream) {
    if (R < 0 || block <= 0 || top_p <= 0 || first < 0 || last < 0 || first + last > top_p) return LSA_ERR_ARG;
    if (R == 0) return LSA_OK;
    positional_picks_kernel<<<(unsigned)((R + 127) / 128), 128, 0, stream>>>(positions, R, block, bpb, rows,
                                                                             (int)top_p, (int)first, (int)last, picks);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

int lsa_select_batched(const void* queries, int q_dtype, int64_t R, int64_t ldq, const void* centroids, int c_dtype,
                       int64_t d, const int64_t* table_off, const int32_t* table_rows, int64_t max_rows,
                       const int32_t* positions, int64_t block, int64_t bpb, const int32_t* members, int64_t cap,
                       int64_t top_p, int64_t window, int64_t sink, int64_t top_k, int32_t* lists, int32_t* lengths,
                       void* scratch, int64_t scratch_bytes, int32_t* counters, int64_t n_counters,
                       int64_t max_position, cudaStream_t stream) {
    if (positions == nullptr || table_off == nullptr || table_rows == nullptr || max_rows < 0) return LSA_ERR_ARG;
    return select_fused_launch(queries, q_dtype, R, ldq, centroids, c_dtype, max_rows, d,
                               RowPos{positions, 0, block, table_off, table_rows}, block, bpb, members, cap, top_p,
                               window, sink, top_k, lists, lengths, scratch, scratch_bytes, counters, n_counters,
                               max_position, stream);
}

int lsa_select_fused_grouped(const void* q, int q_dtype, int64_t R, int64_t Hq, int64_t Hkv, int64_t D,
                             const void* centroids, int c_dtype, int64_t N, const int32_t* positions, int64_t block,
                             int64_t bpb, const int32_t* members, int64_t cap, int64_t top_p, int64_t window,
                             int64_t sink, int64_t top_k, int32_t* lists, int32_t* lengths, cudaStream_t stream) {
    // the decode rows select_fused would give to the one-cluster decode kernel, with the
    // index query built in the kernel; anything else is refused (LSA_ERR_ARG) for the caller
    // to regroup and call lsa_select_fused
    if (R < 0 || Hkv <= 0 || Hq <= 0 || Hq % Hkv || D <= 0 || D % 8 || positions == nullptr) return LSA_ERR_ARG;
    const int64_t d = Hkv * D, G = Hq / Hkv;
    if (d > kDecodeMaxD || cap <= 0 || block <= 0 || top_p <= 0 || top_k < 0 || window < 0 || sink < 0)
        return LSA_ERR_ARG;
    if (!aligned16(q) || !aligned16(centroids)) return LSA_ERR_ARG;
    if (q_dtype != kBF16 && q_dtype != kF16 && q_dtype != kF32) return LSA_ERR_ARG;
    if (c_dtype != kBF16 && c_dtype != kF32) return LSA_ERR_ARG;
    const int64_t most = N;
    int cpw = (int)((most + 16 * 16 - 1) / (16 * 16));
    if (cpw < 1) cpw = 1;
    int cs = (int)((most + 16 * cpw - 1) / (16 * cpw));
    if (cs < 1) cs = 1;
    const int ch = (int)((d / 8 + 31) / 32);
    const int dcpw = cpw <= 1 ? 1 : (cpw <= 2 ? 2 : 4);
    const bool decode = R < 256 && cpw <= kMaxColsPerWarp && cs <= 16 && R * most < 8192 && top_p <= 32 &&
                        cap <= kDecodeMaxCap && ch * dcpw * (c_dtype == kF32 ? 2 : 1) <= 8;
    if (!decode) return LSA_ERR_ARG;
    if (R == 0) return LSA_OK;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    attrs[1].id = cudaLaunchAttributeClusterDimension;
    const int dcs = (int)((most + kDecodeSelWarps * dcpw - 1) / (kDecodeSelWarps * dcpw));
    attrs[1].val.clusterDim.x = (unsigned)(dcs < 1 ? 1 : dcs);
    attrs[1].val.clusterDim.y = 1;
    attrs[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t dc = {};
    dc.gridDim = dim3(attrs[1].val.clusterDim.x, (unsigned)R);
    dc.blockDim = dim3(kDecodeSelThreads);
    dc.dynamicSmemBytes = 0;
    dc.stream = stream;
    dc.attrs = attrs;
    dc.numAttrs = 2;
    const RowPos rp{positions, 0, block, nullptr, nullptr};
    const QGroup qg{(int)G, (int)D};
    const int64_t ldq = Hq * D;
    int rc = LSA_ERR_ARG;
    // only the (chunks per lane, columns per warp) pairs the decode condition admits are built
    auto run = [&](auto tq, auto tc) -> int {
        using TQ = decltype(tq);
        using TC = decltype(tc);
        constexpr int wide = sizeof(TC) == 4 ? 2 : 1;
        int out = LSA_ERR_ARG;
        auto go = [&](auto kern) {
            if (dcs > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
                out = LSA_ERR_CUDA;
            else
                out = cudaLaunchKernelEx(&dc, kern, (const TQ*)q, ldq, (const TC*)centroids, N, (int)d, rp, block, bpb,
                                         (int)top_p, members, (int)cap, (int)window, (int)sink, (int)top_k, lists,
                                         lengths, qg) == cudaSuccess
                          ? LSA_OK
                          : LSA_ERR_CUDA;
        };
        auto pick = [&](auto chc) {
            constexpr int CH = decltype(chc)::value;
            if constexpr (CH * wide <= 8) {
                if (dcpw == 1) go(select_decode_kernel<TQ, TC, CH, 1>);
            }
            if constexpr (CH * 2 * wide <= 8) {
                if (dcpw == 2) go(select_decode_kernel<TQ, TC, CH, 2>);
            }
            if constexpr (CH * 4 * wide <= 8) {
                if (dcpw == 4) go(select_decode_kernel<TQ, TC, CH, 4>);
            }
        };
        if (ch <= 1) pick(std::integral_constant<int, 1>{});
        else if (ch <= 2) pick(std::integral_constant<int, 2>{});
        else if (ch <= 4) pick(std::integral_constant<int, 4>{});
        else pick(std::integral_constant<int, 8>{});
        return out;
    };
    if (c_dtype == kBF16) {  // bf16 scoring: the built query read as its bf16 rounding
        if (q_dtype == kBF16) rc = run(GroupMean<__nv_bfloat16, true>{}, __nv_bfloat16{});
        else if (q_dtype == kF16) rc = run(GroupMean<__half, true>{}, __nv_bfloat16{});
        else rc = run(GroupMean<float, true>{}, __nv_bfloat16{});
    } else {  // fp32 scoring
        if (q_dtype == kBF16) rc = run(GroupMean<__nv_bfloat16, false>{}, float{});
        else if (q_dtype == kF16) rc = run(GroupMean<__half, false>{}, float{});
        else rc = run(GroupMean<float, false>{}, float{});
    }
    if (rc != LSA_OK) return rc;
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

int lsa_select_fused(const void* queries, int q_dtype, int64_t R, int64_t ldq, const void* centroids, int c_dtype,
                     int64_t N, int64_t d, const int32_t* positions, int64_t block, int64_t bpb, const int32_t* members,
                     int64_t cap, int64_t top_p, int64_t window, int64_t sink, int64_t top_k, int32_t* lists,
                     int32_t* lengths, void* scratch, int64_t scratch_bytes, int32_t* counters, int64_t n_counters,
                     int64_t max_position, cudaStream_t stream) {
    if (positions == nullptr) return LSA_ERR_ARG;
    return select_fused_launch(queries, q_dtype, R, ldq, centroids, c_dtype, N, d, RowPos{positions, 0, block, nullptr, nullptr}, block,
                               bpb, members, cap, top_p, window, sink, top_k, lists, lengths, scratch, scratch_bytes,
                               counters, n_counters, max_position, stream);
}

// ------------------------------------------------------------------ tile rows (prefill)

int lsa_tile_queries(const void* index_queries, int q_dtype, int64_t T, int64_t ldq, int64_t d, int64_t tile,
                     float* out, cudaStream_t stream) {
    if (T < 0 || d <= 0 || tile <= 0 || ldq < d || (q_dtype != kF32 && q_dtype != kBF16)) return LSA_ERR_ARG;
    if (T == 0) return LSA_OK;
    int64_t tiles = (T + tile - 1) / tile;
    dim3 grid((unsigned)((d + 255) / 256), (unsigned)tiles);
    if (q_dtype == kF32)
        tile_queries_kernel<float><<<grid, 256, 0, stream>>>((const float*)index_queries, T, ldq, d, tile, out);
    else
        tile_queries_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>((const __nv_bfloat16*)index_queries, T, ldq, d,
                                                                       tile, out);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

int64_t lsa_tile_select_scratch(int64_t T, int64_t tile, int64_t d, int64_t N) {
    if (tile <= 0) return 0;
    int64_t tiles = (T + tile - 1) / tile;
    return ((tiles * d * 4 + 255) / 256) * 256 + lsa_select_fused_scratch(tiles, N);
}

int lsa_tile_select(const void* index_queries, int q_dtype, int64_t T, int64_t ldq, int64_t tile,
                    const void* centroids, int c_dtype, int64_t N, int64_t d, int64_t block, int64_t bpb,
                    const int32_t* members, int64_t cap, int64_t top_p, int64_t sink, int64_t top_k, int32_t* lists,
                    int32_t* lengths, void* scratch, int64_t scratch_bytes, int32_t* counters, int64_t n_counters,
                    cudaStream_t stream) {
    if (tile <= 0 || T < 0 || block <= 0 || block % tile) return LSA_ERR_ARG;
    if (scratch_bytes < lsa_tile_select_scratch(T, tile, d, N) || !aligned16(scratch)) return LSA_ERR_ARG;
    if (T == 0) return LSA_OK;
    int64_t tiles = (T + tile - 1) / tile;
    float* tq = (float*)scratch;
    int64_t tq_bytes = ((tiles * d * 4 + 255) / 256) * 256;
    int rc = lsa_tile_queries(index_queries, q_dtype, T, ldq, d, tile, tq, stream);
    if (rc) return rc;
    return select_fused_launch(tq, kF32, tiles, d, centroids, c_dtype, N, d, RowPos{nullptr, tile, block, nullptr, nullptr}, block, bpb,
                               members, cap, top_p, 0, sink, top_k, lists, lengths, (char*)scratch + tq_bytes,
                               scratch_bytes - tq_bytes, counters, n_counters, (tiles - 1) * tile, stream);
}

}  // extern "C"
