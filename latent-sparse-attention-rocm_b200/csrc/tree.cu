// tree.cu - the D-LSA tree beam: levels walked top-down, candidates scored by centroid,
// the best beam_width kept per level, top_p buckets picked at level 0 (sm_100a).
//
// Reference (AIwork4me/latent-sparse-attention-rocm, paths inside that project):
//   beam             src/lsa_rocm_lab/port/_tree.py:318-373 (_beam_pick_rows)
//   growth replay    _tree.py:100-142 (_growth_replay; upstream growth_at)
// Growth in closed form (equal to the replay's loop for every page p; checked on CPU):
//   covered = floor(p * bpb / nb) * nb; made[0] = covered / size;
//   closed[l] = floor(made[l] / nb) * nb, made[l + 1] = closed[l] / size (l < top_level - 1);
//   closed[top_level - 1] = 0; levels = number of levels with made > 0.
// Candidates at level L are the carried children plus [first_open, made[L-1]) (first_open
// = 0 on the row's top level, else closed[L-1]); carried and fresh ranges are disjoint, so
// no dedup is needed. Order: packed key ordered_bits(cdot(q, centroid)) | (0x7FFFFFFF - id),
// descending - score first, the lower id on ties. Scores: canonical fp32 cdot.
//
// Launches: one per node level (top down) and one for level 0. Each launch scores its
// candidates over a grid of CTAs (two candidates per warp, up to two CTAs per SM); the last
// CTA of a row (atomic ticket) keeps the row's best keys - a warp-list top-K when the beam
// / top_p is at most 128, else a full sort - and writes the next level's carried rows (or
// the picks).
#include <cooperative_groups.h>

#include "common.cuh"
#include "topk.cuh"
#include "umma.cuh"
#include "walk.cuh"

namespace cg = cooperative_groups;

namespace lsa {

constexpr int kTreeMaxLevels = 8;

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
constexpr int kTreeSortCap = 8192;

struct TreeGrowth {
    int32_t covered, levels;
    int32_t made[kTreeMaxLevels], closed[kTreeMaxLevels];
};

__device__ __forceinline__ void growth_at(int64_t page, int64_t bpb, int64_t nb, int64_t size, int top_level,
                                          int64_t rows, int n_built, TreeGrowth& g) {
    int64_t end = page * bpb;
    if (end > rows) end = rows;  // a position past the cache sees the cache's buckets
    int64_t covered = end / nb * nb;
    int64_t made = covered / size;
    g.covered = (int32_t)covered;
    g.levels = 0;
    for (int l = 0; l < kTreeMaxLevels; ++l) g.made[l] = g.closed[l] = 0;
    for (int l = 0; l < top_level && l < kTreeMaxLevels; ++l) {
        g.made[l] = (int32_t)made;
        if (made > 0) g.levels = l + 1;
        if (l + 1 < top_level) {
            int64_t closed = made / nb * nb;
            g.closed[l] = (int32_t)closed;
            made = closed / size;
        }
    }
    if (g.levels > n_built) g.levels = n_built;
}

struct TreeLevelArgs {
    const float* q;  // [R, d] fp32 index queries
    int64_t d;
    const int32_t* positions;
    int64_t block, bpb, nb, size, rows;
    int top_level, n_built;
    int L;                       // node level of this launch (0 = buckets)
    const float* centroids;      // level L centroids (L >= 1) or bucket centroids_f32 (L == 0)
    const int64_t* children;     // level L children [n, size] (L >= 1)
    int keep;                    // beam_width (L >= 1) or top_p (L == 0)
    const int32_t* carried_in;   // [R, carry_cap]
    const int32_t* carried_n_in; // [R]
    int32_t* carried_out;        // [R, carry_cap]
    int32_t* carried_n_out;      // [R]
    int carry_cap;
    int32_t* picks;              // [R, top_p] (L == 0)
    int64_t* pick_keys;          // [R, top_p] packed keys of the picks, column + col_offset (may be null)
    int64_t col_offset;
    int64_t* ws_keys;            // [R, cand_cap]
    int cand_cap;
    int32_t* tickets;            // [R]
    int32_t* status;
};

struct TreeCandKeys {
    const int64_t* row;
    int count;
    __device__ int64_t operator()(int i) const { return i < count ? __ldcg(row + i) : kEmpty; }
};

struct TreeBlockSync {
    __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

// KW > 0: the last CTA keeps the best K = 32 KW keys by warp-list sorts and a merge tree
// (keep <= K); KW == 0: it sorts every candidate (bitonic in shared memory).
template <int CHUNKS, int KW>
__global__ void __launch_bounds__(256) tree_level_kernel(TreeLevelArgs a) {
    extern __shared__ int64_t tsm[];
    __shared__ int is_last;
    const int r = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int64_t pos = a.positions[r];
    int64_t page = pos / a.block;
    TreeGrowth g;
    growth_at(page, a.bpb, a.nb, a.size, a.top_level, a.rows, a.n_built, g);
    const bool active = a.L == 0 || g.levels >= a.L;
    int n_carried = 0, fresh0 = 0, fresh1 = 0;
    if (active) {
        if (a.L == 0) {
            n_carried = g.levels > 0 ? a.carried_n_in[r] : 0;
            int64_t vis = page * a.bpb;
            fresh0 = g.levels > 0 ? g.covered : 0;
            fresh1 = (int)(vis < a.rows ? vis : a.rows);
        } else {
            n_carried = g.levels > a.L ? a.carried_n_in[r] : 0;
            fresh0 = g.levels == a.L ? 0 : g.closed[a.L - 1];
            fresh1 = g.made[a.L - 1];
        }
        if (fresh1 < fresh0) fresh1 = fresh0;
    }
    int n_cand = n_carried + (fresh1 - fresh0);
    if (n_cand > a.cand_cap) {  // never for a consistent hierarchy; recorded, then clamped
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(a.status, LSA_ERR_ARG);
        n_cand = a.cand_cap;
    }
    // phase 1: score this CTA's share of the row's candidates
    if (active && n_cand > 0) {
        int nchunks = (int)(a.d >> 3);
        float x[CHUNKS][8];
#pragma unroll
        for (int j = 0; j < CHUNKS; ++j) {
            int ch = lane + 32 * j;
            if (ch < nchunks) load8<float>(a.q + r * a.d + (size_t)ch * 8, x[j]);
        }
        for (int i = blockIdx.x * nw + warp; i < n_cand; i += gridDim.x * nw) {
            int id = i < n_carried ? a.carried_in[(int64_t)r * a.carry_cap + i] : fresh0 + (i - n_carried);
            float s = butterfly_sum(lane_partial_regs<float, CHUNKS>(x, a.centroids + (int64_t)id * a.d, lane,
                                                                     nchunks));
            if (lane == 0) a.ws_keys[(int64_t)r * a.cand_cap + i] = pack_key(s, id);
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = atomicAdd(a.tickets + r, 1);
        is_last = t == (int)gridDim.x - 1;
        if (is_last) a.tickets[r] = 0;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // phase 2 (last CTA of the row): order the candidates, keep the best
    int kept = 0;
    int64_t* best = tsm;  // the kept keys, best first
    if (active && n_cand > 0) {
        if constexpr (KW > 0) {
            constexpr int K = 32 * KW;
            best = tsm + 8 * K;
            group_topk_desc<KW, 8>(TreeCandKeys{a.ws_keys + (int64_t)r * a.cand_cap, n_cand}, n_cand, tsm, best,
                                   warp, lane, TreeBlockSync{});
        } else {
            int n2 = next_pow2(n_cand);
            for (int i = threadIdx.x; i < n2; i += blockDim.x)
                tsm[i] = i < n_cand ? __ldcg(a.ws_keys + (int64_t)r * a.cand_cap + i) : kEmpty;
            __syncthreads();
            bitonic_sort_desc(tsm, n2);
        }
        kept = n_cand < a.keep ? n_cand : a.keep;
    }
    if (a.L == 0) {
        for (int i = threadIdx.x; i < a.keep; i += blockDim.x) {
            a.picks[(int64_t)r * a.keep + i] = i < kept ? key_bucket(best[i]) : -1;
            if (a.pick_keys) {  // same score bits, column rebased (e.g. to a global bucket id)
                int64_t key = kEmpty;
                if (i < kept) {
                    const uint64_t hi = (uint64_t)best[i] & 0xFFFFFFFF00000000ull;
                    key = (int64_t)(hi | (uint32_t)(0x7FFFFFFF - (key_bucket(best[i]) + (int32_t)a.col_offset)));
                }
                a.pick_keys[(int64_t)r * a.keep + i] = key;
            }
        }
    } else {
        int S = (int)a.size;
        for (int i = threadIdx.x; i < kept * S; i += blockDim.x) {
            int node = key_bucket(best[i / S]);
            a.carried_out[(int64_t)r * a.carry_cap + i] = (int32_t)a.children[(int64_t)node * S + (i % S)];
        }
        if (threadIdx.x == 0) a.carried_n_out[r] = active ? kept * S : 0;
    }
}

// ------------------------------------------------------------------ cluster beam (few rows)

// One thread-block cluster per row walks every level in ONE launch (the multi-launch form
// above pays a launch, a ticket round trip and a global key round trip per level):
//   * before griddepcontrol.wait the cluster pulls every node level's centroid rows into L2
//     (the index is read-only here; prefetches cannot observe stale data), and reads the
//     row's position and derives its growth: positions are inputs of the step, which no
//     kernel of this library writes (the ones that let their dependents start early write
//     lists, keys, picks, index queries or outputs); only the index query, which the
//     previous kernel may produce, is read after the wait;
//   * per level, every CTA derives the level's candidate count from the row's growth and the
//     previous level's kept count (the same arithmetic in every CTA), scores its share of the
//     candidates (one warp per two candidates, both rows' loads in flight before the FMAs,
//     canonical fp32 cdot, the row's query staged in shared memory;
//     carried ids read from the leader's shared memory through DSMEM) and stores the packed
//     keys into the leader's shared memory;
//   * one cluster barrier; the leader keeps the best beam_width (top_p at level 0) by warp-list
//     top-K and writes the next level's carried children into its shared memory; a second
//     barrier publishes them. Level 0 writes the picks (and their rebased keys) and, for
//     lsa_tree_select_lists, walks the expansion in the leader: the picked member rows staged
//     in shared memory by 16-byte cp.async (one round trip), then the same walk as the
//     expansion kernel - read lists without a second launch.
// Same picks as the multi-launch form (same candidates, same keys, same order).
constexpr int kTreeCThreads = 512;
constexpr int kTreeCWarps = kTreeCThreads / 32;
constexpr int kTreeCMaxCand = 4096;
constexpr int kTreeMaxD = 2048;                     // index dims (the entry points check d)

struct TreeClusterArgs {
    const float* q;
    int64_t d;
    const int32_t* positions;
    int64_t block, bpb, nb, size, rows;
    int top_level, n_built, beam, top_p;
    const float* lc[kTreeMaxLevels];    // node level l + 1 centroids [n, d] fp32
    const int64_t* lk[kTreeMaxLevels];  // node level l + 1 children [n, size]
    int64_t ln[kTreeMaxLevels];         // node level l + 1 node counts
    const float* bc;                    // bucket centroids_f32 [rows, d]
    int32_t* picks;                     // [R, top_p]
    int64_t* pick_keys;                 // [R, top_p] or null
    int64_t col_offset;
    int cand_cap, carry_cap;
    int32_t* status;
    // the expansion walk (lists != null): members [member_rows, cap], staged at byte offset
    // stage_off of the dynamic shared memory
    const int32_t* members;
    int64_t member_rows;
    int cap, window, sink, top_k, vec16, stage_off;
    int32_t* lists;
    int32_t* lengths;
};

struct SmemKeys {
    const int64_t* k;
    int n;
    __device__ int64_t operator()(int i) const { return i < n ? k[i] : kEmpty; }
};

// One candidate row's lane chunks (fp32, 8 per chunk; chunks past nchunks are not read)
// and the lane's partial of the canonical cdot over them - the order of lane_partial_regs,
// split so two rows' loads can be in flight before either row's FMAs.
template <int CHUNKS>
__device__ __forceinline__ void load_row_chunks(const float* y, int lane, int nchunks, float (&v)[CHUNKS][8]) {
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
        const int c = lane + 32 * j;
        if (c < nchunks) load8<float>(y + (size_t)c * 8, v[j]);
    }
}
// The lane's partial of one row against the query staged in shared memory (qs), in the
// order of lane_partial_regs (chunk by chunk, element by element).
template <int CHUNKS>
__device__ __forceinline__ float lane_partial1(const float* qs, const float (&v)[CHUNKS][8], int lane, int nchunks) {
    float p = 0.0f;
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
        const int c = lane + 32 * j;
        if (c < nchunks) {
            float xv[8];
            load8<float>(qs + (size_t)c * 8, xv);
#pragma unroll
            for (int e = 0; e < 8; ++e) p = __fmaf_rn(xv[e], v[j][e], p);
        }
    }
    return p;
}
// The same for two rows at once (one query chunk read feeds both).
template <int CHUNKS>
__device__ __forceinline__ void lane_partials2(const float* qs, const float (&v1)[CHUNKS][8],
                                               const float (&v2)[CHUNKS][8], int lane, int nchunks, float& p1,
                                               float& p2) {
    p1 = 0.0f;
    p2 = 0.0f;
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
        const int c = lane + 32 * j;
        if (c < nchunks) {
            float xv[8];
            load8<float>(qs + (size_t)c * 8, xv);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                p1 = __fmaf_rn(xv[e], v1[j][e], p1);
                p2 = __fmaf_rn(xv[e], v2[j][e], p2);
            }
        }
    }
}

__device__ __forceinline__ void tc_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

template <int CHUNKS, int KW>
__global__ void __launch_bounds__(kTreeCThreads) tree_cluster_kernel(const TreeClusterArgs a) {
    constexpr int K = 32 * KW;
    extern __shared__ __align__(16) int64_t csm[];
    int64_t* keys = csm;                                             // [cand_cap]
    int64_t* lists = keys + a.cand_cap;                              // [kTreeCWarps * K]
    int64_t* best = lists + kTreeCWarps * K;                         // [K]
    int32_t* carried = reinterpret_cast<int32_t*>(best + K);         // [carry_cap]
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank(), cs = (int)cluster.num_blocks();
    const int r = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // every CTA has started before any DSMEM store (waited on before the first one)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    {
        const int lines = (int)(a.d * 4 / 128);
        for (int l = 0; l < a.n_built; ++l)
            for (int64_t n = (int64_t)rank * kTreeCWarps + warp; n < a.ln[l]; n += (int64_t)cs * kTreeCWarps)
                for (int i = lane; i < lines; i += 32)
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(a.lc[l] + n * a.d) +
                                                                  i * 128));
    }
    const int64_t pos = a.positions[r];
    const int64_t page = pos / a.block;
    TreeGrowth g;
    growth_at(page, a.bpb, a.nb, a.size, a.top_level, a.rows, a.n_built, g);
    pdl_wait();
    pdl_trigger();
    const int nchunks = (int)(a.d >> 3);
    __shared__ __align__(16) float qs[kTreeMaxD];
    for (int i = threadIdx.x; i < nchunks * 2; i += kTreeCThreads)
        reinterpret_cast<float4*>(qs)[i] = reinterpret_cast<const float4*>(a.q + r * a.d)[i];
    __syncthreads();
    int64_t* lead_keys = cluster.map_shared_rank(keys, 0);
    const int32_t* lead_carried = cluster.map_shared_rank(carried, 0);
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // (first phase)
    int carried_n = 0;
    for (int L = a.n_built; L >= 0; --L) {
        const bool active = L == 0 || g.levels >= L;  // the same in every CTA of the row
        if (!active) {
            carried_n = 0;
            continue;
        }
        int n_carried, fresh0, fresh1;
        if (L == 0) {
            n_carried = g.levels > 0 ? carried_n : 0;
            const int64_t vis = page * a.bpb;
            fresh0 = g.levels > 0 ? g.covered : 0;
            fresh1 = (int)(vis < a.rows ? vis : a.rows);
        } else {
            n_carried = g.levels > L ? carried_n : 0;
            fresh0 = g.levels == L ? 0 : g.closed[L - 1];
            fresh1 = g.made[L - 1];
        }
        if (fresh1 < fresh0) fresh1 = fresh0;
        int n_cand = n_carried + (fresh1 - fresh0);
        if (n_cand > a.cand_cap) {  // never for a consistent hierarchy; recorded, then clamped
            if (threadIdx.x == 0 && rank == 0) atomicExch(a.status, LSA_ERR_ARG);
            n_cand = a.cand_cap;
        }
        const float* cent = L > 0 ? a.lc[L - 1] : a.bc;
        // two candidates per warp pass (both rows' loads in flight before the FMAs) while two
        // rows fit the registers (d <= 1024), else one
        constexpr int PAIR = CHUNKS <= 4 ? 2 : 1;
        const int stride = cs * kTreeCWarps;
        for (int i = rank * kTreeCWarps + warp; i < n_cand; i += PAIR * stride) {
            const int id = i < n_carried ? lead_carried[i] : fresh0 + (i - n_carried);
            float v1[CHUNKS][8];
            if constexpr (PAIR == 2) {
                const int i2 = i + stride;
                const bool two = i2 < n_cand;  // (warp-uniform)
                const int id2 = !two ? id : (i2 < n_carried ? lead_carried[i2] : fresh0 + (i2 - n_carried));
                float v2[CHUNKS][8];
                load_row_chunks<CHUNKS>(cent + (int64_t)id * a.d, lane, nchunks, v1);
                load_row_chunks<CHUNKS>(cent + (int64_t)id2 * a.d, lane, nchunks, v2);
                float p1, p2;
                lane_partials2<CHUNKS>(qs, v1, v2, lane, nchunks, p1, p2);
                const float s1 = butterfly_sum(p1);
                const float s2 = butterfly_sum(p2);
                if (lane == 0) {
                    lead_keys[i] = pack_key(s1, id);
                    if (two) lead_keys[i2] = pack_key(s2, id2);
                }
            } else {
                load_row_chunks<CHUNKS>(cent + (int64_t)id * a.d, lane, nchunks, v1);
                const float s1 = butterfly_sum(lane_partial1<CHUNKS>(qs, v1, lane, nchunks));
                if (lane == 0) lead_keys[i] = pack_key(s1, id);
            }
        }
        tc_arrive();
        const int keep = L > 0 ? a.beam : a.top_p;
        const int kept = n_cand < keep ? n_cand : keep;
        if (L == 0 && rank != 0) return;  // nothing of this CTA is read after the last scores
        tc_wait();
        // a node level whose candidates all stay needs no top-K: only the kept SET matters
        // below it (the next level's keys carry the bucket / node id, so the carried order
        // cannot change any pick), and the keys are read in place
        const bool all_kept = L > 0 && n_cand <= keep;
        if (rank == 0) {
            // the picks of a top_p <= 32 walk: 32-key warp lists (half the sort work of the
            // beam's wider lists; the same best 32 keys in the same order)
            bool narrow = false;
            if constexpr (KW > 1) narrow = L == 0 && a.top_p <= 32;
            if (narrow)
                group_topk_desc<1, kTreeCWarps>(SmemKeys{keys, n_cand}, n_cand, lists, best, warp, lane,
                                                TreeBlockSync{});
            else if (!all_kept)
                group_topk_desc<KW, kTreeCWarps>(SmemKeys{keys, n_cand}, n_cand, lists, best, warp, lane,
                                                 TreeBlockSync{});
            if (L == 0) {
                for (int i = threadIdx.x; i < a.top_p; i += kTreeCThreads) {
                    a.picks[(int64_t)r * a.top_p + i] = i < kept ? key_bucket(best[i]) : -1;
                    if (a.pick_keys) {  // same score bits, column rebased (e.g. to a global bucket id)
                        int64_t key = kEmpty;
                        if (i < kept) {
                            const uint64_t hi = (uint64_t)best[i] & 0xFFFFFFFF00000000ull;
                            key = (int64_t)(hi |
                                            (uint32_t)(0x7FFFFFFF - (key_bucket(best[i]) + (int32_t)a.col_offset)));
                        }
                        a.pick_keys[(int64_t)r * a.top_p + i] = key;
                    }
                }
                if (a.lists) {  // the expansion of the picks (best[0, kept); the rest read as -1)
                    __shared__ int scan_smem[33];
                    const int P = a.top_p, cap = a.cap, total = P * cap;
                    int* mem = reinterpret_cast<int*>(reinterpret_cast<char*>(csm) + a.stage_off);
                    int* gather = mem + ((total + 3) & ~3);
                    auto bucket = [&](int pk) -> int64_t {
                        const int64_t b = pk < kept ? (int64_t)key_bucket(best[pk]) : -1;
                        return b >= 0 && b < a.member_rows ? b : -1;
                    };
                    if (a.vec16) {
                        const int q4 = cap / 4;
                        for (int i = threadIdx.x; i < P * q4; i += kTreeCThreads) {
                            const int pk = i / q4, piece = i - pk * q4;
                            const int64_t b = bucket(pk);
                            int* dst = mem + pk * cap + piece * 4;
                            if (b >= 0) cp_async16(smem_u32(dst), a.members + b * cap + piece * 4, 16);
                            else *reinterpret_cast<int4*>(dst) = make_int4(-1, -1, -1, -1);
                        }
                        cp_async_wait_all();
                    } else {
                        for (int i = threadIdx.x; i < total; i += kTreeCThreads) {
                            const int pk = i / cap;
                            const int64_t b = bucket(pk);
                            mem[i] = b >= 0 ? a.members[b * cap + (i - pk * cap)] : -1;
                        }
                    }
                    __syncthreads();
                    const int width = a.top_k + a.window + a.sink;
                    expand_walk<kTreeCThreads>(mem, total, pos, a.window, a.sink, a.top_k,
                                               a.lists + (int64_t)r * width, width, a.lengths + r, scan_smem,
                                               (int)threadIdx.x, TreeBlockSync{}, gather);
                }
                return;
            }
            const int S = (int)a.size;
            const int64_t* kept_keys = all_kept ? keys : best;
            for (int i = threadIdx.x; i < kept * S; i += kTreeCThreads)
                carried[i] = (int32_t)a.lk[L - 1][(int64_t)key_bucket(kept_keys[i / S]) * S + (i % S)];
        }
        carried_n = kept * (int)a.size;
        // the leader's carried list (and its finished reads of the keys) before the next scores
        tc_arrive();
        tc_wait();
    }
}

static int64_t r256(int64_t x) { return (x + 255) / 256 * 256; }

struct TreePlan {
    int carry_cap, cand_cap;
    int64_t keys_bytes, carry_bytes, scratch_bytes, counters;
};

static TreePlan plan_tree(int64_t R, int64_t n_built, const int64_t* level_counts, int64_t beam, int64_t size,
                          int64_t nb, int64_t bpb, int64_t top_p) {
    TreePlan p;
    int64_t carry = beam * size;
    int64_t thr = bpb / nb > 1 ? bpb / nb : 1;
    int64_t cand = carry + nb * thr + 1;  // level 0 bound
    for (int64_t l = 0; l < n_built; ++l) {
        int64_t c = level_counts[l] > carry + nb ? level_counts[l] : carry + nb;
        if (c > cand) cand = c;
    }
    (void)top_p;
    p.carry_cap = (int)(carry > 0 ? carry : 1);
    p.cand_cap = (int)cand;
    p.keys_bytes = r256(R * cand * 8);
    p.carry_bytes = r256(R * p.carry_cap * 4) * 2 + r256(R * 4) * 2;
    p.scratch_bytes = p.keys_bytes + p.carry_bytes;
    p.counters = R + 1;
    return p;
}

// The expansion a tree select may finish with (lsa_tree_select_lists).
struct TreeWalk {
    const int32_t* members;
    int64_t member_rows, cap, window, sink, top_k;
    int32_t* lists;
    int32_t* lengths;
};
constexpr int64_t kTreeWalkSmem = 128 * 1024;  // staged member slots + gathered list, bytes

}  // namespace lsa

using namespace lsa;

extern "C" {

int lsa_tree_plan(int64_t R, int64_t n_built, const int64_t* level_counts, int64_t beam, int64_t size, int64_t nb,
                  int64_t bpb, int64_t top_p, int64_t* scratch_bytes, int64_t* n_counters) {
    if (n_built < 0 || n_built > kTreeMaxLevels || beam <= 0 || size <= 0 || nb <= 0) return LSA_ERR_ARG;
    TreePlan p = plan_tree(R, n_built, level_counts, beam, size, nb, bpb, top_p);
    if (p.cand_cap > kTreeSortCap) return LSA_ERR_ARG;
    if (scratch_bytes) *scratch_bytes = p.scratch_bytes;
    if (n_counters) *n_counters = p.counters;
    return LSA_OK;
}

// Tree beam picks [R, top_p] int32 (-1 padded). level_centroids / level_children /
// level_counts are HOST arrays of n_built entries (device pointers / node counts).
int lsa_tree_select_keys(const float* q, int64_t R, int64_t d, const int32_t* positions, int64_t block, int64_t bpb,
                         int64_t rows, int64_t n_built, const float* const* level_centroids,
                         const int64_t* const* level_children, const int64_t* level_counts,
                         const float* bucket_centroids, int64_t size, int64_t nb, int64_t top_level, int64_t beam,
                         int64_t top_p, int32_t* picks, int64_t* pick_keys, int64_t col_offset, void* scratch,
                         int64_t scratch_bytes, int32_t* counters, int64_t n_counters, cudaStream_t stream);

int lsa_tree_select(const float* q, int64_t R, int64_t d, const int32_t* positions, int64_t block, int64_t bpb,
                    int64_t rows, int64_t n_built, const float* const* level_centroids,
                    const int64_t* const* level_children, const int64_t* level_counts, const float* bucket_centroids,
                    int64_t size, int64_t nb, int64_t top_level, int64_t beam, int64_t top_p, int32_t* picks,
                    void* scratch, int64_t scratch_bytes, int32_t* counters, int64_t n_counters, cudaStream_t stream) {
    return lsa_tree_select_keys(q, R, d, positions, block, bpb, rows, n_built, level_centroids, level_children,
                                level_counts, bucket_centroids, size, nb, top_level, beam, top_p, picks, nullptr, 0,
                                scratch, scratch_bytes, counters, n_counters, stream);
}

// The beam (and, with walk, the expansion when the one-launch cluster form takes the call:
// *walked tells the caller whether the lists are written).
static int tree_select_run(const float* q, int64_t R, int64_t d, const int32_t* positions, int64_t block, int64_t bpb,
                           int64_t rows, int64_t n_built, const float* const* level_centroids,
                           const int64_t* const* level_children, const int64_t* level_counts,
                           const float* bucket_centroids, int64_t size, int64_t nb, int64_t top_level, int64_t beam,
                           int64_t top_p, int32_t* picks, int64_t* pick_keys, int64_t col_offset, void* scratch,
                           int64_t scratch_bytes, int32_t* counters, int64_t n_counters, cudaStream_t stream,
                           const TreeWalk* walk, bool* walked) {
    if (walked) *walked = false;
    if (col_offset < 0 || col_offset + rows > INT32_MAX) return LSA_ERR_ARG;
    if (d <= 0 || d % 8 || d > 2048 || ((uintptr_t)q & 15) || top_level > kTreeMaxLevels || n_built > top_level)
        return LSA_ERR_ARG;
    if (top_p <= 0 || top_p > kTreeSortCap || block <= 0) return LSA_ERR_ARG;
    TreePlan p = plan_tree(R, n_built, level_counts, beam, size, nb, bpb, top_p);
    if (p.cand_cap > kTreeSortCap || scratch_bytes < p.scratch_bytes || n_counters < p.counters) return LSA_ERR_ARG;
    if (R == 0) return LSA_OK;
    char* w = (char*)scratch;
    TreeLevelArgs a;
    a.q = q; a.d = d; a.positions = positions; a.block = block; a.bpb = bpb; a.nb = nb; a.size = size;
    a.rows = rows; a.top_level = (int)top_level; a.n_built = (int)n_built;
    a.ws_keys = (int64_t*)w;
    a.cand_cap = p.cand_cap;
    a.carry_cap = p.carry_cap;
    int32_t* carry[2] = {(int32_t*)(w + p.keys_bytes), (int32_t*)(w + p.keys_bytes + r256(R * p.carry_cap * 4))};
    int32_t* carry_n[2] = {(int32_t*)(w + p.keys_bytes + 2 * r256(R * p.carry_cap * 4)),
                           (int32_t*)(w + p.keys_bytes + 2 * r256(R * p.carry_cap * 4) + r256(R * 4))};
    a.tickets = counters;
    a.status = counters + R;
    a.picks = picks;
    a.pick_keys = pick_keys;
    a.col_offset = col_offset;
    int chunks = (int)((d / 8 + 31) / 32);
    // few rows: the whole beam in one cluster launch per row
    const int ckw = (beam <= 32 && top_p <= 32) ? 1 : ((beam <= 64 && top_p <= 64) ? 2 : ((beam <= 128 && top_p <= 128) ? 4 : 0));
    if (R <= 64 && ckw && p.cand_cap <= kTreeCMaxCand && size <= 64 && chunks <= 8) {
        TreeClusterArgs c;
        c.q = q; c.d = d; c.positions = positions; c.block = block; c.bpb = bpb; c.nb = nb; c.size = size;
        c.rows = rows; c.top_level = (int)top_level; c.n_built = (int)n_built; c.beam = (int)beam;
        c.top_p = (int)top_p;
        for (int l = 0; l < kTreeMaxLevels; ++l) {
            c.lc[l] = l < n_built ? level_centroids[l] : nullptr;
            c.lk[l] = l < n_built ? level_children[l] : nullptr;
            c.ln[l] = l < n_built ? level_counts[l] : 0;
        }
        c.bc = bucket_centroids; c.picks = picks; c.pick_keys = pick_keys; c.col_offset = col_offset;
        c.cand_cap = p.cand_cap; c.carry_cap = p.carry_cap; c.status = counters + R;
        c.members = nullptr; c.member_rows = 0; c.cap = 0; c.window = 0; c.sink = 0; c.top_k = 0; c.vec16 = 0;
        c.stage_off = 0; c.lists = nullptr; c.lengths = nullptr;
        int64_t staged = 0;  // bytes of the walk's shared memory (0: no walk in this launch)
        if (walk) {
            const int64_t slots = top_p * walk->cap;
            const int64_t bytes = ((slots + 3) / 4 * 4 + walk->top_k) * 4;
            if (slots < (1 << 30) && bytes <= kTreeWalkSmem) {
                staged = bytes;
                c.members = walk->members; c.member_rows = walk->member_rows; c.cap = (int)walk->cap;
                c.window = (int)walk->window; c.sink = (int)walk->sink; c.top_k = (int)walk->top_k;
                c.vec16 = walk->cap % 4 == 0 && ((uintptr_t)walk->members & 15) == 0;
                c.lists = walk->lists; c.lengths = walk->lengths;
            }
        }
        const int Kc = 32 * ckw;
        const int base = (int)(p.cand_cap * 8 + (kTreeCWarps + 1) * Kc * 8 + ((p.carry_cap + 3) / 4) * 16);
        c.stage_off = (base + 15) / 16 * 16;
        const int csmem = staged ? c.stage_off + (int)staged : base;
        int most = p.cand_cap;  // scoring warps the widest level can use
        int cs = (most + kTreeCWarps * 2 - 1) / (kTreeCWarps * 2);
        if (cs < 1) cs = 1;
        if (cs > 16) cs = 16;
        cudaLaunchAttribute at[2];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        at[1].id = cudaLaunchAttributeClusterDimension;
        at[1].val.clusterDim.x = (unsigned)cs;
        at[1].val.clusterDim.y = 1;
        at[1].val.clusterDim.z = 1;
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3((unsigned)cs, (unsigned)R);
        lc.blockDim = dim3(kTreeCThreads);
        lc.dynamicSmemBytes = csmem;
        lc.stream = stream;
        lc.attrs = at;
        lc.numAttrs = 2;
        auto go = [&](auto kern) -> int {
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, csmem) != cudaSuccess)
                return LSA_ERR_CUDA;
            if (cs > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
                return LSA_ERR_CUDA;
            if (cudaLaunchKernelEx(&lc, kern, c) != cudaSuccess) return LSA_ERR_CUDA;
            if (walked) *walked = staged > 0;
            return LSA_OK;
        };
#define LSA_TC_KW(CH)                                               \
    do {                                                            \
        if (ckw == 1) return go(tree_cluster_kernel<CH, 1>);        \
        if (ckw == 2) return go(tree_cluster_kernel<CH, 2>);        \
        return go(tree_cluster_kernel<CH, 4>);                      \
    } while (0)
        if (chunks <= 1) LSA_TC_KW(1);
        if (chunks <= 2) LSA_TC_KW(2);
        if (chunks <= 4) LSA_TC_KW(4);
        LSA_TC_KW(8);
#undef LSA_TC_KW
    }
    int smem = next_pow2(p.cand_cap) * 8;
    if (smem < 1024) smem = 1024;
    int sms = 148;
    {
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    int cur = 0;
    for (int64_t L = n_built; L >= 0; --L) {
        a.L = (int)L;
        a.centroids = L > 0 ? level_centroids[L - 1] : bucket_centroids;
        a.children = L > 0 ? level_children[L - 1] : nullptr;
        a.keep = (int)(L > 0 ? beam : top_p);
        a.carried_in = carry[cur];
        a.carried_n_in = carry_n[cur];
        a.carried_out = carry[cur ^ 1];
        a.carried_n_out = carry_n[cur ^ 1];
        int64_t bound = L > 0 ? (level_counts[L - 1] > p.carry_cap + nb ? level_counts[L - 1] : p.carry_cap + nb)
                              : p.cand_cap;
        int64_t want = (bound + 15) / 16;  // 8 warps x 2 candidates per CTA
        int64_t spread = (2 * (int64_t)sms + R - 1) / R;  // about two CTAs per SM over all rows
        unsigned gx = (unsigned)(want < spread ? want : spread);
        if (gx < 1) gx = 1;
        dim3 grid(gx, (unsigned)R);
        // the kept keys: warp-list top-K for keep <= 128 (K keys per warp, merge tree), else a
        // full bitonic sort of the candidates
        const int kw = a.keep <= 32 ? 1 : (a.keep <= 64 ? 2 : (a.keep <= 128 ? 4 : 0));
        const int lsmem = kw ? 9 * 32 * kw * 8 : smem;
#define LSA_TL(CH, KW)                                                                                      \
    do {                                                                                                    \
        auto kern = tree_level_kernel<CH, KW>;                                                              \
        if (lsmem > 40 * 1024 &&                                                                            \
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, lsmem) != cudaSuccess) \
            return LSA_ERR_CUDA;                                                                            \
        kern<<<grid, 256, lsmem, stream>>>(a);                                                              \
    } while (0)
#define LSA_TL_KW(CH)                         \
    do {                                      \
        if (kw == 1) LSA_TL(CH, 1);           \
        else if (kw == 2) LSA_TL(CH, 2);      \
        else if (kw == 4) LSA_TL(CH, 4);      \
        else LSA_TL(CH, 0);                   \
    } while (0)
        if (chunks <= 1) LSA_TL_KW(1);
        else if (chunks <= 2) LSA_TL_KW(2);
        else if (chunks <= 4) LSA_TL_KW(4);
        else LSA_TL_KW(8);
#undef LSA_TL_KW
#undef LSA_TL
        LSA_LAUNCH_CHECK();
        cur ^= 1;
    }
    return LSA_OK;
}

int lsa_tree_select_keys(const float* q, int64_t R, int64_t d, const int32_t* positions, int64_t block, int64_t bpb,
                         int64_t rows, int64_t n_built, const float* const* level_centroids,
                         const int64_t* const* level_children, const int64_t* level_counts,
                         const float* bucket_centroids, int64_t size, int64_t nb, int64_t top_level, int64_t beam,
                         int64_t top_p, int32_t* picks, int64_t* pick_keys, int64_t col_offset, void* scratch,
                         int64_t scratch_bytes, int32_t* counters, int64_t n_counters, cudaStream_t stream) {
    return tree_select_run(q, R, d, positions, block, bpb, rows, n_built, level_centroids, level_children,
                           level_counts, bucket_centroids, size, nb, top_level, beam, top_p, picks, pick_keys,
                           col_offset, scratch, scratch_bytes, counters, n_counters, stream, nullptr, nullptr);
}

int lsa_expand_in_order(const int32_t* picked, int64_t R, int64_t P, int64_t ldp, const int32_t* members,
                        int64_t member_rows, int64_t cap, const int32_t* positions, int64_t window, int64_t sink,
                        int64_t top_k, int32_t* lists, int32_t* lengths, cudaStream_t stream);

// The beam's picks and their expansion into read lists: one launch when the cluster form
// takes the rows and the staged members fit its shared memory, else the beam then the
// expansion kernel - the same lists either way.
int lsa_tree_select_lists(const float* q, int64_t R, int64_t d, const int32_t* positions, int64_t block, int64_t bpb,
                          int64_t rows, int64_t n_built, const float* const* level_centroids,
                          const int64_t* const* level_children, const int64_t* level_counts,
                          const float* bucket_centroids, int64_t size, int64_t nb, int64_t top_level, int64_t beam,
                          int64_t top_p, const int32_t* members, int64_t member_rows, int64_t cap, int64_t window,
                          int64_t sink, int64_t top_k, int32_t* picks, int32_t* lists, int32_t* lengths,
                          void* scratch, int64_t scratch_bytes, int32_t* counters, int64_t n_counters,
                          cudaStream_t stream) {
    if (!members || !picks || !lists || !lengths || cap <= 0 || member_rows < 0 || window < 0 || sink < 0 ||
        top_k < 0)
        return LSA_ERR_ARG;
    TreeWalk w{members, member_rows, cap, window, sink, top_k, lists, lengths};
    bool walked = false;
    int rc = tree_select_run(q, R, d, positions, block, bpb, rows, n_built, level_centroids, level_children,
                             level_counts, bucket_centroids, size, nb, top_level, beam, top_p, picks, nullptr, 0,
                             scratch, scratch_bytes, counters, n_counters, stream, &w, &walked);
    if (rc != LSA_OK || walked || R == 0) return rc;
    return lsa_expand_in_order(picks, R, top_p, top_p, members, member_rows, cap, positions, window, sink, top_k,
                               lists, lengths, stream);
}

}  // extern "C"
