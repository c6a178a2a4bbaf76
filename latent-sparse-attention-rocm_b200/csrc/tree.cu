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
//     (the hierarchy is read-only here; prefetches cannot observe stale data);
//   * per level, every CTA derives the level's candidate count from the row's growth and the
//     previous level's kept count (the same arithmetic in every CTA), scores its share of the
//     candidates (one warp per candidate, canonical fp32 cdot, the row's query in registers;
//     carried ids read from the leader's shared memory through DSMEM) and stores the packed
//     keys into the leader's shared memory;
//   * one cluster barrier; the leader keeps the best beam_width (top_p at level 0) by warp-list
//     top-K and writes the next level's carried children into its shared memory; a second
//     barrier publishes them. Level 0 writes the picks (and their rebased keys).
// Same picks as the multi-launch form (same candidates, same keys, same order).
constexpr int kTreeCThreads = 512;
constexpr int kTreeCWarps = kTreeCThreads / 32;
constexpr int kTreeCMaxCand = 4096;

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
};

struct SmemKeys {
    const int64_t* k;
    int n;
    __device__ int64_t operator()(int i) const { return i < n ? k[i] : kEmpty; }
};

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
    pdl_wait();
    pdl_trigger();
    const int64_t pos = a.positions[r];
    const int64_t page = pos / a.block;
    TreeGrowth g;
    growth_at(page, a.bpb, a.nb, a.size, a.top_level, a.rows, a.n_built, g);
    const int nchunks = (int)(a.d >> 3);
    float x[CHUNKS][8];
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
        const int ch = min(lane + 32 * j, nchunks - 1);
        load8<float>(a.q + r * a.d + (size_t)ch * 8, x[j]);
    }
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
        for (int i = rank * kTreeCWarps + warp; i < n_cand; i += cs * kTreeCWarps) {
            const int id = i < n_carried ? lead_carried[i] : fresh0 + (i - n_carried);
            const float s = butterfly_sum(lane_partial_regs<float, CHUNKS>(x, cent + (int64_t)id * a.d, lane, nchunks));
            if (lane == 0) lead_keys[i] = pack_key(s, id);
        }
        tc_arrive();
        const int keep = L > 0 ? a.beam : a.top_p;
        const int kept = n_cand < keep ? n_cand : keep;
        if (L == 0 && rank != 0) return;  // nothing of this CTA is read after the last scores
        tc_wait();
        if (rank == 0) {
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
                return;
            }
            const int S = (int)a.size;
            for (int i = threadIdx.x; i < kept * S; i += kTreeCThreads)
                carried[i] = (int32_t)a.lk[L - 1][(int64_t)key_bucket(best[i / S]) * S + (i % S)];
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

int lsa_tree_select_keys(const float* q, int64_t R, int64_t d, const int32_t* positions, int64_t block, int64_t bpb,
                         int64_t rows, int64_t n_built, const float* const* level_centroids,
                         const int64_t* const* level_children, const int64_t* level_counts,
                         const float* bucket_centroids, int64_t size, int64_t nb, int64_t top_level, int64_t beam,
                         int64_t top_p, int32_t* picks, int64_t* pick_keys, int64_t col_offset, void* scratch,
                         int64_t scratch_bytes, int32_t* counters, int64_t n_counters, cudaStream_t stream) {
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
        const int Kc = 32 * ckw;
        const int csmem = (int)(p.cand_cap * 8 + (kTreeCWarps + 1) * Kc * 8 + ((p.carry_cap + 3) / 4) * 16);
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
            return cudaLaunchKernelEx(&lc, kern, c) == cudaSuccess ? LSA_OK : LSA_ERR_CUDA;
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

}  // extern "C"
