// build.cu - index space, bucket build (pools + spherical Ward merge + members +
// centroids), positional buckets and node-bucket pairing (sm_100a).
//
// Reference (AIwork4me/latent-sparse-attention-rocm, paths inside that project):
//   make_index_space -> upstream regroup     src/lsa_rocm_lab/port/gates.py:50-59
//   build_buckets_gpu                        src/lsa_rocm_lab/port/pipeline.py:71-116
//   position_buckets                         pipeline.py:378-403
//   _pair_to_size / build_hierarchy_gpu      pipeline.py:136-181
// The upstream Ward kernels are absent from the reference; this file implements the
// merge rules the CPU checker defines, with the same operation sequence (explicit _rn
// intrinsics, no contraction), so labels, members and centroids match it bit-for-bit.
//
// Ward merge, one CTA per cluster block, Gram matrix resident in shared memory:
//   rounds of mutual nearest partners under the size cap (packed int64 cost|index keys),
//   cheapest mutual pairs merged first, at most count - target per round, all merges of
//   a round applied together from the previous Gram matrix. The rounds are incremental: a
//   cluster searches every partner only when it or its partner changed in the last round,
//   and the Gram update visits only the pairs of a merging cluster - the same keys and
//   values as recomputing everything.
// k == nullptr in the regroup kernels: index queries only.
#include "common.cuh"

namespace lsa {

// ------------------------------------------------------------------ index space

// iq[t, h*D+e] = (sum_g q[t, h*G+g, e]) / G ; ik[t] = k[t] / max(|k[t]|, 1e-12), one warp per t.
template <typename T>
__global__ void regroup_kernel(const T* __restrict__ q, const T* __restrict__ k, int64_t Tn, int Hq, int Hkv, int D,
                               float* __restrict__ iq, float* __restrict__ ik) {
    int lane = threadIdx.x & 31;
    int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= Tn) return;
    int G = Hq / Hkv, d = Hkv * D;
    for (int j = lane; j < d; j += 32) {
        int h = j / D, e = j % D;
        float acc = 0.0f;
        for (int g = 0; g < G; ++g) acc = __fadd_rn(acc, to_f32(q[(t * Hq + h * G + g) * D + e]));
        iq[t * d + j] = __fdiv_rn(acc, (float)G);
    }
    if (k == nullptr) return;  // index queries only
    const T* row = k + t * Hkv * D;
    float n = __fsqrt_rn(warp_cdot<T, T>(row, row, d, lane));
    float den = fmaxf(n, 1e-12f);
    for (int j = lane; j < d; j += 32) ik[t * d + j] = __fdiv_rn(to_f32(row[j]), den);
}

// The same per-row arithmetic as regroup_kernel for few rows (decode): one CTA of 256
// threads per row, every thread's query loads in flight together (elements j = tid + 256 i,
// G group members each, summed in group order then divided by G), the key norm by warp 0
// (the canonical warp dot), then every thread divides its elements. Requires G <= 8 and
// d <= 2048.
constexpr int kRegroupThreads = 256;
template <typename T>
__global__ void __launch_bounds__(kRegroupThreads) regroup_row_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                                      int Hq, int Hkv, int D, float* __restrict__ iq,
                                                                      float* __restrict__ ik) {
    __shared__ float den_s;
    // launched with programmatic stream serialization (decode: right after the previous
    // layer's read): q and k are read only after the previous kernel has completed
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int64_t t = blockIdx.x;
    const int tid = threadIdx.x;
    const int G = Hq / Hkv, d = Hkv * D;
    constexpr int kPer = 2048 / kRegroupThreads;
    float qv[kPer][8];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {  // unconditional loads at clamped in-range addresses
        const int j = min(tid + kRegroupThreads * i, d - 1);
        const int h = j / D, e = j % D;
#pragma unroll
        for (int g = 0; g < 8; ++g) qv[i][g] = to_f32(q[(t * Hq + h * G + min(g, G - 1)) * D + e]);
    }
    const T* row = k + t * Hkv * D;
    if (k != nullptr && tid < 32) {
        const float n = __fsqrt_rn(warp_cdot<T, T>(row, row, d, tid));
        if (tid == 0) den_s = fmaxf(n, 1e-12f);
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int j = tid + kRegroupThreads * i;
        if (j < d) {
            float acc = 0.0f;
#pragma unroll
            for (int g = 0; g < 8; ++g)
                if (g < G) acc = __fadd_rn(acc, qv[i][g]);
            iq[t * d + j] = __fdiv_rn(acc, (float)G);
        }
    }
    if (k == nullptr) return;  // index queries only (block-uniform)
    __syncthreads();
    const float den = den_s;
    for (int j = tid; j < d; j += kRegroupThreads) ik[t * d + j] = __fdiv_rn(to_f32(row[j]), den);
}

// regroup through a D-LSA projection map Wt [d_out, d] (fp32, one row per output dim): the
// group mean of q and the concatenated k row of each position, projected by canonical dots
// with Wt's rows (lane = chunk mod 32, fmaf chain in chunk order, butterfly), the projected
// key then normalised by its canonical norm - bit-equal to the checker's regroup_project.
// A CTA takes 8 positions (staged in shared memory) so each warp's load of a map row serves
// 8 positions; 8 warps stride the output dims. Dynamic smem: (16 d + 8 d_out) floats.
constexpr int kProjRows = 8;
template <typename T, int CH>
__global__ void __launch_bounds__(256) regroup_project_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                              int64_t Tn, int Hq, int Hkv, int D,
                                                              const float* __restrict__ Wt, int d_out,
                                                              float* __restrict__ iq, float* __restrict__ ik) {
    extern __shared__ __align__(16) float psm[];
    __shared__ float den_s[kProjRows];
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int d = Hkv * D, G = Hq / Hkv;
    float* xq = psm;                   // [kProjRows][d]
    float* xk = xq + kProjRows * d;    // [kProjRows][d]
    float* pk = xk + kProjRows * d;    // [kProjRows][d_out]
    const int64_t t0 = (int64_t)blockIdx.x * kProjRows;
    const int rows = (int)(Tn - t0 < kProjRows ? Tn - t0 : kProjRows);
    for (int i = threadIdx.x; i < rows * d; i += blockDim.x) {
        const int r = i / d, j = i % d, h = j / D, e = j % D;
        const int64_t t = t0 + r;
        float acc = 0.0f;
        for (int g = 0; g < G; ++g) acc = __fadd_rn(acc, to_f32(q[(t * Hq + h * G + g) * D + e]));
        xq[r * d + j] = __fdiv_rn(acc, (float)G);
        xk[r * d + j] = to_f32(k[t * Hkv * D + j]);
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int nch = d >> 3;
    for (int j = warp; j < d_out; j += nw) {
        float w[CH][8];
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            const int ch = lane + 32 * c;
            if (ch < nch) load8<float>(Wt + (int64_t)j * d + ch * 8, w[c]);
        }
        for (int r = 0; r < rows; ++r) {
            float pq = 0.0f, pkk = 0.0f;
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                const int ch = lane + 32 * c;
                if (ch < nch) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        pq = __fmaf_rn(xq[r * d + ch * 8 + e], w[c][e], pq);
                        pkk = __fmaf_rn(xk[r * d + ch * 8 + e], w[c][e], pkk);
                    }
                }
            }
            pq = butterfly_sum(pq);
            pkk = butterfly_sum(pkk);
            if (lane == 0) {
                iq[(t0 + r) * d_out + j] = pq;
                pk[r * d_out + j] = pkk;
            }
        }
    }
    __syncthreads();
    if (warp < rows) {
        const float n = __fsqrt_rn(warp_cdot<float, float>(pk + warp * d_out, pk + warp * d_out, d_out, lane));
        if (lane == 0) den_s[warp] = fmaxf(n, 1e-12f);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < rows * d_out; i += blockDim.x) {
        const int r = i / d_out, j = i % d_out;
        ik[(t0 + r) * d_out + j] = __fdiv_rn(pk[r * d_out + j], den_s[r]);
    }
}

// out = x / max(|x|, 1e-12) per row (+ bf16 copy, round to nearest even), one warp per row.
__global__ void normalize_kernel(const float* __restrict__ x, int64_t n, int d, float* __restrict__ out,
                                 __nv_bfloat16* __restrict__ out_bf16) {
    int lane = threadIdx.x & 31;
    int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= n) return;
    const float* row = x + r * d;
    float nn = __fsqrt_rn(warp_cdot<float, float>(row, row, d, lane));
    float den = fmaxf(nn, 1e-12f);
    for (int j = lane; j < d; j += 32) {
        float u = __fdiv_rn(row[j], den);
        if (out) out[r * d + j] = u;
        if (out_bf16) out_bf16[r * d + j] = __float2bfloat16_rn(u);
    }
}

// ------------------------------------------------------------------ pools + Gram

__global__ void pools_kernel(const float* __restrict__ keys, int64_t blocks, int block, int pool, int d,
                             float* __restrict__ pools) {
    int64_t P = block / pool;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= blocks * P * d) return;
    int64_t j = i % d, pi = i / d;  // pool index over all blocks
    int64_t g = pi / P, p = pi % P;
    const float* src = keys + (g * block + p * pool) * d + j;
    float acc = 0.0f;
    for (int t = 0; t < pool; ++t) acc = __fadd_rn(acc, src[(int64_t)t * d]);
    pools[i] = acc;
}

// gram[g][i][j] = cdot(s_i, s_j) for the P rows of block g; one warp per (i <= j) pair.
__global__ void gram_kernel(const float* __restrict__ s, int P, int d, float* __restrict__ gram) {
    int lane = threadIdx.x & 31;
    int64_t pair = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int64_t npairs = (int64_t)P * (P + 1) / 2;
    if (pair >= npairs) return;
    int g = blockIdx.y;
    // pair -> (i, j), i <= j, row-major over the upper triangle
    int i = 0;
    int64_t rem = pair;
    while (rem >= P - i) {
        rem -= P - i;
        ++i;
    }
    int j = i + (int)rem;
    const float* base = s + (int64_t)g * P * d;
    float v = warp_cdot<float, float>(base + (int64_t)i * d, base + (int64_t)j * d, d, lane);
    if (lane == 0) {
        gram[((int64_t)g * P + i) * P + j] = v;
        gram[((int64_t)g * P + j) * P + i] = v;
    }
}

// ------------------------------------------------------------------ Ward merge

constexpr int kWardThreads = 512;
constexpr int kMaxP = 128;

__device__ __forceinline__ int64_t pack_cost(float cost, int index) {
    return (int64_t)(((uint64_t)(uint32_t)ordered_bits(cost) << 32) | (uint64_t)(uint32_t)index);
}

__device__ __forceinline__ int64_t warp_min_i64(int64_t v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        int64_t o = __shfl_xor_sync(0xFFFFFFFFu, v, off);
        v = o < v ? o : v;
    }
    return v;
}

// One CTA per block. gram [blocks, P, P] (read), sizes0 [blocks, P], labels [blocks, P].
__global__ void __launch_bounds__(kWardThreads) ward_merge_kernel(const float* __restrict__ gram,
                                                                  const int32_t* __restrict__ sizes0, int P,
                                                                  int target, int cap, int32_t* __restrict__ labels,
                                                                  int32_t* __restrict__ status) {
    extern __shared__ float wsm[];
    float* G = wsm;               // [P][P]
    float* G2 = wsm + P * P;      // [P][P]
    __shared__ float norm[kMaxP];
    __shared__ int alive[kMaxP], sz[kMaxP], root[kMaxP], nn[kMaxP], partner[kMaxP], dying[kMaxP], into[kMaxP];
    __shared__ int64_t nnkey[kMaxP], pkey[kMaxP];
    __shared__ int pa[kMaxP];
    __shared__ int fresh[kMaxP], olist[kMaxP];  // merged last round / this round's merging owners
    __shared__ int m_pairs, count, n_own, n_fresh;
    const int blk = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const float* src = gram + (int64_t)blk * P * P;
    for (int i = tid; i < P * P; i += blockDim.x) G[i] = src[i];
    for (int i = tid; i < P; i += blockDim.x) {
        alive[i] = 1;
        sz[i] = sizes0[(int64_t)blk * P + i];
        root[i] = i;
        fresh[i] = 0;
        nn[i] = -1;
    }
    if (tid == 0) {
        count = P;
        n_fresh = -1;  // the first round searches every cluster's partner
    }
    __syncthreads();
    // the Ward cost of clusters i and j (packed with j): the same arithmetic for every search
    auto key_of = [&](int i, int j, float gii) -> int64_t {
        const float merged = __fadd_rn(__fadd_rn(gii, G[j * P + j]), __fmul_rn(2.0f, G[i * P + j]));
        const float cost = __fsub_rn(__fadd_rn(norm[i], norm[j]), __fsqrt_rn(fmaxf(merged, 0.0f)));
        return pack_cost(cost, j);
    };
    while (count > target) {
        for (int i = tid; i < P; i += blockDim.x) {
            norm[i] = alive[i] ? __fsqrt_rn(G[i * P + i]) : 0.0f;
            partner[i] = -1;
            dying[i] = 0;
        }
        if (tid == 0) {
            m_pairs = 0;
            n_own = 0;
        }
        __syncthreads();
        // nearest feasible partner of every alive cluster (min packed cost|j). A cluster that
        // merged last round, or whose partner merged or was absorbed, searches all clusters;
        // for any other the kept key is still exact (its costs to unchanged clusters did not
        // change) and only last round's merged clusters can beat it.
        const int nf = n_fresh;
        for (int i = warp; i < P; i += nw) {
            if (!alive[i]) continue;  // (warp-uniform)
            const int ni = nn[i];
            const bool all = nf < 0 || fresh[i] || ni < 0 || !alive[ni] || fresh[ni];
            const float gii = G[i * P + i];
            int64_t best = INT64_MAX;
            if (all) {
                for (int j = lane; j < P; j += 32) {
                    if (j == i || !alive[j] || sz[i] + sz[j] > cap) continue;
                    const int64_t key = key_of(i, j, gii);
                    best = key < best ? key : best;
                }
            } else {
                if (lane == 0) best = nnkey[i];
                for (int x = lane; x < nf; x += 32) {
                    const int j = olist[x];
                    if (j == i || !alive[j] || sz[i] + sz[j] > cap) continue;
                    const int64_t key = key_of(i, j, gii);
                    best = key < best ? key : best;
                }
            }
            best = warp_min_i64(best);
            if (lane == 0) {
                nnkey[i] = best;
                nn[i] = best == INT64_MAX ? -1 : (int)(best & 0xFFFFFFFF);
            }
        }
        __syncthreads();
        // mutual pairs (lower index owns the pair)
        for (int i = tid; i < P; i += blockDim.x) {
            if (alive[i] && nn[i] > i && nn[nn[i]] == i) {
                int slot = atomicAdd(&m_pairs, 1);
                pa[slot] = i;
                pkey[slot] = (int64_t)(((uint64_t)nnkey[i] & 0xFFFFFFFF00000000ull) | (uint64_t)(uint32_t)i);
            }
        }
        __syncthreads();
        int m = m_pairs;
        if (m == 0) {
            if (tid == 0) atomicExch(status, LSA_ERR_SHORT);
            __syncthreads();
            break;
        }
        int allowed = count - target;
        for (int x = tid; x < m; x += blockDim.x) {
            int rank = 0;
            for (int y = 0; y < m; ++y) rank += pkey[y] < pkey[x];
            if (rank < allowed) {
                int a = pa[x], b = nn[a];
                partner[a] = b;
                dying[b] = 1;
                into[b] = a;
                olist[atomicAdd(&n_own, 1)] = a;
            }
        }
        __syncthreads();
        // batched Gram update, from the previous matrix: every pair (A <= C) of surviving
        // clusters with at least one merging owner, each visited once (two owners: from the
        // lower one), with A the lower index as the update's arithmetic is written
        const int no = n_own;
        for (int idx = tid; idx < no * P; idx += blockDim.x) {
            const int a1 = olist[idx / P], X = idx % P;
            if (!alive[X] || dying[X] || (partner[X] >= 0 && X < a1)) continue;
            const int A = a1 < X ? a1 : X, C = a1 < X ? X : a1;
            const int b = partner[A], dd = partner[C];
            float val;
            if (A == C) {
                val = __fadd_rn(__fadd_rn(G[A * P + A], G[A * P + b]), __fadd_rn(G[b * P + A], G[b * P + b]));
            } else if (b >= 0 && dd >= 0) {
                val = __fadd_rn(__fadd_rn(G[A * P + C], G[A * P + dd]), __fadd_rn(G[b * P + C], G[b * P + dd]));
            } else if (b >= 0) {
                val = __fadd_rn(G[A * P + C], G[b * P + C]);
            } else {
                val = __fadd_rn(G[A * P + C], G[A * P + dd]);
            }
            G2[A * P + C] = val;
        }
        __syncthreads();
        for (int idx = tid; idx < no * P; idx += blockDim.x) {
            const int a1 = olist[idx / P], X = idx % P;
            if (!alive[X] || dying[X] || (partner[X] >= 0 && X < a1)) continue;
            const int A = a1 < X ? a1 : X, C = a1 < X ? X : a1;
            const float val = G2[A * P + C];
            G[A * P + C] = val;
            G[C * P + A] = val;
        }
        __syncthreads();
        for (int i = tid; i < P; i += blockDim.x) {
            if (partner[i] >= 0) sz[i] += sz[partner[i]];
            int rt = root[i];
            if (dying[rt]) root[i] = into[rt];
        }
        __syncthreads();
        for (int i = tid; i < P; i += blockDim.x) {
            fresh[i] = partner[i] >= 0;
            if (dying[i]) alive[i] = 0;
        }
        if (tid == 0) {
            count -= no;  // each merge absorbs one cluster
            n_fresh = no;
        }
        __syncthreads();
    }
    // label survivors in increasing order of their lowest pool
    for (int i = tid; i < P; i += blockDim.x) {
        int rank = 0;
        for (int j = 0; j < i; ++j) rank += alive[j];
        nn[i] = alive[i] ? rank : -1;
    }
    __syncthreads();
    for (int p = tid; p < P; p += blockDim.x) labels[(int64_t)blk * P + p] = nn[root[p]];
}

// ------------------------------------------------------------------ members + sums

// One CTA per bucket row (block g, label b): members = positions of the block whose key
// label is b, ascending, -1 padded to cap; sums = fp32 sum of member keys in that order.
// key_labels == nullptr: positional labels (t % block) / bucket_size.
__global__ void __launch_bounds__(256) members_kernel(const float* __restrict__ keys, int d,
                                                      const int32_t* __restrict__ pool_labels, int pool, int block,
                                                      int bpb, int bucket_size, int cap, int32_t* __restrict__ members,
                                                      int32_t* __restrict__ sizes, float* __restrict__ sums,
                                                      int32_t* __restrict__ status) {
    extern __shared__ int msm[];  // [block] member list, then scan scratch
    int* list = msm;
    int* scan = msm + block;
    int64_t row = blockIdx.x;
    int64_t g = row / bpb;
    int b = (int)(row % bpb);
    int n_total = 0;
    // stable compaction over the block, blockDim-sized tiles
    for (int t0 = 0; t0 < block; t0 += blockDim.x) {
        int t = t0 + threadIdx.x;
        int lab = -1;
        if (t < block) lab = pool_labels ? pool_labels[g * (block / pool) + t / pool] : t / bucket_size;
        int hit = (t < block && lab == b) ? 1 : 0;
        int total;
        int at = block_exclusive_scan(hit, scan, &total);
        if (hit) list[n_total + at] = (int)(g * block + t);
        n_total += total;
        __syncthreads();
    }
    if (n_total > cap && threadIdx.x == 0) atomicExch(status, LSA_ERR_SHORT);
    int n = n_total < cap ? n_total : cap;
    for (int s = threadIdx.x; s < cap; s += blockDim.x) members[row * cap + s] = s < n ? list[s] : -1;
    if (threadIdx.x == 0) sizes[row] = n;
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        float acc = 0.0f;
        for (int s = 0; s < n; ++s) acc = __fadd_rn(acc, keys[(int64_t)list[s] * d + j]);
        sums[row * d + j] = acc;
    }
}

// ------------------------------------------------------------------ pairing helpers

// labels_out[g, i] = pair_labels[g, labels_in[g, i]] (compose halvings); labels_in == null: identity
__global__ void compose_labels_kernel(const int32_t* __restrict__ labels_in, const int32_t* __restrict__ pair_labels,
                                      int n, int cur, int64_t blocks, int32_t* __restrict__ labels_out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= blocks * n) return;
    int64_t g = i / n;
    int src = labels_in ? labels_in[i] : (int)(i % n);
    labels_out[i] = pair_labels[g * cur + src];
}

// pair sums: out[g, p, j] = run[g, lo, j] + run[g, hi, j] where lo < hi carry label p.
__global__ void pair_sums_kernel(const float* __restrict__ run, const int32_t* __restrict__ pair_labels, int cur,
                                 int d, int64_t blocks, float* __restrict__ out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int half = cur / 2;
    if (i >= blocks * half * d) return;
    int j = (int)(i % d);
    int64_t gp = i / d;
    int64_t g = gp / half;
    int p = (int)(gp % half);
    int lo = -1, hi = -1;
    for (int r = 0; r < cur; ++r)
        if (pair_labels[g * cur + r] == p) {
            if (lo < 0) lo = r;
            else hi = r;
        }
    float a = lo >= 0 ? run[(g * cur + lo) * d + j] : 0.0f;
    float c = hi >= 0 ? run[(g * cur + hi) * d + j] : 0.0f;
    out[i] = __fadd_rn(a, c);
}

// order[g*n + label*size + rank] = g*n + i: children in node order (stable by index).
__global__ void node_order_kernel(const int32_t* __restrict__ labels, int n, int size, int64_t blocks,
                                  int64_t* __restrict__ order) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= blocks * n) return;
    int64_t g = i / n;
    int me = (int)(i % n);
    int lab = labels[i];
    int rank = 0;
    for (int r = 0; r < me; ++r) rank += labels[g * n + r] == lab;
    if (rank < size) order[g * n + (int64_t)lab * size + rank] = i;
}

__global__ void fill_i32_kernel(int32_t* p, int64_t n, int32_t v) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

// ------------------------------------------------------------------ host

static int64_t r256(int64_t x) { return (x + 255) / 256 * 256; }

static unsigned nblk(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

static int ward_smem(int P) { return 2 * P * P * 4; }

static int launch_ward(const float* gram, const int32_t* sizes0, int64_t blocks, int P, int target, int cap,
                       int32_t* labels, int32_t* status, cudaStream_t st) {
    int smem = ward_smem(P);
    if (cudaFuncSetAttribute(ward_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return LSA_ERR_CUDA;
    ward_merge_kernel<<<(unsigned)blocks, kWardThreads, smem, st>>>(gram, sizes0, P, target, cap, labels, status);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

static int launch_gram(const float* s, int64_t blocks, int P, int d, float* gram, cudaStream_t st) {
    int64_t npairs = (int64_t)P * (P + 1) / 2;
    dim3 grid(nblk(npairs, 8), (unsigned)blocks);
    gram_kernel<<<grid, 256, 0, st>>>(s, P, d, gram);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

}  // namespace lsa

using namespace lsa;

extern "C" {

int lsa_regroup(const void* q, const void* k, int dtype, int64_t T, int64_t Hq, int64_t Hkv, int64_t D, float* iq,
                float* ik, cudaStream_t stream) {
    if (Hkv <= 0 || Hq % Hkv || (Hkv * D) % 8 || ((uintptr_t)k & 15) || (D % 8)) return LSA_ERR_ARG;
    if (T == 0) return LSA_OK;
    if (T <= 1024 && Hq / Hkv <= 8 && Hkv * D <= 2048) {  // few rows (decode): a CTA per row
        cudaLaunchAttribute pdl;
        pdl.id = cudaLaunchAttributeProgrammaticStreamSerialization;
        pdl.val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3((unsigned)T);
        lc.blockDim = dim3(kRegroupThreads);
        lc.stream = stream;
        lc.attrs = &pdl;
        lc.numAttrs = 1;
        cudaError_t e;
        if (dtype == kBF16)
            e = cudaLaunchKernelEx(&lc, regroup_row_kernel<__nv_bfloat16>, (const __nv_bfloat16*)q,
                                   (const __nv_bfloat16*)k, (int)Hq, (int)Hkv, (int)D, iq, ik);
        else if (dtype == kF16)
            e = cudaLaunchKernelEx(&lc, regroup_row_kernel<__half>, (const __half*)q, (const __half*)k, (int)Hq,
                                   (int)Hkv, (int)D, iq, ik);
        else if (dtype == kF32)
            e = cudaLaunchKernelEx(&lc, regroup_row_kernel<float>, (const float*)q, (const float*)k, (int)Hq, (int)Hkv,
                                   (int)D, iq, ik);
        else
            return LSA_ERR_ARG;
        return e == cudaSuccess ? LSA_OK : LSA_ERR_CUDA;
    }
    unsigned grid = nblk(T, 8);
    if (dtype == kBF16)
        regroup_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>((const __nv_bfloat16*)q, (const __nv_bfloat16*)k, T,
                                                               (int)Hq, (int)Hkv, (int)D, iq, ik);
    else if (dtype == kF16)
        regroup_kernel<__half><<<grid, 256, 0, stream>>>((const __half*)q, (const __half*)k, T, (int)Hq, (int)Hkv,
                                                        (int)D, iq, ik);
    else if (dtype == kF32)
        regroup_kernel<float><<<grid, 256, 0, stream>>>((const float*)q, (const float*)k, T, (int)Hq, (int)Hkv,
                                                       (int)D, iq, ik);
    else
        return LSA_ERR_ARG;
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

int lsa_regroup_project(const void* q, const void* k, int dtype, int64_t T, int64_t Hq, int64_t Hkv, int64_t D,
                        const float* Wt, int64_t d_out, float* iq, float* ik, cudaStream_t stream) {
    const int64_t d = Hkv * D;
    if (Hkv <= 0 || Hq % Hkv || D <= 0 || d % 8 || d > 2048 || d_out <= 0 || d_out % 8 || d_out > 2048 ||
        ((uintptr_t)Wt & 15) || T < 0)
        return LSA_ERR_ARG;
    if (T == 0) return LSA_OK;
    const int smem = (int)((2 * kProjRows * d + kProjRows * d_out) * sizeof(float));
    cudaLaunchAttribute pdl;
    pdl.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl.val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)((T + kProjRows - 1) / kProjRows));
    lc.blockDim = dim3(256);
    lc.dynamicSmemBytes = smem;
    lc.stream = stream;
    lc.attrs = &pdl;
    lc.numAttrs = 1;
    const int ch = (int)((d / 8 + 31) / 32);
    auto go = [&](auto kern, auto qp, auto kp) -> int {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return LSA_ERR_CUDA;
        return cudaLaunchKernelEx(&lc, kern, qp, kp, T, (int)Hq, (int)Hkv, (int)D, Wt, (int)d_out, iq, ik) ==
                       cudaSuccess
                   ? LSA_OK
                   : LSA_ERR_CUDA;
    };
#define LSA_RP(TT)                                                                                              \
    do {                                                                                                        \
        auto qp = (const TT*)q;                                                                                 \
        auto kp = (const TT*)k;                                                                                 \
        if (ch <= 1) return go(regroup_project_kernel<TT, 1>, qp, kp);                                          \
        if (ch <= 2) return go(regroup_project_kernel<TT, 2>, qp, kp);                                          \
        if (ch <= 4) return go(regroup_project_kernel<TT, 4>, qp, kp);                                          \
        return go(regroup_project_kernel<TT, 8>, qp, kp);                                                       \
    } while (0)
    if (dtype == kBF16) LSA_RP(__nv_bfloat16);
    if (dtype == kF16) LSA_RP(__half);
    if (dtype == kF32) LSA_RP(float);
#undef LSA_RP
    return LSA_ERR_ARG;
}

int lsa_normalize_rows(const float* x, int64_t n, int64_t d, float* out, void* out_bf16, cudaStream_t stream) {
    if (d % 8 || ((uintptr_t)x & 15)) return LSA_ERR_ARG;
    if (n == 0) return LSA_OK;
    normalize_kernel<<<nblk(n, 8), 256, 0, stream>>>(x, n, (int)d, out, (__nv_bfloat16*)out_bf16);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

int64_t lsa_build_buckets_workspace(int64_t T, int64_t d, int64_t block, int64_t pool) {
    if (block <= 0 || pool <= 0) return -1;
    int64_t blocks = T / block, P = block / pool;
    return r256(blocks * P * d * 4) + r256(blocks * P * P * 4) + r256(blocks * P * 4) * 2;
}

// build_buckets_gpu: index keys [T, d] fp32 -> centroids (fp32 + bf16), members, sizes, key
// sums for the T / block closed blocks. status (device int32) receives LSA_ERR_SHORT when a
// block cannot reach bpb buckets under cap.
int lsa_build_buckets(const float* keys, int64_t T, int64_t d, int64_t block, int64_t pool, int64_t bpb, int64_t cap,
                      float* centroids_f32, void* centroids_bf16, int32_t* members, int32_t* sizes, float* key_sums,
                      void* workspace, int64_t workspace_bytes, int32_t* status, cudaStream_t stream) {
    if (block <= 0 || pool <= 0 || block % pool || bpb <= 0 || cap <= 0 || d % 8 || d > 2048) return LSA_ERR_ARG;
    int64_t P = block / pool;
    if (P > kMaxP || P < 1) return LSA_ERR_ARG;
    if (workspace_bytes < lsa_build_buckets_workspace(T, d, block, pool)) return LSA_ERR_ARG;
    int64_t blocks = T / block;
    if (blocks == 0) return LSA_OK;
    char* w = (char*)workspace;
    float* pools = (float*)w;
    float* gram = (float*)(w + r256(blocks * P * d * 4));
    int32_t* sizes0 = (int32_t*)(w + r256(blocks * P * d * 4) + r256(blocks * P * P * 4));
    int32_t* plabels = sizes0 + r256(blocks * P * 4) / 4;
    int rc;
    pools_kernel<<<nblk(blocks * P * d, 256), 256, 0, stream>>>(keys, blocks, (int)block, (int)pool, (int)d, pools);
    LSA_LAUNCH_CHECK();
    if ((rc = launch_gram(pools, blocks, (int)P, (int)d, gram, stream))) return rc;
    fill_i32_kernel<<<nblk(blocks * P, 256), 256, 0, stream>>>(sizes0, blocks * P, (int32_t)pool);
    LSA_LAUNCH_CHECK();
    if ((rc = launch_ward(gram, sizes0, blocks, (int)P, (int)bpb, (int)cap, plabels, status, stream))) return rc;
    int msmem = (int)(block + 64) * 4;
    members_kernel<<<(unsigned)(blocks * bpb), 256, msmem, stream>>>(keys, (int)d, plabels, (int)pool, (int)block,
                                                                   (int)bpb, 1, (int)cap, members, sizes, key_sums,
                                                                   status);
    LSA_LAUNCH_CHECK();
    return lsa_normalize_rows(key_sums, blocks * bpb, d, centroids_f32, centroids_bf16, stream);
}

int lsa_position_buckets(const float* keys, int64_t T, int64_t d, int64_t block, int64_t bucket_size, int64_t cap,
                         float* centroids_f32, void* centroids_bf16, int32_t* members, int32_t* sizes, float* key_sums,
                         int32_t* status, cudaStream_t stream) {
    if (block <= 0 || bucket_size <= 0 || block % bucket_size || cap < bucket_size || d % 8) return LSA_ERR_ARG;
    int64_t blocks = T / block, bpb = block / bucket_size;
    if (blocks == 0) return LSA_OK;
    int msmem = (int)(block + 64) * 4;
    members_kernel<<<(unsigned)(blocks * bpb), 256, msmem, stream>>>(keys, (int)d, nullptr, 1, (int)block, (int)bpb,
                                                                   (int)bucket_size, (int)cap, members, sizes,
                                                                   key_sums, status);
    LSA_LAUNCH_CHECK();
    return lsa_normalize_rows(key_sums, blocks * bpb, d, centroids_f32, centroids_bf16, stream);
}

int64_t lsa_pair_to_size_workspace(int64_t blocks, int64_t n, int64_t d) {
    return r256(blocks * n * d * 4) * 2 + r256(blocks * n * n * 4) + r256(blocks * n * 4) * 3;
}

// _pair_to_size over [blocks, n, d] sums: log2(size) halvings. labels [blocks, n] (node of
// each row), order [blocks * n] int64 (rows in node order, absolute), node_sums
// [blocks, n / size, d].
int lsa_pair_to_size(const float* sums, int64_t blocks, int64_t n, int64_t d, int64_t size, int32_t* labels,
                     int64_t* order, float* node_sums, void* workspace, int64_t workspace_bytes, int32_t* status,
                     cudaStream_t stream) {
    if (n <= 0 || n > kMaxP || size <= 0 || (size & (size - 1)) || n % size || d % 8) return LSA_ERR_ARG;
    if (workspace_bytes < lsa_pair_to_size_workspace(blocks, n, d)) return LSA_ERR_ARG;
    if (blocks == 0) return LSA_OK;
    char* w = (char*)workspace;
    float* runA = (float*)w;
    float* runB = (float*)(w + r256(blocks * n * d * 4));
    float* gram = (float*)(w + 2 * r256(blocks * n * d * 4));
    int32_t* ones = (int32_t*)(w + 2 * r256(blocks * n * d * 4) + r256(blocks * n * n * 4));
    int32_t* plab = ones + r256(blocks * n * 4) / 4;
    int32_t* comp = plab + r256(blocks * n * 4) / 4;
    int rc;
    if (cudaMemcpyAsync(runA, sums, blocks * n * d * 4, cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
        return LSA_ERR_CUDA;
    fill_i32_kernel<<<nblk(blocks * n, 256), 256, 0, stream>>>(ones, blocks * n, 1);
    LSA_LAUNCH_CHECK();
    int cur = (int)n;
    bool first = true;
    float* run = runA;
    float* nxt = runB;
    for (int64_t s = size; s > 1; s >>= 1) {
        if ((rc = launch_gram(run, blocks, cur, (int)d, gram, stream))) return rc;
        if ((rc = launch_ward(gram, ones, blocks, cur, cur / 2, 2, plab, status, stream))) return rc;
        compose_labels_kernel<<<nblk(blocks * n, 256), 256, 0, stream>>>(first ? nullptr : labels, plab, (int)n, cur,
                                                                          blocks, comp);
        LSA_LAUNCH_CHECK();
        if (cudaMemcpyAsync(labels, comp, blocks * n * 4, cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
            return LSA_ERR_CUDA;
        pair_sums_kernel<<<nblk(blocks * (cur / 2) * d, 256), 256, 0, stream>>>(run, plab, cur, (int)d, blocks, nxt);
        LSA_LAUNCH_CHECK();
        float* t = run;
        run = nxt;
        nxt = t;
        cur /= 2;
        first = false;
    }
    if (first) {  // size == 1: every row is its own node
        compose_labels_kernel<<<nblk(blocks * n, 256), 256, 0, stream>>>(nullptr, ones, (int)n, (int)n, blocks, comp);
        LSA_LAUNCH_CHECK();
    }
    if (cudaMemcpyAsync(node_sums, run, blocks * cur * d * 4, cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
        return LSA_ERR_CUDA;
    node_order_kernel<<<nblk(blocks * n, 256), 256, 0, stream>>>(labels, (int)n, (int)size, blocks, order);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

}  // extern "C"
