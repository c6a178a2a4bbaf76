/*
 * lsa_b200.h - C ABI of the B200 (sm_100a) Latent Sparse Attention select + read kernels.
 *
 * Library: latent-sparse-attention-rocm_b200/lsa_b200/liblsa_b200.so (built by
 * latent-sparse-attention-rocm_b200/build.py). Every entry point takes plain device
 * pointers, sizes and a cudaStream_t, launches asynchronously on that stream and
 * returns a status: LSA_OK, or LSA_ERR_ARG for rejected arguments, LSA_ERR_CUDA for a
 * failed launch. Kernels that wait on the device bound every wait and record
 * LSA_ERR_TIMEOUT in a device status word instead of hanging; the bucket builds record
 * LSA_ERR_SHORT there when a block cannot reach its bucket count under the cap.
 *
 * Dtype codes: 0 = fp32, 1 = fp16, 2 = bf16; the selects' query code also takes 3 = fp32
 * storage read as its bf16 rounding (lsa_select_fused, lsa_select_batched: the bf16 scoring
 * of an fp32 index query with no separate cast). "Counters" arguments are int32 device
 * arrays that must be zero before the call; the kernels leave them zero, so one
 * buffer serves every later call on the same stream (and CUDA-graph replays).
 * Calls sharing a scratch or counters buffer must not overlap on the GPU.
 *
 * Each declaration names the reference interface it replaces: AIwork4me/
 * latent-sparse-attention-rocm, file:line inside that project.
 */
#ifndef LSA_B200_H
#define LSA_B200_H

#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LSA_OK 0
#define LSA_ERR_ARG (-1)
#define LSA_ERR_CUDA (-2)
#define LSA_ERR_TIMEOUT (-3)
#define LSA_ERR_SHORT (-4)
#define LSA_ERR_SIZE (-5)

/* ---------------------------------------------------------------- peer-memory exchange */

/* The sharded decode steps' all-gathers over peer memory (no reference counterpart: the
 * reference is single-GPU; these replace torch.distributed.all_gather_into_tensor / NCCL for
 * the small per-step exchanges). Each rank allocates an arena and shares its CUDA IPC handle
 * (64 bytes); every rank opens every peer's handle. */
int lsa_peer_arena_alloc(int64_t bytes, void** ptr, void* handle);
int lsa_peer_arena_open(const void* handle, void** ptr);
int lsa_peer_arena_close(void* ptr);
int lsa_peer_arena_free(void* ptr);
/* out [world][bytes] = every rank's src [bytes] (bytes a multiple of 16). bases[world]: every
 * rank's arena as mapped in this process (bases[rank] = own); the channel's world uint32 flags
 * at flag_off and its two receive buffers of world x bytes at recv_off in every arena; ctrl: 4
 * device uint32 of this rank for the channel (zero at rest but the epoch). Two launches: the
 * push stores into every rank's arena and publishes the epoch flag; the pull waits (bounded,
 * 1 s; LSA_ERR_TIMEOUT in *status) for every rank's flag and copies the receive buffer out.
 * Every rank makes the same sequence of calls per channel. CUDA-graph safe. */
int lsa_peer_all_gather(const void* src, void* out, int64_t bytes, int rank, int world, void* const* bases,
                        int64_t flag_off, int64_t recv_off, uint32_t* ctrl, int32_t* status, cudaStream_t stream);

/* ---------------------------------------------------------------- index space */

/* make_index_space -> upstream regroup (src/lsa_rocm_lab/port/gates.py:50-59).
 * q [T, Hq, D], k [T, Hkv, D] (dtype) -> index queries / unit index keys [T, Hkv*D] fp32.
 * k = NULL: index queries only (ik unused). */
int lsa_regroup(const void* q, const void* k, int dtype, int64_t T, int64_t Hq, int64_t Hkv, int64_t D, float* iq,
                float* ik, cudaStream_t stream);

/* regroup through a D-LSA projection map (the reference's "model-specific distilled
 * projections", docs/ROADMAP.md:41-43, whose upstream map format is absent; this build's
 * definition): Wt [d_out, Hkv*D] fp32 (16-byte aligned, one row per output dimension);
 * index query = canonical dots of the group-mean query with Wt's rows, index key = the
 * concatenated key row's canonical dots with Wt's rows, normalised by their canonical norm.
 * d and d_out multiples of 8, at most 2048. -> iq / ik [T, d_out] fp32. */
int lsa_regroup_project(const void* q, const void* k, int dtype, int64_t T, int64_t Hq, int64_t Hkv, int64_t D,
                        const float* Wt, int64_t d_out, float* iq, float* ik, cudaStream_t stream);

/* F.normalize of each row (pipeline.py:113, :179), optional bf16 copy (round to nearest even). */
int lsa_normalize_rows(const float* x, int64_t n, int64_t d, float* out, void* out_bf16, cudaStream_t stream);

/* ---------------------------------------------------------------- bucket build */

int64_t lsa_build_buckets_workspace(int64_t T, int64_t d, int64_t block, int64_t pool);

/* build_buckets_gpu (src/lsa_rocm_lab/port/pipeline.py:71-116): pools, spherical Ward merge
 * (upstream triton_ward.ward_merge, :97), members (bucket_members_from_labels, :101) and
 * centroids (:108-114) of the T / block closed blocks. keys [T, d] fp32; outputs
 * centroids_f32 / centroids_bf16 [rows, d], members [rows, cap] int32 (-1 padded),
 * sizes [rows], key_sums [rows, d] fp32; rows = (T / block) * bpb. status: device int32. */
int lsa_build_buckets(const float* keys, int64_t T, int64_t d, int64_t block, int64_t pool, int64_t bpb, int64_t cap,
                      float* centroids_f32, void* centroids_bf16, int32_t* members, int32_t* sizes, float* key_sums,
                      void* workspace, int64_t workspace_bytes, int32_t* status, cudaStream_t stream);

/* position_buckets (pipeline.py:378-403): runs of bucket_size consecutive keys. */
int lsa_position_buckets(const float* keys, int64_t T, int64_t d, int64_t block, int64_t bucket_size, int64_t cap,
                         float* centroids_f32, void* centroids_bf16, int32_t* members, int32_t* sizes,
                         float* key_sums, int32_t* status, cudaStream_t stream);

int64_t lsa_pair_to_size_workspace(int64_t blocks, int64_t n, int64_t d);

/* _pair_to_size (pipeline.py:136-150; upstream cluster_node_buckets iterated): log2(size)
 * halvings of each block of n rows. labels [blocks, n], order [blocks * n] int64 (rows in
 * node order, the children table of build_hierarchy_gpu, :173-179), node_sums. */
int lsa_pair_to_size(const float* sums, int64_t blocks, int64_t n, int64_t d, int64_t size, int32_t* labels,
                     int64_t* order, float* node_sums, void* workspace, int64_t workspace_bytes, int32_t* status,
                     cudaStream_t stream);

/* ---------------------------------------------------------------- select */

/* _production_scores (pipeline.py:217-232): scores [R, N] fp32 = canonical fp32 dot of each
 * query row with each centroid. (q, c) dtypes: (bf16, bf16), (fp32, fp32), (fp32, bf16). */
int lsa_bucket_scores(const void* queries, int q_dtype, int64_t R, int64_t ldq, const void* centroids, int c_dtype,
                      int64_t N, int64_t d, float* scores, int64_t lds, cudaStream_t stream);

/* visible_counts (pipeline.py:184-186): min(rows, pos / block * bpb). */
int lsa_visible_counts(const int32_t* positions, int64_t R, int64_t block, int64_t bpb, int64_t rows, int32_t* counts,
                       cudaStream_t stream);

/* The listing, whole path (upstream TopK.listed, pipeline.py:266-267): every column packed
 * (ordered_bits(score) << 32 | 0x7FFFFFFF - col), EMPTY (INT64_MIN) at or past lengths[r]. */
int lsa_pack_keys(const float* scores, int64_t R, int64_t N, int64_t lds, const int32_t* lengths, int64_t* keys,
                  int64_t ldk, cudaStream_t stream);

/* best_first_keys (pipeline.py:189-214): slots >= counts[r] masked EMPTY (counts may be
 * NULL), the k greatest keys sorted descending into out [R, ldo]. */
int lsa_best_first_keys(const int64_t* keys, int64_t R, int64_t N, int64_t ldk, int64_t k, const int32_t* counts,
                        int64_t* out, int64_t ldo, cudaStream_t stream);

/* upstream keys.unpack_ids (pipeline.py:268): key -> bucket id, EMPTY -> -1. */
int lsa_unpack_ids(const int64_t* keys, int64_t n, int32_t* ids, cudaStream_t stream);

/* select_fused.select_topk_scores (src/lsa_rocm_lab/port/select_fused.py:83-137): scores ->
 * the min(top_p, N) greatest packed keys of the live columns, sorted, EMPTY tail to ldo. */
int lsa_select_topk_scores(const float* scores, int64_t R, int64_t N, int64_t lds, const int32_t* lengths,
                           int64_t top_p, int64_t* out, int64_t ldo, cudaStream_t stream);

/* upstream expansion.expand_in_order (pipeline.py:269-271): picked bucket ids [R, P] (-1 =
 * none) -> read lists [R, top_k + window + sink] (-1 padded) and lengths [R]. */
int lsa_expand_in_order(const int32_t* picked, int64_t R, int64_t P, int64_t ldp, const int32_t* members,
                        int64_t member_rows, int64_t cap, const int32_t* positions, int64_t window, int64_t sink,
                        int64_t top_k, int32_t* lists, int32_t* lengths, cudaStream_t stream);

/* select_fused.expand_in_order_from_keys (select_fused.py:217-280): the walk reading packed keys. */
int lsa_expand_from_keys(const int64_t* keys, int64_t R, int64_t P, int64_t ldk, const int32_t* members,
                         int64_t member_rows, int64_t cap, const int32_t* positions, int64_t window, int64_t sink,
                         int64_t top_k, int32_t* lists, int32_t* lengths, cudaStream_t stream);

int64_t lsa_select_fused_scratch(int64_t R, int64_t N);

/* flat_select with LSA_SELECT_IMPL=fused (pipeline.py:274-316): ONE launch from index queries
 * to read lists - scoring over many CTAs, the last CTA of a row sorts and expands.
 * counters: R int32 tickets (zero at rest), and with R + 1 the status word counters[R]:
 * rows wider than one cluster with bf16 centroids, top_p <= 128 and cap % 4 == 0 then take
 * the persistent streaming kernel (TMA bulk copies of the centroid rows), whose bounded
 * waits record LSA_ERR_TIMEOUT there. max_position < 0: size the grid for every column. */
int lsa_select_fused(const void* queries, int q_dtype, int64_t R, int64_t ldq, const void* centroids, int c_dtype,
                     int64_t N, int64_t d, const int32_t* positions, int64_t block, int64_t bpb, const int32_t* members,
                     int64_t cap, int64_t top_p, int64_t window, int64_t sink, int64_t top_k, int32_t* lists,
                     int32_t* lengths, void* scratch, int64_t scratch_bytes, int32_t* counters, int64_t n_counters,
                     int64_t max_position, cudaStream_t stream);

/* make_index_space + flat_select (fused) for decode rows in one launch (gates.py:50-59 then
 * pipeline.py:274-316): q [R, Hq, D] raw queries (q_dtype fp32 / fp16 / bf16); the index
 * query of a row is built in the kernel with lsa_regroup's arithmetic (the group mean of
 * each KV head's query heads, read as its bf16 rounding for bf16 centroids), so the lists
 * equal lsa_regroup followed by lsa_select_fused byte for byte. Rows the one-cluster decode
 * select takes (R < 256, top_p <= 32, cap <= 128, N <= 1024 columns, Hkv*D <= 2048 in
 * chunks that fit its registers) only: anything else returns LSA_ERR_ARG and the caller
 * regroups and calls lsa_select_fused. No scratch, no counters. */
int lsa_select_fused_grouped(const void* q, int q_dtype, int64_t R, int64_t Hq, int64_t Hkv, int64_t D,
                             const void* centroids, int c_dtype, int64_t N, const int32_t* positions, int64_t block,
                             int64_t bpb, const int32_t* members, int64_t cap, int64_t top_p, int64_t window,
                             int64_t sink, int64_t top_k, int32_t* lists, int32_t* lengths, cudaStream_t stream);

/* cfg 2's positional block-sparse arm (pipeline.py:378-403 builds its buckets; the static
 * pattern is this build's definition): per row, of the v visible buckets the first `first`,
 * the last `last` and top_p - first - last strided in between (first + floor(i * (v - first
 * - last) / (top_p - first - last))), ascending, unique, -1 padded; every visible bucket
 * when v <= top_p. picks [R, top_p] int32, then lsa_expand_in_order. */
int lsa_positional_picks(const int32_t* positions, int64_t R, int64_t block, int64_t bpb, int64_t rows, int64_t top_p,
                         int64_t first, int64_t last, int32_t* picks, cudaStream_t stream);

/* Batched decode (one query row per sequence, sequences of different lengths): the fused
 * selection of flat_select (pipeline.py:274-316) for every row in one launch, row r reading
 * its own sequence's buckets = rows [table_off[r], table_off[r] + table_rows[r]) of the
 * concatenated centroid [sum rows, d] and member [sum rows, cap] tables (member ids are
 * positions within the row's sequence). max_rows = the largest table_rows[r] (the scratch
 * key stride). Each row's result equals flat_select on its own sequence's buckets. The
 * reference has no batched select (its gates build per sequence, gates.py:59). Counters
 * as lsa_select_fused (R tickets, + 1 status word to allow the streaming kernel). */
int64_t lsa_select_batched_scratch(int64_t R, int64_t max_rows);
int lsa_select_batched(const void* queries, int q_dtype, int64_t R, int64_t ldq, const void* centroids, int c_dtype,
                       int64_t d, const int64_t* table_off, const int32_t* table_rows, int64_t max_rows,
                       const int32_t* positions, int64_t block, int64_t bpb, const int32_t* members, int64_t cap,
                       int64_t top_p, int64_t window, int64_t sink, int64_t top_k, int32_t* lists, int32_t* lengths,
                       void* scratch, int64_t scratch_bytes, int32_t* counters, int64_t n_counters,
                       int64_t max_position, cudaStream_t stream);

/* ---------------------------------------------------------------- fused decode */

/* flat_select (LSA_SELECT_IMPL=fused scoring with bf16 queries and centroids,
 * pipeline.py:274-316) followed by lsa_read (read_kernel_tiled.py:41-89) for R <= 4 query
 * rows of ONE sequence, in one cooperative launch (one CTA per SM): grid-wide scoring, one
 * bounded grid barrier, per-CTA top-32 and expansion into shared memory, split reads with a
 * ticket merge. top_p <= 32, D = 128, Hq / Hkv in {4, 8}, dtype bf16 or fp16; q [R, Hq, D],
 * k/v [Tk, Hkv, D]. lists [R, top_k + window + sink] / lengths [R] receive the read lists
 * when non-null (bit-equal to flat_select). Scratch and counters (zero at rest; the kernel
 * leaves them zero) from lsa_decode_fused_plan. No reference counterpart: the reference runs
 * select and read as separate launches (its ROADMAP item 3 names this fusion). */
int lsa_decode_fused_plan(int64_t R, int64_t Hq, int64_t Hkv, int64_t N, int64_t cap, int64_t width,
                          int64_t* scratch_bytes, int64_t* n_counters);
int lsa_decode_fused(const void* index_queries, int64_t R, int64_t ldq, const void* centroids, int64_t N, int64_t d,
                     const int32_t* members, int64_t cap, const int32_t* positions, int64_t block, int64_t bpb,
                     int64_t top_p, int64_t window, int64_t sink, int64_t top_k, const void* q, const void* k,
                     const void* v, int dtype, int64_t Tk, int64_t Hq, int64_t Hkv, int64_t D, float scale, void* out,
                     int32_t* lists, int32_t* lengths, void* scratch, int64_t scratch_bytes, int32_t* counters,
                     int64_t n_counters, cudaStream_t stream);

/* ---------------------------------------------------------------- prefill (tile rows) */

/* Per-64-query-tile selection of the prefill arm. The reference selects per row only
 * (pipeline.py:248-316); a tile row scores the fp32 sum of its rows' bf16 index queries,
 * which ranks buckets like the tile mean.
 * lsa_tile_queries: tq [tiles, d] fp32 = sum over the tile's rows, in row order, of
 * bf16(index query) (q_dtype fp32 or bf16). */
int lsa_tile_queries(const void* index_queries, int q_dtype, int64_t T, int64_t ldq, int64_t d, int64_t tile,
                     float* out, cudaStream_t stream);

int64_t lsa_tile_select_scratch(int64_t T, int64_t tile, int64_t d, int64_t N);

/* flat_select's composition (scores -> packed keys -> best-first top_p -> expansion,
 * pipeline.py:248-271) over tile rows: visible = the blocks closed before the tile's first
 * row (visible_counts, pipeline.py:184-186, at the tile start); the walk keeps the first
 * top_k members of the picks below the tile's block start, then the sinks
 * [0, min(sink, block_start)) (window 0). lists [tiles, top_k + sink] int32 (-1 padded),
 * lengths [tiles]. Counters: tiles int32, zero at rest. block % tile == 0. */
int lsa_tile_select(const void* index_queries, int q_dtype, int64_t T, int64_t ldq, int64_t tile,
                    const void* centroids, int c_dtype, int64_t N, int64_t d, int64_t block, int64_t bpb,
                    const int32_t* members, int64_t cap, int64_t top_p, int64_t sink, int64_t top_k, int32_t* lists,
                    int32_t* lengths, void* scratch, int64_t scratch_bytes, int32_t* counters, int64_t n_counters,
                    cudaStream_t stream);

/* The prefill read (read numerics: src/lsa_rocm_lab/port/read_kernel_tiled.py:41-89): row t
 * of q [B, T, Hq, 128] attends over its tile's list (tile_lists [B, tiles, ldl], lengths
 * [B, tiles]; ids outside [0, Tk) skipped) and then, causally, its open block
 * [t / block * block, t] of k/v [B, Tk, Hkv, 128]. dtype bf16 or fp16; Hq / Hkv in
 * {4, 8, 16}; tile a multiple of 256 / (Hq / Hkv); block a multiple of tile. out like q.
 * status: device int32, LSA_ERR_TIMEOUT written there if a bounded device wait expired. */
int lsa_sparse_prefill(const void* q, const void* k, const void* v, int dtype, const int32_t* tile_lists,
                       const int32_t* tile_lengths, int64_t ldl, int64_t B, int64_t T, int64_t Tk, int64_t Hq,
                       int64_t Hkv, int64_t D, int64_t tile, int64_t block, float scale, void* out, int32_t* status,
                       cudaStream_t stream);

/* ---------------------------------------------------------------- tree */

int lsa_tree_plan(int64_t R, int64_t n_built, const int64_t* level_counts, int64_t beam, int64_t size, int64_t nb,
                  int64_t bpb, int64_t top_p, int64_t* scratch_bytes, int64_t* n_counters);

/* tree_select (pipeline.py:319-337; src/lsa_rocm_lab/port/_tree.py:318-373 beam,
 * :100-142 growth): picks [R, top_p] int32 (-1 padded). level_centroids, level_children
 * and level_counts are HOST arrays of n_built device pointers / node counts. */
int lsa_tree_select(const float* q, int64_t R, int64_t d, const int32_t* positions, int64_t block, int64_t bpb,
                    int64_t rows, int64_t n_built, const float* const* level_centroids,
                    const int64_t* const* level_children, const int64_t* level_counts, const float* bucket_centroids,
                    int64_t size, int64_t nb, int64_t top_level, int64_t beam, int64_t top_p, int32_t* picks,
                    void* scratch, int64_t scratch_bytes, int32_t* counters, int64_t n_counters, cudaStream_t stream);

/* lsa_tree_select plus the picks' packed keys [R, top_p] (score bits unchanged, bucket column
 * + col_offset, EMPTY past the picks): a sequence shard's candidates in global bucket ids,
 * ready for the cross-shard best-first merge (lsa_best_first_keys). No reference counterpart:
 * the reference decodes one sequence on one device. */
int lsa_tree_select_keys(const float* q, int64_t R, int64_t d, const int32_t* positions, int64_t block, int64_t bpb,
                         int64_t rows, int64_t n_built, const float* const* level_centroids,
                         const int64_t* const* level_children, const int64_t* level_counts,
                         const float* bucket_centroids, int64_t size, int64_t nb, int64_t top_level, int64_t beam,
                         int64_t top_p, int32_t* picks, int64_t* pick_keys, int64_t col_offset, void* scratch,
                         int64_t scratch_bytes, int32_t* counters, int64_t n_counters, cudaStream_t stream);

/* tree_select with its expansion (src/lsa_rocm_lab/port/_tree.py:34-60: the beam's picks, then
 * expand_in_order into read lists): lsa_tree_select's picks plus lists [R, top_k + window +
 * sink] int32 (-1 padded) and lengths [R] int32, equal to lsa_expand_in_order(picks, R, top_p,
 * top_p, members, ...). members [member_rows, cap] int32. One launch when the beam's cluster
 * form takes the call (<= 64 rows) and top_p * cap + top_k slots fit 128 KB of shared memory,
 * else the beam and the expansion kernel. Scratch / counters as lsa_tree_plan reports. The
 * launch reads positions (and the read-only index) before it waits for the previous kernel
 * in the stream: a kernel that writes them must not let its dependents start early. */
int lsa_tree_select_lists(const float* q, int64_t R, int64_t d, const int32_t* positions, int64_t block, int64_t bpb,
                          int64_t rows, int64_t n_built, const float* const* level_centroids,
                          const int64_t* const* level_children, const int64_t* level_counts,
                          const float* bucket_centroids, int64_t size, int64_t nb, int64_t top_level, int64_t beam,
                          int64_t top_p, const int32_t* members, int64_t member_rows, int64_t cap, int64_t window,
                          int64_t sink, int64_t top_k, int32_t* picks, int32_t* lists, int32_t* lengths,
                          void* scratch, int64_t scratch_bytes, int32_t* counters, int64_t n_counters,
                          cudaStream_t stream);

/* ---------------------------------------------------------------- read */

/* Split plan of lsa_sparse_read: splits per (row, KV head), scratch bytes, counters (the
 * last counter is the status word). splits_req <= 0 chooses from the SM count. */
int lsa_sparse_read_plan(int64_t B, int64_t Tq, int64_t Hq, int64_t Hkv, int64_t D, int64_t width, int64_t splits_req,
                         int64_t* splits, int64_t* scratch_bytes, int64_t* n_counters);

/* sparse_read / sparse_read_tiled / sparse_read_auto (src/lsa_rocm_lab/port/read_kernel.py:80-120,
 * read_kernel_tiled.py:92-156): q [B, Tq, Hq, D], k/v [B, Tk, Hkv, D] (dtype, D in {64, 128},
 * Hq / Hkv <= 8), ids [B*Tq, width] int32, lengths [B*Tq] int32 -> out like q. */
int lsa_sparse_read(const void* q, const void* k, const void* v, int dtype, const int32_t* ids,
                    const int32_t* lengths, int64_t B, int64_t Tq, int64_t Tk, int64_t Hq, int64_t Hkv, int64_t D,
                    int64_t width, float scale, void* out, void* scratch, int64_t scratch_bytes, int32_t* counters,
                    int64_t n_counters, int64_t splits, cudaStream_t stream);

/* No counterpart in the reference: lsa_sparse_read for callers that cannot allocate
 * device memory (a server whose device memory is one arena owned by its own allocator,
 * a plugin host that forbids cudaMalloc once serving). The split partials and counters
 * live in fixed __device__ arrays of this library: at most 8 MiB of scratch and 65536
 * counters per call. The entry point plans without the persistent grid (so the figures of
 * lsa_sparse_read_plan do not apply to it), checks that plan against both limits itself
 * and returns LSA_ERR_SIZE, launching nothing, for a call beyond them. It calls no
 * allocator. The first call on each device resolves the arrays' addresses, so make it
 * before any stream capture; each call zeroes the counters it uses; calls share the
 * arrays, so calls that overlap on the GPU race. status (may be null): 4 bytes the device
 * can write (device memory, or mapped pinned host memory); once the call's work on
 * `stream` has completed it holds 0, or LSA_ERR_TIMEOUT when a bounded wait of the read
 * expired (the output is then incomplete). */
int lsa_sparse_read_noalloc(const void* q, const void* k, const void* v, int dtype, const int32_t* ids,
                            const int32_t* lengths, int64_t B, int64_t Tq, int64_t Tk, int64_t Hq, int64_t Hkv,
                            int64_t D, int64_t width, float scale, void* out, int64_t splits, int32_t* status,
                            cudaStream_t stream);

/* Sequence-shard partial read (no reference counterpart; the read numerics are
 * read_kernel_tiled.py:41-89 restricted to this shard's keys): ids are global positions and
 * k/v hold positions [id_base, id_base + Tk); ids outside are skipped. out32 [B*Tq, Hq, D]
 * fp32 normalised output over this shard's keys, lse [B*Tq, Hq] their log2-sum-exp of the
 * scaled scores (-inf when the shard holds none of the row's keys). Scratch / counters as
 * lsa_sparse_read. */
int lsa_sparse_read_partial(const void* q, const void* k, const void* v, int dtype, const int32_t* ids,
                            const int32_t* lengths, int64_t B, int64_t Tq, int64_t Tk, int64_t Hq, int64_t Hkv,
                            int64_t D, int64_t width, float scale, int64_t id_base, float* out32, float* lse,
                            void* scratch, int64_t scratch_bytes, int32_t* counters, int64_t n_counters,
                            int64_t splits, cudaStream_t stream);

/* The log-sum-exp merge of P shard partials: o [P, n, D] fp32, lse [P, n] -> out [n, D] in
 * dtype, equal to one read over the union of the shards' (disjoint) key sets. */
int lsa_merge_partials(const float* o, const float* lse, int64_t P, int64_t n, int64_t D, int dtype, void* out,
                       cudaStream_t stream);

/* ---------------------------------------------------------------- paged KV cache */

/* The expansion walk's MAP_SLOTS path (select_fused.py:147-148, 177-199) as a pass over
 * finished read lists: out[r, j] = slot_table[slot_rows[r], lists[r, j]] for j < lengths[r]
 * (walked members, window and sinks alike), -1 past the length or for positions outside
 * [0, table_cols) or a slot row outside [0, table_rows). slot_table [table_rows, ld_table]
 * int32 maps each sequence's positions to physical slots of a KV pool; reading the mapped
 * lists over the pool (k/v [1, slots, Hkv, D], one list row per query row) equals reading
 * the position lists over each sequence's own cache. R <= 65535. */
int lsa_map_slots(const int32_t* lists, const int32_t* lengths, int64_t R, int64_t width, const int32_t* slot_table,
                  int64_t table_rows, int64_t table_cols, int64_t ld_table, const int32_t* slot_rows, int32_t* out,
                  cudaStream_t stream);

/* ---------------------------------------------------------------- self-test */

/* The bounded wait every kernel uses (no reference counterpart): a one-thread kernel waits on
 * an mbarrier of its own with the same helper. arrive != 0: the phase completes, *status = 0;
 * arrive == 0: nothing arrives, the wait gives up after limit_ns (<= 2 s) and *status =
 * LSA_ERR_TIMEOUT. Tests the failure path without a fault or a hang. */
int lsa_wait_selftest(int32_t* status, int64_t limit_ns, int arrive, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LSA_B200_H */
