// read.cu - gather attention over each row's read list (sm_100a).
//
// Reference semantics (AIwork4me/latent-sparse-attention-rocm,
// src/lsa_rocm_lab/port/read_kernel_tiled.py:41-89): for row r and query head h (KV head
// h / (Hq / Hkv)), the ids >= 0 among the first min(length, width) slots are read;
// s = (q . k) * scale in fp32; fp32 online softmax from a finite -3e38 running max;
// o = sum p v / l; a row with no listed key gives zeros; duplicates count per occurrence;
// the output takes q's dtype. Ids outside [0, Tk) are skipped, never dereferenced.
//
// B200 design: split-K flash decoding. One CTA (8 warps) per (row, KV head, split) serves
// all G query heads of the KV head, so each gathered K/V row crosses HBM once per group.
// The CTA's ids are fetched in stages (128 ids for 16-bit types): every warp issues one
// cp.async.bulk (TMA bulk copy) per listed K row and V row of its 16 slots straight into
// shared memory, completion counted by an mbarrier (one expect_tx arrival per warp), three
// stages in flight; the ids of the next stage to issue load while the current stage waits
// and computes, so no id round trip sits between a freed buffer and its refill. A lane holds
// 8 elements (one 16-byte vector) of a row; 16 lanes cover a Dh = 128 row.
// Split partials (m, l, o) merge three ways:
//   * 1 split: the CTA writes the output;
//   * <= 16 splits: the splits of a (row, KV head) form one thread-block cluster and merge
//     through distributed shared memory - every CTA combines a slice of the outputs;
//   * more: partials go to global scratch and the last CTA (atomic ticket) merges them.
// Launches carry programmatic stream serialization: the kernel calls griddepcontrol.wait
// before its first global read, so it may be resident before its producer finishes.
// Every mbarrier wait is bounded (2 s of %globaltimer); on expiry the CTA records
// LSA_ERR_TIMEOUT in the status counter and leaves after a second bounded wait.
#include <cooperative_groups.h>

#include <mutex>

#include "common.cuh"
#include "umma.cuh"

namespace cg = cooperative_groups;

namespace lsa {

constexpr int kReadThreads = 256;  // 8 warps
constexpr int kMaxClusterSplits = 16;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegBig = -3.0e38f;

template <typename T>
struct StageIds {
    static constexpr int value = sizeof(T) == 4 ? 64 : 128;
};
constexpr int kReadStages = 3;  // K/V stages in flight (ring of shared-memory buffers)

// Four 8x8 b16 matrices from shared memory (lane l addresses row l & 7 of matrix l >> 3).
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D[16x8] += A[16x16] B[16x8], fp32 accumulate; A, B both bf16 or both fp16.
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1);

template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                        uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two fp32 values as one register of the 16-bit type (lo in the low half).
template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<float>(float, float) { return 0u; }
template <>
__device__ __forceinline__ void mma16816<float>(float (&)[4], uint32_t, uint32_t, uint32_t, uint32_t, uint32_t,
                                                uint32_t) {}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

enum Combine : int { kSingle = 0, kCluster = 1, kTicket = 2 };

struct ReadArgs {
    const void* q;
    const void* k;
    const void* v;
    const int32_t* ids;
    const int32_t* lengths;
    void* out;
    float* part_o;   // [R*Hkv, splits, G, D]   (ticket combine)
    float* part_ml;  // [R*Hkv, splits, G, 2]
    int32_t* tickets;
    int32_t* status;
    int32_t* queue;  // persistent read: [0] next work item, [1] CTAs done (zero at rest)
    int64_t Tq, Tk;
    int Hq, Hkv, G, width, splits, span, combine;
    float scale_log2;  // scale * log2(e)
    // partial mode (sequence shards): ids are global positions, this call's K/V hold
    // positions [id_base, id_base + Tk); fp32 normalised output and log2-sum-exp per
    // (row, q head) instead of `out`
    int id_base;
    float* out32;
    float* lse;
};

// Final write of one output element (and, in partial mode, the row-head's log2-sum-exp).
template <typename T, int D>
__device__ __forceinline__ void write_out(const ReadArgs& a, int64_t rq, int e, float O, float M, float L) {
    const float val = L > 0.0f ? O / L : 0.0f;
    if (a.out32) {
        a.out32[rq * D + e] = val;
        if (e == 0) a.lse[rq] = L > 0.0f ? M + log2f(L) : -INFINITY;
    } else {
        reinterpret_cast<T*>(a.out)[rq * D + e] = from_f32<T>(val);
    }
}

// The last CTA of unit rh (row * Hkv + h) merges the splits' partials (part_o / part_ml in
// global memory) and writes the output: the split weights are staged in shared memory
// (wts: splits * G + 2 G floats), then every output sums its splits with independent loads.
struct CtaSync {
    __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

template <typename T, int D, typename Sync = CtaSync>
__device__ void merge_splits(const ReadArgs& a, int rh, int64_t row, int h, float* wts, int tid, Sync sync = Sync{}) {
    const int G = a.G;
    float* tot = wts + a.splits * G;  // [G] totals, then [G] maxima
    float* wmax = tot + G;
    for (int i = tid; i < a.splits * G; i += kReadThreads) wts[i] = __ldcg(a.part_ml + ((int64_t)rh * a.splits * G + i) * 2);
    sync();
    if (tid < G) {
        float M = kNegBig;
        for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, wts[sp * G + tid]);
        float L = 0.0f;
        for (int sp = 0; sp < a.splits; ++sp) {
            float f = exp2f(wts[sp * G + tid] - M);
            L += __ldcg(a.part_ml + (((int64_t)rh * a.splits + sp) * G + tid) * 2 + 1) * f;
            wts[sp * G + tid] = f;
        }
        tot[tid] = L;
        wmax[tid] = M;
    }
    sync();
    for (int o = tid; o < G * D; o += kReadThreads) {
        int g = o / D, e = o % D;
        float O = 0.0f;
#pragma unroll 8
        for (int sp = 0; sp < a.splits; ++sp)
            O += wts[sp * G + g] * __ldcg(a.part_o + (((int64_t)rh * a.splits + sp) * G + g) * D + e);
        write_out<T, D>(a, (row * a.Hq) + h * G + g, e, O, wmax[g], tot[g]);
    }
}

// One stage of the tensor-core path for one warp: the warp's SPW = 8 J staged slots (K rows
// at kaddr, V rows at vaddr, row stride D + 8 elements, listed flags fl). S = q K^T as
// mma.m16n8k16 with the query heads as M (rows >= G are zero); the scores stay in registers
// and become the P operand of O += P V (FA2 fragment reuse); (mrow, lrow) is the running
// max / sum of row lane / 4 in the exp2 domain.
template <typename T, int D, int J>
__device__ __forceinline__ void mma_stage(uint32_t kaddr, uint32_t vaddr, const unsigned char* fl,
                                          const uint32_t (&qa)[D / 16][2], float (&o)[D / 8][4], float& mrow,
                                          float& lrow, float scale_log2, int lane) {
    constexpr int ROWS = D + 8, DC = D / 16, NT = D / 8, SPW = 8 * J;
    const int tq = lane & 3;
    float sc[J][4];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
#pragma unroll
        for (int q4 = 0; q4 < DC / 2; ++q4) {  // 4 dim blocks of 8 per ldmatrix.x4
            uint32_t b0, b1, b2, b3;
            uint32_t addr = kaddr + ((8 * j + (lane & 7)) * ROWS + (4 * q4 + (lane >> 3)) * 8) * 2;
            ldsm_x4(addr, b0, b1, b2, b3);
            mma16816<T>(sc[j], qa[2 * q4][0], 0u, qa[2 * q4][1], 0u, b0, b1);
            mma16816<T>(sc[j], qa[2 * q4 + 1][0], 0u, qa[2 * q4 + 1][1], 0u, b2, b3);
        }
    }
    // scores of row gq for keys 8j + 2tq + {0, 1}; unlisted slots never count
    float sv[2 * J];
    float mx = kNegBig;
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            bool valid = fl[8 * j + 2 * tq + e] != 0;
            float v = valid ? sc[j][e] * scale_log2 : -INFINITY;
            sv[2 * j + e] = v;
            mx = fmaxf(mx, v);
        }
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 2));
    float mnew = fmaxf(mrow, mx);
    float alpha = exp2f(mrow - mnew);
    mrow = mnew;
    float p[2 * J];
    float psum = 0.0f;
#pragma unroll
    for (int i = 0; i < 2 * J; ++i) {
        p[i] = exp2f(sv[i] - mnew);
        psum += p[i];
    }
    lrow = lrow * alpha + psum;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        o[nt][0] *= alpha;
        o[nt][1] *= alpha;
    }
    // the P operand covers k16 = 16 keys; with 8 slots per warp its upper half is zero
    uint32_t pa0 = pack2<T>(p[0], p[1]), pa2 = J == 2 ? pack2<T>(p[2 % (2 * J)], p[3 % (2 * J)]) : 0u;
    // V rows of unlisted slots hold stale shared memory: zero their fragment halves
    // (b0/b2 carry keys 2tq, 2tq + 1; b1/b3 keys 8 + 2tq, 9 + 2tq) so 0 * garbage
    // cannot turn into NaN inside the MMA
    const uint32_t vm0 = (fl[2 * tq] ? 0x0000FFFFu : 0u) | (fl[2 * tq + 1] ? 0xFFFF0000u : 0u);
    const uint32_t vm1 = J == 2 ? ((fl[(8 + 2 * tq) % SPW] ? 0x0000FFFFu : 0u) |
                                   (fl[(9 + 2 * tq) % SPW] ? 0xFFFF0000u : 0u))
                                : 0u;
#pragma unroll
    for (int np = 0; np < NT / 2; ++np) {
        uint32_t b0, b1, b2, b3;
        // with 8 slots the upper key half re-reads this warp's rows (masked to zero)
        int key = (lane & 7) + (J == 2 ? 8 * ((lane >> 3) & 1) : 0);
        int dblk = 2 * np + (lane >> 4);
        ldsm_x4_t(vaddr + (key * ROWS + dblk * 8) * 2, b0, b1, b2, b3);
        mma16816<T>(o[2 * np], pa0, 0u, pa2, 0u, b0 & vm0, b1 & vm1);
        mma16816<T>(o[2 * np + 1], pa0, 0u, pa2, 0u, b2 & vm0, b3 & vm1);
    }
}

template <typename T, int D, int GMAX>
__global__ void __launch_bounds__(kReadThreads) sparse_read_kernel(ReadArgs a) {
    constexpr int STAGE = StageIds<T>::value;
    constexpr int LPR = D / 8;          // lanes per key row (8 elements per lane)
    constexpr int GPW = 32 / LPR;       // key rows per warp step
    constexpr int NW = kReadThreads / 32;
    constexpr int NG = NW * GPW;        // row groups in the CTA
    constexpr int PER = STAGE / NG;     // slots of a group in a stage
    constexpr bool MMA = sizeof(T) == 2;      // tensor-core path for 16-bit inputs
    constexpr int NGE = MMA ? NW : NG;        // partial-state owners merged at the end
    constexpr int ROWS = MMA ? D + 8 : D;     // smem row stride (elements): +16 B keeps ldmatrix conflict-free
    constexpr int ROWB = D * sizeof(T);       // bytes copied per row
    constexpr int STAGE_BYTES = STAGE * ROWS * (int)sizeof(T);
    constexpr int IDW = STAGE / NW;     // id slots a warp issues per stage
    constexpr int SPW = IDW;            // slots a warp computes per stage (tensor-core path)
    constexpr int J = SPW / 8;          // n8 key tiles per warp
    static_assert(SPW == 8 || SPW == 16, "a warp computes one or two n8 key tiles");
    static_assert(2 * IDW <= 32, "a warp issues the K and V rows of its slots in one pass");
    constexpr int NST = kReadStages;
    extern __shared__ __align__(128) unsigned char smem[];
    T* sK = reinterpret_cast<T*>(smem);                      // [NST][STAGE][D]
    T* sV = reinterpret_cast<T*>(smem + NST * STAGE_BYTES);  // [NST][STAGE][D]
    __shared__ __align__(8) uint64_t bars[NST];
    __shared__ unsigned char sflag[NST * STAGE];              // slot listed and in range
    __shared__ int is_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = warp * GPW + lane / LPR;
    const int lg = lane % LPR;
    const int rh = blockIdx.x / a.splits;  // row * Hkv + kv head
    const int split = blockIdx.x % a.splits;
    const int64_t row = rh / a.Hkv;
    const int h = rh % a.Hkv;
    const int64_t b = row / a.Tq;
    const int G = a.G;

    if (tid == 0) {
#pragma unroll
        for (int i = 0; i < NST; ++i) mbar_init(&bars[i], NW);  // one expect_tx arrival per warp per stage
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_wait();  // inputs produced by the previous kernel are visible past this point
    pdl_trigger();

    const int s0 = split * a.span;
    const int32_t* idrow = a.ids + row * a.width;
    const T* kbase = reinterpret_cast<const T*>(a.k) + (b * a.Tk * a.Hkv + h) * D;
    const T* vbase = reinterpret_cast<const T*>(a.v) + (b * a.Tk * a.Hkv + h) * D;
    const int64_t tstride = (int64_t)a.Hkv * D;  // elements between consecutive positions
    // Every warp issues the copies of its own IDW slots per stage: lanes [0, IDW) the K rows,
    // lanes [IDW, 2 IDW) the V rows of the same slots.
    const bool issuer = lane < 2 * IDW;
    const bool is_v = lane >= IDW;
    const int my_slot = warp * IDW + (lane % IDW);
    auto load_id = [&](int stage) -> int {  // needs no length: loads overlap the length load
        int at = s0 + stage * STAGE + my_slot;
        return (issuer && at < s0 + a.span && at < a.width) ? idrow[at] - a.id_base : -1;
    };
    int id_first[NST];
#pragma unroll
    for (int i = 0; i < NST; ++i) id_first[i] = load_id(i);
    int id_next = load_id(NST);  // the stage issued when buffer 0 frees
    int len = a.lengths[row];
    len = len < 0 ? 0 : (len > a.width ? a.width : len);
    const int s1 = min(s0 + a.span, len);
    const int n_ids = s1 > s0 ? s1 - s0 : 0;
    const int n_stages = (n_ids + STAGE - 1) / STAGE;

    auto issue = [&](int stage, int id) {
        int buf = stage % NST;
        int at = s0 + stage * STAGE + my_slot;
        bool ok = issuer && at < s1 && id >= 0 && id < a.Tk;
        uint32_t n = __popc(__ballot_sync(0xFFFFFFFFu, ok));
        if (lane == 0) mbar_arrive_expect_tx(&bars[buf], n * ROWB);
        if (issuer && !is_v) sflag[buf * STAGE + my_slot] = ok ? 1 : 0;
        __syncwarp();
        if (ok) {
            T* dst = (is_v ? sV : sK) + ((size_t)buf * STAGE + my_slot) * ROWS;
            const T* src = (is_v ? vbase : kbase) + (int64_t)id * tstride;
            bulk_g2s(dst, src, ROWB, &bars[buf]);
        }
    };

#pragma unroll
    for (int i = 0; i < NST; ++i)
        if (i < n_stages) issue(i, id_first[i]);
    __syncthreads();  // slot flags visible to every group
    // on an expired wait: thread 0 waits (bounded) for every stage still in flight
    auto drain = [&](int st) {
        if (tid == 0)
            for (int s2 = st; s2 < n_stages && s2 < st + NST; ++s2) mbar_wait_bounded(&bars[s2 % NST], (s2 / NST) & 1);
    };

    bool failed = false;
    float* red = reinterpret_cast<float*>(smem);  // [NGE][GMAX][D] group partials (after the loop)
    float* redml = red + NGE * GMAX * D;          // [NGE][GMAX][2]
    float* po = redml + NGE * GMAX * 2;           // [GMAX][D]  the CTA's partial
    float* pml = po + GMAX * D;                   // [GMAX][2]

    if constexpr (MMA) {
        // Tensor-core path (16-bit inputs): warp w owns slots [16 w, 16 w + 16) of a stage.
        // S = q K^T as mma.m16n8k16 with the query heads as M (rows >= G are zero), the
        // scores stay in registers and become the P operand of O += P V (FA2 fragment reuse).
        const int gq = lane >> 2, tq = lane & 3;
        constexpr int DC = D / 16;  // k16 chunks over the head dim
        constexpr int NT = D / 8;   // n8 output tiles over the head dim
        uint32_t qa[DC][2];         // rows gq of the A operand (rows gq + 8 are zero padding)
#pragma unroll
        for (int dc = 0; dc < DC; ++dc) {
            const T* qp = reinterpret_cast<const T*>(a.q) + ((row * a.Hq) + h * G + gq) * D + dc * 16 + 2 * tq;
            qa[dc][0] = gq < G ? *reinterpret_cast<const uint32_t*>(qp) : 0u;
            qa[dc][1] = gq < G ? *reinterpret_cast<const uint32_t*>(qp + 8) : 0u;
        }
        float o[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
        float mrow = kNegBig, lrow = 0.0f;  // row gq (this thread's share of l; quad-summed at the end)
        for (int st = 0; st < n_stages; ++st) {
            int buf = st % NST;
            bool ok = mbar_wait_bounded(&bars[buf], (st / NST) & 1);
            if (__syncthreads_or(!ok)) {  // block-uniform: every thread leaves together
                drain(st);  // copies in flight
                __syncthreads();
                failed = true;
                break;
            }
            const int kb = warp * SPW;  // first slot of this warp
            const unsigned char* fl = sflag + buf * STAGE + kb;
            bool any = __any_sync(0xFFFFFFFFu, lane < SPW && fl[lane % SPW]);
            if (any)
                mma_stage<T, D, J>(smem_u32(sK + ((size_t)buf * STAGE + kb) * ROWS),
                                   smem_u32(sV + ((size_t)buf * STAGE + kb) * ROWS), fl, qa, o, mrow, lrow,
                                   a.scale_log2, lane);
            __syncthreads();  // every warp is done with this buffer
            if (st + NST < n_stages) {
                issue(st + NST, id_next);
                id_next = load_id(st + NST + 1);
            }
        }
        if (!failed) {
            lrow += __shfl_xor_sync(0xFFFFFFFFu, lrow, 1);
            lrow += __shfl_xor_sync(0xFFFFFFFFu, lrow, 2);
            if (gq < G) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    red[(warp * GMAX + gq) * D + nt * 8 + 2 * tq] = o[nt][0];
                    red[(warp * GMAX + gq) * D + nt * 8 + 2 * tq + 1] = o[nt][1];
                }
                if (tq == 0) {
                    redml[(warp * GMAX + gq) * 2] = mrow;
                    redml[(warp * GMAX + gq) * 2 + 1] = lrow;
                }
            }
        }
    } else {
        // CUDA-core path (fp32 inputs): 16 lanes hold a row, 8 elements each.
        float qr[GMAX][8];
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            if (g < G) {
                const T* qp = reinterpret_cast<const T*>(a.q) + ((row * a.Hq) + h * G + g) * D + lg * 8;
                load8<T>(qp, qr[g]);
#pragma unroll
                for (int e = 0; e < 8; ++e) qr[g][e] *= a.scale_log2;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) qr[g][e] = 0.0f;
            }
        }
        float m[GMAX], l[GMAX], acc[GMAX][8];
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
            m[g] = kNegBig;
            l[g] = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[g][e] = 0.0f;
        }
        for (int st = 0; st < n_stages; ++st) {
            int buf = st % NST;
            bool ok = mbar_wait_bounded(&bars[buf], (st / NST) & 1);
            if (__syncthreads_or(!ok)) {
                drain(st);
                __syncthreads();
                failed = true;
                break;
            }
            float s[PER][GMAX];
            bool kept[PER];
#pragma unroll
            for (int u = 0; u < PER; ++u) {
                int j = grp + NG * u;
                kept[u] = sflag[buf * STAGE + j] != 0;
#pragma unroll
                for (int g = 0; g < GMAX; ++g) s[u][g] = kNegBig;
                if (kept[u]) {
                    float kv[8];
                    load8<T>(sK + ((size_t)buf * STAGE + j) * ROWS + lg * 8, kv);
#pragma unroll
                    for (int g = 0; g < GMAX; ++g) {
                        float p = 0.0f;
#pragma unroll
                        for (int e = 0; e < 8; ++e) p = fmaf(qr[g][e], kv[e], p);
                        s[u][g] = p;
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < PER; ++u)
#pragma unroll
                for (int g = 0; g < GMAX; ++g)
#pragma unroll
                    for (int off = LPR / 2; off >= 1; off >>= 1)
                        s[u][g] += __shfl_xor_sync(0xFFFFFFFFu, s[u][g], off);
#pragma unroll
            for (int g = 0; g < GMAX; ++g) {
                float mx = m[g];
#pragma unroll
                for (int u = 0; u < PER; ++u)
                    if (kept[u]) mx = fmaxf(mx, s[u][g]);
                float alpha = exp2f(m[g] - mx);
                l[g] *= alpha;
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[g][e] *= alpha;
                m[g] = mx;
            }
#pragma unroll
            for (int u = 0; u < PER; ++u) {
                if (!kept[u]) continue;
                int j = grp + NG * u;
                float vv[8];
                load8<T>(sV + ((size_t)buf * STAGE + j) * ROWS + lg * 8, vv);
#pragma unroll
                for (int g = 0; g < GMAX; ++g) {
                    float p = exp2f(s[u][g] - m[g]);
                    l[g] += p;
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(p, vv[e], acc[g][e]);
                }
            }
            __syncthreads();
            if (st + NST < n_stages) {
                issue(st + NST, id_next);
                id_next = load_id(st + NST + 1);
            }
        }
        if (!failed) {
#pragma unroll
            for (int g = 0; g < GMAX; ++g) {
#pragma unroll
                for (int e = 0; e < 8; ++e) red[(grp * GMAX + g) * D + lg * 8 + e] = acc[g][e];
                if (lg == 0) {
                    redml[(grp * GMAX + g) * 2] = m[g];
                    redml[(grp * GMAX + g) * 2 + 1] = l[g];
                }
            }
        }
    }
    if (failed) {
        if (tid == 0) atomicExch(a.status, LSA_ERR_TIMEOUT);
        if (a.combine == kCluster) cg::this_cluster().sync();  // peers reach both barriers below
        if (a.combine == kCluster) cg::this_cluster().sync();
        return;
    }

    // merge the NGE row groups of the CTA
    __syncthreads();
    for (int o = tid; o < G * D; o += kReadThreads) {
        int g = o / D, e = o % D;
        float M = kNegBig;
#pragma unroll 4
        for (int r = 0; r < NGE; ++r) M = fmaxf(M, redml[(r * GMAX + g) * 2]);
        float L = 0.0f, O = 0.0f;
#pragma unroll 4
        for (int r = 0; r < NGE; ++r) {
            float f = exp2f(redml[(r * GMAX + g) * 2] - M);
            L += redml[(r * GMAX + g) * 2 + 1] * f;
            O += red[(r * GMAX + g) * D + e] * f;
        }
        if (a.combine == kSingle) {
            write_out<T, D>(a, (row * a.Hq) + h * G + g, e, O, M, L);
        } else if (a.combine == kCluster) {
            po[g * D + e] = O;
            if (e == 0) {
                pml[g * 2] = M;
                pml[g * 2 + 1] = L;
            }
        } else {
            int64_t pidx = ((int64_t)rh * a.splits + split) * G + g;
            a.part_o[pidx * D + e] = O;
            if (e == 0) {
                a.part_ml[pidx * 2] = M;
                a.part_ml[pidx * 2 + 1] = L;
            }
        }
    }
    if (a.combine == kSingle) return;

    if (a.combine == kCluster) {
        // every CTA of the cluster merges a slice of the outputs from all ranks' partials
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();
        const int S = a.splits;
        const int total = G * D;
        const int chunk = (total + S - 1) / S;
        const int o0 = split * chunk;
        for (int o = o0 + tid; o < min(o0 + chunk, total); o += kReadThreads) {
            int g = o / D, e = o % D;
            float mr[kMaxClusterSplits];
            float M = kNegBig;
#pragma unroll
            for (int r = 0; r < kMaxClusterSplits; ++r) {
                if (r < S) {
                    const float* peer = cluster.map_shared_rank(pml, r);
                    mr[r] = peer[g * 2];
                    M = fmaxf(M, mr[r]);
                }
            }
            float L = 0.0f, O = 0.0f;
#pragma unroll
            for (int r = 0; r < kMaxClusterSplits; ++r) {
                if (r < S) {
                    const float* peer_ml = cluster.map_shared_rank(pml, r);
                    const float* peer_o = cluster.map_shared_rank(po, r);
                    float f = exp2f(mr[r] - M);
                    L += peer_ml[g * 2 + 1] * f;
                    O += peer_o[g * D + e] * f;
                }
            }
            write_out<T, D>(a, (row * a.Hq) + h * G + g, e, O, M, L);
        }
        cluster.sync();  // keep this CTA's partial alive until every peer has read it
        return;
    }

    __threadfence();
    __syncthreads();
    if (tid == 0) {
        int t = atomicAdd(a.tickets + rh, 1);
        is_last = t == a.splits - 1;
        if (is_last) a.tickets[rh] = 0;
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    merge_splits<T, D>(a, rh, row, h, red, tid);
}

// ------------------------------------------------------------------ decode read (latency path)

// A handful of (row, KV head) units (single-sequence decode: 8 units of ~2k ids): one
// cluster of up to 16 CTAs per unit, each CTA a contiguous slice of <= 256 list slots held
// in shared memory at once, so the whole slice is ONE memory round trip after the ids:
//   * after griddepcontrol.wait one load per thread brings the slice's ids, the row length
//     and the query fragments (one round trip);
//   * every K and V row of the slice is copied by 16-byte cp.async pieces (warp-wide, a
//     slot's rows contiguous across lanes) in two commit groups (slots below 128, the
//     rest), so the tensor-core stage of the first 128 slots runs while the tail lands;
//   * the compute is the split kernel's mma_stage (S = q K^T and O += P V on mma.sync with
//     the query heads as M); warps merge in shared memory with per-head weights computed
//     once; output slice c belongs to cluster rank c, and every CTA stores its partial of
//     each slice straight into the owner's shared-memory inbox (remote stores only: no
//     remote load round trips), so one cluster barrier separates the pushes from the
//     owners' merges.
// No scratch, no counters, no spin: a call needs no workspace.
constexpr int kDecodeReadSplits = 16;
constexpr int kDecodeReadMaxSpan = kReadThreads;  // one id per thread

template <typename T, int D, int GMAX>
static constexpr int decode_red_bytes() {
    // warp partials [NW][GMAX][D + 4] and (max, sum) [NW][GMAX][2], warp weights [NW][GMAX],
    // the CTA's (max, sum) [GMAX][2], rank weights [16][GMAX], the slice's (max, sum) [GMAX][2]
    return (kReadThreads / 32 * GMAX * (D + 4) + kReadThreads / 32 * GMAX * 3 + GMAX * 2 +
            kDecodeReadSplits * GMAX + GMAX * 2) * 4;
}

// One warp's tensor-core pass over J n8 tiles of staged slots (8 J rows at kaddr / vaddr,
// row stride D + 8 elements, listed flags fl), J in 1..4: S = q K^T with the query heads as M
// (two accumulation chains per tile: even and odd k16 chunks), the online softmax update,
// then O += P V in ceil(J / 2) k16 steps. Rows past the warp's J tiles are never addressed:
// the upper half of an odd last k16 step re-reads the lower half (masked to zero).
template <typename T, int D, int J>
__device__ __forceinline__ void mma_pass(uint32_t kaddr, uint32_t vaddr, const unsigned char* fl,
                                         const uint32_t (&qa)[D / 16][2], float (&o)[D / 8][4], float& mrow,
                                         float& lrow, float scale_log2, int lane) {
    constexpr int ROWS = D + 8, DC = D / 16, NT = D / 8, KT = (J + 1) / 2;
    const int tq = lane & 3;
    float sc[J][2];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        float s0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, s1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int q4 = 0; q4 < DC / 2; ++q4) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4(kaddr + ((8 * j + (lane & 7)) * ROWS + (4 * q4 + (lane >> 3)) * 8) * 2, b0, b1, b2, b3);
            mma16816<T>(s0, qa[2 * q4][0], 0u, qa[2 * q4][1], 0u, b0, b1);
            mma16816<T>(s1, qa[2 * q4 + 1][0], 0u, qa[2 * q4 + 1][1], 0u, b2, b3);
        }
        sc[j][0] = s0[0] + s1[0];
        sc[j][1] = s0[1] + s1[1];
    }
    float sv[2 * J];
    float mx = kNegBig;
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const float v = fl[8 * j + 2 * tq + e] ? sc[j][e] * scale_log2 : -INFINITY;
            sv[2 * j + e] = v;
            mx = fmaxf(mx, v);
        }
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 2));
    const float mnew = fmaxf(mrow, mx);
    const float alpha = exp2f(mrow - mnew);
    mrow = mnew;
    float pr[2 * J];
    float psum = 0.0f;
#pragma unroll
    for (int i = 0; i < 2 * J; ++i) {
        pr[i] = exp2f(sv[i] - mnew);
        psum += pr[i];
    }
    lrow = lrow * alpha + psum;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        o[nt][0] *= alpha;
        o[nt][1] *= alpha;
    }
#pragma unroll
    for (int kt = 0; kt < KT; ++kt) {
        const bool hi = 2 * kt + 1 < J;  // the step's upper 8 keys exist
        const uint32_t pa0 = pack2<T>(pr[4 * kt], pr[4 * kt + 1]);
        const uint32_t pa2 = hi ? pack2<T>(pr[(4 * kt + 2) % (2 * J)], pr[(4 * kt + 3) % (2 * J)]) : 0u;
        // V rows of unlisted slots hold stale shared memory: zero their fragment halves so
        // 0 * garbage cannot turn into NaN inside the MMA
        const unsigned char* f = fl + 16 * kt;
        const uint32_t vm0 = (f[2 * tq] ? 0x0000FFFFu : 0u) | (f[2 * tq + 1] ? 0xFFFF0000u : 0u);
        const uint32_t vm1 = hi ? ((f[8 + 2 * tq] ? 0x0000FFFFu : 0u) | (f[9 + 2 * tq] ? 0xFFFF0000u : 0u)) : 0u;
        const int key = 16 * kt + (lane & 7) + (hi ? 8 * ((lane >> 3) & 1) : 0);
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vaddr + (key * ROWS + (2 * np + (lane >> 4)) * 8) * 2, b0, b1, b2, b3);
            mma16816<T>(o[2 * np], pa0, 0u, pa2, 0u, b0 & vm0, b1 & vm1);
            mma16816<T>(o[2 * np + 1], pa0, 0u, pa2, 0u, b2 & vm0, b3 & vm1);
        }
    }
}

template <typename T, int D, int GMAX, int J>
__global__ void __launch_bounds__(kReadThreads, 2) decode_read_kernel(ReadArgs a, int nslots) {
    constexpr int SPW = 8 * J;  // slots per warp
    static_assert(sizeof(T) == 2, "16-bit inputs");
    constexpr int ROWS = D + 8;  // +16 B per row keeps ldmatrix conflict-free
    constexpr int NW = kReadThreads / 32;
    constexpr int LPR = D / 8;  // 16-byte pieces per row
    extern __shared__ __align__(128) unsigned char smem[];
    T* sK = reinterpret_cast<T*>(smem);                  // [nslots][ROWS]
    T* sV = sK + (size_t)nslots * ROWS;                  // [nslots][ROWS]
    __shared__ int sid[kDecodeReadMaxSpan];
    __shared__ unsigned char sflag[kDecodeReadMaxSpan];
    // partials pushed here by the cluster's CTAs: [splits][chunk] outputs + [splits][GMAX][2]
    __shared__ float inbox[GMAX * D + kDecodeReadSplits * GMAX * 2 + kDecodeReadSplits];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x, rh = blockIdx.y;
    const int64_t row = rh / a.Hkv;
    const int h = rh % a.Hkv;
    const int64_t b = row / a.Tq;
    const int G = a.G;
    const int s0 = split * a.span;
    // first cluster phase: every CTA of the cluster has started before any of them stores
    // into a peer's inbox (waited on just before the pushes)
    if (gridDim.x > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    pdl_wait();  // the list and lengths are the previous kernel's output
    pdl_trigger();
    int id = -1;
    if (tid < a.span && s0 + tid < a.width) id = a.ids[row * a.width + s0 + tid] - a.id_base;
    int len = a.lengths[row];
    len = len < 0 ? 0 : (len > a.width ? a.width : len);
    const int gq = lane >> 2, tq = lane & 3;
    constexpr int DC = D / 16, NT = D / 8;
    uint32_t qa[DC][2];
#pragma unroll
    for (int dc = 0; dc < DC; ++dc) {
        const T* qp = reinterpret_cast<const T*>(a.q) + ((row * a.Hq) + h * G + gq) * D + dc * 16 + 2 * tq;
        qa[dc][0] = gq < G ? *reinterpret_cast<const uint32_t*>(qp) : 0u;
        qa[dc][1] = gq < G ? *reinterpret_cast<const uint32_t*>(qp + 8) : 0u;
    }
    const int n_here = max(0, min(s0 + a.span, len) - s0);
    const bool ok = tid < n_here && id >= 0 && id < a.Tk;
    sid[tid] = ok ? id : -1;
    sflag[tid] = ok ? 1 : 0;
    __syncthreads();
    const T* kbase = reinterpret_cast<const T*>(a.k) + (b * a.Tk * a.Hkv + h) * D;
    const T* vbase = reinterpret_cast<const T*>(a.v) + (b * a.Tk * a.Hkv + h) * D;
    const int64_t tstride = (int64_t)a.Hkv * D;
    // every warp copies the K and V rows of exactly the slots it computes on and waits only
    // for its own copies: a warp starts its tensor pass as soon as its rows have landed
    const int kb = warp * SPW;  // this warp's slots: one pass over the whole slice
    {
        const int nw = max(0, min(SPW, n_here - kb));
        for (int i = lane; i < nw * 2 * LPR; i += 32) {
            const int j = kb + i / (2 * LPR), pc = i % (2 * LPR);
            const int idj = sid[j];
            if (idj >= 0) {
                const bool isv = pc >= LPR;
                const int e = (pc % LPR) * 8;
                const T* src = (isv ? vbase : kbase) + (int64_t)idj * tstride + e;
                cp_async16(smem_u32((isv ? sV : sK) + (size_t)j * ROWS + e), src, 16);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }

    float o[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
    float mrow = kNegBig, lrow = 0.0f;
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
    {
        if (kb < n_here) {
            const unsigned char* fl = sflag + kb;
            if (__any_sync(0xFFFFFFFFu, fl[lane % SPW] != 0))
                mma_pass<T, D, J>(smem_u32(sK + (size_t)kb * ROWS), smem_u32(sV + (size_t)kb * ROWS), fl, qa, o,
                                  mrow, lrow, a.scale_log2, lane);
        }
    }
    __syncthreads();  // the K/V buffers become the reduction buffers
    constexpr int RS = D + 4;                     // padded row: the fragment stores hit distinct banks
    float* red = reinterpret_cast<float*>(smem);  // [NW][GMAX][RS]
    float* redml = red + NW * GMAX * RS;          // [NW][GMAX][2]
    float* wf = redml + NW * GMAX * 2;            // [NW][GMAX] weights of the warps' partials
    float* cml = wf + NW * GMAX;                  // [GMAX][2] the CTA's (max, sum)
    lrow += __shfl_xor_sync(0xFFFFFFFFu, lrow, 1);
    lrow += __shfl_xor_sync(0xFFFFFFFFu, lrow, 2);
    if (gq < G) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            *reinterpret_cast<float2*>(red + (warp * GMAX + gq) * RS + nt * 8 + 2 * tq) = make_float2(o[nt][0], o[nt][1]);
        if (tq == 0) {
            redml[(warp * GMAX + gq) * 2] = mrow;
            redml[(warp * GMAX + gq) * 2 + 1] = lrow;
        }
    }
    __syncthreads();
    if (tid < NW * G) {  // (warp, query head): the head's max over the warps, this warp's weight
        const int w = tid / G, g = tid % G;
        float M = kNegBig;
#pragma unroll
        for (int w2 = 0; w2 < NW; ++w2) M = fmaxf(M, redml[(w2 * GMAX + g) * 2]);
        wf[w * GMAX + g] = exp2f(redml[(w * GMAX + g) * 2] - M);
        if (w == 0) cml[g * 2] = M;
    }
    __syncthreads();
    if (tid < G) {
        float L = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) L += redml[(w * GMAX + tid) * 2 + 1] * wf[w * GMAX + tid];
        cml[tid * 2 + 1] = L;
    }
    __syncthreads();
    const int S = (int)gridDim.x;
    if (S == 1) {
        for (int oi = tid; oi < G * D; oi += kReadThreads) {
            const int g = oi / D, e = oi % D;
            float O = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; ++w) O += red[(w * GMAX + g) * RS + e] * wf[w * GMAX + g];
            write_out<T, D>(a, (row * a.Hq) + h * G + g, e, O, cml[g * 2], cml[g * 2 + 1]);
        }
        return;
    }
    // the cluster merge: output slice c (chunk outputs) belongs to rank c; every CTA stores
    // its partial of each slice straight into the owner's inbox (remote stores, no remote
    // loads), one cluster barrier, then each owner merges its slice from its own memory
    cg::cluster_group cluster = cg::this_cluster();
    const int total = G * D, chunk = (total + S - 1) / S;
    float* in_o = inbox;                                // [S][chunk]
    float* in_ml = inbox + S * chunk;                   // [S][GMAX][2] (S * chunk < G * D + 16)
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // (first phase)
    for (int oi = tid; oi < total; oi += kReadThreads) {
        const int g = oi / D, e = oi % D;
        float O = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) O += red[(w * GMAX + g) * RS + e] * wf[w * GMAX + g];
        const int owner = oi / chunk;
        cluster.map_shared_rank(in_o, owner)[split * chunk + (oi - owner * chunk)] = O;
    }
    if (tid < S * G) {
        const int owner = tid / G, g = tid % G;
        float* dst = cluster.map_shared_rank(in_ml, owner) + (split * GMAX + g) * 2;
        dst[0] = cml[g * 2];
        dst[1] = cml[g * 2 + 1];
    }
    cluster.sync();  // every partial is in its owner's inbox; nothing remote is touched after this
    const int o0 = split * chunk;
    // the heads this slice touches: [g0, g1]; per (rank, head) weight against the head's max
    const int g0 = o0 / D, g1 = (min(o0 + chunk, total) - 1) / D;
    float* rw = cml + GMAX * 2;                    // [S][GMAX]
    float* rml = rw + kDecodeReadSplits * GMAX;    // [GMAX][2]
    if (tid < S * G) {
        const int r = tid / G, g = tid % G;
        if (g >= g0 && g <= g1) {
            float M = kNegBig;
            for (int r2 = 0; r2 < S; ++r2) M = fmaxf(M, in_ml[(r2 * GMAX + g) * 2]);
            rw[r * GMAX + g] = exp2f(in_ml[(r * GMAX + g) * 2] - M);
            if (r == 0) rml[g * 2] = M;
        }
    }
    __syncthreads();
    if (tid < G && tid >= g0 && tid <= g1) {
        float L = 0.0f;
        for (int r = 0; r < S; ++r) L += in_ml[(r * GMAX + tid) * 2 + 1] * rw[r * GMAX + tid];
        rml[tid * 2 + 1] = L;
    }
    __syncthreads();
    for (int i = tid; i < chunk && o0 + i < total; i += kReadThreads) {
        const int g = (o0 + i) / D, e = (o0 + i) % D;
        float O = 0.0f;
        for (int r = 0; r < S; ++r) O += in_o[r * chunk + i] * rw[r * GMAX + g];
        write_out<T, D>(a, (row * a.Hq) + h * G + g, e, O, rml[g * 2], rml[g * 2 + 1]);
    }
}

template <typename T, int D, int GMAX>
static int decode_smem_bytes(int nslots) {
    const int kv = 2 * nslots * (D + 8) * (int)sizeof(T);
    const int red = decode_red_bytes<T, D, GMAX>();
    return kv > red ? kv : red;
}

// Splits of the decode read for `units` (row, KV head) units of `width` slots, or 0 when
// the call is not a decode-sized one (the split / persistent kernels take it).
static int decode_read_splits(int64_t units, int64_t width, int sms) {
    if (units <= 0 || width <= 0) return 0;
    int s = (int)((width + kDecodeReadMaxSpan - 1) / kDecodeReadMaxSpan);  // at most 256 slots per CTA
    if (s > kDecodeReadSplits) return 0;
    int64_t want = (width + 127) / 128;  // at least ~128 slots per CTA are worth a CTA
    if (want > kDecodeReadSplits) want = kDecodeReadSplits;
    if (want > s) s = (int)want;
    if (units * s > 2 * (int64_t)sms) return 0;  // more than one wave of two CTAs per SM
    return s;
}

template <typename T, int D, int GMAX, int J>
static int launch_decode_read_j(ReadArgs a, int64_t units, int splits, cudaStream_t st) {
    const int nslots = (a.span + 8 * J - 1) / (8 * J) * (8 * J);  // whole warps of 8 J slots
    const int smem = decode_smem_bytes<T, D, GMAX>(nslots);
    auto kern = decode_read_kernel<T, D, GMAX, J>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
            cudaSuccess)
        return LSA_ERR_CUDA;
    if (splits > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
        return LSA_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)splits, (unsigned)units);
    cfg.blockDim = dim3(kReadThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    attrs[1].id = cudaLaunchAttributeClusterDimension;
    attrs[1].val.clusterDim.x = (unsigned)splits;
    attrs[1].val.clusterDim.y = 1;
    attrs[1].val.clusterDim.z = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, kern, a, nslots) != cudaSuccess) return LSA_ERR_CUDA;
    return LSA_OK;
}

// slots per warp: 8 J with J the fewest n8 tiles that cover the slice in one pass
template <typename T, int D, int GMAX>
static int launch_decode_read(ReadArgs a, int64_t units, int splits, cudaStream_t st) {
    a.splits = splits;
    a.span = (a.width + splits - 1) / splits;
    const int per_warp = (a.span + kReadThreads / 32 - 1) / (kReadThreads / 32);
    if (per_warp <= 8) return launch_decode_read_j<T, D, GMAX, 1>(a, units, splits, st);
    if (per_warp <= 16) return launch_decode_read_j<T, D, GMAX, 2>(a, units, splits, st);
    if (per_warp <= 24) return launch_decode_read_j<T, D, GMAX, 3>(a, units, splits, st);
    return launch_decode_read_j<T, D, GMAX, 4>(a, units, splits, st);
}

template <typename T, int D>
static int dispatch_decode(const ReadArgs& a, int64_t units, int splits, cudaStream_t st) {
    if (a.G <= 1) return launch_decode_read<T, D, 1>(a, units, splits, st);
    if (a.G <= 2) return launch_decode_read<T, D, 2>(a, units, splits, st);
    if (a.G <= 4) return launch_decode_read<T, D, 4>(a, units, splits, st);
    if (a.G <= 8) return launch_decode_read<T, D, 8>(a, units, splits, st);
    return LSA_ERR_ARG;
}

// ------------------------------------------------------------------ persistent read

// Bandwidth-bound batches (at least one (row, KV head) unit per SM, 16-bit inputs): a
// persistent grid of one CTA per SM takes work items = (row, split, KV head) from a global
// queue (atomic counter: SMs that run slower take fewer items). Four producer warps feed a ring of three
// 128-id stages with 16-byte cp.async row pieces (full / empty mbarriers) while eight
// consumer warps run the tensor-core stage, so the copy issue never waits behind the math
// (measured: 256-byte TMA bulk copies per row issue too slowly for this - the SM takes one
// every ~10-15 cycles and a warp's copy instruction issues its lanes one after another).
// The ring spans items: the next item's rows are in flight while the current one finishes
// (no per-CTA prologue, no partly filled last wave). At an item's last stage the consumer
// warps merge their partials in the consumed stage (before releasing it), write the
// item's split partial, and the unit's last split (atomic ticket) writes the output with
// merge_splits. Queue counters: [0] next item, [1] CTAs done; the last CTA resets both.
constexpr int kPersistStage = 128;    // ids per stage
constexpr int kPersistProducers = 4;  // producer warps
constexpr int kPersistThreads = kReadThreads + 32 * kPersistProducers;

template <typename T, int D, int GMAX>
constexpr int persist_smem_bytes() {
    return 2 * kReadStages * kPersistStage * (D + 8) * (int)sizeof(T);
}

struct ConsumerSync {  // the consumer warps' named barrier (the producer warps never join it)
    __device__ __forceinline__ void operator()() const {
        asm volatile("bar.sync 1, %0;" ::"n"(kReadThreads) : "memory");
    }
};

__device__ __forceinline__ void producer_sync() {
    asm volatile("bar.sync 2, %0;" ::"n"(32 * kPersistProducers) : "memory");
}

// Named-barrier vote: true on every participating thread when any of them passes true, so
// a wait that expired on one thread sends the whole group out together.
template <int BAR, int COUNT>
__device__ __forceinline__ bool group_any(bool x) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)x), "n"(BAR), "n"(COUNT)
        : "memory");
    return r != 0;
}

// cp.async completion tracking without a reserved arrival: the barrier's pending count
// rises now and falls when this thread's earlier cp.async copies land
__device__ __forceinline__ void cp_async_track(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

struct PersistStage {
    int rh, split, first, last;  // rh < 0: no more work
};

template <typename T, int D, int GMAX>
__global__ void __launch_bounds__(kPersistThreads, 1) sparse_read_persist_kernel(ReadArgs a, int n_items) {
    constexpr int STAGE = kPersistStage;
    constexpr int NW = kReadThreads / 32;  // consumer warps
    constexpr int SPW = STAGE / NW;        // slots a consumer warp computes per stage (16)
    constexpr int J = SPW / 8;
    constexpr int NST = kReadStages;
    constexpr int ROWS = D + 8;
    constexpr int ROWB = D * sizeof(T);
    constexpr int STAGE_BYTES = STAGE * ROWS * (int)sizeof(T);  // the K (or V) rows of one stage
    constexpr int DC = D / 16, NT = D / 8;
    constexpr int NP = 32 * kPersistProducers;
    static_assert(sizeof(T) == 2, "tensor-core path only");
    static_assert(STAGE == NP, "a producer thread owns one slot of every stage");
    static_assert(NW * GMAX * D * 4 + NW * GMAX * 2 * 4 <= 2 * STAGE_BYTES, "the warp partials fit one stage");
    // stage buf = its K rows then its V rows (contiguous, so the warp partials of an item's
    // last stage can use the whole consumed stage)
    extern __shared__ __align__(128) unsigned char smem[];
    auto stage_k = [&](int buf) { return reinterpret_cast<T*>(smem + (size_t)buf * 2 * STAGE_BYTES); };
    auto stage_v = [&](int buf) { return reinterpret_cast<T*>(smem + ((size_t)buf * 2 + 1) * STAGE_BYTES); };
    __shared__ __align__(8) uint64_t full[NST], empty[NST];
    __shared__ unsigned char sflag[NST * STAGE];
    __shared__ PersistStage smeta[NST];
    __shared__ int pdesc[2][4];  // the producers' current item: rh, split, s0, s1 (rh < 0: stop)
    __shared__ int is_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = a.G;
    if (tid == 0) {
#pragma unroll
        for (int i = 0; i < NST; ++i) {
            mbar_init(&full[i], NP);   // one release arrival per producer thread (+ its tracked copies)
            mbar_init(&empty[i], NW);  // one arrival per consumer warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_wait();
    pdl_trigger();

    if (warp >= NW) {  // producer warps: producer thread pt copies slot pt of every stage
        const int pt = tid - kReadThreads;
        bool ok = true;
        int g = 0;
        for (int seq = 0;; ++seq) {
            int* d = pdesc[seq & 1];
            if (pt == 0) {
                const int it = atomicAdd(a.queue, 1);
                if (it >= n_items) {
                    d[0] = -1;
                    // every CTA takes items until the queue runs dry, then counts itself done;
                    // the last one resets the queue for the next launch
                    if (atomicAdd(a.queue + 1, 1) == (int)gridDim.x - 1) {
                        a.queue[0] = 0;
                        a.queue[1] = 0;
                    }
                } else {
                    // item order (row, split, KV head), heads fastest: the Hkv items that read
                    // the same positions of a row are taken side by side
                    const int h = it % a.Hkv, rs = it / a.Hkv;
                    const int split = rs % a.splits;
                    const int rh = (rs / a.splits) * a.Hkv + h;
                    int len = a.lengths[rh / a.Hkv];
                    len = len < 0 ? 0 : (len > a.width ? a.width : len);
                    const int s0 = split * a.span;
                    d[0] = rh;
                    d[1] = split;
                    d[2] = s0;
                    d[3] = max(s0, min(s0 + a.span, len));
                }
            }
            producer_sync();
            const int rh = d[0], split = d[1], s0 = d[2], s1 = d[3];
            // an item with no id keeps one empty stage, so its split still posts a partial
            const int n_st = rh < 0 ? 1 : max(1, (s1 - s0 + STAGE - 1) / STAGE);
            const int64_t row = rh < 0 ? 0 : rh / a.Hkv;
            const int h = rh < 0 ? 0 : rh % a.Hkv;
            const int64_t kv0 = ((row / a.Tq) * a.Tk * a.Hkv + h) * D;  // (b, position 0, h)
            for (int st = 0; st < n_st; ++st, ++g) {
                const int buf = g % NST;
                const bool waited = mbar_wait_bounded(&empty[buf], ((g / NST) & 1) ^ 1);
                if (group_any<2, 32 * kPersistProducers>(!waited)) {
                    ok = false;
                    break;
                }
                if (pt == 0) smeta[buf] = PersistStage{rh, split, st == 0, st == n_st - 1};
                int id = -1;
                if (rh >= 0) {
                    const int at = s0 + st * STAGE + pt;  // coalesced id loads
                    id = at < s1 ? a.ids[row * a.width + at] - a.id_base : -1;
                    if (id >= a.Tk) id = -1;
                }
                sflag[buf * STAGE + pt] = id >= 0 ? 1 : 0;
                // 16-byte pieces of the warp's 32 slots: lanes 0-15 a slot's K row, 16-31 its V row
                const int piece = lane & 15;
                const bool v_half = lane >= 16;
                const int slot0 = pt - lane;
                T* dst0 = (v_half ? stage_v(buf) : stage_k(buf)) + (size_t)slot0 * ROWS + piece * (16 / (int)sizeof(T));
                const T* src0 = reinterpret_cast<const T*>(v_half ? a.v : a.k) + kv0 + piece * (16 / (int)sizeof(T));
#pragma unroll 8
                for (int j = 0; j < 32; ++j) {
                    const int idj = __shfl_sync(0xFFFFFFFFu, id, j);
                    if (idj >= 0 && piece * 16 < ROWB)
                        cp_async16(smem_u32(dst0 + (size_t)j * ROWS), src0 + (int64_t)idj * a.Hkv * D, 16);
                }
                cp_async_track(&full[buf]);  // the phase also waits for these copies
                mbar_arrive(&full[buf]);      // release: the slot flags and stage record above
            }
            if (!ok || rh < 0) break;
        }
        if (!ok && lane == 0) {  // the consumers stopped: wait (bounded) for the copies in flight
            atomicExch(a.status, LSA_ERR_TIMEOUT);
            for (int s2 = max(0, g - NST); s2 < g; ++s2) mbar_wait_bounded(&full[s2 % NST], (s2 / NST) & 1);
        }
        return;
    }

    // consumer warps
    const int gq = lane >> 2, tq = lane & 3;
    uint32_t qa[DC][2];
    float o[NT][4];
    float mrow = kNegBig, lrow = 0.0f;
    for (int g = 0;; ++g) {
        const int buf = g % NST;
        const bool waited = mbar_wait_bounded(&full[buf], (g / NST) & 1);
        if (group_any<1, kReadThreads>(!waited)) {  // the consumers leave together
            if (tid == 0) atomicExch(a.status, LSA_ERR_TIMEOUT);
            return;
        }
        const PersistStage m = smeta[buf];
        if (m.rh < 0) return;  // no more work (the stop stage is never released)
        const int rh = m.rh;
        const int64_t row = rh / a.Hkv;
        const int h = rh % a.Hkv;
        if (m.first) {  // a new item: its query rows, fresh state
#pragma unroll
            for (int dc = 0; dc < DC; ++dc) {
                const T* qp = reinterpret_cast<const T*>(a.q) + ((row * a.Hq) + h * G + gq) * D + dc * 16 + 2 * tq;
                qa[dc][0] = gq < G ? *reinterpret_cast<const uint32_t*>(qp) : 0u;
                qa[dc][1] = gq < G ? *reinterpret_cast<const uint32_t*>(qp + 8) : 0u;
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
            mrow = kNegBig;
            lrow = 0.0f;
        }
        const unsigned char* fl = sflag + buf * STAGE + warp * SPW;
        if (__any_sync(0xFFFFFFFFu, lane < SPW && fl[lane % SPW]))
            mma_stage<T, D, J>(smem_u32(stage_k(buf) + (size_t)warp * SPW * ROWS),
                               smem_u32(stage_v(buf) + (size_t)warp * SPW * ROWS), fl, qa, o, mrow, lrow,
                               a.scale_log2, lane);
        if (m.last) {
            // the item's last stage: the warps' partials meet in this consumed stage
            ConsumerSync{}();
            float* red = reinterpret_cast<float*>(stage_k(buf));  // [NW][GMAX][D]
            float* redml = red + NW * GMAX * D;                    // [NW][GMAX][2]
            float l4 = lrow;
            l4 += __shfl_xor_sync(0xFFFFFFFFu, l4, 1);
            l4 += __shfl_xor_sync(0xFFFFFFFFu, l4, 2);
            if (gq < G) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    red[(warp * GMAX + gq) * D + nt * 8 + 2 * tq] = o[nt][0];
                    red[(warp * GMAX + gq) * D + nt * 8 + 2 * tq + 1] = o[nt][1];
                }
                if (tq == 0) {
                    redml[(warp * GMAX + gq) * 2] = mrow;
                    redml[(warp * GMAX + gq) * 2 + 1] = l4;
                }
            }
            ConsumerSync{}();
            for (int oi = tid; oi < G * D; oi += kReadThreads) {
                const int gg = oi / D, e = oi % D;
                float M = kNegBig;
#pragma unroll
                for (int r = 0; r < NW; ++r) M = fmaxf(M, redml[(r * GMAX + gg) * 2]);
                float L = 0.0f, O = 0.0f;
#pragma unroll
                for (int r = 0; r < NW; ++r) {
                    const float f = exp2f(redml[(r * GMAX + gg) * 2] - M);
                    L += redml[(r * GMAX + gg) * 2 + 1] * f;
                    O += red[(r * GMAX + gg) * D + e] * f;
                }
                const int64_t pidx = ((int64_t)rh * a.splits + m.split) * G + gg;
                a.part_o[pidx * D + e] = O;
                if (e == 0) {
                    a.part_ml[pidx * 2] = M;
                    a.part_ml[pidx * 2 + 1] = L;
                }
            }
            __threadfence();
            ConsumerSync{}();
            if (tid == 0) {
                const int t = atomicAdd(a.tickets + rh, 1);
                is_last = t == a.splits - 1;
                if (is_last) a.tickets[rh] = 0;
            }
            ConsumerSync{}();
            if (is_last) {
                __threadfence();
                merge_splits<T, D>(a, rh, row, h, red, tid, ConsumerSync{});
            }
            ConsumerSync{}();  // every consumer is done with the stage
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[buf]);
    }
}

struct ReadPlan {
    int splits, span, combine;
    int64_t part_o_bytes, part_ml_bytes, scratch_bytes, counters;
    bool persist = false;  // 16-bit inputs take sparse_read_persist_kernel over `grid` CTAs
    int64_t grid = 0;
};

static int num_sms() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

static int64_t round256(int64_t x) { return (x + 255) / 256 * 256; }

template <typename T, int D, int GMAX>
static constexpr int read_smem_bytes() {
    constexpr int STAGE = StageIds<T>::value;
    constexpr bool MMA = sizeof(T) == 2;
    constexpr int NG = (kReadThreads / 32) * (32 / (D / 8));
    constexpr int NGE = MMA ? kReadThreads / 32 : NG;
    constexpr int ROWS = MMA ? D + 8 : D;
    constexpr int stage_bytes = 2 * kReadStages * STAGE * ROWS * (int)sizeof(T);
    constexpr int red_bytes = (NGE * GMAX * D + NGE * GMAX * 2 + GMAX * D + GMAX * 2) * 4;
    return stage_bytes > red_bytes ? stage_bytes : red_bytes;
}

// How many clusters of each size (1..16 read CTAs) one device holds at once, probed once
// per device on the heaviest instantiation. A size the GPCs cannot place reports 0.
static const int* cluster_capacity() {
    static int table[128][kMaxClusterSplits + 1];
    static bool probed[128] = {false};
    static std::mutex m;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) dev = 0;
    std::lock_guard<std::mutex> lock(m);
    if (!probed[dev]) {
        auto kern = sparse_read_kernel<__nv_bfloat16, 128, 8>;
        constexpr int smem = read_smem_bytes<__nv_bfloat16, 128, 8>();
        bool ok = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess &&
                  cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                       cudaSharedmemCarveoutMaxShared) == cudaSuccess &&
                  cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
        for (int c = 0; c <= kMaxClusterSplits; ++c) {
            table[dev][c] = 0;
            if (!ok || c < 1) continue;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(c);
            cfg.blockDim = dim3(kReadThreads);
            cfg.dynamicSmemBytes = smem;
            cudaLaunchAttribute attr;
            attr.id = cudaLaunchAttributeClusterDimension;
            attr.val.clusterDim.x = c;
            attr.val.clusterDim.y = 1;
            attr.val.clusterDim.z = 1;
            cfg.attrs = &attr;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess) table[dev][c] = n;
        }
        cudaGetLastError();  // a refused probe leaves no sticky error
        probed[dev] = true;
    }
    return table[dev];
}

// splits: CTAs per (row, KV head). Auto (splits_req <= 0): about four CTAs per SM over the
// whole launch, at least 128 ids per split, at most one cluster. A count above the cluster
// limit merges through the ticket path.
static ReadPlan plan_read(int64_t R, int64_t Hkv, int64_t G, int64_t D, int64_t width, int64_t splits_req, int sms,
                          bool allow_persist = true) {
    ReadPlan p;
    int64_t units = R * Hkv;
    if (splits_req <= 0 && allow_persist && units >= 16 && width > 0 && (D == 64 || D == 128)) {
        // batches of at least 16 (row, KV head) units: the persistent grid (one CTA per SM)
        // beat the split kernel at every size measured from 16 units up (two 2116-id decode
        // rows: 12.7 vs 19.7 us; 64 x 4164-id rows: 264 vs 311 us); a single decode row (8
        // units) stays on the split kernel (9.1 vs 12.4 us). Items per SM: about four when the
        // units alone fill the SMs (more balance costs split merges), else enough splits for
        // about one item per SM; at least 512 (resp. 256) ids per item. Splits merge by ticket.
        const int64_t slots = (int64_t)sms;
        int64_t s, by_len;
        if (units >= slots) {
            s = (4 * slots + units - 1) / units;
            by_len = width / 512;
        } else {
            s = (slots + units - 1) / units;
            by_len = width / 256;
        }
        if (s > by_len) s = by_len;
        if (s < 1) s = 1;
        const int64_t items = units * s;
        const int64_t grid = items < slots ? items : slots;
        p.splits = (int)s;
        p.span = (int)((width + s - 1) / s);
        p.combine = kTicket;
        p.persist = true;
        p.grid = grid;
        p.part_o_bytes = round256(units * s * G * D * 4);
        p.part_ml_bytes = round256(units * s * G * 2 * 4);
        p.scratch_bytes = p.part_o_bytes + p.part_ml_bytes;
        p.counters = units + 3;  // tickets, the status word, the work queue and its done count
        return p;
    }
    const int* cap = cluster_capacity();
    int64_t s = splits_req;
    if (s <= 0) {
        int64_t target = 4 * (int64_t)sms;
        s = (target + units - 1) / (units > 0 ? units : 1);
        int64_t by_len = (width + 127) / 128;
        if (s > by_len) s = by_len;
        if (s > kMaxClusterSplits) s = kMaxClusterSplits;
        // the largest cluster size whose clusters all fit the device at once (portable 8 floor)
        while (s > 8 && cap[s] < units) --s;
    }
    int64_t max_splits = width > 0 ? width : 1;
    if (s > max_splits) s = max_splits;
    if (s < 1) s = 1;
    p.splits = (int)s;
    p.span = (int)((width + s - 1) / s);
    bool placeable = s <= kMaxClusterSplits && (s <= 8 || cap[s] > 0);
    p.combine = s == 1 ? kSingle : (placeable ? kCluster : kTicket);
    bool scratch = p.combine == kTicket;
    p.part_o_bytes = scratch ? round256(units * s * G * D * 4) : 0;
    p.part_ml_bytes = scratch ? round256(units * s * G * 2 * 4) : 0;
    p.scratch_bytes = p.part_o_bytes + p.part_ml_bytes;
    p.counters = units + 1;  // one ticket per (row, KV head) + the status word
    return p;
}

template <typename T, int D, int GMAX>
static int launch_read(const ReadArgs& a, int64_t ctas, cudaStream_t st) {
    constexpr int smem = read_smem_bytes<T, D, GMAX>();
    auto kern = sparse_read_kernel<T, D, GMAX>;
    // the largest shared-memory carveout, so two 16-bit CTAs (three stages each) share an SM
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
            cudaSuccess)
        return LSA_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3(kReadThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    int n = 0;
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
    if (a.combine == kCluster) {
        if (a.splits > 8 &&
            cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
            return LSA_ERR_CUDA;
        attrs[n].id = cudaLaunchAttributeClusterDimension;
        attrs[n].val.clusterDim.x = (unsigned)a.splits;
        attrs[n].val.clusterDim.y = 1;
        attrs[n].val.clusterDim.z = 1;
        ++n;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = n;
    if (cudaLaunchKernelEx(&cfg, kern, a) != cudaSuccess) return LSA_ERR_CUDA;
    return LSA_OK;
}

template <typename T, int D, int GMAX>
static int launch_persist(const ReadArgs& a, int64_t grid, int n_items, cudaStream_t st) {
    constexpr int smem = persist_smem_bytes<T, D, GMAX>();
    auto kern = sparse_read_persist_kernel<T, D, GMAX>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
            cudaSuccess)
        return LSA_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kPersistThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, a, n_items) != cudaSuccess) return LSA_ERR_CUDA;
    return LSA_OK;
}

template <typename T, int D>
static int dispatch_persist(const ReadArgs& a, int64_t grid, int n_items, cudaStream_t st) {
    if (a.G <= 1) return launch_persist<T, D, 1>(a, grid, n_items, st);
    if (a.G <= 2) return launch_persist<T, D, 2>(a, grid, n_items, st);
    if (a.G <= 4) return launch_persist<T, D, 4>(a, grid, n_items, st);
    if (a.G <= 8) return launch_persist<T, D, 8>(a, grid, n_items, st);
    return LSA_ERR_ARG;
}

template <typename T, int D>
static int dispatch_g(const ReadArgs& a, int64_t ctas, cudaStream_t st) {
    if (a.G <= 1) return launch_read<T, D, 1>(a, ctas, st);
    if (a.G <= 2) return launch_read<T, D, 2>(a, ctas, st);
    if (a.G <= 4) return launch_read<T, D, 4>(a, ctas, st);
    if (a.G <= 8) return launch_read<T, D, 8>(a, ctas, st);
    return LSA_ERR_ARG;
}

template <typename T>
static int dispatch_d(const ReadArgs& a, int D, int64_t ctas, cudaStream_t st) {
    if (D == 64) return dispatch_g<T, 64>(a, ctas, st);
    if (D == 128) return dispatch_g<T, 128>(a, ctas, st);
    return LSA_ERR_ARG;
}

int sparse_read_launch(const void* q, const void* k, const void* v, int dtype, const int32_t* ids,
                       const int32_t* lengths, int64_t B, int64_t Tq, int64_t Tk, int64_t Hq, int64_t Hkv, int64_t D,
                       int64_t width, float scale, void* out, void* scratch, int64_t scratch_bytes, int32_t* counters,
                       int64_t n_counters, int64_t splits, cudaStream_t stream, int64_t id_base = 0,
                       float* out32 = nullptr, float* lse = nullptr, bool allow_persist = true) {
    if (B < 0 || Tq < 0 || Tk < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || width < 0) return LSA_ERR_ARG;
    if (D != 64 && D != 128) return LSA_ERR_ARG;
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out | (uintptr_t)scratch | (uintptr_t)out32) & 15)
        return LSA_ERR_ARG;
    if ((out32 == nullptr) != (lse == nullptr) || id_base < 0 || id_base > INT32_MAX) return LSA_ERR_ARG;
    int64_t R = B * Tq;
    if (R == 0) return LSA_OK;
    int64_t G = Hq / Hkv;
    if (G > 8) return LSA_ERR_ARG;
    ReadPlan p = plan_read(R, Hkv, G, D, width, splits, num_sms(), allow_persist);
    if (scratch_bytes < p.scratch_bytes || n_counters < p.counters || !counters) return LSA_ERR_ARG;
    char* w = (char*)scratch;
    ReadArgs a;
    a.q = q; a.k = k; a.v = v; a.ids = ids; a.lengths = lengths; a.out = out;
    a.part_o = (float*)w;
    a.part_ml = (float*)(w + p.part_o_bytes);
    a.tickets = counters;
    a.status = counters + R * Hkv;
    a.queue = counters + R * Hkv + 1;
    a.Tq = Tq; a.Tk = Tk;
    a.Hq = (int)Hq; a.Hkv = (int)Hkv; a.G = (int)G; a.width = (int)width;
    a.splits = p.splits; a.span = p.span; a.combine = p.combine;
    a.scale_log2 = scale * kLog2e;
    a.id_base = (int)id_base;
    a.out32 = out32;
    a.lse = lse;
    int64_t ctas = R * Hkv * p.splits;
    // decode-sized calls (fewer than 16 units, splits not forced): the latency kernel
    if (splits <= 0 && R * Hkv < 16 && (dtype == kBF16 || dtype == kF16)) {
        const int ds = decode_read_splits(R * Hkv, width, num_sms());
        if (ds > 0) {
            if (dtype == kBF16)
                return D == 64 ? dispatch_decode<__nv_bfloat16, 64>(a, R * Hkv, ds, stream)
                               : dispatch_decode<__nv_bfloat16, 128>(a, R * Hkv, ds, stream);
            return D == 64 ? dispatch_decode<__half, 64>(a, R * Hkv, ds, stream)
                           : dispatch_decode<__half, 128>(a, R * Hkv, ds, stream);
        }
    }
    if (p.persist && (dtype == kBF16 || dtype == kF16)) {
        const int n_items = (int)ctas;
        if (dtype == kBF16)
            return D == 64 ? dispatch_persist<__nv_bfloat16, 64>(a, p.grid, n_items, stream)
                           : dispatch_persist<__nv_bfloat16, 128>(a, p.grid, n_items, stream);
        return D == 64 ? dispatch_persist<__half, 64>(a, p.grid, n_items, stream)
                       : dispatch_persist<__half, 128>(a, p.grid, n_items, stream);
    }
    if (dtype == kBF16) return dispatch_d<__nv_bfloat16>(a, (int)D, ctas, stream);
    if (dtype == kF16) return dispatch_d<__half>(a, (int)D, ctas, stream);
    if (dtype == kF32) return dispatch_d<float>(a, (int)D, ctas, stream);
    return LSA_ERR_ARG;
}

}  // namespace lsa

extern "C" {

// Plan of lsa_sparse_read: split count, scratch bytes (any content) and the number of int32
// counters (zero before the call; the kernel leaves them zero; the last one is the status
// word, LSA_ERR_TIMEOUT after an expired wait). splits_req <= 0 picks splits from the SM count.
int lsa_sparse_read_plan(int64_t B, int64_t Tq, int64_t Hq, int64_t Hkv, int64_t D, int64_t width, int64_t splits_req,
                         int64_t* splits, int64_t* scratch_bytes, int64_t* n_counters) {
    if (Hkv <= 0 || Hq % Hkv || width < 0) return LSA_ERR_ARG;
    lsa::ReadPlan p = lsa::plan_read(B * Tq, Hkv, Hq / Hkv, D, width, splits_req, lsa::num_sms());
    if (splits) *splits = p.splits;
    if (scratch_bytes) *scratch_bytes = p.scratch_bytes;
    if (n_counters) *n_counters = p.counters;
    return LSA_OK;
}

int lsa_sparse_read(const void* q, const void* k, const void* v, int dtype, const int32_t* ids,
                    const int32_t* lengths, int64_t B, int64_t Tq, int64_t Tk, int64_t Hq, int64_t Hkv, int64_t D,
                    int64_t width, float scale, void* out, void* scratch, int64_t scratch_bytes, int32_t* counters,
                    int64_t n_counters, int64_t splits, cudaStream_t stream) {
    return lsa::sparse_read_launch(q, k, v, dtype, ids, lengths, B, Tq, Tk, Hq, Hkv, D, width, scale, out, scratch,
                                   scratch_bytes, counters, n_counters, splits, stream);
}

/* Sequence-shard partial read: lists hold global positions; k/v hold positions
 * [id_base, id_base + Tk) of every batch row. Writes the fp32 normalised output over this
 * shard's listed keys and its log2-sum-exp per (row, q head) (-inf: no key here). */
int lsa_sparse_read_partial(const void* q, const void* k, const void* v, int dtype, const int32_t* ids,
                            const int32_t* lengths, int64_t B, int64_t Tq, int64_t Tk, int64_t Hq, int64_t Hkv,
                            int64_t D, int64_t width, float scale, int64_t id_base, float* out32, float* lse,
                            void* scratch, int64_t scratch_bytes, int32_t* counters, int64_t n_counters,
                            int64_t splits, cudaStream_t stream) {
    if (out32 == nullptr || lse == nullptr) return LSA_ERR_ARG;
    return lsa::sparse_read_launch(q, k, v, dtype, ids, lengths, B, Tq, Tk, Hq, Hkv, D, width, scale, nullptr,
                                   scratch, scratch_bytes, counters, n_counters, splits, stream, id_base, out32, lse);
}

}  // extern "C"

namespace lsa {

// out[i, :] = sum_p o[p, i, :] 2^(lse[p, i] - M) / sum_p 2^(lse[p, i] - M), M = max_p lse[p, i]:
// the softmax over the union of the parts' disjoint key sets. One warp per row-head.
template <typename T>
__global__ void merge_partials_kernel(const float* __restrict__ o, const float* __restrict__ lse, int P, int64_t n,
                                      int D, T* __restrict__ out) {
    const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (i >= n) return;
    float M = -INFINITY;
    for (int p = 0; p < P; ++p) M = fmaxf(M, lse[(int64_t)p * n + i]);
    float W = 0.0f;
    for (int p = 0; p < P; ++p) {
        const float x = lse[(int64_t)p * n + i];
        W += x == -INFINITY ? 0.0f : exp2f(x - M);
    }
    for (int e = lane; e < D; e += 32) {
        float acc = 0.0f;
        for (int p = 0; p < P; ++p) {
            const float x = lse[(int64_t)p * n + i];
            if (x != -INFINITY) acc += o[((int64_t)p * n + i) * D + e] * exp2f(x - M);
        }
        out[i * D + e] = from_f32<T>(W > 0.0f ? acc / W : 0.0f);
    }
}

}  // namespace lsa

extern "C" {

/* Merge P shard partials (o [P, n, D] fp32 normalised, lse [P, n] log2-sum-exp) into
 * out [n, D] of dtype (the result of one read over the union of the shards' keys). */
int lsa_merge_partials(const float* o, const float* lse, int64_t P, int64_t n, int64_t D, int dtype, void* out,
                       cudaStream_t stream) {
    if (P <= 0 || n < 0 || D <= 0) return LSA_ERR_ARG;
    if (n == 0) return LSA_OK;
    const unsigned grid = (unsigned)((n * 32 + 255) / 256);
    if (dtype == lsa::kBF16)
        lsa::merge_partials_kernel<__nv_bfloat16>
            <<<grid, 256, 0, stream>>>(o, lse, (int)P, n, (int)D, (__nv_bfloat16*)out);
    else if (dtype == lsa::kF16)
        lsa::merge_partials_kernel<__half><<<grid, 256, 0, stream>>>(o, lse, (int)P, n, (int)D, (__half*)out);
    else if (dtype == lsa::kF32)
        lsa::merge_partials_kernel<float><<<grid, 256, 0, stream>>>(o, lse, (int)P, n, (int)D, (float*)out);
    else
        return LSA_ERR_ARG;
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ no-allocation entry
//
// Some callers cannot call cudaMalloc at all: an inference server whose device memory is
// one pre-reserved arena owned by its own allocator, or a plugin host that forbids
// allocation once serving has started. lsa_sparse_read_noalloc serves them: the split
// partials and counters of the read live in fixed device arrays of this library instead of
// caller-provided buffers. The arrays are file-scope __device__ storage, so every GPU that
// loads the library holds them (8 MiB + 256 KiB) until the process exits.
namespace lsa {

constexpr int64_t kNoAllocScratchBytes = 8ll << 20;  // split partials (m, l, o)
constexpr int64_t kNoAllocCounters = 1 << 16;        // tickets + status word

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ __align__(256) int32_t g_noalloc_counters[kNoAllocCounters];

// Host copies of the arrays' device addresses, one entry per device. In host code the
// array names above are host-side stand-ins, not device addresses; only these may be
// handed to a kernel.
struct NoAllocSlot {
    void* scratch = nullptr;
    int32_t* counters = nullptr;
};
static NoAllocSlot g_noalloc_slots[128];
static std::mutex g_noalloc_mutex;

static int noalloc_setup(NoAllocSlot* out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return LSA_ERR_CUDA;
    if (dev < 0 || dev >= 128) return LSA_ERR_ARG;
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    NoAllocSlot& slot = g_noalloc_slots[dev];
    if (slot.scratch == nullptr) {  // first call on this device (the device is current)
        void* s = nullptr;
        void* c = nullptr;
        if (cudaGetSymbolAddress(&s, g_noalloc_scratch) != cudaSuccess) return LSA_ERR_CUDA;
        if (cudaGetSymbolAddress(&c, g_noalloc_counters) != cudaSuccess) return LSA_ERR_CUDA;
        slot.scratch = s;
        slot.counters = static_cast<int32_t*>(c);
    }
    *out = slot;
    return LSA_OK;
}

}  // namespace lsa

extern "C" {

// lsa_sparse_read without caller buffers. Limits: the plan's scratch must fit 8 MiB and
// its counters 65536, checked here against the plan this entry uses (no persistent grid);
// larger calls return LSA_ERR_SIZE and launch nothing. The first call on each device
// resolves the arrays' addresses (cudaGetSymbolAddress), so make it before any stream
// capture. Each call zeroes the counters it uses (cudaMemsetAsync) and then launches the
// read; calls share the arrays, so calls that overlap on the GPU (different streams, or
// devices sharing a context) race and must be serialised by the caller. The read's status
// word (0, or LSA_ERR_TIMEOUT after an expired bounded wait) lives in the shared counters
// and the next call's zeroing would erase it, so it is copied (cudaMemcpyAsync, 4 bytes,
// on `stream`) to the caller's `status` when one is given.
int lsa_sparse_read_noalloc(const void* q, const void* k, const void* v, int dtype, const int32_t* ids,
                            const int32_t* lengths, int64_t B, int64_t Tq, int64_t Tk, int64_t Hq, int64_t Hkv,
                            int64_t D, int64_t width, float scale, void* out, int64_t splits, int32_t* status,
                            cudaStream_t stream) {
    if (Hkv <= 0 || Hq % Hkv || width < 0 || D <= 0 || B < 0 || Tq < 0) return LSA_ERR_ARG;
    // the fixed arrays take the cluster / ticket plans only (the persistent plan's split
    // partials can outgrow them)
    lsa::ReadPlan p = lsa::plan_read(B * Tq, Hkv, Hq / Hkv, D, width, splits, lsa::num_sms(), false);
    if (p.scratch_bytes > lsa::kNoAllocScratchBytes || p.counters > lsa::kNoAllocCounters) return LSA_ERR_SIZE;
    lsa::NoAllocSlot slot;
    int rc = lsa::noalloc_setup(&slot);
    if (rc != LSA_OK) return rc;
    if (cudaMemsetAsync(slot.counters, 0, (size_t)p.counters * sizeof(int32_t), stream) != cudaSuccess)
        return LSA_ERR_CUDA;
    rc = lsa::sparse_read_launch(q, k, v, dtype, ids, lengths, B, Tq, Tk, Hq, Hkv, D, width, scale, out, slot.scratch,
                                 lsa::kNoAllocScratchBytes, slot.counters, lsa::kNoAllocCounters, splits, stream, 0,
                                 nullptr, nullptr, false);
    if (rc != LSA_OK || status == nullptr) return rc;
    // the status word of the launch: counters[rows * KV heads] (zeroed above, so 0 when the
    // kernel that ran keeps no status)
    const int32_t* word = slot.counters + B * Tq * Hkv;
    if (cudaMemcpyAsync(status, word, sizeof(int32_t), cudaMemcpyDefault, stream) != cudaSuccess) return LSA_ERR_CUDA;
    return LSA_OK;
}

}  // extern "C"
