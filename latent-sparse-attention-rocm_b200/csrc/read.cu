// read.cu - gather attention over each row's read list (sm_100a).
//
// Reference semantics (AIwork4me/latent-sparse-attention-rocm,
// src/lsa_rocm_lab/port/read_kernel_tiled.py:41-89): for row r and query head h (KV head
// h / (Hq / Hkv)), the ids >= 0 among the first min(length, width) slots are read;
// s = (q . k) * scale in fp32; fp32 online softmax from a finite -3e38 running max;
// o = sum p v / l; a row with no listed key gives zeros; duplicates count per occurrence;
// the output takes q's dtype.
//
// B200 design: split-K flash decoding. One CTA per (row, KV head, split) serves all G
// query heads of the KV head, so each gathered K/V row is read from HBM once for the
// group. The CTA's ids are fetched in stages of 64: warp 0 issues one cp.async.bulk
// (TMA bulk copy) per listed K row and per V row straight into shared memory, completion
// tracked by an mbarrier (expect_tx bytes), two stages in flight. Each 16-byte lane vector
// carries 8 elements of a row. Partial (m, l, o) per split go to a workspace; the last CTA
// of a (row, KV head) - atomic ticket - merges them. With one split the CTA writes the
// output directly. Every mbarrier wait is bounded (2 s of %globaltimer): on expiry the
// CTA records LSA_ERR_TIMEOUT in the workspace status word and leaves.
#include <mutex>

#include "common.cuh"

namespace lsa {

constexpr int kStageIds = 64;      // ids per pipeline stage
constexpr int kReadThreads = 128;  // 4 warps
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegBig = -3.0e38f;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx_arrive(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
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

// Bounded wait: true when the phase completed, false after ~2 s.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > 2000000000ull) return false;
    }
    return true;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

struct ReadArgs {
    const void* q;
    const void* k;
    const void* v;
    const int32_t* ids;
    const int32_t* lengths;
    void* out;
    float* part_o;   // [R*Hkv, splits, G, D]
    float* part_ml;  // [R*Hkv, splits, G, 2]
    int32_t* tickets;
    int32_t* status;
    int64_t Tq, Tk;
    int Hq, Hkv, G, width, splits, span;
    float scale_log2;  // scale * log2(e)
};

template <typename T, int D, int GMAX>
__global__ void __launch_bounds__(kReadThreads) sparse_read_kernel(ReadArgs a) {
    constexpr int LPR = D / 8;         // lanes per key row (8 elements per lane)
    constexpr int GPW = 32 / LPR;      // key rows per warp step
    constexpr int NG = 4 * GPW;        // row groups in the CTA
    constexpr int ROWB = D * sizeof(T);
    constexpr int STAGE_BYTES = kStageIds * ROWB;
    extern __shared__ __align__(128) unsigned char smem[];
    T* sK = reinterpret_cast<T*>(smem);                      // [2][kStageIds][D]
    T* sV = reinterpret_cast<T*>(smem + 2 * STAGE_BYTES);    // [2][kStageIds][D]
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ int is_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = warp * GPW + lane / LPR;  // row group of this lane
    const int lg = lane % LPR;                // lane within the group
    const int rh = blockIdx.x / a.splits;     // row * Hkv + kv head
    const int split = blockIdx.x % a.splits;
    const int64_t row = rh / a.Hkv;
    const int h = rh % a.Hkv;
    const int64_t b = row / a.Tq;
    const int G = a.G;

    int len = a.lengths[row];
    len = len < 0 ? 0 : (len > a.width ? a.width : len);
    const int s0 = split * a.span;
    const int s1 = min(s0 + a.span, len);
    const int n_ids = s1 > s0 ? s1 - s0 : 0;
    const int n_stages = (n_ids + kStageIds - 1) / kStageIds;
    const int32_t* idrow = a.ids + row * a.width;
    const T* kbase = reinterpret_cast<const T*>(a.k) + (b * a.Tk * a.Hkv + h) * D;
    const T* vbase = reinterpret_cast<const T*>(a.v) + (b * a.Tk * a.Hkv + h) * D;
    const int64_t tstride = (int64_t)a.Hkv * D;  // elements between consecutive positions

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    // warp 0 issues one stage: bulk copies of every listed K and V row of the stage
    auto issue = [&](int stage) {
        int buf = stage & 1;
        int base = s0 + stage * kStageIds;
        int cnt = min(kStageIds, s1 - base);
        int idv[2];
        bool ok[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            int j = lane + 32 * u;
            idv[u] = j < cnt ? idrow[base + j] : -1;
            ok[u] = idv[u] >= 0 && idv[u] < a.Tk;
        }
        uint32_t n = __popc(__ballot_sync(0xFFFFFFFFu, ok[0])) + __popc(__ballot_sync(0xFFFFFFFFu, ok[1]));
        if (lane == 0) mbar_expect_tx_arrive(&bars[buf], n * 2u * ROWB);
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (ok[u]) {
                int j = lane + 32 * u;
                bulk_g2s(sK + ((size_t)buf * kStageIds + j) * D, kbase + (int64_t)idv[u] * tstride, ROWB, &bars[buf]);
                bulk_g2s(sV + ((size_t)buf * kStageIds + j) * D, vbase + (int64_t)idv[u] * tstride, ROWB, &bars[buf]);
            }
        }
    };

    if (warp == 0) {
        if (n_stages > 0) issue(0);
        if (n_stages > 1) issue(1);
    }

    // q of the group's heads, this lane's 8 dims, pre-scaled into the log2 domain
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

    bool failed = false;
    for (int st = 0; st < n_stages; ++st) {
        int buf = st & 1;
        bool ok = mbar_wait_bounded(&bars[buf], (st >> 1) & 1);
        if (__syncthreads_or(!ok)) {  // block-uniform: every thread leaves together
            // give copies still in flight a second bounded window before the CTA exits
            if (tid == 0) mbar_wait_bounded(&bars[buf], (st >> 1) & 1);
            __syncthreads();
            failed = true;
            break;
        }
        int base = s0 + st * kStageIds;
        int cnt = min(kStageIds, s1 - base);
        constexpr int PER = kStageIds / NG;  // slots of this group in the stage
        float s[PER][GMAX];
        bool kept[PER];
#pragma unroll
        for (int u = 0; u < PER; ++u) {
            int j = grp + NG * u;
            int id = j < cnt ? idrow[base + j] : -1;
            kept[u] = id >= 0 && id < a.Tk;
#pragma unroll
            for (int g = 0; g < GMAX; ++g) s[u][g] = kNegBig;
            if (kept[u]) {
                float kv[8];
                load8<T>(sK + ((size_t)buf * kStageIds + j) * D + lg * 8, kv);
#pragma unroll
                for (int g = 0; g < GMAX; ++g) {
                    float p = 0.0f;
#pragma unroll
                    for (int e = 0; e < 8; ++e) p = fmaf(qr[g][e], kv[e], p);
                    s[u][g] = p;
                }
            }
        }
        // reduce the partial dots across the LPR lanes of each group
#pragma unroll
        for (int u = 0; u < PER; ++u)
#pragma unroll
            for (int g = 0; g < GMAX; ++g)
#pragma unroll
                for (int off = LPR / 2; off >= 1; off >>= 1) s[u][g] += __shfl_xor_sync(0xFFFFFFFFu, s[u][g], off);
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
            load8<T>(sV + ((size_t)buf * kStageIds + j) * D + lg * 8, vv);
#pragma unroll
            for (int g = 0; g < GMAX; ++g) {
                float p = exp2f(s[u][g] - m[g]);
                l[g] += p;
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(p, vv[e], acc[g][e]);
            }
        }
        __syncthreads();  // every group is done with this buffer
        if (warp == 0 && st + 2 < n_stages) issue(st + 2);
    }
    if (failed) {
        if (lane == 0) atomicExch(a.status, LSA_ERR_TIMEOUT);
        return;
    }

    // merge the NG row groups of the CTA (stage buffers are free now)
    float* red = reinterpret_cast<float*>(smem);  // [NG][GMAX][D] then m,l [NG][GMAX][2]
    float* redml = red + NG * GMAX * D;
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
#pragma unroll
        for (int e = 0; e < 8; ++e) red[(grp * GMAX + g) * D + lg * 8 + e] = acc[g][e];
        if (lg == 0) {
            redml[(grp * GMAX + g) * 2] = m[g];
            redml[(grp * GMAX + g) * 2 + 1] = l[g];
        }
    }
    __syncthreads();
    const bool single = a.splits == 1;
    for (int o = tid; o < G * D; o += kReadThreads) {
        int g = o / D, e = o % D;
        float M = kNegBig;
        for (int r = 0; r < NG; ++r) M = fmaxf(M, redml[(r * GMAX + g) * 2]);
        float L = 0.0f, O = 0.0f;
        for (int r = 0; r < NG; ++r) {
            float f = exp2f(redml[(r * GMAX + g) * 2] - M);
            L += redml[(r * GMAX + g) * 2 + 1] * f;
            O += red[(r * GMAX + g) * D + e] * f;
        }
        if (single) {
            float val = L > 0.0f ? O / L : 0.0f;
            reinterpret_cast<T*>(a.out)[((row * a.Hq) + h * G + g) * D + e] = from_f32<T>(val);
        } else {
            int64_t pidx = ((int64_t)rh * a.splits + split) * G + g;
            a.part_o[pidx * D + e] = O;
            if (e == 0) {
                a.part_ml[pidx * 2] = M;
                a.part_ml[pidx * 2 + 1] = L;
            }
        }
    }
    if (single) return;

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
    for (int o = tid; o < G * D; o += kReadThreads) {
        int g = o / D, e = o % D;
        float M = kNegBig;
        for (int sp = 0; sp < a.splits; ++sp)
            M = fmaxf(M, __ldcg(a.part_ml + (((int64_t)rh * a.splits + sp) * G + g) * 2));
        float L = 0.0f, O = 0.0f;
        for (int sp = 0; sp < a.splits; ++sp) {
            int64_t pidx = ((int64_t)rh * a.splits + sp) * G + g;
            float f = exp2f(__ldcg(a.part_ml + pidx * 2) - M);
            L += __ldcg(a.part_ml + pidx * 2 + 1) * f;
            O += __ldcg(a.part_o + pidx * D + e) * f;
        }
        float val = L > 0.0f ? O / L : 0.0f;
        reinterpret_cast<T*>(a.out)[((row * a.Hq) + h * G + g) * D + e] = from_f32<T>(val);
    }
}

struct ReadPlan {
    int splits, span;
    int64_t part_o_bytes, part_ml_bytes, scratch_bytes, counters;
};

static int num_sms() {
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

static int64_t round256(int64_t x) { return (x + 255) / 256 * 256; }

// splits: CTAs per (row, KV head). Auto (splits_req <= 0): enough CTAs for two per SM,
// at most one split per 16 ids of the width.
static ReadPlan plan_read(int64_t R, int64_t Hkv, int64_t G, int64_t D, int64_t width, int64_t splits_req, int sms) {
    ReadPlan p;
    int64_t units = R * Hkv;
    int64_t max_splits = (width + 15) / 16;
    if (max_splits < 1) max_splits = 1;
    int64_t s = splits_req;
    if (s <= 0) {
        int64_t target = 2 * (int64_t)sms;
        s = (target + units - 1) / (units > 0 ? units : 1);
    }
    if (s > max_splits) s = max_splits;
    if (s < 1) s = 1;
    p.splits = (int)s;
    p.span = (int)((width + s - 1) / s);
    p.part_o_bytes = s > 1 ? round256(units * s * G * D * 4) : 0;
    p.part_ml_bytes = s > 1 ? round256(units * s * G * 2 * 4) : 0;
    p.scratch_bytes = p.part_o_bytes + p.part_ml_bytes;
    p.counters = units + 1;  // one ticket per (row, KV head) + the status word
    return p;
}

template <typename T, int D, int GMAX>
static int launch_read(const ReadArgs& a, int64_t ctas, cudaStream_t st) {
    constexpr int smem = 4 * kStageIds * D * (int)sizeof(T);
    auto kern = sparse_read_kernel<T, D, GMAX>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return LSA_ERR_CUDA;
    kern<<<(unsigned)ctas, kReadThreads, smem, st>>>(a);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
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
                       int64_t n_counters, int64_t splits, cudaStream_t stream) {
    if (B < 0 || Tq < 0 || Tk < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || width < 0) return LSA_ERR_ARG;
    if (D != 64 && D != 128) return LSA_ERR_ARG;
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out | (uintptr_t)scratch) & 15) return LSA_ERR_ARG;
    int64_t R = B * Tq;
    if (R == 0) return LSA_OK;
    int64_t G = Hq / Hkv;
    if (G > 8) return LSA_ERR_ARG;
    ReadPlan p = plan_read(R, Hkv, G, D, width, splits, num_sms());
    if (scratch_bytes < p.scratch_bytes || n_counters < p.counters || !counters) return LSA_ERR_ARG;
    char* w = (char*)scratch;
    ReadArgs a;
    a.q = q; a.k = k; a.v = v; a.ids = ids; a.lengths = lengths; a.out = out;
    a.part_o = (float*)w;
    a.part_ml = (float*)(w + p.part_o_bytes);
    a.tickets = counters;
    a.status = counters + R * Hkv;
    a.Tq = Tq; a.Tk = Tk;
    a.Hq = (int)Hq; a.Hkv = (int)Hkv; a.G = (int)G; a.width = (int)width;
    a.splits = p.splits; a.span = p.span;
    a.scale_log2 = scale * kLog2e;
    int64_t ctas = R * Hkv * p.splits;
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
// its counters 65536 (lsa_sparse_read_plan reports both); larger calls return
// LSA_ERR_SIZE and launch nothing. The first call on each device resolves the arrays'
// addresses (cudaGetSymbolAddress), so make it before any stream capture. Each call
// zeroes the counters it uses (cudaMemsetAsync) and then launches the read; calls share
// the arrays, so calls that overlap on the GPU (different streams, or devices sharing a
// context) race and must be serialised by the caller.
int lsa_sparse_read_noalloc(const void* q, const void* k, const void* v, int dtype, const int32_t* ids,
                            const int32_t* lengths, int64_t B, int64_t Tq, int64_t Tk, int64_t Hq, int64_t Hkv,
                            int64_t D, int64_t width, float scale, void* out, int64_t splits, cudaStream_t stream) {
    if (Hkv <= 0 || Hq % Hkv || width < 0 || D <= 0) return LSA_ERR_ARG;
    lsa::ReadPlan p = lsa::plan_read(B * Tq, Hkv, Hq / Hkv, D, width, splits, lsa::num_sms());
    if (p.scratch_bytes > lsa::kNoAllocScratchBytes || p.counters > lsa::kNoAllocCounters) return LSA_ERR_SIZE;
    lsa::NoAllocSlot slot;
    int rc = lsa::noalloc_setup(&slot);
    if (rc != LSA_OK) return rc;
    if (cudaMemsetAsync(slot.counters, 0, (size_t)p.counters * sizeof(int32_t), stream) != cudaSuccess)
        return LSA_ERR_CUDA;
    return lsa::sparse_read_launch(q, k, v, dtype, ids, lengths, B, Tq, Tk, Hq, Hkv, D, width, scale, out,
                                   slot.scratch, lsa::kNoAllocScratchBytes, slot.counters, lsa::kNoAllocCounters,
                                   splits, stream);
}

}  // extern "C"
