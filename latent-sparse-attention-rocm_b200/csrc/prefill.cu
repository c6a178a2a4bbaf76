// prefill.cu - the sparse prefill read on the 5th-generation tensor cores (sm_100a).
//
// The prefill arm reads, for every query row t, the list of its 64-query tile (the picked
// members of closed blocks, then the sinks: lsa_tile_select) followed by the row's own open
// block [block_start, t], causally. Read numerics follow the reference's sparse read
// (AIwork4me/latent-sparse-attention-rocm, src/lsa_rocm_lab/port/read_kernel_tiled.py:41-89):
// ids outside [0, Tk) among the first `length` entries are skipped, s = (q . k) * scale in
// fp32, softmax over the row's keys, o = sum p v / l, rows with no key read as zeros, the
// output has q's dtype.
//
// One CTA = one query tile x one KV head. Its rows are (query, q head of the KV head's
// group) pairs, split into two halves of 128 rows (M = 128 each); both halves read the same
// keys, so every K/V row the CTA gathers feeds 256 rows of tensor-core work. Per chunk of
// 128 keys of the CTA's list:
//   S_h  = Q_h K^T     tcgen05.mma kind::f16, Q and K in 128B-swizzled shared memory, S in TMEM
//   softmax            one thread per row: S row from TMEM, running max / sum (exp2 domain,
//                      the O rescale deferred until the max grows by more than 2^8); P is
//                      written back over S in TMEM (two 16-bit values per column)
//   O_h += P_h V       tcgen05.mma with A = P from TMEM and V as an MN-major smem operand
// TMEM columns: S_0/P_0 [0,128), S_1/P_1 [128,256), O_0 [256,384), O_1 [384,512).
// Rows reach shared memory by cp.async from six loader warps (16 B per copy into the
// 128B-swizzled layout): Q once, K and V per chunk into 3 + 2 stages. Many small copies in
// flight beat TMA row gathers here: a tile::gather4 moves 512 B and the copy engine takes
// roughly 75 cycles per gather, about 7 B/clk per SM.
// Each half has its own MMA issuing warp: S_h(j), then PV_h(j) in two parts as the half's
// softmax publishes P_h(j) for the first and the last 64 keys, then S_h(j+1). The two
// softmax warpgroups take turns (h0 chunk j, h1 chunk j, h0 chunk j+1, ...), so one half's
// exponentials run while the tensor pipe runs the other half's MMAs. tcgen05 operations of
// one thread run in order, so S_h(j+1) overwrites P_h(j) only after PV_h(j) has read it, and
// O_h is current whenever the softmax sees S_h(j+1). Two issuers because one thread issues
// one MMA per ~180 cycles (measured on B200: 128 x 128 x 16 MMAs from one thread reach half
// the pipe's rate, from two threads all of it).
// Warp roles (16 warps): warps 0 / 1 issue half 0's / half 1's MMAs (warp 0 also owns the
// TMEM allocation); warps 2-3 and 12-15 load Q, K and V; warps 4-7 / 8-11 run the softmax of
// half 0 / half 1.
//
// Every wait is bounded (1 s of %globaltimer, warp-uniform); a wait that expires raises a
// CTA-wide abort flag, every role leaves its loop, the MMA warp drains its MMAs and the
// loaders their copies before the TMEM is released, and LSA_ERR_TIMEOUT lands in the
// status word.
#include "common.cuh"
#include "umma.cuh"

namespace lsa {
namespace {

constexpr int kPfThreads = 512;
constexpr int kLoaders = 192;  // warps 2-3 and 12-15
constexpr int kChunk = 128;                // keys per step
constexpr int kTileBytes = 128 * 128 * 2;  // one 128 x 128 16-bit operand tile (two 16 KB blocks)
constexpr int kBlockBytes = 16384;         // one 64-column block of a tile
constexpr int kKStages = 3;
constexpr int kVStages = 2;
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + 2 * kTileBytes;
constexpr int kOffV = kOffK + kKStages * kTileBytes;
constexpr int kOffBar = kOffV + kVStages * kTileBytes;

enum : int {
    kBarQ = 0,
    kBarKFull = 1,                      // kKStages
    kBarKEmpty = kBarKFull + kKStages,  // kKStages
    kBarVFull = kBarKEmpty + kKStages,  // kVStages
    kBarVEmpty = kBarVFull + kVStages,  // kVStages
    kBarSFull = kBarVEmpty + kVStages,  // 2 halves
    kBarPFull = kBarSFull + 2,          // 4: (half, first / last 64 keys of P)
    kBarODone = kBarPFull + 4,          // 2 halves
    kBarDrain = kBarODone + 2,          // 2 issuers
    kBarTurn = kBarDrain + 2,           // 2: half h may run its exponentials
    kNumBars = kBarTurn + 2
};

constexpr int kOffMisc = kOffBar + kNumBars * 8;  // TMEM base (u32), abort flag (int)
constexpr int kSmemBytes = kOffMisc + 16 + 1024;  // + slack to align the base to 1024 B
static_assert(kSmemBytes <= 232448, "prefill shared memory exceeds the per-CTA limit");

constexpr uint64_t kWaitNs = 1000000000ull;

struct PrefillArgs {
    const void* q;
    const void* k;
    const void* v;
    const int32_t* lists;    // [B, tiles, ldl]
    const int32_t* lengths;  // [B, tiles]
    void* out;
    int64_t T, Tk, tiles, ldl;
    int Hq, Hkv, G, QH;  // G = Hq / Hkv; QH = 128 / G queries per half
    int tile, block;
    float scale_log2;
    int32_t* status;
};

// Warp-uniform bounded wait on an mbarrier phase. false: expired or another role aborted.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    bool done = mbar_try_wait(bar, parity);
    if (__all_sync(0xFFFFFFFFu, done)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (!done) done = mbar_try_wait(bar, parity);
        if (__all_sync(0xFFFFFFFFu, done)) return true;
        int stop = 0;
        if ((threadIdx.x & 31) == 0) stop = (*abort_flag != 0) || (global_ns() - t0 > kWaitNs);
        if (__shfl_sync(0xFFFFFFFFu, stop, 0)) {
            if ((threadIdx.x & 31) == 0) *abort_flag = 1;
            return false;
        }
    }
}

__device__ __forceinline__ uint32_t pack2(float a, float b, __nv_bfloat16*) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack2(float a, float b, __half*) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Packed fp32 pairs (sm_100): one instruction does the two lanes' fma / add with the
// rounding of the scalar instruction; a 3-input max.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Byte offset of 16-byte chunk c (0..15) of row r in a 128B-swizzled 128 x 128 tile.
__device__ __forceinline__ uint32_t swz(int r, int c) {
    return (uint32_t)((c >> 3) * kBlockBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// The softmax warpgroup of one half (warps 4-7: half 0, 8-11: half 1), one thread per row.
template <typename T, typename KeyId>
__device__ __forceinline__ void softmax_role(const PrefillArgs& a, uint64_t* bars, volatile int* abort_flag,
                                             uint32_t tmem, const KeyId& key_id, int64_t t0, int64_t bs, int Lt,
                                             int nchunks) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvh = blockIdx.x, b = blockIdx.z;
    const int h = (warp - 4) >> 2, qd = warp & 3, r = qd * 32 + lane;
    const int g = r / a.QH, qi = r % a.QH;
    const int64_t t = t0 + h * a.QH + qi;
    const bool live_row = t < a.T;
    const int limit = live_row ? Lt + (int)(t - bs) : -1;  // last list position this row reads
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t tS = tmem + lane_base + h * 128;
    const uint32_t tO = tmem + lane_base + 256 + h * 128;
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    // ids of the chunk about to be scored (lane l: columns l + 32 m), one chunk ahead
    int idn[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) idn[m] = key_id(lane + 32 * m);
    const float sl = a.scale_log2;
    const float thresh = 8.0f / sl;  // defer the O rescale until the max grows by 2^8
    for (int j = 0; j < nchunks; ++j) {
        uint32_t vm[4];  // columns of this chunk with a readable key
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            vm[m] = __ballot_sync(0xFFFFFFFFu, idn[m] >= 0);
            idn[m] = key_id((j + 1) * kChunk + lane + 32 * m);
        }
        // the halves take turns (h0 chunk j, h1 chunk j, h0 chunk j+1, ...): each turn has the
        // SM's exponential units to itself while the tensor pipe runs the other half's MMAs
        if (h == 1 || j > 0) ok = warp_wait(&bars[kBarTurn + h], (h == 1 ? j : j - 1) & 1, abort_flag);
        if (ok) ok = warp_wait(&bars[kBarSFull + h], j & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        uint32_t sr[128];
        tmem_ld64_wait<0>(tS, sr);
        tmem_ld64_wait<64>(tS + 64, sr);
        const int cmax = limit - j * kChunk;  // columns <= cmax pass the causal bound
        const bool full = (vm[0] & vm[1] & vm[2] & vm[3]) == 0xFFFFFFFFu && cmax >= kChunk - 1;
        if (!__all_sync(0xFFFFFFFFu, full)) {
#pragma unroll
            for (int c = 0; c < 128; ++c) {
                const bool live = ((vm[c >> 5] >> (c & 31)) & 1u) && c <= cmax;
                if (!live) sr[c] = 0xFF800000u;  // -inf
            }
        }
        // row max by 3-input max (4 independent chains over the 128 columns)
        float mx4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) mx4[i] = fmaxf(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1]));
#pragma unroll
        for (int c = 8; c < 128; c += 8)
#pragma unroll
            for (int i = 0; i < 4; ++i)
                mx4[i] = max3f(mx4[i], __uint_as_float(sr[c + 2 * i]), __uint_as_float(sr[c + 2 * i + 1]));
        const float mx = max3f(mx4[0], mx4[1], fmaxf(mx4[2], mx4[3]));
        const float m_new = fmaxf(m_used, mx);
        float alpha = 1.0f;
        const bool resc = m_new > m_used + thresh;
        if (resc) {
            alpha = ex2_approx((m_used - m_new) * sl);
            m_used = m_new;
        }
        const float neg = m_used == -INFINITY ? 0.0f : -m_used * sl;
        // exponents two columns at a time: one packed FMA (fma.rn.f32x2, the same rounding as
        // two fmaf) forms (s sl - m sl) for a column pair, one packed add accumulates the pair
        const uint64_t sl2 = f2_pack(sl, sl), neg2 = f2_pack(neg, neg);
        uint64_t sum2[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) sum2[i] = 0ull;
#pragma unroll
        for (int half = 0; half < 2; ++half) {  // P columns [32 half, 32 half + 32) = keys 64 half ..
            uint32_t pk[32];
#pragma unroll
            for (int c2 = 0; c2 < 32; ++c2) {
                const int c = 64 * half + 2 * c2;
                float x0, x1;
                f2_unpack(ffma2(f2_pack(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), sl2, neg2), x0, x1);
                const float p0 = ex2_approx(x0);
                const float p1 = ex2_approx(x1);
                sum2[c2 & 3] = fadd2(sum2[c2 & 3], f2_pack(p0, p1));
                pk[c2] = pack2(p0, p1, (T*)nullptr);
            }
            // O_h is current here (PV_h(j-1) was issued before S_h(j) and tcgen05 runs in
            // order); its rescale lands before any P of this chunk is published, since PV_h(j)
            // starts on the first 64 keys' P while the last 64 are still being computed
            if (half == 0 && j > 0 && __any_sync(0xFFFFFFFFu, resc)) {
#pragma unroll 1
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t o[32];
                    tmem_ld32_wait(tO + cc * 32, o);
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(tO + cc * 32, o);
                }
            }
            tmem_st32(tS + 32 * half, pk);  // P_h over S_h's first 64 columns
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bars[kBarPFull + 2 * h + half]);  // keys [64 half, 64 half + 64) of P_h
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kBarTurn + (1 - h)]);
        float sm8[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) f2_unpack(sum2[i], sm8[2 * i], sm8[2 * i + 1]);
        l = l * alpha + (((sm8[0] + sm8[1]) + (sm8[2] + sm8[3])) + ((sm8[4] + sm8[5]) + (sm8[6] + sm8[7])));
    }
    if (ok && nchunks > 0) ok = warp_wait(&bars[kBarODone + h], 0, abort_flag);
    T* orow = static_cast<T*>(a.out) + (((int64_t)b * a.T + t) * a.Hq + (int64_t)kvh * a.G + g) * 128;
    if (ok && nchunks > 0) {
        tc_fence_after();
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
            uint32_t o[32];
            tmem_ld32_wait(tO + cc * 32, o);
            if (live_row) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    uint4 w;
                    w.x = pack2(__uint_as_float(o[8 * i + 0]) * inv, __uint_as_float(o[8 * i + 1]) * inv, (T*)nullptr);
                    w.y = pack2(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv, (T*)nullptr);
                    w.z = pack2(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv, (T*)nullptr);
                    w.w = pack2(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv, (T*)nullptr);
                    *reinterpret_cast<uint4*>(orow + cc * 32 + i * 8) = w;
                }
            }
        }
    } else if (ok && live_row) {
        for (int i = 0; i < 16; ++i) reinterpret_cast<uint4*>(orow)[i] = make_uint4(0, 0, 0, 0);
    }
}

template <typename T>
__global__ void __launch_bounds__(kPfThreads, 1)
    sparse_prefill_kernel(const PrefillArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(sm);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffMisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + kOffMisc + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvh = blockIdx.x, b = blockIdx.z;
    const int QC = 2 * a.QH;
    const int64_t t0 = (int64_t)(gridDim.y - 1 - blockIdx.y) * QC;  // the longest lists first
    const int64_t tile = t0 / a.tile;
    const int64_t bs = t0 / a.block * a.block;
    const int32_t* list = a.lists + ((int64_t)b * a.tiles + tile) * a.ldl;
    int Lt = a.lengths[(int64_t)b * a.tiles + tile];
    Lt = Lt < 0 ? 0 : (Lt > a.ldl ? (int)a.ldl : Lt);
    const int64_t tend = t0 + QC < a.T ? t0 + QC : a.T;
    const int L = Lt + (int)(tend - bs);  // list, then the open block [bs, tend)
    const int nchunks = (L + kChunk - 1) / kChunk;

    // key row of list position i (-1: skipped)
    auto key_id = [&](int i) -> int {
        if (i >= L) return -1;
        if (i < Lt) {
            int id = __ldg(list + i);
            return (unsigned)id < (unsigned)a.Tk ? id : -1;
        }
        return (int)(bs + (i - Lt));
    };

    if (threadIdx.x == 0) {
        mbar_init(&bars[kBarQ], kLoaders);
        for (int s = 0; s < kKStages; ++s) {
            mbar_init(&bars[kBarKFull + s], kLoaders);
            mbar_init(&bars[kBarKEmpty + s], 2);  // a commit from each half's issuer
        }
        for (int s = 0; s < kVStages; ++s) {
            mbar_init(&bars[kBarVFull + s], kLoaders);
            mbar_init(&bars[kBarVEmpty + s], 2);
        }
        for (int h = 0; h < 2; ++h) {
            mbar_init(&bars[kBarSFull + h], 1);
            mbar_init(&bars[kBarPFull + 2 * h], 128);
            mbar_init(&bars[kBarPFull + 2 * h + 1], 128);
        }
        for (int h = 0; h < 2; ++h) {
            mbar_init(&bars[kBarODone + h], 1);
            mbar_init(&bars[kBarDrain + h], 1);
            mbar_init(&bars[kBarTurn + h], 4);  // one arrival per warp of the other half
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // register split (launch: 512 threads x 128): the MMA/loader warpgroups (0 and 3) give
    // up registers, the two softmax warpgroups take them: 256 x 80 + 256 x 176 = 512 x 128
    if (warp >= 4 && warp < 12) {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 176;" ::: "memory");
        softmax_role<T>(a, bars, abort_flag, tmem, key_id, t0, bs, Lt, nchunks);
    } else {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 80;" ::: "memory");
        if (warp < 2) {
            // ------------------------------------------------------------ MMA issue, warp h: half h
            // One issuing thread sustains one tcgen05.mma per ~180 cycles (measured on B200), about
            // half the tensor pipe's rate at N = 128; the two halves' issuers together keep it full.
            const int h = warp;
            constexpr uint32_t idS = umma_idesc_f16<T>(128, 128, false);
            constexpr uint32_t idPV = umma_idesc_f16<T>(128, 128, true);
            auto issue_s = [&](int j) {  // S_h(j) = Q_h K_j^T; K_j's stage is free once both halves' S are
                if (lane == 0) {
                    fence_proxy_async_smem();  // cp.async (generic proxy) data -> MMA (async proxy)
                    const uint32_t qa = sbase + kOffQ + h * kTileBytes;
                    const uint32_t ka = sbase + kOffK + (j % kKStages) * kTileBytes;
#pragma unroll 1
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t off = (kk >> 2) * kBlockBytes + (kk & 3) * 32;
                        umma_f16_ss(tmem + h * 128, sw128_desc(qa + off, 16, 1024), sw128_desc(ka + off, 16, 1024),
                                    idS, kk > 0);
                    }
                    umma_commit(&bars[kBarSFull + h]);
                    umma_commit(&bars[kBarKEmpty + j % kKStages]);
                }
                __syncwarp();
            };
            auto issue_pv = [&](int j, int part) {  // O_h += P_h(j) V_j over keys [64 part, 64 part + 64)
                if (lane == 0) {
                    fence_proxy_async_smem();
                    const uint32_t va = sbase + kOffV + (j % kVStages) * kTileBytes;
#pragma unroll 1
                    for (int kk = 4 * part; kk < 4 * part + 4; ++kk)
                        umma_f16_ts(tmem + 256 + h * 128, tmem + h * 128 + kk * 8,
                                    sw128_desc(va + kk * 2048, kBlockBytes, 1024), idPV, (j > 0 || kk > 0));
                    if (part == 1) umma_commit(&bars[kBarVEmpty + j % kVStages]);
                }
                __syncwarp();
            };
            auto commit_to = [&](uint64_t* bar) {
                if (lane == 0) umma_commit(bar);
                __syncwarp();
            };
            // per half, in issue order: S_h(j), then PV_h(j) once the softmax has written P_h(j);
            // S_h(j + 1) overwrites P_h(j) only after PV_h(j) read it (one thread's tcgen05
            // operations run in order)
            bool ok = warp_wait(&bars[kBarQ], 0, abort_flag);
            for (int j = 0; ok && j < nchunks; ++j) {
                ok = warp_wait(&bars[kBarKFull + j % kKStages], (j / kKStages) & 1, abort_flag);
                if (!ok) break;
                tc_fence_after();
                issue_s(j);
                ok = warp_wait(&bars[kBarVFull + j % kVStages], (j / kVStages) & 1, abort_flag);
                if (ok) ok = warp_wait(&bars[kBarPFull + 2 * h], j & 1, abort_flag);
                if (!ok) break;
                tc_fence_after();
                issue_pv(j, 0);
                ok = warp_wait(&bars[kBarPFull + 2 * h + 1], j & 1, abort_flag);
                if (!ok) break;
                tc_fence_after();
                issue_pv(j, 1);
            }
            if (ok && nchunks > 0) commit_to(&bars[kBarODone + h]);
            // every MMA this warp issued completes before the TMEM is released
            commit_to(&bars[kBarDrain + h]);
            mbar_wait_bounded(&bars[kBarDrain + h], 0);
            __syncwarp();
        } else {
            // ------------------------------------------------------------ loads (warps 2-3, 12-15)
            // 192 threads, 16 B per cp.async, 128B-swizzled destinations: Q once, then K_j and
            // V_j per chunk into their stages (skipped ids zero-fill their rows: masked anyway)
            const int lt = (warp < 4 ? warp - 2 : warp - 10) * 32 + lane;
            const T* qg = static_cast<const T*>(a.q);
            for (int lin = lt; lin < 4096; lin += kLoaders) {  // 256 rows x 16 chunks
                const int row2 = lin >> 4, c = lin & 15, h = row2 >> 7, r = row2 & 127, g = r / a.QH, qi = r % a.QH;
                const int64_t t = t0 + h * a.QH + qi;
                const bool live = t < a.T;
                const T* src = qg + (((int64_t)b * a.T + (live ? t : 0)) * a.Hq + (int64_t)kvh * a.G + g) * 128 + c * 8;
                cp_async16(sbase + kOffQ + h * kTileBytes + swz(r, c), src, live ? 16u : 0u);
            }
            cp_async_arrive_noinc(&bars[kBarQ]);
            const int64_t row_stride = (int64_t)a.Hkv * 128;
            const T* k0 = static_cast<const T*>(a.k) + ((int64_t)b * a.Tk * a.Hkv + kvh) * 128;
            const T* v0 = static_cast<const T*>(a.v) + ((int64_t)b * a.Tk * a.Hkv + kvh) * 128;
            // copy `it` of a thread: 16-byte chunk (lt + 224 it) & 15 of row (lt + 224 it) >> 4; the
            // rows' ids (shared by K_j and V_j) load into registers before the stage waits
            constexpr int kCopies = (2048 + kLoaders - 1) / kLoaders;
            int idr[kCopies];
            auto load_ids = [&](int j) {
#pragma unroll
                for (int it = 0; it < kCopies; ++it) {
                    const int lin = lt + kLoaders * it;
                    idr[it] = lin < 2048 ? key_id(j * kChunk + (lin >> 4)) : -1;
                }
            };
            auto issue = [&](uint32_t dst, const T* src0) {
#pragma unroll
                for (int it = 0; it < kCopies; ++it) {
                    const int lin = lt + kLoaders * it;
                    if (lin < 2048) {
                        const int row = lin >> 4, c = lin & 15, id = idr[it];
                        cp_async16(dst + swz(row, c), src0 + (int64_t)(id < 0 ? 0 : id) * row_stride + c * 8,
                                   id < 0 ? 0u : 16u);
                    }
                }
            };
            if (nchunks > 0) load_ids(0);
            for (int j = 0; j < nchunks; ++j) {
                const int sk = j % kKStages, sv = j % kVStages;
                if (j >= kKStages && !warp_wait(&bars[kBarKEmpty + sk], (j / kKStages - 1) & 1, abort_flag)) break;
                issue(sbase + kOffK + sk * kTileBytes, k0);
                cp_async_arrive_noinc(&bars[kBarKFull + sk]);
                if (j >= kVStages && !warp_wait(&bars[kBarVEmpty + sv], (j / kVStages - 1) & 1, abort_flag)) break;
                issue(sbase + kOffV + sv * kTileBytes, v0);
                cp_async_arrive_noinc(&bars[kBarVFull + sv]);
                if (j + 1 < nchunks) load_ids(j + 1);
            }
            cp_async_wait_all();
            __syncwarp();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
    if (threadIdx.x == 0 && *abort_flag) atomicExch(a.status, LSA_ERR_TIMEOUT);
}

template <typename T>
int launch_prefill(const PrefillArgs& a, int64_t B, cudaStream_t stream) {
    auto kern = sparse_prefill_kernel<T>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess)
        return LSA_ERR_CUDA;
    const int QC = 2 * a.QH;
    dim3 grid((unsigned)a.Hkv, (unsigned)((a.T + QC - 1) / QC), (unsigned)B);
    kern<<<grid, kPfThreads, kSmemBytes, stream>>>(a);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

}  // namespace
}  // namespace lsa

using namespace lsa;

extern "C" {

int lsa_sparse_prefill(const void* q, const void* k, const void* v, int dtype, const int32_t* tile_lists,
                       const int32_t* tile_lengths, int64_t ldl, int64_t B, int64_t T, int64_t Tk, int64_t Hq,
                       int64_t Hkv, int64_t D, int64_t tile, int64_t block, float scale, void* out, int32_t* status,
                       cudaStream_t stream) {
    if (B < 0 || T < 0 || D != 128 || Hkv <= 0 || Hq % Hkv || Tk < T || ldl < 0 || tile <= 0 || block <= 0)
        return LSA_ERR_ARG;
    const int64_t G = Hq / Hkv;
    if (G != 4 && G != 8 && G != 16) return LSA_ERR_ARG;
    const int64_t QH = 128 / G;
    if (tile % (2 * QH) || block % tile) return LSA_ERR_ARG;
    if (status == nullptr || Tk > INT32_MAX) return LSA_ERR_ARG;
    auto al16 = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
    if (!al16(q) || !al16(k) || !al16(v) || !al16(out)) return LSA_ERR_ARG;
    if (B == 0 || T == 0) return LSA_OK;
    PrefillArgs a;
    a.q = q;
    a.k = k;
    a.v = v;
    a.lists = tile_lists;
    a.lengths = tile_lengths;
    a.out = out;
    a.T = T;
    a.Tk = Tk;
    a.tiles = (T + tile - 1) / tile;
    a.ldl = ldl;
    a.Hq = (int)Hq;
    a.Hkv = (int)Hkv;
    a.G = (int)G;
    a.QH = (int)QH;
    a.tile = (int)tile;
    a.block = (int)block;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.status = status;
    if (dtype == kBF16) return launch_prefill<__nv_bfloat16>(a, B, stream);
    if (dtype == kF16) return launch_prefill<__half>(a, B, stream);
    return LSA_ERR_ARG;
}

}  // extern "C"
