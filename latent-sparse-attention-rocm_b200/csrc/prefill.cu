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
//   S_h  = Q_h K^T     tcgen05.mma kind::f16; Q, K in 128B-swizzled shared memory; S in TMEM
//   softmax            one thread per row: S row from TMEM, running max / sum (exp2 domain,
//                      the O rescale deferred until the max grows by more than 2^8),
//                      P row (q dtype) into swizzled shared memory
//   O_h += P_h V       tcgen05.mma with V as an MN-major operand; O in TMEM
// TMEM columns: S_0 [0,128), S_1 [128,256), O_0 [256,384), O_1 [384,512).
// Warp roles (12 warps): warp 0 issues the MMAs (one thread) and owns the TMEM allocation;
// warp 1 gathers K rows, warp 2 gathers V rows (cp.async, 16 B per lane, zero-fill for
// skipped ids); warp 3 loads Q; warps 4-7 / 8-11 run the softmax of half 0 / half 1.
// The S MMA of chunk j+1 is issued before the PV MMA of chunk j, so the tensor core works
// on one half while the softmax warps work on the other chunk.
//
// Every wait is bounded (1 s of %globaltimer, warp-uniform); a wait that expires raises a
// CTA-wide abort flag, every role leaves its loop, the MMA warp drains its MMAs before the
// TMEM is released, and LSA_ERR_TIMEOUT lands in the status word.
#include "common.cuh"
#include "umma.cuh"

namespace lsa {
namespace {

constexpr int kPfThreads = 384;
constexpr int kChunk = 128;                 // keys per step
constexpr int kTileBytes = 128 * 128 * 2;   // one 128 x 128 16-bit operand tile (two 16 KB blocks)
constexpr int kBlockBytes = 16384;          // one 64-column block of a tile
constexpr int kKStages = 2;
constexpr int kVStages = 1;
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + 2 * kTileBytes;
constexpr int kOffV = kOffK + kKStages * kTileBytes;
constexpr int kOffP = kOffV + kVStages * kTileBytes;
constexpr int kOffBar = kOffP + 2 * kTileBytes;

enum : int {
    kBarQ = 0,
    kBarKFull = 1,                         // kKStages
    kBarKEmpty = kBarKFull + kKStages,     // kKStages
    kBarVFull = kBarKEmpty + kKStages,     // kVStages
    kBarVEmpty = kBarVFull + kVStages,     // kVStages
    kBarSFull = kBarVEmpty + kVStages,     // 2 halves
    kBarSFree = kBarSFull + 2,             // 2
    kBarPFull = kBarSFree + 2,             // 2
    kBarPFree = kBarPFull + 2,             // 2
    kBarDrain = kBarPFree + 2,
    kNumBars = kBarDrain + 1
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

// Byte offset of 16-byte chunk c (0..15) of row r in a swizzled 128 x 128 tile.
__device__ __forceinline__ uint32_t swz(int r, int c) {
    return (uint32_t)((c >> 3) * kBlockBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// The softmax warpgroup of one half (warps 4-7: half 0, 8-11: half 1), one thread per row.
template <typename T, typename KeyId>
__device__ __forceinline__ void softmax_role(const PrefillArgs& a, uint32_t sbase, uint64_t* bars,
                                             volatile int* abort_flag, uint32_t tmem, const KeyId& key_id, int64_t t0,
                                             int64_t bs, int Lt, int nchunks) {
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
    const uint32_t prow = sbase + kOffP + h * kTileBytes;
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nchunks; ++j) {
        uint32_t vm[4];  // columns of this chunk with a readable key (lane l: column l + 32 m)
#pragma unroll
        for (int m = 0; m < 4; ++m) vm[m] = __ballot_sync(0xFFFFFFFFu, key_id(j * kChunk + lane + 32 * m) >= 0);
        ok = warp_wait(&bars[kBarSFull + h], j & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        uint32_t sr[128];
        tmem_ld64_wait<0>(tS, sr);
        tmem_ld64_wait<64>(tS + 64, sr);
        tc_fence_before();
        mbar_arrive(&bars[kBarSFree + h]);
        const int cmax = limit - j * kChunk;  // columns <= cmax pass the causal bound
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 128; ++c) {
            const bool live = ((vm[c >> 5] >> (c & 31)) & 1u) && c <= cmax;
            const float x = live ? __uint_as_float(sr[c]) * a.scale_log2 : -INFINITY;
            sr[c] = __float_as_uint(x);
            mx = fmaxf(mx, x);
        }
        const float m_new = fmaxf(m_used, mx);
        float alpha = 1.0f;
        const bool resc = m_new > m_used + 8.0f;
        if (resc) {
            alpha = exp2f(m_used - m_new);
            m_used = m_new;
        }
        const float ref = m_used == -INFINITY ? 0.0f : m_used;
        float sum = 0.0f;
#pragma unroll
        for (int c = 0; c < 128; ++c) {
            const float p = exp2f(__uint_as_float(sr[c]) - ref);
            sr[c] = __float_as_uint(p);
            sum += p;
        }
        l = l * alpha + sum;
        if (j > 0) {
            // PV of the previous chunk done: its P buffer is free and O is current
            ok = warp_wait(&bars[kBarPFree + h], (j - 1) & 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
        }
#pragma unroll
        for (int c16 = 0; c16 < 16; ++c16) {
            uint4 w;
            w.x = pack2(__uint_as_float(sr[8 * c16 + 0]), __uint_as_float(sr[8 * c16 + 1]), (T*)nullptr);
            w.y = pack2(__uint_as_float(sr[8 * c16 + 2]), __uint_as_float(sr[8 * c16 + 3]), (T*)nullptr);
            w.z = pack2(__uint_as_float(sr[8 * c16 + 4]), __uint_as_float(sr[8 * c16 + 5]), (T*)nullptr);
            w.w = pack2(__uint_as_float(sr[8 * c16 + 6]), __uint_as_float(sr[8 * c16 + 7]), (T*)nullptr);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(prow + swz(r, c16)), "r"(w.x),
                         "r"(w.y), "r"(w.z), "r"(w.w)
                         : "memory");
        }
        if (j > 0 && __any_sync(0xFFFFFFFFu, resc)) {
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
                uint32_t o[32];
                tmem_ld32_wait(tO + cc * 32, o);
#pragma unroll
                for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                tmem_st32(tO + cc * 32, o);
            }
            tmem_wait_st();
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bars[kBarPFull + h]);
    }
    if (ok && nchunks > 0) ok = warp_wait(&bars[kBarPFree + h], (nchunks - 1) & 1, abort_flag);
    if (ok && nchunks > 0) {
        tc_fence_after();
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        T* orow = static_cast<T*>(a.out) + (((int64_t)b * a.T + t) * a.Hq + (int64_t)kvh * a.G + g) * 128;
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
    } else if (live_row && nchunks == 0) {
        T* orow = static_cast<T*>(a.out) + (((int64_t)b * a.T + t) * a.Hq + (int64_t)kvh * a.G + g) * 128;
        for (int i = 0; i < 16; ++i) reinterpret_cast<uint4*>(orow)[i] = make_uint4(0, 0, 0, 0);
    }
}

template <typename T>
__global__ void __launch_bounds__(kPfThreads, 1) sparse_prefill_kernel(const PrefillArgs a) {
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
    const T* qg = static_cast<const T*>(a.q);
    const T* kg = static_cast<const T*>(a.k);
    const T* vg = static_cast<const T*>(a.v);

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
        mbar_init(&bars[kBarQ], 32);
        for (int s = 0; s < kKStages; ++s) {
            mbar_init(&bars[kBarKFull + s], 32);
            mbar_init(&bars[kBarKEmpty + s], 1);
        }
        for (int s = 0; s < kVStages; ++s) {
            mbar_init(&bars[kBarVFull + s], 32);
            mbar_init(&bars[kBarVEmpty + s], 1);
        }
        for (int h = 0; h < 2; ++h) {
            mbar_init(&bars[kBarSFull + h], 1);
            mbar_init(&bars[kBarSFree + h], 128);
            mbar_init(&bars[kBarPFull + h], 128);
            mbar_init(&bars[kBarPFree + h], 1);
        }
        mbar_init(&bars[kBarDrain], 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // register split (launch: 384 threads x 168): the loader/MMA warpgroup gives up
    // registers, the two softmax warpgroups take them: 128 x 96 + 256 x 192 <= 384 x 168
    if (warp >= 4) {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 192;" ::: "memory");
        softmax_role<T>(a, sbase, bars, abort_flag, tmem, key_id, t0, bs, Lt, nchunks);
    } else {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 96;" ::: "memory");
        if (warp == 0) {
            // ---------------------------------------------------------------- MMA issue
            constexpr uint32_t idS = umma_idesc_f16<T>(128, 128, false);
            constexpr uint32_t idPV = umma_idesc_f16<T>(128, 128, true);
            bool ok = warp_wait(&bars[kBarQ], 0, abort_flag);
            for (int j = 0; ok && j <= nchunks; ++j) {
                if (j < nchunks) {
                    const int s = j % kKStages;
                    ok = warp_wait(&bars[kBarKFull + s], (j / kKStages) & 1, abort_flag);
                    for (int h = 0; ok && h < 2; ++h) {
                        if (j > 0) ok = warp_wait(&bars[kBarSFree + h], (j - 1) & 1, abort_flag);
                        if (!ok) break;
                        if (lane == 0) {
                            fence_proxy_async_smem();
                            tc_fence_after();
                            const uint32_t qa = sbase + kOffQ + h * kTileBytes, ka = sbase + kOffK + s * kTileBytes;
#pragma unroll
                            for (int kk = 0; kk < 8; ++kk) {
                                const uint32_t off = (kk >> 2) * kBlockBytes + (kk & 3) * 32;
                                umma_f16_ss(tmem + h * 128, sw128_desc(qa + off, 16, 1024),
                                            sw128_desc(ka + off, 16, 1024), idS, kk > 0);
                            }
                            umma_commit(&bars[kBarSFull + h]);
                        }
                        __syncwarp();
                    }
                    if (!ok) break;
                    if (lane == 0) umma_commit(&bars[kBarKEmpty + s]);
                    __syncwarp();
                }
                if (j > 0) {
                    const int jj = j - 1, vs = jj % kVStages;
                    ok = warp_wait(&bars[kBarVFull + vs], (jj / kVStages) & 1, abort_flag);
                    for (int h = 0; ok && h < 2; ++h) {
                        ok = warp_wait(&bars[kBarPFull + h], jj & 1, abort_flag);
                        if (!ok) break;
                        if (lane == 0) {
                            fence_proxy_async_smem();
                            tc_fence_after();
                            const uint32_t pa = sbase + kOffP + h * kTileBytes, va = sbase + kOffV + vs * kTileBytes;
#pragma unroll
                            for (int kk = 0; kk < 8; ++kk) {
                                const uint32_t aoff = (kk >> 2) * kBlockBytes + (kk & 3) * 32;
                                umma_f16_ss(tmem + 256 + h * 128, sw128_desc(pa + aoff, 16, 1024),
                                            sw128_desc(va + kk * 2048, kBlockBytes, 1024), idPV, (jj > 0 || kk > 0));
                            }
                            umma_commit(&bars[kBarPFree + h]);
                        }
                        __syncwarp();
                    }
                    if (!ok) break;
                    if (lane == 0) umma_commit(&bars[kBarVEmpty + vs]);
                    __syncwarp();
                }
            }
            // every MMA issued so far completes before the TMEM is released
            if (lane == 0) umma_commit(&bars[kBarDrain]);
            __syncwarp();
            mbar_wait_bounded(&bars[kBarDrain], 0);
            __syncwarp();
        } else if (warp == 1 || warp == 2) {
            // ---------------------------------------------------------------- K / V gathers
            const bool isK = warp == 1;
            const T* src = isK ? kg : vg;
            const int stages = isK ? kKStages : kVStages;
            uint64_t* full = &bars[isK ? kBarKFull : kBarVFull];
            uint64_t* empty = &bars[isK ? kBarKEmpty : kBarVEmpty];
            const uint32_t base = sbase + (isK ? kOffK : kOffV);
            const int64_t row_stride = (int64_t)a.Hkv * 128;
            const T* src0 = src + ((int64_t)b * a.Tk * a.Hkv + kvh) * 128 + (lane & 15) * 8;
            for (int j = 0; j < nchunks; ++j) {
                const int s = j % stages;
                if (j >= stages && !warp_wait(&empty[s], (j / stages - 1) & 1, abort_flag)) break;
                const int i0 = j * kChunk + lane;
                const int id0 = key_id(i0), id1 = key_id(i0 + 32), id2 = key_id(i0 + 64), id3 = key_id(i0 + 96);
                const uint32_t dst0 = base + s * kTileBytes;
#pragma unroll 1
                for (int m = 0; m < 4; ++m) {
                    const int idm = m == 0 ? id0 : (m == 1 ? id1 : (m == 2 ? id2 : id3));
#pragma unroll 4
                    for (int i = 0; i < 16; ++i) {
                        const int row = 32 * m + 2 * i + (lane >> 4);
                        const int kid = __shfl_sync(0xFFFFFFFFu, idm, row & 31);
                        const T* g = src0 + (int64_t)(kid < 0 ? 0 : kid) * row_stride;
                        cp_async16(dst0 + swz(row, lane & 15), g, kid < 0 ? 0u : 16u);
                    }
                }
                cp_async_arrive_noinc(&full[s]);
            }
            cp_async_wait_all();
        } else if (warp == 3) {
            // ---------------------------------------------------------------- Q tile
#pragma unroll 2
            for (int it = 0; it < 128; ++it) {  // 256 rows x 16 chunks over 32 lanes
                const int lin = it * 32 + lane, row2 = lin >> 4, c = lin & 15;
                const int h = row2 >> 7, r = row2 & 127, g = r / a.QH, qi = r % a.QH;
                const int64_t t = t0 + h * a.QH + qi;
                const bool live = t < a.T;
                const T* src = qg + (((int64_t)b * a.T + (live ? t : 0)) * a.Hq + (int64_t)kvh * a.G + g) * 128 + c * 8;
                cp_async16(sbase + kOffQ + h * kTileBytes + swz(r, c), src, live ? 16u : 0u);
            }
            cp_async_arrive_noinc(&bars[kBarQ]);
            cp_async_wait_all();
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
    if (Tk > INT32_MAX || T > INT32_MAX || status == nullptr) return LSA_ERR_ARG;
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
