// peer.cu - an all-gather over peer memory for the sharded decode steps' small exchanges.
//
// Every rank owns one arena (cudaMalloc, shared by CUDA IPC handle); each rank maps every
// peer's arena, so a kernel on this GPU stores straight into a peer's memory over NVLink. A
// channel (one per message size) is a region of every arena: world uint32 flags, then two
// receive buffers of world x bytes (the parity of the gather's epoch picks one).
//
// One gather = two launches on the caller's stream:
//   push: every CTA copies its share of this rank's chunk into slot `rank` of every rank's
//         receive buffer (16-byte stores, peers' memory included), fences at system scope and
//         takes a ticket; the last CTA publishes epoch e in flag `rank` of every rank.
//   pull: thread 0 of every CTA waits (bounded, 1 s of %globaltimer) until all world flags of
//         this rank's arena reached e, then the CTA copies its share of the receive buffer to
//         the output; the last CTA advances the local epoch.
// The epoch lives in device memory (a per-channel control word, zero at rest along with the
// two tickets), so a captured CUDA graph replays correctly. Two receive buffers suffice: a
// rank can only write gather e + 2 into a peer after that peer published e + 1, which the
// peer does after its pull of gather e has copied the buffer out (stream order).
// A flag that never arrives sets LSA_ERR_TIMEOUT in the status word and the pull returns.
// Plain 16-byte stores and loads through the peer mappings only (no bulk or tensor copies).
#include <cstring>

#include "common.cuh"

namespace lsa {
namespace {

constexpr int kPeerMaxRanks = 8;
constexpr int kPeerThreads = 256;
constexpr int kPeerMaxCtas = 16;
constexpr uint64_t kPeerWaitNs = 1000000000ull;

struct PeerGatherArgs {
    const uint4* src;  // this rank's chunk, bytes / 16 pieces
    uint4* out;        // [world][bytes] gathered here
    int64_t n16;       // 16-byte pieces per chunk
    int rank, world;
    uint8_t* base[kPeerMaxRanks];  // every rank's arena as mapped in this process
    int64_t flag_off, recv_off;    // the channel's flags / receive buffers in an arena
    uint32_t* ctrl;                // this rank's control words: [0] epoch, [1] push ticket, [2] pull ticket
    int32_t* status;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(kPeerThreads) peer_push_kernel(const PeerGatherArgs a) {
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(a.ctrl) + 1u;
    const int64_t slot = ((int64_t)(e & 1u) * a.world + a.rank) * a.n16;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int p = 0; p < a.world; ++p) {
        uint4* dst = reinterpret_cast<uint4*>(a.base[p] + a.recv_off) + slot;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.n16; i += stride) dst[i] = a.src[i];
    }
    __threadfence_system();  // this thread's stores reach every peer before the CTA's ticket
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(&a.ctrl[1], 1u) == gridDim.x - 1) {
        a.ctrl[1] = 0u;  // the last CTA: every CTA's stores are out
        __threadfence_system();
        for (int p = 0; p < a.world; ++p)
            st_release_sys(reinterpret_cast<uint32_t*>(a.base[p] + a.flag_off) + a.rank, e);
    }
}

__global__ void __launch_bounds__(kPeerThreads) peer_pull_kernel(const PeerGatherArgs a) {
    __shared__ int ok;
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(a.ctrl) + 1u;
    if (threadIdx.x == 0) {
        const uint32_t* flags = reinterpret_cast<const uint32_t*>(a.base[a.rank] + a.flag_off);
        int good = 1;
        const uint64_t t0 = global_ns();
        for (int p = 0; p < a.world && good; ++p) {
            while ((int32_t)(ld_acquire_sys(flags + p) - e) < 0) {
                if (global_ns() - t0 > kPeerWaitNs) {
                    good = 0;
                    break;
                }
            }
        }
        if (!good) atomicExch(a.status, LSA_ERR_TIMEOUT);
        ok = good;
    }
    __syncthreads();
    if (ok) {
        const uint4* recv = reinterpret_cast<const uint4*>(a.base[a.rank] + a.recv_off) +
                            (int64_t)(e & 1u) * a.world * a.n16;
        const int64_t total = a.world * a.n16, stride = (int64_t)gridDim.x * blockDim.x;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) a.out[i] = recv[i];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&a.ctrl[2], 1u) == gridDim.x - 1) {
            a.ctrl[2] = 0u;
            a.ctrl[0] = e;  // the next gather on this channel is epoch e + 1
        }
    }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

int ctas_for(int64_t n16) {
    const int64_t c = (n16 + kPeerThreads - 1) / kPeerThreads;
    return (int)(c < 1 ? 1 : (c > kPeerMaxCtas ? kPeerMaxCtas : c));
}

}  // namespace
}  // namespace lsa

using namespace lsa;

extern "C" {

int lsa_peer_arena_alloc(int64_t bytes, void** ptr, void* handle) {
    if (bytes <= 0 || ptr == nullptr || handle == nullptr) return LSA_ERR_ARG;
    void* p = nullptr;
    if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return LSA_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return LSA_ERR_CUDA;
    }
    memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return LSA_OK;
}

int lsa_peer_arena_open(const void* handle, void** ptr) {
    if (handle == nullptr || ptr == nullptr) return LSA_ERR_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? LSA_OK : LSA_ERR_CUDA;
}

int lsa_peer_arena_close(void* ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? LSA_OK : LSA_ERR_CUDA; }

int lsa_peer_arena_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? LSA_OK : LSA_ERR_CUDA; }

int lsa_peer_all_gather(const void* src, void* out, int64_t bytes, int rank, int world, void* const* bases,
                        int64_t flag_off, int64_t recv_off, uint32_t* ctrl, int32_t* status, cudaStream_t stream) {
    if (world < 1 || world > kPeerMaxRanks || rank < 0 || rank >= world || bytes < 0 || bytes % 16) return LSA_ERR_ARG;
    if (bases == nullptr || ctrl == nullptr || status == nullptr || flag_off < 0 || recv_off < 0) return LSA_ERR_ARG;
    if (flag_off % 4 || recv_off % 16 || !aligned16(src) || !aligned16(out)) return LSA_ERR_ARG;
    if (bytes == 0) return LSA_OK;
    PeerGatherArgs a;
    a.src = static_cast<const uint4*>(src);
    a.out = static_cast<uint4*>(out);
    a.n16 = bytes / 16;
    a.rank = rank;
    a.world = world;
    for (int p = 0; p < kPeerMaxRanks; ++p) a.base[p] = p < world ? static_cast<uint8_t*>(bases[p]) : nullptr;
    for (int p = 0; p < world; ++p)
        if (a.base[p] == nullptr) return LSA_ERR_ARG;
    a.flag_off = flag_off;
    a.recv_off = recv_off;
    a.ctrl = ctrl;
    a.status = status;
    peer_push_kernel<<<ctas_for(a.n16), kPeerThreads, 0, stream>>>(a);
    LSA_LAUNCH_CHECK();
    peer_pull_kernel<<<ctas_for(a.n16 * world), kPeerThreads, 0, stream>>>(a);
    LSA_LAUNCH_CHECK();
    return LSA_OK;
}

}  // extern "C"
