// walk.cuh - the expansion walk over staged member slots, shared by the selects and the
// tree beam (sm_100a).
#pragma once

#include "common.cuh"

namespace lsa {

// The rank-order walk over staged member slots mem[0, total) (slot p * cap + m holds member
// m of the p-th pick; -1 and ids outside [sink, ws) are skipped): one scan over all slots
// gives every thread its output offset, kept ids go out in slot order up to top_k, then the
// window [ws, pos] and the sinks [0, min(sink, ws)). Run by NT threads (tid in [0, NT)) that
// share the barrier `sync`; mem must be 16-byte aligned.
template <int NT, typename Sync>
__device__ void expand_walk(const int* mem, int total, int64_t pos, int window, int sink, int top_k,
                            int32_t* __restrict__ out, int width, int32_t* length_out, int* scan_smem, int tid,
                            Sync sync, int* gather = nullptr) {
    // gather (top_k ints of shared memory, optional): kept ids land there first and leave in
    // one coalesced copy instead of scattered 4-byte stores per thread
    int32_t* dst = gather ? gather : out;
    int64_t ws = pos + 1 - window;
    if (ws < 0) ws = 0;
    auto keep = [&](int v) { return v >= 0 && v >= sink && (int64_t)v < ws; };
    const int spt = (total + NT - 1) / NT;
    const int first = tid * spt;
    const bool vec = spt % 4 == 0 && first + spt <= total;  // contiguous 16-byte reads of this thread's slots
    int cnt = 0;
    if (vec) {
        for (int i = 0; i < spt; i += 4) {
            int4 v = *reinterpret_cast<const int4*>(mem + first + i);
            cnt += keep(v.x) + keep(v.y) + keep(v.z) + keep(v.w);
        }
    } else {
        for (int i = 0; i < spt; ++i) {
            int s = first + i;
            cnt += (s < total && keep(mem[s]));
        }
    }
    int filled;
    int at = group_exclusive_scan<NT>(cnt, scan_smem, &filled, tid, sync);
    if (vec) {
        for (int i = 0; i < spt && at < top_k; i += 4) {
            int4 v = *reinterpret_cast<const int4*>(mem + first + i);
            const int e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (keep(e[u])) {
                    if (at < top_k) dst[at] = e[u];
                    ++at;
                }
            }
        }
    } else {
        for (int i = 0; i < spt && at < top_k; ++i) {
            int s = first + i;
            if (s < total && keep(mem[s])) {
                dst[at] = mem[s];
                ++at;
            }
        }
    }
    if (filled > top_k) filled = top_k;
    if (gather) {
        sync();
        for (int i = tid; i < filled; i += NT) out[i] = gather[i];
    }
    int nwin = (int)(pos - ws + 1);
    if (nwin < 0) nwin = 0;
    int nsink = (int)(sink < ws ? sink : ws);
    for (int i = tid; i < width - filled; i += NT) {
        int j = filled + i, v = -1;
        if (i < nwin) v = (int)(ws + i);
        else if (i < nwin + nsink) v = i - nwin;
        out[j] = v;
    }
    if (tid == 0) *length_out = filled + nwin + nsink;
}

}  // namespace lsa
