// torch_ops.cpp - the hot-path operators as torch.library ops (namespace "lsa").
//
// A thin C++ layer over the C ABI (include/lsa_b200.h): each op checks its tensors, takes the
// workspace of the current (device, stream), and launches the library's kernels on
// at::cuda::getCurrentCUDAStream(). Registered ops (drop-ins for the reference's operators):
//   lsa::regroup(q, k) -> (index_queries, index_keys)        make_index_space, port/gates.py:50-59
//   lsa::select_fused(index_queries, positions, centroids, members, block, bpb, top_p, window,
//                     sink, top_k) -> (lists, lengths)          flat_select fused, pipeline.py:274-316
//                     (index_queries [R, d], or raw queries [R, Hq, D]: regroup fused in)
//   lsa::sparse_read(q, k, v, ids, lengths, scale) -> out     sparse_read_auto, read_kernel_tiled.py:147
//   lsa::workspace_counters() -> Tensor[]                      the cached counter buffers (checks)
// Meta implementations give FX / torch.compile the output shapes. Workspaces: scratch (any
// content) and int32 counters (zero at rest: the kernels that use them leave them zero) cached
// per (device, stream), grown on demand - the same contract as the C ABI's callers keep.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "../../include/lsa_b200.h"

namespace {

struct Workspace {
    at::Tensor scratch, counters;
};

std::mutex g_ws_mutex;
std::map<std::pair<int, cudaStream_t>, Workspace> g_ws;

Workspace& workspace(const at::Device& dev, cudaStream_t stream, int64_t scratch_bytes, int64_t n_counters) {
    std::lock_guard<std::mutex> lock(g_ws_mutex);
    Workspace& w = g_ws[{dev.index(), stream}];
    if (!w.scratch.defined() || w.scratch.numel() < scratch_bytes)
        w.scratch = at::empty({std::max<int64_t>(scratch_bytes, 256)}, at::TensorOptions().dtype(at::kByte).device(dev));
    if (!w.counters.defined() || w.counters.numel() < n_counters) {
        // a new buffer starts at zero; the old one (if any) is at rest (zero) by contract
        w.counters = at::zeros({std::max<int64_t>(n_counters, 64)}, at::TensorOptions().dtype(at::kInt).device(dev));
    }
    return w;
}

int dtype_code(at::ScalarType t) {
    switch (t) {
        case at::kFloat: return 0;
        case at::kHalf: return 1;
        case at::kBFloat16: return 2;
        default: TORCH_CHECK(false, "lsa: expected fp32 / fp16 / bf16, got ", t);
    }
    return -1;
}

void check_rc(int rc, const char* what) {
    TORCH_CHECK(rc == 0, what, ": the C-ABI entry point returned status ", rc,
                rc == -1 ? " (arguments rejected)" : (rc == -2 ? " (CUDA launch failed)" : ""));
}

std::tuple<at::Tensor, at::Tensor> regroup_cuda(const at::Tensor& q_in, const at::Tensor& k_in) {
    TORCH_CHECK(q_in.is_cuda() && k_in.is_cuda(), "lsa::regroup is a CUDA kernel");
    TORCH_CHECK(q_in.dim() == 3 && k_in.dim() == 3 && q_in.size(0) == k_in.size(0) && q_in.size(2) == k_in.size(2),
                "lsa::regroup: q [T, Hq, D], k [T, Hkv, D]");
    TORCH_CHECK(q_in.scalar_type() == k_in.scalar_type(), "lsa::regroup: q and k share a dtype");
    c10::cuda::CUDAGuard guard(q_in.device());
    auto q = q_in.contiguous(), k = k_in.contiguous();
    const int64_t T = q.size(0), Hq = q.size(1), Hkv = k.size(1), D = q.size(2);
    TORCH_CHECK(Hq % Hkv == 0, "lsa::regroup: query heads must group evenly onto KV heads");
    auto opts = q.options().dtype(at::kFloat);
    auto iq = at::empty({T, Hkv * D}, opts), ik = at::empty({T, Hkv * D}, opts);
    if (T)
        check_rc(lsa_regroup(q.data_ptr(), k.data_ptr(), dtype_code(q.scalar_type()), T, Hq, Hkv, D,
                             iq.data_ptr<float>(), ik.data_ptr<float>(), at::cuda::getCurrentCUDAStream()),
                 "lsa::regroup");
    return {iq, ik};
}

std::tuple<at::Tensor, at::Tensor> select_fused_cuda(const at::Tensor& iq_arg, const at::Tensor& positions_in,
                                                     const at::Tensor& centroids_in, const at::Tensor& members_in,
                                                     int64_t block, int64_t bpb, int64_t top_p, int64_t window,
                                                     int64_t sink, int64_t top_k) {
    TORCH_CHECK(iq_arg.is_cuda() && positions_in.is_cuda() && centroids_in.is_cuda() && members_in.is_cuda(),
                "lsa::select_fused is a CUDA kernel");
    TORCH_CHECK(centroids_in.dim() == 2, "lsa::select_fused: centroids [N, d]");
    c10::cuda::CUDAGuard guard(iq_arg.device());
    const auto cdt = centroids_in.scalar_type();
    TORCH_CHECK(cdt == at::kBFloat16 || cdt == at::kFloat, "lsa::select_fused: bf16 or fp32 centroids");
    at::Tensor iq_in = iq_arg;
    if (iq_arg.dim() == 3) {
        // raw queries [R, Hq, D]: the index queries are built inside the decode select (one
        // launch); rows it does not take are regrouped first and go the two-dimensional way
        auto qr = iq_arg.contiguous();
        const int64_t R = qr.size(0), Hq = qr.size(1), D = qr.size(2), d = centroids_in.size(1);
        TORCH_CHECK(D > 0 && d % D == 0 && Hq % (d / D) == 0,
                    "lsa::select_fused: raw queries [R, Hq, D] need centroids of Hkv * D dims with Hq % Hkv == 0");
        TORCH_CHECK(positions_in.numel() == R, "lsa::select_fused: a position a query");
        const int64_t Hkv = d / D;
        auto c = centroids_in.contiguous();
        auto members = members_in.to(at::kInt).contiguous();
        auto pos = positions_in.to(at::kInt).contiguous();
        const int64_t width = top_k + window + sink;
        auto lists = at::empty({R, width}, qr.options().dtype(at::kInt));
        auto lengths = at::empty({R}, qr.options().dtype(at::kInt));
        if (R == 0) return {lists, lengths};
        auto stream = at::cuda::getCurrentCUDAStream();
        const int rc = lsa_select_fused_grouped(qr.data_ptr(), dtype_code(qr.scalar_type()), R, Hq, Hkv, D,
                                                c.data_ptr(), cdt == at::kFloat ? 0 : 2, c.size(0),
                                                pos.data_ptr<int32_t>(), block, bpb, members.data_ptr<int32_t>(),
                                                members.size(1), top_p, window, sink, top_k,
                                                lists.data_ptr<int32_t>(), lengths.data_ptr<int32_t>(), stream);
        if (rc == LSA_OK) return {lists, lengths};
        TORCH_CHECK(rc == LSA_ERR_ARG, "lsa::select_fused: the C-ABI entry point returned status ", rc);
        iq_in = at::empty({R, d}, qr.options().dtype(at::kFloat));
        check_rc(lsa_regroup(qr.data_ptr(), nullptr, dtype_code(qr.scalar_type()), R, Hq, Hkv, D,
                             iq_in.data_ptr<float>(), nullptr, stream),
                 "lsa::select_fused");
    }
    TORCH_CHECK(iq_in.dim() == 2 && iq_in.size(1) == centroids_in.size(1),
                "lsa::select_fused: index_queries [R, d] (or raw queries [R, Hq, D]), centroids [N, d]");
    TORCH_CHECK(positions_in.numel() == iq_in.size(0), "lsa::select_fused: a position a query");
    at::Tensor q;
    int q_code;
    if (cdt == at::kFloat) {  // fp32 scoring
        q = iq_in.to(at::kFloat).contiguous();
        q_code = 0;
    } else if (iq_in.scalar_type() == at::kFloat) {  // bf16 scoring of fp32 queries, rounded in-kernel
        q = iq_in.contiguous();
        q_code = 3;
    } else {
        q = iq_in.to(at::kBFloat16).contiguous();
        q_code = 2;
    }
    auto c = centroids_in.contiguous();
    auto members = members_in.to(at::kInt).contiguous();
    auto pos = positions_in.to(at::kInt).contiguous();
    const int64_t R = q.size(0), d = q.size(1), N = c.size(0);
    const int64_t width = top_k + window + sink;
    auto lists = at::empty({R, width}, q.options().dtype(at::kInt));
    auto lengths = at::empty({R}, q.options().dtype(at::kInt));
    if (R == 0) return {lists, lengths};
    auto stream = at::cuda::getCurrentCUDAStream();
    Workspace& w = workspace(q.device(), stream, lsa_select_fused_scratch(R, N), R + 1);
    check_rc(lsa_select_fused(q.data_ptr(), q_code, R, d, c.data_ptr(), cdt == at::kFloat ? 0 : 2, N, d,
                              pos.data_ptr<int32_t>(), block, bpb, members.data_ptr<int32_t>(), members.size(1), top_p,
                              window, sink, top_k, lists.data_ptr<int32_t>(), lengths.data_ptr<int32_t>(),
                              w.scratch.data_ptr(), w.scratch.numel(), w.counters.data_ptr<int32_t>(),
                              w.counters.numel(), -1, stream),
             "lsa::select_fused");
    return {lists, lengths};
}

at::Tensor sparse_read_cuda(const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in,
                            const at::Tensor& ids_in, const at::Tensor& lengths_in, double scale) {
    TORCH_CHECK(q_in.is_cuda() && k_in.is_cuda() && v_in.is_cuda(), "lsa::sparse_read is a CUDA kernel");
    TORCH_CHECK(q_in.dim() == 4 && k_in.dim() == 4 && v_in.sizes() == k_in.sizes(),
                "lsa::sparse_read: q [B, Tq, Hq, D], k / v [B, Tk, Hkv, D]");
    TORCH_CHECK(q_in.scalar_type() == k_in.scalar_type() && q_in.scalar_type() == v_in.scalar_type(),
                "lsa::sparse_read: q, k, v share a dtype");
    c10::cuda::CUDAGuard guard(q_in.device());
    auto q = q_in.contiguous(), k = k_in.contiguous(), v = v_in.contiguous();
    const int64_t B = q.size(0), Tq = q.size(1), Hq = q.size(2), D = q.size(3), Tk = k.size(1), Hkv = k.size(2);
    TORCH_CHECK(Hq % Hkv == 0, "lsa::sparse_read: query heads must group evenly onto KV heads");
    const int64_t width = ids_in.size(-1);
    auto ids = ids_in.reshape({-1, width}).to(at::kInt).contiguous();
    auto lens = lengths_in.reshape({-1}).to(at::kInt).contiguous();
    auto out = at::empty_like(q);
    if (B * Tq == 0) return out;
    int64_t splits = 0, scratch_bytes = 0, n_counters = 0;
    check_rc(lsa_sparse_read_plan(B, Tq, Hq, Hkv, D, width, 0, &splits, &scratch_bytes, &n_counters),
             "lsa::sparse_read");
    auto stream = at::cuda::getCurrentCUDAStream();
    Workspace& w = workspace(q.device(), stream, scratch_bytes, n_counters);
    check_rc(lsa_sparse_read(q.data_ptr(), k.data_ptr(), v.data_ptr(), dtype_code(q.scalar_type()),
                             ids.data_ptr<int32_t>(), lens.data_ptr<int32_t>(), B, Tq, Tk, Hq, Hkv, D, width,
                             (float)scale, out.data_ptr(), w.scratch.data_ptr(), w.scratch.numel(),
                             w.counters.data_ptr<int32_t>(), w.counters.numel(), 0, stream),
             "lsa::sparse_read");
    return out;
}

std::vector<at::Tensor> workspace_counters() {
    std::lock_guard<std::mutex> lock(g_ws_mutex);
    std::vector<at::Tensor> out;
    for (auto& kv : g_ws)
        if (kv.second.counters.defined()) out.push_back(kv.second.counters);
    return out;
}

// ------------------------------------------------------------------ shapes (Meta)

std::tuple<at::Tensor, at::Tensor> regroup_meta(const at::Tensor& q, const at::Tensor& k) {
    auto opts = q.options().dtype(at::kFloat);
    return {at::empty({q.size(0), k.size(1) * k.size(2)}, opts), at::empty({q.size(0), k.size(1) * k.size(2)}, opts)};
}

std::tuple<at::Tensor, at::Tensor> select_fused_meta(const at::Tensor& iq, const at::Tensor&, const at::Tensor&,
                                                     const at::Tensor&, int64_t, int64_t, int64_t, int64_t window,
                                                     int64_t sink, int64_t top_k) {
    auto opts = iq.options().dtype(at::kInt);
    return {at::empty({iq.size(0), top_k + window + sink}, opts), at::empty({iq.size(0)}, opts)};
}

at::Tensor sparse_read_meta(const at::Tensor& q, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                            const at::Tensor&, double) {
    return at::empty_like(q);
}

}  // namespace

TORCH_LIBRARY(lsa, m) {
    m.def("regroup(Tensor q, Tensor k) -> (Tensor, Tensor)");
    m.def("select_fused(Tensor index_queries, Tensor positions, Tensor centroids, Tensor members, int block, int bpb, "
          "int top_p, int window, int sink, int top_k) -> (Tensor, Tensor)");
    m.def("sparse_read(Tensor q, Tensor k, Tensor v, Tensor ids, Tensor lengths, float scale) -> Tensor");
    m.def("workspace_counters() -> Tensor[]", &workspace_counters);
}

TORCH_LIBRARY_IMPL(lsa, CUDA, m) {
    m.impl("regroup", &regroup_cuda);
    m.impl("select_fused", &select_fused_cuda);
    m.impl("sparse_read", &sparse_read_cuda);
}

TORCH_LIBRARY_IMPL(lsa, Meta, m) {
    m.impl("regroup", &regroup_meta);
    m.impl("select_fused", &select_fused_meta);
    m.impl("sparse_read", &sparse_read_meta);
}
