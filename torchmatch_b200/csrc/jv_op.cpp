// CUDA implementation of torch.ops.assignment.jonker_dense_batch.
//
// The operator schema "jonker_dense_batch(Tensor costs) -> Tensor" belongs to
// the `assignment` library (tue-p8n/torchmatch 1.0.3,
// sources/torchmatch/assignment/cpu/ops.cpp:486-496).  This file registers
// only the CUDA kernel for it (the reference does the same in
// cuda/dispatch.cu:181-186); the Python loader defines the schema and the
// fake kernel when the reference's CPU extension has not done so already.
//
// Behaviour kept from jonker_dense_batch_cuda (cuda/dispatch.cu:137-177):
// device guard, current-stream execution, refusal inside CUDA graph capture,
// fp32 cast, batch-global +inf sentinel with a host sync to raise on NaN /
// -inf, a fresh int64 (B, N) output.  The same sync reads the device status
// back and raises if a cost tile copy timed out.  The statistics come out of the solve
// itself (check mode); only batches holding +inf are solved a second time.  Widened: rectangular (B, N, M) input
// and max(N, M) up to tm_jv_max_k(); non-contiguous input is made
// contiguous instead of rejected.  All device work goes through the C ABI in
// include/torchmatch_b200.h.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "torchmatch_b200.h"

namespace {

void check_not_capturing(cudaStream_t stream, const char *op_name) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    const cudaError_t e = cudaStreamIsCapturing(stream, &st);
    TORCH_CHECK(e == cudaSuccess, "cudaStreamIsCapturing failed: ", cudaGetErrorString(e));
    TORCH_CHECK(st == cudaStreamCaptureStatusNone, op_name,
                " performs a host-side CUDA synchronization and cannot run inside CUDA "
                "graph capture (e.g. torch.compile(mode=\"reduce-overhead\")); call it "
                "outside the captured region.");
}

std::string status_text(int rc) {
    std::string s = tm_status_string(rc);
    if (rc == TM_ERR_CUDA) {
        s += ": ";
        s += cudaGetErrorString(static_cast<cudaError_t>(tm_last_cuda_error()));
    }
    return s;
}

using FullFn = int (*)(const float *, int64_t, int, int, int64_t *, void *, tm_stream_t);
using UnpackedFn = int (*)(const float *, int64_t, int, int, const tm_jv_unpacked *, void *,
                           tm_stream_t);

// Shared body of the packed ops: checks, capture guard, fp32 cast, then one
// C-ABI call that solves in check mode, reads the 8-byte verdict back
// (raising on NaN / -inf like cuda_common.cuh:245-249) and, only for a
// batch holding +inf, solves again with the batch-global sentinel.
at::Tensor packed_op(const at::Tensor &costs, FullFn fn, const char *name) {
    TORCH_CHECK(costs.is_cuda(), "costs must be a CUDA tensor");
    TORCH_CHECK(costs.dim() == 3, "costs must be 3D (B, N, M), got ", costs.dim());
    TORCH_CHECK(costs.scalar_type() == at::kFloat || costs.scalar_type() == at::kDouble,
                "costs must be float32 or float64, got ", costs.scalar_type());
    const c10::cuda::CUDAGuard guard(costs.device());
    const int64_t B = costs.size(0), N = costs.size(1), M = costs.size(2);
    if (B == 0 || N == 0 || M == 0)
        return at::full({B, N}, -1, costs.options().dtype(at::kLong));
    const int64_t K = std::max(N, M);
    TORCH_CHECK(K <= tm_jv_max_k(), "Batched JV (CUDA) supports max(N, M) <= ", tm_jv_max_k(),
                ", got K=", K);
    cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
    check_not_capturing(stream, name);
    const at::Tensor c = costs.to(at::kFloat).contiguous();
    at::Tensor scratch =
        at::empty({(int64_t)tm_jv_workspace_bytes()}, c.options().dtype(at::kByte));
    at::Tensor out = at::empty({B, N}, costs.options().dtype(at::kLong));
    const int rc = fn(c.const_data_ptr<float>(), B, static_cast<int>(N), static_cast<int>(M),
                      out.mutable_data_ptr<int64_t>(), scratch.mutable_data_ptr(),
                      reinterpret_cast<tm_stream_t>(stream));
    TORCH_CHECK(rc != TM_ERR_NAN, name, ": ", tm_status_string(rc));
    TORCH_CHECK(rc != TM_ERR_NEG_INF, name, ": ", tm_status_string(rc));
    TORCH_CHECK(rc != TM_ERR_TIMEOUT, name, ": ", tm_status_string(rc));
    TORCH_CHECK(rc == TM_OK, "batched JV kernel launch failed: ", status_text(rc));
    return out;
}

at::Tensor jonker_dense_batch_cuda(const at::Tensor &costs) {
    return packed_op(costs, &tm_jonker_dense_batch_f32, "jonker_dense_batch");
}

at::Tensor jonker_compact_batch_cuda(const at::Tensor &costs) {
    return packed_op(costs, &tm_jonker_compact_batch_f32, "jonker_compact_batch");
}

// jonker_dense_batch_unpacked on CUDA (the reference has it on CPU only,
// cpu/ops.cpp:297-417): the same solve, with the compacted outputs written by
// the solve kernel's output stage.  Layout and empty-shape behaviour follow
// the CPU op (cpu/ops.cpp:290-316).
std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor>
unpacked_op(const at::Tensor &costs, UnpackedFn fn, const char *name) {
    TORCH_CHECK(costs.is_cuda(), "costs must be a CUDA tensor");
    TORCH_CHECK(costs.dim() == 3, "costs must be 3D (B, N, M), got ", costs.dim());
    TORCH_CHECK(costs.scalar_type() == at::kFloat || costs.scalar_type() == at::kDouble,
                "costs must be float32 or float64, got ", costs.scalar_type());
    const c10::cuda::CUDAGuard guard(costs.device());
    const int64_t B = costs.size(0), N = costs.size(1), M = costs.size(2);
    const auto lo = costs.options().dtype(at::kLong);
    if (B == 0 || N == 0 || M == 0)
        return {at::empty({B, N, 2}, lo), at::empty({B, N}, lo), at::empty({B, M}, lo),
                at::zeros({B}, lo)};
    const int64_t K = std::max(N, M);
    TORCH_CHECK(K <= tm_jv_max_k(), "Batched JV (CUDA) supports max(N, M) <= ", tm_jv_max_k(),
                ", got K=", K);
    cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
    check_not_capturing(stream, name);
    const at::Tensor c = costs.to(at::kFloat).contiguous();
    at::Tensor scratch =
        at::empty({(int64_t)tm_jv_workspace_bytes()}, c.options().dtype(at::kByte));
    at::Tensor matches = at::empty({B, N, 2}, lo), ur = at::empty({B, N}, lo);
    at::Tensor uc = at::empty({B, M}, lo), nm = at::empty({B}, lo);
    tm_jv_unpacked u{matches.mutable_data_ptr<int64_t>(), ur.mutable_data_ptr<int64_t>(),
                     uc.mutable_data_ptr<int64_t>(), nm.mutable_data_ptr<int64_t>()};
    const int rc = fn(
        c.const_data_ptr<float>(), B, static_cast<int>(N), static_cast<int>(M), &u,
        scratch.mutable_data_ptr(), reinterpret_cast<tm_stream_t>(stream));
    TORCH_CHECK(rc != TM_ERR_NAN, name, ": ", tm_status_string(rc));
    TORCH_CHECK(rc != TM_ERR_NEG_INF, name, ": ", tm_status_string(rc));
    TORCH_CHECK(rc != TM_ERR_TIMEOUT, name, ": ", tm_status_string(rc));
    TORCH_CHECK(rc == TM_OK, "batched JV kernel launch failed: ", status_text(rc));
    return {matches, ur, uc, nm};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor>
jonker_dense_batch_unpacked_cuda(const at::Tensor &costs) {
    return unpacked_op(costs, &tm_jonker_dense_batch_unpacked_f32, "jonker_dense_batch_unpacked");
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor>
jonker_compact_batch_unpacked_cuda(const at::Tensor &costs) {
    return unpacked_op(costs, &tm_jonker_compact_batch_unpacked_f32,
                       "jonker_compact_batch_unpacked");
}

// jonker_dense_batch_async: the same mapping without any host
// synchronisation, so it can be captured in a CUDA graph.  Returns the
// mapping and a one-element int32 status tensor (TM_WS_* bits: 1 NaN,
// 2 -inf, 4 a problem hit a loop bound, 8 a wait timed out) that stays on the
// device; NaN / -inf problems are rows of -1.  No counterpart in the
// reference, whose op refuses capture (cuda/dispatch.cu:97-106).
std::tuple<at::Tensor, at::Tensor> jonker_dense_batch_async_cuda(const at::Tensor &costs) {
    TORCH_CHECK(costs.is_cuda(), "costs must be a CUDA tensor");
    TORCH_CHECK(costs.dim() == 3, "costs must be 3D (B, N, M), got ", costs.dim());
    TORCH_CHECK(costs.scalar_type() == at::kFloat || costs.scalar_type() == at::kDouble,
                "costs must be float32 or float64, got ", costs.scalar_type());
    const c10::cuda::CUDAGuard guard(costs.device());
    const int64_t B = costs.size(0), N = costs.size(1), M = costs.size(2);
    TORCH_CHECK(std::max(N, M) <= tm_jv_max_k(), "Batched JV (CUDA) supports max(N, M) <= ",
                tm_jv_max_k(), ", got K=", std::max(N, M));
    at::Tensor scratch = at::zeros({(int64_t)tm_jv_workspace_bytes() / 4},
                                   costs.options().dtype(at::kInt));
    at::Tensor status = scratch.narrow(0, offsetof(tm_jv_workspace, status) / 4, 1);
    at::Tensor out = at::empty({B, N}, costs.options().dtype(at::kLong));
    if (B == 0 || N == 0) return {out, status.clone()};
    if (M == 0) {
        out.fill_(-1);
        return {out, status.clone()};
    }
    const at::Tensor c = costs.to(at::kFloat).contiguous();
    cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
    const int rc = tm_jonker_dense_batch_async_f32(
        c.const_data_ptr<float>(), B, static_cast<int>(N), static_cast<int>(M),
        out.mutable_data_ptr<int64_t>(), scratch.mutable_data_ptr(),
        reinterpret_cast<tm_stream_t>(stream));
    TORCH_CHECK(rc == TM_OK, "batched JV kernel launch failed: ", status_text(rc));
    // a fresh tensor (stream-ordered copy) rather than a view into scratch
    return {out, status.clone()};
}

// jonker_sqeuclidean_batch(x (B, N, D), y (B, M, D)) -> (B, N) int64: the
// mapping of jonker_dense_batch on the squared-Euclidean costs of the two
// point sets, built inside the solve kernel instead of as a (B, N, M)
// tensor.  No counterpart op in the reference; the result equals
// jonker_dense_batch on the costs of a sequential fp32 producer (see the
// C ABI declaration).
at::Tensor jonker_sqeuclidean_batch_cuda(const at::Tensor &x, const at::Tensor &y) {
    TORCH_CHECK(x.is_cuda() && y.is_cuda(), "x and y must be CUDA tensors");
    TORCH_CHECK(x.device() == y.device(), "x and y must be on the same device");
    TORCH_CHECK(x.dim() == 3 && y.dim() == 3, "x must be (B, N, D) and y (B, M, D)");
    TORCH_CHECK(x.size(0) == y.size(0) && x.size(2) == y.size(2),
                "x (B, N, D) and y (B, M, D) must agree in B and D, got ", x.sizes(), " and ",
                y.sizes());
    TORCH_CHECK(x.scalar_type() == at::kFloat || x.scalar_type() == at::kDouble,
                "x must be float32 or float64, got ", x.scalar_type());
    TORCH_CHECK(y.scalar_type() == at::kFloat || y.scalar_type() == at::kDouble,
                "y must be float32 or float64, got ", y.scalar_type());
    const c10::cuda::CUDAGuard guard(x.device());
    const int64_t B = x.size(0), N = x.size(1), M = y.size(1), D = x.size(2);
    if (B == 0 || N == 0 || M == 0)
        return at::full({B, N}, -1, x.options().dtype(at::kLong));
    const int64_t K = std::max(N, M);
    TORCH_CHECK(K <= tm_jv_max_k(), "Batched JV (CUDA) supports max(N, M) <= ", tm_jv_max_k(),
                ", got K=", K);
    TORCH_CHECK(D <= INT32_MAX, "D too large");
    cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
    check_not_capturing(stream, "jonker_sqeuclidean_batch");
    const at::Tensor xc = x.to(at::kFloat).contiguous(), yc = y.to(at::kFloat).contiguous();
    const size_t ws_bytes = tm_jv_points_workspace_bytes(B, static_cast<int>(N),
                                                         static_cast<int>(M));
    // the caching allocator returns 512-byte aligned blocks
    at::Tensor scratch = at::empty({(int64_t)ws_bytes}, xc.options().dtype(at::kByte));
    at::Tensor out = at::empty({B, N}, x.options().dtype(at::kLong));
    const int rc = tm_jonker_sqeuclidean_batch_f32(
        xc.const_data_ptr<float>(), yc.const_data_ptr<float>(), B, static_cast<int>(N),
        static_cast<int>(M), static_cast<int>(D), out.mutable_data_ptr<int64_t>(),
        scratch.mutable_data_ptr(), ws_bytes, reinterpret_cast<tm_stream_t>(stream));
    TORCH_CHECK(rc != TM_ERR_NAN, "jonker_sqeuclidean_batch: ", tm_status_string(rc));
    TORCH_CHECK(rc != TM_ERR_NEG_INF, "jonker_sqeuclidean_batch: ", tm_status_string(rc));
    TORCH_CHECK(rc != TM_ERR_TIMEOUT, "jonker_sqeuclidean_batch: ", tm_status_string(rc));
    TORCH_CHECK(rc == TM_OK, "batched JV kernel launch failed: ", status_text(rc));
    return out;
}

}  // namespace

TORCH_LIBRARY_IMPL(assignment, CUDA, m) {
    m.impl("jonker_sqeuclidean_batch", &jonker_sqeuclidean_batch_cuda);
    m.impl("jonker_dense_batch_async", &jonker_dense_batch_async_cuda);
    m.impl("jonker_dense_batch", &jonker_dense_batch_cuda);
    m.impl("jonker_dense_batch_unpacked", &jonker_dense_batch_unpacked_cuda);
    m.impl("jonker_compact_batch", &jonker_compact_batch_cuda);
    m.impl("jonker_compact_batch_unpacked", &jonker_compact_batch_unpacked_cuda);
}
