// Bindings of the symmetric-memory plumbing and the reduce-scatter receiver.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <string>

#include "comm_api.h"

namespace {
void check(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e));
}

// Raw device allocation (outside torch's caching allocator) so that the CUDA
// IPC handle covers exactly this buffer.
int64_t symm_alloc(int64_t nbytes) {
  void* p = nullptr;
  check(cudaMalloc(&p, size_t(nbytes)), "symm_alloc");
  check(cudaMemset(p, 0, size_t(nbytes)), "symm_alloc memset");
  return reinterpret_cast<int64_t>(p);
}
void symm_free(int64_t ptr) { check(cudaFree(reinterpret_cast<void*>(ptr)), "symm_free"); }

pybind11::bytes ipc_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  check(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)), "cudaIpcGetMemHandle");
  return pybind11::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}
int64_t ipc_open(const std::string& handle) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<int64_t>(p);
}
void ipc_close(int64_t ptr) {
  check(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)), "cudaIpcCloseMemHandle");
}

// Non-owning tensor view of device memory (lifetime is the caller's).
at::Tensor view_ptr(int64_t ptr, std::vector<int64_t> shape, at::ScalarType dtype, int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), shape, opts);
}

// Copy `bytes` from a local CUDA tensor to a raw device pointer (own kernel).
void copy_to_ptr(int64_t dst, const at::Tensor& src, int64_t bytes, int64_t ctas) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous() && src.numel() * src.element_size() >= bytes);
  const c10::cuda::CUDAGuard guard(src.device());
  const int code = tn5b::comm::copy16(reinterpret_cast<void*>(dst), src.data_ptr(), bytes, int(ctas),
                                      at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(code == 0, "copy_to_ptr failed (", code, ")");
}

// Raw pointer to raw pointer copy with this framework's 16-byte copy kernel
// (either side may be a peer's IPC mapping: push when dst is remote, pull when
// src is remote).
void copy_ptr(int64_t dst, int64_t src, int64_t bytes, int64_t ctas) {
  const int code = tn5b::comm::copy16(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), bytes,
                                      int(ctas), at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(code == 0, "copy_ptr failed (", code, ")");
}

// Bulk-engine pull/copy: src may be a peer's memory, dst is local.
void bulk_copy(int64_t dst, int64_t src, int64_t bytes, int64_t ctas, int64_t chunk, int64_t stages,
               int64_t timeout_ns, const at::Tensor& status) {
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == at::kInt, "status must be a CUDA int32 tensor");
  const c10::cuda::CUDAGuard guard(status.device());
  const int code = tn5b::comm::bulk_copy(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), bytes,
                                         int(ctas), int(chunk), int(stages), uint64_t(timeout_ns),
                                         status.data_ptr<int>(), at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(code == 0, "bulk_copy failed (", code < 0 ? "bad arguments" : cudaGetErrorString(cudaError_t(code)), ")");
}

void rs_reduce(int64_t recv, int64_t flags, int64_t slot_bytes, int64_t rank, int64_t world,
               int64_t rows, int64_t n, int64_t tile_n, int64_t chunk_rows, bool quantized,
               int64_t epoch, at::Tensor& out, const c10::optional<at::Tensor>& residual,
               const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& tile_order,
               bool arrival, const c10::optional<at::Tensor>& claims, const at::Tensor& status,
               int64_t timeout_ns, int64_t max_ctas, const c10::optional<at::Tensor>& stamps) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.is_contiguous());
  TORCH_CHECK(out.size(0) == rows && out.size(1) == n, "rs_reduce: out must be [rows, n]");
  const c10::cuda::CUDAGuard guard(out.device());
  tn5b::comm::RsReduceCall c;
  c.recv = reinterpret_cast<const uint8_t*>(recv);
  c.flags = reinterpret_cast<const uint32_t*>(flags);
  c.slot_bytes = slot_bytes;
  c.rank = int(rank); c.world = int(world);
  c.rows = int(rows); c.n = int(n); c.tile_n = int(tile_n); c.chunk_rows = int(chunk_rows);
  c.quantized = quantized; c.epoch = uint32_t(epoch);
  c.out = out.data_ptr();
  if (residual) {
    TORCH_CHECK(residual->is_contiguous() && residual->scalar_type() == at::kBFloat16 &&
                residual->numel() == rows * n);
    c.residual = residual->data_ptr();
  }
  if (bias) {
    TORCH_CHECK(bias->is_contiguous() && bias->scalar_type() == at::kBFloat16 && bias->numel() == n);
    c.bias = bias->data_ptr();
  }
  if (tile_order) c.tile_order = tile_order->data_ptr<int>();
  c.arrival = arrival;
  if (claims) c.claims = claims->data_ptr<int>();
  c.status = status.data_ptr<int>();
  c.timeout_ns = uint64_t(timeout_ns);
  c.max_ctas = int(max_ctas);
  if (stamps) {
    TORCH_CHECK(stamps->scalar_type() == at::kLong && stamps->is_cuda());
    c.stamps = reinterpret_cast<unsigned long long*>(stamps->data_ptr<int64_t>());
  }
  const int r = tn5b::comm::rs_reduce(c, at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(r == 0, "rs_reduce failed: ", r < 0 ? "bad arguments" : cudaGetErrorString(cudaError_t(r)));
}

void pack_pieces(const at::Tensor& src, int64_t dst) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16 && src.dim() == 2 && src.stride(1) == 1,
              "pack_pieces: src must be a CUDA bf16 [M, N] with unit inner stride");
  const c10::cuda::CUDAGuard guard(src.device());
  const int r = tn5b::comm::pack_pieces(src.data_ptr(), src.stride(0), reinterpret_cast<void*>(dst), int(src.size(0)),
                                        int(src.size(1)), at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(r == 0, "pack_pieces failed: ", r < 0 ? "M % 128, N % 64 and 16-byte alignment required"
                                                    : cudaGetErrorString(cudaError_t(r)));
}

void publish_tiles(int64_t flag_ptrs, int64_t rank, int64_t world, int64_t per_dest, int64_t epoch, int64_t device) {
  const c10::cuda::CUDAGuard guard(c10::Device(c10::kCUDA, int(device)));
  const int r = tn5b::comm::publish_tiles(reinterpret_cast<uint32_t* const*>(flag_ptrs), int(rank), int(world),
                                          int(per_dest), uint32_t(epoch), at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(r == 0, "publish_tiles failed");
}

void wait_probe(int64_t flag, int64_t target, int64_t timeout_ns, const at::Tensor& status) {
  const c10::cuda::CUDAGuard guard(status.device());
  const int r = tn5b::comm::wait_probe(reinterpret_cast<const uint32_t*>(flag), uint32_t(target),
                                       uint64_t(timeout_ns), status.data_ptr<int>(),
                                       at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(r == 0, "wait_probe launch failed");
}
}  // namespace

void register_comm(pybind11::module& m) {
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_free", &symm_free);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("view_ptr", &view_ptr);
  using nogil = pybind11::call_guard<pybind11::gil_scoped_release>;
  m.def("rs_reduce", &rs_reduce, nogil());
  m.def("wait_probe", &wait_probe, nogil());
  m.def("pack_pieces", &pack_pieces, nogil());
  m.def("publish_tiles", &publish_tiles, nogil());
  m.def("copy_to_ptr", &copy_to_ptr, nogil());
  m.def("copy_ptr", &copy_ptr, nogil());
  m.def("bulk_copy", &bulk_copy, nogil());
}
