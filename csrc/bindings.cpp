// Python bindings of the native sm_100a kernels (module tempname_5090_b200._C).
// Every entry validates dtype/device/contiguity, takes the current CUDA stream
// and raises on a failed launch; no entry point falls back to another backend.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "gemm/gemm_api.h"
#include "kernels/kernels_api.h"
#include "comm/comm_api.h"
#include "common/push_lanes.h"

namespace {

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
void check_bf16(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
}
void check_rows(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be 2-D with unit inner stride");
}
void raise_if(int code, const char* what) {
  if (code == 0) return;
  if (code < 0) TORCH_CHECK(false, what, ": ", tn5b::gemm::last_error());
  TORCH_CHECK(false, what, ": ", cudaGetErrorString(cudaError_t(code)));
}
cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }
int* status_ptr(const at::Tensor& s) {
  check_cuda(s, "status");
  TORCH_CHECK(s.scalar_type() == at::kInt && s.numel() >= 1, "status must be int32");
  return s.data_ptr<int>();
}

// out = epilogue(A * B^T).  a_mn / b_mn select MN-major storage ([K,M] / [K,N]).
void gemm(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, at::Tensor& out,
          int64_t epi, const c10::optional<at::Tensor>& bias,
          const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& residual,
          const at::Tensor& status, int64_t bn, int64_t max_ctas,
          const c10::optional<at::Tensor>& tile_order, int64_t pair, int64_t group_m,
          const c10::optional<at::Tensor>& debug) {
  check_bf16(A, "A"); check_bf16(B, "B"); check_bf16(out, "out");
  check_rows(A, "A"); check_rows(B, "B"); check_rows(out, "out");
  const c10::cuda::CUDAGuard guard(A.device());
  tn5b::gemm::GemmCall c;
  c.A = A.data_ptr(); c.lda = A.stride(0); c.a_mn = a_mn;
  c.B = B.data_ptr(); c.ldb = B.stride(0); c.b_mn = b_mn;
  c.M = int(a_mn ? A.size(1) : A.size(0));
  const int64_t ka = a_mn ? A.size(0) : A.size(1);
  c.N = int(b_mn ? B.size(1) : B.size(0));
  const int64_t kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(ka == kb, "gemm: K mismatch ", ka, " vs ", kb);
  c.K = int(ka);
  TORCH_CHECK(out.size(0) == c.M && out.size(1) == c.N, "gemm: out must be [M, N]");
  c.out = out.data_ptr(); c.ldo = out.stride(0);
  c.epi = int(epi);
  if (bias) { check_bf16(*bias, "bias"); TORCH_CHECK(bias->numel() == c.N && bias->is_contiguous()); c.bias = bias->data_ptr(); }
  if (aux) { check_bf16(*aux, "aux"); check_rows(*aux, "aux"); c.aux = aux->data_ptr(); c.ld_aux = aux->stride(0); }
  if (residual) { check_bf16(*residual, "residual"); check_rows(*residual, "residual"); c.residual = residual->data_ptr(); c.ld_res = residual->stride(0); }
  if (tile_order) { check_cuda(*tile_order, "tile_order"); TORCH_CHECK(tile_order->scalar_type() == at::kInt); c.tile_order = tile_order->data_ptr<int>(); }
  c.bn = int(bn);
  c.max_ctas = int(max_ctas);
  c.pair = int(pair);
  if (group_m > 0) c.group_m = int(group_m);
  c.status = status_ptr(status);
  if (debug) {
    check_cuda(*debug, "debug");
    TORCH_CHECK(debug->scalar_type() == at::kLong && debug->numel() >= 8 * int64_t(tn5b::gemm::grid_ctas(c)),
                "debug must be int64 with 8 words per CTA");
    c.debug = reinterpret_cast<unsigned long long*>(debug->data_ptr<int64_t>());
  }
  raise_if(tn5b::gemm::run(c, stream()), "gemm");
}

// GEMM -> reduce-scatter push: tiles of A*B^T go to their owner rank's slot.
void gemm_rs_push(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, int64_t mode,
                  int64_t recv_ptrs, int64_t flag_ptrs, int64_t rank, int64_t world,
                  int64_t chunk_rows, int64_t epoch, int64_t slot_bytes,
                  const at::Tensor& tile_order, const at::Tensor& status, int64_t timeout_ns,
                  int64_t max_ctas, int64_t delay_tile, int64_t delay_ns) {
  check_bf16(A, "A"); check_bf16(B, "B"); check_rows(A, "A"); check_rows(B, "B");
  const c10::cuda::CUDAGuard guard(A.device());
  tn5b::gemm::GemmCall c;
  c.A = A.data_ptr(); c.lda = A.stride(0); c.a_mn = a_mn;
  c.B = B.data_ptr(); c.ldb = B.stride(0); c.b_mn = b_mn;
  c.M = int(a_mn ? A.size(1) : A.size(0));
  c.N = int(b_mn ? B.size(1) : B.size(0));
  const int64_t ka = a_mn ? A.size(0) : A.size(1);
  const int64_t kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(ka == kb, "gemm_rs: K mismatch");
  c.K = int(ka);
  c.mode = int(mode);
  c.rs_recv = reinterpret_cast<uint8_t* const*>(recv_ptrs);
  c.rs_flags = reinterpret_cast<uint32_t* const*>(flag_ptrs);
  c.rank = int(rank); c.world = int(world); c.chunk_rows = int(chunk_rows);
  c.epoch = uint32_t(epoch); c.slot_bytes = slot_bytes;
  check_cuda(tile_order, "tile_order");
  TORCH_CHECK(tile_order.scalar_type() == at::kInt);
  c.tile_order = tile_order.data_ptr<int>();
  c.status = status_ptr(status);
  c.timeout_ns = uint64_t(timeout_ns);
  c.max_ctas = int(max_ctas);
  c.delay_tile = int(delay_tile);
  c.delay_ns = uint64_t(delay_ns);
  raise_if(tn5b::gemm::run(c, stream()), "gemm_rs_push");
}

// GEMM -> reduce-scatter, pull transport: one launch whose GEMM CTAs store the
// partial tiles of A*B^T into this rank's partial buffer and publish them to
// their owners, while its `comm_ctas` reducer CTAs pull this rank's tiles from
// every source and reduce them (ordered, BF16 after every source) into `out`.
// `phase` (bit1 reduce, bit2 GEMM) splits the launch for single-GPU emulation.
void gemm_rs_pull(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, int64_t partial_local,
                  int64_t partial_ptrs, int64_t flag_ptrs, int64_t my_flags, int64_t rank, int64_t world,
                  int64_t epoch, const at::Tensor& tile_order, const at::Tensor& consumer_order, at::Tensor& out,
                  const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& bias,
                  const at::Tensor& status, int64_t timeout_ns, int64_t comm_ctas, int64_t phase,
                  const c10::optional<at::Tensor>& stamps, const c10::optional<at::Tensor>& produced,
                  int64_t delay_tile, int64_t delay_ns, int64_t max_ctas,
                  const c10::optional<at::Tensor>& cta_stamps, int64_t pair) {
  check_bf16(A, "A"); check_bf16(B, "B"); check_rows(A, "A"); check_rows(B, "B");
  check_bf16(out, "out");
  TORCH_CHECK(out.is_contiguous(), "gemm_rs_pull: out must be contiguous");
  const c10::cuda::CUDAGuard guard(A.device());
  tn5b::gemm::GemmCall c;
  c.A = A.data_ptr(); c.lda = A.stride(0); c.a_mn = a_mn;
  c.B = B.data_ptr(); c.ldb = B.stride(0); c.b_mn = b_mn;
  c.M = int(a_mn ? A.size(1) : A.size(0));
  c.N = int(b_mn ? B.size(1) : B.size(0));
  const int64_t ka = a_mn ? A.size(0) : A.size(1);
  const int64_t kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(ka == kb, "gemm_rs_pull: K mismatch");
  c.K = int(ka);
  TORCH_CHECK(world >= 1 && c.M % world == 0 && out.size(0) == c.M / world && out.size(1) == c.N,
              "gemm_rs_pull: out must be [M / world, N]");
  c.mode = 3;
  c.rs_partial_local = reinterpret_cast<void*>(partial_local);
  c.rs_partials = reinterpret_cast<const uint8_t* const*>(partial_ptrs);
  c.rs_flags = reinterpret_cast<uint32_t* const*>(flag_ptrs);
  c.rs_my_flags = reinterpret_cast<const uint32_t*>(my_flags);
  c.rank = int(rank); c.world = int(world);
  c.epoch = uint32_t(epoch);
  check_cuda(tile_order, "tile_order");
  TORCH_CHECK(tile_order.scalar_type() == at::kInt);
  c.tile_order = tile_order.data_ptr<int>();
  check_cuda(consumer_order, "consumer_order");
  TORCH_CHECK(consumer_order.scalar_type() == at::kInt);
  c.rs_consumer_order = consumer_order.data_ptr<int>();
  c.rs_out = out.data_ptr();
  if (residual) {
    check_bf16(*residual, "residual");
    TORCH_CHECK(residual->is_contiguous() && residual->sizes() == out.sizes(), "residual must match out");
    c.rs_residual = residual->data_ptr();
  }
  if (bias) {
    check_bf16(*bias, "bias");
    TORCH_CHECK(bias->is_contiguous() && bias->numel() == c.N, "bias must be [N]");
    c.rs_bias = bias->data_ptr();
  }
  if (stamps) {
    TORCH_CHECK(stamps->is_cuda() && stamps->scalar_type() == at::kLong, "stamps must be CUDA int64");
    c.rs_stamps = reinterpret_cast<unsigned long long*>(stamps->data_ptr<int64_t>());
  }
  if (produced) {
    TORCH_CHECK(produced->is_cuda() && produced->scalar_type() == at::kLong, "produced must be CUDA int64");
    c.rs_produced = reinterpret_cast<unsigned long long*>(produced->data_ptr<int64_t>());
  }
  c.status = status_ptr(status);
  c.timeout_ns = uint64_t(timeout_ns);
  c.comm_ctas = int(comm_ctas);
  c.phase = int(phase);
  c.delay_tile = int(delay_tile);
  c.delay_ns = uint64_t(delay_ns);
  c.max_ctas = int(max_ctas);
  c.pair = int(pair);
  if (cta_stamps) {
    TORCH_CHECK(cta_stamps->is_cuda() && cta_stamps->scalar_type() == at::kLong &&
                    cta_stamps->numel() >= 2 * int64_t(tn5b::gemm::grid_ctas(c)),
                "cta_stamps must be CUDA int64 with 2 words per CTA");
    c.cta_stamps = reinterpret_cast<unsigned long long*>(cta_stamps->data_ptr<int64_t>());
  }
  raise_if(tn5b::gemm::run(c, stream()), "gemm_rs_pull");
}

// The reducer CTAs of the pull reduce-scatter alone (phase 2), for partials
// that were packed and published without a GEMM (single-CTA flag tiles).  The
// GEMM operands of the call are never read: the partial buffer stands in.
void rs_pull_reduce_only(int64_t partial_local, int64_t partial_ptrs, int64_t flag_ptrs, int64_t my_flags,
                         int64_t M, int64_t N, int64_t rank, int64_t world, int64_t epoch,
                         const at::Tensor& consumer_order, at::Tensor& out, const at::Tensor& status,
                         int64_t timeout_ns, int64_t comm_ctas) {
  check_bf16(out, "out");
  TORCH_CHECK(out.is_contiguous() && out.size(0) == M / world && out.size(1) == N, "out must be [M / world, N]");
  const c10::cuda::CUDAGuard guard(out.device());
  tn5b::gemm::GemmCall c;
  c.A = reinterpret_cast<const void*>(partial_local); c.lda = 64;
  c.B = reinterpret_cast<const void*>(partial_local); c.ldb = 64;
  c.M = int(M); c.N = int(N); c.K = 64;
  c.mode = 3; c.phase = 2; c.pair = 0;
  c.rs_partial_local = reinterpret_cast<void*>(partial_local);
  c.rs_partials = reinterpret_cast<const uint8_t* const*>(partial_ptrs);
  c.rs_flags = reinterpret_cast<uint32_t* const*>(flag_ptrs);
  c.rs_my_flags = reinterpret_cast<const uint32_t*>(my_flags);
  c.rank = int(rank); c.world = int(world); c.epoch = uint32_t(epoch);
  check_cuda(consumer_order, "consumer_order");
  c.rs_consumer_order = consumer_order.data_ptr<int>();
  c.tile_order = consumer_order.data_ptr<int>();  // not read in the reduce phase
  c.rs_out = out.data_ptr();
  c.status = status_ptr(status);
  c.timeout_ns = uint64_t(timeout_ns);
  c.comm_ctas = int(comm_ctas);
  raise_if(tn5b::gemm::run(c, stream()), "rs_pull_reduce_only");
}

// All-gather -> GEMM, pull transport: out = epilogue(gather(shards) * B^T).
// `gather` is this rank's symmetric gather buffer [M, K]; its gatherer CTAs
// pull the peers' chunks into it while the GEMM CTAs consume arrived blocks
// (the own chunk straight from `shard`).  published_* are the ranks' block
// flags [world][M / world / 128], pulled_* their "finished reading" counters.
void ag_gemm(const at::Tensor& shard, const at::Tensor& gather, const at::Tensor& B, bool b_mn,
             at::Tensor& out, int64_t epi, const c10::optional<at::Tensor>& bias,
             const c10::optional<at::Tensor>& aux, int64_t gather_ptrs, int64_t published_ptrs,
             int64_t pulled_ptrs, int64_t published_local, int64_t pulled_local, const at::Tensor& ready,
             int64_t rank, int64_t world, int64_t epoch, int64_t pulled_target, int64_t ready_target,
             const at::Tensor& tile_order, const at::Tensor& status, int64_t timeout_ns, int64_t bn,
             int64_t comm_ctas, int64_t phase, const c10::optional<at::Tensor>& cta_stamps,
             const c10::optional<at::Tensor>& block_stamps, int64_t pair) {
  check_bf16(shard, "shard"); check_bf16(gather, "gather"); check_bf16(B, "B"); check_bf16(out, "out");
  TORCH_CHECK(shard.is_contiguous() && gather.is_contiguous(), "shard/gather must be contiguous");
  check_rows(B, "B"); check_rows(out, "out");
  const c10::cuda::CUDAGuard guard(gather.device());
  tn5b::gemm::GemmCall c;
  c.A = gather.data_ptr(); c.lda = gather.stride(0); c.a_mn = 0;
  c.B = B.data_ptr(); c.ldb = B.stride(0); c.b_mn = b_mn;
  c.M = int(gather.size(0)); c.K = int(gather.size(1));
  c.N = int(b_mn ? B.size(1) : B.size(0));
  TORCH_CHECK((b_mn ? B.size(0) : B.size(1)) == c.K, "ag_gemm: K mismatch");
  TORCH_CHECK(out.size(0) == c.M && out.size(1) == c.N, "ag_gemm: out must be [M, N]");
  TORCH_CHECK(shard.numel() * world == gather.numel(), "ag_gemm: shard size mismatch");
  c.out = out.data_ptr(); c.ldo = out.stride(0);
  c.epi = int(epi);
  if (bias) {
    check_bf16(*bias, "bias");
    TORCH_CHECK(bias->is_contiguous() && bias->numel() == c.N, "ag_gemm: bias must be a contiguous [N]");
    c.bias = bias->data_ptr();
  }
  if (aux) { check_bf16(*aux, "aux"); check_rows(*aux, "aux"); c.aux = aux->data_ptr(); c.ld_aux = aux->stride(0); }
  TORCH_CHECK(ready.is_cuda() && ready.scalar_type() == at::kInt &&
                  ready.numel() >= world * (c.M / world / 128) * tn5b::gemm::kReadyStride,
              "ag_gemm: ready must be int32 [world * blocks * ", tn5b::gemm::kReadyStride, "]");
  c.ag = 1;
  c.rank = int(rank); c.world = int(world);
  c.ag_shard = shard.data_ptr();
  // A shard that already is this rank's chunk of the gather buffer is published in place.
  c.ag_own_in_place = shard.data_ptr() == static_cast<void*>(static_cast<uint8_t*>(gather.data_ptr()) +
                                                             rank * shard.numel() * 2);
  c.ag_gather = reinterpret_cast<uint8_t* const*>(gather_ptrs);
  c.ag_published = reinterpret_cast<uint32_t* const*>(published_ptrs);
  c.ag_pulled = reinterpret_cast<uint32_t* const*>(pulled_ptrs);
  c.ag_published_local = reinterpret_cast<const uint32_t*>(published_local);
  c.ag_pulled_local = reinterpret_cast<const uint32_t*>(pulled_local);
  c.ag_ready = reinterpret_cast<uint32_t*>(ready.data_ptr<int>());
  c.ag_epoch = uint32_t(epoch);
  c.ag_pulled_target = uint32_t(pulled_target);
  c.ag_ready_target = uint32_t(ready_target);
  check_cuda(tile_order, "tile_order");
  c.tile_order = tile_order.data_ptr<int>();
  c.status = status_ptr(status);
  c.timeout_ns = uint64_t(timeout_ns);
  c.bn = int(bn);
  c.comm_ctas = int(comm_ctas);
  c.phase = int(phase);
  c.pair = int(pair);
  if (cta_stamps) {
    TORCH_CHECK(cta_stamps->is_cuda() && cta_stamps->scalar_type() == at::kLong &&
                    cta_stamps->numel() >= 2 * int64_t(tn5b::gemm::grid_ctas(c)),
                "cta_stamps must be CUDA int64 with 2 words per CTA");
    c.cta_stamps = reinterpret_cast<unsigned long long*>(cta_stamps->data_ptr<int64_t>());
  }
  if (block_stamps) {
    TORCH_CHECK(block_stamps->is_cuda() && block_stamps->scalar_type() == at::kLong &&
                    block_stamps->numel() >= world * (c.M / world / 128),
                "block_stamps must be CUDA int64 [world * blocks]");
    c.ag_block_stamps = reinterpret_cast<unsigned long long*>(block_stamps->data_ptr<int64_t>());
  }
  raise_if(tn5b::gemm::run(c, stream()), "ag_gemm");
}

// Grid of a fused launch (GEMM CTAs + communication CTAs) for profiling buffers.
int64_t fused_grid(int64_t M, int64_t N, int64_t K, int64_t mode, int64_t ag, int64_t bn, int64_t comm_ctas,
                   int64_t phase, int64_t pair) {
  tn5b::gemm::GemmCall c;
  c.M = int(M); c.N = int(N); c.K = int(K); c.mode = int(mode); c.ag = int(ag); c.bn = int(bn);
  c.comm_ctas = int(comm_ctas); c.phase = int(phase); c.pair = int(pair);
  return tn5b::gemm::grid_ctas(c);
}

int64_t fused_tile_kind(int64_t M, int64_t N, int64_t K, int64_t comm_ctas) {
  return tn5b::gemm::fused_tile_kind(int(M), int(N), int(K), int(comm_ctas));
}

// Mapping probe: the (tile_m, tile_n) pairs the GEMM kernel's CTAs decode for
// each linear tile index of a call of this shape, tile kind and tile order.
at::Tensor gemm_tile_map(int64_t M, int64_t N, int64_t K, int64_t mode, int64_t pair,
                         const c10::optional<at::Tensor>& tile_order, int64_t device) {
  const c10::cuda::CUDAGuard guard(c10::Device(c10::kCUDA, int(device)));
  tn5b::gemm::GemmCall c;
  c.M = int(M); c.N = int(N); c.K = int(K); c.mode = int(mode); c.pair = int(pair);
  if (tile_order) {
    check_cuda(*tile_order, "tile_order");
    TORCH_CHECK(tile_order->scalar_type() == at::kInt);
    c.tile_order = tile_order->data_ptr<int>();
    TORCH_CHECK(tile_order->numel() == tn5b::gemm::tile_count(c), "tile_order length differs from the tile count");
  }
  auto out = at::empty({int64_t(tn5b::gemm::tile_count(c)), 2},
                       at::TensorOptions().dtype(at::kInt).device(at::kCUDA, int(device)));
  raise_if(tn5b::gemm::tile_map(c, out.data_ptr<int>(), stream()), "gemm_tile_map");
  return out;
}

// Number of SMs of the current device.
int64_t sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

}  // namespace

void register_kernels(pybind11::module& m);
void register_comm(pybind11::module& m);

// The push transport's lane layout as the kernels compute it (push_lanes.h):
// (lane_slot_bytes, recv_bytes, flag_words, flag index of every (source, local tile)).
std::tuple<int64_t, int64_t, int64_t, at::Tensor> push_lanes_layout(int64_t rows, int64_t n, int64_t chunk_rows,
                                                                    int64_t world, int64_t tile_n) {
  TORCH_CHECK(chunk_rows > 0 && chunk_rows % 128 == 0 && rows % chunk_rows == 0 && n % tile_n == 0,
              "push lanes: 128 | chunk_rows, chunk_rows | rows, tile_n | n");
  const tn5b::PushLanes L{int(rows), int(n), int(chunk_rows), int(world), int(tile_n)};
  const int tiles_n = int(n / tile_n), tiles = int(rows / 128) * tiles_n;
  at::Tensor idx = at::empty({world, tiles}, at::kLong);
  auto a = idx.accessor<int64_t, 2>();
  for (int s = 0; s < world; ++s)
    for (int t = 0; t < tiles; ++t) a[s][t] = L.flag_index(s, (t / tiles_n) * 128, t % tiles_n);
  return {L.lane_slot_bytes(), L.recv_bytes(), L.flag_words(), idx};
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "tempname_5090_b200 native sm_100a kernels";
  using nogil = pybind11::call_guard<pybind11::gil_scoped_release>;
  m.def("gemm", &gemm, "tcgen05 BF16 GEMM with fused epilogue", nogil());
  m.def("gemm_rs_push", &gemm_rs_push, "tcgen05 GEMM whose epilogue pushes tiles to owners", nogil());
  m.def("gemm_rs_pull", &gemm_rs_pull, "tcgen05 GEMM with in-launch pull reduce-scatter", nogil());
  m.def("rs_pull_reduce_only", &rs_pull_reduce_only, "pull reduce-scatter of packed, published partials", nogil());
  m.def("ag_gemm", &ag_gemm, "all-gather (in-launch pull) fused into a tcgen05 GEMM", nogil());
  m.def("sm_count", &sm_count, "number of SMs of the current device");
  m.def("push_lanes_layout", &push_lanes_layout, "push transport lane layout as the kernels compute it");
  m.def("fused_grid", &fused_grid, "grid of a fused GEMM launch (GEMM + communication CTAs)");
  m.def("fused_tile_kind", &fused_tile_kind, "tile kind the wave model picks for a fused launch");
  m.def("gemm_tile_map", &gemm_tile_map, "device read-back of the GEMM tile order (mapping probe)");
  register_kernels(m);
  register_comm(m);
}
