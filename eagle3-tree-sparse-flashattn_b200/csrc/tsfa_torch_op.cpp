// PyTorch operator binding of libtsfa: torch.ops.tsfa.*
//
// A thin layer over the C ABI (include/tsfa.h) that makes the verify-step
// attention a dispatcher-visible operator, so that torch.compile, CUDA-graph
// capture and fake-tensor tracing see it as one op instead of an opaque
// ctypes call.  It replaces the Triton launch of the reference's bridge
// (eagle_tree_sparse_bridge.py:108-158: out = empty_like(q), grid over
// (q-block, batch x head), 35 kernel arguments) with one call of
// tsfa_run_tree_sparse on the current stream.
//
//   tsfa::run_tree_sparse(q, k, v, tree_mask, prefix_len, block_m, block_n, sm_scale) -> out
//       metadata build from the mask + forward (tsfa_run_tree_sparse)
//   tsfa::build_metadata(tree_mask, block_m, block_n)
//       -> (row_ptr, col_idx, blk_type, mixed_mask_payload, mixed_mask_offset, counts)
//       K1 at fixed capacity (n_q_blocks * n_tree_blocks tiles) with
//       counts = {nnz, n_mixed} on the device: no host read, so it traces and
//       captures; the reference-sized tensors are the first nnz entries.
//   tsfa::workspace(device, nbytes)
//       the per-(device, stream) work buffer the ops use, shared with the
//       ctypes binding's calls (eager helper, not for tracing).
//
// Every tensor argument must be a CUDA tensor; the kernels are in libtsfa.so
// and there is no CPU implementation.  The Meta implementations give the
// output shapes for tracing.  Errors map to c10::Error with the library's
// status text (the Python layer re-raises the reference's exception types).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cmath>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "tsfa.h"

namespace {

int mask_code(const at::Tensor& m) {
  switch (m.scalar_type()) {
    case at::kBool: case at::kByte: case at::kChar: return TSFA_MASK_B8;
    case at::kShort: return TSFA_MASK_I16;
    case at::kInt: return TSFA_MASK_I32;
    case at::kLong: return TSFA_MASK_I64;
    case at::kHalf: return TSFA_MASK_F16;
    case at::kBFloat16: return TSFA_MASK_BF16;
    case at::kFloat: return TSFA_MASK_F32;
    case at::kDouble: return TSFA_MASK_F64;
    default: TORCH_CHECK_TYPE(false, "tsfa: unsupported tree_mask dtype ", m.scalar_type());
  }
  return -1;
}

// Status -> exception: ValueError for TSFA_ERR_VALUE (the reference's
// ValueErrors, tsfa.py:85-88 and bridge.py:91-93), NotImplementedError for a
// shape or layout this build does not handle, RuntimeError otherwise.
void check_status(int st, const char* what) {
  if (st == TSFA_OK) return;
  TORCH_CHECK_VALUE(st != TSFA_ERR_VALUE, what, ": ", tsfa_status_string(st), " (status ", st, ")");
  TORCH_CHECK_NOT_IMPLEMENTED(st != TSFA_ERR_UNSUPPORTED, what, ": ", tsfa_status_string(st), " (status ", st, ")");
  if (st == TSFA_ERR_CUDA)
    TORCH_CHECK(false, what, ": ", tsfa_status_string(st), " (status ", st, ") [", tsfa_last_error(), "]");
  TORCH_CHECK(false, what, ": ", tsfa_status_string(st), " (status ", st, ")");
}

// One work buffer per (device, stream), grown on demand; its first
// TSFA_SYNC_BYTES are zeroed once when it is allocated (the kernels leave
// their counters at zero).
at::Tensor workspace(size_t bytes, const at::Device& dev, cudaStream_t stream) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, at::Tensor> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto& buf = cache[{dev.index(), stream}];
  if (!buf.defined() || (size_t)buf.numel() < bytes) {
    size_t n = std::max<size_t>(std::max<size_t>(bytes, TSFA_SYNC_BYTES), 1u << 20);
    size_t p2 = 1;
    while (p2 < n) p2 <<= 1;
    buf = at::empty({(int64_t)p2}, at::TensorOptions().dtype(at::kByte).device(dev));
    buf.narrow(0, 0, TSFA_SYNC_BYTES).zero_();
  }
  return buf;
}

int qkv_code(const at::Tensor& t) {
  if (t.scalar_type() == at::kBFloat16) return TSFA_DTYPE_BF16;
  if (t.scalar_type() == at::kHalf) return TSFA_DTYPE_F16;
  TORCH_CHECK_TYPE(false, "tsfa: query/key/value must be bfloat16 or float16, got ", t.scalar_type());
  return -1;
}

// TMA wants unit stride on head_dim, 16-byte aligned rows and base: views
// that have them are used in place, others get one contiguous copy.
at::Tensor kernel_ready(const at::Tensor& t) {
  bool ok = t.stride(3) == 1 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15u) == 0;
  for (int i = 0; i < 3; ++i) ok = ok && t.stride(i) % 8 == 0;
  return ok ? t : t.contiguous();
}

at::Tensor run_tree_sparse_cuda(const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in,
                                const at::Tensor& tree_mask, int64_t prefix_len, int64_t block_m, int64_t block_n,
                                double sm_scale) {
  TORCH_CHECK(q_in.is_cuda() && k_in.is_cuda() && v_in.is_cuda() && tree_mask.is_cuda(),
              "tsfa: CUDA tensors expected");
  TORCH_CHECK(q_in.dim() == 4 && k_in.dim() == 4 && v_in.dim() == 4, "tsfa: q, k, v must be 4-D");
  const at::Tensor q = kernel_ready(q_in), k = kernel_ready(k_in), v = kernel_ready(v_in);
  TORCH_CHECK(tree_mask.dim() == 2, "tsfa: tree_mask must be [q_len, q_len]");
  const c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
  at::Tensor mask = tree_mask.numel() && tree_mask.stride(1) != 1 ? tree_mask.contiguous() : tree_mask;
  at::Tensor out = at::empty(q.sizes(), q.options().memory_format(at::MemoryFormat::Contiguous));
  TsfaFwdArgs a{};
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.o = out.data_ptr();
  for (int i = 0; i < 4; ++i) {
    a.q_stride[i] = q.stride(i);
    a.k_stride[i] = k.stride(i);
    a.v_stride[i] = v.stride(i);
    a.o_stride[i] = out.stride(i);
  }
  a.batch = (int32_t)q.size(0);
  a.num_heads = (int32_t)q.size(1);
  a.q_len = (int32_t)q.size(2);
  a.head_dim = (int32_t)q.size(3);
  a.num_kv_heads = (int32_t)k.size(1);
  a.kv_len = (int32_t)k.size(2);
  a.prefix_len = (int32_t)prefix_len;
  a.dtype = qkv_code(q);
  TORCH_CHECK(k.scalar_type() == q.scalar_type() && v.scalar_type() == q.scalar_type(),
              "tsfa: q, k, v must share one dtype");
  TORCH_CHECK(k.sizes() == v.sizes() && k.size(0) == q.size(0) && k.size(3) == q.size(3),
              "tsfa: shape mismatch between query/key/value");
  a.sm_scale = (float)sm_scale;
  a.block_m = (int32_t)block_m;
  a.block_n = (int32_t)block_n;
  size_t need = 0;
  check_status(tsfa_run_workspace_bytes(&a, &need), "tsfa_run_workspace_bytes");
  at::Tensor ws = workspace(need, q.device(), stream);
  const int64_t T = q.size(2);
  check_status(tsfa_run_tree_sparse(&a, mask.numel() ? mask.data_ptr() : nullptr, mask_code(mask),
                                    mask.numel() ? mask.stride(0) : T, ws.data_ptr(), (size_t)ws.numel(), stream),
               "tsfa_run_tree_sparse");
  return out;
}

at::Tensor run_tree_sparse_meta(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                const at::Tensor& tree_mask, int64_t prefix_len, int64_t block_m, int64_t block_n,
                                double sm_scale) {
  return at::empty(q.sizes(), q.options().memory_format(at::MemoryFormat::Contiguous));
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor> meta_buffers(
    const at::Tensor& mask, int64_t block_m, int64_t block_n) {
  TsfaMetaDims d{};
  check_status(tsfa_meta_dims((int32_t)mask.size(0), (int32_t)block_m, (int32_t)block_n, &d), "tsfa_meta_dims");
  auto i32 = mask.options().dtype(at::kInt);
  return {at::empty({d.n_q_blocks + 1}, i32), at::empty({d.tile_capacity}, i32),
          at::empty({d.tile_capacity}, mask.options().dtype(at::kChar)), at::empty({d.payload_capacity}, i32),
          at::empty({d.tile_capacity}, i32), at::empty({2}, i32)};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor> build_metadata_cuda(
    const at::Tensor& tree_mask, int64_t block_m, int64_t block_n) {
  TORCH_CHECK(tree_mask.is_cuda(), "tsfa: CUDA tensor expected");
  TORCH_CHECK(tree_mask.dim() == 2 && tree_mask.size(0) == tree_mask.size(1), "tree_mask must be square");
  const c10::cuda::CUDAGuard guard(tree_mask.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(tree_mask.device().index()).stream();
  at::Tensor mask = tree_mask.numel() && tree_mask.stride(1) != 1 ? tree_mask.contiguous() : tree_mask;
  auto bufs = meta_buffers(mask, block_m, block_n);
  TsfaMeta m{};
  m.row_ptr = std::get<0>(bufs).data_ptr<int32_t>();
  m.col_idx = std::get<1>(bufs).numel() ? std::get<1>(bufs).data_ptr<int32_t>() : nullptr;
  m.blk_type = std::get<2>(bufs).numel() ? std::get<2>(bufs).data_ptr<int8_t>() : nullptr;
  m.mixed_mask_payload = std::get<3>(bufs).numel() ? std::get<3>(bufs).data_ptr<int32_t>() : nullptr;
  m.mixed_mask_offset = std::get<4>(bufs).numel() ? std::get<4>(bufs).data_ptr<int32_t>() : nullptr;
  m.counts = std::get<5>(bufs).data_ptr<int32_t>();
  const int32_t T = (int32_t)mask.size(0);
  size_t need = 0;
  check_status(tsfa_meta_workspace_bytes(T, (int32_t)block_m, (int32_t)block_n, &need), "tsfa_meta_workspace_bytes");
  at::Tensor ws = workspace(need, mask.device(), stream);
  check_status(tsfa_meta_build(mask.numel() ? mask.data_ptr() : nullptr, mask_code(mask),
                               mask.numel() ? mask.stride(0) : T, T, (int32_t)block_m, (int32_t)block_n, &m,
                               ws.data_ptr(), (size_t)ws.numel(), stream),
               "tsfa_meta_build");
  return bufs;
}

// The work buffer the ops use on `device` and its current stream, at least
// `nbytes` long: the Python binding's other native calls share it, so the
// device status block read after any of them is this one.
at::Tensor workspace_op(c10::Device device, int64_t nbytes) {
  TORCH_CHECK(device.is_cuda(), "tsfa: workspace on a CUDA device expected");
  const c10::cuda::CUDAGuard guard(device);
  at::Device dev(at::kCUDA, c10::cuda::current_device());
  return workspace((size_t)std::max<int64_t>(nbytes, 0), dev, c10::cuda::getCurrentCUDAStream(dev.index()).stream());
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor> build_metadata_meta(
    const at::Tensor& tree_mask, int64_t block_m, int64_t block_n) {
  return meta_buffers(tree_mask, block_m, block_n);
}

}  // namespace

TORCH_LIBRARY(tsfa, m) {
  m.def("run_tree_sparse(Tensor q, Tensor k, Tensor v, Tensor tree_mask, int prefix_len, int block_m, "
        "int block_n, float sm_scale) -> Tensor");
  m.def("build_metadata(Tensor tree_mask, int block_m, int block_n) -> (Tensor, Tensor, Tensor, Tensor, "
        "Tensor, Tensor)");
  // eager helper for the binding's other calls (not meant for tracing)
  m.def("workspace(Device device, int nbytes) -> Tensor", &workspace_op);
}

TORCH_LIBRARY_IMPL(tsfa, CUDA, m) {
  m.impl("run_tree_sparse", &run_tree_sparse_cuda);
  m.impl("build_metadata", &build_metadata_cuda);
}

TORCH_LIBRARY_IMPL(tsfa, Meta, m) {
  m.impl("run_tree_sparse", &run_tree_sparse_meta);
  m.impl("build_metadata", &build_metadata_meta);
}
