// PyTorch adapter for libtpsa: registers the reference operator schemas on
// the CUDA dispatch key.  Mirrors the reference adapter
// operator/torch_adapter/triangle_paged_attention_torch.cpp (checks :29-97,
// functional :101-138, out :140-178, workspace :180-261, registrations
// :265-304) with the NPU device replaced by CUDA and aclnn replaced by the
// C ABI in include/tpsa.h.
#include <ATen/ATen.h>
#include <ATen/MemoryOverlap.h>
#include <c10/core/DeviceGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "../../include/tpsa.h"

namespace trianglemix_b200 {
namespace {

void check_inputs(const at::Tensor& query, const at::Tensor& key_cache,
                  const at::Tensor& value_cache, const at::Tensor& block_table) {
  TORCH_CHECK(query.is_cuda(), "query must be a CUDA tensor");
  TORCH_CHECK(key_cache.is_cuda() && value_cache.is_cuda() && block_table.is_cuda(),
              "key_cache, value_cache, and block_table must be CUDA tensors");
  TORCH_CHECK(query.scalar_type() == at::ScalarType::BFloat16, "query must be BF16");
  TORCH_CHECK(key_cache.scalar_type() == at::ScalarType::BFloat16 &&
                  value_cache.scalar_type() == at::ScalarType::BFloat16,
              "key_cache and value_cache must be BF16");
  TORCH_CHECK(block_table.scalar_type() == at::ScalarType::Int, "block_table must be INT32");
  TORCH_CHECK(query.device() == key_cache.device() && query.device() == value_cache.device() &&
                  query.device() == block_table.device(),
              "all inputs must be on the same CUDA device");
  TORCH_CHECK(query.is_contiguous() && key_cache.is_contiguous() &&
                  value_cache.is_contiguous() && block_table.is_contiguous(),
              "all inputs must be contiguous");
  TORCH_CHECK(query.dim() == 3 && query.size(1) == TPSA_QUERY_HEADS &&
                  query.size(2) == TPSA_HEAD_DIM,
              "query must be [Tq, 32, 128]");
  TORCH_CHECK(key_cache.dim() == 4 && key_cache.size(1) == TPSA_PAGE_SIZE &&
                  key_cache.size(2) == TPSA_KV_HEADS && key_cache.size(3) == TPSA_HEAD_DIM,
              "key_cache must be [pages, 128, 8, 128]");
  TORCH_CHECK(value_cache.sizes() == key_cache.sizes(),
              "value_cache shape must equal key_cache shape");
  TORCH_CHECK(block_table.dim() == 2 && block_table.size(0) == 1,
              "block_table must be [1, max_pages]");
}

void check_output(const at::Tensor& query, const at::Tensor& key_cache,
                  const at::Tensor& value_cache, const at::Tensor& block_table,
                  const at::Tensor& output) {
  TORCH_CHECK(output.is_cuda(), "out must be a CUDA tensor");
  TORCH_CHECK(output.device() == query.device(), "out must be on the same CUDA device as query");
  TORCH_CHECK(output.scalar_type() == at::ScalarType::BFloat16, "out must be BF16");
  TORCH_CHECK(output.sizes() == query.sizes(), "out shape must exactly match query");
  TORCH_CHECK(output.is_contiguous(), "out must be contiguous");
  at::assert_no_internal_overlap(output);
  at::assert_no_overlap(output, query);
  at::assert_no_overlap(output, key_cache);
  at::assert_no_overlap(output, value_cache);
  at::assert_no_overlap(output, block_table);
}

void check_status(tpsa_status status) {
  TORCH_CHECK(status == TPSA_OK, tpsa_last_error()[0] != '\0' ? tpsa_last_error()
                                                              : tpsa_status_string(status));
}

void run(const at::Tensor& query, const at::Tensor& key_cache, const at::Tensor& value_cache,
         const at::Tensor& block_table, int64_t query_start, int64_t seq_len, int64_t prompt_len,
         double scale, at::Tensor& output) {
  uint64_t bytes = 0;
  check_status(tpsa_workspace_size(query.size(0), query_start, seq_len, prompt_len, &bytes));
  at::Tensor workspace;
  if (bytes > 0) {
    workspace = at::empty({static_cast<int64_t>(bytes)},
                          query.options().dtype(at::ScalarType::Byte));
  }
  const auto stream = c10::cuda::getCurrentCUDAStream(query.device().index());
  check_status(tpsa_paged_attention(
      query.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
      block_table.data_ptr<int32_t>(), output.data_ptr(), query.size(0), key_cache.size(0),
      block_table.size(1), query_start, seq_len, prompt_len, static_cast<float>(scale),
      bytes > 0 ? workspace.data_ptr() : nullptr, bytes, stream.stream()));
}

}  // namespace

at::Tensor triangle_paged_sparse_attention(const at::Tensor& query, const at::Tensor& key_cache,
                                           const at::Tensor& value_cache,
                                           const at::Tensor& block_table, int64_t query_start,
                                           int64_t seq_len, int64_t prompt_len, double scale) {
  check_inputs(query, key_cache, value_cache, block_table);
  c10::OptionalDeviceGuard device_guard(query.device());
  at::Tensor output = at::empty_like(query);
  run(query, key_cache, value_cache, block_table, query_start, seq_len, prompt_len, scale, output);
  return output;
}

at::Tensor& triangle_paged_sparse_attention_out(const at::Tensor& query,
                                                const at::Tensor& key_cache,
                                                const at::Tensor& value_cache,
                                                const at::Tensor& block_table,
                                                int64_t query_start, int64_t seq_len,
                                                int64_t prompt_len, double scale,
                                                at::Tensor& output) {
  check_inputs(query, key_cache, value_cache, block_table);
  check_output(query, key_cache, value_cache, block_table, output);
  c10::OptionalDeviceGuard device_guard(query.device());
  run(query, key_cache, value_cache, block_table, query_start, seq_len, prompt_len, scale, output);
  return output;
}

int64_t triangle_paged_sparse_attention_workspace_size(
    const at::Tensor& query, const at::Tensor& key_cache, const at::Tensor& value_cache,
    const at::Tensor& block_table, int64_t query_start, int64_t seq_len, int64_t prompt_len,
    double scale) {
  check_inputs(query, key_cache, value_cache, block_table);
  c10::OptionalDeviceGuard device_guard(query.device());
  (void)scale;
  uint64_t bytes = 0;
  check_status(tpsa_workspace_size(query.size(0), query_start, seq_len, prompt_len, &bytes));
  return static_cast<int64_t>(bytes);
}

}  // namespace trianglemix_b200

TORCH_LIBRARY(trianglemix_reference, ops) {
  ops.def(
      "triangle_paged_sparse_attention("
      "Tensor query, Tensor key_cache, Tensor value_cache, "
      "Tensor block_table, int query_start, int seq_len, "
      "int prompt_len, float scale) -> Tensor");
  ops.def(
      "triangle_paged_sparse_attention_workspace_size("
      "Tensor query, Tensor key_cache, Tensor value_cache, "
      "Tensor block_table, int query_start, int seq_len, "
      "int prompt_len, float scale) -> int");
}

TORCH_LIBRARY_IMPL(trianglemix_reference, CUDA, ops) {
  ops.impl("triangle_paged_sparse_attention", &trianglemix_b200::triangle_paged_sparse_attention);
  ops.impl("triangle_paged_sparse_attention_workspace_size",
           &trianglemix_b200::triangle_paged_sparse_attention_workspace_size);
}

TORCH_LIBRARY_FRAGMENT(trianglemix, ops) {
  ops.def(
      "triangle_paged_sparse_attention.out("
      "Tensor query, Tensor key_cache, Tensor value_cache, "
      "Tensor block_table, int query_start, int seq_len, "
      "int prompt_len, float scale, *, Tensor(a!) out) -> Tensor(a!)");
}

TORCH_LIBRARY_IMPL(trianglemix, CUDA, ops) {
  ops.impl("triangle_paged_sparse_attention.out",
           &trianglemix_b200::triangle_paged_sparse_attention_out);
}

// The name the reference registers from its in-tree vLLM-Ascend build
// (README.md:34-36 of the reference: torch.ops._C_ascend.
// npu_triangle_paged_sparse_attention, an out-variant operator), bound to the
// same out implementation: same arguments, same gates, caller-owned output.
TORCH_LIBRARY_FRAGMENT(_C_ascend, ops) {
  ops.def(
      "npu_triangle_paged_sparse_attention("
      "Tensor query, Tensor key_cache, Tensor value_cache, "
      "Tensor block_table, int query_start, int seq_len, "
      "int prompt_len, float scale, *, Tensor(a!) out) -> Tensor(a!)");
}

TORCH_LIBRARY_IMPL(_C_ascend, CUDA, ops) {
  ops.impl("npu_triangle_paged_sparse_attention",
           &trianglemix_b200::triangle_paged_sparse_attention_out);
}
