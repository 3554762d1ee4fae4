// torch operator registration of the drop-in kernels: torch.ops.omni_b200.*
//
// A thin layer over the C ABI of libomni_b200.so (include/omni_b200.h): each op
// checks its tensors, takes the current CUDA stream of the tensors' device and
// calls the matching omni_* entry point; a non-zero return code raises with the
// library's message.  Registering the ops with the dispatcher (TORCH_LIBRARY)
// makes them visible to torch.compile (fake kernels are registered from Python in
// omni_b200/torch_ops.py) and capturable in CUDA graphs (no host reads, no
// allocation but the op's own outputs).  Schemas follow the reference's Python
// signatures of these kernels:
//   sample_topk_topp           sglang_omni/models/qwen3_tts/sampling_kernels.py:836-846
//   gather_codec_embedding_and_add  sglang_omni/models/qwen3_tts/predictor_kernels.py:87-94
//   codebook_step              sglang_omni/utils/predictor_layers.py:963-968
//   add_rmsnorm_rounded        sglang_omni/utils/predictor_layers.py:603-622
//   paged_decode_attention     RadixAttention decode (qwen3_omni/components/thinker_model.py:373-379)
//   linear                     the bf16 projections (nn.Linear layout)
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "omni_b200.h"

namespace {

void* stream_of(const at::Tensor& t) { return c10::cuda::getCurrentCUDAStream(t.get_device()).stream(); }

void check_rc(int rc, const char* op) { TORCH_CHECK(rc == 0, "omni_b200::", op, ": ", omni_last_error()); }

void check_rows(const at::Tensor& t, int64_t rows, at::ScalarType dt, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 1 && t.size(0) == rows && t.is_contiguous() && t.scalar_type() == dt,
              name, " must be a contiguous CUDA vector of ", rows, " ", c10::toString(dt));
}

at::Tensor sample_topk_topp(const at::Tensor& logits, const at::Tensor& temperatures, const at::Tensor& top_ks,
                            const at::Tensor& top_ps, const at::Tensor& seeds, const at::Tensor& positions,
                            int64_t max_top_k, bool has_top_p) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1,
              "logits must be bf16 [rows, vocab] with unit column stride");
  const int64_t rows = logits.size(0);
  check_rows(temperatures, rows, at::kFloat, "temperatures");
  check_rows(top_ks, rows, at::kLong, "top_ks");
  check_rows(top_ps, rows, at::kFloat, "top_ps");
  check_rows(seeds, rows, at::kLong, "seeds");
  check_rows(positions, rows, at::kLong, "positions");
  c10::cuda::CUDAGuard g(logits.device());
  auto out = at::empty({rows}, logits.options().dtype(at::kLong));
  if (rows == 0) return out;
  check_rc(omni_sample_topk_topp(logits.data_ptr(), rows, logits.size(1), logits.stride(0),
                                 temperatures.data_ptr<float>(), top_ks.data_ptr<int64_t>(), top_ps.data_ptr<float>(),
                                 seeds.data_ptr<int64_t>(), positions.data_ptr<int64_t>(), (int32_t)max_top_k,
                                 has_top_p ? 1 : 0, out.data_ptr<int64_t>(), stream_of(logits)),
           "sample_topk_topp");
  return out;
}

bool gather_codec_embedding_and_add(const at::Tensor& token_ids, const at::Tensor& embedding_weight,
                                    at::Tensor gathered, at::Tensor accumulated) {
  TORCH_CHECK(token_ids.is_cuda() && token_ids.dim() == 1 && token_ids.is_contiguous() &&
                  (token_ids.scalar_type() == at::kLong || token_ids.scalar_type() == at::kInt),
              "token_ids must be a contiguous CUDA int64 / int32 vector");
  TORCH_CHECK(embedding_weight.dim() == 2 && gathered.dim() == 2 && accumulated.dim() == 2 &&
                  embedding_weight.is_contiguous() && gathered.is_contiguous() && accumulated.is_contiguous() &&
                  embedding_weight.scalar_type() == at::kBFloat16 && gathered.scalar_type() == at::kBFloat16 &&
                  accumulated.scalar_type() == at::kBFloat16,
              "tables and rows must be contiguous bf16 matrices");
  const int64_t rows = token_ids.size(0), hidden = embedding_weight.size(1);
  TORCH_CHECK(gathered.size(0) == rows && accumulated.size(0) == rows && gathered.size(1) == hidden &&
                  accumulated.size(1) == hidden, "gathered / accumulated must be [rows, hidden]");
  c10::cuda::CUDAGuard g(token_ids.device());
  if (rows == 0) return true;
  check_rc(omni_gather_embedding_add(token_ids.data_ptr(), token_ids.scalar_type() == at::kInt ? 1 : 0, rows,
                                     embedding_weight.data_ptr(), hidden, gathered.data_ptr(), accumulated.data_ptr(),
                                     nullptr, 0, nullptr, stream_of(token_ids)),
           "gather_codec_embedding_and_add");
  return true;
}

at::Tensor codebook_step(const at::Tensor& logits, const at::Tensor& embedding_weight, at::Tensor codes,
                         at::Tensor summed) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1,
              "logits must be bf16 [rows, vocab]");
  const int64_t rows = logits.size(0), hidden = embedding_weight.size(1);
  TORCH_CHECK(codes.scalar_type() == at::kLong && codes.dim() == 1 && codes.size(0) == rows, "codes: int64 [rows]");
  TORCH_CHECK(summed.scalar_type() == at::kBFloat16 && summed.dim() == 2 && summed.size(0) == rows &&
                  summed.size(1) == hidden && summed.stride(1) == 1 && summed.stride(0) == hidden,
              "summed: contiguous bf16 [rows, hidden]");
  TORCH_CHECK(embedding_weight.scalar_type() == at::kBFloat16 && embedding_weight.is_contiguous(),
              "embedding_weight: contiguous bf16");
  c10::cuda::CUDAGuard g(logits.device());
  auto next = at::empty({rows, 1, hidden}, summed.options());
  if (rows == 0) return next;
  check_rc(omni_codebook_step(logits.data_ptr(), rows, logits.size(1), logits.stride(0), embedding_weight.data_ptr(),
                              hidden, codes.data_ptr<int64_t>(), codes.stride(0), next.data_ptr(), summed.data_ptr(),
                              stream_of(logits)),
           "codebook_step");
  return next;
}

void add_rmsnorm_rounded(at::Tensor x, at::Tensor residual, const at::Tensor& weight, double eps) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.sizes() == residual.sizes() && x.scalar_type() == at::kBFloat16 &&
                  residual.scalar_type() == at::kBFloat16 && weight.scalar_type() == at::kBFloat16 &&
                  x.stride(1) == 1 && residual.stride(1) == 1 && weight.is_contiguous() &&
                  weight.numel() == x.size(1),
              "add_rmsnorm_rounded: bf16 x, residual [rows, hidden] and weight [hidden]");
  c10::cuda::CUDAGuard g(x.device());
  if (x.size(0) == 0) return;
  check_rc(omni_rmsnorm(x.data_ptr(), x.stride(0), residual.data_ptr(), residual.stride(0), residual.data_ptr(),
                        residual.stride(0), weight.data_ptr(), (float)eps, x.data_ptr(), x.stride(0), x.size(0),
                        x.size(1), stream_of(x)),
           "add_rmsnorm_rounded");
}

void paged_decode_attention(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                            const at::Tensor& page_indptr, const at::Tensor& page_indices, const at::Tensor& seq_lens,
                            double sm_scale, at::Tensor out, at::Tensor workspace, int64_t work_capacity) {
  TORCH_CHECK(q.is_cuda() && q.dim() == 3 && k_cache.dim() == 3 && v_cache.sizes() == k_cache.sizes() &&
                  out.sizes() == q.sizes(),
              "q / out [rows, Hq, D], caches [slots, Hkv, D]");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k_cache.scalar_type() == at::kBFloat16 &&
                  v_cache.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16,
              "bf16 operands");
  TORCH_CHECK(q.stride(2) == 1 && q.stride(1) == q.size(2) && out.stride(2) == 1 && out.stride(1) == out.size(2) &&
                  k_cache.is_contiguous() && v_cache.is_contiguous(),
              "heads must be packed within a row");
  const int64_t rows = q.size(0);
  check_rows(page_indptr, rows + 1, at::kInt, "page_indptr");
  check_rows(seq_lens, rows, at::kLong, "seq_lens");
  TORCH_CHECK(page_indices.is_cuda() && page_indices.scalar_type() == at::kInt && page_indices.is_contiguous(),
              "page_indices: contiguous int32");
  TORCH_CHECK(workspace.is_cuda() && workspace.is_contiguous(), "workspace: contiguous device buffer");
  c10::cuda::CUDAGuard g(q.device());
  check_rc(omni_paged_decode_attention(q.data_ptr(), q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
                                       page_indptr.data_ptr<int32_t>(), page_indices.data_ptr<int32_t>(),
                                       seq_lens.data_ptr<int64_t>(), nullptr, rows, (int32_t)q.size(1),
                                       (int32_t)k_cache.size(1), (int32_t)q.size(2), 16, 1, work_capacity,
                                       (float)sm_scale, out.data_ptr(), out.stride(0), workspace.data_ptr(),
                                       workspace.numel() * workspace.element_size(), 0, stream_of(q)),
           "paged_decode_attention");
}

void linear(const at::Tensor& x, const at::Tensor& w, at::Tensor out, int64_t epilogue,
            const c10::optional<at::Tensor>& residual) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && w.dim() == 2 && out.dim() == 2 && x.size(1) == w.size(1) &&
                  out.size(0) == x.size(0),
              "x [rows, K], w [N, K], out [rows, N]");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && x.stride(1) == 1 &&
                  w.is_contiguous() && out.stride(1) == 1,
              "bf16 operands with unit column strides");
  c10::cuda::CUDAGuard g(x.device());
  const at::Tensor* r = residual.has_value() ? &residual.value() : nullptr;
  check_rc(omni_linear(x.data_ptr(), x.size(0), x.size(1), x.stride(0), w.data_ptr(), w.size(0), (int32_t)epilogue,
                       r ? r->data_ptr() : nullptr, r ? r->stride(0) : 0, out.data_ptr(), out.stride(0), nullptr, 0,
                       0, stream_of(x)),
           "linear");
}

}  // namespace

TORCH_LIBRARY(omni_b200, m) {
  m.def("sample_topk_topp(Tensor logits, Tensor temperatures, Tensor top_ks, Tensor top_ps, Tensor seeds, "
        "Tensor positions, int max_top_k, bool has_top_p) -> Tensor");
  m.def("gather_codec_embedding_and_add(Tensor token_ids, Tensor embedding_weight, Tensor(a!) gathered, "
        "Tensor(b!) accumulated) -> bool");
  m.def("codebook_step(Tensor logits, Tensor embedding_weight, Tensor(a!) codes, Tensor(b!) summed) -> Tensor");
  m.def("add_rmsnorm_rounded(Tensor(a!) x, Tensor(b!) residual, Tensor weight, float eps) -> ()");
  m.def("paged_decode_attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor page_indptr, Tensor page_indices, "
        "Tensor seq_lens, float sm_scale, Tensor(a!) out, Tensor(b!) workspace, int work_capacity) -> ()");
  m.def("linear(Tensor x, Tensor w, Tensor(a!) out, int epilogue, Tensor? residual=None) -> ()");
}

TORCH_LIBRARY_IMPL(omni_b200, CUDA, m) {
  m.impl("sample_topk_topp", &sample_topk_topp);
  m.impl("gather_codec_embedding_and_add", &gather_codec_embedding_and_add);
  m.impl("codebook_step", &codebook_step);
  m.impl("add_rmsnorm_rounded", &add_rmsnorm_rounded);
  m.impl("paged_decode_attention", &paged_decode_attention);
  m.impl("linear", &linear);
}
