// Python bindings of the llmserve_b200 sm_100a kernels (module llmserve_b200._C).
#include <torch/extension.h>

namespace lsb {
void rms_norm(at::Tensor out, at::Tensor x, at::Tensor w, double eps);
void add_rms_norm(at::Tensor out, at::Tensor res_out, at::Tensor x, at::Tensor residual, at::Tensor w, double eps);
void silu_and_mul(at::Tensor out, at::Tensor x);
void embedding(at::Tensor out, at::Tensor ids, at::Tensor table, at::Tensor status);
void qkv_rope(at::Tensor q_out, at::Tensor k_out, at::Tensor qkv, at::Tensor positions, at::Tensor cos_sin,
              at::Tensor q_w, at::Tensor k_w, double eps, at::Tensor k_cache, at::Tensor v_cache,
              at::Tensor slot_mapping, int64_t nh, int64_t nkv, int64_t hd, bool store, at::Tensor status);
void store_kvcache(at::Tensor k, at::Tensor v, at::Tensor k_cache, at::Tensor v_cache, at::Tensor slots,
                   at::Tensor status);
void commit_tree_kv(at::Tensor tk, at::Tensor tv, at::Tensor kc, at::Tensor vc, at::Tensor nodes, at::Tensor slots,
                    at::Tensor status);
void splitk_reduce(at::Tensor out, at::Tensor partials);
void splitk_reduce_add_rmsnorm(at::Tensor out, at::Tensor res_out, at::Tensor partials, at::Tensor residual,
                               at::Tensor w, double eps);
void argmax_rows(at::Tensor out_idx, at::Tensor out_val, at::Tensor logits);
void sample_rows(at::Tensor out, at::Tensor logits, at::Tensor temps, int64_t seed);
void decode_attention(at::Tensor out, at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor block_tables,
                      at::Tensor context_lens, double scale, at::Tensor part_o, at::Tensor part_ml, at::Tensor counters,
                      int64_t max_splits, int64_t partition, int64_t grid_z, at::Tensor status);
void prefill_attention(at::Tensor out, at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor cu_q,
                       at::Tensor seqlens_k, at::Tensor block_tables, double scale, int64_t max_seqlen_q,
                       at::Tensor status);
void tree_attention(at::Tensor out, at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor bt, int64_t prefix_len,
                    at::Tensor tk, at::Tensor tv, at::Tensor mask_bits, double scale, at::Tensor status);
void gemm_bf16(at::Tensor out, at::Tensor x, at::Tensor w, at::Tensor partials, int64_t splits, at::Tensor status,
               int64_t max_stages);
int64_t comm_alloc(int64_t nbytes);
void comm_free(int64_t p);
at::Tensor comm_ipc_handle(int64_t p);
int64_t comm_open_handle(at::Tensor handle);
void comm_close_handle(int64_t p);
void comm_set_spin_limit(int64_t polls);
void row_parallel_finish(std::vector<int64_t> ag, int64_t inbox, int64_t ctrl, int64_t out, int64_t res_out,
                         at::Tensor res_in, at::Tensor w, int64_t rank, int64_t S, int64_t T, int64_t N,
                         int64_t rows_per_rank, double eps, int64_t phases, at::Tensor status);
void vocab_argmax_exchange(std::vector<int64_t> flags, at::Tensor vals, at::Tensor idx, int64_t vocab_start,
                           at::Tensor out, int64_t rank, at::Tensor status);
int64_t comm_control_bytes();
void gemm_bf16_to_owners(at::Tensor x, at::Tensor w, int64_t n, bool packed, std::vector<int64_t> inboxes,
                         int64_t rank, int64_t rows_per_rank, int64_t splits, bool reduce, int64_t epoch_ptr,
                         at::Tensor status, int64_t max_stages);
void gemm_bf16_reduced(at::Tensor out, at::Tensor x, at::Tensor w, int64_t n, bool packed, at::Tensor plane,
                       int64_t splits, at::Tensor status, int64_t max_stages);
void gemm_bf16_silu_reduced(at::Tensor out, at::Tensor x, at::Tensor w, int64_t n, bool packed, int64_t splits,
                            at::Tensor status, int64_t max_stages);
void awq_gemm_reduced(at::Tensor out, at::Tensor x, at::Tensor qtiles, at::Tensor sztiles, int64_t n, int64_t splits,
                      at::Tensor status);
void awq_gemm_to_owners(at::Tensor x, at::Tensor qtiles, at::Tensor sztiles, int64_t n, std::vector<int64_t> inboxes,
                        int64_t rank, int64_t rows_per_rank, int64_t splits, bool reduce, int64_t epoch_ptr,
                        at::Tensor status);
void gemm_bf16_silu(at::Tensor out, at::Tensor x, at::Tensor w, at::Tensor status, int64_t max_stages);
void splitk_silu(at::Tensor out, at::Tensor partials);
void silu_and_mul_interleaved(at::Tensor out, at::Tensor x);
void gemm_bf16_silu_packed(at::Tensor out, at::Tensor x, at::Tensor w, int64_t n, at::Tensor status,
                           int64_t max_stages);
void gemm_bf16_packed(at::Tensor out, at::Tensor x, at::Tensor w, int64_t n, at::Tensor partials, int64_t splits,
                      at::Tensor status, int64_t max_stages);
void decode_attention_tma(at::Tensor out, at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor block_tables,
                          at::Tensor context_lens, double scale, at::Tensor part_o, at::Tensor part_ml,
                          at::Tensor counters, int64_t max_splits, int64_t partition, int64_t nq,
                          at::Tensor status);
bool decode_tma_supported(int64_t block_size, int64_t head_dim);
bool prefill_tc_supported(int64_t block_size, int64_t head_dim);
bool tree_tc_supported(int64_t n_q, int64_t nh, int64_t nkv, int64_t n_tree, int64_t block_size, int64_t head_dim);
void tree_attention_tc(at::Tensor out, at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor bt, int64_t prefix_len,
                       at::Tensor tk, at::Tensor tv, at::Tensor mask_bits, double scale, at::Tensor status);
void prefill_attention_tc(at::Tensor out, at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor cu_q,
                          at::Tensor seqlens_k, at::Tensor block_tables, double scale, int64_t max_q,
                          at::Tensor status);
void awq_gemm(at::Tensor out, at::Tensor x, at::Tensor qtiles, at::Tensor sztiles, int64_t n, at::Tensor partials,
              int64_t splits, at::Tensor status);
void greedy_accept(at::Tensor out, at::Tensor target, at::Tensor draft, at::Tensor start);
void feed_ids(at::Tensor out, at::Tensor ids, at::Tensor feed, at::Tensor prev, at::Tensor status);
void kv_push(at::Tensor src_k, at::Tensor src_v, at::Tensor dst_k, at::Tensor dst_v, at::Tensor src_ids,
             at::Tensor dst_ids, at::Tensor status);
}  // namespace lsb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "llmserve_b200 sm_100a kernels";
  m.def("rms_norm", &lsb::rms_norm);
  m.def("add_rms_norm", &lsb::add_rms_norm);
  m.def("silu_and_mul", &lsb::silu_and_mul);
  m.def("embedding", &lsb::embedding);
  m.def("qkv_rope", &lsb::qkv_rope);
  m.def("store_kvcache", &lsb::store_kvcache);
  m.def("commit_tree_kv", &lsb::commit_tree_kv);
  m.def("splitk_reduce", &lsb::splitk_reduce);
  m.def("splitk_reduce_add_rmsnorm", &lsb::splitk_reduce_add_rmsnorm);
  m.def("argmax_rows", &lsb::argmax_rows);
  m.def("sample_rows", &lsb::sample_rows);
  m.def("decode_attention_tma", &lsb::decode_attention_tma);
  m.def("gemm_bf16_packed", &lsb::gemm_bf16_packed);
  m.def("awq_gemm", &lsb::awq_gemm);
  m.def("decode_tma_supported", &lsb::decode_tma_supported);
  m.def("decode_attention", &lsb::decode_attention, py::arg("out"), py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("block_tables"), py::arg("context_lens"), py::arg("scale"), py::arg("part_o"), py::arg("part_ml"),
        py::arg("counters"), py::arg("max_splits"), py::arg("partition"), py::arg("grid_z"), py::arg("status"));
  m.def("prefill_attention", &lsb::prefill_attention);
  m.def("prefill_attention_tc", &lsb::prefill_attention_tc);
  m.def("prefill_tc_supported", &lsb::prefill_tc_supported);
  m.def("tree_attention", &lsb::tree_attention);
  m.def("tree_attention_tc", &lsb::tree_attention_tc);
  m.def("tree_tc_supported", &lsb::tree_tc_supported);
  m.def("comm_alloc", &lsb::comm_alloc);
  m.def("comm_free", &lsb::comm_free);
  m.def("comm_ipc_handle", &lsb::comm_ipc_handle);
  m.def("comm_open_handle", &lsb::comm_open_handle);
  m.def("comm_close_handle", &lsb::comm_close_handle);
  m.def("comm_set_spin_limit", &lsb::comm_set_spin_limit);
  m.def("row_parallel_finish", &lsb::row_parallel_finish);
  m.def("vocab_argmax_exchange", &lsb::vocab_argmax_exchange);
  m.def("comm_control_bytes", &lsb::comm_control_bytes);
  m.def("gemm_bf16_to_owners", &lsb::gemm_bf16_to_owners);
  m.def("gemm_bf16_reduced", &lsb::gemm_bf16_reduced);
  m.def("gemm_bf16_silu_reduced", &lsb::gemm_bf16_silu_reduced);
  m.def("awq_gemm_to_owners", &lsb::awq_gemm_to_owners);
  m.def("awq_gemm_reduced", &lsb::awq_gemm_reduced);
  m.def("gemm_bf16_silu", &lsb::gemm_bf16_silu);
  m.def("splitk_silu", &lsb::splitk_silu);
  m.def("silu_and_mul_interleaved", &lsb::silu_and_mul_interleaved);
  m.def("gemm_bf16_silu_packed", &lsb::gemm_bf16_silu_packed);
  m.def("kv_push", &lsb::kv_push);
  m.def("feed_ids", &lsb::feed_ids);
  m.def("greedy_accept", &lsb::greedy_accept);
  m.def("gemm_bf16", &lsb::gemm_bf16, py::arg("out"), py::arg("x"), py::arg("w"), py::arg("partials"),
        py::arg("splits"), py::arg("status"), py::arg("max_stages") = 0);
}
