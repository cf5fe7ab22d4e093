// Python bindings of the qwen38_b200 sm_100a kernels.
#include <torch/extension.h>

void q38_linear(torch::Tensor x, torch::Tensor w, int64_t N, torch::Tensor out, int64_t epi, torch::Tensor ws,
                torch::Tensor counters, torch::Tensor err);
void q38_lm_head_argmax(torch::Tensor x, torch::Tensor w, int64_t N, torch::Tensor out_val, torch::Tensor out_idx,
                        int64_t vocab_offset, torch::Tensor part_val, torch::Tensor part_idx, torch::Tensor ws,
                        torch::Tensor counters, torch::Tensor err, c10::optional<torch::Tensor> samp_scale,
                        c10::optional<torch::Tensor> samp_key);
void q38_linear_rs(torch::Tensor x, torch::Tensor w, int64_t N, torch::Tensor ws, torch::Tensor counters,
                   torch::Tensor err, std::vector<int64_t> recv_ptrs, std::vector<int64_t> count_ptrs, int64_t rank,
                   int64_t rows_cap);
void q38_rs_reduce_bcast(int64_t recv_local, int64_t count_local, int64_t count_target, torch::Tensor x,
                         int64_t x_mc, int64_t flag_mc, int64_t rank, int64_t world, int64_t rows_cap,
                         int64_t slots, torch::Tensor err);
void q38_rs_wait(int64_t flag_local, int64_t target, torch::Tensor err);
void q38_rms_norm_wait(torch::Tensor x, torch::Tensor w, double eps, torch::Tensor out, int64_t flag_local,
                       int64_t target, torch::Tensor err);
void q38_linear_push(torch::Tensor x, torch::Tensor w, int64_t N, torch::Tensor ws, torch::Tensor counters,
                     torch::Tensor err, std::vector<int64_t> recv_ptrs, int64_t rank, int64_t slot,
                     int64_t block_words, torch::Tensor epochs, int64_t mc_ptr,
                     c10::optional<torch::Tensor> mx_scales);
void q38_linear_mx(torch::Tensor x, torch::Tensor wq, torch::Tensor wsc, int64_t N, torch::Tensor out, int64_t epi,
                   torch::Tensor ws, torch::Tensor counters, torch::Tensor err);
void q38_rms_norm_ar(torch::Tensor x, c10::optional<torch::Tensor> w, double eps, c10::optional<torch::Tensor> out,
                     int64_t recv_local, torch::Tensor epochs, int64_t slot, int64_t world, int64_t block_words,
                     torch::Tensor err);
int64_t q38_linear_trace(torch::Tensor x, torch::Tensor w, int64_t N, torch::Tensor out, int64_t epi,
                         torch::Tensor ws, torch::Tensor counters, torch::Tensor err, torch::Tensor trace,
                         c10::optional<torch::Tensor> mx_scales);
void q38_clear_map_cache();
void q38_gdn_set_trace(c10::optional<torch::Tensor> trace);
void q38_gdn_recurrent(int64_t mode, torch::Tensor proj, torch::Tensor window, torch::Tensor state,
                       torch::Tensor conv_w, torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor norm_w,
                       c10::optional<torch::Tensor> out, int64_t rows, c10::optional<torch::Tensor> rows_dev,
                       int64_t nk, int64_t nv, int64_t D, double eps);
void q38_attn_prep(torch::Tensor proj, int64_t q_off, int64_t k_off, int64_t v_off, int64_t nq, int64_t nkv,
                   int64_t D, int64_t rd, torch::Tensor qn, torch::Tensor kn, torch::Tensor inv_freq,
                   double rope_scale, double eps, torch::Tensor pos, c10::optional<torch::Tensor> q_out,
                   torch::Tensor kcache, torch::Tensor vcache, c10::optional<torch::Tensor> block_table,
                   int64_t block_size, torch::Tensor err);
void q38_attn_decode(torch::Tensor q, torch::Tensor kcache, torch::Tensor vcache,
                     c10::optional<torch::Tensor> block_table, int64_t block_size, torch::Tensor qpos, double scale,
                     int64_t causal, c10::optional<torch::Tensor> gate, int64_t gate_off, torch::Tensor out,
                     torch::Tensor part_o, torch::Tensor part_ml, int64_t max_keys, c10::optional<torch::Tensor> err);
void q38_attn_decode_window(torch::Tensor q, torch::Tensor kcache, torch::Tensor vcache,
                            c10::optional<torch::Tensor> block_table, int64_t block_size, torch::Tensor qpos,
                            double scale, int64_t causal, c10::optional<torch::Tensor> gate, int64_t gate_off,
                            torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml, int64_t max_keys,
                            int64_t window, c10::optional<torch::Tensor> err);
std::vector<std::pair<int64_t, int64_t>> q38_attn_key_groups(int64_t nchunks);
void q38_draft_conv(torch::Tensor x, torch::Tensor dyn, int64_t tap0, torch::Tensor base, int64_t group,
                    c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> resid);
void q38_draft_select(torch::Tensor feats, torch::Tensor cand, torch::Tensor unary, torch::Tensor anchor,
                      torch::Tensor pred, torch::Tensor succ, torch::Tensor out, torch::Tensor err);
void q38_attn_prefill(torch::Tensor q, torch::Tensor kcache, torch::Tensor vcache,
                      c10::optional<torch::Tensor> block_table, int64_t block_size, torch::Tensor qpos, double scale,
                      c10::optional<torch::Tensor> gate, torch::Tensor out);
void q38_gdn_chunk_prefill(torch::Tensor proj, torch::Tensor window, torch::Tensor state, torch::Tensor conv_w,
                           torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor norm_w, torch::Tensor out,
                           torch::Tensor work, int64_t nk, int64_t nv, double eps);
size_t q38_gdn_chunk_workspace_bytes(int64_t S, int64_t nv);
void q38_markov_select(torch::Tensor logits, torch::Tensor pred, torch::Tensor succ, torch::Tensor anchor,
                       torch::Tensor out, int64_t vocab_offset, torch::Tensor rec_val, torch::Tensor rec_idx,
                       torch::Tensor state, std::vector<int64_t> recv_ptrs, int64_t rank, torch::Tensor err);
void q38_rms_norm(torch::Tensor x, torch::Tensor w, double eps, torch::Tensor out);
void q38_rms_norm_split(torch::Tensor x, torch::Tensor parts, int64_t S, c10::optional<torch::Tensor> w, double eps,
                        c10::optional<torch::Tensor> out);
int64_t q38_swap_splits(int64_t N, int64_t K);
int64_t q38_linear_split(torch::Tensor x, torch::Tensor w, int64_t N, torch::Tensor residual, torch::Tensor parts,
                         torch::Tensor ws, torch::Tensor counters, torch::Tensor err,
                         c10::optional<torch::Tensor> mx_scales);
void q38_embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out);
void q38_markov_step(torch::Tensor logits_row, torch::Tensor pred, torch::Tensor succ, torch::Tensor prev,
                     torch::Tensor out, c10::optional<torch::Tensor> out_val, torch::Tensor part_val,
                     torch::Tensor part_idx, int64_t vocab_offset, bool write_prev);

torch::Tensor q38_peer_alloc(int64_t bytes, int64_t device);
torch::Tensor q38_ipc_handle(torch::Tensor buf);
int64_t q38_ipc_open(torch::Tensor handle, int64_t device);
void q38_ipc_close(int64_t ptr);
void q38_allreduce_residual(std::vector<int64_t> data_ptrs, std::vector<int64_t> flag_ptrs, int64_t rank,
                            int64_t slot, int64_t slot_floats, torch::Tensor residual, torch::Tensor epochs,
                            torch::Tensor err);
void q38_argmax_allreduce(std::vector<int64_t> data_ptrs, std::vector<int64_t> flag_ptrs, int64_t rank,
                          int64_t slot, int64_t slot_floats, torch::Tensor val, torch::Tensor idx, torch::Tensor out,
                          torch::Tensor epochs, torch::Tensor err);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "qwen38_b200 sm_100a kernels";
  m.def("linear", &q38_linear);
  m.def("lm_head_argmax", &q38_lm_head_argmax);
  m.def("linear_push", &q38_linear_push);
  m.def("linear_rs", &q38_linear_rs);
  m.def("rs_reduce_bcast", &q38_rs_reduce_bcast);
  m.def("rs_wait", &q38_rs_wait);
  m.def("rms_norm_wait", &q38_rms_norm_wait);
  m.def("rms_norm_ar", &q38_rms_norm_ar);
  m.def("linear_trace", &q38_linear_trace);
  m.def("clear_map_cache", &q38_clear_map_cache);
  m.def("gdn_recurrent", &q38_gdn_recurrent);
  m.def("gdn_set_trace", &q38_gdn_set_trace);
  m.def("gdn_chunk_prefill", &q38_gdn_chunk_prefill);
  m.def("gdn_chunk_workspace_bytes", &q38_gdn_chunk_workspace_bytes);
  m.def("attn_prep", &q38_attn_prep);
  m.def("attn_decode", &q38_attn_decode);
  m.def("attn_decode_window", &q38_attn_decode_window);
  m.def("draft_conv", &q38_draft_conv);
  m.def("draft_select", &q38_draft_select);
  m.def("attn_prefill", &q38_attn_prefill);
  m.def("attn_key_groups", &q38_attn_key_groups);
  m.def("rms_norm", &q38_rms_norm);
  m.def("rms_norm_split", &q38_rms_norm_split);
  m.def("swap_splits", &q38_swap_splits);
  m.def("linear_split", &q38_linear_split);
  m.def("linear_mx", &q38_linear_mx);
  m.def("embedding", &q38_embedding);
  m.def("markov_step", &q38_markov_step);
  m.def("markov_select", &q38_markov_select);
  m.def("peer_alloc", &q38_peer_alloc);
  m.def("ipc_handle", &q38_ipc_handle);
  m.def("ipc_open", &q38_ipc_open);
  m.def("ipc_close", &q38_ipc_close);
  m.def("allreduce_residual", &q38_allreduce_residual);
  m.def("argmax_allreduce", &q38_argmax_allreduce);
}
