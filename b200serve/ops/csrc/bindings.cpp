// Python bindings of the b200serve CUDA extension.
#include <torch/extension.h>

void rmsnorm_fused(std::vector<torch::Tensor> parts, c10::optional<torch::Tensor> residual_in,
                   c10::optional<torch::Tensor> residual_out, torch::Tensor w, torch::Tensor out, double eps);
void rmsnorm_fused_wait(std::vector<torch::Tensor> parts, c10::optional<torch::Tensor> residual_in,
                        c10::optional<torch::Tensor> residual_out, torch::Tensor w, torch::Tensor out, double eps,
                        int64_t flags_ptr, int64_t epoch_ptr, int64_t err_ptr, int64_t n_flags);
void rmsnorm_lamport(std::vector<torch::Tensor> parts, c10::optional<torch::Tensor> residual_in,
                     c10::optional<torch::Tensor> residual_out, torch::Tensor w, torch::Tensor out, double eps,
                     int64_t err_ptr, bool skip_prior_wait);
std::vector<int64_t> gemm_partial_plan(int64_t M, int64_t N, int64_t K, int64_t num_sms);
std::vector<int64_t> gemm_tc_partial(torch::Tensor act, torch::Tensor w, int64_t packed_n, torch::Tensor part);
void rmsnorm_partial(torch::Tensor like, torch::Tensor part, int64_t kb, int64_t ctas, int64_t total, int64_t tile,
                     c10::optional<torch::Tensor> residual_in, c10::optional<torch::Tensor> residual_out,
                     torch::Tensor w, torch::Tensor out, double eps);
void qkv_post_partial(torch::Tensor like, torch::Tensor part, int64_t kb, int64_t ctas, int64_t total,
                      int64_t tile, c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> qn_w,
                      c10::optional<torch::Tensor> kn_w, torch::Tensor cos_sin, torch::Tensor positions,
                      torch::Tensor slots, torch::Tensor q_out, torch::Tensor k_cache, torch::Tensor v_cache,
                      c10::optional<torch::Tensor> k_scale, c10::optional<torch::Tensor> v_scale, int64_t nq,
                      int64_t nkv, double eps);
int64_t gguf_gemv_splits(int64_t N, int64_t K);
void gguf_gemv(torch::Tensor x, torch::Tensor codes, torch::Tensor meta, int64_t N, int64_t bits, int64_t group,
               int64_t mode, int64_t S, torch::Tensor out, int64_t ldo, int64_t col0, torch::Tensor push_ptrs,
               int64_t mc_ptr);
void silu_mul_partial(torch::Tensor part, int64_t kb, int64_t ctas, int64_t total, int64_t tile, int64_t M, int64_t I,
                      torch::Tensor out, int64_t inter);
std::vector<int64_t> gguf_stream_plan(int64_t N, int64_t K, int64_t num_sms);
std::vector<int64_t> gguf_stream(torch::Tensor x, std::vector<torch::Tensor> codes, std::vector<torch::Tensor> metas,
                                 std::vector<int64_t> ns, std::vector<int64_t> bits, std::vector<int64_t> groups,
                                 int64_t mode, torch::Tensor out, int64_t ldo, torch::Tensor ws, torch::Tensor counters,
                                 torch::Tensor push_ptrs, int64_t mc_ptr, int64_t num_sms, int64_t wait_ms,
                                 int64_t table);
void gguf_dequant_packed(torch::Tensor codes, torch::Tensor meta, int64_t N, int64_t K, int64_t bits, int64_t group,
                         torch::Tensor out, int64_t table);
void gemm_grouped_ep(torch::Tensor act, torch::Tensor w_packed, int64_t N, int64_t E, torch::Tensor offsets,
                     int64_t max_rows, torch::Tensor out, torch::Tensor ws, torch::Tensor counters, int64_t epi,
                     int64_t ag_flags_ptr, int64_t ag_n, int64_t ag_epoch_ptr, torch::Tensor comb_meta,
                     int64_t comb_k, int64_t comb_rows, torch::Tensor comb_dst_ptrs, int64_t ldo,
                     torch::Tensor flag_ptrs, torch::Tensor tile_done, int64_t push_tiles, int64_t err_ptr);
void ep_count(torch::Tensor ids, int64_t valid, int64_t per, int64_t me, torch::Tensor pos, torch::Tensor cnt_ptrs,
              torch::Tensor flag_ptrs, int64_t epoch_ptr);
void ep_dispatch(torch::Tensor x, torch::Tensor ids, torch::Tensor wts, torch::Tensor pos, int64_t valid, int64_t per,
                 int64_t me, int64_t cnt_all_ptr, int64_t wait_flags_ptr, torch::Tensor cnt_ptrs,
                 torch::Tensor rows_ptrs, torch::Tensor meta_ptrs, torch::Tensor dflag_ptrs, int64_t epoch_ptr,
                 torch::Tensor done, int64_t err_ptr);
void gemm_tc_push(torch::Tensor act, torch::Tensor w, torch::Tensor dst_ptrs, int64_t ldo, torch::Tensor flag_ptrs,
                  int64_t epoch_ptr, torch::Tensor tile_done, c10::optional<torch::Tensor> bias, torch::Tensor ws,
                  torch::Tensor counters, int64_t err_ptr, int64_t packed_n, int64_t rs_rows, int64_t lamport, int64_t mc_ptr);
int64_t ipc_malloc(int64_t bytes);
void ipc_free(int64_t ptr);
torch::Tensor ipc_handle(int64_t ptr);
int64_t ipc_open(torch::Tensor handle);
void ipc_close(int64_t ptr);
torch::Tensor host_error_word();
int64_t read_host_word(int64_t host_ptr, int64_t index, bool reset);
void epoch_inc(int64_t epoch_ptr);
void qkv_post(torch::Tensor qkv, c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> qn_w,
              c10::optional<torch::Tensor> kn_w, torch::Tensor cos_sin, torch::Tensor positions,
              torch::Tensor slots, torch::Tensor q_out, torch::Tensor k_cache, torch::Tensor v_cache, int64_t nq,
              int64_t nkv, double eps);
void silu_mul(torch::Tensor gu, torch::Tensor act);
void gelu_tanh_mul(torch::Tensor gu, torch::Tensor act);
void softcap_(torch::Tensor x, double cap);
void layernorm_rows(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> b, double eps, torch::Tensor out);
void gelu_rows(torch::Tensor x, bool tanh_approx);
void vision_qkv_rope(torch::Tensor qkv, torch::Tensor cos_sin, int64_t heads, int64_t hd, torch::Tensor slots,
                     torch::Tensor q_out, torch::Tensor k_cache, torch::Tensor v_cache);
void row_sigmoid_scale(torch::Tensor x, torch::Tensor g);
void embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out);
void paged_decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                            torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor out,
                            torch::Tensor part_acc, torch::Tensor part_ml, double scale, int64_t tps,
                            int64_t nsplit, int64_t window, double softcap);
void paged_prefill_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                             torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor q_start,
                             torch::Tensor cu_q, torch::Tensor out, double scale, int64_t max_q, int64_t window,
                             double softcap);
void paged_decode_attention_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                               torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor out,
                               torch::Tensor part_acc, torch::Tensor part_ml, double scale, int64_t tps,
                               int64_t nsplit);
void topk_softmax(torch::Tensor logits, int64_t k, bool renorm, torch::Tensor w_out, torch::Tensor id_out);
void moe_permute(torch::Tensor ids, int64_t k, int64_t e0, int64_t E, torch::Tensor offsets, torch::Tensor pos,
                 torch::Tensor sorted_tok);
void gather_rows(torch::Tensor x, torch::Tensor rows, torch::Tensor count, torch::Tensor out);
void moe_combine(torch::Tensor y, torch::Tensor w, torch::Tensor pos, int64_t k, torch::Tensor out);
void gguf_gemm(torch::Tensor x, torch::Tensor codes, torch::Tensor meta, int64_t N, int64_t bits, int64_t group,
               torch::Tensor out);
void paged_decode_attention_q4(torch::Tensor q, torch::Tensor k_codes, torch::Tensor v_codes, torch::Tensor k_scale,
                               torch::Tensor v_scale, torch::Tensor block_tables, torch::Tensor seq_lens,
                               torch::Tensor out, torch::Tensor part_acc, torch::Tensor part_ml, double scale,
                               int64_t tps, int64_t nsplit);
void qkv_post_q4(torch::Tensor qkv, c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> qn_w,
                 c10::optional<torch::Tensor> kn_w, torch::Tensor cos_sin, torch::Tensor positions,
                 torch::Tensor slots, torch::Tensor q_out, torch::Tensor k_codes, torch::Tensor v_codes,
                 torch::Tensor k_scale, torch::Tensor v_scale, int64_t nq, int64_t nkv, double eps);
void paged_prefill_attention_q4(torch::Tensor q, torch::Tensor k_codes, torch::Tensor v_codes, torch::Tensor k_scale,
                                torch::Tensor v_scale, torch::Tensor block_tables, torch::Tensor seq_lens,
                                torch::Tensor q_start, torch::Tensor cu_q, torch::Tensor out, double scale,
                                int64_t max_q);
std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K, int64_t epi, int64_t num_sms);
void gemm_tc(torch::Tensor act, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> bias,
             c10::optional<torch::Tensor> residual, torch::Tensor ws, torch::Tensor counters, int64_t epi,
             int64_t force_splits, int64_t packed_n);
int64_t gemm_error_flag(bool reset);
void gemm_set_trace(int64_t ptr, int64_t slots);
void gemm_grouped(torch::Tensor act, torch::Tensor w_packed, int64_t N, int64_t E, torch::Tensor offsets,
                  int64_t max_rows, torch::Tensor out, torch::Tensor ws, torch::Tensor counters, int64_t epi);
void argmax_rows(torch::Tensor logits, torch::Tensor out_idx, torch::Tensor out_val, int64_t index_offset);
void argmax_merge(torch::Tensor vals, torch::Tensor idx, torch::Tensor out);
void sample_rows(torch::Tensor logits, torch::Tensor params, torch::Tensor pen_ids, torch::Tensor pen_counts,
                 torch::Tensor pen_vals, torch::Tensor out, int64_t cluster);

void paged_decode_attention_tq(torch::Tensor q_rot, torch::Tensor q_jl, torch::Tensor k_codes, torch::Tensor k_sign,
                               torch::Tensor k_meta, torch::Tensor v_codes, torch::Tensor v_meta,
                               torch::Tensor code_vals, torch::Tensor block_tables, torch::Tensor seq_lens,
                               torch::Tensor out, torch::Tensor part_acc, torch::Tensor part_ml, double scale,
                               int64_t tps, int64_t nsplit);
void tq_qkv(torch::Tensor q, torch::Tensor k_stage, torch::Tensor v_stage, torch::Tensor slots, torch::Tensor S,
            torch::Tensor cents, torch::Tensor thr, int64_t kbits, int64_t vbits, double alpha, torch::Tensor q_rot,
            torch::Tensor q_jl, torch::Tensor k_codes, torch::Tensor k_sign, torch::Tensor k_meta,
            torch::Tensor v_codes, torch::Tensor v_meta, torch::Tensor win_k, torch::Tensor win_v,
            torch::Tensor win_slots);
void paged_decode_combine(torch::Tensor part_acc, torch::Tensor part_ml, torch::Tensor seq_lens, torch::Tensor out,
                          int64_t nkv, int64_t G, int64_t nsplit, int64_t tps);
void tq_dequant(torch::Tensor block_ids, torch::Tensor k_codes, torch::Tensor k_sign, torch::Tensor k_meta,
                torch::Tensor v_codes, torch::Tensor v_meta, torch::Tensor S, torch::Tensor code_vals,
                torch::Tensor out_k, torch::Tensor out_v);

void gemm_tc_ag(torch::Tensor act, torch::Tensor w, torch::Tensor out, c10::optional<torch::Tensor> bias,
                torch::Tensor ws, torch::Tensor counters, int64_t epi, int64_t packed_n, int64_t ag_flags_ptr,
                int64_t ag_n, int64_t ag_epoch_ptr);

void rmsnorm_rs_ag(std::vector<torch::Tensor> parts, c10::optional<torch::Tensor> residual_in,
                   c10::optional<torch::Tensor> residual_out, torch::Tensor w, double eps, int64_t flags_ptr,
                   int64_t epoch_ptr, int64_t err_ptr, torch::Tensor dst_ptrs, torch::Tensor ag_flag_ptrs,
                   int64_t row0, int64_t T, torch::Tensor done, int64_t n_flags);

void publish_flags(torch::Tensor flag_ptrs, int64_t epoch_ptr);
void flag_wait(int64_t flags_ptr, int64_t n, int64_t epoch_ptr, int64_t err_ptr, double timeout_ms);
void set_flag_wait_ms(double ms);
double get_flag_wait_ms();
void flag_pingpong(int64_t mine_ptr, int64_t peer_ptr, int64_t iters, int64_t initiator, int64_t mode,
                   torch::Tensor out);

void gemm_tc_qkv(torch::Tensor act, torch::Tensor w, int64_t packed_n, c10::optional<torch::Tensor> bias,
                 c10::optional<torch::Tensor> q_norm, c10::optional<torch::Tensor> k_norm, torch::Tensor cos_sin,
                 torch::Tensor positions, torch::Tensor slots, torch::Tensor q_out, torch::Tensor k_cache,
                 torch::Tensor v_cache, int64_t nq, int64_t nkv, double eps, torch::Tensor ws,
                 torch::Tensor counters, int64_t ag_flags_ptr, int64_t ag_n, int64_t ag_epoch_ptr);

void moe_combine_push(torch::Tensor y, torch::Tensor w, torch::Tensor pos, int64_t k, int64_t T, int64_t H,
                      torch::Tensor dst_ptrs, torch::Tensor flag_ptrs, int64_t epoch_ptr, torch::Tensor done);

void paged_prefill_attention_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor q_start,
                                torch::Tensor cu_q, torch::Tensor out, double scale, int64_t max_q);
int64_t prefill_tc_error(bool reset);

void q4_dequant_pages(torch::Tensor block_ids, torch::Tensor codes, torch::Tensor scales, torch::Tensor out);
void deltanet_layer(torch::Tensor y, torch::Tensor conv_w, torch::Tensor A, torch::Tensor dt_bias,
                    torch::Tensor norm_w, torch::Tensor conv_state, torch::Tensor rec_state,
                    c10::optional<torch::Tensor> cu_q, torch::Tensor q_start, torch::Tensor slots, torch::Tensor xc,
                    torch::Tensor gb, torch::Tensor out, int64_t nk, int64_t nv, int64_t D, double eps,
                    c10::optional<torch::Tensor> o_raw);
void sigmoid_gate_mul(torch::Tensor attn, torch::Tensor gate);
void shortconv_layer(torch::Tensor y, torch::Tensor conv_w, torch::Tensor conv_state,
                     c10::optional<torch::Tensor> cu_q, torch::Tensor q_start, torch::Tensor slots,
                     torch::Tensor out);

// Error words of the bounds-checked build, one per translation unit with checked indices.
#define B200_BOUNDS_UNITS(X)                                                                    \
  X(norm_rope) X(attention_decode) X(attention_decode_tc) X(attention_prefill) X(attention_prefill_tc) \
  X(kv_turboquant) X(deltanet) X(shortconv) X(ep_a2a) X(vision)
#define B200_BOUNDS_DECL(u) int64_t bounds_error_##u(bool reset);
B200_BOUNDS_UNITS(B200_BOUNDS_DECL)
#undef B200_BOUNDS_DECL

// {unit: first recorded error code} for the units with a recorded error (empty in release builds).
static py::dict bounds_errors(bool reset) {
  py::dict d;
#define B200_BOUNDS_READ(u)                         \
  {                                                 \
    const int64_t v = bounds_error_##u(reset);      \
    if (v) d[#u] = v;                               \
  }
  B200_BOUNDS_UNITS(B200_BOUNDS_READ)
#undef B200_BOUNDS_READ
  return d;
}

static bool bounds_checked() {
#ifdef B200_BOUNDS_CHECK
  return true;
#else
  return false;
#endif
}

void paged_decode_attention_tc_part(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                    torch::Tensor block_tables, torch::Tensor seq_lens, torch::Tensor tok_lo,
                                    torch::Tensor part_acc, torch::Tensor part_ml, double scale, int64_t tps,
                                    int64_t nsplit, int64_t split_base, int64_t nsplit_total);
void paged_decode_attention_tq_part(torch::Tensor q_rot, torch::Tensor q_jl, torch::Tensor k_codes,
                                    torch::Tensor k_sign, torch::Tensor k_meta, torch::Tensor v_codes,
                                    torch::Tensor v_meta, torch::Tensor code_vals, torch::Tensor block_tables,
                                    torch::Tensor seq_lens, torch::Tensor part_acc, torch::Tensor part_ml, double scale,
                                    int64_t tps, int64_t nsplit, int64_t split_base, int64_t nsplit_total);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("paged_decode_attention_tc_part", &paged_decode_attention_tc_part);
  m.def("paged_decode_attention_tq_part", &paged_decode_attention_tq_part);
  m.def("paged_decode_combine", &paged_decode_combine);
  m.def("bounds_errors", &bounds_errors, py::arg("reset") = true);
  m.def("bounds_checked", &bounds_checked);
  m.doc() = "b200serve sm_100a kernels";
  m.def("rmsnorm_fused", &rmsnorm_fused);
  m.def("qkv_post", &qkv_post);
  m.def("rmsnorm_fused_wait", &rmsnorm_fused_wait);
  m.def("rmsnorm_rs_ag", &rmsnorm_rs_ag);
  m.def("gemm_tc_push", &gemm_tc_push, py::arg("act"), py::arg("w"), py::arg("dst_ptrs"), py::arg("ldo"),
        py::arg("flag_ptrs"), py::arg("epoch_ptr"), py::arg("tile_done"), py::arg("bias"), py::arg("ws"),
        py::arg("counters"), py::arg("err_ptr"), py::arg("packed_n"), py::arg("rs_rows"), py::arg("lamport") = 0,
        py::arg("mc_ptr") = 0);
  m.def("gemm_partial_plan", &gemm_partial_plan);
  m.def("gguf_gemv_splits", &gguf_gemv_splits);
  m.def("gguf_gemv", &gguf_gemv);
  m.def("gemm_grouped_ep", &gemm_grouped_ep);
  m.def("ep_count", &ep_count);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("gguf_dequant_packed", &gguf_dequant_packed);
  m.def("silu_mul_partial", &silu_mul_partial, py::arg("part"), py::arg("kb"), py::arg("ctas"), py::arg("total"),
        py::arg("tile"), py::arg("M"), py::arg("I"), py::arg("out"), py::arg("inter") = 0);
  m.def("gguf_stream_plan", &gguf_stream_plan);
  m.def("gguf_stream", &gguf_stream);
  m.def("gemm_tc_partial", &gemm_tc_partial);
  m.def("rmsnorm_partial", &rmsnorm_partial);
  m.def("qkv_post_partial", &qkv_post_partial);
  m.def("rmsnorm_lamport", &rmsnorm_lamport);
  m.def("ipc_malloc", &ipc_malloc);
  m.def("ipc_free", &ipc_free);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("host_error_word", &host_error_word);
  m.def("read_host_word", &read_host_word);
  m.def("epoch_inc", &epoch_inc);
  m.def("flag_wait", &flag_wait, py::arg("flags_ptr"), py::arg("n"), py::arg("epoch_ptr"), py::arg("err_ptr"),
        py::arg("timeout_ms") = -1.0);
  m.def("set_flag_wait_ms", &set_flag_wait_ms);
  m.def("publish_flags", &publish_flags);
  m.def("get_flag_wait_ms", &get_flag_wait_ms);
  m.def("flag_pingpong", &flag_pingpong);
  m.def("silu_mul", &silu_mul);
  m.def("gelu_tanh_mul", &gelu_tanh_mul);
  m.def("softcap_", &softcap_);
  m.def("layernorm_rows", &layernorm_rows);
  m.def("gelu_rows", &gelu_rows);
  m.def("vision_qkv_rope", &vision_qkv_rope);
  m.def("row_sigmoid_scale", &row_sigmoid_scale);
  m.def("embedding", &embedding);
  m.def("paged_decode_attention", &paged_decode_attention);
  m.def("paged_prefill_attention", &paged_prefill_attention);
  m.def("paged_prefill_attention_tc", &paged_prefill_attention_tc);
  m.def("q4_dequant_pages", &q4_dequant_pages);
  m.def("deltanet_layer", &deltanet_layer);
  m.def("sigmoid_gate_mul", &sigmoid_gate_mul);
  m.def("shortconv_layer", &shortconv_layer);
  m.def("prefill_tc_error", &prefill_tc_error);
  m.def("paged_decode_attention_tc", &paged_decode_attention_tc);
  m.def("topk_softmax", &topk_softmax);
  m.def("moe_permute", &moe_permute);
  m.def("gather_rows", &gather_rows);
  m.def("moe_combine", &moe_combine);
  m.def("moe_combine_push", &moe_combine_push);
  m.def("gguf_gemm", &gguf_gemm);
  m.def("paged_decode_attention_q4", &paged_decode_attention_q4);
  m.def("qkv_post_q4", &qkv_post_q4);
  m.def("paged_prefill_attention_q4", &paged_prefill_attention_q4);
  m.def("gemm_plan", &gemm_plan);
  m.def("gemm_tc", &gemm_tc);
  m.def("gemm_tc_ag", &gemm_tc_ag);
  m.def("gemm_tc_qkv", &gemm_tc_qkv);
  m.def("gemm_error_flag", &gemm_error_flag);
  m.def("gemm_set_trace", &gemm_set_trace);
  m.def("gemm_grouped", &gemm_grouped);
  m.def("argmax_rows", &argmax_rows);
  m.def("argmax_merge", &argmax_merge);
  m.def("sample_rows", &sample_rows, py::arg("logits"), py::arg("params"), py::arg("pen_ids"), py::arg("pen_counts"),
        py::arg("pen_vals"), py::arg("out"), py::arg("cluster") = 0);
  m.def("paged_decode_attention_tq", &paged_decode_attention_tq);
  m.def("tq_qkv", &tq_qkv);
  m.def("tq_dequant", &tq_dequant);
}
