// Operator registry of the sm_100a kernel library: ``torch.ops.isb.*``.
//
// Parity: the reference registers its CUDA ops with ``TORCH_LIBRARY(nanovllm)``
// (``nanovllm/csrc/ops.cpp:48-80``); this library exposes the kernels of this
// engine the same way so they are graph-capturable torch ops.

#include <torch/extension.h>

namespace isb {
at::Tensor gemm(const at::Tensor& a, const at::Tensor& b, int64_t epilogue, int64_t splits);
std::tuple<at::Tensor, at::Tensor> lm_head_sample(const at::Tensor& h, const at::Tensor& w, const at::Tensor& temps,
                                                  const at::Tensor& rng, int64_t vocab_offset);
int64_t gemm_error_word();
at::Tensor gemm_timeline(const at::Tensor& a, const at::Tensor& b, int64_t splits);
at::Tensor gemm_accum_timeline(const at::Tensor& a, const at::Tensor& b, at::Tensor acc, int64_t splits);
void gemm_accum(const at::Tensor& a, const at::Tensor& b, at::Tensor acc, int64_t splits);
at::Tensor gemm_accum_norm(const at::Tensor& a, const at::Tensor& b, at::Tensor acc, at::Tensor residual,
                           const at::Tensor& w, double eps, bool zc);
at::Tensor add_rmsnorm_acc(at::Tensor acc, at::Tensor residual, const at::Tensor& w, double eps, bool zc);
at::Tensor silu_mul_acc(at::Tensor acc, int64_t rows);
at::Tensor rmsnorm(const at::Tensor& x, const at::Tensor& w, double eps, bool zc);
at::Tensor add_rmsnorm(const at::Tensor& x, at::Tensor residual, const at::Tensor& w, double eps, bool zc);
std::tuple<at::Tensor, at::Tensor> embed_rmsnorm(const at::Tensor& ids, const at::Tensor& table, const at::Tensor& w,
                                                 double eps, bool zc);
at::Tensor embed(const at::Tensor& ids, const at::Tensor& table, int64_t vocab_start);
at::Tensor gdn_decode(const at::Tensor& proj, const at::Tensor& slots, const at::Tensor& conv_w, const at::Tensor& A_log,
                      const at::Tensor& dt_bias, const at::Tensor& norm_w, at::Tensor rec, at::Tensor conv, int64_t hk,
                      int64_t hv, int64_t dk, int64_t dv, double eps);
void gdn_chunk_debug(const at::Tensor& buf);
at::Tensor gdn_prefill_chunked(const at::Tensor& proj, const at::Tensor& cu_seqlens, const at::Tensor& slots,
                               const at::Tensor& chunk_info, int64_t nc, const at::Tensor& conv_w,
                               const at::Tensor& A_log, const at::Tensor& dt_bias, const at::Tensor& norm_w,
                               at::Tensor rec, at::Tensor conv, int64_t hk, int64_t hv, double eps);
at::Tensor gdn_prefill(const at::Tensor& proj, const at::Tensor& cu_seqlens, const at::Tensor& slots,
                       const at::Tensor& conv_w, const at::Tensor& A_log, const at::Tensor& dt_bias,
                       const at::Tensor& norm_w, at::Tensor rec, at::Tensor conv, int64_t hk, int64_t hv, int64_t dk,
                       int64_t dv, double eps, int64_t max_seqlen);
at::Tensor gdn_scan_history(const at::Tensor& proj, const at::Tensor& cu_seqlens, const at::Tensor& slots,
                            const at::Tensor& conv_w, const at::Tensor& A_log, const at::Tensor& dt_bias,
                            const at::Tensor& norm_w, at::Tensor rec, at::Tensor conv, int64_t hk, int64_t hv,
                            double eps, bool write_final, const c10::optional<at::Tensor>& hist_row,
                            c10::optional<at::Tensor> hist_rec, c10::optional<at::Tensor> hist_conv,
                            c10::optional<at::Tensor> rec_k, c10::optional<at::Tensor> rec_delta,
                            c10::optional<at::Tensor> rec_g);
void gdn_replay_commit(at::Tensor rec, const at::Tensor& slots, const at::Tensor& keys, const at::Tensor& deltas,
                       const at::Tensor& gs, const at::Tensor& lens, int64_t steps);
void gdn_conv_commit(at::Tensor conv, const at::Tensor& hist, const at::Tensor& slots, const at::Tensor& bounds,
                     int64_t steps);
std::tuple<at::Tensor, at::Tensor> attn_prepare(const at::Tensor& qkv, const at::Tensor& positions,
                                                const at::Tensor& slot_mapping, const at::Tensor& qn,
                                                const at::Tensor& kn, const at::Tensor& cos_sin, at::Tensor kc,
                                                at::Tensor vc, int64_t Hq, int64_t Hkv, int64_t hd, double eps,
                                                bool gated, bool zc);
at::Tensor attention_decode(const at::Tensor& q, const at::Tensor& gate, const at::Tensor& kc, const at::Tensor& vc,
                            const at::Tensor& ctx_lens, const at::Tensor& block_tables, double scale, bool gated);
at::Tensor attention_decode_tc(const at::Tensor& q, const at::Tensor& gate, const at::Tensor& kc, const at::Tensor& vc,
                               const at::Tensor& ctx_lens, const at::Tensor& block_tables, double scale, bool gated);
at::Tensor attention_prefill(const at::Tensor& q, const at::Tensor& gate, const at::Tensor& kc, const at::Tensor& vc,
                             const at::Tensor& cu_q, const at::Tensor& ctx_lens, const at::Tensor& block_tables,
                             double scale, bool gated, int64_t max_seqlen_q);
at::Tensor attention_prefill_tc(const at::Tensor& q, const at::Tensor& gate, const at::Tensor& kc, const at::Tensor& vc,
                                const at::Tensor& cu_q, const at::Tensor& ctx_lens, const at::Tensor& block_tables,
                                double scale, bool gated, int64_t max_seqlen_q);
int64_t attn_tc_error_word();
int64_t gdn_error_word();
void quantize_state_int8(const at::Tensor& state, at::Tensor q, at::Tensor scale);
void dequantize_state_int8(const at::Tensor& q, const at::Tensor& scale, at::Tensor out);
void copy_kv_page(at::Tensor kc, at::Tensor vc, int64_t src, int64_t dst, int64_t n);

int64_t attn_error_word();
int64_t comm_error_word();
void tp_gemm_rs_norm(const at::Tensor& a, const at::Tensor& b, const at::Tensor& slots, int64_t slot_rows,
                     const at::Tensor& flags, int64_t rank, const at::Tensor& slots_local, at::Tensor residual,
                     const at::Tensor& w, at::Tensor xout, at::Tensor ctl, double eps, bool zc);
int64_t tp_gemm_rs(const at::Tensor& a, const at::Tensor& b, const at::Tensor& slots, int64_t slot_rows,
                   at::Tensor staging, const at::Tensor& flags, int64_t rank, int64_t own_rows, int64_t splits,
                   bool one_shot);
void tp_norm_allgather(const at::Tensor& slots, at::Tensor residual, const at::Tensor& w, const at::Tensor& xdst,
                       const at::Tensor& ag_flags, at::Tensor ctl, int64_t T, int64_t own_rows, int64_t rank,
                       int64_t rs_incr, double eps, bool zc, bool wait_gather, bool one_shot);
std::tuple<at::Tensor, at::Tensor> symm_alloc(int64_t nbytes);
int64_t symm_open(const at::Tensor& handle);
void symm_close(int64_t ptr);
at::Tensor xrank_argmax(const at::Tensor& val, const at::Tensor& idx, const at::Tensor& xbufs,
                        const at::Tensor& peer_flags, at::Tensor my_flags, const at::Tensor& my_xbuf, int64_t rank,
                        int64_t max_rows);
void comm_set_wait_timeout(int64_t ns);
at::Tensor step_status(const at::Tensor& toks, const at::Tensor& words);
int64_t gemm_error_word_address();
int64_t attn_error_word_address();
int64_t comm_error_word_address();
int64_t attn_tc_error_word_address();
int64_t gdn_error_word_address();

// Device addresses of the error words, in the bit order of ``step_status`` / ``error_word``:
// gemm, attention, communication, tensor-core attention, GDN.
at::Tensor error_word_addresses() {
  return at::tensor({gemm_error_word_address(), attn_error_word_address(), comm_error_word_address(),
                     attn_tc_error_word_address(), gdn_error_word_address()},
                    at::TensorOptions().dtype(at::kLong));
}

int64_t error_word() {
  return gemm_error_word() | (attn_error_word() << 8) | (comm_error_word() << 16) | (attn_tc_error_word() << 24) |
         (gdn_error_word() << 32);
}
}  // namespace isb

TORCH_LIBRARY(isb, m) {
  m.def("gemm(Tensor a, Tensor b, int epilogue, int splits=0) -> Tensor");
  m.def("lm_head_sample(Tensor hidden, Tensor weight, Tensor temps, Tensor rng, int vocab_offset) -> (Tensor, Tensor)");
  m.def("rmsnorm(Tensor x, Tensor w, float eps, bool zero_centered) -> Tensor");
  m.def("add_rmsnorm(Tensor x, Tensor(a!) residual, Tensor w, float eps, bool zero_centered) -> Tensor");
  m.def("embed_rmsnorm(Tensor ids, Tensor table, Tensor w, float eps, bool zero_centered) -> (Tensor, Tensor)");
  m.def("embed(Tensor ids, Tensor table, int vocab_start) -> Tensor");
  m.def(
      "gdn_decode(Tensor(c!) proj, Tensor slots, Tensor conv_w, Tensor A_log, Tensor dt_bias, Tensor norm_w, "
      "Tensor(a!) rec, Tensor(b!) conv, int hk, int hv, int dk, int dv, float eps) -> Tensor");
  m.def(
      "gdn_prefill_chunked(Tensor proj, Tensor cu_seqlens, Tensor slots, Tensor chunk_info, int nc, Tensor conv_w, "
      "Tensor A_log, Tensor dt_bias, Tensor norm_w, Tensor(a!) rec, Tensor(b!) conv, int hk, int hv, float eps) "
      "-> Tensor");
  m.def(
      "gdn_prefill(Tensor(c!) proj, Tensor cu_seqlens, Tensor slots, Tensor conv_w, Tensor A_log, Tensor dt_bias, "
      "Tensor norm_w, Tensor(a!) rec, Tensor(b!) conv, int hk, int hv, int dk, int dv, float eps, int max_seqlen) "
      "-> Tensor");
  m.def(
      "gdn_scan_history(Tensor(h!) proj, Tensor cu_seqlens, Tensor slots, Tensor conv_w, Tensor A_log, Tensor dt_bias, "
      "Tensor norm_w, Tensor(a!) rec, Tensor(b!) conv, int hk, int hv, float eps, bool write_final, "
      "Tensor? hist_row, Tensor(c!)? hist_rec, Tensor(d!)? hist_conv, Tensor(e!)? rec_k, Tensor(f!)? rec_delta, "
      "Tensor(g!)? rec_g) -> Tensor");
  m.def(
      "gdn_replay_commit(Tensor(a!) rec, Tensor slots, Tensor keys, Tensor deltas, Tensor gs, Tensor lens, "
      "int steps) -> ()");
  m.def("gdn_conv_commit(Tensor(a!) conv, Tensor hist, Tensor slots, Tensor bounds, int steps) -> ()");
  m.def(
      "attn_prepare(Tensor(c!) qkv, Tensor positions, Tensor slot_mapping, Tensor qn, Tensor kn, Tensor cos_sin, "
      "Tensor(a!) k_cache, Tensor(b!) v_cache, int Hq, int Hkv, int hd, float eps, bool gated, bool zero_centered) "
      "-> (Tensor, Tensor)");
  m.def(
      "attention_decode(Tensor q, Tensor gate, Tensor k_cache, Tensor v_cache, Tensor context_lens, "
      "Tensor block_tables, float scale, bool gated) -> Tensor");
  m.def(
      "attention_decode_tc(Tensor q, Tensor gate, Tensor k_cache, Tensor v_cache, Tensor context_lens, "
      "Tensor block_tables, float scale, bool gated) -> Tensor");
  m.def(
      "attention_prefill_tc(Tensor q, Tensor gate, Tensor kc, Tensor vc, Tensor cu_q, Tensor ctx_lens, "
      "Tensor block_tables, float scale, bool gated, int max_seqlen_q) -> Tensor");
  m.def(
      "attention_prefill(Tensor q, Tensor gate, Tensor k_cache, Tensor v_cache, Tensor cu_seqlens_q, "
      "Tensor context_lens, Tensor block_tables, float scale, bool gated, int max_seqlen_q) -> Tensor");
  m.def("quantize_state_int8(Tensor state, Tensor(a!) q, Tensor(b!) scale) -> ()");
  m.def("dequantize_state_int8(Tensor q, Tensor scale, Tensor(a!) out) -> ()");
  m.def("copy_kv_page(Tensor(a!) k_cache, Tensor(b!) v_cache, int src, int dst, int n) -> ()");
  m.def("error_word() -> int");
  m.def("gemm_timeline(Tensor a, Tensor b, int splits) -> Tensor");
  m.def("gemm_accum_timeline(Tensor a, Tensor b, Tensor(a!) acc, int splits) -> Tensor");
  m.def("gemm_accum(Tensor a, Tensor b, Tensor(a!) acc, int splits=0) -> ()");
  m.def("gemm_accum_norm(Tensor a, Tensor b, Tensor(a!) acc, Tensor(b!) residual, Tensor w, float eps, "
        "bool zero_centered) -> Tensor");
  m.def("add_rmsnorm_acc(Tensor(a!) acc, Tensor(b!) residual, Tensor w, float eps, bool zero_centered) -> Tensor");
  m.def("silu_mul_acc(Tensor(a!) acc, int rows) -> Tensor");
  m.def("tp_gemm_rs_norm(Tensor a, Tensor b, Tensor slots, int slot_rows, Tensor flags, int rank, Tensor slots_local, "
        "Tensor(a!) residual, Tensor w, Tensor(b!) xout, Tensor(c!) ctl, float eps, bool zero_centered) -> ()");
  m.def("tp_gemm_rs(Tensor a, Tensor b, Tensor slots, int slot_rows, Tensor(a!) staging, Tensor flags, "
        "int rank, int own_rows, int splits=0, bool one_shot=False) -> int");
  m.def("tp_norm_allgather(Tensor slots, Tensor(b!) residual, Tensor w, Tensor xdst, Tensor ag_flags, "
        "Tensor(c!) ctl, int T, int own_rows, int rank, int rs_incr, float eps, bool zero_centered, "
        "bool wait_gather, bool one_shot=False) -> ()");
  m.def("comm_set_wait_timeout(int ns) -> ()");
  m.def("step_status(Tensor toks, Tensor words) -> Tensor");
  m.def("error_word_addresses() -> Tensor");
  m.def("gdn_chunk_debug(Tensor buf) -> ()");
  m.def("symm_alloc(int nbytes) -> (Tensor, Tensor)");
  m.def("symm_open(Tensor handle) -> int");
  m.def("symm_close(int ptr) -> ()");
  m.def("xrank_argmax(Tensor val, Tensor idx, Tensor xbufs, Tensor peer_flags, Tensor(a!) my_flags, Tensor my_xbuf, "
        "int rank, int max_rows) -> Tensor");
}

TORCH_LIBRARY_IMPL(isb, CUDA, m) {
  m.impl("gemm", &isb::gemm);
  m.impl("lm_head_sample", &isb::lm_head_sample);
  m.impl("rmsnorm", &isb::rmsnorm);
  m.impl("add_rmsnorm", &isb::add_rmsnorm);
  m.impl("embed_rmsnorm", &isb::embed_rmsnorm);
  m.impl("embed", &isb::embed);
  m.impl("gdn_decode", &isb::gdn_decode);
  m.impl("gdn_prefill", &isb::gdn_prefill);
  m.impl("gdn_prefill_chunked", &isb::gdn_prefill_chunked);
  m.impl("attention_prefill_tc", &isb::attention_prefill_tc);
  m.impl("gdn_scan_history", &isb::gdn_scan_history);
  m.impl("gdn_replay_commit", &isb::gdn_replay_commit);
  m.impl("gdn_conv_commit", &isb::gdn_conv_commit);
  m.impl("attn_prepare", &isb::attn_prepare);
  m.impl("attention_decode", &isb::attention_decode);
  m.impl("attention_decode_tc", &isb::attention_decode_tc);
  m.impl("attention_prefill", &isb::attention_prefill);
  m.impl("quantize_state_int8", &isb::quantize_state_int8);
  m.impl("dequantize_state_int8", &isb::dequantize_state_int8);
  m.impl("copy_kv_page", &isb::copy_kv_page);
  m.impl("gemm_timeline", &isb::gemm_timeline);
  m.impl("gemm_accum_timeline", &isb::gemm_accum_timeline);
  m.impl("gemm_accum", &isb::gemm_accum);
  m.impl("gemm_accum_norm", &isb::gemm_accum_norm);
  m.impl("add_rmsnorm_acc", &isb::add_rmsnorm_acc);
  m.impl("silu_mul_acc", &isb::silu_mul_acc);
  m.impl("tp_gemm_rs", &isb::tp_gemm_rs);
  m.impl("tp_gemm_rs_norm", &isb::tp_gemm_rs_norm);
  m.impl("tp_norm_allgather", &isb::tp_norm_allgather);
  m.impl("step_status", &isb::step_status);
  m.impl("xrank_argmax", &isb::xrank_argmax);
}

TORCH_LIBRARY_IMPL(isb, CompositeExplicitAutograd, m) {
  m.impl("gdn_chunk_debug", &isb::gdn_chunk_debug);
  m.impl("error_word", &isb::error_word);
  m.impl("symm_alloc", &isb::symm_alloc);
  m.impl("symm_open", &isb::symm_open);
  m.impl("symm_close", &isb::symm_close);
  m.impl("comm_set_wait_timeout", &isb::comm_set_wait_timeout);
  m.impl("error_word_addresses", &isb::error_word_addresses);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) { m.doc() = "sm_100a kernels (torch.ops.isb)"; }
