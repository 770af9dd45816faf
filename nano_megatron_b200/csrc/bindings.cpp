// Python bindings of the sm_100a kernel library (module nano_megatron_b200._C).
#include <torch/extension.h>

#include "launch_counter.h"

void gemm_tc(at::Tensor a, bool a_mn, at::Tensor b, bool b_mn, at::Tensor c, int64_t epi,
             c10::optional<at::Tensor> residual, c10::optional<at::Tensor> alpha_t, double alpha,
             double beta, c10::optional<at::Tensor> aux, int64_t swiglu_up_row,
             c10::optional<at::Tensor> positions, c10::optional<at::Tensor> inv_freq,
             int64_t head_dim, int64_t rope_cols, int64_t pos_div, at::Tensor status,
             int64_t bn_override, int64_t max_ctas, c10::optional<at::Tensor> rope_cs,
             c10::optional<at::Tensor> ce_part);
void flash_attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse,
                    double softmax_scale, bool causal, int64_t q_offset, int64_t k_offset);
void flash_attn_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor dout,
                    at::Tensor lse, at::Tensor dq, at::Tensor dk, at::Tensor dv,
                    at::Tensor delta_ws, at::Tensor dq_acc_ws, double softmax_scale, bool causal,
                    int64_t q_offset, int64_t k_offset, c10::optional<at::Tensor> q_pos,
                    c10::optional<at::Tensor> k_pos, c10::optional<at::Tensor> inv_freq);
void flash_attn_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor lse,
                       double softmax_scale, bool causal, int64_t q_offset, int64_t k_offset,
                       at::Tensor status, int64_t pull_src, c10::optional<at::Tensor> pull_dst,
                       int64_t pull_flag, int64_t pull_epoch);
void flash_attn_bwd_prep(at::Tensor o, at::Tensor dout, at::Tensor delta, at::Tensor dq_acc);
void flash_attn_bwd_dq_convert(at::Tensor dq_acc, at::Tensor dq, c10::optional<at::Tensor> q_pos,
                               c10::optional<at::Tensor> inv_freq);
int64_t attn_bwd_softmax_groups();
int64_t attn_bwd_trace_slots();
void flash_attn_bwd_tc_kv(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor dout,
                          at::Tensor lse, at::Tensor delta, at::Tensor dq_acc, at::Tensor dk,
                          at::Tensor dv, double softmax_scale, bool causal, int64_t q_offset,
                          int64_t k_offset, c10::optional<at::Tensor> k_pos,
                          c10::optional<at::Tensor> inv_freq, at::Tensor status,
                          int64_t pull_src, c10::optional<at::Tensor> pull_dst,
                          int64_t pull_flag, int64_t pull_epoch, c10::optional<at::Tensor> k_cs,
                          c10::optional<at::Tensor> trace, int64_t dq_slot_stride);
void set_deterministic(bool on);
bool get_deterministic();
void slots_sum(at::Tensor slots, at::Tensor out, bool accumulate);
void rmsnorm_fwd(at::Tensor x, at::Tensor w, at::Tensor y, at::Tensor rstd, double eps);
void rmsnorm_bwd(at::Tensor x, at::Tensor w, at::Tensor dy, at::Tensor rstd, at::Tensor dx,
                 c10::optional<at::Tensor> dw, c10::optional<at::Tensor> dres);
void swiglu_fwd(at::Tensor gu, at::Tensor h);
void swiglu_bwd(at::Tensor gu, at::Tensor dh, at::Tensor dgu);
void rope_inplace(at::Tensor x, int64_t ncols, int64_t head_dim, at::Tensor pos,
                  at::Tensor inv_freq, bool inverse);
void embedding_fwd(at::Tensor ids, at::Tensor w, int64_t vstart, at::Tensor out);
void embedding_bwd(at::Tensor ids, at::Tensor dy, at::Tensor grad, int64_t vstart);
void ce_stats(at::Tensor logits, at::Tensor labels, int64_t vstart, at::Tensor stats);
void ce_finish(at::Tensor logits, at::Tensor labels, int64_t vstart, at::Tensor stats,
               int64_t shards, at::Tensor loss_row, bool write_grad);
void ce_fused(at::Tensor logits, at::Tensor labels, at::Tensor loss_row, bool write_grad);
void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v,
                c10::optional<at::Tensor> p_bf16, double lr, double beta1, double beta2,
                double eps, double wd, int64_t step, c10::optional<at::Tensor> grad_scale,
                c10::optional<at::Tensor> lr_t);
at::Tensor sumsq_partials(at::Tensor x);
void gemm_tc_ag(at::Tensor a_local, std::vector<int64_t> shard_ptrs,
                std::vector<int64_t> shard_ptrs_odd, int64_t lda, at::Tensor b, bool b_mn,
                at::Tensor c, int64_t epi, c10::optional<at::Tensor> xfull,
                c10::optional<at::Tensor> aux, int64_t swiglu_up_row,
                c10::optional<at::Tensor> positions, c10::optional<at::Tensor> inv_freq,
                int64_t head_dim, int64_t rope_cols, int64_t pos_div, int64_t rank,
                int64_t flags_ptr, int64_t epoch_ptr, at::Tensor status,
                c10::optional<at::Tensor> rope_cs, c10::optional<at::Tensor> gather_ready,
                c10::optional<at::Tensor> ce_part);
void gemm_tc_rs(at::Tensor a, bool a_mn, at::Tensor b, bool b_mn,
                std::vector<int64_t> staging_ptrs, std::vector<int64_t> staging_ptrs_odd,
                int64_t rows_per_rank, int64_t n_out, int64_t rank, int64_t epoch_ptr,
                at::Tensor status, c10::optional<at::Tensor> alpha_t,
                c10::optional<at::Tensor> out, c10::optional<at::Tensor> residual,
                std::vector<int64_t> tile_flag_ptrs);
void tp_embedding_scatter(at::Tensor ids, at::Tensor w, int64_t vstart, int64_t rows_per_rank,
                          std::vector<int64_t> slots_even, std::vector<int64_t> slots_odd,
                          int64_t epoch_ptr);
void tp_embedding_collect(int64_t slot_even, int64_t slot_odd, at::Tensor out, int64_t tp,
                          int64_t flags_ptr, int64_t epoch_ptr, at::Tensor status);
void tp_embedding_bwd_gather(at::Tensor ids, std::vector<int64_t> slots_even,
                             std::vector<int64_t> slots_odd, int64_t rows_per_rank, int64_t H,
                             at::Tensor grad, int64_t vstart, int64_t flags_ptr,
                             int64_t epoch_ptr, at::Tensor status);
void tp_ce_stats_scatter(at::Tensor logits, at::Tensor labels, int64_t vstart, int64_t rank,
                         std::vector<int64_t> slots_even, std::vector<int64_t> slots_odd,
                         int64_t epoch_ptr);
void ce_from_parts(at::Tensor logits, at::Tensor labels, at::Tensor parts, int64_t nparts,
                   at::Tensor loss_row, bool write_grad);
void tp_ce_parts_scatter(at::Tensor logits, at::Tensor labels, int64_t vstart, at::Tensor parts,
                         int64_t nparts, int64_t rank, std::vector<int64_t> slots_even,
                         std::vector<int64_t> slots_odd, int64_t epoch_ptr);
void tp_ce_finish_gather(at::Tensor logits, at::Tensor labels, int64_t vstart, int64_t stats_even,
                         int64_t stats_odd, int64_t tp, at::Tensor loss_row, bool write_grad,
                         int64_t flags_ptr, int64_t epoch_ptr, at::Tensor status);
std::tuple<at::Tensor, pybind11::bytes> symm_alloc(int64_t bytes, int64_t device);
int64_t symm_open(pybind11::bytes handle, int64_t device);
void symm_close(int64_t ptr, int64_t device);
void peer_signal(std::vector<int64_t> targets, int64_t epoch_ptr);
void ag_publish(at::Tensor x, int64_t even_ptr, int64_t odd_ptr, int64_t epoch_ptr);
void rs_reduce(int64_t staging_even, int64_t staging_odd, int64_t tp, at::Tensor out,
               c10::optional<at::Tensor> residual, int64_t flags_ptr, int64_t epoch_ptr,
               at::Tensor status);
int64_t replica_reduce_blocks(int64_t len, int64_t device);
void replica_reduce(std::vector<int64_t> grad_ptrs, int64_t self, int64_t off, int64_t len,
                    at::Tensor segments, at::Tensor partials, int64_t flags_ptr,
                    int64_t epoch_ptr, at::Tensor status);
void replica_adamw_gather(std::vector<int64_t> grad_ptrs, std::vector<int64_t> param_ptrs,
                          int64_t self, int64_t off, int64_t len, at::Tensor master,
                          at::Tensor exp_avg, at::Tensor exp_avg_sq, double lr, double beta1,
                          double beta2, double eps, double wd, int64_t step,
                          c10::optional<at::Tensor> grad_scale, c10::optional<at::Tensor> lr_t);
void replica_wait(int64_t flags_ptr, int64_t n, int64_t epoch_ptr, at::Tensor status);
void cp_pull(int64_t src, at::Tensor dst, int64_t flag_ptr, int64_t epoch_ptr, at::Tensor status);
void cp_push(at::Tensor src, int64_t dst_even, int64_t dst_odd, int64_t epoch_ptr);
void cp_reduce(at::Tensor acc, std::vector<int64_t> slots_even, std::vector<int64_t> slots_odd,
               int64_t mask, int64_t flags_ptr, int64_t epoch_ptr, at::Tensor status);
void scale_inplace(at::Tensor x, double s);
void dropout_apply(at::Tensor x, at::Tensor y, double p, int64_t seed);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "nano_megatron_b200 sm_100a kernels (tcgen05 GEMM, flash attention, fused ops)";
  m.def("gemm_tc", &gemm_tc, "tcgen05 GEMM with fused epilogues", py::arg("a"), py::arg("a_mn"),
        py::arg("b"), py::arg("b_mn"), py::arg("c"), py::arg("epi"), py::arg("residual"),
        py::arg("alpha_t"), py::arg("alpha"), py::arg("beta"), py::arg("aux"),
        py::arg("swiglu_up_row"), py::arg("positions"), py::arg("inv_freq"), py::arg("head_dim"),
        py::arg("rope_cols"), py::arg("pos_div"), py::arg("status"), py::arg("bn_override"),
        py::arg("max_ctas"), py::arg("rope_cs") = py::none(), py::arg("ce_part") = py::none());
  m.def("flash_attn_fwd", &flash_attn_fwd);
  m.def("flash_attn_bwd", &flash_attn_bwd);
  m.def("flash_attn_fwd_tc", &flash_attn_fwd_tc,
        "tcgen05/TMEM causal flash attention forward (optionally pulling the next ring block)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"),
        py::arg("softmax_scale"), py::arg("causal"), py::arg("q_offset"), py::arg("k_offset"),
        py::arg("status"), py::arg("pull_src") = 0, py::arg("pull_dst") = py::none(),
        py::arg("pull_flag") = 0, py::arg("pull_epoch") = 0);
  m.def("flash_attn_bwd_prep", &flash_attn_bwd_prep);
  m.def("flash_attn_bwd_dq_convert", &flash_attn_bwd_dq_convert);
  m.def("flash_attn_bwd_tc_kv", &flash_attn_bwd_tc_kv,
        "tcgen05/TMEM attention backward (dK, dV, dQ acc; optionally pulling the next ring block)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("dout"), py::arg("lse"),
        py::arg("delta"), py::arg("dq_acc"), py::arg("dk"), py::arg("dv"),
        py::arg("softmax_scale"), py::arg("causal"), py::arg("q_offset"), py::arg("k_offset"),
        py::arg("k_pos"), py::arg("inv_freq"), py::arg("status"), py::arg("pull_src") = 0,
        py::arg("pull_dst") = py::none(), py::arg("pull_flag") = 0, py::arg("pull_epoch") = 0,
        py::arg("k_cs") = py::none(), py::arg("trace") = py::none(),
        py::arg("dq_slot_stride") = 0);
  m.def("set_deterministic", &set_deterministic,
        "process-wide deterministic kernel mode (fixed-order reductions instead of atomics)");
  m.def("get_deterministic", &get_deterministic);
  m.def("slots_sum", &slots_sum, "out (+)= sum over the leading dim of slots, in order",
        py::arg("slots"), py::arg("out"), py::arg("accumulate"));
  m.def("attn_bwd_trace_slots", &attn_bwd_trace_slots,
        "timestamps per CTA written by the attention backward's optional phase trace");
  m.def("attn_bwd_softmax_groups", &attn_bwd_softmax_groups,
        "softmax warp groups of the attention backward (NMB_ATTN_BWD_SOFTMAX_GROUPS)");
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("rope_inplace", &rope_inplace);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("ce_stats", &ce_stats);
  m.def("ce_finish", &ce_finish);
  m.def("ce_fused", &ce_fused);
  m.def("adamw_step", &adamw_step);
  m.def("sumsq_partials", &sumsq_partials);
  m.def("scale_inplace", &scale_inplace);
  m.def("dropout_apply", &dropout_apply, "counter-based (Philox-4x32-10) dropout, mask = f(seed, index)");
  m.def("gemm_tc_ag", &gemm_tc_ag, "AG->GEMM: A rows gathered from TP peers' symmetric shards",
        py::arg("a_local"), py::arg("shard_ptrs"), py::arg("shard_ptrs_odd"), py::arg("lda"),
        py::arg("b"), py::arg("b_mn"), py::arg("c"), py::arg("epi"), py::arg("xfull"),
        py::arg("aux"), py::arg("swiglu_up_row"), py::arg("positions"), py::arg("inv_freq"),
        py::arg("head_dim"), py::arg("rope_cols"), py::arg("pos_div"), py::arg("rank"),
        py::arg("flags_ptr"), py::arg("epoch_ptr"), py::arg("status"),
        py::arg("rope_cs") = py::none(), py::arg("gather_ready") = py::none(),
        py::arg("ce_part") = py::none());
  m.def("gemm_tc_rs", &gemm_tc_rs, "GEMM->RS: partial tiles stored into the owner's staging",
        py::arg("a"), py::arg("a_mn"), py::arg("b"), py::arg("b_mn"), py::arg("staging_ptrs"),
        py::arg("staging_ptrs_odd"), py::arg("rows_per_rank"), py::arg("n_out"),
        py::arg("rank"), py::arg("epoch_ptr"), py::arg("status"),
        py::arg("alpha_t") = py::none(), py::arg("out") = py::none(),
        py::arg("residual") = py::none(), py::arg("tile_flag_ptrs") = std::vector<int64_t>());
  m.def("tp_embedding_scatter", &tp_embedding_scatter,
        "TP embedding: rows of this vocabulary shard stored into the sequence owners' slots");
  m.def("tp_embedding_collect", &tp_embedding_collect,
        "TP embedding: wait for every rank, copy this rank's slot out");
  m.def("tp_embedding_bwd_gather", &tp_embedding_bwd_gather,
        "TP embedding backward: dY rows of this vocabulary shard read from the owners' slots");
  m.def("tp_ce_stats_scatter", &tp_ce_stats_scatter,
        "TP cross-entropy: per-row shard statistics stored into every rank's slot");
  m.def("ce_from_parts", &ce_from_parts,
        "cross-entropy from the LM-head GEMM's per-tile (max, sum exp): row loss + in-place grad");
  m.def("tp_ce_parts_scatter", &tp_ce_parts_scatter,
        "vocab-parallel CE: per-tile statistics merged and stored into every TP rank's slot");
  m.def("tp_ce_finish_gather", &tp_ce_finish_gather,
        "TP cross-entropy: merge every rank's statistics, loss and in-place gradient");
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("peer_signal", &peer_signal);
  m.def("ag_publish", &ag_publish);
  m.def("rs_reduce", &rs_reduce);
  m.def("replica_reduce_blocks", &replica_reduce_blocks);
  m.def("replica_reduce", &replica_reduce,
        "DP: sum this rank's shard over all replicas' gradient buffers (peer loads) in place, "
        "with per-block partial squared norms");
  m.def("replica_adamw_gather", &replica_adamw_gather,
        "DP: AdamW over this rank's shard, bf16 result stored into every replica's parameters");
  m.def("replica_wait", &replica_wait, "DP: bounded wait for every replica's flag");
  m.def("cp_pull", &cp_pull, "CP ring: pull a peer's published block into local memory");
  m.def("cp_push", &cp_push, "CP ring: store a dK/dV partial into its owner's return slot");
  m.def("cp_reduce", &cp_reduce, "CP ring: add the returned partials once every rank signalled");
  m.def("launch_count", []() { return nmb::launch_counter().load(); },
        "number of kernel launches issued by this library so far (graph replays included)");
  m.def("record_graph_launches", [](int64_t n) { nmb::launch_counter() += n; },
        "count `n` library kernels launched by one CUDA-graph replay");
}
