// Host entry points of the sm_100a kernels.
#pragma once
#include <torch/extension.h>

#include <vector>

namespace pm {
// gemm_dense.cu, gemm_moe_fwd.cu, gemm_moe_bwd.cu (kernel template in gemm_sm100.cuh)
void dense_gemm(torch::Tensor a, torch::Tensor b, torch::Tensor out, bool a_mn, bool b_mn, bool accumulate);
void moe_fc1_swiglu(torch::Tensor x, torch::Tensor w1, torch::Tensor offsets, torch::Tensor scale, torch::Tensor h,
                    c10::optional<torch::Tensor> gu_out, int64_t align, c10::optional<torch::Tensor> gather_idx);
void moe_grouped_gemm(torch::Tensor a, torch::Tensor w, torch::Tensor offsets, torch::Tensor out, bool b_mn,
                      int64_t align);
void moe_fc2_dgrad_dswiglu(torch::Tensor dy, torch::Tensor w2, torch::Tensor offsets, torch::Tensor gu,
                           torch::Tensor scale, torch::Tensor dgu, torch::Tensor dscale, int64_t align);
void moe_wgrad(torch::Tensor a, torch::Tensor b, torch::Tensor offsets, torch::Tensor dw, bool accumulate,
               c10::optional<torch::Tensor> gather_idx);

// norm_rope.cu
std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps);
std::vector<torch::Tensor> add_rmsnorm_fwd(torch::Tensor x, torch::Tensor res, torch::Tensor w, double eps);
torch::Tensor rmsnorm_bwd_add(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dw,
                              torch::Tensor dres);
torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dw);
std::vector<torch::Tensor> qkv_rope_fwd(torch::Tensor qkv, torch::Tensor pos, torch::Tensor rope,
                                        c10::optional<torch::Tensor> qw, c10::optional<torch::Tensor> kw, int64_t Hq,
                                        int64_t Hkv, int64_t D, int64_t q_group, int64_t k_group, double eps);
torch::Tensor qkv_rope_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor qkv, torch::Tensor pos,
                           torch::Tensor rope, c10::optional<torch::Tensor> qw, c10::optional<torch::Tensor> kw,
                           torch::Tensor rq, torch::Tensor rk, c10::optional<torch::Tensor> dqw,
                           c10::optional<torch::Tensor> dkw, int64_t Hq, int64_t Hkv, int64_t D, int64_t q_group,
                           int64_t k_group);

// moe_route.cu
std::vector<torch::Tensor> router_topk_fwd(torch::Tensor logits, c10::optional<torch::Tensor> bias, int64_t K,
                                           bool renorm);
torch::Tensor router_topk_bwd(torch::Tensor logits, c10::optional<torch::Tensor> bias, torch::Tensor idx,
                              torch::Tensor dw, c10::optional<torch::Tensor> aux, bool renorm);
std::vector<torch::Tensor> moe_plan(torch::Tensor idx, c10::optional<torch::Tensor> lut,
                                    c10::optional<torch::Tensor> weights, int64_t num_slots, int64_t capacity,
                                    int64_t align);
void gather_rows(torch::Tensor src, torch::Tensor row_token, c10::optional<torch::Tensor> end, torch::Tensor out);
void sum_rows(torch::Tensor src, torch::Tensor row_of, torch::Tensor out);
torch::Tensor gather_scalar(torch::Tensor vals, torch::Tensor row_of);

// optim.cu
std::vector<torch::Tensor> adamw_build_table(std::vector<torch::Tensor> params, std::vector<torch::Tensor> grads,
                                             std::vector<torch::Tensor> exp_avg, std::vector<torch::Tensor> exp_avg_sq,
                                             std::vector<c10::optional<torch::Tensor>> shadows);
void adamw_step(torch::Tensor table, torch::Tensor meta, double lr, double beta1, double beta2, double eps, double wd,
                int64_t step, c10::optional<torch::Tensor> grad_scale);
std::vector<torch::Tensor> sq_norm_build_table(std::vector<torch::Tensor> grads, std::vector<double> weights);
void sq_norm(torch::Tensor table, torch::Tensor meta, torch::Tensor out);

// attention_sm100.cu
std::vector<torch::Tensor> attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, int64_t S,
                                    c10::optional<torch::Tensor> doc_lo);
std::vector<torch::Tensor> attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o,
                                    torch::Tensor lse, torch::Tensor dout, int64_t S, c10::optional<torch::Tensor> doc_hi);

// loss.cu
void ce_fwd_bwd(torch::Tensor logits, torch::Tensor labels, int64_t ignore_index, double grad_scale,
                torch::Tensor loss_sum, c10::optional<torch::Tensor> row_loss);

// p2p.cu
void p2p_put_rows(torch::Tensor src, c10::optional<torch::Tensor> src_row, torch::Tensor dst_rank, torch::Tensor dst_row,
                  c10::optional<torch::Tensor> n_dev, int64_t n_host, torch::Tensor peers, int64_t region_off,
                  int64_t ld);
void p2p_put_words(torch::Tensor vals, torch::Tensor dst_rank, torch::Tensor dst_idx, c10::optional<torch::Tensor> n_dev,
                   int64_t n_host, torch::Tensor peers, int64_t region_off);
void p2p_allgather_words(torch::Tensor vals, torch::Tensor peers, int64_t region_off, int64_t my_rank);
void p2p_barrier(torch::Tensor peers, int64_t flags_off, int64_t my_rank, int64_t epoch, double timeout_s,
                 torch::Tensor status);
void p2p_reduce_f32(torch::Tensor out, torch::Tensor peers, torch::Tensor ranks, int64_t region_off);
void p2p_sum_f32(torch::Tensor out, torch::Tensor peers, torch::Tensor src_rank, torch::Tensor src_off);
void p2p_pull(torch::Tensor dst, torch::Tensor peers, int64_t src_rank, int64_t region_off);

// fused expert-parallel dispatch / combine over peer memory (ep_fused.cu)
int64_t ep_scratch_ints(int64_t world, int64_t slots);
void ep_phase_marks(c10::optional<torch::Tensor> buf);
void ep_dispatch(torch::Tensor x, torch::Tensor idx, torch::Tensor w, torch::Tensor dest_tab, torch::Tensor slot_tab,
                 torch::Tensor peers, std::vector<int64_t> geo, torch::Tensor scratch, torch::Tensor status,
                 int64_t epoch, double timeout_s, torch::Tensor pos, torch::Tensor dst, torch::Tensor offsets,
                 torch::Tensor row_scale);
void ep_combine(torch::Tensor rows, c10::optional<torch::Tensor> dscale, torch::Tensor pos, torch::Tensor dst,
                torch::Tensor offsets, torch::Tensor peers, std::vector<int64_t> geo, torch::Tensor scratch,
                torch::Tensor status, int64_t epoch, double timeout_s, torch::Tensor out,
                c10::optional<torch::Tensor> dw_out);
void ep_scatter(torch::Tensor dy, torch::Tensor pos, torch::Tensor dst, torch::Tensor offsets, torch::Tensor peers,
                std::vector<int64_t> geo, torch::Tensor scratch, torch::Tensor status, int64_t epoch,
                double timeout_s);

// Ulysses sequence-parallel exchange over peer memory (sp_exchange.cu)
void sp_exchange(torch::Tensor in, torch::Tensor out, torch::Tensor peers, std::vector<int64_t> geo,
                 torch::Tensor scratch, torch::Tensor status, int64_t epoch, double timeout_s);

int device_error(bool reset);
}  // namespace pm

// Per-translation-unit error words (see common.cuh).
int pm_error_gemm_dense(bool reset);
int pm_error_gemm_moe_fwd(bool reset);
int pm_error_gemm_moe_bwd(bool reset);
int pm_error_norm(bool reset);
int pm_error_route(bool reset);
int pm_error_optim(bool reset);
int pm_error_loss(bool reset);
int pm_error_attn(bool reset);
int pm_error_p2p(bool reset);
