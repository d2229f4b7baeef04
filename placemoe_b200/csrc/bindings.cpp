// Python bindings of the sm_100a kernels (one extension module, built in-tree).
#include <torch/extension.h>

#include "ops.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "placemoe_b200 sm_100a kernels";
  // tcgen05 GEMMs
  m.def("dense_gemm", &pm::dense_gemm);
  m.def("moe_fc1_swiglu", &pm::moe_fc1_swiglu);
  m.def("moe_grouped_gemm", &pm::moe_grouped_gemm);
  m.def("moe_fc2_dgrad_dswiglu", &pm::moe_fc2_dgrad_dswiglu);
  m.def("moe_wgrad", &pm::moe_wgrad);
  // norms / rotary
  m.def("rmsnorm_fwd", &pm::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &pm::rmsnorm_bwd);
  m.def("add_rmsnorm_fwd", &pm::add_rmsnorm_fwd, "h = x + res (bf16), y = rmsnorm(h): returns [h, y, rstd]");
  m.def("rmsnorm_bwd_add", &pm::rmsnorm_bwd_add, "rmsnorm backward plus the residual-path gradient");
  m.def("qkv_rope_fwd", &pm::qkv_rope_fwd);
  m.def("qkv_rope_bwd", &pm::qkv_rope_bwd);
  // routing
  m.def("router_topk_fwd", &pm::router_topk_fwd);
  m.def("router_topk_bwd", &pm::router_topk_bwd);
  m.def("moe_plan", &pm::moe_plan);
  m.def("gather_rows", &pm::gather_rows);
  m.def("sum_rows", &pm::sum_rows);
  m.def("gather_scalar", &pm::gather_scalar);
  // optimizer
  m.def("adamw_build_table", &pm::adamw_build_table);
  m.def("adamw_step", &pm::adamw_step);
  m.def("sq_norm_build_table", &pm::sq_norm_build_table);
  m.def("sq_norm", &pm::sq_norm);
  // attention
  m.def("attn_fwd", &pm::attn_fwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("S"),
        py::arg("doc_lo") = py::none());
  m.def("attn_bwd", &pm::attn_bwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"),
        py::arg("dout"), py::arg("S"), py::arg("doc_hi") = py::none());
  // loss
  m.def("ce_fwd_bwd", &pm::ce_fwd_bwd);
  // peer-to-peer data plane
  m.def("p2p_put_rows", &pm::p2p_put_rows);
  m.def("p2p_put_words", &pm::p2p_put_words);
  m.def("p2p_allgather_words", &pm::p2p_allgather_words);
  m.def("p2p_barrier", &pm::p2p_barrier);
  m.def("p2p_reduce_f32", &pm::p2p_reduce_f32);
  m.def("p2p_sum_f32", &pm::p2p_sum_f32);
  m.def("p2p_pull", &pm::p2p_pull);
  // fused expert-parallel dispatch / combine (one cooperative kernel per phase)
  m.def("ep_scratch_ints", &pm::ep_scratch_ints);
  m.def("ep_phase_marks", &pm::ep_phase_marks, "int64[24] buffer for per-phase timestamps of the EP kernels");
  m.def("ep_dispatch", &pm::ep_dispatch);
  m.def("ep_combine", &pm::ep_combine);
  m.def("ep_scatter", &pm::ep_scatter);
  m.def("sp_exchange", &pm::sp_exchange);
  m.def("device_error", &pm::device_error, "read (and optionally clear) the kernels' error words");
#ifdef PLACEMOE_DEBUG_BOUNDS
  m.def("debug_bounds", [] { return true; }, "built with the index checks of the debug build");
#else
  m.def("debug_bounds", [] { return false; }, "built with the index checks of the debug build");
#endif
}
