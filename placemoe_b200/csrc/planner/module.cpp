// pybind11 module of the PlaceMoE planner cores.
#include <torch/extension.h>

#include "planner.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "placemoe_b200 planner C++ cores";
  m.def("accumulate_route_stats", &pmp::accumulate_route_stats, "demand/affinity accumulation for one source rank");
  m.def("evaluate_routes", &pmp::evaluate_routes, "exact one-level route replay of one step");
  m.def("evaluate_routes_batch", &pmp::evaluate_routes_batch,
        "exact one-level route replay of several steps (S tensors per step), one result row per step");
  m.def("optimize_mapping", &pmp::optimize_mapping, "mapping coordinate descent (in place)");
  m.def("refine_partition", &pmp::refine_partition, "capacity-constrained pairwise exchange (in place)");
  m.def("optimize_mapping_normalized", &pmp::optimize_mapping_normalized,
        "scale-normalised mapping proposal (in place); returns [peak load, sweeps, changes]");
  m.def("community_intersection_hits", &pmp::community_intersection_hits, "tokens whose community mask meets X");
  m.def("community_mask_histogram", &pmp::community_mask_histogram,
        "tokens per (source unit, community mask), summed over steps of `sources_per_step` sources",
        py::arg("routes"), py::arg("community"), py::arg("ranks_per_unit"), py::arg("num_communities"),
        py::arg("sources_per_step") = 0);
  m.def("optimize_community_mapping", &pmp::optimize_community_mapping,
        "block mapping of (source unit, community) -> destination unit");
}
