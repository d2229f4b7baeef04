// CPU cores of the PlaceMoE planner (declarations).
#pragma once
#include <torch/extension.h>

#include <tuple>
#include <vector>

namespace pmp {
void accumulate_route_stats(torch::Tensor routes, int64_t source_rank, torch::Tensor demand, torch::Tensor affinity);
torch::Tensor evaluate_routes(std::vector<torch::Tensor> routes, torch::Tensor mapping, torch::Tensor slot_rank,
                              double row_bytes, double meta_bytes);
torch::Tensor evaluate_routes_batch(std::vector<torch::Tensor> routes, torch::Tensor mapping, torch::Tensor slot_rank,
                                    double row_bytes, double meta_bytes);
double optimize_mapping(torch::Tensor demand, torch::Tensor affinity, torch::Tensor slot_to_logical,
                        torch::Tensor slot_rank, torch::Tensor mapping, double omega, double lambda_local,
                        double gamma, int64_t sweeps);
int64_t refine_partition(torch::Tensor affinity, torch::Tensor weight, torch::Tensor labels, torch::Tensor item_expert,
                         torch::Tensor ranks_per_group, double omega, double gamma, int64_t limit);
std::vector<double> optimize_mapping_normalized(torch::Tensor demand, torch::Tensor affinity,
                                                torch::Tensor slot_to_logical, torch::Tensor slot_rank,
                                                torch::Tensor mapping, int64_t ranks_per_node,
                                                double assignment_weight, double node_weight, double rank_weight,
                                                int64_t sweeps);
torch::Tensor community_intersection_hits(torch::Tensor hist);
torch::Tensor community_mask_histogram(std::vector<torch::Tensor> routes, torch::Tensor community,
                                       int64_t ranks_per_unit, int64_t num_communities);
std::tuple<torch::Tensor, double, int64_t, int64_t> optimize_community_mapping(
    torch::Tensor allowed, torch::Tensor assignments, torch::Tensor hits, double comm_ms_per_token,
    double ms_per_assignment, int64_t ranks_per_unit, int64_t row_limit, int64_t beam_width, int64_t sweeps);
}  // namespace pmp
