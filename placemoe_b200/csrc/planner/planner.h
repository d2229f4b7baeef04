// CPU cores of the PlaceMoE planner (declarations).
#pragma once
#include <torch/extension.h>

#include <vector>

namespace pmp {
void accumulate_route_stats(torch::Tensor routes, int64_t source_rank, torch::Tensor demand, torch::Tensor affinity);
torch::Tensor evaluate_routes(std::vector<torch::Tensor> routes, torch::Tensor mapping, torch::Tensor slot_rank,
                              double row_bytes, double meta_bytes);
double optimize_mapping(torch::Tensor demand, torch::Tensor affinity, torch::Tensor slot_to_logical,
                        torch::Tensor slot_rank, torch::Tensor mapping, double omega, double lambda_local,
                        double gamma, int64_t sweeps);
int64_t refine_partition(torch::Tensor affinity, torch::Tensor weight, torch::Tensor labels, torch::Tensor item_expert,
                         torch::Tensor ranks_per_group, double omega, double gamma, int64_t limit);
}  // namespace pmp
