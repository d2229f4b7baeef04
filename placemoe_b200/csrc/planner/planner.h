// CPU cores of the PlaceMoE planner (declarations).
#pragma once
#include <torch/extension.h>

#include <ATen/Parallel.h>

#include <algorithm>
#include <atomic>
#include <thread>
#include <tuple>
#include <vector>

namespace pmp {

// fn(i) for i in [0, items) on up to at::get_num_threads() threads (the caller's torch thread
// setting); items are claimed dynamically, so fn must be safe to run concurrently for distinct i.
template <typename F>
void run_pool(int64_t items, F&& fn) {
  const int64_t nt = std::max<int64_t>(1, std::min<int64_t>(items, at::get_num_threads()));
  if (nt == 1) {
    for (int64_t i = 0; i < items; ++i) fn(i);
    return;
  }
  std::atomic<int64_t> next{0};
  std::vector<std::thread> pool;
  pool.reserve(nt);
  for (int64_t w = 0; w < nt; ++w)
    pool.emplace_back([&] {
      for (int64_t i = next.fetch_add(1); i < items; i = next.fetch_add(1)) fn(i);
    });
  for (auto& th : pool) th.join();
}

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
                                       int64_t ranks_per_unit, int64_t num_communities, int64_t sources_per_step);
std::tuple<torch::Tensor, double, int64_t, int64_t> optimize_community_mapping(
    torch::Tensor allowed, torch::Tensor assignments, torch::Tensor hits, double comm_ms_per_token,
    double ms_per_assignment, int64_t ranks_per_unit, int64_t row_limit, int64_t beam_width, int64_t sweeps);
}  // namespace pmp
