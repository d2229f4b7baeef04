// CPU cores of the PlaceMoE planner: route statistics.
//
// demand[s, e]      = number of (token, slot) assignments from source rank s to logical expert e
// affinity[s, i, j] = number of tokens on source rank s whose top-k contains both i and j (i != j),
//                     symmetric with a zero diagonal.
//
// Semantics follow veomni/distributed/moe/hiermoe/placemoe/statistics.py:30-61
// (profile_route_statistics); the reference builds the pair counts with one
// bincount per (lhs, rhs) top-k column pair, this core does one pass over the
// tokens with the k*(k-1)/2 pairs of each token accumulated directly.
#include <torch/extension.h>

#include <cstdint>
#include <stdexcept>
#include <vector>

#include "planner.h"

namespace pmp {

void accumulate_route_stats(torch::Tensor routes, int64_t source_rank, torch::Tensor demand, torch::Tensor affinity) {
  TORCH_CHECK(routes.dim() == 2, "routes must be [tokens, top_k]");
  TORCH_CHECK(demand.dim() == 2 && demand.scalar_type() == torch::kFloat64, "demand must be float64 [S, E]");
  TORCH_CHECK(affinity.dim() == 3 && affinity.scalar_type() == torch::kFloat64, "affinity must be float64 [S, E, E]");
  auto r = routes.to(torch::kCPU, torch::kInt64).contiguous();
  const int64_t T = r.size(0), K = r.size(1);
  const int64_t E = demand.size(1);
  TORCH_CHECK(source_rank >= 0 && source_rank < demand.size(0), "source rank out of range");
  TORCH_CHECK(demand.is_contiguous() && affinity.is_contiguous(), "outputs must be contiguous");
  const int64_t* rp = r.data_ptr<int64_t>();
  double* dem = demand.data_ptr<double>() + source_rank * E;
  double* aff = affinity.data_ptr<double>() + source_rank * E * E;
  for (int64_t i = 0; i < T * K; ++i) {
    const int64_t e = rp[i];
    if (e < 0 || e >= E) throw std::invalid_argument("Routing sample contains an invalid logical expert ID.");
  }
  for (int64_t t = 0; t < T; ++t) {
    const int64_t* row = rp + t * K;
    for (int64_t a = 0; a < K; ++a) {
      dem[row[a]] += 1.0;
      for (int64_t b = a + 1; b < K; ++b) {
        const int64_t i = row[a], j = row[b];
        if (i == j) continue;
        aff[i * E + j] += 1.0;
        aff[j * E + i] += 1.0;
      }
    }
  }
}

}  // namespace pmp
