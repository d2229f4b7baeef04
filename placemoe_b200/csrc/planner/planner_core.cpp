// CPU cores of the PlaceMoE planner: exact route replay, mapping coordinate
// descent and capacity-constrained partition refinement.
//
// All three are the planner's hot loops (see the reference's
// scripts/profile/build_hiermoe_hierarchical_init_layout.py:515-647,
// veomni/distributed/moe/hiermoe/placemoe/mapping.py:253-332 and
// partition.py:160-212).  On a single NVSwitch domain the topology has one
// level, so the evaluator only counts per-destination-GPU unique rows.
#include <torch/extension.h>

#include <ATen/Parallel.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <limits>
#include <thread>
#include <vector>

#include "planner.h"

namespace pmp {

// ---------------------------------------------------------------------------
// Exact route replay.
//
// routes[i]: [T_i, k] logical experts chosen by tokens of source rank i % S
//            (S = mapping.size(0)); routes[i] belongs to step i / S.
// mapping:   [S, E] physical slot used by source s for expert e.
// slot_rank: [N] rank holding each slot.
// For every token: destination ranks = rank(mapping[s, e_j]); each remote
// destination receives the hidden row once (deduplicated) plus `meta_bytes`
// per assignment.  Returns float64 [n_steps, 5 + 3R], one row per step:
//   [0] max over ranks of max(send_bytes, recv_bytes)
//   [1] max over ranks of assignments
//   [2] total remote unique rows      [3] total remote assignments
//   [4] total assignments             [5 .. 5+R) send bytes per rank
//   [5+R .. 5+2R) recv bytes          [5+2R .. 5+3R) assignments per rank
//
// The (step, source) pairs are independent: they run on a pool of
// at::get_num_threads() threads (the caller's torch thread setting, which
// the planner process pins to its CPU set), each into its own integer
// counters, and are summed in a fixed order afterwards, so the result does not
// depend on the thread count.  Counting is in integers (rows and assignments
// per destination); bytes are formed once per step.
// ---------------------------------------------------------------------------
namespace {

struct SourceCounts {
  std::vector<int64_t> rows, asg;  // per destination rank: remote unique rows / remote assignments received
  std::vector<int64_t> load;       // per destination rank: all assignments (local ones included)
  int64_t total = 0;
  bool bad = false;
};

template <typename Idx>
void replay_source(const Idx* r, int64_t T, int64_t K, const uint8_t* dest, int64_t E, int64_t src, int64_t R,
                   SourceCounts& c) {
  c.rows.assign(R, 0);
  c.asg.assign(R, 0);
  c.load.assign(R, 0);
  int32_t cnt[64];
  for (int64_t t = 0; t < T; ++t) {
    uint64_t mask = 0;
    const Idx* row = r + t * K;
    for (int64_t j = 0; j < K; ++j) {
      const int64_t e = (int64_t)row[j];
      if (e < 0 || e >= E) { c.bad = true; return; }
      const int d = dest[e];
      const uint64_t bit = 1ull << d;
      if (!(mask & bit)) { mask |= bit; cnt[d] = 0; }
      ++cnt[d];
    }
    for (uint64_t m = mask; m; m &= m - 1) {
      const int d = __builtin_ctzll(m);
      c.load[d] += cnt[d];
      if (d == src) continue;
      c.rows[d] += 1;
      c.asg[d] += cnt[d];
    }
  }
  c.total = T * K;
}

}  // namespace

torch::Tensor evaluate_routes_batch(std::vector<torch::Tensor> routes, torch::Tensor mapping, torch::Tensor slot_rank,
                                    double row_bytes, double meta_bytes) {
  auto M = mapping.to(torch::kInt64).contiguous();
  auto Rk = slot_rank.to(torch::kInt64).contiguous();
  TORCH_CHECK(M.dim() == 2, "mapping must be [S, E]");
  const int64_t S = M.size(0), E = M.size(1);
  TORCH_CHECK(S > 0 && (int64_t)routes.size() % S == 0, "routes must hold S tensors per step");
  const int64_t steps = (int64_t)routes.size() / S;
  const int64_t* mp = M.data_ptr<int64_t>();
  const int64_t* rp = Rk.data_ptr<int64_t>();
  const int64_t N = Rk.numel();
  int64_t R = 0;
  for (int64_t i = 0; i < N; ++i) {
    TORCH_CHECK(rp[i] >= 0, "slot rank must be non-negative");
    R = std::max(R, rp[i] + 1);
  }
  TORCH_CHECK(R <= 64, "route replay supports up to 64 ranks");
  TORCH_CHECK(S <= R, "more sources than ranks");
  // destination rank of every (source, expert), validated once
  std::vector<uint8_t> dest(S * E);
  for (int64_t i = 0; i < S * E; ++i) {
    TORCH_CHECK(mp[i] >= 0 && mp[i] < N, "mapping slot out of range");
    dest[i] = (uint8_t)rp[mp[i]];
  }
  std::vector<torch::Tensor> rt(routes.size());
  for (size_t i = 0; i < routes.size(); ++i) {
    auto x = routes[i];
    if (x.scalar_type() != torch::kInt32 && x.scalar_type() != torch::kInt64) x = x.to(torch::kInt64);
    rt[i] = x.contiguous();
    TORCH_CHECK(rt[i].dim() == 2, "routes must be [T, k]");
  }
  std::vector<SourceCounts> part(routes.size());
  run_pool((int64_t)routes.size(), [&](int64_t i) {
    const int64_t s = i % S;
    const auto& x = rt[i];
    if (x.scalar_type() == torch::kInt32)
      replay_source(x.data_ptr<int32_t>(), x.size(0), x.size(1), dest.data() + s * E, E, s, R, part[i]);
    else
      replay_source(x.data_ptr<int64_t>(), x.size(0), x.size(1), dest.data() + s * E, E, s, R, part[i]);
  });
  for (const auto& c : part) TORCH_CHECK(!c.bad, "route expert out of range");
  auto out = torch::zeros({steps, 5 + 3 * R}, torch::kFloat64);
  double* o = out.data_ptr<double>();
  std::vector<int64_t> recv_rows(R), recv_asg(R), load(R);
  for (int64_t st = 0; st < steps; ++st) {
    double* row = o + st * (5 + 3 * R);
    std::fill(recv_rows.begin(), recv_rows.end(), 0);
    std::fill(recv_asg.begin(), recv_asg.end(), 0);
    std::fill(load.begin(), load.end(), 0);
    int64_t rows_remote = 0, asg_remote = 0, asg_total = 0;
    for (int64_t s = 0; s < S; ++s) {
      const auto& c = part[st * S + s];
      int64_t sent_rows = 0, sent_asg = 0;
      for (int64_t d = 0; d < R; ++d) {
        recv_rows[d] += c.rows[d];
        recv_asg[d] += c.asg[d];
        load[d] += c.load[d];
        sent_rows += c.rows[d];
        sent_asg += c.asg[d];
      }
      row[5 + s] = row_bytes * (double)sent_rows + meta_bytes * (double)sent_asg;
      rows_remote += sent_rows;
      asg_remote += sent_asg;
      asg_total += c.total;
    }
    double peak_bytes = 0, peak_asg = 0;
    for (int64_t d = 0; d < R; ++d) {
      const double recv = row_bytes * (double)recv_rows[d] + meta_bytes * (double)recv_asg[d];
      row[5 + R + d] = recv;
      row[5 + 2 * R + d] = (double)load[d];
      peak_bytes = std::max(peak_bytes, std::max(row[5 + d], recv));
      peak_asg = std::max(peak_asg, (double)load[d]);
    }
    row[0] = peak_bytes;
    row[1] = peak_asg;
    row[2] = (double)rows_remote;
    row[3] = (double)asg_remote;
    row[4] = (double)asg_total;
  }
  return out;
}

torch::Tensor evaluate_routes(std::vector<torch::Tensor> routes, torch::Tensor mapping, torch::Tensor slot_rank,
                              double row_bytes, double meta_bytes) {
  TORCH_CHECK(mapping.dim() == 2 && mapping.size(0) == (int64_t)routes.size(), "mapping must be [S, E]");
  return evaluate_routes_batch(std::move(routes), mapping, slot_rank, row_bytes, meta_bytes)[0];
}

// ---------------------------------------------------------------------------
// Mapping coordinate descent.
//
// Objective (time units, lower is better):
//   J(M) = - omega  * sum_s sum_{e<f} A[s,e,f] [rank(M[s,e]) == rank(M[s,f])]
//          - lambda * sum_s sum_e D[s,e] [rank(M[s,e]) == s]
//          + gamma  * max_r load_r,     load_r = sum_{s,e} D[s,e] [rank(M[s,e]) == r]
// The first term is co-selection reuse (a token that picks e and f sends one
// row to a shared destination), the second keeps traffic on the source GPU,
// the third is the expert-compute critical path.  Each sweep revisits every
// (source, expert) with more than one copy and moves it to the copy with the
// best objective delta.  `mapping` is updated in place; returns J.
// ---------------------------------------------------------------------------
double optimize_mapping(torch::Tensor demand, torch::Tensor affinity, torch::Tensor slot_to_logical,
                        torch::Tensor slot_rank, torch::Tensor mapping, double omega, double lambda_local,
                        double gamma, int64_t sweeps) {
  auto D = demand.to(torch::kFloat64).contiguous();
  auto A = affinity.to(torch::kFloat64).contiguous();
  auto L = slot_to_logical.to(torch::kInt64).contiguous();
  auto R = slot_rank.to(torch::kInt64).contiguous();
  TORCH_CHECK(mapping.scalar_type() == torch::kInt64 && mapping.is_contiguous(), "mapping must be contiguous int64");
  const int64_t S = D.size(0), E = D.size(1), N = L.numel();
  const double* d = D.data_ptr<double>();
  const double* a = A.data_ptr<double>();
  const int64_t* l = L.data_ptr<int64_t>();
  const int64_t* rk = R.data_ptr<int64_t>();
  int64_t* m = mapping.data_ptr<int64_t>();
  int64_t P = 0;
  for (int64_t i = 0; i < N; ++i) P = std::max(P, rk[i] + 1);
  std::vector<std::vector<int64_t>> copies(E);
  for (int64_t i = 0; i < N; ++i)
    if (l[i] >= 0) copies[l[i]].push_back(i);
  // aff_rank[s][e][r] = sum_f A[s,e,f] [rank(M[s,f]) == r]
  std::vector<double> aff_rank(S * E * P, 0.0), load(P, 0.0);
  for (int64_t s = 0; s < S; ++s)
    for (int64_t f = 0; f < E; ++f) {
      const int64_t r = rk[m[s * E + f]];
      load[r] += d[s * E + f];
      for (int64_t e = 0; e < E; ++e) aff_rank[(s * E + e) * P + r] += a[(s * E + e) * E + f];
    }
  auto objective = [&]() {
    double reuse = 0, local = 0, peak = 0;
    for (int64_t s = 0; s < S; ++s)
      for (int64_t e = 0; e < E; ++e) {
        const int64_t r = rk[m[s * E + e]];
        reuse += 0.5 * aff_rank[(s * E + e) * P + r];
        if (r == s) local += d[s * E + e];
      }
    for (int64_t r = 0; r < P; ++r) peak = std::max(peak, load[r]);
    return -omega * reuse - lambda_local * local + gamma * peak;
  };
  for (int64_t sw = 0; sw < sweeps; ++sw) {
    int64_t moves = 0;
    for (int64_t s = 0; s < S; ++s) {
      for (int64_t e = 0; e < E; ++e) {
        if (copies[e].size() < 2) continue;
        const int64_t cur = m[s * E + e];
        const int64_t rc = rk[cur];
        const double de = d[s * E + e];
        // peak load with this (s,e) removed
        double best_delta = 0.0;
        int64_t best = cur;
        double base_peak = 0;
        for (int64_t r = 0; r < P; ++r) base_peak = std::max(base_peak, load[r]);
        for (int64_t c : copies[e]) {
          if (c == cur) continue;
          const int64_t rn = rk[c];
          if (rn == rc) continue;
          const double reuse_delta = aff_rank[(s * E + e) * P + rn] - aff_rank[(s * E + e) * P + rc];
          const double local_delta = (rn == s ? de : 0.0) - (rc == s ? de : 0.0);
          double peak = 0;
          for (int64_t r = 0; r < P; ++r) {
            double v = load[r];
            if (r == rc) v -= de;
            if (r == rn) v += de;
            peak = std::max(peak, v);
          }
          const double delta = -omega * reuse_delta - lambda_local * local_delta + gamma * (peak - base_peak);
          if (delta < best_delta - 1e-12) { best_delta = delta; best = c; }
        }
        if (best != cur) {
          const int64_t rn = rk[best];
          m[s * E + e] = best;
          load[rc] -= de;
          load[rn] += de;
          for (int64_t g = 0; g < E; ++g) {
            const double v = a[(s * E + g) * E + e];
            aff_rank[(s * E + g) * P + rc] -= v;
            aff_rank[(s * E + g) * P + rn] += v;
          }
          ++moves;
        }
      }
    }
    if (moves == 0) break;
  }
  return objective();
}

// ---------------------------------------------------------------------------
// Capacity-constrained partition refinement by pairwise exchange.
//
// items: n copies with demand w[i], affinity A[i,j] (symmetric), label[i] in
// [0, G) with fixed group capacities.  Objective:
//   -omega * sum_{i<j same group} A[i,j] + gamma * max_g load_g / ranks_g
// An exchange swaps the groups of two items; exchanges that would put two
// copies of the same logical expert (item_expert) into one group are
// rejected.  Greedy best-improvement steps, at most `limit` of them.
// Returns the number of exchanges made (labels updated in place).
// ---------------------------------------------------------------------------
int64_t refine_partition(torch::Tensor affinity, torch::Tensor weight, torch::Tensor labels, torch::Tensor item_expert,
                         torch::Tensor ranks_per_group, double omega, double gamma, int64_t limit) {
  auto A = affinity.to(torch::kFloat64).contiguous();
  auto W = weight.to(torch::kFloat64).contiguous();
  auto X = item_expert.to(torch::kInt64).contiguous();
  auto RG = ranks_per_group.to(torch::kFloat64).contiguous();
  TORCH_CHECK(labels.scalar_type() == torch::kInt64 && labels.is_contiguous(), "labels must be contiguous int64");
  const int64_t n = W.numel(), G = RG.numel();
  const double* a = A.data_ptr<double>();
  const double* w = W.data_ptr<double>();
  const int64_t* x = X.data_ptr<int64_t>();
  const double* rg = RG.data_ptr<double>();
  int64_t* lab = labels.data_ptr<int64_t>();
  std::vector<double> to_group(n * G, 0.0), load(G, 0.0);
  for (int64_t i = 0; i < n; ++i) {
    load[lab[i]] += w[i];
    for (int64_t j = 0; j < n; ++j) to_group[i * G + lab[j]] += a[i * n + j];
  }
  // expert presence per group (duplicate-copy constraint)
  int64_t max_e = 0;
  for (int64_t i = 0; i < n; ++i) max_e = std::max(max_e, x[i] + 1);
  std::vector<int> present(G * std::max<int64_t>(max_e, 1), 0);
  for (int64_t i = 0; i < n; ++i)
    if (x[i] >= 0) present[lab[i] * max_e + x[i]] += 1;
  int64_t done = 0;
  for (; done < limit; ++done) {
    double cur_peak = 0;
    for (int64_t g = 0; g < G; ++g) cur_peak = std::max(cur_peak, load[g] / rg[g]);
    double best = -1e-12;
    int64_t bi = -1, bj = -1;
    for (int64_t i = 0; i < n; ++i) {
      const int64_t gi = lab[i];
      for (int64_t j = i + 1; j < n; ++j) {
        const int64_t gj = lab[j];
        if (gi == gj) continue;
        if (x[i] >= 0 && x[i] != x[j] && present[gj * max_e + x[i]] > 0) continue;
        if (x[j] >= 0 && x[i] != x[j] && present[gi * max_e + x[j]] > 0) continue;
        const double gain = to_group[i * G + gj] - to_group[i * G + gi] + to_group[j * G + gi] -
                            to_group[j * G + gj] - 2.0 * a[i * n + j];
        double peak = 0;
        for (int64_t g = 0; g < G; ++g) {
          double v = load[g];
          if (g == gi) v += w[j] - w[i];
          if (g == gj) v += w[i] - w[j];
          peak = std::max(peak, v / rg[g]);
        }
        const double delta = -omega * gain + gamma * (peak - cur_peak);
        if (delta < best) { best = delta; bi = i; bj = j; }
      }
    }
    if (bi < 0) break;
    const int64_t gi = lab[bi], gj = lab[bj];
    for (int64_t k = 0; k < n; ++k) {
      to_group[k * G + gi] += a[k * n + bj] - a[k * n + bi];
      to_group[k * G + gj] += a[k * n + bi] - a[k * n + bj];
    }
    load[gi] += w[bj] - w[bi];
    load[gj] += w[bi] - w[bj];
    if (x[bi] >= 0) { present[gi * max_e + x[bi]] -= 1; present[gj * max_e + x[bi]] += 1; }
    if (x[bj] >= 0) { present[gj * max_e + x[bj]] -= 1; present[gi * max_e + x[bj]] += 1; }
    lab[bi] = gj;
    lab[bj] = gi;
  }
  return done;
}

}  // namespace pmp
