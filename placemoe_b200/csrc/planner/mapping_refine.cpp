// Mapping proposals for the PlaceMoE planner beyond the calibrated coordinate descent.
//
// optimize_mapping_normalized
//   Coordinate descent over (source GPU, expert) choices with a scale-free
//   score: co-selection reward on the candidate's node and GPU (normalised by
//   the total co-selection mass, plus the assignment's own demand when the
//   candidate is local) minus a weighted projected peak GPU load (normalised
//   by the total demand).  Sweeping `assignment_weight` spans proposals from
//   communication-only to compute-balanced; the exact route replay picks.
//   The per-source reward tables are kept incrementally: moving expert e from
//   GPU a to GPU b moves column A[s, :, e] from a's row to b's row.
//
// community_intersection_hits / community_mask_histogram / optimize_community_mapping
//   Block mapping: experts are grouped into C communities, and every source
//   unit (a node, or a GPU on a one-level topology) picks one destination
//   unit per community.  A token of unit u whose experts fall in the set of
//   communities `mask` is sent once to every destination unit that serves one
//   of them, so the rows leaving u are  sum over destinations v != u of
//   hits[u][communities sent to v],  with hits[u][X] = tokens of u whose mask
//   meets X.  hits comes from the mask histogram by a subset-sum transform:
//   hits[X] = total - (tokens whose mask lies inside the complement of X).
//   Rows per source unit are enumerated (or built by a bounded beam over
//   communities), a beam over source units combines them under the proxy cost
//   comm_ms_per_token * remote rows + ms_per_assignment * peak unit
//   assignments / ranks_per_unit, and coordinate sweeps over (unit, community)
//   blocks polish the result.
//
// Reference parity: optimize_mapping_normalized, community_intersection_hits
// and optimize_community_mapping of
// veomni/distributed/moe/hiermoe/placemoe/mapping.py:445-810.
#include <torch/extension.h>

#include <algorithm>
#include <cstdint>
#include <numeric>
#include <tuple>
#include <vector>

#include "planner.h"

namespace pmp {

// ---------------------------------------------------------------------------------------- normalized
std::vector<double> optimize_mapping_normalized(torch::Tensor demand, torch::Tensor affinity,
                                                torch::Tensor slot_to_logical, torch::Tensor slot_rank,
                                                torch::Tensor mapping, int64_t ranks_per_node,
                                                double assignment_weight, double node_weight, double rank_weight,
                                                int64_t sweeps) {
  TORCH_CHECK(demand.dtype() == torch::kFloat64 && affinity.dtype() == torch::kFloat64, "fp64 statistics");
  TORCH_CHECK(mapping.dtype() == torch::kInt64 && slot_to_logical.dtype() == torch::kInt64 &&
                  slot_rank.dtype() == torch::kInt64, "int64 tables");
  TORCH_CHECK(ranks_per_node > 0 && sweeps >= 0, "ranks_per_node > 0, sweeps >= 0");
  TORCH_CHECK(assignment_weight >= 0 && node_weight >= 0 && rank_weight >= 0, "non-negative weights");
  const int64_t S = demand.size(0), E = demand.size(1), N = slot_to_logical.size(0);
  TORCH_CHECK(affinity.sizes() == torch::IntArrayRef({S, E, E}) && mapping.sizes() == demand.sizes(), "shapes");
  auto D = demand.accessor<double, 2>();
  auto A = affinity.accessor<double, 3>();
  auto L = slot_to_logical.accessor<int64_t, 1>();
  auto R = slot_rank.accessor<int64_t, 1>();
  auto M = mapping.accessor<int64_t, 2>();
  int64_t W = S;
  for (int64_t i = 0; i < N; ++i) W = std::max(W, R[i] + 1);
  const int64_t nodes = (W + ranks_per_node - 1) / ranks_per_node;
  std::vector<std::vector<int64_t>> copies(E);
  for (int64_t i = 0; i < N; ++i)
    if (L[i] >= 0) copies[L[i]].push_back(i);
  std::vector<double> load(W, 0.0);
  double tot_a = 0.0, tot_d = 0.0;
  for (int64_t s = 0; s < S; ++s)
    for (int64_t e = 0; e < E; ++e) {
      load[R[M[s][e]]] += D[s][e];
      tot_d += D[s][e];
      for (int64_t f = 0; f < E; ++f) tot_a += A[s][e][f];
    }
  tot_a = std::max(tot_a, 1.0);
  tot_d = std::max(tot_d, 1.0);
  std::vector<double> rank_aff(W * E), node_aff(nodes * E);
  int64_t done = 0, changes = 0;
  for (int64_t sweep = 0; sweep < sweeps; ++sweep) {
    int64_t moved = 0;
    for (int64_t s = 0; s < S; ++s) {
      std::fill(rank_aff.begin(), rank_aff.end(), 0.0);
      std::fill(node_aff.begin(), node_aff.end(), 0.0);
      for (int64_t f = 0; f < E; ++f) {
        const int64_t rf = R[M[s][f]];
        for (int64_t e = 0; e < E; ++e) {
          rank_aff[rf * E + e] += A[s][e][f];
          node_aff[(rf / ranks_per_node) * E + e] += A[s][e][f];
        }
      }
      std::vector<int64_t> order(E);
      std::iota(order.begin(), order.end(), 0);
      std::stable_sort(order.begin(), order.end(), [&](int64_t a, int64_t b) { return D[s][a] > D[s][b]; });
      for (int64_t e : order) {
        if (copies[e].size() <= 1) continue;
        const int64_t cur = M[s][e], rc = R[cur];
        const double amt = D[s][e];
        int64_t pick = cur;
        double best = 0.0;
        int64_t best_rank = 0;
        bool have = false;
        for (int64_t c : copies[e]) {
          const int64_t rho = R[c], node = rho / ranks_per_node;
          double peak = 0.0;
          for (int64_t r = 0; r < W; ++r) {
            double v = load[r];
            if (r == rc) v -= amt;
            if (r == rho) v += amt;
            peak = std::max(peak, v);
          }
          const double node_reward = node_aff[node * E + e] + (node == s / ranks_per_node ? amt : 0.0);
          const double rank_reward = rank_aff[rho * E + e] + (rho == s ? amt : 0.0);
          const double score = node_weight * node_reward / tot_a + rank_weight * rank_reward / tot_a -
                               assignment_weight * peak / tot_d;
          // higher score wins; ties go to the lower GPU, then the lower slot
          if (!have || score > best || (score == best && (rho < best_rank || (rho == best_rank && c < pick)))) {
            have = true;
            best = score;
            best_rank = rho;
            pick = c;
          }
        }
        if (pick == cur) continue;
        const int64_t rp = R[pick];
        load[rc] -= amt;
        load[rp] += amt;
        M[s][e] = pick;
        for (int64_t f = 0; f < E; ++f) {
          rank_aff[rc * E + f] -= A[s][f][e];
          rank_aff[rp * E + f] += A[s][f][e];
          node_aff[(rc / ranks_per_node) * E + f] -= A[s][f][e];
          node_aff[(rp / ranks_per_node) * E + f] += A[s][f][e];
        }
        ++moved;
      }
    }
    ++done;
    changes += moved;
    if (moved == 0) break;
  }
  return {*std::max_element(load.begin(), load.end()), (double)done, (double)changes};
}

// ---------------------------------------------------------------------------------------- community
torch::Tensor community_intersection_hits(torch::Tensor hist) {
  TORCH_CHECK(hist.dim() == 2 && hist.dtype() == torch::kInt64, "histogram: int64 [unit, 2^C]");
  const int64_t U = hist.size(0), K = hist.size(1);
  TORCH_CHECK(K > 0 && (K & (K - 1)) == 0, "histogram width must be a power of two");
  int C = 0;
  while ((int64_t(1) << C) < K) ++C;
  auto h = hist.contiguous();
  auto out = torch::zeros_like(h);
  const int64_t* hp = h.data_ptr<int64_t>();
  int64_t* op = out.data_ptr<int64_t>();
  std::vector<int64_t> inside(K);
  for (int64_t u = 0; u < U; ++u) {
    std::copy(hp + u * K, hp + (u + 1) * K, inside.begin());
    for (int b = 0; b < C; ++b)  // inside[m] = tokens whose mask is a subset of m
      for (int64_t m = 0; m < K; ++m)
        if (m & (int64_t(1) << b)) inside[m] += inside[m ^ (int64_t(1) << b)];
    const int64_t total = inside[K - 1];
    for (int64_t x = 0; x < K; ++x) op[u * K + x] = total - inside[(K - 1) & ~x];
  }
  return out;
}

namespace {
template <typename Idx>
bool mask_histogram_source(const Idx* rp, int64_t T, int64_t k, const int64_t* comm, int64_t E, int64_t* row) {
  for (int64_t t = 0; t < T; ++t) {
    int64_t mask = 0;
    for (int64_t j = 0; j < k; ++j) {
      const int64_t e = (int64_t)rp[t * k + j];
      if (e < 0 || e >= E) return false;
      if (comm[e] >= 0) mask |= int64_t(1) << comm[e];
    }
    row[mask] += 1;
  }
  return true;
}
}  // namespace

torch::Tensor community_mask_histogram(std::vector<torch::Tensor> routes, torch::Tensor community,
                                       int64_t ranks_per_unit, int64_t num_communities, int64_t sources_per_step) {
  TORCH_CHECK(num_communities > 0 && num_communities <= 20, "1..20 communities");
  const int64_t n = (int64_t)routes.size();
  const int64_t S = sources_per_step > 0 ? sources_per_step : n;
  TORCH_CHECK(n % S == 0 && S % ranks_per_unit == 0 && ranks_per_unit > 0,
              "routes hold whole steps of sources, split into units");
  auto cm = community.to(torch::kInt64).contiguous();
  const int64_t* comm = cm.data_ptr<int64_t>();
  const int64_t E = cm.numel();
  const int64_t U = S / ranks_per_unit, K = int64_t(1) << num_communities;
  auto out = torch::zeros({U, K}, torch::kInt64);
  int64_t* op = out.data_ptr<int64_t>();
  std::vector<torch::Tensor> rt(routes.size());
  for (size_t s = 0; s < routes.size(); ++s) {
    auto r = routes[s];
    if (r.scalar_type() != torch::kInt32 && r.scalar_type() != torch::kInt64) r = r.to(torch::kInt64);
    rt[s] = r.contiguous();
    TORCH_CHECK(rt[s].dim() == 2, "routes: [tokens, k]");
  }
  // units own disjoint rows of the histogram: one unit per pool item, its sources of every step in order
  std::vector<char> bad(U, 0);
  run_pool(U, [&](int64_t u) {
    std::vector<int64_t> row(K, 0);  // thread-local: short rows of neighbouring units share cache lines
    for (int64_t i = 0; i < n; ++i) {
      if ((i % S) / ranks_per_unit != u) continue;
      const auto& r = rt[i];
      const int64_t T = r.size(0), k = r.size(1);
      const bool ok = r.scalar_type() == torch::kInt32
                          ? mask_histogram_source(r.data_ptr<int32_t>(), T, k, comm, E, row.data())
                          : mask_histogram_source(r.data_ptr<int64_t>(), T, k, comm, E, row.data());
      if (!ok) bad[u] = 1;
    }
    std::copy(row.begin(), row.end(), op + u * K);
  });
  for (int64_t u = 0; u < U; ++u) TORCH_CHECK(!bad[u], "expert id out of range");
  return out;
}

namespace {

struct Row {
  double cost;
  std::vector<int64_t> dest;  // destination unit per community
  double remote;
  std::vector<double> asg;  // assignments per destination unit
};

bool row_less(const Row& a, const Row& b) {
  if (a.cost != b.cost) return a.cost < b.cost;
  return a.dest < b.dest;
}

double remote_rows(const int64_t* hits_u, const std::vector<int64_t>& dest, int64_t src_unit, int64_t U) {
  std::vector<int64_t> sub(U, 0);
  for (size_t c = 0; c < dest.size(); ++c) sub[dest[c]] |= int64_t(1) << c;
  double r = 0.0;
  for (int64_t v = 0; v < U; ++v)
    if (v != src_unit && sub[v]) r += (double)hits_u[sub[v]];
  return r;
}

}  // namespace

// Returns (destination [U, C] int64, proxy cost, sweeps, changes).
std::tuple<torch::Tensor, double, int64_t, int64_t> optimize_community_mapping(
    torch::Tensor allowed, torch::Tensor assignments, torch::Tensor hits, double comm_ms_per_token,
    double ms_per_assignment, int64_t ranks_per_unit, int64_t row_limit, int64_t beam_width, int64_t sweeps) {
  // allowed [C, U] bool-as-int64: unit v serves every expert of community c
  TORCH_CHECK(allowed.dim() == 2 && assignments.dim() == 2 && hits.dim() == 2, "2-D inputs");
  const int64_t C = allowed.size(0), U = allowed.size(1);
  TORCH_CHECK(C > 0 && C <= 20 && assignments.size(0) == U && assignments.size(1) == C, "assignments [U, C]");
  TORCH_CHECK(hits.size(0) == U && hits.size(1) == (int64_t(1) << C), "hits [U, 2^C]");
  TORCH_CHECK(row_limit > 0 && beam_width > 0 && ranks_per_unit > 0, "positive limits");
  auto al = allowed.to(torch::kInt64).contiguous();
  auto as = assignments.to(torch::kFloat64).contiguous();
  auto hi = hits.to(torch::kInt64).contiguous();
  const int64_t* alp = al.data_ptr<int64_t>();
  const double* asp = as.data_ptr<double>();
  const int64_t* hp = hi.data_ptr<int64_t>();
  const int64_t K = int64_t(1) << C;
  std::vector<std::vector<int64_t>> units(C);
  for (int64_t c = 0; c < C; ++c) {
    for (int64_t v = 0; v < U; ++v)
      if (alp[c * U + v]) units[c].push_back(v);
    TORCH_CHECK(!units[c].empty(), "a community has no unit serving all of its experts");
  }
  auto proxy = [&](double remote, const std::vector<double>& asg) {
    return comm_ms_per_token * remote +
           ms_per_assignment * (*std::max_element(asg.begin(), asg.end())) / (double)ranks_per_unit;
  };
  // ---- candidate destination rows of every source unit
  std::vector<std::vector<Row>> rows_of(U);
  for (int64_t u = 0; u < U; ++u) {
    const int64_t* hu = hp + u * K;
    double product = 1.0;
    for (int64_t c = 0; c < C; ++c) product *= (double)units[c].size();
    std::vector<Row> rows;
    if (product <= (double)(row_limit * beam_width)) {
      std::vector<size_t> idx(C, 0);
      while (true) {
        Row r;
        r.dest.resize(C);
        r.asg.assign(U, 0.0);
        for (int64_t c = 0; c < C; ++c) {
          r.dest[c] = units[c][idx[c]];
          r.asg[r.dest[c]] += asp[u * C + c];
        }
        r.remote = remote_rows(hu, r.dest, u, U);
        r.cost = proxy(r.remote, r.asg);
        rows.push_back(std::move(r));
        int64_t c = C - 1;
        while (c >= 0 && ++idx[c] == units[c].size()) idx[c--] = 0;
        if (c < 0) break;
      }
    } else {  // bounded beam over the communities, in order
      std::vector<Row> partial(1);
      partial[0].asg.assign(U, 0.0);
      for (int64_t c = 0; c < C; ++c) {
        std::vector<Row> grown;
        for (const Row& p : partial)
          for (int64_t v : units[c]) {
            Row r = p;
            r.dest.push_back(v);
            r.asg[v] += asp[u * C + c];
            r.remote = remote_rows(hu, r.dest, u, U);  // communities beyond c are not placed yet
            r.cost = proxy(r.remote, r.asg);
            grown.push_back(std::move(r));
          }
        std::sort(grown.begin(), grown.end(), row_less);
        if ((int64_t)grown.size() > row_limit) grown.resize(row_limit);
        partial = std::move(grown);
      }
      rows = std::move(partial);
    }
    std::sort(rows.begin(), rows.end(), row_less);
    if ((int64_t)rows.size() > row_limit) rows.resize(row_limit);
    rows_of[u] = std::move(rows);
  }
  // ---- beam over source units
  struct State {
    double cost, remote;
    std::vector<double> asg;
    std::vector<int64_t> pick;  // row index per source unit
    std::vector<int64_t> key;   // concatenated destination rows (tie-break)
  };
  std::vector<State> beam(1);
  beam[0] = {0.0, 0.0, std::vector<double>(U, 0.0), {}, {}};
  for (int64_t u = 0; u < U; ++u) {
    std::vector<State> grown;
    for (const State& st : beam)
      for (size_t i = 0; i < rows_of[u].size(); ++i) {
        const Row& r = rows_of[u][i];
        State n = st;
        n.remote += r.remote;
        for (int64_t v = 0; v < U; ++v) n.asg[v] += r.asg[v];
        n.cost = proxy(n.remote, n.asg);
        n.pick.push_back((int64_t)i);
        n.key.insert(n.key.end(), r.dest.begin(), r.dest.end());
        grown.push_back(std::move(n));
      }
    std::sort(grown.begin(), grown.end(), [](const State& a, const State& b) {
      if (a.cost != b.cost) return a.cost < b.cost;
      return a.key < b.key;
    });
    if ((int64_t)grown.size() > beam_width) grown.resize(beam_width);
    beam = std::move(grown);
  }
  std::vector<std::vector<int64_t>> dest(U);
  std::vector<double> remote(U), asg = beam[0].asg;
  for (int64_t u = 0; u < U; ++u) {
    dest[u] = rows_of[u][beam[0].pick[u]].dest;
    remote[u] = remote_rows(hp + u * K, dest[u], u, U);
  }
  // ---- coordinate sweeps over (source unit, community) blocks, largest first
  std::vector<std::tuple<double, int64_t, int64_t>> order;
  for (int64_t u = 0; u < U; ++u)
    for (int64_t c = 0; c < C; ++c) order.emplace_back(-asp[u * C + c], u, c);
  std::sort(order.begin(), order.end());
  auto total_cost = [&]() { return proxy(std::accumulate(remote.begin(), remote.end(), 0.0), asg); };
  int64_t done = 0, changes = 0;
  for (int64_t sweep = 0; sweep < sweeps; ++sweep) {
    int64_t moved = 0;
    for (const auto& [neg, u, c] : order) {
      const double amount = -neg;
      const int64_t cur = dest[u][c];
      const double now = total_cost();
      double best = now;
      int64_t best_v = cur;
      for (int64_t v : units[c]) {
        if (v == cur) continue;
        std::vector<int64_t> trial = dest[u];
        trial[c] = v;
        const double r_u = remote_rows(hp + u * K, trial, u, U);
        std::vector<double> a2 = asg;
        a2[cur] -= amount;
        a2[v] += amount;
        const double saved = remote[u];
        remote[u] = r_u;
        const double cost = proxy(std::accumulate(remote.begin(), remote.end(), 0.0), a2);
        remote[u] = saved;
        if (cost < best || (cost == best && v < best_v && best_v != cur)) {
          best = cost;
          best_v = v;
        }
      }
      if (best_v == cur || best >= now - 1e-12) continue;
      dest[u][c] = best_v;
      asg[cur] -= amount;
      asg[best_v] += amount;
      remote[u] = remote_rows(hp + u * K, dest[u], u, U);
      ++moved;
    }
    ++done;
    changes += moved;
    if (moved == 0) break;
  }
  auto out = torch::empty({U, C}, torch::kInt64);
  for (int64_t u = 0; u < U; ++u)
    for (int64_t c = 0; c < C; ++c) out[u][c] = dest[u][c];
  return {out, total_cost(), done, changes};
}

}  // namespace pmp
