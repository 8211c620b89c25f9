// Shared-budget tier allocation: the exact-row multiple-choice knapsack that
// picks one tree tier per request for the next packed wave (host code).
//
// Specification (continuous_tree_block_decode.py:706-795, with the cost model
// of :619-641): request i choosing option k takes options[k] + 1 target rows
// (tier nodes plus the root row) and earns weights[i] * utilities[i][k].
// Requests are taken in order; for every exact row total the best allocation
// so far is kept (a larger reward wins unless the two are within 1e-12, then
// the lexicographically smaller allocation), and the final allocation
// maximises reward / wave_cost(rows), ties going to fewer rows.  Rows that
// first become reachable are visited in the order they first appear, which
// decides near-ties exactly as the reference does.  Arithmetic is IEEE fp64 in
// the reference's evaluation order (reward + weight * utility; cost =
// left + fraction * (right - left)), so allocations are bit-identical.
//
// The table holds, per request step and row total, the reward and a back
// pointer (previous row total, option); allocations are rebuilt from back
// pointers only to break exact ties.
#include <cmath>
#include <vector>

#include "common.cuh"

namespace sg {
namespace {

struct Cell {
  double reward;
  int prev;    // row total before this request; -2 = unreachable
  int option;  // option index chosen for this request
};

struct Problem {
  int R, T, budget;
  const double* weights;
  const int32_t* options;
  const double* utilities;  // [R, T]
  double fixed;             // > 0, or NaN when a curve is given
  const int32_t* curve_rows;
  const double* curve_cost;
  int curve_points;
};

double wave_cost(const Problem& p, int rows) {
  if (p.curve_points == 0) return p.fixed + static_cast<double>(rows);
  if (rows <= p.curve_rows[0]) return p.curve_cost[0];
  for (int s = 0; s + 1 < p.curve_points; ++s) {
    const int lr = p.curve_rows[s], rr = p.curve_rows[s + 1];
    if (rows <= rr) {
      const double fraction = static_cast<double>(rows - lr) / static_cast<double>(rr - lr);
      const double span = p.curve_cost[s + 1] - p.curve_cost[s];
      const double step = fraction * span;
      return p.curve_cost[s] + step;
    }
  }
  return p.curve_cost[p.curve_points - 1];
}

// Options (by index) of the allocation ending at row total `rows` after
// `steps` requests, in request order.
void rebuild(const std::vector<std::vector<Cell>>& table, int steps, int rows, std::vector<int>& out) {
  out.assign(steps, 0);
  for (int i = steps; i > 0; --i) {
    const Cell& c = table[i][rows];
    out[i - 1] = c.option;
    rows = c.prev;
  }
}

int validate(const Problem& p) {
  if (p.R < 1 || p.T < 1 || p.weights == nullptr || p.options == nullptr || p.utilities == nullptr)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers: empty problem");
  if (p.options[0] < 1) return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers: tier options must be >= 1");
  for (int k = 1; k < p.T; ++k)
    if (p.options[k] <= p.options[k - 1])
      return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers: tier options must be strictly increasing");
  if (static_cast<int64_t>(p.budget) < static_cast<int64_t>(p.R) * (p.options[0] + 1))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers: row budget below one smallest tier per request");
  const bool has_curve = p.curve_points > 0;
  if (has_curve == std::isfinite(p.fixed))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers: give either a fixed row equivalent or a cost curve");
  if (!has_curve && !(p.fixed > 0.0))
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers: fixed row equivalent must be positive");
  if (has_curve) {
    if (p.curve_rows == nullptr || p.curve_cost == nullptr)
      return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers: null cost curve");
    for (int s = 0; s < p.curve_points; ++s) {
      if (p.curve_rows[s] < 1 || !std::isfinite(p.curve_cost[s]) || !(p.curve_cost[s] > 0.0))
        return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers: cost curve points need rows >= 1, cost > 0");
      if (s > 0 && (p.curve_rows[s] <= p.curve_rows[s - 1] || p.curve_cost[s] < p.curve_cost[s - 1]))
        return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers: cost curve must be increasing in rows, "
                                             "non-decreasing in cost");
    }
  }
  for (int i = 0; i < p.R; ++i) {
    if (!std::isfinite(p.weights[i]) || p.weights[i] < 0.0)
      return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers: weights must be finite and >= 0");
    for (int k = 0; k < p.T; ++k) {
      const double u = p.utilities[static_cast<size_t>(i) * p.T + k];
      if (!std::isfinite(u) || u < 1.0)
        return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers: utilities must be finite and >= 1");
    }
  }
  return SG_OK;
}

}  // namespace
}  // namespace sg

extern "C" int sg_allocate_tiers(int32_t num_requests, const double* weights, int32_t num_options,
                                 const int32_t* options, const double* utilities, int32_t row_budget,
                                 double fixed_row_equivalent, const int32_t* curve_rows, const double* curve_cost,
                                 int32_t curve_points, int32_t* allocation) {
  using namespace sg;
  if (allocation == nullptr || curve_points < 0) return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers: bad output");
  Problem p{num_requests, num_options, row_budget, weights, options, utilities, fixed_row_equivalent, curve_rows,
            curve_cost, curve_points};
  int st = validate(p);
  if (st != SG_OK) return st;
  const int B = p.budget;
  std::vector<std::vector<Cell>> table(p.R + 1, std::vector<Cell>(B + 1, Cell{0.0, -2, -1}));
  table[0][0] = Cell{0.0, -1, -1};
  std::vector<int> reached{0}, next;
  std::vector<int> a, b;
  for (int i = 0; i < p.R; ++i) {
    next.clear();
    std::vector<Cell>& row = table[i + 1];
    for (int used : reached) {
      const double base = table[i][used].reward;
      for (int k = 0; k < p.T; ++k) {
        const int rows = used + p.options[k] + 1;
        if (rows > B) continue;
        const double earned = p.weights[i] * p.utilities[static_cast<size_t>(i) * p.T + k];
        const double reward = base + earned;
        Cell& cur = row[rows];
        if (cur.prev == -2) {
          cur = Cell{reward, used, k};
          next.push_back(rows);
          continue;
        }
        bool take = reward > cur.reward + 1e-12;
        if (!take && std::fabs(reward - cur.reward) <= 1e-12) {
          // lexicographic order of the two allocations (options increase
          // with their index, so indices compare like tier sizes)
          rebuild(table, i, used, a);
          a.push_back(k);
          rebuild(table, i, cur.prev, b);
          b.push_back(cur.option);
          take = a < b;
        }
        if (take) cur = Cell{reward, used, k};
      }
    }
    reached.swap(next);
    if (reached.empty()) return fail(SG_ERR_CAPACITY, "sg_allocate_tiers: no feasible wave under the row budget");
  }
  int best = -1;
  double best_ratio = 0.0;
  for (int rows : reached) {
    const double ratio = table[p.R][rows].reward / wave_cost(p, rows);
    if (best < 0 || ratio > best_ratio || (ratio == best_ratio && rows < best)) {
      best = rows;
      best_ratio = ratio;
    }
  }
  rebuild(table, p.R, best, a);
  for (int i = 0; i < p.R; ++i) allocation[i] = p.options[a[i]];
  return SG_OK;
}
