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
#include <climits>
#include <cmath>
#include <cstdio>
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

// Checks of the problem's shape and cost model (host data in both entries).
int validate_shape(const Problem& p, const char* who) {
  char msg[160];
  auto bad = [&](const char* what) {
    std::snprintf(msg, sizeof(msg), "%s: %s", who, what);
    return fail(SG_ERR_INVALID_ARGUMENT, msg);
  };
  if (p.R < 1 || p.T < 1 || p.weights == nullptr || p.options == nullptr || p.utilities == nullptr)
    return bad("empty problem");
  if (p.options[0] < 1) return bad("tier options must be >= 1");
  for (int k = 1; k < p.T; ++k)
    if (p.options[k] <= p.options[k - 1]) return bad("tier options must be strictly increasing");
  if (static_cast<int64_t>(p.budget) < static_cast<int64_t>(p.R) * (p.options[0] + 1))
    return bad("row budget below one smallest tier per request");
  const bool has_curve = p.curve_points > 0;
  if (has_curve == std::isfinite(p.fixed)) return bad("give either a fixed row equivalent or a cost curve");
  if (!has_curve && !(p.fixed > 0.0)) return bad("fixed row equivalent must be positive");
  if (has_curve) {
    if (p.curve_rows == nullptr || p.curve_cost == nullptr) return bad("null cost curve");
    for (int s = 0; s < p.curve_points; ++s) {
      if (p.curve_rows[s] < 1 || !std::isfinite(p.curve_cost[s]) || !(p.curve_cost[s] > 0.0))
        return bad("cost curve points need rows >= 1, cost > 0");
      if (s > 0 && (p.curve_rows[s] <= p.curve_rows[s - 1] || p.curve_cost[s] < p.curve_cost[s - 1]))
        return bad("cost curve must be increasing in rows, non-decreasing in cost");
    }
  }
  return SG_OK;
}

int validate(const Problem& p) {
  int st = validate_shape(p, "sg_allocate_tiers");
  if (st != SG_OK) return st;
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

// ---------------------------------------------------------------------------
// The same knapsack as one CTA on the device, for weights and utilities that
// the tree kernels left in device memory (no host round trip per wave).
//
// Per request step every reachable row total is one thread's cell.  The host
// loop visits (previous row total in first-reached order, option) pairs in
// order and updates a cell with each pair that lands on it; a cell's
// candidates are therefore processed in the order of their key
// rank(previous) * T + option, and the next step's first-reached order is
// the order of each cell's smallest key.  Ranks are rebuilt every step from a
// bitmap of those keys, so the device visits candidates in exactly the host's
// order and applies the same fp64 comparisons: allocations are identical.
// The lexicographic tie rule compares two allocations that end in the same
// cell; every reached cell also keeps the lexicographic rank of its
// allocation among the step's allocations (rank of the key lex(previous) * T
// + option, rebuilt by the same bitmap count), so a tie is two comparisons of
// ranks and options instead of a walk along the back pointers.
// ---------------------------------------------------------------------------
namespace sg {
namespace {

constexpr int kAllocThreads = 512;
constexpr int kAllocMaxOptions = 8;
constexpr int kAllocMaxBudget = 4096;
constexpr int kAllocMaxCurve = 64;

struct DeviceProblem {
  int R, T, B;
  int options[kAllocMaxOptions];
  double fixed;
  int curve_points;
  int curve_rows[kAllocMaxCurve];
  double curve_cost[kAllocMaxCurve];
  const double* weights;    // device [R]
  const double* utilities;  // device [R, T]
  int32_t* allocation;      // device [R]
  int32_t* status;          // device word (atomicMax of error codes), or null
  int32_t* links;           // device [(R + 1) * (B + 1)]: previous row total * 8 + option, -1 unreached
};

__device__ double device_wave_cost(const DeviceProblem& p, int rows) {
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

__device__ __forceinline__ void alloc_report(const DeviceProblem& p, int code) {
  if (p.status != nullptr) atomicMax(p.status, code);
}

// Warp 0 turns the key bitmap into per-word exclusive prefix counts
// (word_base) and returns the total through *total (read after a barrier).
__device__ void scan_bits(const uint32_t* bits, int key_words, int* word_base, int* total) {
  const int lane = threadIdx.x & 31;
  const int per = (key_words + 31) / 32;
  const int begin = min(key_words, lane * per), end = min(key_words, begin + per);
  int local = 0;
  for (int j = begin; j < end; ++j) local += __popc(bits[j]);
  int incl = local;
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  int run = incl - local;
  for (int j = begin; j < end; ++j) {
    word_base[j] = run;
    run += __popc(bits[j]);
  }
  if (lane == 31) *total = incl;
}

template <int TT>
__global__ void __launch_bounds__(kAllocThreads) allocate_tiers_kernel(const DeviceProblem p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int cells = p.B + 1;
  constexpr int T = TT;  // options (a template parameter: exact unrolling)
  double* reward = reinterpret_cast<double*>(smem);                // [2][cells]
  int* rank = reinterpret_cast<int*>(reward + 2 * cells);          // [2][cells] first-reached rank
  int* lex = rank + 2 * cells;                                     // [2][cells] lexicographic rank
  const int key_words = (cells * T + 31) / 32;
  uint32_t* bits = reinterpret_cast<uint32_t*>(lex + 2 * cells);   // [2][key_words] first-reached keys
  uint32_t* lbits = bits + 2 * key_words;                          // [2][key_words] lexicographic keys
  int* word_base = reinterpret_cast<int*>(lbits + 2 * key_words);  // [key_words]
  int* lword_base = word_base + key_words;                         // [key_words]
  __shared__ double earned_s[2][kAllocMaxOptions];
  __shared__ int bad;
  __shared__ int reached;
  __shared__ int lreached;
  __shared__ double best_ratio[32];
  __shared__ int best_rows[32];
  const int tid = threadIdx.x;

  if (tid == 0) bad = 0;
  __syncthreads();
  for (int j = tid; j < p.R * T; j += kAllocThreads) {
    const double u = p.utilities[j];
    if (!isfinite(u) || u < 1.0) bad = 1;
  }
  for (int i = tid; i < p.R; i += kAllocThreads) {
    const double w = p.weights[i];
    if (!isfinite(w) || w < 0.0) bad = 1;
  }
  for (int c = tid; c < cells; c += kAllocThreads) {
    rank[c] = c == 0 ? 0 : -1;
    lex[c] = 0;
    reward[c] = 0.0;
    p.links[c] = c == 0 ? -1 : -2;
  }
  for (int j = tid; j < 4 * key_words; j += kAllocThreads) bits[j] = 0u;
  if (tid < T) earned_s[0][tid] = p.weights[0] * p.utilities[tid];
  __syncthreads();
  if (bad) {
    alloc_report(p, SG_ERR_INVALID_ARGUMENT);
    for (int i = tid; i < p.R; i += kAllocThreads) p.allocation[i] = -1;
    return;
  }
  int cur = 0;
  for (int i = 0; i < p.R; ++i) {
    const int* rank_prev = rank + cur * cells;
    int* rank_next = rank + (cur ^ 1) * cells;
    const int* lex_prev = lex + cur * cells;
    int* lex_next = lex + (cur ^ 1) * cells;
    uint32_t* lbits_now = lbits + (i & 1) * key_words;
    uint32_t* lbits_other = lbits + ((i & 1) ^ 1) * key_words;
    const double* reward_prev = reward + cur * cells;
    double* reward_next = reward + (cur ^ 1) * cells;
    uint32_t* bits_now = bits + (i & 1) * key_words;
    uint32_t* bits_other = bits + ((i & 1) ^ 1) * key_words;
    int32_t* links_next = p.links + static_cast<size_t>(i + 1) * cells;
    // the next step's earned rewards load while this step runs
    if (tid < T && i + 1 < p.R)
      earned_s[(i + 1) & 1][tid] = p.weights[i + 1] * p.utilities[static_cast<size_t>(i + 1) * T + tid];
    double earned[T];
    int opts[T];
#pragma unroll
    for (int k = 0; k < T; ++k) {
      earned[k] = earned_s[i & 1][k];
      opts[k] = p.options[k];
    }
    // the other bitmap was read by the previous step's rank conversion,
    // which ended with a barrier: clear it for the next step
    for (int j = tid; j < key_words; j += kAllocThreads) {
      bits_other[j] = 0u;
      lbits_other[j] = 0u;
    }
    for (int c = tid; c < cells; c += kAllocThreads) {
      // candidate k: previous row total c - options[k] - 1, key rank * T + k
      int key[T];
#pragma unroll
      for (int k = 0; k < T; ++k) {
        const int u = c - opts[k] - 1;
        key[k] = (u >= 0 && rank_prev[u] >= 0) ? rank_prev[u] * T + k : INT_MAX;
      }
      // visit candidates in increasing key order (the host's order)
      double best = 0.0;
      int best_used = -1, best_opt = -1, first_key = INT_MAX;
      unsigned done = 0u;
#pragma unroll
      for (int step = 0; step < T; ++step) {
        int kmin = -1, vmin = INT_MAX;
#pragma unroll
        for (int k = 0; k < T; ++k)
          if (!((done >> k) & 1u) && key[k] < vmin) {
            vmin = key[k];
            kmin = k;
          }
        if (kmin < 0) break;
        done |= 1u << kmin;
        int u = 0;
        double e = 0.0;
#pragma unroll
        for (int k = 0; k < T; ++k)
          if (k == kmin) {
            u = c - opts[k] - 1;
            e = earned[k];
          }
        const double r = reward_prev[u] + e;
        if (best_used < 0) {
          best = r;
          best_used = u;
          best_opt = kmin;
          first_key = vmin;
          continue;
        }
        bool take = r > best + 1e-12;
        if (!take && fabs(r - best) <= 1e-12) {
          // lexicographic order of (allocation of u, kmin) and (allocation
          // of best_used, best_opt): the prefixes' ranks, then the options
          const int la = lex_prev[u], lb = lex_prev[best_used];
          take = la < lb || (la == lb && kmin < best_opt);
        }
        if (take) {
          best = r;
          best_used = u;
          best_opt = kmin;
        }
      }
      if (best_used < 0) {
        rank_next[c] = -1;
        links_next[c] = -2;
        continue;
      }
      reward_next[c] = best;
      links_next[c] = best_used * 8 + best_opt;
      rank_next[c] = first_key;  // first-reached key; turned into a rank below
      atomicOr(&bits_now[first_key >> 5], 1u << (first_key & 31));
      const int lkey = lex_prev[best_used] * T + best_opt;  // unique per cell
      lex_next[c] = lkey;
      atomicOr(&lbits_now[lkey >> 5], 1u << (lkey & 31));
    }
    __syncthreads();
    if (tid < 32) scan_bits(bits_now, key_words, word_base, &reached);
    else if (tid < 64) scan_bits(lbits_now, key_words, lword_base, &lreached);
    __syncthreads();
    if (reached == 0) {
      alloc_report(p, SG_ERR_CAPACITY);
      for (int r = tid; r < p.R; r += kAllocThreads) p.allocation[r] = -1;
      return;
    }
    for (int c = tid; c < cells; c += kAllocThreads) {
      const int key = rank_next[c];
      if (key >= 0) {
        rank_next[c] = word_base[key >> 5] + __popc(bits_now[key >> 5] & ((1u << (key & 31)) - 1u));
        const int lkey = lex_next[c];
        lex_next[c] = lword_base[lkey >> 5] + __popc(lbits_now[lkey >> 5] & ((1u << (lkey & 31)) - 1u));
      }
    }
    __syncthreads();
    cur ^= 1;
  }
  // largest reward / cost, ties to fewer rows
  const int* rank_last = rank + cur * cells;
  const double* reward_last = reward + cur * cells;
  double my_ratio = 0.0;
  int my_rows = -1;
  for (int c = tid; c < cells; c += kAllocThreads) {
    if (rank_last[c] < 0) continue;
    const double ratio = reward_last[c] / device_wave_cost(p, c);
    if (my_rows < 0 || ratio > my_ratio || (ratio == my_ratio && c < my_rows)) {
      my_ratio = ratio;
      my_rows = c;
    }
  }
  const int lane = tid & 31, warp = tid >> 5;
  for (int o = 16; o > 0; o >>= 1) {
    const double r = __shfl_down_sync(0xffffffffu, my_ratio, o);
    const int c = __shfl_down_sync(0xffffffffu, my_rows, o);
    if (c >= 0 && (my_rows < 0 || r > my_ratio || (r == my_ratio && c < my_rows))) {
      my_ratio = r;
      my_rows = c;
    }
  }
  if (lane == 0) {
    best_ratio[warp] = my_ratio;
    best_rows[warp] = my_rows;
  }
  __syncthreads();
  if (tid == 0) {
    double r = best_ratio[0];
    int rows = best_rows[0];
    for (int w = 1; w < kAllocThreads / 32; ++w) {
      const int c = best_rows[w];
      if (c >= 0 && (rows < 0 || best_ratio[w] > r || (best_ratio[w] == r && c < rows))) {
        r = best_ratio[w];
        rows = c;
      }
    }
    for (int s = p.R; s > 0; --s) {
      const int link = p.links[static_cast<size_t>(s) * cells + rows];
      p.allocation[s - 1] = p.options[link & 7];
      rows = link >> 3;
    }
  }
}

size_t allocate_smem_bytes(int T, int B) {
  const size_t cells = static_cast<size_t>(B) + 1;
  const size_t key_words = (cells * T + 31) / 32;
  return cells * 2 * sizeof(double) + cells * 4 * sizeof(int) + key_words * 4 * 4 + key_words * 2 * 4;
}

}  // namespace
}  // namespace sg

extern "C" size_t sg_allocate_tiers_device_workspace_bytes(int32_t num_requests, int32_t row_budget) {
  if (num_requests < 1 || row_budget < 0) return 0;
  return static_cast<size_t>(num_requests + 1) * (static_cast<size_t>(row_budget) + 1) * sizeof(int32_t);
}

extern "C" int sg_allocate_tiers_device(int32_t num_requests, const double* weights, int32_t num_options,
                                        const int32_t* options, const double* utilities, int32_t row_budget,
                                        double fixed_row_equivalent, const int32_t* curve_rows,
                                        const double* curve_cost, int32_t curve_points, int32_t* allocation,
                                        int32_t* status, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace sg;
  if (allocation == nullptr || curve_points < 0)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers_device: bad output");
  Problem hp{num_requests, num_options, row_budget, weights, options, utilities, fixed_row_equivalent,
             curve_rows, curve_cost, curve_points};
  int st = validate_shape(hp, "sg_allocate_tiers_device");
  if (st != SG_OK) return st;
  if (num_options > kAllocMaxOptions || row_budget > kAllocMaxBudget || curve_points > kAllocMaxCurve)
    return fail(SG_ERR_UNSUPPORTED, "sg_allocate_tiers_device: at most 8 options, 4096 rows, 64 curve points");
  const size_t need = sg_allocate_tiers_device_workspace_bytes(num_requests, row_budget);
  if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 3u) != 0) {
    set_error("sg_allocate_tiers_device: workspace of %zu bytes, %zu needed (4-byte aligned)", workspace_bytes, need);
    return SG_ERR_WORKSPACE;
  }
  if ((reinterpret_cast<uintptr_t>(weights) & 7u) != 0 || (reinterpret_cast<uintptr_t>(utilities) & 7u) != 0 ||
      (reinterpret_cast<uintptr_t>(allocation) & 3u) != 0 || (reinterpret_cast<uintptr_t>(status) & 3u) != 0)
    return fail(SG_ERR_INVALID_ARGUMENT, "sg_allocate_tiers_device: misaligned pointer");
  DeviceProblem p = {};
  p.R = num_requests;
  p.T = num_options;
  p.B = row_budget;
  for (int k = 0; k < num_options; ++k) p.options[k] = options[k];
  p.fixed = fixed_row_equivalent;
  p.curve_points = curve_points;
  for (int s = 0; s < curve_points; ++s) {
    p.curve_rows[s] = curve_rows[s];
    p.curve_cost[s] = curve_cost[s];
  }
  p.weights = weights;
  p.utilities = utilities;
  p.allocation = allocation;
  p.status = status;
  p.links = static_cast<int32_t*>(workspace);
  const size_t smem = allocate_smem_bytes(num_options, row_budget);
  static std::atomic<int> limits[kAllocMaxOptions + 1][kMaxDevices];
  auto run = [&](auto kernel) -> int {
    const int s = ensure_dynamic_smem(kernel, smem, limits[num_options]);
    if (s != SG_OK) return s;
    kernel<<<1, kAllocThreads, smem, static_cast<cudaStream_t>(stream)>>>(p);
    return check_launch("allocate_tiers_kernel");
  };
  switch (num_options) {
    case 1: return run(allocate_tiers_kernel<1>);
    case 2: return run(allocate_tiers_kernel<2>);
    case 3: return run(allocate_tiers_kernel<3>);
    case 4: return run(allocate_tiers_kernel<4>);
    case 5: return run(allocate_tiers_kernel<5>);
    case 6: return run(allocate_tiers_kernel<6>);
    case 7: return run(allocate_tiers_kernel<7>);
    default: return run(allocate_tiers_kernel<8>);
  }
}
