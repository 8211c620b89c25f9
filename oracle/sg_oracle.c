/*
 * TEST INFRASTRUCTURE — CPU oracle for the specgrove_b200 acceptance walk and
 * KV commit.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg may load this library; the product path never does.
 *
 * It restates, in plain C, the reference's uniform-driven tree acceptance:
 *
 *   scan rule    fused_tree_sampling.py:538-627 (fused_tree_sample_scan_kernel):
 *                at the visited node of depth d, threshold = u[d] * row_total,
 *                token = first index whose inclusive prefix > threshold
 *                (fallback V-1), child = first edge with (parent, token), stop
 *                when there is no child or depth == max_depth.
 *   sparse exit  fused_tree_sampling.py:688-824: route among the children by
 *                cumulative child probability against u[2d]; on exit, draw from
 *                the row with the children removed against u[2d+1] (fallback:
 *                last non-child token).
 *   follow       fused_tree_sampling.py:120-151 (walk pre-drawn posterior
 *                tokens; the law of sampling.py:903-950).
 *   KV commit    continuous_tree_block_decode.py:215-261
 *                (append_packed_sequence: dst row i <- src row keep[i]).
 *
 * Two arithmetics are provided for the probability sums:
 *   - exact:  every fp32 p becomes floor(p * 2^64) in unsigned 128-bit
 *             integers; sums are exact and order-independent.  This is the
 *             arithmetic the CUDA kernels implement, so GPU and oracle
 *             decisions must agree bit for bit.
 *   - fp64:   a sequential fp64 running sum, the reference CPU rule of
 *             fused_tree_sampling.py:2607-2612 (cumsum in fp64) with the
 *             kernel's strict comparison.  Used to pin the exact arithmetic
 *             against the reference's own rounding.
 *
 * The uniform stream for "no explicit uniforms" is Philox4x32-10 (Salmon et
 * al., SC 2011) keyed by (seed) with counter (node, request lo, request hi, 0);
 * the CUDA library uses the same published generator.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef unsigned __int128 u128;

enum { RULE_SCAN = 0, RULE_SPARSE_EXIT = 1 };
enum { ARITH_EXACT = 0, ARITH_FP64 = 1 };

/* ---- exact 64.64 masses ------------------------------------------------ */

static int mass_of(float p, u128* out) {
  uint32_t bits;
  memcpy(&bits, &p, 4);
  if ((bits & 0x7fffffffu) == 0u) {
    *out = 0;
    return 0;
  }
  uint32_t e = (bits >> 23) & 0xffu;
  if ((bits >> 31) || e >= 167u) {
    *out = 0;
    return 1;
  }
  uint64_t m = bits & 0x7fffffu;
  int eff = 1;
  if (e) {
    m |= 0x800000u;
    eff = (int)e;
  }
  int s = eff - 86; /* p * 2^64 = m * 2^(eff - 86) */
  if (s >= 0)
    *out = ((u128)m) << s;
  else
    *out = (-s < 64) ? (u128)(m >> (-s)) : 0;
  return 0;
}

/* floor(u * total) for u in [0, 1), exact. */
static u128 mass_scale(double u, u128 total) {
  uint64_t bits;
  memcpy(&bits, &u, 8);
  uint64_t e = (bits >> 52) & 0x7ffu;
  uint64_t m = bits & ((1ull << 52) - 1);
  int shift;
  if (e == 0) {
    shift = 1074;
  } else {
    m |= 1ull << 52;
    shift = 1075 - (int)e;
  }
  if (m == 0) return 0;
  /* total < 2^122 and m < 2^53: split the product to stay within 128 bits */
  u128 lo = (u128)(uint64_t)total * m;          /* < 2^117 */
  u128 hi = (u128)(uint64_t)(total >> 64) * m;  /* < 2^111, weight 2^64 */
  /* value = (hi << 64) + lo, shifted right by `shift` */
  if (shift >= 64 + 128) return 0;
  u128 result;
  if (shift >= 64) {
    int s2 = shift - 64;
    u128 carry_lo = lo >> 64; /* lo's upper part contributes at weight 2^64 */
    u128 top = hi + carry_lo; /* (hi + floor(lo / 2^64)) at weight 2^64 */
    result = (s2 >= 128) ? 0 : (top >> s2);
  } else {
    /* shift in [1, 63]: result = floor(((hi << 64) + lo) / 2^shift) */
    u128 lo_part = lo >> shift;
    u128 hi_part = hi << (64 - shift);
    result = hi_part + lo_part;
  }
  return result;
}

/* ---- Philox4x32-10 ------------------------------------------------------ */

static void philox(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    uint32_t n1 = (uint32_t)p1;
    uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    uint32_t n3 = (uint32_t)p0;
    c[0] = n0;
    c[1] = n1;
    c[2] = n2;
    c[3] = n3;
  }
}

static double u53(uint32_t a, uint32_t b) {
  uint64_t v = ((uint64_t)b << 32) | a;
  return (double)(v >> 11) * (1.0 / 9007199254740992.0);
}

void sgo_node_uniforms(uint64_t seed, uint64_t request, uint32_t node, double* route, double* exit_) {
  uint32_t c[4] = {node, (uint32_t)request, (uint32_t)(request >> 32), 0u};
  philox(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  *route = u53(c[0], c[1]);
  *exit_ = u53(c[2], c[3]);
}

/* ---- one inverse-CDF draw over a row ------------------------------------ */

static int is_child_token(int64_t t, const int64_t* child_tok, int k) {
  for (int c = 0; c < k; ++c)
    if (child_tok[c] == t) return 1;
  return 0;
}

/* Returns the drawn token or -1 when the (masked) row total is zero. */
static int64_t draw_row(const float* row, int64_t V, double u, const int64_t* mask_tok, int k,
                        int arith, int* bad) {
  if (arith == ARITH_EXACT) {
    u128 total = 0, m;
    for (int64_t t = 0; t < V; ++t) {
      *bad |= mass_of(row[t], &m);
      if (k && is_child_token(t, mask_tok, k)) continue;
      total += m;
    }
    if (total == 0) return -1;
    u128 thr = mass_scale(u, total), run = 0;
    for (int64_t t = 0; t < V; ++t) {
      if (k && is_child_token(t, mask_tok, k)) continue;
      mass_of(row[t], &m);
      run += m;
      if (run > thr) return t;
    }
    return -1;
  } else {
    double total = 0.0;
    for (int64_t t = 0; t < V; ++t) {
      if (k && is_child_token(t, mask_tok, k)) continue;
      total += (double)row[t];
    }
    double thr = u * total, run = 0.0;
    for (int64_t t = 0; t < V; ++t) {
      if (k && is_child_token(t, mask_tok, k)) continue;
      run += (double)row[t];
      if (thr < run) return t;
    }
    return -1;
  }
}

static int find_child(const int64_t* par, const int64_t* tok, int n, int64_t cur, int64_t token) {
  for (int j = 1; j < n; ++j)
    if (par[j] == cur && tok[j] == token) return j;
  return -1;
}

static int walk_one(const float* probs, int64_t V, const int64_t* par, const int64_t* tok, int n,
                    int32_t D, int32_t rule, const double* ut, uint64_t seed, uint64_t request,
                    int arith, int64_t* out) {
  int bad = 0;
  for (int i = 0; i < D + 2; ++i) out[i] = -1;
  if (n < 1 || par[0] != -1) return 3;
  for (int j = 1; j < n; ++j)
    if (par[j] < 0 || par[j] >= j || tok[j] < 0 || tok[j] >= V) return 3;
  int64_t* child_tok = (int64_t*)malloc(sizeof(int64_t) * (size_t)n);
  int* child_node = (int*)malloc(sizeof(int) * (size_t)n);
  int cur = 0, accepted = 0;
  for (int depth = 0; depth <= D; ++depth) {
    const float* row = probs + (int64_t)cur * V;
    double u_main, u_exit = 0.0;
    if (ut) {
      if (rule == RULE_SPARSE_EXIT) {
        u_main = ut[2 * depth];
        u_exit = ut[2 * depth + 1];
      } else {
        u_main = ut[depth];
      }
    } else {
      sgo_node_uniforms(seed, request, (uint32_t)cur, &u_main, &u_exit);
    }
    int k = 0;
    if (rule == RULE_SPARSE_EXIT) {
      for (int j = 1; j < n; ++j)
        if (par[j] == cur) {
          child_node[k] = j;
          child_tok[k] = tok[j];
          ++k;
        }
      int route = -1;
      if (arith == ARITH_EXACT) {
        u128 thr = mass_scale(u_main, ((u128)1) << 64), cum = 0, m;
        for (int c = 0; c < k; ++c) {
          bad |= mass_of(row[child_tok[c]], &m);
          cum += m;
          if (cum > thr) {
            route = child_node[c];
            break;
          }
        }
      } else {
        double cum = 0.0;
        for (int c = 0; c < k; ++c) {
          cum += (double)row[child_tok[c]];
          if (u_main < cum) {
            route = child_node[c];
            break;
          }
        }
      }
      if (route >= 0 && depth < D) {
        out[accepted++] = route;
        cur = route;
        continue;
      }
      int64_t token = draw_row(row, V, u_exit, child_tok, k, arith, &bad);
      if (token < 0) {
        for (int64_t t = V - 1; t >= 0; --t)
          if (!is_child_token(t, child_tok, k)) {
            token = t;
            break;
          }
      }
      out[D] = accepted;
      out[D + 1] = token;
      break;
    }
    int64_t token = draw_row(row, V, u_main, NULL, 0, arith, &bad);
    if (token < 0) token = V - 1;
    int child = find_child(par, tok, n, cur, token);
    if (child >= 0 && depth < D) {
      out[accepted++] = child;
      cur = child;
      continue;
    }
    out[D] = accepted;
    out[D + 1] = token;
    break;
  }
  free(child_tok);
  free(child_node);
  return bad ? 4 : 0;
}

/*
 * Batched walk over packed rows; argument meaning as sg_tree_accept_probs in
 * include/specgrove_b200.h, with host pointers.  Returns the worst status.
 */
int sgo_tree_accept_probs(const float* probs, int64_t vocab, const int64_t* row_offsets,
                          const int64_t* parents, const int64_t* tokens, int32_t num_trees,
                          int32_t max_depth, int32_t rule, const double* uniforms,
                          int32_t uniform_stride, uint64_t seed, const int64_t* request_ids,
                          int32_t arith, int64_t* out) {
  int worst = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(max : worst)
  for (int t = 0; t < num_trees; ++t) {
    int64_t r0 = row_offsets[t];
    int n = (int)(row_offsets[t + 1] - r0);
    const double* ut = uniforms ? uniforms + (int64_t)t * uniform_stride : NULL;
    uint64_t req = request_ids ? (uint64_t)request_ids[t] : (uint64_t)t;
    int st = walk_one(probs + r0 * vocab, vocab, parents + r0, tokens + r0, n, max_depth, rule, ut,
                      seed, req, arith, out + (int64_t)t * (max_depth + 2));
    if (st > worst) worst = st;
  }
  return worst;
}

/*
 * Direct-logits scan rule (fused_tree_sampling.py:942-1115, the kernel of
 * tree_verify_ancestral_logits_fused_scan(_batched), :2417-2533): at the
 * visited node x_j = double(logit_j) / T, w_j = exp(x_j - max x); the token
 * is the first index whose inclusive prefix of w exceeds u[depth] * sum(w)
 * (fallback V - 1).  ARITH_EXACT sums floor(w * 2^64) exactly (the CUDA
 * kernel's arithmetic), ARITH_FP64 is the reference kernel's fp64 running sum.
 * Logits are fp32 here (bf16 rows are widened exactly by the caller).
 */
static u128 weight_mass(double w) {
  return w >= 1.0 ? ((u128)1) << 64 : (u128)(uint64_t)(w * 18446744073709551616.0);
}

static int64_t draw_logit_row(const float* row, int64_t V, double inv, double u, int arith, int* bad) {
  float m = -INFINITY;
  for (int64_t t = 0; t < V; ++t) {
    if (row[t] != row[t]) *bad = 1;
    if (row[t] > m) m = row[t];
  }
  const double xmax = (double)m * inv;
  if (arith == ARITH_EXACT) {
    u128 total = 0;
    for (int64_t t = 0; t < V; ++t) total += weight_mass(exp((double)row[t] * inv - xmax));
    if (total == 0) return -1;
    u128 thr = mass_scale(u, total), run = 0;
    for (int64_t t = 0; t < V; ++t) {
      run += weight_mass(exp((double)row[t] * inv - xmax));
      if (run > thr) return t;
    }
    return -1;
  }
  double total = 0.0;
  for (int64_t t = 0; t < V; ++t) total += exp((double)row[t] * inv - xmax);
  double thr = u * total, run = 0.0;
  for (int64_t t = 0; t < V; ++t) {
    run += exp((double)row[t] * inv - xmax);
    if (thr < run) return t;
  }
  return -1;
}

int sgo_tree_accept_logits(const float* logits, int64_t vocab, const int64_t* row_offsets, const int64_t* parents,
                           const int64_t* tokens, int32_t num_trees, int32_t max_depth, double temperature,
                           const double* uniforms, int32_t uniform_stride, uint64_t seed,
                           const int64_t* request_ids, int32_t arith, int64_t* out) {
  int worst = 0;
  const double inv = 1.0 / temperature;
#pragma omp parallel for schedule(dynamic, 1) reduction(max : worst)
  for (int t = 0; t < num_trees; ++t) {
    const int64_t r0 = row_offsets[t];
    const int n = (int)(row_offsets[t + 1] - r0);
    const int64_t* par = parents + r0;
    const int64_t* tok = tokens + r0;
    int64_t* o = out + (int64_t)t * (max_depth + 2);
    for (int i = 0; i < max_depth + 2; ++i) o[i] = -1;
    int st = 0, bad = 0;
    if (n < 1 || par[0] != -1) st = 3;
    for (int j = 1; j < n && !st; ++j)
      if (par[j] < 0 || par[j] >= j || tok[j] < 0 || tok[j] >= vocab) st = 3;
    const uint64_t req = request_ids ? (uint64_t)request_ids[t] : (uint64_t)t;
    int cur = 0, accepted = 0;
    for (int depth = 0; depth <= max_depth && !st; ++depth) {
      double u, unused;
      if (uniforms)
        u = uniforms[(int64_t)t * uniform_stride + depth];
      else
        sgo_node_uniforms(seed, req, (uint32_t)cur, &u, &unused);
      int64_t token = draw_logit_row(logits + (r0 + cur) * vocab, vocab, inv, u, arith, &bad);
      if (token < 0) token = vocab - 1;
      const int child = find_child(par, tok, n, cur, token);
      if (child >= 0 && depth < max_depth) {
        o[accepted++] = child;
        cur = child;
        continue;
      }
      o[max_depth] = accepted;
      o[max_depth + 1] = token;
      break;
    }
    if (bad && st == 0) st = 4;
    if (st > worst) worst = st;
  }
  return worst;
}

/* Walk pre-drawn posterior tokens (fused_tree_sampling.py:120-151). */
int sgo_tree_follow(const int64_t* posterior, const int64_t* row_offsets, const int64_t* parents,
                    const int64_t* tokens, int32_t num_trees, int32_t max_depth, int64_t* out) {
  for (int t = 0; t < num_trees; ++t) {
    int64_t r0 = row_offsets[t];
    int n = (int)(row_offsets[t + 1] - r0);
    int64_t* o = out + (int64_t)t * (max_depth + 2);
    for (int i = 0; i < max_depth + 2; ++i) o[i] = -1;
    int cur = 0, accepted = 0;
    int64_t bonus = posterior[r0];
    for (int depth = 0; depth < max_depth; ++depth) {
      int child = find_child(parents + r0, tokens + r0, n, cur, bonus);
      if (child < 0) break;
      o[accepted++] = child;
      cur = child;
      bonus = posterior[r0 + cur];
    }
    o[max_depth] = accepted;
    o[max_depth + 1] = bonus;
  }
  return 0;
}

/* KV commit: for every plane, dst row dst_rows[i] <- src row src_rows[i]
 * (continuous_tree_block_decode.py:215-261).  Rows are gathered before any
 * store so the in-place compaction has the reference's gather semantics. */
int sgo_kv_commit(void* dst, int64_t dst_plane_rows, const void* src, int64_t src_plane_rows,
                  int64_t num_planes, int64_t row_bytes, const int64_t* src_rows,
                  const int64_t* dst_rows, int64_t num_rows) {
  unsigned char* tmp = (unsigned char*)malloc((size_t)(num_rows * row_bytes) + 1);
  int status = 0;
  for (int64_t pl = 0; pl < num_planes; ++pl) {
    const unsigned char* s = (const unsigned char*)src + pl * src_plane_rows * row_bytes;
    unsigned char* d = (unsigned char*)dst + pl * dst_plane_rows * row_bytes;
    for (int64_t i = 0; i < num_rows; ++i) {
      if (src_rows[i] < 0 || src_rows[i] >= src_plane_rows) {
        status = 5;
        continue;
      }
      memcpy(tmp + i * row_bytes, s + src_rows[i] * row_bytes, (size_t)row_bytes);
    }
    for (int64_t i = 0; i < num_rows; ++i) {
      if (dst_rows[i] < 0 || dst_rows[i] >= dst_plane_rows || src_rows[i] < 0 ||
          src_rows[i] >= src_plane_rows) {
        status = 5;
        continue;
      }
      memcpy(d + dst_rows[i] * row_bytes, tmp + i * row_bytes, (size_t)row_bytes);
    }
  }
  free(tmp);
  return status;
}

/* Exact mass of one fp32 value as (lo, hi) limbs, exposed for unit tests. */
int sgo_mass_of(float p, uint64_t* lo, uint64_t* hi) {
  u128 m;
  int bad = mass_of(p, &m);
  *lo = (uint64_t)m;
  *hi = (uint64_t)(m >> 64);
  return bad;
}

void sgo_mass_scale(double u, uint64_t tlo, uint64_t thi, uint64_t* lo, uint64_t* hi) {
  u128 total = ((u128)thi << 64) | tlo;
  u128 r = mass_scale(u, total);
  *lo = (uint64_t)r;
  *hi = (uint64_t)(r >> 64);
}

/* ---- terminal-mass verifier ---------------------------------------------
 * Restates sampling.py:542-735 (tree_block_verify_terminal_mass, exit_mode
 * "internal", prefix_mode "batched") with explicit uniforms, in the
 * arithmetic of the CUDA kernel (specgrove_b200/csrc/terminal_mass.cu): row
 * masses as exact 64.64 sums converted once to the nearest double,
 * normalisation / prefix products / terminal masses in fp64 in node order,
 * the terminal node as the first node whose running terminal mass exceeds
 * u0 * total, the bonus token by the exact fixed-point inverse CDF over the
 * terminal node's row without its children's tokens.  Output layout as
 * sgo_tree_accept_probs.  Returns the worst status (3 tree, 4 probability).
 */
static double u128_to_double(u128 m) {
  uint64_t hi = (uint64_t)(m >> 64), lo = (uint64_t)m;
  if (hi == 0) return (double)lo;
  int lz = __builtin_clzll(hi);
  uint64_t top = lz ? (hi << lz) | (lo >> (64 - lz)) : hi;
  uint64_t rest = lz ? (lo << lz) : lo;
  uint64_t v = top | (rest != 0 ? 1ull : 0ull);
  return ldexp((double)v, 64 - lz);
}

static int terminal_one(const float* probs, int64_t V, const int64_t* par, const int64_t* tok, int n,
                        int32_t D, double u_node, double u_bonus, int64_t* out) {
  int bad = 0;
  for (int i = 0; i < D + 2; ++i) out[i] = -1;
  if (n < 1 || n > 256 || par[0] != -1) return 3;
  int* dep = (int*)calloc((size_t)n, sizeof(int));
  for (int j = 1; j < n; ++j) {
    if (par[j] < 0 || par[j] >= j || tok[j] < 0 || tok[j] >= V) { free(dep); return 3; }
    dep[j] = dep[par[j]] + 1;
    if (dep[j] > D) { free(dep); return 3; }
    for (int i = 1; i < j; ++i)
      if (par[i] == par[j] && tok[i] == tok[j]) { free(dep); return 3; }
  }
  u128* covered = (u128*)calloc((size_t)n, sizeof(u128));
  u128* total = (u128*)calloc((size_t)n, sizeof(u128));
  u128* edge = (u128*)calloc((size_t)n, sizeof(u128));
  char* internal = (char*)calloc((size_t)n, 1);
  double* prefix = (double*)calloc((size_t)n, sizeof(double));
  double* term = (double*)calloc((size_t)n, sizeof(double));
  int status = 0, pick = -1;
  for (int j = 1; j < n; ++j) {
    bad |= mass_of(probs[(int64_t)par[j] * V + tok[j]], &edge[j]);
    covered[par[j]] += edge[j];
    internal[par[j]] = 1;
  }
  for (int j = 0; j < n; ++j) {
    if (!internal[j]) continue;
    u128 s = 0, m;
    for (int64_t t = 0; t < V; ++t) {
      bad |= mass_of(probs[(int64_t)j * V + t], &m);
      s += m;
    }
    total[j] = s;
  }
  double total_term = 0.0;
  prefix[0] = 1.0;
  for (int j = 0; j < n && !status; ++j) {
    if (j > 0) prefix[j] = prefix[par[j]] * (u128_to_double(edge[j]) / u128_to_double(total[par[j]]));
    double exit_frac = 1.0;
    if (internal[j]) {
      if (total[j] == 0 || total[j] < covered[j]) { status = 4; break; }
      exit_frac = u128_to_double(total[j] - covered[j]) / u128_to_double(total[j]);
    }
    term[j] = prefix[j] * exit_frac;
    total_term += term[j];
  }
  if (bad) status = 4;
  if (!status && total_term > 0.0 && isfinite(total_term)) {
    double thr = u_node * total_term, cum = 0.0;
    for (int j = 0; j < n; ++j) {
      cum += term[j];
      if (term[j] > 0.0) pick = j;
      if (cum > thr && term[j] > 0.0) break;
    }
  }
  if (!status && pick < 0) status = 4;
  if (!status) {
    const float* row = probs + (int64_t)pick * V;
    u128 exit_total, m;
    if (internal[pick]) {
      exit_total = total[pick] - covered[pick];
    } else {
      exit_total = 0;
      for (int64_t t = 0; t < V; ++t) {
        bad |= mass_of(row[t], &m);
        exit_total += m;
      }
    }
    for (int64_t t = 0; t < V; ++t) bad |= mass_of(row[t], &m);  /* the terminal row is read whole */
    if (bad || exit_total == 0) {
      status = 4;
    } else {
      u128 thr = mass_scale(u_bonus, exit_total), run = 0;
      int64_t bonus = -1;
      for (int64_t t = 0; t < V && bonus < 0; ++t) {
        int excluded = 0;
        for (int j = 1; j < n; ++j) excluded |= par[j] == pick && tok[j] == t;
        if (excluded) continue;
        mass_of(row[t], &m);
        run += m;
        if (run > thr) bonus = t;
      }
      if (bonus < 0) {
        status = 4;
      } else {
        int count = dep[pick];
        for (int x = pick, i = count - 1; x != 0; x = (int)par[x], --i) out[i] = x;
        out[D] = count;
        out[D + 1] = bonus;
      }
    }
  }
  free(dep); free(covered); free(total); free(edge); free(internal); free(prefix); free(term);
  return status;
}

int sgo_tree_verify_terminal_mass(const float* probs, int64_t vocab, const int64_t* row_offsets,
                                  const int64_t* parents, const int64_t* tokens, int32_t num_trees,
                                  int32_t max_depth, const double* uniforms, int32_t uniform_stride,
                                  uint64_t seed, const int64_t* request_ids, int64_t* out) {
  int worst = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(max : worst)
  for (int t = 0; t < num_trees; ++t) {
    int64_t r0 = row_offsets[t];
    int n = (int)(row_offsets[t + 1] - r0);
    double u0, u1;
    if (uniforms) {
      u0 = uniforms[(int64_t)t * uniform_stride];
      u1 = uniforms[(int64_t)t * uniform_stride + 1];
    } else {
      uint64_t req = request_ids ? (uint64_t)request_ids[t] : (uint64_t)t;
      uint32_t c[4] = {0u, (uint32_t)req, (uint32_t)(req >> 32), 2u};
      philox(c, (uint32_t)seed, (uint32_t)(seed >> 32));
      u0 = u53(c[0], c[1]);
      u1 = u53(c[2], c[3]);
    }
    int st = terminal_one(probs + r0 * vocab, vocab, parents + r0, tokens + r0, n, max_depth, u0, u1,
                          out + (int64_t)t * (max_depth + 2));
    if (st > worst) worst = st;
  }
  return worst;
}
