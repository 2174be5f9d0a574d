// Host-side planners: the B200 counterpart of the reference planners' host
// logic (row folding, tiling, core assignment, load balancing).
//
//   reference                                          here
//   fold empty rows (load_balanced_new_DM.cpp:50-61)   empty rows become zero-fill units
//   N per core (host_code_utils.cpp:32-66)             fixed 128-column tiles (MMA M)
//   core grid (load_balanced_new_DM.cpp:71-107)        one persistent CTA per SM
//   serpentine LB (load_balanced_new_DM.cpp:346-393)   serpentine_order() over work units
//   no-LB variant (load_balanced_new_DM.cpp:339-344)   contiguous split (opts.no_load_balance)
//   SDDMM even split (bsr_sddmm_multicore_naive.cpp:266-310)  4-segment units, same balancer
//
// Nothing here touches the GPU, so every branch is testable on CPU.
#include <algorithm>
#include <climits>
#include <cstring>
#include <cstdlib>
#include <numeric>
#include <queue>
#include <string>
#include <system_error>
#include <thread>

#include "bsp_internal.h"

namespace bsp {

int spmm_smem_bytes(int stages, int stage_bytes, bool c_f32);
int sddmm_smem_bytes(int stages, int stage_bytes);

namespace {

int pow2_at_least(int x) {
  int p = 32;
  while (p < x) p <<= 1;
  return p;
}

// Largest multiple of 32 that divides R and is <= 256 (the MMA N limit).
int slab_height(int R) {
  if (R <= 256) return R;
  for (int d = 256; d >= 32; d -= 32)
    if (R % d == 0) return d;
  return 32;
}

}  // namespace

// Threads for a host planning pass over `items` independent items: at most
// 16 and the machine's cores, at least `min_items` items each, and the
// per-thread scratch (`scratch_bytes`) within 256 MB.  BSP_PLANNER_THREADS
// overrides the count (the plans do not depend on it).
// A planning thread may carry a cap on the threads it spawns (the batch path
// plans several patterns at once and shares the cores among them).
static thread_local int tl_thread_cap = 0;

void set_planner_thread_cap(int cap) { tl_thread_cap = cap; }

static int planner_threads(int64_t items, int64_t min_items, int64_t scratch_bytes) {
  // the core count is read once (the C library parses /sys on every query)
  static const unsigned cores = std::max(1u, std::thread::hardware_concurrency());
  int t = static_cast<int>(std::min<unsigned>(16, cores));
  if (tl_thread_cap > 0) t = std::min(t, tl_thread_cap);
  if (const char* env = std::getenv("BSP_PLANNER_THREADS")) {
    const int v = std::atoi(env);
    if (v > 0) return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(v, items)));
  }
  t = static_cast<int>(std::min<int64_t>(t, std::max<int64_t>(1, items / std::max<int64_t>(1, min_items))));
  t = static_cast<int>(std::min<int64_t>(t, std::max<int64_t>(1, (int64_t(256) << 20) / std::max<int64_t>(1, scratch_bytes))));
  return t;
}

// fn(thread, begin, end) over `nt` contiguous ranges of [0, n); the first
// failing status (in range order) is returned.
template <class F>
static bsp_status parallel_ranges(int64_t n, int nt, F&& fn) {
  if (nt <= 1) return fn(0, int64_t(0), n);
  std::vector<bsp_status> res(static_cast<size_t>(nt), BSP_OK);
  std::vector<std::string> msg(static_cast<size_t>(nt));  // error messages are per thread
  std::vector<std::thread> th;
  auto body = [&](int t) {
    try {
      res[static_cast<size_t>(t)] = fn(t, n * t / nt, n * (t + 1) / nt);
      if (res[static_cast<size_t>(t)] != BSP_OK) msg[static_cast<size_t>(t)] = bsp_last_error_string();
    } catch (const std::bad_alloc&) {
      res[static_cast<size_t>(t)] = BSP_ERR_ALLOC;
      msg[static_cast<size_t>(t)] = "host allocation failed in the planner";
    }
  };
  try {
    for (int t = 1; t < nt; ++t) th.emplace_back(body, t);
  } catch (const std::system_error&) {
    for (auto& x : th) x.join();
    th.clear();
    return fn(0, int64_t(0), n);  // no threads to be had: one pass
  }
  body(0);
  for (auto& x : th) x.join();
  for (int t = 0; t < nt; ++t)
    if (res[static_cast<size_t>(t)] != BSP_OK) return set_error(res[static_cast<size_t>(t)], msg[static_cast<size_t>(t)]);
  return BSP_OK;
}

static bsp_status spmm_stage_counts(bsp_spmm_plan* p);
static bsp_status rowstack_stage_lists(bsp_spmm_plan* p);
static bsp_status pair_stage_lists(bsp_spmm_plan* p);

// The reference's zig-zag balancer generalised to any item list: items sorted
// by weight (heaviest first, ties by index), then each pass deals the next
// `parts` heaviest items to parts 0..P-1 and the `parts` lightest remaining
// ones to parts P-1..0 (load_balanced_new_DM.cpp:371-393).
void serpentine_order(const std::vector<int64_t>& weight, int parts,
                      std::vector<std::vector<int32_t>>* per_part) {
  const int64_t n = static_cast<int64_t>(weight.size());
  std::vector<int32_t> perm(n);
  std::iota(perm.begin(), perm.end(), 0);
  std::stable_sort(perm.begin(), perm.end(),
                   [&](int32_t a, int32_t b) { return weight[a] > weight[b]; });
  per_part->assign(parts, {});
  int64_t assigned = 0, it = 1;
  while (assigned < n) {
    int64_t k = std::min<int64_t>(parts, n - assigned);
    int64_t sub = 0;
    for (int64_t w = 0; w < k; ++w) {
      if (assigned++ >= n) break;
      (*per_part)[w].push_back(perm[parts * (it - 1) + sub]);
      ++sub;
    }
    k = std::min<int64_t>(parts, n - assigned);
    sub = parts - k;
    for (int64_t w = parts; w > parts - k; --w) {
      if (assigned++ >= n) break;
      (*per_part)[w - 1].push_back(perm[n - parts * it + sub]);
      ++sub;
    }
    ++it;
  }
}

// Items in their given order, each to the part with the least weight so far
// (ties: lowest part).  Parts then run their lists in that order, so items
// that are close in the given order run at about the same time (shared
// operands stay in L2) while the parts' totals stay balanced.
static void ordered_greedy(const std::vector<int64_t>& weight, int parts,
                           std::vector<std::vector<int32_t>>* per_part) {
  per_part->assign(parts, {});
  std::vector<std::pair<int64_t, int32_t>> heap;
  heap.reserve(parts);
  for (int p = 0; p < parts; ++p) heap.push_back({0, p});
  auto cmp = [](const std::pair<int64_t, int32_t>& a, const std::pair<int64_t, int32_t>& b) {
    return a.first != b.first ? a.first > b.first : a.second > b.second;
  };
  std::make_heap(heap.begin(), heap.end(), cmp);
  for (size_t i = 0; i < weight.size(); ++i) {
    std::pop_heap(heap.begin(), heap.end(), cmp);
    auto& top = heap.back();
    (*per_part)[top.second].push_back(static_cast<int32_t>(i));
    top.first += weight[i];
    std::push_heap(heap.begin(), heap.end(), cmp);
  }
}

// Longest processing time first: items by weight (heaviest first, ties by
// index), each to the part with the least weight so far; each part's list is
// then put back in index order.
static void lpt_order(const std::vector<int64_t>& weight, int parts,
                      std::vector<std::vector<int32_t>>* per_part) {
  std::vector<int32_t> order(weight.size());
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) { return weight[a] > weight[b]; });
  std::vector<int64_t> sorted_w(order.size());
  for (size_t i = 0; i < order.size(); ++i) sorted_w[i] = weight[order[i]];
  ordered_greedy(sorted_w, parts, per_part);
  for (auto& v : *per_part) {
    for (auto& x : v) x = order[x];
    std::sort(v.begin(), v.end());
  }
}

static void contiguous_split(int64_t n, int parts, std::vector<std::vector<int32_t>>* per_part) {
  per_part->assign(parts, {});
  for (int p = 0; p < parts; ++p) {
    const int64_t b = n * p / parts, e = n * (p + 1) / parts;
    for (int64_t i = b; i < e; ++i) (*per_part)[p].push_back(static_cast<int32_t>(i));
  }
}

// Contiguous runs of items with about equal total weight: part p ends at the
// first item where the running total reaches (p + 1) / parts of the whole.
static void contiguous_weighted_split(const std::vector<int64_t>& weight, int parts,
                                      std::vector<std::vector<int32_t>>* per_part) {
  per_part->assign(parts, {});
  int64_t total = 0;
  for (int64_t w : weight) total += w;
  int64_t acc = 0;
  int p = 0;
  const int64_t n = static_cast<int64_t>(weight.size());
  for (int64_t i = 0; i < n; ++i) {
    // keep at least one item for every later part
    while (p < parts - 1 && acc * parts >= total * (p + 1) && n - i >= parts - p - 1 &&
           !(*per_part)[p].empty())
      ++p;
    if (p < parts - 1 && n - i == parts - p - 1 && !(*per_part)[p].empty()) ++p;
    (*per_part)[p].push_back(static_cast<int32_t>(i));
    acc += weight[static_cast<size_t>(i)];
  }
}

static bsp_status check_pattern(const int32_t* row_ptr, const int32_t* col_idx, int64_t nbr,
                                int64_t nbc, int64_t nnzb) {
  if (row_ptr[0] != 0) return set_error(BSP_ERR_INVALID_ARG, "row_ptr[0] must be 0");
  for (int64_t i = 0; i < nbr; ++i)
    if (row_ptr[i + 1] < row_ptr[i])
      return set_error(BSP_ERR_INVALID_ARG, "row_ptr must be non-decreasing");
  if (row_ptr[nbr] != nnzb)
    return set_error(BSP_ERR_INVALID_ARG, "row_ptr[last] must equal nnzb");
  for (int64_t b = 0; b < nnzb; ++b)
    if (col_idx[b] < 0 || col_idx[b] >= nbc)
      return set_error(BSP_ERR_INVALID_ARG, "col_idx out of range at block " + std::to_string(b));
  return BSP_OK;
}

bsp_status plan_spmm_host(bsp_spmm_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                          int sm_count, int max_smem, const bsp_spmm_opts* opts) {
  bsp_spmm_opts o;
  memset(&o, 0, sizeof(o));
  if (opts) o = *opts;
  const int64_t M = p->M, K = p->K, N = p->N;
  const int R = p->R, C = p->C;
  if (R <= 0 || C <= 0 || R % 32 || C % 32)
    return set_error(BSP_ERR_INVALID_ARG, "block dims R, C must be positive multiples of 32");
  if (M <= 0 || K <= 0 || M % R || K % C)
    return set_error(BSP_ERR_INVALID_ARG, "M % R and K % C must be 0");
  if (N <= 0 || N % 8) return set_error(BSP_ERR_INVALID_ARG, "N must be a positive multiple of 8");
  if (p->nnzb < 0 || p->nnzb * R >= (int64_t(1) << 31) || K >= (int64_t(1) << 31) ||
      M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31))
    return set_error(BSP_ERR_UNSUPPORTED, "matrix too large for 32-bit TMA coordinates");
  const int64_t nbr = M / R, nbc = K / C;
  bsp_status st = check_pattern(row_ptr, col_idx, nbr, nbc, p->nnzb);
  if (st != BSP_OK) return st;
  // DDA runs on the row-stacked kernel unless the caller asks for one of the
  // swap-AB variants (group_mma 2: one MMA per block, 3: stacked swap-AB).
  // DDA: group_mma 4 forces the single-CTA row-stacked kernel, 5 the CTA-pair
  // kernel (2-SM MMA).  By default both schedules are built and the one with
  // the shorter estimated critical path wins: a pair stage moves twice the
  // rows for ~0.74x the time of a single-CTA stage (measured on B200 from
  // 10% density up), but pairing 8 block-rows instead of 4 widens each
  // unit's column union, which costs more than it saves below ~20% block
  // density.
  if (p->strategy == BSP_DDA && o.group_mma != 2 && o.group_mma != 3) {
    if (o.group_mma == 4 || sm_count < 2) return plan_spmm_rowstack(p, row_ptr, col_idx, sm_count, max_smem, opts);
    if (o.group_mma == 5) return plan_spmm_pair(p, row_ptr, col_idx, sm_count, max_smem, opts);
    if (o.group_mma == 6)
      return spmm_twin_eligible(p) ? plan_spmm_twin(p, row_ptr, col_idx, sm_count, max_smem, opts)
                                   : plan_spmm_pair(p, row_ptr, col_idx, sm_count, max_smem, opts);
    // a pair CTA loads one 128-column half of a 256-column tile: with N <= 128
    // one of the two would load nothing but out-of-range zeros
    if (p->N <= 128) return plan_spmm_rowstack(p, row_ptr, col_idx, sm_count, max_smem, opts);
    // Both schedules without their stage lists (the choice needs only the
    // stage counts); the lists are then built for the winner alone.
    // The two are built at once, the pair schedule on a second host thread.
    bsp_spmm_plan pair;
    pair.M = p->M;
    pair.K = p->K;
    pair.N = p->N;
    pair.R = p->R;
    pair.C = p->C;
    pair.nnzb = p->nnzb;
    pair.c_type = p->c_type;
    pair.strategy = p->strategy;
    bsp_status st2 = BSP_OK;
    const int cap = tl_thread_cap;
    std::thread pair_thread([&, cap]() {
      tl_thread_cap = cap;
      st2 = plan_spmm_pair(&pair, row_ptr, col_idx, sm_count, max_smem, opts, false);
    });
    bsp_status st1 = plan_spmm_rowstack(p, row_ptr, col_idx, sm_count, max_smem, opts, false);
    pair_thread.join();
    if (st1 != BSP_OK) return plan_spmm_pair(p, row_ptr, col_idx, sm_count, max_smem, opts);
    auto longest = [](const bsp_spmm_plan* q, int step) {
      int64_t m = 0;
      for (size_t c = 0; c + step < q->h_cta_stage_begin.size(); c += step)
        m = std::max<int64_t>(m, q->h_cta_stage_begin[c + 1] - q->h_cta_stage_begin[c]);
      return m;
    };
    const int64_t s1 = longest(p, 1);
    if (st2 != BSP_OK) return rowstack_stage_lists(p);
    const int64_t s2 = longest(&pair, 2);  // per pair: the leader's list (both lists are equal length)
    if (74 * s2 < 100 * s1) {  // pair time ~ 0.74 x its stages vs single-CTA stages
      bsp_device* dev = p->dev;
      *p = std::move(pair);
      p->dev = dev;
      return pair_stage_lists(p);
    }
    return rowstack_stage_lists(p);
  }
  p->variant = 0;

  const int Rs = slab_height(R);
  const int kc = (C % 64 == 0) ? 64 : 32;
  const int ntiles_total = static_cast<int>((N + kTileN - 1) / kTileN);
  int G = 1, NT = 1;
  switch (p->strategy) {
    case BSP_NAIVE:
      break;
    case BSP_SNF:
      NT = o.n_tiles > 0 ? o.n_tiles : std::min({kMaxNTiles, 256 / Rs, ntiles_total});
      break;
    case BSP_DDA:
      NT = o.n_tiles > 0 ? o.n_tiles : std::min({2, 256 / Rs, ntiles_total});
      NT = std::max(NT, 1);
      G = o.group_rows > 0 ? o.group_rows : std::max(1, std::min(kMaxGroupRows, 256 / (NT * Rs)));
      break;
    default:
      return set_error(BSP_ERR_INVALID_ARG, "unknown strategy");
  }
  NT = std::max(1, std::min(NT, ntiles_total));
  if (G < 1 || G > kMaxGroupRows || NT > kMaxNTiles)
    return set_error(BSP_ERR_INVALID_ARG, "group_rows must be 1..8 and n_tiles 1..4");
  if (2 * NT * G * Rs > kTmemCols)
    return set_error(BSP_ERR_INVALID_ARG,
                     "2 * n_tiles * group_rows * slab height exceeds the 512 TMEM columns");
  p->Rs = Rs;
  p->kc = kc;
  p->G = G;
  p->NT = NT;
  // Stacked issue (one MMA of N = G*Rs per k-step and tile) covers G = 1 too;
  // only DDA with group_mma = 2 issues one MMA per present block.
  p->stacked = (G == 1 || o.group_mma != 2) ? 1 : 0;

  // ---- steps and units ----
  const int stride = 1 + G;
  p->step_stride = stride;
  std::vector<int32_t>& steps = p->h_steps;
  steps.clear();
  std::vector<SpmmUnit> units;
  std::vector<int64_t> weight;
  const int nkc = C / kc;
  const int esz = p->c_type == BSP_F32 ? 4 : 2;
  std::vector<std::pair<int32_t, int32_t>> cols;  // (col, g) for a group
  for (int64_t r0 = 0; r0 < nbr; r0 += G) {
    const int nrows = static_cast<int>(std::min<int64_t>(G, nbr - r0));
    const int32_t s_begin = static_cast<int32_t>(steps.size() / stride);
    int32_t mask = 0;
    for (int g = 0; g < nrows; ++g)
      if (row_ptr[r0 + g + 1] > row_ptr[r0 + g]) mask |= 1 << g;
    if (G == 1) {
      for (int32_t b = row_ptr[r0]; b < row_ptr[r0 + 1]; ++b) {
        steps.push_back(col_idx[b]);
        steps.push_back(b);
      }
    } else {
      // merge the member rows' blocks by column: one step per distinct column
      // (a repeated column inside one row opens a new step)
      std::vector<std::pair<int32_t, int32_t>> items;  // (col, block)
      std::vector<int8_t> owner;
      for (int g = 0; g < nrows; ++g)
        for (int32_t b = row_ptr[r0 + g]; b < row_ptr[r0 + g + 1]; ++b)
          items.push_back({col_idx[b], b});
      std::stable_sort(items.begin(), items.end(),
                       [](const std::pair<int32_t, int32_t>& a,
                          const std::pair<int32_t, int32_t>& b) { return a.first < b.first; });
      int64_t cur = -1;
      for (const auto& it : items) {
        int g = 0;
        while (!(it.second >= row_ptr[r0 + g] && it.second < row_ptr[r0 + g + 1])) ++g;
        const bool open = cur >= 0 && steps[cur * stride] == it.first &&
                          steps[cur * stride + 1 + g] < 0;
        if (!open) {
          cur = static_cast<int64_t>(steps.size() / stride);
          steps.push_back(it.first);
          for (int k = 0; k < G; ++k) steps.push_back(-1);
        }
        steps[cur * stride + 1 + g] = it.second;
      }
    }
    const int32_t s_end = static_cast<int32_t>(steps.size() / stride);
    // bytes this group's steps stage per 128-column tile, for the balancer
    int64_t a_blocks = 0;
    for (int32_t s = s_begin; s < s_end; ++s)
      for (int g = 0; g < G; ++g) a_blocks += steps[s * stride + 1 + g] >= 0;
    for (int r_off = 0; r_off < R; r_off += Rs) {
      for (int t0 = 0; t0 < ntiles_total; t0 += NT) {
        SpmmUnit u;
        u.row0 = static_cast<int32_t>(r0);
        u.nrows = nrows;
        u.r_off = r_off;
        u.n0 = t0 * kTileN;
        u.nt = std::min(NT, ntiles_total - t0);
        u.step_begin = s_begin;
        u.step_end = s_end;
        u.row_mask = mask;
        units.push_back(u);
        const int64_t smem_in = int64_t(nkc) * ((s_end - s_begin) * int64_t(u.nt) * kc * kTileN * 2 +
                                                a_blocks * int64_t(Rs) * kc * 2);
        const int64_t out = int64_t(nrows) * u.nt * kTileN * Rs * esz;
        weight.push_back(smem_in + out);
      }
    }
  }
  p->n_steps = static_cast<int64_t>(steps.size() / stride);
  if (steps.empty()) {  // keep a valid (never read) table
    steps.push_back(0);
    for (int k = 0; k < G; ++k) steps.push_back(-1);
  }

  // ---- CTA assignment ----
  int grid = o.max_ctas > 0 ? std::min(o.max_ctas, sm_count) : sm_count;
  grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(grid, units.size())));
  std::vector<std::vector<int32_t>> per;
  if (o.no_load_balance)
    contiguous_split(static_cast<int64_t>(units.size()), grid, &per);
  else
    serpentine_order(weight, grid, &per);
  p->h_units.clear();
  p->h_cta_begin.assign(1, 0);
  for (int c = 0; c < grid; ++c) {
    for (int32_t idx : per[c]) p->h_units.push_back(units[idx]);
    p->h_cta_begin.push_back(static_cast<int32_t>(p->h_units.size()));
  }
  p->n_units = static_cast<int64_t>(units.size());
  p->grid = grid;

  // ---- shared memory / TMEM ----
  int stage_bytes = NT * kc * 256 + G * Rs * kc * 2;
  stage_bytes = (stage_bytes + 1023) / 1024 * 1024;
  const int fixed = spmm_smem_bytes(0, stage_bytes, p->c_type == BSP_F32);
  int stages = (max_smem - fixed) / stage_bytes;
  stages = std::min(stages, 32);
  if (stages < 2)
    return set_error(BSP_ERR_UNSUPPORTED, "block too large: fewer than 2 pipeline stages fit");
  // Producer warps issue stages round-robin; each owns stage slots congruent
  // to it, so the ring length is a multiple of their number.
  int nprod = std::min(spmm_max_producers(), stages);
  if (o.producers > 0) nprod = std::min(nprod, o.producers);
  stages = stages / nprod * nprod;
  p->nprod = nprod;
  p->stage_bytes = stage_bytes;
  p->stages = stages;
  p->smem_bytes = spmm_smem_bytes(stages, stage_bytes, p->c_type == BSP_F32);
  p->tmem_cols = pow2_at_least(2 * NT * G * Rs);
  p->timeout_ns = static_cast<uint64_t>(o.timeout_ms > 0 ? o.timeout_ms : 2000) * 1000000ull;
  return BSP_OK;
}

// Row-stacked schedule (spmm_rowstack.cu).  An "entry" is an Rs-row slab of a
// block-row (Rs = 128, 64 or 32, the largest that divides R); G = 128 / Rs
// consecutive entries form the 128 rows of one MMA.  A unit is one entry group
// x 256 output columns; its steps are the distinct block-columns of the
// group's rows, each listing per entry the block to multiply (or -1).
// Split-K for the row-stacked kernels: a long unit is cut into parts over
// consecutive ranges of its steps; each part accumulates a partial tile, and
// the part that finishes last adds the others' partials (left in a workspace
// by them) and stores the tile.  parts[i] (1 = whole) for units of balancer
// weight weight[i] and nsteps[i] steps: several target part weights are
// tried (cut every unit above the target into parts of about that weight),
// and the cut whose serpentine deal has the shortest makespan is kept if it
// beats the uncut deal by 3%.  Each part is charged its partial's write plus
// the final sum's read of all n partials: the merge is bound by L2 round
// trips on the merging CTA's critical path, so parts are also capped at 8
// (16-part merges of config 5's longest rows cost more than they balanced;
// 8 parts leave one GPU's config 5 unchanged and shorten the slowest CTA of
// an 8-GPU row panel holding a 1000-block row by 16%).
static void ordered_greedy(const std::vector<int64_t>& weight, int parts,
                           std::vector<std::vector<int32_t>>* per_part);
// ordered: the units are dealt in their given order (ordered_greedy), the
// parts of a cut unit in its place; otherwise by the serpentine balancer.
static std::vector<int32_t> choose_splits(const std::vector<int64_t>& weight, const std::vector<int32_t>& nsteps,
                                          int ctas, int64_t partial_bytes, bool ordered = false) {
  constexpr int kMaxSplit = 8, kMinPartSteps = 4;
  const size_t n = weight.size();
  std::vector<int32_t> best(n, 1);
  if (n == 0 || ctas < 2) return best;
  auto makespan = [&](const std::vector<int32_t>& np) {
    std::vector<int64_t> items;
    for (size_t i = 0; i < n; ++i)
      for (int k = 0; k < np[i]; ++k) {
        const int64_t lo = int64_t(nsteps[i]) * k / np[i], hi = int64_t(nsteps[i]) * (k + 1) / np[i];
        items.push_back(np[i] == 1 ? weight[i]
                                   : weight[i] * (hi - lo) / std::max(1, nsteps[i]) + (1 + np[i]) * partial_bytes);
      }
    const int grid = static_cast<int>(std::min<int64_t>(ctas, static_cast<int64_t>(items.size())));
    std::vector<std::vector<int32_t>> per;
    if (ordered) ordered_greedy(items, grid, &per);
    else serpentine_order(items, grid, &per);
    int64_t worst = 0;
    for (const auto& v : per) {
      int64_t t = 0;
      for (int32_t idx : v) t += items[static_cast<size_t>(idx)];
      worst = std::max(worst, t);
    }
    return worst;
  };
  const int64_t base = makespan(best);
  int64_t best_m = base, total = 0;
  for (int64_t w : weight) total += w;
  std::vector<int32_t> cand(n);
  for (double f : {0.1, 0.15, 0.2, 0.3, 0.4, 0.5, 0.6, 0.75, 0.9, 1.0, 1.1, 1.25, 1.5, 2.0}) {
    const int64_t target = std::max<int64_t>(1, static_cast<int64_t>(static_cast<double>(total) / ctas * f));
    bool any = false;
    for (size_t i = 0; i < n; ++i) {
      cand[i] = 1;
      if (weight[i] > target && nsteps[i] >= 2 * kMinPartSteps) {
        const int64_t want = (weight[i] + target - 1) / target;
        cand[i] = static_cast<int32_t>(std::min<int64_t>({kMaxSplit, nsteps[i] / kMinPartSteps, want}));
        any |= cand[i] > 1;
      }
    }
    if (!any) continue;
    // no deal beats the mean load with the parts' added traffic: skip the
    // deal when even that bound cannot improve on the best so far
    int64_t added = 0;
    for (size_t i = 0; i < n; ++i)
      if (cand[i] > 1) added += int64_t(cand[i]) * (1 + cand[i]) * partial_bytes;
    if ((total + added) / ctas >= best_m) continue;
    const int64_t m = makespan(cand);
    if (m < best_m) {
      best_m = m;
      best = cand;
    }
  }
  // Equal-sized units leave the deal's last round part-filled (n mod ctas
  // units): halving only the m heaviest units, m = ctas * ceil(n / ctas) - n
  // (or one round more), makes the item count a multiple of the CTAs.
  {
    std::vector<int32_t> order(n);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) { return weight[a] > weight[b]; });
    const int64_t nn = static_cast<int64_t>(n);
    const int64_t m1 = (nn + ctas - 1) / ctas * ctas - nn;
    for (int64_t m : {m1, m1 + ctas}) {
      if (m <= 0 || m > nn) continue;
      std::fill(cand.begin(), cand.end(), 1);
      for (int64_t r = 0; r < m; ++r)
        if (nsteps[static_cast<size_t>(order[r])] >= 2 * kMinPartSteps) cand[static_cast<size_t>(order[r])] = 2;
      const int64_t m_span = makespan(cand);
      if (m_span < best_m) {
        best_m = m_span;
        best = cand;
      }
    }
  }
  if (best_m * 100 > base * 97) std::fill(best.begin(), best.end(), 1);
  return best;
}

bsp_status plan_spmm_rowstack(bsp_spmm_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                              int sm_count, int max_smem, const bsp_spmm_opts* opts, bool stage_lists) {
  bsp_spmm_opts o;
  memset(&o, 0, sizeof(o));
  if (opts) o = *opts;
  const int R = p->R, C = p->C;
  const int64_t nbr = p->M / R;
  const int Rs = (R % 128 == 0) ? 128 : (R % 64 == 0) ? 64 : 32;
  const int slabs = R / Rs;
  const int G = 128 / Rs;
  // Wide units (opts.n_tiles = 4, N a multiple of 512): 512 output columns
  // in one accumulator (all of TMEM, no double buffering), two N = 256 MMAs
  // per k-step, 32-deep k-chunks so that a stage (a 512-column B slice and the
  // entries' blocks) stays at 40 KB.  Each A block is then loaded once per 512
  // columns instead of once per 256.
  const bool wide = o.n_tiles == 4 && p->N % 512 == 0;
  const int kc = (C % 64 == 0 && !wide) ? 64 : 32;
  const int nkc = C / kc;
  const int64_t n_entries = nbr * slabs;
  // 256-column tiles (MMA N = 256); a B of at most 128 columns gets 128-column
  // tiles (MMA N = 128) instead of a 256-column box half out of range
  const int tile_n = wide ? 512 : p->N <= 128 ? 128 : 256;
  const int ntiles = static_cast<int>((p->N + tile_n - 1) / tile_n);
  if (n_entries >= (int64_t(1) << 31))
    return set_error(BSP_ERR_UNSUPPORTED, "too many block-rows");
  p->variant = 1;
  p->Rs = Rs;
  p->kc = kc;
  p->G = G;
  p->NT = tile_n / 128;  // 128-column tiles per unit
  p->stacked = 1;
  const int stride = 1 + G;
  p->step_stride = stride;
  std::vector<int32_t>& steps = p->h_steps;
  steps.clear();
  std::vector<SpmmUnit> units;
  std::vector<int64_t> weight;
  const int esz = p->c_type == BSP_F32 ? 4 : 2;
  std::vector<std::pair<int32_t, int32_t>> items;  // (col, g * 2^24-free: block id)
  std::vector<int8_t> item_g;
  // Stacking order.  The G block-rows of a unit step through the union of
  // their block-columns, so rows of very different lengths (power-law rows)
  // stacked together leave most slots of the long row's steps empty.  Rows
  // stacked by length (longest first) are kept when that shortens the total
  // of the unions by 5% or more.
  p->h_entry_rows.clear();
  if (slabs == 1 && G > 1 && nbr > G && !o.no_load_balance) {
    const int64_t nbc = p->K / C;
    std::vector<int64_t> stamp(static_cast<size_t>(nbc), -1);
    auto union_total = [&](const std::vector<int32_t>* order) {
      int64_t tot = 0;
      for (int64_t e0 = 0; e0 < nbr; e0 += G)
        for (int64_t e = e0; e < std::min<int64_t>(nbr, e0 + G); ++e) {
          const int64_t i = order ? (*order)[static_cast<size_t>(e)] : e;
          for (int32_t b = row_ptr[i]; b < row_ptr[i + 1]; ++b)
            if (stamp[static_cast<size_t>(col_idx[b])] != e0) {
              stamp[static_cast<size_t>(col_idx[b])] = e0;
              ++tot;
            }
        }
      return tot;
    };
    const int64_t t_id = union_total(nullptr);
    std::fill(stamp.begin(), stamp.end(), -1);
    std::vector<int32_t> by_len(static_cast<size_t>(nbr));
    std::iota(by_len.begin(), by_len.end(), 0);
    std::stable_sort(by_len.begin(), by_len.end(), [&](int32_t a, int32_t b) {
      return row_ptr[a + 1] - row_ptr[a] > row_ptr[b + 1] - row_ptr[b];
    });
    if (union_total(&by_len) * 100 <= t_id * 95) p->h_entry_rows.swap(by_len);
  }
  const std::vector<int32_t>& perm = p->h_entry_rows;
  for (int64_t e0 = 0; e0 < n_entries; e0 += G) {
    const int nent = static_cast<int>(std::min<int64_t>(G, n_entries - e0));
    const int32_t s_begin = static_cast<int32_t>(steps.size() / stride);
    int32_t mask = 0;
    items.clear();
    item_g.clear();
    for (int g = 0; g < nent; ++g) {
      const int64_t i = perm.empty() ? (e0 + g) / slabs : perm[static_cast<size_t>(e0 + g)];
      if (row_ptr[i + 1] > row_ptr[i]) mask |= 1 << g;
      for (int32_t b = row_ptr[i]; b < row_ptr[i + 1]; ++b) {
        items.push_back({col_idx[b], b});
        item_g.push_back(static_cast<int8_t>(g));
      }
    }
    std::vector<int32_t> order(items.size());
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(),
                     [&](int32_t a, int32_t b) { return items[a].first < items[b].first; });
    int64_t cur = -1;
    int64_t a_loads = 0;
    for (int32_t k : order) {
      const int g = item_g[k];
      const bool open = cur >= 0 && steps[cur * stride] == items[k].first &&
                        steps[cur * stride + 1 + g] < 0;
      if (!open) {
        cur = static_cast<int64_t>(steps.size() / stride);
        steps.push_back(items[k].first);
        for (int q = 0; q < G; ++q) steps.push_back(-1);
      }
      steps[cur * stride + 1 + g] = items[k].second;
      ++a_loads;
    }
    const int32_t s_end = static_cast<int32_t>(steps.size() / stride);
    for (int t = 0; t < ntiles; ++t) {
      SpmmUnit u;
      u.row0 = static_cast<int32_t>(e0);
      u.nrows = nent;
      u.r_off = 0;
      u.n0 = t * tile_n;
      u.nt = 1;
      u.step_begin = s_begin;
      u.step_end = s_end;
      u.row_mask = mask;
      units.push_back(u);
      const int64_t smem_in = int64_t(nkc) * ((s_end - s_begin) * int64_t(kc) * tile_n * 2 +
                                              a_loads * int64_t(Rs) * kc * 2);
      weight.push_back(smem_in + int64_t(nent) * Rs * tile_n * esz + 4096);
    }
  }
  p->n_steps = static_cast<int64_t>(steps.size() / stride);
  if (steps.empty()) {
    steps.push_back(0);
    for (int q = 0; q < G; ++q) steps.push_back(-1);
  }
  int grid = o.max_ctas > 0 ? std::min(o.max_ctas, sm_count) : sm_count;
  // When B does not fit in L2 (with room for A), the units run tile by tile:
  // units in column-tile-major order, each dealt to the least-loaded CTA in
  // that order, so all CTAs work on one B panel (K x tile_n) at a time and
  // it is read from DRAM about once instead of once per row group.
  const bool l2_order = !o.no_load_balance && ntiles > 1 && p->K * p->N * 2 > (int64_t(64) << 20);
  if (l2_order) {
    std::vector<int32_t> idx(units.size());
    std::iota(idx.begin(), idx.end(), 0);
    std::stable_sort(idx.begin(), idx.end(), [&](int32_t a, int32_t b) {
      if (units[a].n0 != units[b].n0) return units[a].n0 < units[b].n0;
      return units[a].row0 < units[b].row0;
    });
    std::vector<SpmmUnit> su(units.size());
    std::vector<int64_t> sw(units.size());
    for (size_t i = 0; i < idx.size(); ++i) {
      su[i] = units[static_cast<size_t>(idx[i])];
      sw[i] = weight[static_cast<size_t>(idx[i])];
    }
    units.swap(su);
    weight.swap(sw);
  }
  // split-K (not with the contiguous split; opts.group_rows = -1 turns it off)
  p->n_split_slots = 0;
  p->split_units = 0;
  if (!o.no_load_balance && o.group_rows != -1) {
    std::vector<int32_t> nst(units.size());
    for (size_t i = 0; i < units.size(); ++i) nst[i] = units[i].step_end - units[i].step_begin;
    const std::vector<int32_t> np = choose_splits(weight, nst, grid, int64_t(128) * tile_n * 4, l2_order);
    std::vector<SpmmUnit> su;
    std::vector<int64_t> sw;
    for (size_t i = 0; i < units.size(); ++i) {
      if (np[i] == 1) {
        su.push_back(units[i]);
        sw.push_back(weight[i]);
        continue;
      }
      for (int k = 0; k < np[i]; ++k) {
        SpmmUnit v = units[i];
        v.step_begin = units[i].step_begin + static_cast<int32_t>(int64_t(nst[i]) * k / np[i]);
        v.step_end = units[i].step_begin + static_cast<int32_t>(int64_t(nst[i]) * (k + 1) / np[i]);
        v.nt = np[i] | (k << 8);
        v.r_off = static_cast<int32_t>(p->n_split_slots);
        su.push_back(v);
        sw.push_back(weight[i] * (v.step_end - v.step_begin) / std::max(1, nst[i]) +
                     (1 + np[i]) * int64_t(128) * tile_n * 4);
      }
      p->n_split_slots += np[i];
      ++p->split_units;
    }
    units.swap(su);
    weight.swap(sw);
  }
  grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(grid, units.size())));
  std::vector<std::vector<int32_t>> per;
  if (o.no_load_balance)
    contiguous_split(static_cast<int64_t>(units.size()), grid, &per);
  else if (l2_order)
    ordered_greedy(weight, grid, &per);
  else
    serpentine_order(weight, grid, &per);
  p->h_units.clear();
  p->h_cta_begin.assign(1, 0);
  for (int c = 0; c < grid; ++c) {
    for (int32_t idx : per[c]) p->h_units.push_back(units[idx]);
    p->h_cta_begin.push_back(static_cast<int32_t>(p->h_units.size()));
  }
  p->n_units = static_cast<int64_t>(units.size());
  p->grid = grid;
  // With 32-wide blocks a step is only two MMAs, and one full/empty barrier
  // hand-off per stage costs about as long as two MMAs take.  A stage then
  // carries two consecutive steps so that each hand-off moves four MMAs:
  // on B200 that beats the deeper one-step ring at every density from 5%.
  int nsub = 1;
  if (kc == 32 && nkc == 1 && o.steps_per_stage != 1 && !wide) nsub = 2;
  const int sub_bytes = (tile_n / 64) * kc * 128 + G * Rs * kc * 2;
  p->sub_bytes = sub_bytes;
  p->nsub = nsub;
  int stage_bytes = nsub * sub_bytes;
  stage_bytes = (stage_bytes + 1023) / 1024 * 1024;
  const int max_stages = std::min(rowstack_max_stages(), (max_smem - 2048) / stage_bytes);
  if (max_stages < 2) return set_error(BSP_ERR_UNSUPPORTED, "block too large for the pipeline");
  // Each producer warp owns the ring slots congruent to it, so the ring length
  // is a multiple of the producer count: pick the count that keeps the most
  // stages (ties: more producers).
  int nprod = 1, stages = max_stages;
  if (o.producers > 0) {
    nprod = std::min({o.producers, rowstack_max_producers(), max_stages});
    stages = max_stages / nprod * nprod;
  } else {
    for (int q = 2; q <= std::min(rowstack_max_producers(), max_stages); ++q) {
      const int sq = max_stages / q * q;
      if (sq >= stages - (stages > 6 ? 1 : 0)) {  // accept losing one stage of a deep ring
        nprod = q;
        stages = sq;
      }
    }
  }
  p->nprod = nprod;
  p->stage_bytes = stage_bytes;
  p->stages = stages;
  p->smem_bytes = 2048 + stages * stage_bytes;
  // A 16 KiB staging area through which the epilogue stores C (and its peer
  // copies) as whole 128-byte lines, when it fits beside the ring without
  // costing a stage.
  p->xfer_off = 0;
  if (p->smem_bytes + 16384 <= max_smem) {
    p->xfer_off = 1024 + stages * stage_bytes;
    p->smem_bytes += 16384;
  }
  p->tmem_cols = wide ? 512 : 2 * tile_n;
  p->n_acc = wide ? 1 : 2;
  p->timeout_ns = static_cast<uint64_t>(o.timeout_ms > 0 ? o.timeout_ms : 2000) * 1000000ull;

  bsp_status st = spmm_stage_counts(p);
  if (st != BSP_OK || !stage_lists) return st;
  return rowstack_stage_lists(p);
}

// Row-stacked schedule for CTA pairs (2-SM MMA, spmm_pair.cu).  A pair unit
// is 2G entries (256 output rows) x 256 columns; CTA rank r of the pair holds
// entries r*G .. r*G+G-1 (its 128 TMEM lanes) and loads B columns
// n0 + 128 r .. +127.  Every entry slot is loaded at every step: an absent
// block comes from a TMA box entirely above the A tensor (y = -Rs), which
// the TMA fills with zeros, so each stage moves a fixed number of bytes and
// no slot ever needs clearing.  Units and stage lists are per CTA (the two
// CTAs of a pair walk the same stage sequence with their own coordinates).
bsp_status plan_spmm_pair(bsp_spmm_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                          int sm_count, int max_smem, const bsp_spmm_opts* opts, bool stage_lists) {
  bsp_spmm_opts o;
  memset(&o, 0, sizeof(o));
  if (opts) o = *opts;
  const int R = p->R, C = p->C;
  const int64_t nbr = p->M / R;
  const int Rs = (R % 128 == 0) ? 128 : (R % 64 == 0) ? 64 : 32;
  const int slabs = R / Rs;
  const int G = 128 / Rs;  // entries per CTA
  const int G2 = 2 * G;    // entries per pair unit
  const int kc = (C % 64 == 0) ? 64 : 32;
  const int nkc = C / kc;
  const int64_t n_entries = nbr * slabs;
  const int ntiles = static_cast<int>((p->N + 255) / 256);
  if (n_entries >= (int64_t(1) << 31)) return set_error(BSP_ERR_UNSUPPORTED, "too many block-rows");
  p->variant = 2;
  p->Rs = Rs;
  p->kc = kc;
  p->G = G;
  p->NT = 2;
  p->stacked = 1;
  const int stride = 1 + G2;
  p->step_stride = stride;
  std::vector<int32_t>& steps = p->h_steps;
  steps.clear();
  struct PairUnit {
    int64_t e0;
    int nent;
    int32_t s_begin, s_end, n0;
    int32_t mask;  // present entries (bit g of the 2G)
    int32_t np = 1, part = 0, slot0 = 0;  // split-K: part of np; rank r's slots start at slot0 + r * np
  };
  std::vector<PairUnit> units;
  std::vector<int64_t> weight;
  const int esz = p->c_type == BSP_F32 ? 4 : 2;
  std::vector<std::pair<int32_t, int32_t>> items;
  std::vector<int8_t> item_g;
  for (int64_t e0 = 0; e0 < n_entries; e0 += G2) {
    const int nent = static_cast<int>(std::min<int64_t>(G2, n_entries - e0));
    const int32_t s_begin = static_cast<int32_t>(steps.size() / stride);
    int32_t mask = 0;
    items.clear();
    item_g.clear();
    for (int g = 0; g < nent; ++g) {
      const int64_t i = (e0 + g) / slabs;
      if (row_ptr[i + 1] > row_ptr[i]) mask |= 1 << g;
      for (int32_t b = row_ptr[i]; b < row_ptr[i + 1]; ++b) {
        items.push_back({col_idx[b], b});
        item_g.push_back(static_cast<int8_t>(g));
      }
    }
    std::vector<int32_t> order(items.size());
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(),
                     [&](int32_t a, int32_t b) { return items[a].first < items[b].first; });
    int64_t cur = -1;
    for (int32_t k : order) {
      const int g = item_g[k];
      const bool open = cur >= 0 && steps[cur * stride] == items[k].first && steps[cur * stride + 1 + g] < 0;
      if (!open) {
        cur = static_cast<int64_t>(steps.size() / stride);
        steps.push_back(items[k].first);
        for (int q = 0; q < G2; ++q) steps.push_back(-1);
      }
      steps[cur * stride + 1 + g] = items[k].second;
    }
    const int32_t s_end = static_cast<int32_t>(steps.size() / stride);
    for (int t = 0; t < ntiles; ++t) {
      units.push_back({e0, nent, s_begin, s_end, t * 256, mask, 1, 0, 0});
      // bytes staged per CTA: B half + all entry slots per step, plus its C rows
      weight.push_back(int64_t(s_end - s_begin) * nkc * (int64_t(kc) * 128 * 2 + int64_t(G) * Rs * kc * 2) +
                       int64_t(G) * Rs * 256 * esz + 4096);
    }
  }
  p->n_steps = static_cast<int64_t>(steps.size() / stride);
  int npairs = (o.max_ctas > 0 ? std::min(o.max_ctas, sm_count) : sm_count) / 2;
  // B larger than L2: pair units run tile by tile (see plan_spmm_rowstack)
  const bool l2_order = !o.no_load_balance && ntiles > 1 && p->K * p->N * 2 > (int64_t(64) << 20);
  if (l2_order) {
    std::stable_sort(units.begin(), units.end(), [](const PairUnit& a, const PairUnit& b) { return a.n0 < b.n0; });
    // weights follow the units: recompute them in the new order
    weight.clear();
    for (const PairUnit& u : units)
      weight.push_back(int64_t(u.s_end - u.s_begin) * nkc * (int64_t(kc) * 128 * 2 + int64_t(G) * Rs * kc * 2) +
                       int64_t(G) * Rs * 256 * esz + 4096);
  }
  // split-K over pair units (each rank keeps its own partial tile)
  p->n_split_slots = 0;
  p->split_units = 0;
  if (!o.no_load_balance && o.group_rows != -1) {
    std::vector<int32_t> nst(units.size());
    for (size_t i = 0; i < units.size(); ++i) nst[i] = units[i].s_end - units[i].s_begin;
    const std::vector<int32_t> np = choose_splits(weight, nst, npairs, int64_t(128) * 256 * 4, l2_order);
    std::vector<PairUnit> su;
    std::vector<int64_t> sw;
    for (size_t i = 0; i < units.size(); ++i) {
      if (np[i] == 1) {
        su.push_back(units[i]);
        sw.push_back(weight[i]);
        continue;
      }
      for (int k = 0; k < np[i]; ++k) {
        PairUnit v = units[i];
        v.s_begin = units[i].s_begin + static_cast<int32_t>(int64_t(nst[i]) * k / np[i]);
        v.s_end = units[i].s_begin + static_cast<int32_t>(int64_t(nst[i]) * (k + 1) / np[i]);
        v.np = np[i];
        v.part = k;
        v.slot0 = static_cast<int32_t>(p->n_split_slots);
        su.push_back(v);
        sw.push_back(weight[i] * (v.s_end - v.s_begin) / std::max(1, nst[i]) + (1 + np[i]) * int64_t(128) * 256 * 4);
      }
      p->n_split_slots += 2 * np[i];
      ++p->split_units;
    }
    units.swap(su);
    weight.swap(sw);
  }
  npairs = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(npairs, units.size())));
  std::vector<std::vector<int32_t>> per;
  if (o.no_load_balance)
    contiguous_split(static_cast<int64_t>(units.size()), npairs, &per);
  else if (l2_order)
    ordered_greedy(weight, npairs, &per);
  else
    serpentine_order(weight, npairs, &per);

  // stages: nsub consecutive (step, k-chunk) items per stage, as in the
  // single-CTA kernel (two 32-wide block-columns = 4 MMAs per hand-off)
  int nsub = 1;
  if (kc == 32 && nkc == 1 && o.steps_per_stage != 1) nsub = 2;
  const int b_half = 2 * kc * 128;               // two 64-column boxes
  const int sub_bytes = b_half + G * Rs * kc * 2;
  p->sub_bytes = sub_bytes;
  p->nsub = nsub;
  int stage_bytes = nsub * sub_bytes;
  stage_bytes = (stage_bytes + 1023) / 1024 * 1024;
  const int max_stages = std::min(rowstack_max_stages(), (max_smem - 2048 - 16384) / stage_bytes);
  if (max_stages < 2) return set_error(BSP_ERR_UNSUPPORTED, "block too large for the pipeline");
  int nprod = 1, stages = max_stages;
  if (o.producers > 0) {
    nprod = std::min({o.producers, rowstack_max_producers(), max_stages});
    stages = max_stages / nprod * nprod;
  } else {
    for (int q = 2; q <= std::min(rowstack_max_producers(), max_stages); ++q) {
      const int sq = max_stages / q * q;
      if (sq >= stages - (stages > 6 ? 1 : 0)) {
        nprod = q;
        stages = sq;
      }
    }
  }
  p->nprod = nprod;
  p->stage_bytes = stage_bytes;
  p->stages = stages;
  p->xfer_off = 1024 + stages * stage_bytes;  // staging area of the C stores
  p->smem_bytes = 2048 + stages * stage_bytes + 16384;
  p->tmem_cols = 512;
  p->timeout_ns = static_cast<uint64_t>(o.timeout_ms > 0 ? o.timeout_ms : 2000) * 1000000ull;
  p->grid = 2 * npairs;

  // per-CTA units (CTA 2c + r = rank r of pair c); both CTAs of a pair walk
  // the same step sequence, each with its own entries and B half
  p->h_units.clear();
  p->h_cta_begin.assign(1, 0);
  for (int c = 0; c < npairs; ++c) {
    for (int r = 0; r < 2; ++r) {
      for (int32_t idx : per[c]) {
        const PairUnit& pu = units[idx];
        SpmmUnit u;
        u.row0 = static_cast<int32_t>(pu.e0 + r * G);
        u.nrows = std::max(0, std::min(G, pu.nent - r * G));
        u.r_off = pu.np > 1 ? pu.slot0 + r * pu.np : 0;
        u.n0 = pu.n0;
        u.nt = pu.np | (pu.part << 8);
        u.step_begin = pu.s_begin;
        u.step_end = pu.s_end;
        u.row_mask = (pu.mask >> (r * G)) & ((1 << G) - 1);
        p->h_units.push_back(u);
      }
      p->h_cta_begin.push_back(static_cast<int32_t>(p->h_units.size()));
    }
  }
  if (steps.empty()) {
    steps.push_back(0);
    for (int q = 0; q < G2; ++q) steps.push_back(-1);
  }
  // one unit record per CTA of each pair unit
  p->n_units = static_cast<int64_t>(p->h_units.size());
  bsp_status st = spmm_stage_counts(p);
  if (st != BSP_OK || !stage_lists) return st;
  return pair_stage_lists(p);
}

// Stages in each CTA's list (row-stacked and pair schedules): a unit without
// blocks takes one empty stage, the others ceil(steps * k-chunks / nsub).
static bsp_status spmm_stage_counts(bsp_spmm_plan* p) {
  const int nkc = p->C / p->kc;
  p->h_cta_stage_begin.assign(1, 0);
  p->h_stage_list.clear();
  int64_t total = 0;
  for (size_t c = 0; c + 1 < p->h_cta_begin.size(); ++c) {
    for (int32_t ui = p->h_cta_begin[c]; ui < p->h_cta_begin[c + 1]; ++ui) {
      const int64_t n = static_cast<int64_t>(p->h_units[ui].step_end - p->h_units[ui].step_begin) * nkc;
      total += n == 0 ? 1 : (n + p->nsub - 1) / p->nsub;
    }
    if (total >= (int64_t(1) << 31)) return set_error(BSP_ERR_UNSUPPORTED, "schedule too long");
    p->h_cta_stage_begin.push_back(static_cast<int32_t>(total));
  }
  return BSP_OK;
}

// The row-stacked kernel's per-CTA stage lists, CTAs split over host threads
// (each CTA's list depends only on its own units).  The kernel's smem ring is
// in lockstep with each CTA's stage sequence (stage k uses slot k % stages),
// so the host can tell exactly which entry slots still hold an older block
// and must be zeroed before a stage where that entry is absent.
static bsp_status rowstack_stage_lists(bsp_spmm_plan* p) {
  const int W = kRsStageWords;
  const int G = p->G, Rs = p->Rs, R = p->R, C = p->C, kc = p->kc, nkc = C / kc, slabs = R / Rs;
  const int nsub = p->nsub, stages = p->stages, stride = p->step_stride;
  const bool b3d = (p->N % 64 == 0);
  const uint32_t all = (1u << G) - 1u;
  const int64_t grid = static_cast<int64_t>(p->h_cta_begin.size()) - 1;
  p->h_stage_list.resize(static_cast<size_t>(p->h_cta_stage_begin.back()) * W);
  const std::vector<int32_t>& steps = p->h_steps;
  // a thread pays for itself from a few thousand stages on
  const int64_t nst = p->h_cta_stage_begin.back();
  return parallel_ranges(grid, planner_threads(std::min<int64_t>(grid, nst / 4096), 1, 0), [&](int, int64_t c0, int64_t c1) {
    std::vector<uint32_t> dirty(static_cast<size_t>(stages) * nsub);  // per (slot, sub-step)
    for (int64_t c = c0; c < c1; ++c) {
      int32_t* out = p->h_stage_list.data() + static_cast<size_t>(p->h_cta_stage_begin[c]) * W;
      std::fill(dirty.begin(), dirty.end(), all);  // unknown contents until first written
      int64_t k = 0;
      for (int32_t ui = p->h_cta_begin[c]; ui < p->h_cta_begin[c + 1]; ++ui) {
        const SpmmUnit& u = p->h_units[ui];
        const int nsteps = u.step_end - u.step_begin;
        if (nsteps == 0) {
          int32_t e[kRsStageWords] = {RS_F_FIRST | RS_F_LAST | RS_F_EMPTY};
          memcpy(out, e, sizeof(e));
          out += W;
          ++k;
          continue;
        }
        int slab_off[4] = {0, 0, 0, 0};
        for (int g = 0; g < G; ++g) slab_off[g] = static_cast<int>((u.row0 + g) % slabs) * Rs;
        // the unit's (step, k-chunk) sequence, nsub of them per stage
        const int nitems = nsteps * nkc;
        for (int s0 = 0; s0 < nitems; s0 += nsub) {
          const int nin = std::min(nsub, nitems - s0);
          int32_t e[kRsStageWords];
          for (int q = 0; q < W; ++q) e[q] = (q >= 5 && q <= 12) ? -1 : 0;
          uint32_t flags = 0, np = 0;
          const int slot = static_cast<int>(k % stages);
          for (int sub = 0; sub < nin; ++sub) {
            const int s_ = s0 + sub;
            const int j = s_ / nkc, kci = s_ % nkc;
            const int32_t* st = &steps[static_cast<size_t>(u.step_begin + j) * stride];
            uint32_t present = 0;
            for (int g = 0; g < G; ++g)
              if (g < u.nrows && st[1 + g] >= 0) {
                present |= 1u << g;
                ++np;
                e[5 + 4 * sub + g] = st[1 + g] * R + slab_off[g];
              }
            uint32_t& d = dirty[static_cast<size_t>(slot) * nsub + sub];
            const uint32_t zero = ~present & all & d;
            d = present;
            flags |= (present << (4 * sub)) | (zero << (8 + 4 * sub));
            e[3 + sub] = st[0] * C + kci * kc;
            e[2] = kci * kc;  // a stage never mixes k-chunks when nsub == 2 (nkc == 1)
          }
          flags |= np << 16;
          if (s0 == 0) flags |= RS_F_FIRST;
          if (s0 + nin >= nitems) flags |= RS_F_LAST;
          if (nin == 2) flags |= RS_F_TWO;
          e[0] = static_cast<int32_t>(flags);
          e[1] = b3d ? u.n0 / 64 : u.n0;
          memcpy(out, e, sizeof(e));
          out += W;
          ++k;
        }
      }
    }
    return BSP_OK;
  });
}

// The CTA-pair kernel's per-CTA stage lists (CTA 2c + r = rank r of pair c),
// built a pair at a time over host threads.  The host replays each CTA's smem
// ring: a slot is loaded when its entry has a block in the sub-step, or when
// it is absent but still holds an older block (then from a box above the A
// tensor, which the TMA fills with zeros); absent slots that are already zero
// are not touched.  So every shared-memory write stays a TMA write.  Flags
// bits 0..7 mark the slots to load.  Both CTAs' copies complete on the
// leader's full barrier, so the leader's descriptor carries the pair's count
// of loaded slots (bits 16..20), from which it arms the barrier.
static bsp_status pair_stage_lists(bsp_spmm_plan* p) {
  const int W = kRsStageWords;
  const int G = p->G, Rs = p->Rs, R = p->R, C = p->C, kc = p->kc, nkc = C / kc, slabs = R / Rs;
  const int nsub = p->nsub, stride = p->step_stride, stages = p->stages;
  const bool b3d = (p->N % 64 == 0);
  const uint32_t all = (1u << G) - 1u;
  const int64_t npairs = (static_cast<int64_t>(p->h_cta_begin.size()) - 1) / 2;
  p->h_stage_list.resize(static_cast<size_t>(p->h_cta_stage_begin.back()) * W);
  const std::vector<int32_t>& steps = p->h_steps;
  // a thread pays for itself from a few thousand stages on
  const int64_t nst = p->h_cta_stage_begin.back();
  return parallel_ranges(npairs, planner_threads(std::min<int64_t>(npairs, nst / 4096), 1, 0),
                         [&](int, int64_t c0, int64_t c1) {
    std::vector<uint32_t> dirty(static_cast<size_t>(stages) * nsub);  // per (slot, sub-step)
    for (int64_t pc = c0; pc < c1; ++pc) {
      for (int r = 0; r < 2; ++r) {
        const int64_t cta = 2 * pc + r;
        int32_t* out = p->h_stage_list.data() + static_cast<size_t>(p->h_cta_stage_begin[cta]) * W;
        std::fill(dirty.begin(), dirty.end(), all);  // unknown contents until first written
        int64_t k = 0;
        for (int32_t ui = p->h_cta_begin[cta]; ui < p->h_cta_begin[cta + 1]; ++ui) {
          const SpmmUnit& u = p->h_units[ui];
          const int nsteps = u.step_end - u.step_begin;
          if (nsteps == 0) {
            int32_t e[kRsStageWords] = {RS_F_FIRST | RS_F_LAST | RS_F_EMPTY};
            memcpy(out, e, sizeof(e));
            out += W;
            ++k;
            continue;
          }
          int slab_off[4] = {0, 0, 0, 0};
          for (int g = 0; g < G; ++g) slab_off[g] = static_cast<int>((u.row0 + g) % slabs) * Rs;
          const int nitems = nsteps * nkc;
          for (int s0 = 0; s0 < nitems; s0 += nsub) {
            const int nin = std::min(nsub, nitems - s0);
            int32_t e[kRsStageWords];
            for (int q = 0; q < W; ++q) e[q] = (q >= 5 && q <= 12) ? -1 : 0;
            uint32_t flags = 0;
            const int slot = static_cast<int>(k % stages);
            for (int sub = 0; sub < nin; ++sub) {
              const int s_ = s0 + sub;
              const int j = s_ / nkc, kci = s_ % nkc;
              const int32_t* st = &steps[static_cast<size_t>(u.step_begin + j) * stride];
              uint32_t present = 0;
              for (int g = 0; g < G; ++g) {
                const int gg = r * G + g;
                if (g < u.nrows && st[1 + gg] >= 0) {
                  present |= 1u << g;
                  e[5 + 4 * sub + g] = st[1 + gg] * R + slab_off[g];
                }
              }
              uint32_t& d = dirty[static_cast<size_t>(slot) * nsub + sub];
              const uint32_t stale = ~present & all & d;  // zero-filled by a box above the tensor
              for (int g = 0; g < G; ++g)
                if ((stale >> g) & 1u) e[5 + 4 * sub + g] = -Rs;
              d = present;
              flags |= (present | stale) << (4 * sub);
              e[3 + sub] = st[0] * C + kci * kc;
              e[2] = kci * kc;
            }
            if (s0 == 0) flags |= RS_F_FIRST;
            if (s0 + nin >= nitems) flags |= RS_F_LAST;
            if (nin == 2) flags |= RS_F_TWO;
            e[0] = static_cast<int32_t>(flags);
            e[1] = b3d ? u.n0 / 64 + 2 * r : u.n0 + 128 * r;
            memcpy(out, e, sizeof(e));
            out += W;
            ++k;
          }
        }
      }
      // the leader's descriptors carry the pair's count of loaded slots
      int32_t* lead = p->h_stage_list.data() + static_cast<size_t>(p->h_cta_stage_begin[2 * pc]) * W;
      const int32_t* peer = p->h_stage_list.data() + static_cast<size_t>(p->h_cta_stage_begin[2 * pc + 1]) * W;
      const int64_t n_lead = p->h_cta_stage_begin[2 * pc + 1] - p->h_cta_stage_begin[2 * pc];
      const int64_t n_peer = p->h_cta_stage_begin[2 * pc + 2] - p->h_cta_stage_begin[2 * pc + 1];
      if (n_lead != n_peer) return set_error(BSP_ERR_STATE, "pair stage lists differ in length");
      for (int64_t i = 0; i < n_lead; ++i) {
        const uint32_t fl = static_cast<uint32_t>(lead[i * W]), fp = static_cast<uint32_t>(peer[i * W]);
        const uint32_t np = static_cast<uint32_t>(__builtin_popcount(fl & 0xFFu) + __builtin_popcount(fp & 0xFFu));
        lead[i * W] = static_cast<int32_t>(fl | (np << 16));
      }
    }
    return BSP_OK;
  });
}

// ---- twin units on CTA pairs (variant 3) -------------------------------------
bool spmm_twin_eligible(const bsp_spmm_plan* p) { return p->C == 32 && p->R % 32 == 0 && p->N > 128; }

// Two pair units (row groups g and g + 1 of 8 entries, the same 256-column
// tile) run as one work item on a CTA pair: their steps are the union of
// their columns, each B slice is loaded once for both, and each unit keeps
// its own accumulator (TMEM columns 0-255 and 256-511 of both CTAs).  A unit
// multiplies only at the columns where one of its entries holds a block; its
// absent entries of such a column are zero boxes.  Items are dealt longest
// first to the least-loaded pair.
bsp_status plan_spmm_twin(bsp_spmm_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                          int sm_count, int max_smem, const bsp_spmm_opts* opts, bool stage_lists) {
  bsp_spmm_opts o;
  memset(&o, 0, sizeof(o));
  if (opts) o = *opts;
  const int R = p->R, Rs = 32, slabs = R / 32, G = 4, G2 = 8;
  const int64_t nbr = p->M / R;
  const int64_t n_entries = nbr * slabs;
  const int ntiles = static_cast<int>((p->N + 255) / 256);
  if (n_entries >= (int64_t(1) << 31)) return set_error(BSP_ERR_UNSUPPORTED, "too many block-rows");
  p->variant = 3;
  p->Rs = Rs;
  p->kc = 32;
  p->G = G;
  p->NT = 2;
  p->stacked = 1;
  p->nsub = 1;
  const int stride = 1 + 2 * G2;  // column, then the block of each of the 16 entries (or -1)
  p->step_stride = stride;
  p->n_split_slots = 0;
  p->split_units = 0;
  std::vector<int32_t>& steps = p->h_steps;
  steps.clear();
  struct Twin {
    int64_t e0;      // first entry of unit a (unit b: e0 + 8)
    int nent_a, nent_b;
    int32_t s_begin, s_end, n0;
    int32_t mask;    // present entries: bits 0-7 unit a, 8-15 unit b
  };
  std::vector<Twin> twins;
  std::vector<int64_t> weight;
  const int esz = p->c_type == BSP_F32 ? 4 : 2;
  std::vector<std::pair<int32_t, int32_t>> items;
  std::vector<int8_t> item_g;
  for (int64_t e0 = 0; e0 < n_entries; e0 += 2 * G2) {
    const int nent = static_cast<int>(std::min<int64_t>(2 * G2, n_entries - e0));
    const int32_t s_begin = static_cast<int32_t>(steps.size() / stride);
    int32_t mask = 0;
    int64_t mmas = 0;
    items.clear();
    item_g.clear();
    for (int g = 0; g < nent; ++g) {
      const int64_t i = (e0 + g) / slabs;
      if (row_ptr[i + 1] > row_ptr[i]) mask |= 1 << g;
      for (int32_t b = row_ptr[i]; b < row_ptr[i + 1]; ++b) {
        items.push_back({col_idx[b], b});
        item_g.push_back(static_cast<int8_t>(g));
      }
    }
    std::vector<int32_t> order(items.size());
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(),
                     [&](int32_t a, int32_t b) { return items[a].first < items[b].first; });
    int64_t cur = -1;
    for (int32_t k : order) {
      const int g = item_g[k];
      // a column repeated in a row of an entry opens a further step
      const bool open = cur >= 0 && steps[cur * stride] == items[k].first && steps[cur * stride + 1 + g] < 0;
      if (!open) {
        cur = static_cast<int64_t>(steps.size() / stride);
        steps.push_back(items[k].first);
        for (int q = 0; q < 2 * G2; ++q) steps.push_back(-1);
      }
      steps[cur * stride + 1 + g] = items[k].second;
    }
    const int32_t s_end = static_cast<int32_t>(steps.size() / stride);
    for (int32_t s = s_begin; s < s_end; ++s) {
      bool ua = false, ub = false;
      for (int g = 0; g < G2; ++g) ua |= steps[static_cast<size_t>(s) * stride + 1 + g] >= 0;
      for (int g = G2; g < 2 * G2; ++g) ub |= steps[static_cast<size_t>(s) * stride + 1 + g] >= 0;
      mmas += (ua ? 1 : 0) + (ub ? 1 : 0);
    }
    for (int t = 0; t < ntiles; ++t) {
      twins.push_back({e0, std::min(nent, G2), std::max(0, nent - G2), s_begin, s_end, t * 256, mask});
      // per step: both units' MMAs (~2 x 156 cycles each) vs the stage's
      // staging; per item: two 128 x 256 tiles of C per CTA
      weight.push_back(mmas * 2 * 32 * 128 * 2 + int64_t(s_end - s_begin) * 8192 + 2 * int64_t(G) * Rs * 256 * esz +
                       8192);
    }
  }
  p->n_steps = static_cast<int64_t>(steps.size() / stride);
  int npairs = (o.max_ctas > 0 ? std::min(o.max_ctas, sm_count) : sm_count) / 2;
  // split-K over twins (both units' partials meet in the plan's workspace):
  // parts of consecutive union steps, kept only when they shorten the deal
  struct TwinPart {
    int32_t twin, part, np;
    int32_t s_begin, s_end;
    int32_t slot0;  // unit a's slots (rank r: slot0 + r * np), unit b's follow at slot0 + 2 * np
  };
  std::vector<TwinPart> parts;
  std::vector<int64_t> pw;
  {
    std::vector<int32_t> nst(twins.size());
    for (size_t i = 0; i < twins.size(); ++i) nst[i] = twins[i].s_end - twins[i].s_begin;
    std::vector<int32_t> np(twins.size(), 1);
    if (!o.no_load_balance && o.group_rows != -1)
      np = choose_splits(weight, nst, std::max(1, npairs), 2 * int64_t(128) * 256 * 4);
    for (size_t i = 0; i < twins.size(); ++i) {
      int32_t slot0 = 0;
      if (np[i] > 1) {
        slot0 = static_cast<int32_t>(p->n_split_slots);
        p->n_split_slots += 4 * np[i];
        ++p->split_units;
      }
      for (int k = 0; k < np[i]; ++k) {
        const int32_t lo = twins[i].s_begin + static_cast<int32_t>(int64_t(nst[i]) * k / np[i]);
        const int32_t hi = twins[i].s_begin + static_cast<int32_t>(int64_t(nst[i]) * (k + 1) / np[i]);
        parts.push_back({static_cast<int32_t>(i), k, np[i], lo, hi, slot0});
        pw.push_back(np[i] == 1 ? weight[i]
                                : weight[i] * (hi - lo) / std::max(1, nst[i]) + (1 + np[i]) * 2 * int64_t(128) * 256 * 4);
      }
    }
  }
  npairs = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(npairs, parts.size())));
  std::vector<std::vector<int32_t>> per;
  if (o.no_load_balance)
    contiguous_split(static_cast<int64_t>(parts.size()), npairs, &per);
  else
    serpentine_order(pw, npairs, &per);
  // ring: one block-column per stage, B half (8 KB) + 8 entry slots (2 KB each)
  const int a_slot = Rs * 32 * 2;
  const int stage_bytes = 2 * 32 * 128 + G2 * a_slot;
  p->sub_bytes = stage_bytes;
  const int max_stages = std::min(rowstack_max_stages(), (max_smem - 2048 - 16384) / stage_bytes);
  if (max_stages < 2) return set_error(BSP_ERR_UNSUPPORTED, "twin stages do not fit in shared memory");
  int nprod = 1, stages = max_stages;
  if (o.producers > 0) {
    nprod = std::min({o.producers, rowstack_max_producers(), max_stages});
    stages = max_stages / nprod * nprod;
  } else {
    for (int q = 2; q <= std::min(rowstack_max_producers(), max_stages); ++q) {
      const int sq = max_stages / q * q;
      if (sq >= stages - (stages > 6 ? 1 : 0)) {
        nprod = q;
        stages = sq;
      }
    }
  }
  p->nprod = nprod;
  p->stage_bytes = stage_bytes;
  p->stages = stages;
  p->xfer_off = 1024 + stages * stage_bytes;  // staging area of the C stores
  p->smem_bytes = 2048 + stages * stage_bytes + 16384;
  p->tmem_cols = 512;
  p->timeout_ns = static_cast<uint64_t>(o.timeout_ms > 0 ? o.timeout_ms : 2000) * 1000000ull;
  p->grid = 2 * npairs;
  // per CTA: the unit records of its twins in order, unit a then unit b (the
  // epilogue alternates accumulators 0 / 1 with them); both carry the twin's
  // step range
  p->h_units.clear();
  p->h_cta_begin.assign(1, 0);
  for (int c = 0; c < npairs; ++c) {
    for (int r = 0; r < 2; ++r) {
      for (int32_t idx : per[c]) {
        const TwinPart& tp = parts[static_cast<size_t>(idx)];
        const Twin& tw = twins[static_cast<size_t>(tp.twin)];
        for (int x = 0; x < 2; ++x) {
          const int nent = x ? tw.nent_b : tw.nent_a;
          // does unit x multiply anywhere in this part (pair-wide)?
          bool acc = false;
          for (int32_t s = tp.s_begin; s < tp.s_end && !acc; ++s)
            for (int g = 0; g < G2; ++g) acc |= steps[static_cast<size_t>(s) * stride + 1 + x * G2 + g] >= 0;
          SpmmUnit u;
          u.row0 = static_cast<int32_t>(tw.e0 + x * G2 + r * G);
          u.nrows = std::max(0, std::min(G, nent - r * G));
          u.r_off = tp.np > 1 ? tp.slot0 + x * 2 * tp.np + r * tp.np : 0;
          u.n0 = tw.n0;
          u.nt = tp.np | (tp.part << 8) | (tp.np > 1 && !acc ? kUnitNoAcc : 0);
          u.step_begin = tp.s_begin;
          u.step_end = tp.s_end;
          u.row_mask = (tw.mask >> (x * G2 + r * G)) & ((1 << G) - 1);
          p->h_units.push_back(u);
        }
      }
      p->h_cta_begin.push_back(static_cast<int32_t>(p->h_units.size()));
    }
  }
  if (steps.empty()) {
    steps.push_back(0);
    for (int q = 0; q < 2 * G2; ++q) steps.push_back(-1);
  }
  p->n_units = static_cast<int64_t>(p->h_units.size());
  // stage counts: one stage per union step of each twin (one for an empty twin)
  p->h_cta_stage_begin.assign(1, 0);
  p->h_stage_list.clear();
  int64_t total = 0;
  for (size_t c = 0; c + 1 < p->h_cta_begin.size(); ++c) {
    for (int32_t ui = p->h_cta_begin[c]; ui < p->h_cta_begin[c + 1]; ui += 2) {
      const int64_t n = p->h_units[ui].step_end - p->h_units[ui].step_begin;
      total += n == 0 ? 1 : n;
    }
    if (total >= (int64_t(1) << 31)) return set_error(BSP_ERR_UNSUPPORTED, "schedule too long");
    p->h_cta_stage_begin.push_back(static_cast<int32_t>(total));
  }
  if (!stage_lists) return BSP_OK;
  const int W = kRsStageWords;
  const bool b3d = (p->N % 64 == 0);
  const int64_t grid = static_cast<int64_t>(p->h_cta_begin.size()) - 1;
  p->h_stage_list.resize(static_cast<size_t>(p->h_cta_stage_begin.back()) * W);
  // a thread pays for itself from a few thousand stages on
  const int64_t nst = p->h_cta_stage_begin.back();
  return parallel_ranges(grid, planner_threads(std::min<int64_t>(grid, nst / 4096), 1, 0), [&](int, int64_t c0, int64_t c1) {
    for (int64_t cta = c0; cta < c1; ++cta) {
      const int r = static_cast<int>(cta % 2);
      int32_t* out = p->h_stage_list.data() + static_cast<size_t>(p->h_cta_stage_begin[cta]) * W;
      for (int32_t ui = p->h_cta_begin[cta]; ui < p->h_cta_begin[cta + 1]; ui += 2) {
        const SpmmUnit& ua = p->h_units[ui];
        const int nsteps = ua.step_end - ua.step_begin;
        const int32_t bz = b3d ? ua.n0 / 64 + 2 * r : ua.n0 + 128 * r;
        if (nsteps == 0) {
          int32_t e[kRsStageWords] = {TW_F_FIRST_A | TW_F_LAST_A | TW_F_FIRST_B | TW_F_LAST_B | TW_F_EMPTY, bz};
          memcpy(out, e, sizeof(e));
          out += W;
          continue;
        }
        // each unit's first and last multiplying step (pair-wide: all 8 entries)
        int first[2] = {-1, -1}, last[2] = {-1, -1};
        for (int s = 0; s < nsteps; ++s) {
          const int32_t* st = &steps[static_cast<size_t>(ua.step_begin + s) * stride];
          for (int x = 0; x < 2; ++x) {
            bool any = false;
            for (int g = 0; g < G2; ++g) any |= st[1 + x * G2 + g] >= 0;
            if (any) {
              if (first[x] < 0) first[x] = s;
              last[x] = s;
            }
          }
        }
        for (int s = 0; s < nsteps; ++s) {
          const int32_t* st = &steps[static_cast<size_t>(ua.step_begin + s) * stride];
          int32_t e[kRsStageWords];
          for (int q = 0; q < W; ++q) e[q] = 0;
          uint32_t flags = 0;
          for (int x = 0; x < 2; ++x) {
            // a unit without blocks opens and closes on the twin's first stage
            const bool fx = first[x] < 0 ? s == 0 : s == first[x];
            const bool lx = first[x] < 0 ? s == 0 : s == last[x];
            if (fx) flags |= x ? TW_F_FIRST_B : TW_F_FIRST_A;
            if (lx) flags |= x ? TW_F_LAST_B : TW_F_LAST_A;
            bool any = false;
            for (int g = 0; g < G2; ++g) any |= st[1 + x * G2 + g] >= 0;
            if (!any) continue;
            flags |= x ? TW_F_MMA_B : TW_F_MMA_A;
            const SpmmUnit& u = p->h_units[ui + x];
            for (int g = 0; g < G; ++g) {
              const int slot = 4 * x + g;
              flags |= 1u << slot;
              const int32_t blk = g < u.nrows ? st[1 + x * G2 + r * G + g] : -1;
              e[4 + slot] = blk >= 0 ? blk * R + static_cast<int>((u.row0 + g) % slabs) * Rs : -Rs;
            }
          }
          e[0] = static_cast<int32_t>(flags);
          e[1] = bz;
          e[3] = st[0] * 32;
          memcpy(out, e, sizeof(e));
          out += W;
        }
      }
    }
    return BSP_OK;
  });
}

bsp_status plan_sddmm_host(bsp_sddmm_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                           int sm_count, int max_smem, const bsp_sddmm_opts* opts) {
  bsp_sddmm_opts o;
  memset(&o, 0, sizeof(o));
  if (opts) o = *opts;
  const int64_t M = p->M, N = p->N, K = p->K;
  const int R = p->R, C = p->C;
  if (R <= 0 || C <= 0 || R % 32 || C % 32)
    return set_error(BSP_ERR_INVALID_ARG, "block dims R, C must be positive multiples of 32");
  if (M <= 0 || N <= 0 || M % R || N % C)
    return set_error(BSP_ERR_INVALID_ARG, "M % R and N % C must be 0");
  if (K <= 0 || K % 32) return set_error(BSP_ERR_INVALID_ARG, "K must be a positive multiple of 32");
  if (M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31) || K >= (int64_t(1) << 31) ||
      p->nnzb < 0 || p->nnzb >= (int64_t(1) << 31))
    return set_error(BSP_ERR_UNSUPPORTED, "matrix too large for 32-bit coordinates");
  const int64_t nbr = M / R, nbc = N / C;
  bsp_status st = check_pattern(row_ptr, col_idx, nbr, nbc, p->nnzb);
  if (st != BSP_OK) return st;
  if (p->strategy != BSP_NAIVE && p->strategy != BSP_DDA && p->strategy != BSP_SNF)
    return set_error(BSP_ERR_INVALID_ARG, "unknown strategy");

  // Default: the row-stacked kernel (N = 128/256 MMAs).  group_mma == 2 keeps
  // the swap-AB kernel (one 4-segment unit per block-row slab).
  if (o.group_mma != 2) return plan_sddmm_rowstack(p, row_ptr, col_idx, sm_count, max_smem, &o);
  p->variant = 0;
  const int Rs = slab_height(R);
  const int kc = (K % 64 == 0) ? 64 : 32;
  p->Rs = Rs;
  p->kc = kc;
  p->keep_a = 0;

  std::vector<SddmmUnit> units;
  for (int64_t i = 0; i < nbr; ++i) {
    for (int r_off = 0; r_off < R; r_off += Rs) {
      SddmmUnit u;
      memset(&u, 0, sizeof(u));
      u.row = static_cast<int32_t>(i);
      u.r_off = r_off;
      for (int32_t b = row_ptr[i]; b < row_ptr[i + 1]; ++b) {
        for (int c0 = 0; c0 < C; c0 += 32) {
          u.blk[u.nseg] = b;
          u.col[u.nseg] = col_idx[b] * C + c0;
          if (++u.nseg == 4) {
            units.push_back(u);
            u.nseg = 0;
          }
        }
      }
      if (u.nseg > 0) units.push_back(u);
    }
  }
  int grid = o.max_ctas > 0 ? std::min(o.max_ctas, sm_count) : sm_count;
  grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(grid, units.size())));
  std::vector<std::vector<int32_t>> per;
  if (o.no_load_balance || p->strategy == BSP_DDA) {
    // DDA keeps a block-row's units together on one CTA, so that the row's
    // A slab is reused from L2/smem by consecutive units.
    contiguous_split(static_cast<int64_t>(units.size()), grid, &per);
  } else {
    std::vector<int64_t> w(units.size());
    for (size_t k = 0; k < units.size(); ++k) w[k] = units[k].nseg;
    serpentine_order(w, grid, &per);
  }
  p->h_units.clear();
  p->h_cta_begin.assign(1, 0);
  for (int c = 0; c < grid; ++c) {
    for (int32_t idx : per[c]) p->h_units.push_back(units[idx]);
    p->h_cta_begin.push_back(static_cast<int32_t>(p->h_units.size()));
  }
  p->n_units = static_cast<int64_t>(units.size());
  p->grid = grid;

  int stage_bytes = Rs * kc * 2 + 4 * kc * 64;
  stage_bytes = (stage_bytes + 1023) / 1024 * 1024;
  int stages = std::min(32, (max_smem - sddmm_smem_bytes(0, stage_bytes)) / stage_bytes);
  if (stages < 2) return set_error(BSP_ERR_UNSUPPORTED, "block too large for the pipeline");
  p->stage_bytes = stage_bytes;
  p->stages = stages;
  p->smem_bytes = sddmm_smem_bytes(stages, stage_bytes);
  p->tmem_cols = pow2_at_least(2 * Rs);
  p->timeout_ns = static_cast<uint64_t>(o.timeout_ms > 0 ? o.timeout_ms : 2000) * 1000000ull;
  return BSP_OK;
}

// Row-stacked SDDMM schedule.  Output rows are taken 128 at a time (one TMA
// box of A, four 32-row slabs = TMEM lane quarters).  For each such group the
// union of the mask's block-columns over the block-rows it touches is cut
// into 32-column segments, and the segments into units of nseg_max (4 or 8,
// MMA N = 128 or 256).  blk[q][s] names the mask block that slab q of
// segment s lands in (-1: not in the mask; the tile is computed but not
// written).  A block-column repeated within one mask row gets a second layer
// of units, so every output block is written exactly once.
bsp_status plan_sddmm_rowstack(bsp_sddmm_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                               int sm_count, int max_smem, const bsp_sddmm_opts* opts) {
  const bsp_sddmm_opts& o = *opts;
  const int64_t M = p->M, K = p->K;
  const int R = p->R, C = p->C;
  const int kc = (K % 64 == 0) ? 64 : 32;
  const int nkc = static_cast<int>(K / kc);
  p->variant = 1;
  p->Rs = 32;
  p->kc = kc;
  p->keep_a = 0;
  const int64_t ngroups = (M + 127) / 128;
  const int segs_per_block = C / 32;

  // (block-column, block index) of every mask block of block-row br, sorted
  // by column (stable: repeated columns keep their order, one layer each).
  auto row_pairs = [&](int64_t br, std::vector<std::pair<int32_t, int32_t>>* out) {
    out->clear();
    for (int32_t b = row_ptr[br]; b < row_ptr[br + 1]; ++b) out->push_back({col_idx[b], b});
    std::stable_sort(out->begin(), out->end(),
                     [](const std::pair<int32_t, int32_t>& x, const std::pair<int32_t, int32_t>& y) {
                       return x.first < y.first;
                     });
  };
  struct GroupSegs {
    int64_t g;
    int layer;
    std::vector<int32_t> cols;  // block-columns of this layer, ascending
  };
  std::vector<GroupSegs> layers;
  std::vector<std::vector<std::pair<int32_t, int32_t>>> slab_pairs(4);
  std::vector<int64_t> slab_br(4);
  int64_t units8 = 0, units4 = 0;
  std::vector<std::vector<std::pair<int32_t, int32_t>>> group_rows;
  for (int64_t g = 0; g < ngroups; ++g) {
    const int64_t r_lo = g * 128, r_hi = std::min<int64_t>(M, r_lo + 128);
    const int64_t br0 = r_lo / R, br1 = (r_hi - 1) / R + 1;
    group_rows.assign(static_cast<size_t>(br1 - br0), {});
    int max_layer = 0;
    for (int64_t br = br0; br < br1; ++br) {
      auto& v = group_rows[static_cast<size_t>(br - br0)];
      row_pairs(br, &v);
      int run = 0;
      for (size_t k = 0; k < v.size(); ++k) {
        run = (k > 0 && v[k].first == v[k - 1].first) ? run + 1 : 0;
        max_layer = std::max(max_layer, run);
      }
    }
    for (int layer = 0; layer <= max_layer; ++layer) {
      GroupSegs gs;
      gs.g = g;
      gs.layer = layer;
      for (const auto& v : group_rows) {
        int run = 0;
        for (size_t k = 0; k < v.size(); ++k) {
          run = (k > 0 && v[k].first == v[k - 1].first) ? run + 1 : 0;
          if (run == layer) gs.cols.push_back(v[k].first);
        }
      }
      std::sort(gs.cols.begin(), gs.cols.end());
      gs.cols.erase(std::unique(gs.cols.begin(), gs.cols.end()), gs.cols.end());
      if (gs.cols.empty()) continue;
      const int64_t nseg = static_cast<int64_t>(gs.cols.size()) * segs_per_block;
      units8 += (nseg + 7) / 8;
      units4 += (nseg + 3) / 4;
      layers.push_back(std::move(gs));
    }
  }
  int nseg_max = 8;
  if (o.n_tiles == 1) nseg_max = 4;
  else if (o.n_tiles == 0 && units8 < sm_count && units4 > units8) nseg_max = 4;
  p->nseg_max = nseg_max;

  std::vector<SddmmRsUnit> units;
  std::vector<int64_t> weight;
  for (const GroupSegs& gs : layers) {
    const int64_t row0 = gs.g * 128;
    // per slab q: the (column, block) pairs of this layer
    for (int q = 0; q < 4; ++q) {
      slab_pairs[q].clear();
      const int64_t row = row0 + 32 * q;
      slab_br[q] = row < M ? row / R : -1;
      if (slab_br[q] < 0) continue;
      std::vector<std::pair<int32_t, int32_t>> v;
      row_pairs(slab_br[q], &v);
      int run = 0;
      for (size_t k = 0; k < v.size(); ++k) {
        run = (k > 0 && v[k].first == v[k - 1].first) ? run + 1 : 0;
        if (run == gs.layer) slab_pairs[q].push_back(v[k]);
      }
    }
    std::vector<int32_t> segs;
    for (int32_t j : gs.cols)
      for (int c0 = 0; c0 < C; c0 += 32) segs.push_back(static_cast<int32_t>(int64_t(j) * C + c0));
    for (size_t s0 = 0; s0 < segs.size(); s0 += nseg_max) {
      SddmmRsUnit u;
      memset(&u, 0, sizeof(u));
      u.row0 = static_cast<int32_t>(row0);
      u.nseg = static_cast<int32_t>(std::min<size_t>(nseg_max, segs.size() - s0));
      for (int s_ = 0; s_ < kSddmmRsMaxSeg; ++s_) {
        u.seg_col[s_] = s_ < u.nseg ? segs[s0 + s_] : -1;
        for (int q = 0; q < 4; ++q) {
          u.blk[q][s_] = -1;
          if (s_ >= u.nseg || slab_br[q] < 0) continue;
          const int32_t j = u.seg_col[s_] / C;
          const auto& sp = slab_pairs[q];
          auto it = std::lower_bound(sp.begin(), sp.end(), std::make_pair(j, INT32_MIN));
          if (it != sp.end() && it->first == j) u.blk[q][s_] = it->second;
        }
      }
      units.push_back(u);
      weight.push_back(static_cast<int64_t>(u.nseg) * nkc + 2);
    }
  }
  int grid = o.max_ctas > 0 ? std::min(o.max_ctas, sm_count) : sm_count;
  grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(grid, units.size())));
  std::vector<std::vector<int32_t>> per;
  if (o.no_load_balance || p->strategy == BSP_DDA) {
    // CDA: a row group's units stay together on one CTA (A rows reused)
    contiguous_split(static_cast<int64_t>(units.size()), grid, &per);
  } else if (p->strategy == BSP_SNF) {
    // SnF: contiguous runs balanced by weight, so each CTA loads a row
    // group's A tile once and streams the group's B segments past it
    contiguous_weighted_split(weight, grid, &per);
  } else {
    serpentine_order(weight, grid, &per);
  }
  p->h_units.clear();
  p->h_rs_units.clear();
  p->h_cta_begin.assign(1, 0);
  for (int c = 0; c < grid; ++c) {
    for (int32_t idx : per[c]) p->h_rs_units.push_back(units[idx]);
    p->h_cta_begin.push_back(static_cast<int32_t>(p->h_rs_units.size()));
  }
  p->n_units = static_cast<int64_t>(units.size());
  p->grid = grid;

  // Resident A (CDA and SnF; opts.group_rows = -1 turns it off): two
  // 128 x K A tiles beside a ring of B-only stages, when K <= 256 and at
  // least two stages still fit.
  const int a_tile = 128 * static_cast<int>(K) * 2;
  const int b_stage = (nseg_max * kc * 64 + 1023) / 1024 * 1024;
  p->keep_a = (p->strategy == BSP_DDA || p->strategy == BSP_SNF) && o.group_rows != -1 && K <= 256 &&
                      (max_smem - 2048 - 2 * a_tile) / b_stage >= 2
                  ? 1
                  : 0;
  if (p->keep_a) {
    // runs of equal row0 in each CTA's list: pad[0] = run index << 1 | first, pad[1] = last
    for (int c = 0; c < grid; ++c) {
      int32_t run = -1;
      for (int32_t ui = p->h_cta_begin[c]; ui < p->h_cta_begin[c + 1]; ++ui) {
        SddmmRsUnit& u = p->h_rs_units[ui];
        const bool first = ui == p->h_cta_begin[c] || u.row0 != p->h_rs_units[ui - 1].row0;
        if (first) {
          ++run;
          if (ui > p->h_cta_begin[c]) p->h_rs_units[ui - 1].pad[1] = 1;
        }
        u.pad[0] = (run << 1) | (first ? 1 : 0);
        u.pad[1] = 0;
      }
      if (p->h_cta_begin[c + 1] > p->h_cta_begin[c]) p->h_rs_units[p->h_cta_begin[c + 1] - 1].pad[1] = 1;
    }
  }

  const int stage_bytes = p->keep_a ? b_stage : (128 * kc * 2 + nseg_max * kc * 64 + 1023) / 1024 * 1024;
  const int ring_smem = max_smem - 2048 - (p->keep_a ? 2 * a_tile : 0);
  const int max_stages = std::min(sddmm_rowstack_max_stages(), ring_smem / stage_bytes);
  if (max_stages < 2) return set_error(BSP_ERR_UNSUPPORTED, "stage too large for the pipeline");
  int nprod = 1, stages = max_stages;
  if (o.producers > 0) {
    nprod = std::min({o.producers, sddmm_rowstack_max_producers(), max_stages});
    stages = max_stages / nprod * nprod;
  } else {
    // More producer warps beat one more stage here (measured on B200 with the
    // config 4 mask: one producer over 5 stages 35 us, two over 4 and three
    // over 3 both 29 us), so up to one stage of the ring is given up for them.
    for (int q = 2; q <= std::min(sddmm_rowstack_max_producers(), max_stages); ++q) {
      const int sq = max_stages / q * q;
      if (sq >= 2 && sq >= max_stages - 1) {
        nprod = q;
        stages = sq;
      }
    }
  }
  p->nprod = nprod;
  p->stage_bytes = stage_bytes;
  p->stages = stages;
  p->smem_bytes = 2048 + (p->keep_a ? 2 * a_tile : 0) + stages * stage_bytes;
  p->tmem_cols = pow2_at_least(2 * 32 * nseg_max);
  p->timeout_ns = static_cast<uint64_t>(o.timeout_ms > 0 ? o.timeout_ms : 2000) * 1000000ull;
  return BSP_OK;
}

// SpGEMM schedule (C_bsr = A_bsr * B_bsr).  The output pattern is computed
// first (bsr_matrix.hpp:741-810: block (i, j) exists when some A[i, k] and
// B[k, j] are stored; columns ascending).  Output rows are then cut into
// 32-row slabs ("entries"), four per group (MMA M = 128); the union of the
// group's output block-columns is cut into 32-column segments, nseg_max per
// unit (MMA N).  A unit's steps are the block indices k for which one of its
// entries' rows stores A[i, k] and one of its columns stores B[k, j], in
// ascending order.  A k repeated inside a row of A (or a column repeated in
// row k of B) gives layered steps, one per pair of repeats, so every stored
// block product is taken exactly once.
// Cut one step's slots into TMA boxes.  ay[e]: first A row of entry e's slab
// (-1 absent); bb[s] / bt[s]: block of B and 32-column slice of segment s
// (block -1 absent).  A run of slots that are all absent, or whose data is
// contiguous (A slabs 32 rows apart; B segments of one slice in consecutive
// blocks), is covered by power-of-two boxes of at most 1 << la_log2 /
// 1 << lb_log2 slots, largest first.
static SpgemmStep spgemm_boxes(const int32_t* ay, const int32_t* bb, const int32_t* bt, int nseg,
                               int la_log2, int lb_log2) {
  SpgemmStep st;
  memset(&st, 0, sizeof(st));
  int nbox = 0;
  auto emit_a = [&](int e0, int len) {
    while (len > 0) {
      int l = la_log2;
      while ((1 << l) > len) --l;
      const int L = 1 << l;
      st.a_y[nbox] = ay[e0] >= 0 ? ay[e0] : -32 * L;
      st.a_meta[nbox] = static_cast<uint8_t>(kSpgemmBoxValid | e0 | (l << 3));
      ++nbox;
      e0 += L;
      len -= L;
    }
  };
  for (int e = 0; e < kSpgemmEnt;) {
    int r = e + 1;
    while (r < kSpgemmEnt && ((ay[e] < 0 && ay[r] < 0) || (ay[e] >= 0 && ay[r] == ay[r - 1] + 32))) ++r;
    emit_a(e, r - e);
    e = r;
  }
  nbox = 0;
  auto emit_b = [&](int s0, int len) {
    while (len > 0) {
      int l = lb_log2;
      while ((1 << l) > len) --l;
      const int L = 1 << l;
      st.b_z[nbox] = bb[s0] >= 0 ? bb[s0] : -L;
      st.b_meta[nbox] = static_cast<uint8_t>(kSpgemmBoxValid | s0 | (l << 3) | ((bt[s0] & 3) << 5));
      ++nbox;
      s0 += L;
      len -= L;
    }
  };
  for (int s_ = 0; s_ < nseg;) {
    int r = s_ + 1;
    while (r < nseg && ((bb[s_] < 0 && bb[r] < 0) ||
                        (bb[s_] >= 0 && bb[r] == bb[r - 1] + 1 && bt[r] == bt[s_])))
      ++r;
    emit_b(s_, r - s_);
    s_ = r;
  }
  return st;
}

static int spgemm_box_count(const SpgemmStep& st) {
  int n = 0;
  for (int i = 0; i < kSpgemmEnt; ++i) n += (st.a_meta[i] & kSpgemmBoxValid) ? 1 : 0;
  for (int i = 0; i < kSpgemmMaxSeg; ++i) n += (st.b_meta[i] & kSpgemmBoxValid) ? 1 : 0;
  return n;
}

struct SgBuildCtx {
  const bsp_spgemm_plan* p;
  const int32_t *a_rp, *a_ci, *b_rp, *b_ci;
  int64_t nbk, nbc;
  int spr, segs_per_col;
  int64_t n_ent;
  int nkc;
};

struct SgBuildOut {
  std::vector<SpgemmUnit> units;
  std::vector<int64_t> weight;
  std::vector<SpgemmStep> steps;  // step_begin of the units counts from this range's first step
  int64_t n_steps = 0, n_boxes = 0;
};

// The units and steps of output groups [g_begin, g_end) for nseg_max
// segments per unit.  count_only: only n_steps (no tables).
static bsp_status sg_build_groups(const SgBuildCtx& c, int nseg_max, int64_t g_begin, int64_t g_end,
                                  bool count_only, SgBuildOut* out) {
  const bsp_spgemm_plan* p = c.p;
  const int32_t *a_rp = c.a_rp, *a_ci = c.a_ci, *b_rp = c.b_rp, *b_ci = c.b_ci;
  const int64_t nbk = c.nbk, nbc = c.nbc, n_ent = c.n_ent;
  const int spr = c.spr, segs_per_col = c.segs_per_col, Ra = p->Ra;
  auto& units = out->units;
  auto& weight = out->weight;
  auto& steps = out->steps;
  out->n_steps = 0;
  out->n_boxes = 0;
  const int cpu = std::max(1, nseg_max / segs_per_col);  // block-columns per unit
  std::vector<int32_t> colpos(static_cast<size_t>(nbc), -1), colstamp(static_cast<size_t>(nbc), -1);
  std::vector<int32_t> kstamp(static_cast<size_t>(nbk), -1);
  std::vector<int32_t> cols, ks;
  // Per local block-row q of the group (at most 4): A blocks of column k
  // (a_first / a_cnt into rowpairs[q], valid where a_stamp == g) and the
  // output index of block-column j (o_idx, valid where o_stamp == g).
  const int64_t rows_per_group = (kSpgemmEnt + spr - 1) / spr;
  std::vector<int32_t> a_first_k(static_cast<size_t>(rows_per_group * nbk)),
      a_cnt_k(static_cast<size_t>(rows_per_group * nbk)), a_stamp(static_cast<size_t>(rows_per_group * nbk), -1);
  std::vector<int32_t> o_idx, o_stamp;
  if (!count_only) {
    o_idx.resize(static_cast<size_t>(rows_per_group * nbc));
    o_stamp.assign(static_cast<size_t>(rows_per_group * nbc), -1);
  }
  // B blocks of the group's k's bucketed by unit (counting sort), k ascending
  std::vector<int32_t> cb_off, cb_k, cb_b, fill;
  std::vector<std::vector<int32_t>> bl(kSpgemmMaxSeg);  // B blocks of row k per unit column
  // (k, A block) of each distinct block-row of the group, sorted by k (stable)
  std::vector<std::vector<std::pair<int32_t, int32_t>>> rowpairs;
  for (int64_t g = g_begin; g < g_end; ++g) {
    const int32_t g32 = static_cast<int32_t>(g);
    const int64_t e0 = g * kSpgemmEnt, e1 = std::min<int64_t>(n_ent, e0 + kSpgemmEnt);
    const int64_t r0 = e0 / spr, r1 = (e1 - 1) / spr + 1;  // block-rows [r0, r1)
    cols.clear();
    for (int64_t i = r0; i < r1; ++i)
      for (int32_t q = p->out_row_ptr[i]; q < p->out_row_ptr[i + 1]; ++q) {
        const int32_t j = p->out_col_idx[q];
        if (!count_only) {
          const size_t oi = static_cast<size_t>((i - r0) * nbc + j);
          o_stamp[oi] = g32;
          o_idx[oi] = q;
        }
        if (colstamp[j] != g32) {
          colstamp[j] = g32;
          cols.push_back(j);
        }
      }
    if (cols.empty()) continue;
    std::sort(cols.begin(), cols.end());
    for (size_t q = 0; q < cols.size(); ++q) colpos[cols[q]] = static_cast<int32_t>(q);
    const int64_t nchunks = (static_cast<int64_t>(cols.size()) + cpu - 1) / cpu;
    rowpairs.resize(static_cast<size_t>(r1 - r0));
    ks.clear();
    for (int64_t i = r0; i < r1; ++i) {
      auto& v = rowpairs[static_cast<size_t>(i - r0)];
      v.clear();
      for (int32_t a = a_rp[i]; a < a_rp[i + 1]; ++a) {
        v.push_back({a_ci[a], a});
        if (kstamp[a_ci[a]] != g32) {
          kstamp[a_ci[a]] = g32;
          ks.push_back(a_ci[a]);
        }
      }
      std::stable_sort(v.begin(), v.end(),
                       [](const std::pair<int32_t, int32_t>& x, const std::pair<int32_t, int32_t>& y) {
                         return x.first < y.first;
                       });
      for (size_t t = 0; t < v.size(); ++t) {
        const size_t ai = static_cast<size_t>((i - r0) * nbk + v[t].first);
        if (a_stamp[ai] != g32) {
          a_stamp[ai] = g32;
          a_first_k[ai] = static_cast<int32_t>(t);
          a_cnt_k[ai] = 0;
        }
        ++a_cnt_k[ai];
      }
    }
    std::sort(ks.begin(), ks.end());
    cb_off.assign(static_cast<size_t>(nchunks + 1), 0);
    for (int32_t k : ks)
      for (int32_t b = b_rp[k]; b < b_rp[k + 1]; ++b) ++cb_off[static_cast<size_t>(colpos[b_ci[b]] / cpu + 1)];
    for (int64_t q = 0; q < nchunks; ++q) cb_off[q + 1] += cb_off[q];
    cb_k.resize(static_cast<size_t>(cb_off[nchunks]));
    cb_b.resize(static_cast<size_t>(cb_off[nchunks]));
    fill.assign(cb_off.begin(), cb_off.end() - 1);
    for (int32_t k : ks)
      for (int32_t b = b_rp[k]; b < b_rp[k + 1]; ++b) {
        const size_t at = static_cast<size_t>(fill[static_cast<size_t>(colpos[b_ci[b]] / cpu)]++);
        cb_k[at] = k;
        cb_b[at] = b;
      }
    for (int64_t ch = 0; ch < nchunks; ++ch) {
      SpgemmUnit u;
      memset(&u, 0, sizeof(u));
      const int64_t j0 = ch * cpu;
      const int ncols = static_cast<int>(std::min<int64_t>(cpu, static_cast<int64_t>(cols.size()) - j0));
      u.n_ent = static_cast<int32_t>(e1 - e0);
      u.nseg = std::min(nseg_max, ncols * segs_per_col);
      if (!count_only) {
        // segments slice-major: segment s is 32-column slice s / ncols of
        // column s % ncols, so that a slice of consecutive stored blocks of a
        // row of B lands in consecutive segments (one TMA box)
        for (int s_ = 0; s_ < kSpgemmMaxSeg; ++s_) u.seg_x[s_] = s_ < u.nseg ? (s_ / ncols) * 32 : 0;
        for (int e = 0; e < kSpgemmEnt; ++e) {
          const int64_t E = e0 + e;
          u.ent_r[e] = E < e1 ? static_cast<int32_t>(E % spr) * 32 : 0;
          for (int s_ = 0; s_ < kSpgemmMaxSeg; ++s_) {
            u.out_blk[e][s_] = -1;
            if (E >= e1 || s_ >= u.nseg) continue;
            const int32_t j = cols[static_cast<size_t>(j0 + s_ % ncols)];
            const size_t oi = static_cast<size_t>((E / spr - r0) * nbc + j);
            if (o_stamp[oi] == g32) u.out_blk[e][s_] = o_idx[oi];
          }
        }
      }
      u.step_begin = static_cast<int32_t>(out->n_steps);
      if (out->n_steps >= (int64_t(1) << 31) - 4096)
        return set_error(BSP_ERR_UNSUPPORTED, "SpGEMM schedule too large");
      for (int32_t t0 = cb_off[ch]; t0 < cb_off[ch + 1];) {
        const int32_t k = cb_k[t0];
        int32_t t1 = t0;
        // B blocks of row k per unit column, A blocks of column k per entry
        for (auto& l : bl) l.clear();
        int lb_max = 0;
        for (; t1 < cb_off[ch + 1] && cb_k[t1] == k; ++t1) {
          auto& l = bl[static_cast<size_t>(colpos[b_ci[cb_b[t1]]] - j0)];
          l.push_back(cb_b[t1]);
          lb_max = std::max(lb_max, static_cast<int>(l.size()));
        }
        t0 = t1;
        int32_t a_first[kSpgemmEnt], a_cnt[kSpgemmEnt];
        int la_max = 0;
        for (int e = 0; e < kSpgemmEnt; ++e) {
          a_first[e] = 0;
          a_cnt[e] = 0;
          const int64_t E = e0 + e;
          if (E >= e1) continue;
          const size_t ai = static_cast<size_t>((E / spr - r0) * nbk + k);
          if (a_stamp[ai] != g32) continue;
          a_first[e] = a_first_k[ai];
          a_cnt[e] = a_cnt_k[ai];
          la_max = std::max(la_max, static_cast<int>(a_cnt[e]));
        }
        if (count_only) {
          out->n_steps += static_cast<int64_t>(la_max) * lb_max;
          continue;
        }
        for (int la = 0; la < la_max; ++la)
          for (int lb = 0; lb < lb_max; ++lb) {
            int32_t ay[kSpgemmEnt], bb[kSpgemmMaxSeg], bt[kSpgemmMaxSeg];
            for (int e = 0; e < kSpgemmEnt; ++e) {
              ay[e] = -1;
              if (la < a_cnt[e]) {
                const auto& v = rowpairs[static_cast<size_t>((e0 + e) / spr - r0)];
                ay[e] = v[static_cast<size_t>(a_first[e] + la)].second * Ra + u.ent_r[e];
              }
            }
            for (int s_ = 0; s_ < u.nseg; ++s_) {
              const auto& l = bl[static_cast<size_t>(s_ % ncols)];
              bb[s_] = lb < static_cast<int>(l.size()) ? l[static_cast<size_t>(lb)] : -1;
              bt[s_] = s_ / ncols;
            }
            steps.push_back(spgemm_boxes(ay, bb, bt, u.nseg, p->la_log2, p->lb_log2));
            out->n_boxes += spgemm_box_count(steps.back());
            ++out->n_steps;
          }
      }
      u.n_steps = static_cast<int32_t>(out->n_steps - u.step_begin);
      if (u.n_steps == 0 || count_only) continue;  // (an empty unit cannot happen: every unit column has a product)
      units.push_back(u);
      weight.push_back(static_cast<int64_t>(u.n_steps) * c.nkc + 2);
    }
  }
  return BSP_OK;
}

bsp_status plan_spgemm_host(bsp_spgemm_plan* p, const int32_t* a_rp, const int32_t* a_ci,
                            const int32_t* b_rp, const int32_t* b_ci, int sm_count, int max_smem,
                            const bsp_spmm_opts* opts) {
  bsp_spmm_opts o;
  memset(&o, 0, sizeof(o));
  if (opts) o = *opts;
  const int64_t M = p->M, K = p->K, N = p->N;
  const int Ra = p->Ra, Ca = p->Ca, Cb = p->Cb;
  auto ok_blk = [](int x) { return x == 32 || x == 64 || x == 128; };
  if (!ok_blk(Ra) || !ok_blk(Ca) || !ok_blk(Cb))
    return set_error(BSP_ERR_UNSUPPORTED, "SpGEMM block sizes must be 32, 64 or 128");
  if (M <= 0 || K <= 0 || N <= 0 || M % Ra || K % Ca || N % Cb)
    return set_error(BSP_ERR_INVALID_ARG, "M % Ra, K % Ca and N % Cb must be 0");
  if (p->nnzb_a < 0 || p->nnzb_b < 0 || p->nnzb_a * Ra >= (int64_t(1) << 31) ||
      p->nnzb_b * Ca >= (int64_t(1) << 31) || M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31))
    return set_error(BSP_ERR_UNSUPPORTED, "matrix too large for 32-bit TMA coordinates");
  const int64_t nbr = M / Ra, nbk = K / Ca, nbc = N / Cb;
  bsp_status st = check_pattern(a_rp, a_ci, nbr, nbk, p->nnzb_a);
  if (st != BSP_OK) return st;
  st = check_pattern(b_rp, b_ci, nbk, nbc, p->nnzb_b);
  if (st != BSP_OK) return st;

  // ---- output pattern (symbolic product), block-rows split over threads ----
  // (int32 stamps: one per output block-column and thread, so the thread
  // count also stays under a 256 MB budget for them)
  const int nt_sym = planner_threads(nbr, 64, nbc * 4);
  std::vector<std::vector<int32_t>> sym_cols(static_cast<size_t>(nt_sym));
  std::vector<int64_t> sym_pairs(static_cast<size_t>(nt_sym), 0);
  p->out_row_ptr.assign(static_cast<size_t>(nbr + 1), 0);
  st = parallel_ranges(nbr, nt_sym, [&](int t, int64_t i0, int64_t i1) {
    std::vector<int32_t> stamp(static_cast<size_t>(nbc), -1);
    auto& oc = sym_cols[static_cast<size_t>(t)];
    for (int64_t i = i0; i < i1; ++i) {
      const size_t start = oc.size();
      for (int32_t a = a_rp[i]; a < a_rp[i + 1]; ++a) {
        const int32_t k = a_ci[a];
        sym_pairs[static_cast<size_t>(t)] += b_rp[k + 1] - b_rp[k];
        for (int32_t b = b_rp[k]; b < b_rp[k + 1]; ++b) {
          const int32_t j = b_ci[b];
          if (stamp[j] != static_cast<int32_t>(i)) {
            stamp[j] = static_cast<int32_t>(i);
            oc.push_back(j);
          }
        }
      }
      std::sort(oc.begin() + static_cast<std::ptrdiff_t>(start), oc.end());
      p->out_row_ptr[i + 1] = static_cast<int32_t>(oc.size() - start);  // row length for now
    }
    return BSP_OK;
  });
  if (st != BSP_OK) return st;
  int64_t pairs = 0, out_total = 0;
  for (int t = 0; t < nt_sym; ++t) {
    pairs += sym_pairs[static_cast<size_t>(t)];
    out_total += static_cast<int64_t>(sym_cols[static_cast<size_t>(t)].size());
  }
  if (out_total >= (int64_t(1) << 31)) return set_error(BSP_ERR_UNSUPPORTED, "output has too many blocks");
  for (int64_t i = 0; i < nbr; ++i) p->out_row_ptr[i + 1] += p->out_row_ptr[i];
  p->out_col_idx.clear();
  p->out_col_idx.reserve(static_cast<size_t>(out_total));
  for (auto& v : sym_cols) {
    p->out_col_idx.insert(p->out_col_idx.end(), v.begin(), v.end());
    std::vector<int32_t>().swap(v);
  }
  p->pairs = pairs;
  const int64_t out_nnzb = static_cast<int64_t>(p->out_col_idx.size());
  if (out_nnzb * Ra * Cb >= (int64_t(1) << 40))
    return set_error(BSP_ERR_UNSUPPORTED, "output too large");

  // ---- stage geometry ----
  const int kc = Ca == 32 ? 32 : 64;
  const int nkc = Ca / kc;
  p->kc = kc;
  p->nkc = nkc;
  const int spr = Ra / 32;                      // slabs (entries) per output block-row
  const int segs_per_col = Cb / 32;             // segments per output block-column
  const int64_t n_ent = nbr * spr;
  const int64_t ngroups = (n_ent + kSpgemmEnt - 1) / kSpgemmEnt;

  // largest boxes the tensors can hold (a box may not exceed its tensor)
  p->la_log2 = 0;
  while (p->la_log2 < 2 && (int64_t(32) << (p->la_log2 + 1)) <= p->nnzb_a * Ra) ++p->la_log2;
  p->lb_log2 = 0;
  while (p->lb_log2 < 3 && (int64_t(1) << (p->lb_log2 + 1)) <= p->nnzb_b) ++p->lb_log2;

  const SgBuildCtx ctx{p, a_rp, a_ci, b_rp, b_ci, nbk, nbc, spr, segs_per_col, n_ent, nkc};
  // Groups split over threads; each range's units and steps are appended in
  // range order, so the schedule does not depend on the thread count.
  const int64_t scratch_per_thread = (nbc + nbk) * 48;
  auto run = [&](int nseg, bool count_only, std::vector<SpgemmUnit>* units, std::vector<int64_t>* weight,
                 int64_t* n_steps, int64_t* n_boxes) -> bsp_status {
    const int nt = planner_threads(ngroups, 8, scratch_per_thread);
    std::vector<SgBuildOut> parts(static_cast<size_t>(nt));
    bsp_status s2 = parallel_ranges(ngroups, nt, [&](int t, int64_t g0, int64_t g1) {
      return sg_build_groups(ctx, nseg, g0, g1, count_only, &parts[static_cast<size_t>(t)]);
    });
    if (s2 != BSP_OK) return s2;
    *n_steps = 0;
    *n_boxes = 0;
    int64_t n_units = 0;
    for (const auto& q : parts) {
      *n_steps += q.n_steps;
      *n_boxes += q.n_boxes;
      n_units += static_cast<int64_t>(q.units.size());
    }
    if (*n_steps >= (int64_t(1) << 31) - 4096) return set_error(BSP_ERR_UNSUPPORTED, "SpGEMM schedule too large");
    if (count_only) return BSP_OK;
    units->clear();
    weight->clear();
    units->reserve(static_cast<size_t>(n_units));
    weight->reserve(static_cast<size_t>(n_units));
    p->h_steps.clear();
    p->h_steps.reserve(static_cast<size_t>(*n_steps));
    for (auto& q : parts) {
      const int32_t off = static_cast<int32_t>(p->h_steps.size());
      for (SpgemmUnit u : q.units) {
        u.step_begin += off;
        units->push_back(u);
      }
      weight->insert(weight->end(), q.weight.begin(), q.weight.end());
      p->h_steps.insert(p->h_steps.end(), q.steps.begin(), q.steps.end());
      std::vector<SpgemmStep>().swap(q.steps);
    }
    return BSP_OK;
  };
  // MMA N = 256 (8 segments) unless the caller asks for 128; when 256-wide
  // tiles would be mostly empty, N = 128 is taken if its schedule moves fewer
  // operand bytes (a step costs about its bytes: the smem fill rate bounds it).
  // The choice needs only step counts, so only the chosen width is built.
  std::vector<SpgemmUnit> units;
  std::vector<int64_t> weight;
  int nseg_max = (o.n_tiles == 1) ? 4 : 8;
  if (o.n_tiles == 0) {
    int64_t n8 = 0, b8 = 0;
    st = run(8, true, nullptr, nullptr, &n8, &b8);
    if (st != BSP_OK) return st;
    const double fill = n8 > 0 ? static_cast<double>(pairs) * spr * segs_per_col /
                                     (static_cast<double>(n8) * kSpgemmEnt * 8)
                               : 1.0;
    if (fill < 0.5) {
      int64_t n4 = 0, b4 = 0;
      st = run(4, true, nullptr, nullptr, &n4, &b4);
      if (st != BSP_OK) return st;
      auto sub = [&](int n) { return static_cast<double>(kSpgemmEnt * 32 * kc * 2 + n * kc * 64); };
      if (static_cast<double>(n4) * sub(4) < static_cast<double>(n8) * sub(8)) nseg_max = 4;
    }
  }
  int64_t n_steps_total = 0;
  st = run(nseg_max, false, &units, &weight, &n_steps_total, &p->n_boxes);
  if (st != BSP_OK) return st;
  p->nseg_max = nseg_max;
  p->n_steps = static_cast<int64_t>(p->h_steps.size());

  int grid = o.max_ctas > 0 ? std::min(o.max_ctas, sm_count) : sm_count;
  grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(grid, units.size())));
  std::vector<std::vector<int32_t>> per;
  // no_load_balance: 0 ordered greedy (default), 1 contiguous split, 2 serpentine
  if (o.no_load_balance == 1) contiguous_split(static_cast<int64_t>(units.size()), grid, &per);
  else if (o.no_load_balance == 2) serpentine_order(weight, grid, &per);
  else ordered_greedy(weight, grid, &per);
  p->h_units.clear();
  p->h_cta_begin.assign(1, 0);
  for (int cta = 0; cta < grid; ++cta) {
    for (int32_t idx : per[cta]) p->h_units.push_back(units[idx]);
    p->h_cta_begin.push_back(static_cast<int32_t>(p->h_units.size()));
  }
  p->n_units = static_cast<int64_t>(units.size());
  p->grid = units.empty() ? 0 : grid;

  const int a_slot = 32 * kc * 2;
  const int sub_bytes = kSpgemmEnt * a_slot + nseg_max * kc * 64;
  int sps = o.steps_per_stage > 0 ? std::min(4, o.steps_per_stage) : (kc == 32 ? 2 : 1);
  int max_stages = 0;
  for (;; sps = std::max(1, sps / 2)) {
    max_stages = std::min(spgemm_max_stages(), (max_smem - 2048) / (sps * sub_bytes));
    if (max_stages >= 2 || sps == 1) break;
  }
  if (max_stages < 2) return set_error(BSP_ERR_UNSUPPORTED, "stage too large for the pipeline");
  const int stage_bytes = sps * sub_bytes;
  // Issuing the many small boxes of a stage is the producers' bottleneck, so
  // as many producer warps as can own stages, even at the cost of a ring slot.
  const int nprod = std::min({o.producers > 0 ? o.producers : spgemm_max_producers(),
                              spgemm_max_producers(), max_stages});
  const int stages = max_stages / nprod * nprod;
  p->sps = sps;
  p->sub_bytes = sub_bytes;
  p->nprod = nprod;
  p->stage_bytes = stage_bytes;
  p->stages = stages;
  p->smem_bytes = 2048 + stages * stage_bytes;
  p->tmem_cols = pow2_at_least(2 * 32 * nseg_max);
  p->timeout_ns = static_cast<uint64_t>(o.timeout_ms > 0 ? o.timeout_ms : 2000) * 1000000ull;
  return BSP_OK;
}

// Fused attention schedule: query rows in units of 128 (four block-rows of
// the 32 x 32 mask); per unit the sorted union of its block-rows' mask
// columns (a column repeated within a row counts once) cut into chunks of four
// key blocks, each with the bits of the (block-row, key block) pairs the mask
// holds.  Units (and parts) are dealt longest first to the least-loaded CTA.
bsp_status plan_attn_host(bsp_attn_plan* p, const int32_t* row_ptr, const int32_t* col_idx,
                          int sm_count, int max_smem, const bsp_spmm_opts* opts) {
  bsp_spmm_opts o;
  memset(&o, 0, sizeof(o));
  if (opts) o = *opts;
  const int64_t S = p->S;
  if (p->d != 64 && p->d != 128) return set_error(BSP_ERR_UNSUPPORTED, "attention head size must be 64 or 128");
  if (S <= 0 || S % 32 || S >= (int64_t(1) << 31))
    return set_error(BSP_ERR_INVALID_ARG, "sequence length must be a positive multiple of 32");
  const int64_t nbr = S / 32;
  bsp_status st = check_pattern(row_ptr, col_idx, nbr, nbr, p->nnzb);
  if (st != BSP_OK) return st;
  if (attn_smem_bytes(static_cast<int>(p->d)) > max_smem)
    return set_error(BSP_ERR_UNSUPPORTED, "not enough shared memory for the attention pipeline");
  const int64_t ngroups = (nbr + 3) / 4;
  p->h_units.clear();
  p->h_chunks.clear();
  p->mask_blocks = 0;
  std::vector<int64_t> weight;
  std::vector<int64_t> stamp(static_cast<size_t>(nbr), -1);
  std::vector<int32_t> cols;
  std::vector<std::vector<int32_t>> rowcols(4);
  for (int64_t g = 0; g < ngroups; ++g) {
    AttnUnit u;
    memset(&u, 0, sizeof(u));
    u.row0 = static_cast<int32_t>(g * 128);
    u.chunk_begin = static_cast<int32_t>(p->h_chunks.size());
    cols.clear();
    for (int q = 0; q < 4; ++q) {
      rowcols[q].clear();
      const int64_t i = g * 4 + q;
      if (i >= nbr) continue;
      for (int32_t b = row_ptr[i]; b < row_ptr[i + 1]; ++b) rowcols[q].push_back(col_idx[b]);
      std::sort(rowcols[q].begin(), rowcols[q].end());
      rowcols[q].erase(std::unique(rowcols[q].begin(), rowcols[q].end()), rowcols[q].end());
      p->mask_blocks += static_cast<int64_t>(rowcols[q].size());
      for (int32_t c : rowcols[q])
        if (stamp[c] != g) {
          stamp[c] = g;
          cols.push_back(c);
        }
    }
    std::sort(cols.begin(), cols.end());
    for (size_t c0 = 0; c0 < cols.size(); c0 += kAttnSlots) {
      AttnChunk ch;
      memset(&ch, 0, sizeof(ch));
      for (int s_ = 0; s_ < kAttnSlots; ++s_) {
        ch.kb[s_] = -1;
        if (c0 + s_ >= cols.size()) continue;
        const int32_t c = cols[c0 + s_];
        ch.kb[s_] = c;
        for (int q = 0; q < 4; ++q)
          if (std::binary_search(rowcols[q].begin(), rowcols[q].end(), c)) ch.bits |= 1u << (4 * q + s_);
      }
      p->h_chunks.push_back(ch);
    }
    u.n_chunks = static_cast<int32_t>(p->h_chunks.size()) - u.chunk_begin;
    u.n_parts = 1;
    u.counter = -1;
    p->h_units.push_back(u);
  }
  p->n_chunks = static_cast<int64_t>(p->h_chunks.size());
  int grid = o.max_ctas > 0 ? std::min(o.max_ctas, sm_count) : sm_count;
  // Split units.  Cost model (fitted to B200 timings, d = 128): a chunk keeps
  // the tensor pipe busy ~1.55 us; a unit's epilogue costs ~1.3 us, a split
  // part's (partial write, counter, and on the last part the merge) about
  // 5 + 2 * (parts - 1) us, on the critical path of its CTA.  By default several target lengths are tried:
  // every unit longer than the target is cut into parts of about that length,
  // all items are dealt longest first, and the split with the smallest
  // estimated makespan is kept.  n_tiles > 0 instead cuts every unit into
  // parts of about that many chunks; group_rows = -1 never splits.
  constexpr int64_t kChunkNs = 1550, kEpiNs = 1300, kSplitEpiNs = 5000, kSplitPartNs = 2000;
  std::vector<int64_t> np_of(p->h_units.size(), 1);
  if (o.group_rows >= 0 && o.n_tiles > 0) {
    for (size_t i = 0; i < p->h_units.size(); ++i) {
      const int64_t n = p->h_units[i].n_chunks;
      if (n > o.n_tiles + o.n_tiles / 4)
        np_of[i] = std::min<int64_t>(kAttnMaxParts, (n + o.n_tiles - 1) / o.n_tiles);
    }
  } else if (o.group_rows >= 0 && !p->h_units.empty()) {
    int64_t total = 0, longest = 0;
    for (const AttnUnit& u : p->h_units) {
      total += u.n_chunks * kChunkNs + kEpiNs;
      longest = std::max<int64_t>(longest, u.n_chunks);
    }
    // makespan of dealing the items longest first to the least-loaded CTA
    auto makespan = [&](const std::vector<int64_t>& np) {
      std::vector<int64_t> items;
      for (size_t i = 0; i < p->h_units.size(); ++i) {
        const int64_t n = p->h_units[i].n_chunks;
        for (int64_t k = 0; k < np[i]; ++k) {
          const int64_t len = n * (k + 1) / np[i] - n * k / np[i];
          items.push_back(len * kChunkNs + (np[i] > 1 ? kSplitEpiNs + kSplitPartNs * (np[i] - 1) : kEpiNs));
        }
      }
      std::sort(items.begin(), items.end(), std::greater<int64_t>());
      std::priority_queue<int64_t, std::vector<int64_t>, std::greater<int64_t>> load;
      for (int c = 0; c < grid; ++c) load.push(0);
      int64_t worst = 0;
      for (int64_t w : items) {
        int64_t l = load.top();
        load.pop();
        l += w;
        worst = std::max(worst, l);
        load.push(l);
      }
      return worst;
    };
    int64_t best = makespan(np_of);
    std::vector<int64_t> cand(p->h_units.size());
    const double avg_chunks = static_cast<double>(total) / grid / kChunkNs;
    for (double f : {0.6, 0.75, 0.9, 1.0, 1.1, 1.2, 1.3, 1.4, 1.5, 1.75, 2.0, 2.5}) {
      const int64_t target = std::max<int64_t>(2, static_cast<int64_t>(avg_chunks * f));
      if (target >= longest) continue;
      for (size_t i = 0; i < p->h_units.size(); ++i) {
        const int64_t n = p->h_units[i].n_chunks;
        cand[i] = n > target ? std::min<int64_t>({kAttnMaxParts, n / 2, (n + target - 1) / target}) : 1;
        cand[i] = std::max<int64_t>(1, cand[i]);
      }
      const int64_t m = makespan(cand);
      if (m < best) {
        best = m;
        np_of = cand;
      }
    }
  }
  std::vector<AttnUnit> parts;
  p->n_slots = 0;
  p->n_counters = 0;
  for (size_t i = 0; i < p->h_units.size(); ++i) {
    const AttnUnit& u = p->h_units[i];
    const int64_t np = np_of[i];
    if (np == 1) {
      parts.push_back(u);
      continue;
    }
    for (int64_t k = 0; k < np; ++k) {
      AttnUnit v = u;
      const int64_t b = u.n_chunks * k / np, e = u.n_chunks * (k + 1) / np;
      v.chunk_begin = u.chunk_begin + static_cast<int32_t>(b);
      v.n_chunks = static_cast<int32_t>(e - b);
      v.n_parts = static_cast<int32_t>(np);
      v.part = static_cast<int32_t>(k);
      v.slot0 = static_cast<int32_t>(p->n_slots);
      v.counter = static_cast<int32_t>(p->n_counters);
      parts.push_back(v);
    }
    p->n_slots += np;
    ++p->n_counters;
  }
  p->h_units.swap(parts);
  for (const AttnUnit& u : p->h_units) weight.push_back(static_cast<int64_t>(u.n_chunks) * 4 + 1);
  p->n_units = static_cast<int64_t>(p->h_units.size());
  grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(grid, p->n_units)));
  std::vector<std::vector<int32_t>> per;
  if (o.no_load_balance == 1) contiguous_split(p->n_units, grid, &per);
  else lpt_order(weight, grid, &per);
  std::vector<AttnUnit> ordered;
  p->h_cta_begin.assign(1, 0);
  for (int c = 0; c < grid; ++c) {
    for (int32_t idx : per[c]) ordered.push_back(p->h_units[idx]);
    p->h_cta_begin.push_back(static_cast<int32_t>(ordered.size()));
  }
  p->h_units.swap(ordered);
  p->grid = grid;
  p->smem_bytes = attn_smem_bytes(static_cast<int>(p->d));
  p->tmem_cols = 512;
  p->timeout_ns = static_cast<uint64_t>(o.timeout_ms > 0 ? o.timeout_ms : 2000) * 1000000ull;
  return BSP_OK;
}

// Operand bytes a SpMM plan moves with TMA into shared memory (the B200
// counterpart of the reference's per-core DRAM read counts of in0 = A and
// in1 = B, block_spmm/scripts/count_dram_reads.py): out[0] A bytes, out[1] B
// bytes, out[2] A boxes, out[3] B boxes.  Zero boxes for absent blocks read
// nothing and are not counted.
void spmm_plan_traffic(const bsp_spmm_plan& p, int64_t out[4]) {
  out[0] = out[1] = out[2] = out[3] = 0;
  const int64_t kc = p.kc, Rs = p.Rs;
  if (p.variant == 0) {
    const int stride = p.step_stride;
    const int64_t nkc = p.C / p.kc;
    for (const SpmmUnit& u : p.h_units)
      for (int32_t s = u.step_begin; s < u.step_end; ++s) {
        int64_t present = 0;
        for (int g = 0; g < p.G; ++g) present += p.h_steps[static_cast<size_t>(s) * stride + 1 + g] >= 0;
        out[0] += nkc * present * Rs * kc * 2;
        out[2] += nkc * present;
        out[1] += nkc * int64_t(u.nt) * kc * kTileN * 2;
        out[3] += nkc * int64_t(u.nt) * 2;  // two 64-column boxes per 128-column tile
      }
    return;
  }
  const size_t W = kRsStageWords;
  if (p.variant == 3) {
    // twins: one block-column per stage; this CTA's B half, and the A slots
    // of the units that multiply there (present blocks; zero boxes not counted)
    for (size_t k = 0; k + W <= p.h_stage_list.size(); k += W) {
      const uint32_t flags = static_cast<uint32_t>(p.h_stage_list[k]);
      if (flags & TW_F_EMPTY) continue;
      out[1] += kc * 128 * 2;
      out[3] += 2;
      for (int s = 0; s < 8; ++s)
        if (((flags >> s) & 1u) && p.h_stage_list[k + 4 + s] >= 0) {
          out[0] += Rs * kc * 2;
          out[2] += 1;
        }
    }
    return;
  }
  const int64_t b_cols = p.variant == 2 ? 128 : 128 * p.NT;  // a pair CTA loads half of the 256 columns
  for (size_t k = 0; k + W <= p.h_stage_list.size(); k += W) {
    const uint32_t flags = static_cast<uint32_t>(p.h_stage_list[k]);
    if (flags & RS_F_EMPTY) continue;
    const int nsub = (flags & RS_F_TWO) ? 2 : 1;
    out[1] += nsub * kc * b_cols * 2;
    out[3] += nsub * (b_cols / 64);
    for (int sub = 0; sub < nsub; ++sub)
      for (int g = 0; g < 4; ++g)
        if (p.h_stage_list[k + 5 + 4 * sub + g] >= 0) {
          out[0] += Rs * kc * 2;
          out[2] += 1;
        }
  }
}

}  // namespace bsp
