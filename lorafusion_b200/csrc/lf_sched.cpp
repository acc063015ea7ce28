// Host-side packing and sharding of the fused batch.
//
// lf_greedy_pack restates greedy_pack (lorafusion/scheduler/milp_packer.py:36-72) with the same
// output bit for bit; the first-fit search is a max segment tree over the bins' free rows
// (leftmost bin with room in O(log bins)) instead of a linear scan.  lf_assign_rows gives each
// rank its rows for one process per GPU, keeping every adapter on one rank where it fits.
#include <stdint.h>

#include <algorithm>
#include <numeric>
#include <vector>

#include "../../include/lorafusion_b200.h"

namespace {

// Max segment tree over a fixed number of leaves (bins not yet opened hold -1).
class FirstFit {
 public:
  explicit FirstFit(int n) : size_(1) {
    while (size_ < n) size_ <<= 1;
    tree_.assign(2 * size_, -1);
  }
  void set(int i, int v) {
    int k = i + size_;
    tree_[k] = v;
    for (k >>= 1; k >= 1; k >>= 1) tree_[k] = std::max(tree_[2 * k], tree_[2 * k + 1]);
  }
  int get(int i) const { return tree_[i + size_]; }
  // Leftmost leaf with value >= need, or -1.
  int leftmost(int need) const {
    if (tree_[1] < need) return -1;
    int k = 1;
    while (k < size_) k = tree_[2 * k] >= need ? 2 * k : 2 * k + 1;
    return k - size_;
  }

 private:
  int size_;
  std::vector<int> tree_;
};

}  // namespace

extern "C" int lf_greedy_pack(const int32_t* adapter_ids, const int32_t* rows, int32_t n_adapters,
                              int32_t tile_capacity, int32_t max_entries, int32_t* bin_start, int32_t* entry_adapter,
                              int32_t* entry_rows, int32_t* n_entries, int32_t* n_bins) {
  if (tile_capacity <= 0 || n_adapters < 0 || max_entries < 0 || !n_entries || !n_bins) return LF_ERR_INVALID_ARG;
  if (n_adapters > 0 && (!adapter_ids || !rows)) return LF_ERR_INVALID_ARG;
  struct Chunk {
    int32_t adapter, rows;
  };
  std::vector<Chunk> chunks;
  int64_t count = 0;
  for (int32_t a = 0; a < n_adapters; ++a)
    if (rows[a] > 0) count += (static_cast<int64_t>(rows[a]) + tile_capacity - 1) / tile_capacity;
  *n_entries = static_cast<int32_t>(std::min<int64_t>(count, INT32_MAX));
  *n_bins = 0;
  if (count > max_entries) return LF_ERR_CAPACITY;
  if (count > 0 && (!bin_start || !entry_adapter || !entry_rows)) return LF_ERR_INVALID_ARG;
  chunks.reserve(static_cast<size_t>(count));
  for (int32_t a = 0; a < n_adapters; ++a)
    for (int32_t left = rows[a]; left > 0; left -= std::min(left, tile_capacity))
      chunks.push_back({adapter_ids[a], std::min(left, tile_capacity)});
  std::stable_sort(chunks.begin(), chunks.end(), [](const Chunk& x, const Chunk& y) { return x.rows > y.rows; });

  // Place every chunk, remembering its bin; then lay the bins out in CSR order.
  FirstFit ff(static_cast<int>(std::max<int64_t>(count, 1)));
  std::vector<int32_t> bin_of(chunks.size()), bin_count;
  int32_t bins = 0;
  for (size_t i = 0; i < chunks.size(); ++i) {
    int b = ff.leftmost(chunks[i].rows);
    if (b < 0) {
      b = bins++;
      bin_count.push_back(0);
      ff.set(b, tile_capacity);
    }
    ff.set(b, ff.get(b) - chunks[i].rows);
    bin_of[i] = b;
    ++bin_count[b];
  }
  bin_start[0] = 0;
  for (int32_t b = 0; b < bins; ++b) bin_start[b + 1] = bin_start[b] + bin_count[b];
  std::vector<int32_t> fill(bin_start, bin_start + bins);
  for (size_t i = 0; i < chunks.size(); ++i) {  // chunks arrive in each bin's insertion order
    const int32_t e = fill[bin_of[i]]++;
    entry_adapter[e] = chunks[i].adapter;
    entry_rows[e] = chunks[i].rows;
  }
  *n_bins = bins;
  return LF_OK;
}

extern "C" int lf_assign_rows(const int32_t* bin_start, const int32_t* entry_adapter, const int32_t* entry_rows,
                              int32_t n_bins, int32_t world_size, int32_t granule_rows, int32_t max_ranges,
                              int64_t* range_start, int64_t* range_end, int32_t* range_rank, int32_t* n_ranges) {
  if (world_size <= 0 || granule_rows <= 0 || n_bins < 0 || max_ranges < 0 || !n_ranges) return LF_ERR_INVALID_ARG;
  *n_ranges = 0;
  if (n_bins == 0) return LF_OK;
  if (!bin_start || !entry_adapter || !entry_rows) return LF_ERR_INVALID_ARG;
  const int32_t n_entries = bin_start[n_bins];
  // entries in global row order; adapters in order of first appearance
  std::vector<int64_t> e_start(n_entries);
  std::vector<int32_t> adapter_of_entry(n_entries), first_seen;
  std::vector<int32_t> ids(entry_adapter, entry_adapter + n_entries);
  std::sort(ids.begin(), ids.end());
  ids.erase(std::unique(ids.begin(), ids.end()), ids.end());
  const int n_ad = static_cast<int>(ids.size());
  std::vector<int64_t> total_of(n_ad, 0);
  std::vector<int32_t> order_seen(n_ad, -1);
  int64_t cur = 0, total = 0;
  for (int32_t e = 0; e < n_entries; ++e) {
    const int a = static_cast<int>(std::lower_bound(ids.begin(), ids.end(), entry_adapter[e]) - ids.begin());
    adapter_of_entry[e] = a;
    e_start[e] = cur;
    cur += entry_rows[e];
    total_of[a] += entry_rows[e];
    if (order_seen[a] < 0) order_seen[a] = static_cast<int32_t>(first_seen.size()), first_seen.push_back(a);
  }
  total = cur;
  const int64_t share = std::max<int64_t>(1, (total + world_size - 1) / world_size);
  const int64_t cap = (share + granule_rows - 1) / granule_rows * granule_rows;
  // adapters, most rows first (ties: first appearance), to ranks: whole into the rank they fit
  // best (least room left, then lowest rank); an adapter that fits nowhere is cut over the ranks
  // with most room (then lowest rank), each taking what it has room for
  std::vector<int> by_size(first_seen.begin(), first_seen.end());
  std::stable_sort(by_size.begin(), by_size.end(), [&](int x, int y) { return total_of[x] > total_of[y]; });
  std::vector<int64_t> load(world_size, 0);
  std::vector<std::vector<std::pair<int, int64_t>>> parts(n_ad);  // (rank, rows) in order
  for (int a : by_size) {
    int64_t left = total_of[a];
    int best = -1;
    for (int k = 0; k < world_size; ++k)
      if (load[k] + left <= cap && (best < 0 || cap - load[k] - left < cap - load[best] - left)) best = k;
    if (best >= 0) {
      parts[a].push_back({best, left});
      load[best] += left;
      continue;
    }
    while (left > 0) {
      int most = 0;
      for (int k = 1; k < world_size; ++k)
        if (load[k] < load[most]) most = k;
      const int64_t room = cap - load[most];
      const int64_t take = room > 0 ? std::min(room, left) : left;  // no room anywhere: the least-loaded rank
      parts[a].push_back({most, take});
      load[most] += take;
      left -= take;
    }
  }
  // each adapter's rows, in global order, go to its parts in order: emit row ranges
  std::vector<size_t> part_i(n_ad, 0);
  std::vector<int64_t> part_used(n_ad, 0);
  int32_t n = 0;
  auto emit = [&](int64_t s0, int64_t e0, int32_t r) {
    if (n > 0 && n <= max_ranges && range_rank && range_end && range_rank[n - 1] == r && range_end[n - 1] == s0) {
      range_end[n - 1] = e0;  // extend the previous range
      return;
    }
    if (n < max_ranges && range_start && range_end && range_rank) {
      range_start[n] = s0;
      range_end[n] = e0;
      range_rank[n] = r;
    }
    ++n;
  };
  for (int32_t e = 0; e < n_entries; ++e) {
    const int a = adapter_of_entry[e];
    int64_t s0 = e_start[e], rows_left = entry_rows[e];
    while (rows_left > 0) {
      const auto& pr = parts[a][part_i[a]];
      const int64_t take = std::min(rows_left, pr.second - part_used[a]);
      emit(s0, s0 + take, pr.first);
      s0 += take;
      rows_left -= take;
      part_used[a] += take;
      if (part_used[a] == pr.second) {
        ++part_i[a];
        part_used[a] = 0;
      }
    }
  }
  *n_ranges = n;
  return n <= max_ranges ? LF_OK : LF_ERR_CAPACITY;
}
