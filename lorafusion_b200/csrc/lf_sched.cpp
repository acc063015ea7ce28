// Host-side packing and sharding of the fused batch.
//
// lf_greedy_pack restates greedy_pack (lorafusion/scheduler/milp_packer.py:36-72) with the same
// output bit for bit; the first-fit search is a max segment tree over the bins' free rows
// (leftmost bin with room in O(log bins)) instead of a linear scan.  lf_assign_bins gives each
// rank whole bins for one process per GPU.
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

extern "C" int lf_assign_bins(const int32_t* bin_start, const int32_t* entry_adapter, const int32_t* entry_rows,
                              int32_t n_bins, int32_t world_size, int32_t granule_rows, int32_t* bin_rank) {
  if (world_size <= 0 || granule_rows <= 0 || n_bins < 0) return LF_ERR_INVALID_ARG;
  if (n_bins == 0) return LF_OK;
  if (!bin_start || !entry_adapter || !entry_rows || !bin_rank) return LF_ERR_INVALID_ARG;
  std::vector<int64_t> rows(n_bins, 0);
  std::vector<int32_t> adapter_of(n_bins, 0);  // the bin's adapter when `single`
  std::vector<char> single(n_bins, 0);          // every entry of the bin holds one and the same adapter
  int64_t total = 0;
  for (int32_t b = 0; b < n_bins; ++b) {
    single[b] = bin_start[b + 1] > bin_start[b];
    for (int32_t e = bin_start[b]; e < bin_start[b + 1]; ++e) {
      rows[b] += entry_rows[e];
      if (e == bin_start[b]) adapter_of[b] = entry_adapter[e];
      else if (entry_adapter[e] != adapter_of[b]) single[b] = 0;
    }
    total += rows[b];
  }
  const int64_t share = std::max<int64_t>(1, (total + world_size - 1) / world_size);
  const int64_t cap = (share + granule_rows - 1) / granule_rows * granule_rows;

  // Bundles: runs of consecutive bins of one single adapter, at most `share` rows each; a bin
  // with several adapters (or none) is a bundle of its own.
  std::vector<std::vector<int32_t>> bundles;
  std::vector<int32_t> cur;
  int32_t cur_adapter = 0;
  int64_t cur_rows = 0;
  for (int32_t b = 0; b < n_bins; ++b) {
    if (!cur.empty() && (!single[b] || adapter_of[b] != cur_adapter || cur_rows + rows[b] > share)) {
      bundles.push_back(cur);
      cur.clear();
      cur_rows = 0;
    }
    cur.push_back(b);
    cur_rows += rows[b];
    cur_adapter = adapter_of[b];
    if (!single[b]) {
      bundles.push_back(cur);
      cur.clear();
      cur_rows = 0;
    }
  }
  if (!cur.empty()) bundles.push_back(cur);

  std::vector<int64_t> bundle_rows(bundles.size(), 0);
  for (size_t i = 0; i < bundles.size(); ++i)
    for (int32_t b : bundles[i]) bundle_rows[i] += rows[b];
  std::vector<size_t> order(bundles.size());
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(),
                   [&](size_t x, size_t y) { return bundle_rows[x] > bundle_rows[y]; });
  std::vector<int64_t> load(world_size, 0);
  auto place = [&](const std::vector<int32_t>& members, int64_t n) {
    int best = -1;
    for (int k = 0; k < world_size; ++k)
      if (load[k] + n <= cap && (best < 0 || cap - load[k] - n < cap - load[best] - n)) best = k;
    if (best < 0) return false;
    for (int32_t b : members) bin_rank[b] = best;
    load[best] += n;
    return true;
  };
  for (size_t i : order) {
    if (place(bundles[i], bundle_rows[i])) continue;
    std::vector<int32_t> members = bundles[i];
    std::stable_sort(members.begin(), members.end(), [&](int32_t x, int32_t y) { return rows[x] > rows[y]; });
    for (int32_t b : members) {
      if (place({b}, rows[b])) continue;
      int least = 0;
      for (int k = 1; k < world_size; ++k)
        if (load[k] < load[least]) least = k;
      bin_rank[b] = least;
      load[least] += rows[b];
    }
  }
  return LF_OK;
}
