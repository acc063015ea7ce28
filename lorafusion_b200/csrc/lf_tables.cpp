// Host-side routing tables: routes (contiguous row ranges -> adapter slot) are cut
// along the fixed 128-row tile grid of the fused batch into "segment tiles"
// (route x tile).  Every kernel walks these tables; no kernel needs per-row lookups.
//
// Follows the route semantics of lorafusion/ops/config.py:29-69 (TileRoute,
// TileRoutingConfig.validate) and the per-route work of lorafusion/ops/mock_ops.py:40-46,71-93.
#include <algorithm>
#include <cstring>
#include <numeric>
#include <vector>

#include "../../include/lorafusion_b200.h"

namespace {

constexpr int kMaxSlotRank = 64;  // largest rank one (virtual) slot carries

int pad_rank(int r) {
  if (r <= 16) return 16;
  if (r <= 32) return 32;
  return 64;
}

}  // namespace

extern "C" int32_t lf_plan_table_words(int32_t n_routes, int32_t total_rows, int32_t n_slots) {
  if (n_routes < 0 || total_rows < 0 || n_slots < 0) return -1;
  const int64_t n_tiles = (static_cast<int64_t>(total_rows) + LF_TILE_ROWS - 1) / LF_TILE_ROWS;
  // every route adds at most (tiles it spans) segment tiles; sum <= n_routes + n_tiles
  const int64_t n_st = static_cast<int64_t>(n_routes) + n_tiles;
  const int64_t n_pairs = (n_tiles + 1) / 2;
  const int64_t words = (n_tiles + 1) + 6 * n_st + (n_slots + 1) + n_st + n_slots + (n_slots + 1) + n_slots +
                        3 * n_st + (n_pairs + 1) + 3 * n_st + (n_tiles + 1) + 16;
  return words > 0x7fffffff ? -1 : static_cast<int32_t>(words);
}

extern "C" int lf_plan_tables(const int32_t* route_start, const int32_t* route_end, const int32_t* route_slot,
                              int32_t n_routes, int32_t total_rows, const int32_t* slot_rank,
                              const float* slot_scale, int32_t n_slots, int32_t* table, int32_t table_capacity,
                              lf_plan_info* info) {
  if (!info || !table || n_routes < 0 || total_rows < 0 || n_slots < 0) return LF_ERR_INVALID_ARG;
  if (n_routes > 0 && (!route_start || !route_end || !route_slot)) return LF_ERR_INVALID_ARG;
  if (n_slots > 0 && (!slot_rank || !slot_scale)) return LF_ERR_INVALID_ARG;
  std::memset(info, 0, sizeof(*info));

  // validation: same checks as TileRoutingConfig.validate, plus slot range
  int64_t expect = 0;
  for (int32_t i = 0; i < n_routes; ++i) {
    if (route_start[i] != expect) return LF_ERR_ROUTING;
    if (route_end[i] < route_start[i]) return LF_ERR_ROUTING;
    if (route_slot[i] < 0 || route_slot[i] >= n_slots) return LF_ERR_ROUTING;
    expect = route_end[i];
  }
  if (expect != total_rows) return LF_ERR_ROUTING;

  // A slot of rank r > 64 becomes ceil(r / 64) consecutive virtual slots of ranks 64, ..., 64 and
  // the remainder, over the same rows: y = sum over chunks c of s (x A_c^T) B_c^T is the same
  // product, and every kernel adds all the LoRA terms of a row.  `vslot0[s]` is the first virtual
  // slot of input slot s; the tables and info->n_slots count virtual slots.
  std::vector<int32_t> vslot0(n_slots + 1, 0), vrank, vslot_of;
  int max_rank = 1;
  for (int32_t s = 0; s < n_slots; ++s) {
    if (slot_rank[s] <= 0) return LF_ERR_INVALID_ARG;
    max_rank = std::max(max_rank, static_cast<int>(slot_rank[s]));
    for (int32_t c0 = 0; c0 < slot_rank[s]; c0 += kMaxSlotRank) {
      vrank.push_back(std::min(kMaxSlotRank, slot_rank[s] - c0));
      vslot_of.push_back(s);
    }
    vslot0[s + 1] = static_cast<int32_t>(vrank.size());
  }
  const int32_t n_vslots = static_cast<int32_t>(vrank.size());
  const int r_pad = pad_rank(std::min(max_rank, kMaxSlotRank));

  const int32_t n_tiles = (total_rows + LF_TILE_ROWS - 1) / LF_TILE_ROWS;

  // segment tiles in route order == row order (the virtual slots of a route one after another)
  std::vector<int32_t> st_tile, st_lo, st_hi, st_slot, st_route;
  std::vector<int32_t> tile_first(n_tiles + 1, 0);
  for (int32_t i = 0; i < n_routes; ++i) {
    int32_t r0 = route_start[i], r1 = route_end[i];
    while (r0 < r1) {
      const int32_t t = r0 / LF_TILE_ROWS;
      const int32_t tile_end = std::min<int64_t>(static_cast<int64_t>(t + 1) * LF_TILE_ROWS, r1);
      for (int32_t v = vslot0[route_slot[i]]; v < vslot0[route_slot[i] + 1]; ++v) {
        st_tile.push_back(t);
        st_lo.push_back(r0 - t * LF_TILE_ROWS);
        st_hi.push_back(tile_end - t * LF_TILE_ROWS);
        st_slot.push_back(v);
        st_route.push_back(i);
      }
      r0 = tile_end;
    }
  }
  n_slots = n_vslots;  // from here on: virtual slots
  const int32_t n_st = static_cast<int32_t>(st_tile.size());
  for (int32_t j = 0; j < n_st; ++j) tile_first[st_tile[j] + 1]++;
  for (int32_t t = 0; t < n_tiles; ++t) tile_first[t + 1] += tile_first[t];

  // per-slot lists (route order)
  std::vector<int32_t> slot_first(n_slots + 1, 0), slot_list(n_st);
  for (int32_t j = 0; j < n_st; ++j) slot_first[st_slot[j] + 1]++;
  for (int32_t s = 0; s < n_slots; ++s) slot_first[s + 1] += slot_first[s];
  {
    std::vector<int32_t> fill(slot_first.begin(), slot_first.end() - 1);
    for (int32_t j = 0; j < n_st; ++j) slot_list[fill[st_slot[j]]++] = j;
  }
  std::vector<int32_t> rank_prefix(n_slots + 1, 0);
  for (int32_t s = 0; s < n_slots; ++s) rank_prefix[s + 1] = rank_prefix[s] + vrank[s];
  std::vector<int32_t> order(n_slots);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) {
    return (slot_first[a + 1] - slot_first[a]) > (slot_first[b + 1] - slot_first[b]);
  });

  // shrink units: runs of consecutive segment tiles of one row tile, N = run * r_pad <= 64
  const int32_t group = std::max(1, 64 / r_pad);
  std::vector<int32_t> u_tile, u_st0, u_nst, tile_unit(n_tiles + 1, 0);
  for (int32_t t = 0; t < n_tiles; ++t) {
    tile_unit[t] = static_cast<int32_t>(u_tile.size());
    for (int32_t j = tile_first[t]; j < tile_first[t + 1]; j += group) {
      u_tile.push_back(t);
      u_st0.push_back(j);
      u_nst.push_back(std::min(group, tile_first[t + 1] - j));
    }
  }
  const int32_t n_units = static_cast<int32_t>(u_tile.size());
  tile_unit[n_tiles] = n_units;

  // pair LoRA stages: segment tiles of row tiles 2p and 2p+1 matched by slot, in row order
  const int32_t n_pairs = (n_tiles + 1) / 2;
  std::vector<int32_t> pair_first(n_pairs + 1, 0), pl_a, pl_b, pl_slot;
  for (int32_t p = 0; p < n_pairs; ++p) {
    const int32_t t0 = 2 * p, t1 = 2 * p + 1;
    const int32_t a_b = tile_first[t0], a_e = tile_first[t0 + 1];
    const int32_t b_b = t1 < n_tiles ? tile_first[t1] : 0, b_e = t1 < n_tiles ? tile_first[t1 + 1] : 0;
    std::vector<char> used(static_cast<size_t>(std::max(0, b_e - b_b)), 0);
    for (int32_t j = a_b; j < a_e; ++j) {
      int32_t match = n_st;
      for (int32_t k = b_b; k < b_e; ++k)
        if (!used[k - b_b] && st_slot[k] == st_slot[j]) {
          match = k;
          used[k - b_b] = 1;
          break;
        }
      pl_a.push_back(j);
      pl_b.push_back(match);
      pl_slot.push_back(st_slot[j]);
    }
    for (int32_t k = b_b; k < b_e; ++k)
      if (!used[k - b_b]) {
        pl_a.push_back(n_st);
        pl_b.push_back(k);
        pl_slot.push_back(st_slot[k]);
      }
    pair_first[p + 1] = static_cast<int32_t>(pl_a.size());
  }
  const int32_t n_pl = static_cast<int32_t>(pl_a.size());

  // lay out the sections
  int32_t w = 0;
  auto take = [&](int32_t n) {
    const int32_t o = w;
    w += n;
    return o;
  };
  info->off_tile_st = take(n_tiles + 1);
  info->off_st_tile = take(n_st);
  info->off_st_lo = take(n_st);
  info->off_st_hi = take(n_st);
  info->off_st_slot = take(n_st);
  info->off_st_route = take(n_st);
  info->off_st_scale = take(n_st);
  info->off_slot_st = take(n_slots + 1);
  info->off_slot_list = take(n_st);
  info->off_slot_rank = take(n_slots);
  info->off_rank_prefix = take(n_slots + 1);
  info->off_slot_order = take(n_slots);
  info->off_unit_tile = take(n_units);
  info->off_unit_st0 = take(n_units);
  info->off_unit_nst = take(n_units);
  info->off_pair_lora = take(n_pairs + 1);
  info->off_pl_a = take(n_pl);
  info->off_pl_b = take(n_pl);
  info->off_pl_slot = take(n_pl);
  info->off_tile_unit = take(n_tiles + 1);
  if (w > table_capacity) {
    info->table_words = w;  // what a retry needs
    return LF_ERR_CAPACITY;
  }

  auto put = [&](int32_t off, const std::vector<int32_t>& v) {
    if (!v.empty()) std::memcpy(table + off, v.data(), v.size() * sizeof(int32_t));
  };
  put(info->off_tile_st, tile_first);
  put(info->off_st_tile, st_tile);
  put(info->off_st_lo, st_lo);
  put(info->off_st_hi, st_hi);
  put(info->off_st_slot, st_slot);
  put(info->off_st_route, st_route);
  for (int32_t j = 0; j < n_st; ++j) {
    const float s = slot_scale[vslot_of[st_slot[j]]];
    std::memcpy(table + info->off_st_scale + j, &s, sizeof(float));
  }
  put(info->off_slot_st, slot_first);
  put(info->off_slot_list, slot_list);
  put(info->off_slot_rank, vrank);
  put(info->off_rank_prefix, rank_prefix);
  put(info->off_slot_order, order);
  put(info->off_unit_tile, u_tile);
  put(info->off_unit_st0, u_st0);
  put(info->off_unit_nst, u_nst);
  put(info->off_pair_lora, pair_first);
  put(info->off_pl_a, pl_a);
  put(info->off_pl_b, pl_b);
  put(info->off_pl_slot, pl_slot);
  put(info->off_tile_unit, tile_unit);
  info->n_pair_lora = n_pl;

  info->total_rows = total_rows;
  info->n_routes = n_routes;
  info->n_slots = n_slots;
  info->n_tiles = n_tiles;
  info->n_segtiles = n_st;
  info->r_pad = r_pad;
  info->max_rank = max_rank;
  info->rank_total = rank_prefix[n_slots];
  info->n_shrink_units = n_units;
  info->table_words = w;
  return LF_OK;
}
