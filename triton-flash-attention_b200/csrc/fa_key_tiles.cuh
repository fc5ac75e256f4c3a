// fa_key_tiles.cuh -- the work decomposition shared by the key-row-major
// backward kernels (dK/dV, and the fused passes that also produce dQ).
//
// A work tile is BM keys of one (batch, kv head); its items are the (query
// head of the group, BQ-row query tile) pairs that see those keys, in the
// order head-major, then query tile.  Under a causal mask a tile starts at
// the first query tile holding a row at or after its first key, as the
// reference's dK/dV loop does (triton_flash_attention/attention.py:428-505,
// start_n .. N_CTX); a sliding window (packed layout only) also ends it at
// the last query that sees the tile's last key.  Tiles are numbered key
// tile major, so snake_unit's heaviest-first order walks the causally
// longest tiles first.
#pragma once

#include "fa_common.cuh"

namespace fa {

struct KeyTile {
  int kv0, b, kvh, i_start, per_head, n_items;
  Seq sq;
};

template <bool VL, int BM, int BQ>
__device__ __forceinline__ KeyTile key_tile_of(const AttnShape& shp, int t) {
  const int BHkv = shp.B * shp.Hkv;
  const int kv_tile = t / BHkv;
  const int bhk = t % BHkv;
  KeyTile w;
  w.b = bhk / shp.Hkv;
  w.kvh = bhk % shp.Hkv;
  w.kv0 = kv_tile * BM;
  w.sq = seq_of_v<VL>(shp, w.b);
  const int n_qt = w.kv0 < w.sq.nk ? (w.sq.nq + BQ - 1) / BQ : 0;
  int i_start = 0;
  if (shp.causal) {
    // first query tile holding a row at or after this tile's first key
    const long long first_row = (long long)w.kv0 + shp.k_off - shp.q_off;
    i_start = first_row <= 0 ? 0 : int(first_row / BQ);
    if (i_start > n_qt) i_start = n_qt;
  }
  int n_qt_w = n_qt;
  if (VL && shp.causal && shp.window > 0) {  // windows come with the packed layout only
    // sliding window: the last query that sees this tile's last key
    const long long last_row = (long long)w.kv0 + BM - 1 + shp.window - 1 + shp.k_off - shp.q_off;
    const long long i_end = last_row < 0 ? 0 : last_row / BQ + 1;
    if (i_end < n_qt_w) n_qt_w = int(i_end);
  }
  w.i_start = i_start;
  w.per_head = n_qt_w > i_start ? n_qt_w - i_start : 0;
  w.n_items = w.per_head * (shp.Hq / shp.Hkv);
  return w;
}

// Walks the items of a CTA's non-empty tiles in issue order (the producers
// use it to fetch an item's lse2 / Delta a few items ahead).
template <bool VL, int BM, int BQ>
struct KeyItemCursor {
  int k, it;
  KeyTile w;
  // the first item of the first non-empty tile at snake position >= k
  __device__ __forceinline__ bool seek(const AttnShape& shp, int cta, int n_cta, int n_tiles) {
    for (;; ++k) {
      const int t = snake_unit(cta, k, n_cta, n_tiles);
      if (t >= n_tiles) return false;
      w = key_tile_of<VL, BM, BQ>(shp, t);
      if (w.n_items > 0) {
        it = 0;
        return true;
      }
    }
  }
  __device__ __forceinline__ bool next(const AttnShape& shp, int cta, int n_cta, int n_tiles) {
    if (++it < w.n_items) return true;
    ++k;
    return seek(shp, cta, n_cta, n_tiles);
  }
};

}  // namespace fa
