// fa_common.cuh -- shared geometry and parameter blocks of the attention
// kernels.
#pragma once

#include "sm100_ptx.cuh"

namespace fa {

// Geometry of an (R x D) fp16 tile as a TMA load with swizzle leaves it in
// shared memory: D is cut into boxes of BOX elements (one swizzle row of SW
// bytes each); box b holds rows 0..R-1 of columns [b*BOX, (b+1)*BOX) and sits
// R*SW bytes after box b-1.
template <int D>
struct TileGeom {
  static constexpr int SW = D >= 64 ? 128 : 64;  // swizzle width in bytes
  static constexpr int BOX = SW / 2;             // fp16 elements per box row
  static constexpr int NBOX = D / BOX;
  static_assert(D == 32 || D == 64 || D == 128, "head dim");
};

// Byte offset of the 16-wide K slice `ks` inside a K-major (R x D) tile, and
// of rows [16 ks, 16 ks + 16) inside an MN-major tile (compile-time).
template <int D, int R>
__host__ __device__ constexpr uint32_t k_major_off(int ks) {
  using G = TileGeom<D>;
  return uint32_t((ks * 16) / G::BOX) * uint32_t(R * G::SW) + uint32_t((ks * 16) % G::BOX) * 2u;
}
template <int D>
__host__ __device__ constexpr uint32_t mn_major_off(int ks) {
  return uint32_t(ks) * 16u * uint32_t(TileGeom<D>::SW);
}
// Descriptor bases: advance with sdesc_at(base, k_major_off / mn_major_off).
template <int D>
__device__ __forceinline__ SDesc desc_k_base(uint32_t tile_saddr) {
  using G = TileGeom<D>;
  return sdesc<G::SW>(tile_saddr, 16u, 8u * G::SW);
}
template <int D, int R>
__device__ __forceinline__ SDesc desc_mn_base(uint32_t tile_saddr) {
  using G = TileGeom<D>;
  return sdesc<G::SW>(tile_saddr, uint32_t(R * G::SW), 8u * G::SW);
}

// Problem description shared by the attention kernels (element strides).
struct AttnShape {
  int B, Hq, Hkv, Nq, Nk;
  int q_off, k_off;  // global positions of query row 0 and key row 0
  int causal;
  float scale;       // softmax scale
  float scale_log2;  // scale * log2(e)
  int* status;       // device status word (see CtaCtl)
};

// Number of K/V tiles of width BN a block of query rows [r0, r0 + rows)
// touches; 0 when every key is masked for all of them.
__device__ __forceinline__ int kv_tiles_for_rows(const AttnShape& s, int r0, int rows, int BN) {
  if (r0 >= s.Nq) return 0;
  int last = s.Nk - 1;
  if (s.causal) {
    const int last_row = (r0 + rows < s.Nq ? r0 + rows : s.Nq) - 1;
    const long long lim = (long long)last_row + s.q_off - s.k_off;
    if (lim < 0) return 0;
    if (lim < last) last = int(lim);
  }
  return last / BN + 1;
}

// Persistent kernels: the k-th work unit of CTA c when G CTAs share n units
// numbered heaviest first.  Snake order over rounds of G evens out the work
// per CTA; returns n when the CTA has no k-th unit.
__device__ __forceinline__ int snake_unit(int c, int k, int G, int n) {
  const int t = k * G + ((k & 1) ? G - 1 - c : c);
  return t < n ? t : n;
}

}  // namespace fa
