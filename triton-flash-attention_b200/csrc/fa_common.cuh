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
  // Packed variable-length batches: when cu_q is not null, batch b owns
  // query rows [cu_q[b], cu_q[b+1]) and key rows [cu_k[b], cu_k[b+1]) of
  // tensors packed as (total, heads, D); Nq / Nk are then the longest
  // sequence lengths, and lse / Delta are laid out (Hq, total_q).
  const int* cu_q;
  const int* cu_k;
  int total_q, total_k;
  // Paged K/V (forward only): when block_table is not null, batch b has
  // seqlen_k[b] keys, and key row j lives at row j % page_size of page
  // block_table[b * bt_stride + j / page_size] of the (pages * page_size,
  // Hkv, D) caches; the causal mask is then bottom-right aligned (query i of
  // nq sees keys j <= i + nk - nq), the convention of a KV cache.
  const int* seqlen_k;
  const int* block_table;
  int bt_stride, page_size;
  // Forward only: when pack_g > 1, a 128-row query tile holds pack_g query
  // heads of one K/V head (a GQA group) x 128 / pack_g query rows, so each
  // K/V tile is read once for the whole group (decode, short queries).
  int pack_g;
  // Sliding window (causal only): when window > 0, a query sees only the
  // window keys ending at its own position, j > pos - window.
  int window;
  // Columns of the outputs the kernels store: qk_cols of dQ / dK, v_cols of
  // O / dV.  The kernels compute at their template width D; a narrower
  // tensor (value head size != query/key head size) is read through a tensor
  // map whose extent is its own width, so the TMA fills the missing columns
  // with zeros (they add nothing to Q K^T, P V or the gradients), and its
  // output columns at or past the width are not stored.  Multiples of 32.
  int qk_cols, v_cols;
};

// Dense boolean mask (dense layout only), a kernel parameter of its own so
// that the unmasked kernels keep their parameter block: key k is visible to
// query row r of head h in batch b only if bit (k & 31) of word
// bits[b * sb + h * sh + r * sn + (k >> 5)] is set; a row holds
// roundup(Nk, 128) / 32 words, so a 128-key tile is one aligned 16-byte
// load.  bits_t is the same mask transposed (a row per key, a bit per query,
// roundup(Nq, 128) / 32 words a row) for the kernels whose threads own key
// rows.  Strides in words; a stride of 0 broadcasts.  bits == nullptr: no
// mask.
struct MaskBits {
  const uint32_t* bits = nullptr;
  long long sb = 0, sh = 0, sn = 0;
  const uint32_t* bits_t = nullptr;
  long long tsb = 0, tsh = 0, tsn = 0;
};

// Attention dropout (a kernel parameter of its own): P is kept where the
// position's random byte is at least t (so p = t / 256, t in [1, 255]) and
// the kept values are scaled by r = 1 / (1 - t / 256).  The random bytes are
// a stateless function of (seed, batch * Hq + head, query, key), so the
// forward and the backward kernels regenerate the same ones in any order:
//   key_bh  = mix32(seed_lo ^ mix32(seed_hi + bh * 0x9E3779B9))
//   key2    = mix32(key_bh ^ ((q >> 17) << 16 | (k >> 17)))
//   word    = mix32(key2 ^ (((q >> 1) & 0xFFFF) << 16 | ((k >> 1) & 0xFFFF)))
//   byte    = word >> 8 * (2 * (q & 1) + (k & 1))
// -- one 32-bit word for each 2 x 2 block of (query, key) positions, so a
// thread that owns a query row and one that owns a key row each use two of
// its four bytes.  mix32 is the "lowbias32" integer hash published by
// C. Wellons (hash-prospector): xorshift 16, multiply 0x7feb352d, xorshift
// 15, multiply 0x846ca68b, xorshift 16.  t == 0: no dropout.
struct DropArgs {
  uint32_t t = 0;
  float r = 1.f;
  uint32_t seed_lo = 0, seed_hi = 0;
};

// Split-KV forward (a kernel parameter of its own): the key tiles of every
// unit are cut into n ranges of `tiles` key tiles; range s writes its partial
// O (normalised by its own row sums) at o + s * o_stride and its base-2
// log-sum-exp at lse + s * lse_stride, for a combine pass to merge.
struct SplitArgs {
  int n = 1;
  int tiles = 0;
  long long o_stride = 0;
  long long lse_stride = 0;
};

__host__ __device__ __forceinline__ uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}
__device__ __forceinline__ uint32_t drop_key_bh(const DropArgs& dr, int bh) {
  return mix32(dr.seed_lo ^ mix32(dr.seed_hi + uint32_t(bh) * 0x9E3779B9u));
}
// key2 of the (query, key) positions whose indices agree above bit 16
__device__ __forceinline__ uint32_t drop_key2(uint32_t key_bh, int q, int k) {
  return mix32(key_bh ^ ((uint32_t(q) >> 17) << 16 | (uint32_t(k) >> 17)));
}
__device__ __forceinline__ uint32_t drop_word(uint32_t key2, int q, int k) {
  return mix32(key2 ^ ((((uint32_t(q) >> 1) & 0xFFFFu) << 16) | ((uint32_t(k) >> 1) & 0xFFFFu)));
}
// Lane mask (0xFFFF per kept 16-bit lane) of an element pair: bytes b0 (low
// lane) and b1 (high lane) of word.  sel = b0 | 0x40 | b1 << 8 | 0x4000 moves
// them to bits 0-7 and 16-23 (byte_perm), tt = (256 - t) * 0x10001 carries
// each into bit 8 / 24 iff byte >= t.
__host__ __device__ constexpr uint32_t keep_sel(int b0, int b1) {
  return uint32_t(b0) | 0x40u | (uint32_t(b1) << 8) | 0x4000u;
}
__device__ __forceinline__ uint32_t keep_mask2(uint32_t word, uint32_t sel, uint32_t tt) {
  const uint32_t z = __byte_perm(word, 0u, sel) + tt;
  return ((z >> 8) & 0x00010001u) * 0xFFFFu;
}
// Words of the block pairs (2j, 2j + 1) that lanes l and l ^ 1 share (rows,
// or key rows, 2i and 2i + 1 lie in one 2 x 2 block): this lane hashes the
// one of index 2j + odd and takes the other from its partner.
__device__ __forceinline__ void shared_words(uint32_t mine, int odd, uint32_t& w_even, uint32_t& w_odd) {
  const uint32_t other = __shfl_xor_sync(0xffffffffu, mine, 1);
  w_even = odd ? other : mine;
  w_odd = odd ? mine : other;
}

// Hides the columns of s whose bit in words is clear (bit c & 31 of word
// c >> 5; 1 = visible).
template <int N>
__device__ __forceinline__ void apply_mask_bits(float (&s)[N], const uint32_t (&words)[(N + 31) / 32]) {
#pragma unroll
  for (int c = 0; c < N; ++c) s[c] = ((words[c >> 5] >> (c & 31)) & 1u) ? s[c] : -INFINITY;
}

// Rows of batch b: query rows [q0, q0 + nq) and key rows [k0, k0 + nk) of
// the tensors, and tb, b's coordinate in the 4-D tensor maps (0 when packed).
struct Seq {
  int q0, nq, k0, nk, tb;
  int diag;  // added to a query's position for the causal limit (bottom-right alignment)
};
__device__ __forceinline__ Seq seq_of(const AttnShape& s, int b) {
  Seq r;
  r.diag = 0;
  if (s.cu_q) {
    r.q0 = __ldg(s.cu_q + b);
    r.nq = __ldg(s.cu_q + b + 1) - r.q0;
    if (s.block_table) {
      r.k0 = 0;
      r.nk = __ldg(s.seqlen_k + b);
      r.diag = r.nk - r.nq;
    } else {
      r.k0 = __ldg(s.cu_k + b);
      r.nk = __ldg(s.cu_k + b + 1) - r.k0;
    }
    r.tb = 0;
  } else {
    r.q0 = 0;
    r.nq = s.Nq;
    r.k0 = 0;
    r.nk = s.Nk;
    r.tb = b;
  }
  return r;
}
// Compile-time variants for kernels instantiated per layout: VL = packed.
template <bool VL>
__device__ __forceinline__ Seq seq_of_v(const AttnShape& s, int b) {
  if constexpr (VL) {
    Seq r;
    r.diag = 0;
    r.q0 = __ldg(s.cu_q + b);
    r.nq = __ldg(s.cu_q + b + 1) - r.q0;
    r.k0 = __ldg(s.cu_k + b);
    r.nk = __ldg(s.cu_k + b + 1) - r.k0;
    r.tb = 0;
    return r;
  } else {
    Seq r;
    r.q0 = 0;
    r.nq = s.Nq;
    r.k0 = 0;
    r.nk = s.Nk;
    r.tb = b;
    r.diag = 0;
    return r;
  }
}
template <bool VL>
__device__ __forceinline__ long long row_stat_index_v(const AttnShape& s, const Seq& q, int b, int h, int r) {
  if constexpr (VL) return (long long)h * s.total_q + q.q0 + r;
  else return ((long long)b * s.Hq + h) * s.Nq + r;
}
// Index of query row r (local to batch b) of head h in lse / Delta.
__device__ __forceinline__ long long row_stat_index(const AttnShape& s, const Seq& q, int b, int h, int r) {
  return s.cu_q ? (long long)h * s.total_q + q.q0 + r : ((long long)b * s.Hq + h) * s.Nq + r;
}

// Number of K/V tiles of width BN a block of query rows [r0, r0 + rows) of
// a batch touches; 0 when every key is masked for all of them.
__device__ __forceinline__ int kv_tiles_for_rows(const AttnShape& s, const Seq& q, int r0, int rows, int BN) {
  if (r0 >= q.nq || q.nk <= 0) return 0;
  int last = q.nk - 1;
  if (s.causal) {
    const int last_row = (r0 + rows < q.nq ? r0 + rows : q.nq) - 1;
    const long long lim = (long long)last_row + s.q_off - s.k_off + q.diag;
    if (lim < 0) return 0;
    if (lim < last) last = int(lim);
  }
  return last / BN + 1;
}

// First K/V tile of width BN that a block of query rows starting at r0 of a
// batch touches: 0 unless a sliding window hides the keys before it.
__device__ __forceinline__ int kv_first_tile(const AttnShape& s, const Seq& q, int r0, int BN) {
  if (s.window <= 0) return 0;
  const long long lo = (long long)r0 + s.q_off - s.k_off + q.diag - s.window + 1;  // first visible key
  return lo <= 0 ? 0 : int(lo / BN);
}

// Persistent kernels: the k-th work unit of CTA c when G CTAs share n units
// numbered heaviest first.  Snake order over rounds of G evens out the work
// per CTA; returns n when the CTA has no k-th unit.
__device__ __forceinline__ int snake_unit(int c, int k, int G, int n) {
  const int t = k * G + ((k & 1) ? G - 1 - c : c);
  return t < n ? t : n;
}

}  // namespace fa
