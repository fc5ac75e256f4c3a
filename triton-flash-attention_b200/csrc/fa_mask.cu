// fa_mask.cu -- packs a dense boolean attention mask into the bit rows the
// attention kernels read (MaskBits::bits and bits_t).
//
// The input is a byte per (query, key) position (a torch.bool tensor; any
// nonzero byte = visible) with arbitrary element strides, so broadcast
// dimensions (stride 0) need no copy.  The output is two bit matrices per
// (batch, head) of the mask:
//   bits   (Nq rows of roundup(Nk, 128) / 32 words): bit k & 31 of word k >> 5
//          of row q is position (q, k) -- read by the kernels whose threads
//          own query rows (forward, dQ);
//   bits_t (Nk rows of roundup(Nq, 128) / 32 words): the transpose -- read by
//          the kernels whose threads own key rows (dK/dV, fused backward).
// Rows are padded to whole 128-position tiles with zero bits (hidden), so a
// tile's bits are one aligned 16-byte load.
#include "fa_kernels.h"

namespace fa {

// One warp per 32 x 32 block of positions: lane l holds key k0 + l and reads
// the block's 32 query rows (32 consecutive bytes per row when the key
// stride is 1).  A ballot per row yields that row's word of bits; each lane
// gathers its key's 32 query bits into the word of bits_t.  Positions past
// Nq or Nk read as hidden.  Every word of both outputs is written.
__global__ void __launch_bounds__(256)
    fa_mask_pack_kernel(const uint8_t* __restrict__ m, long long sb, long long sh, long long sq, long long sk, int Hm,
                        int Nq, int Nk, int words_k, int words_q, uint32_t* __restrict__ bits,
                        uint32_t* __restrict__ bits_t, long long n_blocks) {
  const int lane = threadIdx.x & 31;
  const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long blk = warp0; blk < n_blocks; blk += n_warps) {  // uniform per warp
    const int kb = int(blk % words_k);
    const long long rest = blk / words_k;
    const int qb = int(rest % words_q);
    const long long bh = rest / words_q;
    const long long b = bh / Hm;
    const long long h = bh % Hm;
    const int k = kb * 32 + lane;
    const bool k_in = k < Nk;
    const uint8_t* col = m + b * sb + h * sh + (k_in ? (long long)k * sk : 0);
    // all 32 loads first, so that they are in flight together
    uint32_t byte[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int q = qb * 32 + i;
      byte[i] = (k_in && q < Nq) ? uint32_t(__ldg(col + (long long)q * sq)) : 0u;
    }
    uint32_t tword = 0, row_word = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const bool bit = byte[i] != 0;
      const uint32_t w = __ballot_sync(0xffffffffu, bit);
      if (lane == i) row_word = w;
      tword |= uint32_t(bit) << i;
    }
    const int q = qb * 32 + lane;
    if (q < Nq) bits[(bh * Nq + q) * words_k + kb] = row_word;
    if (k_in) bits_t[(bh * Nk + k) * words_q + qb] = tword;
  }
}

// Bits 0..7 of x moved to bits 0, 4, 8, ..., 28.
__device__ __forceinline__ uint32_t spread4(uint32_t x) {
  x = (x | (x << 12)) & 0x000F000Fu;
  x = (x | (x << 6)) & 0x03030303u;
  x = (x | (x << 3)) & 0x11111111u;
  return x;
}

// The same packing, 4 bytes a lane: one warp per 32 query rows x one
// 128-key tile.  Lane l loads keys 4l .. 4l+3 of each row (one 128-byte line
// per row and load); four ballots per row (one per byte position) hold the
// row's 128 bits, which lane i interleaves into the row's 4 words and
// stores as one 16-byte store; each lane also gathers its 4 keys' 32 query
// bits for bits_t.  Needs a key stride of 1, 4-byte aligned rows and Nk a
// multiple of 4 (checked by the host).
__global__ void __launch_bounds__(256)
    fa_mask_pack_vec_kernel(const uint8_t* __restrict__ m, long long sb, long long sh, long long sq, int Hm, int Nq,
                            int Nk, int words_k, int words_q, uint32_t* __restrict__ bits,
                            uint32_t* __restrict__ bits_t, long long n_blocks) {
  const int lane = threadIdx.x & 31;
  const int tiles_k = words_k / 4;
  const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long blk = warp0; blk < n_blocks; blk += n_warps) {  // uniform per warp
    const int kt = int(blk % tiles_k);
    const long long rest = blk / tiles_k;
    const int qb = int(rest % words_q);
    const long long bh = rest / words_q;
    const long long b = bh / Hm;
    const long long h = bh % Hm;
    const int k = kt * 128 + 4 * lane;  // this lane's first key
    const bool k_in = k < Nk;           // Nk % 4 == 0: all four keys or none
    const uint8_t* col = m + b * sb + h * sh + (k_in ? k : 0);
    uint32_t v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int q = qb * 32 + i;
      v[i] = (k_in && q < Nq) ? __ldg(reinterpret_cast<const uint32_t*>(col + (long long)q * sq)) : 0u;
    }
    uint32_t t0 = 0, t1 = 0, t2 = 0, t3 = 0;  // bits_t words of keys k .. k+3
    uint32_t r0 = 0, r1 = 0, r2 = 0, r3 = 0;  // ballots of row qb*32 + lane
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const bool e0 = (v[i] & 0x000000FFu) != 0, e1 = (v[i] & 0x0000FF00u) != 0;
      const bool e2 = (v[i] & 0x00FF0000u) != 0, e3 = (v[i] & 0xFF000000u) != 0;
      const uint32_t b0 = __ballot_sync(0xffffffffu, e0), b1 = __ballot_sync(0xffffffffu, e1);
      const uint32_t b2 = __ballot_sync(0xffffffffu, e2), b3 = __ballot_sync(0xffffffffu, e3);
      if (lane == i) {
        r0 = b0;
        r1 = b1;
        r2 = b2;
        r3 = b3;
      }
      t0 |= uint32_t(e0) << i;
      t1 |= uint32_t(e1) << i;
      t2 |= uint32_t(e2) << i;
      t3 |= uint32_t(e3) << i;
    }
    // word j of the row: keys 32j .. 32j+31 = lanes 8j .. 8j+7, key 4l + c at bit 4(l - 8j) + c
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      w[j] = spread4((r0 >> (8 * j)) & 0xFFu) | (spread4((r1 >> (8 * j)) & 0xFFu) << 1) |
             (spread4((r2 >> (8 * j)) & 0xFFu) << 2) | (spread4((r3 >> (8 * j)) & 0xFFu) << 3);
    const int q = qb * 32 + lane;
    if (q < Nq)
      *reinterpret_cast<uint4*>(bits + (bh * Nq + q) * words_k + kt * 4) = make_uint4(w[0], w[1], w[2], w[3]);
    if (k_in) {
      uint32_t* dst = bits_t + (bh * Nk + k) * words_q + qb;
      dst[0] = t0;
      dst[words_q] = t1;
      dst[2 * words_q] = t2;
      dst[3 * words_q] = t3;
    }
  }
}

int launch_mask_pack(const void* mask, long long sb, long long sh, long long sq, long long sk, int Bm, int Hm, int Nq,
                     int Nk, uint32_t* bits, uint32_t* bits_t, cudaStream_t stream) {
  const int words_k = (Nk + 127) / 128 * 4;
  const int words_q = (Nq + 127) / 128 * 4;
  const long long cap = (long long)device_sm_count() * 16;
  const uintptr_t addr = reinterpret_cast<uintptr_t>(mask);
  if (sk == 1 && Nk % 4 == 0 && addr % 4 == 0 && sb % 4 == 0 && sh % 4 == 0 && sq % 4 == 0) {
    const long long n_blocks = (long long)Bm * Hm * words_q * (words_k / 4);
    long long ctas = (n_blocks + 7) / 8;  // 8 warps a CTA
    if (ctas > cap) ctas = cap;
    if (ctas < 1) ctas = 1;
    fa_mask_pack_vec_kernel<<<unsigned(ctas), 256, 0, stream>>>(static_cast<const uint8_t*>(mask), sb, sh, sq, Hm,
                                                                Nq, Nk, words_k, words_q, bits, bits_t, n_blocks);
    return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
  }
  const long long n_blocks = (long long)Bm * Hm * words_q * words_k;
  long long ctas = (n_blocks + 7) / 8;  // 8 warps a CTA
  if (ctas > cap) ctas = cap;
  if (ctas < 1) ctas = 1;
  fa_mask_pack_kernel<<<unsigned(ctas), 256, 0, stream>>>(static_cast<const uint8_t*>(mask), sb, sh, sq, sk, Hm, Nq,
                                                          Nk, words_k, words_q, bits, bits_t, n_blocks);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

}  // namespace fa
