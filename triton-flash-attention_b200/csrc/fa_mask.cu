// fa_mask.cu -- packs a dense boolean attention mask into the bit rows the
// attention kernels read (AttnShape::mask and mask_t).
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
    uint32_t tword = 0, row_word = 0;
#pragma unroll 4
    for (int i = 0; i < 32; ++i) {
      const int q = qb * 32 + i;
      const bool bit = k_in && q < Nq && col[(long long)q * sq] != 0;
      const uint32_t w = __ballot_sync(0xffffffffu, bit);
      if (lane == i) row_word = w;
      tword |= uint32_t(bit) << i;
    }
    const int q = qb * 32 + lane;
    if (q < Nq) bits[(bh * Nq + q) * words_k + kb] = row_word;
    if (k_in) bits_t[(bh * Nk + k) * words_q + qb] = tword;
  }
}

int launch_mask_pack(const void* mask, long long sb, long long sh, long long sq, long long sk, int Bm, int Hm, int Nq,
                     int Nk, uint32_t* bits, uint32_t* bits_t, cudaStream_t stream) {
  const int words_k = (Nk + 127) / 128 * 4;
  const int words_q = (Nq + 127) / 128 * 4;
  const long long n_blocks = (long long)Bm * Hm * words_q * words_k;
  long long ctas = (n_blocks + 7) / 8;  // 8 warps a CTA
  const long long cap = (long long)device_sm_count() * 16;
  if (ctas > cap) ctas = cap;
  if (ctas < 1) ctas = 1;
  fa_mask_pack_kernel<<<unsigned(ctas), 256, 0, stream>>>(static_cast<const uint8_t*>(mask), sb, sh, sq, sk, Hm, Nq,
                                                          Nk, words_k, words_q, bits, bits_t, n_blocks);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

}  // namespace fa
