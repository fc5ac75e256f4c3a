// fa_kernels.h -- internal launch interface between the C ABI (fa_capi.cu)
// and the kernel translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include "../../include/fa_b200.h"
#include "fa_common.cuh"

namespace fa {

// Operand element types (dtype fields below).
enum : int { DT_F16 = 0, DT_BF16 = 1 };

struct FwdArgs {
  CUtensorMap tmap_q, tmap_k, tmap_v;  // 4-D {D, N, H, B}, box {<=64, 128, 1, 1}
  AttnShape shape;
  int dtype;  // DT_F16 or DT_BF16: q, k, v and o
  void* o;
  long long o_sb, o_sh, o_sn;
  float* lse;
  MaskBits mask;  // dense boolean mask (bits == nullptr: none)
  DropArgs drop;  // attention dropout (t == 0: none)
  SplitArgs split;  // split-KV partial outputs (n == 1: none)
  cudaStream_t stream;
};

struct BwdArgs {
  CUtensorMap tmap_q, tmap_k, tmap_v, tmap_do;  // 4-D maps of the operand type
  AttnShape shape;
  int dtype;  // DT_F16 or DT_BF16: q, k, v, dO and the non-fp32 outputs
  const float* lse;
  const float* delta;
  void* dq;  // fa_bwd_dq output (operand type, or fp32 when accumulate_fp32)
  long long dq_sb, dq_sh, dq_sn;
  void* dk;
  void* dv;
  long long dk_sb, dk_sh, dk_sn;
  long long dv_sb, dv_sh, dv_sn;
  int accumulate_fp32;
  MaskBits mask;  // dense boolean mask (bits == nullptr: none)
  DropArgs drop;  // attention dropout (t == 0: none)
  cudaStream_t stream;
};

// Number of SMs of the current device (cached per device); persistent
// kernels launch at most one CTA per SM.
inline int device_sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// The text of the CUDA runtime error behind the last FA_ERR_CUDA status
// (cudaGetErrorString's static string), for fa_status_string.
void record_cuda_error(cudaError_t e);
const char* last_cuda_error_text();

int launch_fwd(const FwdArgs& a, int D);
int launch_bwd_dq(const BwdArgs& a, int D);
int launch_bwd_dkdv(const BwdArgs& a, int D);
// zero_acc: when not null, the contiguous [B, H, N, D] fp32 buffer is zeroed
// on the way (the fused backward's dQ accumulator).
int launch_bwd_delta(const void* o, long long o_sb, long long o_sh, long long o_sn, const void* dO,
                     long long do_sb, long long do_sh, long long do_sn, float* delta, float* zero_acc, int B, int H,
                     int N, int D, int dtype, cudaStream_t stream);
// Fused dK/dV + dQ backward (every D; D = 128 runs fa_bwd_fused128.cu, with
// no boolean mask or dropout).  The fp32 dQ accumulator is a.dq; the D = 128
// kernel reduce-adds into it through tmap_dq, the D <= 64 kernels add into it
// directly (tmap_dq unused).
int launch_bwd_fused(const BwdArgs& a, const CUtensorMap& tmap_dq, int D);
int launch_bwd_fused128(const BwdArgs& a, const CUtensorMap& tmap_dq);
// acc_w: the accumulator's row width (0: D); dq receives its first D columns.
int launch_dq_convert(const float* acc, void* dq, long long sb, long long sh, long long sn, int B, int H, int N, int D,
                      int dtype, cudaStream_t stream, int acc_w = 0);
// Dense boolean mask (bytes, element strides {sb, sh, sq, sk}, Bm x Hm x Nq x
// Nk) -> bits (Bm, Hm, Nq, roundup(Nk, 128) / 32) and bits_t (Bm, Hm, Nk,
// roundup(Nq, 128) / 32) uint32 words, contiguous.
int launch_mask_pack(const void* mask, long long sb, long long sh, long long sq, long long sk, int Bm, int Hm, int Nq,
                     int Nk, uint32_t* bits, uint32_t* bits_t, cudaStream_t stream);
int launch_combine_splits(const void* o_part, const float* lse_part, void* o, float* lse, int S, int total_q, int H,
                          int D, int dtype, cudaStream_t stream);
int launch_merge_partial(float* o_acc, float* lse_acc, const void* o_part, const float* lse_part, long long rows,
                         int D, int dtype, cudaStream_t stream);

// Query-tile / key-tile sizes the host needs for TMA box shapes.
namespace dq_cfg {
constexpr int BM = 128;  // query rows per tile
constexpr int BN = 128;  // keys per key tile
}  // namespace dq_cfg
namespace dkdv_cfg {
constexpr int BM = 128;  // key rows per tile (the MMA M dimension)
constexpr int BQ = 64;   // query rows per tile (D = 128)
constexpr int BQ_WIDE = 128;  // query rows per item (D <= 64)
}  // namespace dkdv_cfg
// Query rows per item of the fused backward (its Q / dO tensor-map boxes).
constexpr int fused_item_rows(int D) { return D <= 64 ? dkdv_cfg::BQ_WIDE : dkdv_cfg::BQ; }

}  // namespace fa
