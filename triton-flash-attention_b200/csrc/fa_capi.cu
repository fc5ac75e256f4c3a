// fa_capi.cu -- the extern "C" boundary (include/fa_b200.h): argument
// validation, TMA descriptor encoding and kernel dispatch.  No exceptions and
// no torch types cross it; every entry point returns an FA_ERR_* code.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <mutex>

#include "fa_kernels.h"

namespace fa {
namespace {

__device__ int g_device_status;  // one word per device (each device loads its own copy)

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Device address of this device's status word (looked up once per device).
int* status_ptr() {
  static int* ptrs[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool supported_d(int D) { return D == 32 || D == 64 || D == 128; }

// 4-D tensor map (fp16 or bf16 elements) over (B, H, N, D) with element
// strides {sb, sh, sn, 1}.  The box is {min(D, 64), rows, 1, 1} with the
// swizzle the kernels' shared memory descriptors assume (128 B for D >= 64,
// 64 B for D = 32).  extent > 0 (< D) declares a tensor only extent columns
// wide read by a width-D kernel: the TMA fills columns extent..D-1 with zeros.
int make_map(CUtensorMap* map, const void* ptr, int B, int H, int N, int D, const int64_t* strides, int rows,
             int dtype, int heads_per_box = 1, int extent = 0) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return FA_ERR_DRIVER;
  if (!aligned16(ptr)) return FA_ERR_MISALIGNED;
  for (int i = 0; i < 3; ++i)
    if (strides[i] <= 0 || (strides[i] * 2) % 16 != 0) return FA_ERR_MISALIGNED;
  const int box_d = D >= 64 ? 64 : 32;
  cuuint64_t dims[4] = {cuuint64_t(extent > 0 ? extent : D), cuuint64_t(N), cuuint64_t(H), cuuint64_t(B)};
  cuuint64_t gstr[3] = {cuuint64_t(strides[2]) * 2, cuuint64_t(strides[1]) * 2, cuuint64_t(strides[0]) * 2};
  cuuint32_t box[4] = {cuuint32_t(box_d), cuuint32_t(rows), cuuint32_t(heads_per_box), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType ty = dtype == DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, ty, 4, const_cast<void*>(ptr), dims, gstr, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   D >= 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FA_OK : FA_ERR_TENSOR_MAP;
}

int check_shape(int B, int Hq, int Hkv, int Nq, int Nk, int D) {
  if (!supported_d(D)) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Nq <= 0 || Nk <= 0) return FA_ERR_BAD_SHAPE;
  if (Hq % Hkv != 0) return FA_ERR_BAD_SHAPE;
  return FA_OK;
}

bool out_strides_ok(const void* p, const int64_t* s, int elem_bytes) {
  if (!aligned16(p)) return false;
  for (int i = 0; i < 3; ++i)
    if (s[i] <= 0 || (s[i] * elem_bytes) % 16 != 0) return false;
  return true;
}

AttnShape make_shape(int B, int Hq, int Hkv, int Nq, int Nk, float scale, int causal, int q_off, int k_off) {
  AttnShape s;
  s.B = B;
  s.Hq = Hq;
  s.Hkv = Hkv;
  s.Nq = Nq;
  s.Nk = Nk;
  s.q_off = q_off;
  s.k_off = k_off;
  s.causal = causal ? 1 : 0;
  s.scale = scale;
  s.scale_log2 = float(double(scale) * 1.4426950408889634);
  s.status = status_ptr();
  s.cu_q = nullptr;
  s.cu_k = nullptr;
  s.total_q = 0;
  s.total_k = 0;
  s.seqlen_k = nullptr;
  s.block_table = nullptr;
  s.bt_stride = 0;
  s.page_size = 0;
  s.pack_g = 0;
  s.window = 0;
  s.qk_cols = 1 << 20;  // no narrower tensor: every column is stored
  s.v_cols = 1 << 20;
  return s;
}

// GQA packing of the forward (AttnShape::pack_g): a query tile holds the G
// query heads of a K/V head x 128 / G rows, so K/V is read once per group.
// Worth it when the query side is short -- decode and short chunks, where
// one unit then covers all of a sequence's queries -- and not for long
// causal queries, whose diagonal tiles it would make mostly masked.
int gqa_pack(int Hq, int Hkv, int max_q) {
  const int G = Hq / Hkv;
  if (G < 2 || G > 64 || (G & (G - 1)) != 0) return 0;
  return max_q * G <= 256 ? G : 0;
}

// The forward's query tensor map: a 128-row box of one head, or with GQA
// packing 128 / G rows of G consecutive heads.
int make_q_map(CUtensorMap* map, const void* q, int B, int H, int N, int D, const int64_t* strides, int dtype,
               int pack, int extent = 0) {
  return pack > 1 ? make_map(map, q, B, H, N, D, strides, 128 / pack, dtype, pack, extent)
                  : make_map(map, q, B, H, N, D, strides, 128, dtype, 1, extent);
}

int fwd_impl(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq, int Hkv, int Nq,
             int Nk, int D, const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
             const int64_t* o_strides, float softmax_scale, int causal, int q_offset, int k_offset, void* stream,
             int dtype) {
  int rc = check_shape(B, Hq, Hkv, Nq, Nk, D);
  if (rc) return rc;
  if (!q || !k || !v || !o || !lse || !q_strides || !k_strides || !v_strides || !o_strides) return FA_ERR_BAD_SHAPE;
  if (!std::isfinite(softmax_scale)) return FA_ERR_BAD_SHAPE;
  if (!out_strides_ok(o, o_strides, 2)) return FA_ERR_MISALIGNED;
  FwdArgs a;
  const int pack = gqa_pack(Hq, Hkv, Nq);
  if ((rc = make_q_map(&a.tmap_q, q, B, Hq, Nq, D, q_strides, dtype, pack))) return rc;
  if ((rc = make_map(&a.tmap_k, k, B, Hkv, Nk, D, k_strides, 128, dtype))) return rc;
  if ((rc = make_map(&a.tmap_v, v, B, Hkv, Nk, D, v_strides, 128, dtype))) return rc;
  a.shape = make_shape(B, Hq, Hkv, Nq, Nk, softmax_scale, causal, q_offset, k_offset);
  a.shape.pack_g = pack;
  a.dtype = dtype;
  a.o = o;
  a.o_sb = o_strides[0];
  a.o_sh = o_strides[1];
  a.o_sn = o_strides[2];
  a.lse = lse;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_fwd(a, D);
}

int delta_impl(const void* o, const void* dO, float* delta, int B, int H, int N, int D, const int64_t* o_strides,
               const int64_t* do_strides, void* stream, int dtype) {
  if (!supported_d(D)) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  if (B <= 0 || H <= 0 || N <= 0) return FA_ERR_BAD_SHAPE;
  if (!o || !dO || !delta || !o_strides || !do_strides) return FA_ERR_BAD_SHAPE;
  if (!out_strides_ok(o, o_strides, 2) || !out_strides_ok(dO, do_strides, 2)) return FA_ERR_MISALIGNED;
  return launch_bwd_delta(o, o_strides[0], o_strides[1], o_strides[2], dO, do_strides[0], do_strides[1],
                          do_strides[2], delta, nullptr, B, H, N, D, dtype, static_cast<cudaStream_t>(stream));
}

int preprocess_impl(const void* o, const void* dO, float* delta, float* dq_accum, int B, int H, int N, int D,
                    const int64_t* o_strides, const int64_t* do_strides, void* stream, int dtype) {
  if (!supported_d(D)) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  if (B <= 0 || H <= 0 || N <= 0) return FA_ERR_BAD_SHAPE;
  if (!o || !dO || !delta || !o_strides || !do_strides) return FA_ERR_BAD_SHAPE;
  if (!out_strides_ok(o, o_strides, 2) || !out_strides_ok(dO, do_strides, 2)) return FA_ERR_MISALIGNED;
  if (dq_accum && !aligned16(dq_accum)) return FA_ERR_MISALIGNED;
  return launch_bwd_delta(o, o_strides[0], o_strides[1], o_strides[2], dO, do_strides[0], do_strides[1],
                          do_strides[2], delta, dq_accum, B, H, N, D, dtype, static_cast<cudaStream_t>(stream));
}

// 4-D fp32 tensor map over the contiguous (B, H, N, D) dQ accumulator, with
// the box the fused kernel at D = 128 stages its partials in: one warp's
// {32, 64, 1, 1} piece without swizzle.  (At D <= 64 the fused kernel adds
// its partials with vector reductions and takes no map.)
int make_acc_map(CUtensorMap* map, float* ptr, int B, int H, int N, int D) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return FA_ERR_DRIVER;
  if (!aligned16(ptr)) return FA_ERR_MISALIGNED;
  cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(N), cuuint64_t(H), cuuint64_t(B)};
  cuuint64_t gstr[3] = {cuuint64_t(D) * 4, cuuint64_t(N) * D * 4, cuuint64_t(H) * N * D * 4};
  cuuint32_t box[4] = {32, cuuint32_t(fused_item_rows(D)), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ptr, dims, gstr, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FA_OK : FA_ERR_TENSOR_MAP;
}

int convert_impl(const float* acc, void* dq, int B, int H, int N, int D, const int64_t* dq_strides, void* stream,
                 int dtype) {
  if (!supported_d(D)) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  if (B <= 0 || H <= 0 || N <= 0) return FA_ERR_BAD_SHAPE;
  if (!acc || !dq || !dq_strides) return FA_ERR_BAD_SHAPE;
  if (!aligned16(acc) || !out_strides_ok(dq, dq_strides, 2)) return FA_ERR_MISALIGNED;
  return launch_dq_convert(acc, dq, dq_strides[0], dq_strides[1], dq_strides[2], B, H, N, D, dtype,
                           static_cast<cudaStream_t>(stream));
}

int dq_impl(const void* q, const void* k, const void* v, const void* dO, const float* lse, const float* delta,
            void* dq, int B, int Hq, int Hkv, int Nq, int Nk, int D, const int64_t* q_strides,
            const int64_t* k_strides, const int64_t* v_strides, const int64_t* do_strides,
            const int64_t* dq_strides, float softmax_scale, int causal, int q_offset, int k_offset,
            int accumulate_fp32, void* stream, int dtype) {
  int rc = check_shape(B, Hq, Hkv, Nq, Nk, D);
  if (rc) return rc;
  if (!q || !k || !v || !dO || !lse || !delta || !dq) return FA_ERR_BAD_SHAPE;
  if (!q_strides || !k_strides || !v_strides || !do_strides || !dq_strides) return FA_ERR_BAD_SHAPE;
  if (!std::isfinite(softmax_scale)) return FA_ERR_BAD_SHAPE;
  if (!out_strides_ok(dq, dq_strides, accumulate_fp32 ? 4 : 2)) return FA_ERR_MISALIGNED;
  BwdArgs a;
  a.dtype = dtype;
  if ((rc = make_map(&a.tmap_q, q, B, Hq, Nq, D, q_strides, dq_cfg::BM, dtype))) return rc;
  if ((rc = make_map(&a.tmap_do, dO, B, Hq, Nq, D, do_strides, dq_cfg::BM, dtype))) return rc;
  const int bn = dq_cfg::BN;
  if ((rc = make_map(&a.tmap_k, k, B, Hkv, Nk, D, k_strides, bn, dtype))) return rc;
  if ((rc = make_map(&a.tmap_v, v, B, Hkv, Nk, D, v_strides, bn, dtype))) return rc;
  a.shape = make_shape(B, Hq, Hkv, Nq, Nk, softmax_scale, causal, q_offset, k_offset);
  a.lse = lse;
  a.delta = delta;
  a.dq = dq;
  a.dq_sb = dq_strides[0];
  a.dq_sh = dq_strides[1];
  a.dq_sn = dq_strides[2];
  a.dk = a.dv = nullptr;
  a.dk_sb = a.dk_sh = a.dk_sn = a.dv_sb = a.dv_sh = a.dv_sn = 0;
  a.accumulate_fp32 = accumulate_fp32 ? 1 : 0;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_bwd_dq(a, D);
}

int dkdv_impl(const void* q, const void* k, const void* v, const void* dO, const float* lse, const float* delta,
              void* dk, void* dv, int B, int Hq, int Hkv, int Nq, int Nk, int D, const int64_t* q_strides,
              const int64_t* k_strides, const int64_t* v_strides, const int64_t* do_strides,
              const int64_t* dk_strides, const int64_t* dv_strides, float softmax_scale, int causal, int q_offset,
              int k_offset, int accumulate_fp32, void* stream, int dtype) {
  int rc = check_shape(B, Hq, Hkv, Nq, Nk, D);
  if (rc) return rc;
  if (!q || !k || !v || !dO || !lse || !delta || !dk || !dv) return FA_ERR_BAD_SHAPE;
  if (!q_strides || !k_strides || !v_strides || !do_strides || !dk_strides || !dv_strides) return FA_ERR_BAD_SHAPE;
  if (!std::isfinite(softmax_scale)) return FA_ERR_BAD_SHAPE;
  const int eb = accumulate_fp32 ? 4 : 2;
  if (!out_strides_ok(dk, dk_strides, eb) || !out_strides_ok(dv, dv_strides, eb)) return FA_ERR_MISALIGNED;
  BwdArgs a;
  a.dtype = dtype;
  const int bq = D <= 64 ? dkdv_cfg::BQ_WIDE : dkdv_cfg::BQ;
  if ((rc = make_map(&a.tmap_q, q, B, Hq, Nq, D, q_strides, bq, dtype))) return rc;
  if ((rc = make_map(&a.tmap_do, dO, B, Hq, Nq, D, do_strides, bq, dtype))) return rc;
  if ((rc = make_map(&a.tmap_k, k, B, Hkv, Nk, D, k_strides, dkdv_cfg::BM, dtype))) return rc;
  if ((rc = make_map(&a.tmap_v, v, B, Hkv, Nk, D, v_strides, dkdv_cfg::BM, dtype))) return rc;
  a.shape = make_shape(B, Hq, Hkv, Nq, Nk, softmax_scale, causal, q_offset, k_offset);
  a.lse = lse;
  a.delta = delta;
  a.dq = nullptr;
  a.dq_sb = a.dq_sh = a.dq_sn = 0;
  a.dk = dk;
  a.dv = dv;
  a.dk_sb = dk_strides[0];
  a.dk_sh = dk_strides[1];
  a.dk_sn = dk_strides[2];
  a.dv_sb = dv_strides[0];
  a.dv_sh = dv_strides[1];
  a.dv_sn = dv_strides[2];
  a.accumulate_fp32 = accumulate_fp32 ? 1 : 0;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_bwd_dkdv(a, D);
}

int fused_impl(const void* q, const void* k, const void* v, const void* dO, const float* lse, const float* delta,
               float* dq_accum, void* dk, void* dv, int B, int Hq, int Hkv, int Nq, int Nk, int D,
               const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
               const int64_t* do_strides, const int64_t* dk_strides, const int64_t* dv_strides, float softmax_scale,
               int causal, int q_offset, int k_offset, int accumulate_fp32, void* stream, int dtype) {
  int rc = check_shape(B, Hq, Hkv, Nq, Nk, D);
  if (rc) return rc;
  if (!q || !k || !v || !dO || !lse || !delta || !dq_accum || !dk || !dv) return FA_ERR_BAD_SHAPE;
  if (!q_strides || !k_strides || !v_strides || !do_strides || !dk_strides || !dv_strides) return FA_ERR_BAD_SHAPE;
  if (!std::isfinite(softmax_scale)) return FA_ERR_BAD_SHAPE;
  const int eb = accumulate_fp32 ? 4 : 2;
  if (!out_strides_ok(dk, dk_strides, eb) || !out_strides_ok(dv, dv_strides, eb)) return FA_ERR_MISALIGNED;
  BwdArgs a;
  a.dtype = dtype;
  const int bq = fused_item_rows(D);
  if ((rc = make_map(&a.tmap_q, q, B, Hq, Nq, D, q_strides, bq, dtype))) return rc;
  if ((rc = make_map(&a.tmap_do, dO, B, Hq, Nq, D, do_strides, bq, dtype))) return rc;
  if ((rc = make_map(&a.tmap_k, k, B, Hkv, Nk, D, k_strides, dkdv_cfg::BM, dtype))) return rc;
  if ((rc = make_map(&a.tmap_v, v, B, Hkv, Nk, D, v_strides, dkdv_cfg::BM, dtype))) return rc;
  CUtensorMap tmap_dq = {};
  if (D == 128 && (rc = make_acc_map(&tmap_dq, dq_accum, B, Hq, Nq, D))) return rc;
  a.shape = make_shape(B, Hq, Hkv, Nq, Nk, softmax_scale, causal, q_offset, k_offset);
  a.lse = lse;
  a.delta = delta;
  a.dq = dq_accum;
  a.dq_sb = a.dq_sh = a.dq_sn = 0;
  a.dk = dk;
  a.dv = dv;
  a.dk_sb = dk_strides[0];
  a.dk_sh = dk_strides[1];
  a.dk_sn = dk_strides[2];
  a.dv_sb = dv_strides[0];
  a.dv_sh = dv_strides[1];
  a.dv_sn = dv_strides[2];
  a.accumulate_fp32 = accumulate_fp32 ? 1 : 0;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_bwd_fused(a, tmap_dq, D);
}

int merge_impl(float* o_acc, float* lse_acc, const void* o_part, const float* lse_part, int B, int H, int N, int D,
               void* stream, int dtype) {
  if (!supported_d(D)) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  if (B <= 0 || H <= 0 || N <= 0) return FA_ERR_BAD_SHAPE;
  if (!o_acc || !lse_acc || !o_part || !lse_part) return FA_ERR_BAD_SHAPE;
  if (!aligned16(o_acc) || !aligned16(o_part)) return FA_ERR_MISALIGNED;
  return launch_merge_partial(o_acc, lse_acc, o_part, lse_part, (long long)B * H * N, D, dtype,
                              static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// Packed variable-length batches (no counterpart in the reference): q, o,
// dO, dq are contiguous (total_q, Hq, D), k, v, dk, dv contiguous
// (total_k, Hkv, D); batch b owns rows [cu_q[b], cu_q[b+1]) and
// [cu_k[b], cu_k[b+1]).  The kernels are the dense ones, reading the packed
// tensors through (1, H, total, D) tensor maps at the batch's row offset.

// Element strides {batch, head, row} of a contiguous (total, H, D) tensor
// seen as (1, H, total, D).
struct PackedStrides {
  int64_t v[3];
  PackedStrides(int total, int H, int D) {
    v[0] = int64_t(total > 0 ? total : 1) * H * D;
    v[1] = D;
    v[2] = int64_t(H) * D;
  }
};

int check_varlen(const int* cu_q, const int* cu_k, int B, int Hq, int Hkv, int max_q, int max_k, int total_q,
                 int total_k, int D) {
  if (!supported_d(D)) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0) return FA_ERR_BAD_SHAPE;
  if (max_q <= 0 || max_k <= 0 || total_q <= 0 || total_k <= 0) return FA_ERR_BAD_SHAPE;
  if (!cu_q || !cu_k) return FA_ERR_BAD_SHAPE;
  return FA_OK;
}

AttnShape varlen_shape(const int* cu_q, const int* cu_k, int B, int Hq, int Hkv, int max_q, int max_k, int total_q,
                       int total_k, float scale, int causal) {
  AttnShape sh = make_shape(B, Hq, Hkv, max_q, max_k, scale, causal, 0, 0);
  sh.cu_q = cu_q;
  sh.cu_k = cu_k;
  sh.total_q = total_q;
  sh.total_k = total_k;
  return sh;
}

int fwd_varlen_impl(const void* q, const void* k, const void* v, void* o, float* lse, const int* cu_q,
                    const int* cu_k, int B, int Hq, int Hkv, int max_q, int max_k, int total_q, int total_k, int D,
                    float softmax_scale, int causal, int window, void* stream, int dtype) {
  int rc = check_varlen(cu_q, cu_k, B, Hq, Hkv, max_q, max_k, total_q, total_k, D);
  if (rc) return rc;
  if (!q || !k || !v || !o || !lse || !std::isfinite(softmax_scale)) return FA_ERR_BAD_SHAPE;
  if (window < 0 || (window > 0 && !causal)) return FA_ERR_BAD_SHAPE;
  const PackedStrides sq(total_q, Hq, D), sk(total_k, Hkv, D);
  if (!out_strides_ok(o, sq.v, 2)) return FA_ERR_MISALIGNED;
  FwdArgs a;
  const int pack = gqa_pack(Hq, Hkv, max_q);
  if ((rc = make_q_map(&a.tmap_q, q, 1, Hq, total_q, D, sq.v, dtype, pack))) return rc;
  if ((rc = make_map(&a.tmap_k, k, 1, Hkv, total_k, D, sk.v, 128, dtype))) return rc;
  if ((rc = make_map(&a.tmap_v, v, 1, Hkv, total_k, D, sk.v, 128, dtype))) return rc;
  a.shape = varlen_shape(cu_q, cu_k, B, Hq, Hkv, max_q, max_k, total_q, total_k, softmax_scale, causal);
  a.shape.pack_g = pack;
  a.shape.window = window;
  a.dtype = dtype;
  a.o = o;
  a.o_sb = 0;
  a.o_sh = sq.v[1];
  a.o_sn = sq.v[2];
  a.lse = lse;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_fwd(a, D);
}

int bwd_varlen_impl(const void* q, const void* k, const void* v, const void* o, const void* dO, const float* lse,
                    void* dq, void* dk, void* dv, float* delta, float* dq_accum, const int* cu_q, const int* cu_k,
                    int B, int Hq, int Hkv, int max_q, int max_k, int total_q, int total_k, int D,
                    float softmax_scale, int causal, int window, int deterministic, void* stream, int dtype) {
  int rc = check_varlen(cu_q, cu_k, B, Hq, Hkv, max_q, max_k, total_q, total_k, D);
  if (rc) return rc;
  if (window < 0 || (window > 0 && !causal)) return FA_ERR_BAD_SHAPE;
  if (!q || !k || !v || !o || !dO || !lse || !dq || !dk || !dv || !delta) return FA_ERR_BAD_SHAPE;
  if (!std::isfinite(softmax_scale)) return FA_ERR_BAD_SHAPE;
  const bool fused = !deterministic;
  if (fused && !dq_accum) return FA_ERR_BAD_SHAPE;
  const PackedStrides sq(total_q, Hq, D), sk(total_k, Hkv, D);
  if (!out_strides_ok(o, sq.v, 2) || !out_strides_ok(dO, sq.v, 2) || !out_strides_ok(dq, sq.v, 2) ||
      !out_strides_ok(dk, sk.v, 2) || !out_strides_ok(dv, sk.v, 2) || !aligned16(delta) ||
      (fused && !aligned16(dq_accum)))
    return FA_ERR_MISALIGNED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Delta (Hq, total_q) and, for the fused pass, the zeroed (Hq, total_q, D) accumulator
  if ((rc = launch_bwd_delta(o, sq.v[0], sq.v[1], sq.v[2], dO, sq.v[0], sq.v[1], sq.v[2], delta,
                             fused ? dq_accum : nullptr, 1, Hq, total_q, D, dtype, st)))
    return rc;
  BwdArgs a;
  a.dtype = dtype;
  a.shape = varlen_shape(cu_q, cu_k, B, Hq, Hkv, max_q, max_k, total_q, total_k, softmax_scale, causal);
  a.shape.window = window;
  a.lse = lse;
  a.delta = delta;
  a.dk = dk;
  a.dv = dv;
  a.dk_sb = a.dv_sb = 0;
  a.dk_sh = a.dv_sh = sk.v[1];
  a.dk_sn = a.dv_sn = sk.v[2];
  a.accumulate_fp32 = 0;
  a.stream = st;
  if (fused) {
    if ((rc = make_map(&a.tmap_q, q, 1, Hq, total_q, D, sq.v, fused_item_rows(D), dtype))) return rc;
    if ((rc = make_map(&a.tmap_do, dO, 1, Hq, total_q, D, sq.v, fused_item_rows(D), dtype))) return rc;
    if ((rc = make_map(&a.tmap_k, k, 1, Hkv, total_k, D, sk.v, dkdv_cfg::BM, dtype))) return rc;
    if ((rc = make_map(&a.tmap_v, v, 1, Hkv, total_k, D, sk.v, dkdv_cfg::BM, dtype))) return rc;
    CUtensorMap tmap_dq = {};
    if (D == 128 && (rc = make_acc_map(&tmap_dq, dq_accum, 1, Hq, total_q, D))) return rc;
    a.dq = dq_accum;
    a.dq_sb = a.dq_sh = a.dq_sn = 0;
    if ((rc = launch_bwd_fused(a, tmap_dq, D))) return rc;
    return launch_dq_convert(dq_accum, dq, sq.v[0], sq.v[1], sq.v[2], 1, Hq, total_q, D, dtype, st);
  }
  // split path: dQ kernel, then dK/dV kernel
  if ((rc = make_map(&a.tmap_q, q, 1, Hq, total_q, D, sq.v, dq_cfg::BM, dtype))) return rc;
  if ((rc = make_map(&a.tmap_do, dO, 1, Hq, total_q, D, sq.v, dq_cfg::BM, dtype))) return rc;
  if ((rc = make_map(&a.tmap_k, k, 1, Hkv, total_k, D, sk.v, dq_cfg::BN, dtype))) return rc;
  if ((rc = make_map(&a.tmap_v, v, 1, Hkv, total_k, D, sk.v, dq_cfg::BN, dtype))) return rc;
  a.dq = dq;
  a.dq_sb = 0;
  a.dq_sh = sq.v[1];
  a.dq_sn = sq.v[2];
  if ((rc = launch_bwd_dq(a, D))) return rc;
  const int bq = D <= 64 ? dkdv_cfg::BQ_WIDE : dkdv_cfg::BQ;
  if ((rc = make_map(&a.tmap_q, q, 1, Hq, total_q, D, sq.v, bq, dtype))) return rc;
  if ((rc = make_map(&a.tmap_do, dO, 1, Hq, total_q, D, sq.v, bq, dtype))) return rc;
  if ((rc = make_map(&a.tmap_k, k, 1, Hkv, total_k, D, sk.v, dkdv_cfg::BM, dtype))) return rc;
  if ((rc = make_map(&a.tmap_v, v, 1, Hkv, total_k, D, sk.v, dkdv_cfg::BM, dtype))) return rc;
  a.dq = nullptr;
  a.dq_sb = a.dq_sh = a.dq_sn = 0;
  return launch_bwd_dkdv(a, D);
}

// ---------------------------------------------------------------------------
// Paged K/V forward (no counterpart in the reference): packed queries as in
// the varlen calls, keys and values in (num_pages * page_size, Hkv, D)
// caches addressed through a (B, bt_stride) block table.
int fwd_paged_impl(const void* q, const void* k_cache, const void* v_cache, void* o, float* lse, const int* cu_q,
                   const int* seqlens_k, const int* block_table, int B, int Hq, int Hkv, int max_q, int max_k,
                   int total_q, int num_pages, int page_size, int bt_stride, int D, float softmax_scale, int causal,
                   int window, void* stream, int dtype, int splits = 1) {
  if (!supported_d(D)) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0 || max_q <= 0 || max_k <= 0 || total_q <= 0 ||
      num_pages <= 0 || bt_stride <= 0)
    return FA_ERR_BAD_SHAPE;
  // a power of two of at least 16 rows: a key tile of 128 is whole pieces of
  // pages, each starting on a swizzle-atom boundary of the shared tile
  if (page_size < 16 || (page_size & (page_size - 1)) != 0) return FA_ERR_BAD_SHAPE;
  if ((long long)num_pages * page_size > 0x7fffffffLL) return FA_ERR_BAD_SHAPE;
  if (!q || !k_cache || !v_cache || !o || !lse || !cu_q || !seqlens_k || !block_table) return FA_ERR_BAD_SHAPE;
  if (!std::isfinite(softmax_scale)) return FA_ERR_BAD_SHAPE;
  if (window < 0 || (window > 0 && !causal)) return FA_ERR_BAD_SHAPE;
  const PackedStrides sq(total_q, Hq, D), sk(num_pages * page_size, Hkv, D);
  if (!out_strides_ok(o, sq.v, 2)) return FA_ERR_MISALIGNED;
  int rc;
  FwdArgs a;
  const int pr = page_size < 128 ? page_size : 128;
  const int pack = gqa_pack(Hq, Hkv, max_q);
  // split-KV: GQA-packed query tiles and no window; o and lse hold the
  // splits' partials, (splits, total_q, Hq, D) and (splits, Hq, total_q)
  const int key_tiles = (max_k + 127) / 128;
  if (splits < 1 || splits > FA_MAX_KV_SPLITS || splits > key_tiles) return FA_ERR_BAD_SHAPE;
  if (splits > 1 && (pack < 2 || window > 0)) return FA_ERR_BAD_SHAPE;
  if ((rc = make_q_map(&a.tmap_q, q, 1, Hq, total_q, D, sq.v, dtype, pack))) return rc;
  if ((rc = make_map(&a.tmap_k, k_cache, 1, Hkv, num_pages * page_size, D, sk.v, pr, dtype))) return rc;
  if ((rc = make_map(&a.tmap_v, v_cache, 1, Hkv, num_pages * page_size, D, sk.v, pr, dtype))) return rc;
  a.shape = make_shape(B, Hq, Hkv, max_q, max_k, softmax_scale, causal, 0, 0);
  a.shape.cu_q = cu_q;
  a.shape.total_q = total_q;
  a.shape.seqlen_k = seqlens_k;
  a.shape.block_table = block_table;
  a.shape.bt_stride = bt_stride;
  a.shape.page_size = page_size;
  a.shape.pack_g = pack;
  a.shape.window = window;
  a.dtype = dtype;
  a.o = o;
  a.o_sb = 0;
  a.o_sh = sq.v[1];
  a.o_sn = sq.v[2];
  a.lse = lse;
  if (splits > 1) {
    a.split.n = splits;
    a.split.tiles = (key_tiles + splits - 1) / splits;
    a.split.o_stride = (long long)total_q * Hq * D;
    a.split.lse_stride = (long long)Hq * total_q;
  }
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_fwd(a, D);
}

int combine_impl(const void* o_part, const float* lse_part, void* o, float* lse, int splits, int total_q, int H, int D,
                 void* stream, int dtype) {
  if (!supported_d(D)) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  if (splits < 1 || splits > FA_MAX_KV_SPLITS || total_q <= 0 || H <= 0) return FA_ERR_BAD_SHAPE;
  if (!o_part || !lse_part || !o || !lse) return FA_ERR_BAD_SHAPE;
  if (!aligned16(o_part) || !aligned16(o)) return FA_ERR_MISALIGNED;
  return launch_combine_splits(o_part, lse_part, o, lse, splits, total_q, H, D, dtype,
                               static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// fwd_dense_impl / bwd_dense_impl: the dense-layout forward and whole
// backward with the options the plain calls lack -- a value head size of
// its own, a packed boolean mask, dropout -- behind fa_*_vdim, fa_*_masked
// and fa_*_dropout.
//
// Value head size Dv different from the query/key head size D (the
// reference hands these inputs to PyTorch, attention.py:639-646).  The
// kernels run at width W = max(D, Dv): the narrower operands are read
// through tensor maps whose extent is their own width, so the TMA fills
// the missing columns with zeros -- zero columns of Q and K leave Q K^T
// unchanged, zero columns of V and dO give zero columns of O, dP's
// reduction is unchanged and the padded gradient columns are zero -- and
// the kernels store only the first D columns of dQ / dK and the first Dv of
// O / dV (AttnShape::qk_cols, v_cols).  The MMAs on the padded columns are
// wasted work: W = max(D, Dv) sets the cost.
//
// Dense boolean masks (fa_mask_pack, fa_fwd_masked, fa_bwd_masked; the
// reference has none, README.md:93): the kernels take the packed bit rows
// through a MaskBits kernel parameter, in instantiations of their own.  A mask
// goes with the dense layout, no GQA packing of the forward, no window and
// no position offsets.
//
// Dropout (fa_fwd_dropout, fa_bwd_dropout; the reference has none): a
// DropArgs kernel parameter (threshold, scale, seed) in instantiations of
// their own; the backward always runs the separate dQ and dK/dV kernels,
// whose threads hold P and dS of an element together.

// A packed mask's word strides {batch, head, row}: non-negative, 16-byte
// aligned rows of at least `words` words.
bool mask_ok(const uint32_t* bits, const int64_t* st, int words) {
  if (!bits || !st || !aligned16(bits)) return false;
  if (st[0] < 0 || st[1] < 0 || st[2] < words) return false;
  for (int i = 0; i < 3; ++i)
    if (st[i] % 4 != 0) return false;
  return true;
}

int fwd_dense_impl(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq, int Hkv, int Nq,
                  int Nk, int D, int Dv, const int64_t* q_strides, const int64_t* k_strides,
                  const int64_t* v_strides, const int64_t* o_strides, float softmax_scale, int causal, void* stream,
                  int dtype, const uint32_t* mask = nullptr, const int64_t* mask_strides = nullptr,
                  const DropArgs* drop = nullptr) {
  if (!supported_d(D) || !supported_d(Dv)) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  const int W = D > Dv ? D : Dv;
  int rc = check_shape(B, Hq, Hkv, Nq, Nk, W);
  if (rc) return rc;
  if (!q || !k || !v || !o || !lse || !q_strides || !k_strides || !v_strides || !o_strides) return FA_ERR_BAD_SHAPE;
  if (!std::isfinite(softmax_scale)) return FA_ERR_BAD_SHAPE;
  if (!out_strides_ok(o, o_strides, 2)) return FA_ERR_MISALIGNED;
  if (mask && !mask_ok(mask, mask_strides, (Nk + 127) / 128 * 4)) return FA_ERR_MISALIGNED;
  FwdArgs a;
  const int pack = (mask || drop) ? 0 : gqa_pack(Hq, Hkv, Nq);
  if ((rc = make_q_map(&a.tmap_q, q, B, Hq, Nq, W, q_strides, dtype, pack, D))) return rc;
  if ((rc = make_map(&a.tmap_k, k, B, Hkv, Nk, W, k_strides, 128, dtype, 1, D))) return rc;
  if ((rc = make_map(&a.tmap_v, v, B, Hkv, Nk, W, v_strides, 128, dtype, 1, Dv))) return rc;
  a.shape = make_shape(B, Hq, Hkv, Nq, Nk, softmax_scale, causal, 0, 0);
  a.shape.pack_g = pack;
  a.shape.qk_cols = D;
  a.shape.v_cols = Dv;
  if (mask) {
    a.mask.bits = mask;
    a.mask.sb = mask_strides[0];
    a.mask.sh = mask_strides[1];
    a.mask.sn = mask_strides[2];
  }
  if (drop) a.drop = *drop;
  a.dtype = dtype;
  a.o = o;
  a.o_sb = o_strides[0];
  a.o_sh = o_strides[1];
  a.o_sn = o_strides[2];
  a.lse = lse;
  a.stream = static_cast<cudaStream_t>(stream);
  return launch_fwd(a, W);
}

int bwd_dense_impl(const void* q, const void* k, const void* v, const void* o, const void* dO, const float* lse,
                  void* dq, void* dk, void* dv, float* delta, float* dq_accum, int B, int Hq, int Hkv, int Nq, int Nk,
                  int D, int Dv, const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                  const int64_t* o_strides, const int64_t* do_strides, const int64_t* dq_strides,
                  const int64_t* dk_strides, const int64_t* dv_strides, float softmax_scale, int causal,
                  int deterministic, void* stream, int dtype, const uint32_t* mask = nullptr,
                  const int64_t* mask_strides = nullptr, const uint32_t* mask_t = nullptr,
                  const int64_t* mask_t_strides = nullptr, const DropArgs* drop = nullptr) {
  if (!supported_d(D) || !supported_d(Dv)) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  const int W = D > Dv ? D : Dv;
  int rc = check_shape(B, Hq, Hkv, Nq, Nk, W);
  if (rc) return rc;
  if (!q || !k || !v || !o || !dO || !lse || !dq || !dk || !dv || !delta) return FA_ERR_BAD_SHAPE;
  if (!q_strides || !k_strides || !v_strides || !o_strides || !do_strides || !dq_strides || !dk_strides ||
      !dv_strides)
    return FA_ERR_BAD_SHAPE;
  if (!std::isfinite(softmax_scale)) return FA_ERR_BAD_SHAPE;
  // dropout runs the separate dQ and dK/dV kernels, whose threads hold P and
  // dS of an element together
  const bool fused = W <= 64 && !deterministic && !drop;
  if (fused && !dq_accum) return FA_ERR_BAD_SHAPE;
  if (!out_strides_ok(o, o_strides, 2) || !out_strides_ok(dO, do_strides, 2) || !out_strides_ok(dq, dq_strides, 2) ||
      !out_strides_ok(dk, dk_strides, 2) || !out_strides_ok(dv, dv_strides, 2) || !aligned16(delta) ||
      (fused && !aligned16(dq_accum)))
    return FA_ERR_MISALIGNED;
  if ((mask || mask_t) && (!mask_ok(mask, mask_strides, (Nk + 127) / 128 * 4) ||
                           !mask_ok(mask_t, mask_t_strides, (Nq + 127) / 128 * 4)))
    return FA_ERR_MISALIGNED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Delta = rowsum(O * dO) over the Dv columns
  if ((rc = launch_bwd_delta(o, o_strides[0], o_strides[1], o_strides[2], dO, do_strides[0], do_strides[1],
                             do_strides[2], delta, nullptr, B, Hq, Nq, Dv, dtype, st)))
    return rc;
  BwdArgs a;
  a.dtype = dtype;
  a.shape = make_shape(B, Hq, Hkv, Nq, Nk, softmax_scale, causal, 0, 0);
  a.shape.qk_cols = D;
  a.shape.v_cols = Dv;
  if (mask) {
    a.mask.bits = mask;
    a.mask.sb = mask_strides[0];
    a.mask.sh = mask_strides[1];
    a.mask.sn = mask_strides[2];
    a.mask.bits_t = mask_t;
    a.mask.tsb = mask_t_strides[0];
    a.mask.tsh = mask_t_strides[1];
    a.mask.tsn = mask_t_strides[2];
  }
  if (drop) a.drop = *drop;
  a.lse = lse;
  a.delta = delta;
  a.dk = dk;
  a.dv = dv;
  a.dk_sb = dk_strides[0];
  a.dk_sh = dk_strides[1];
  a.dk_sn = dk_strides[2];
  a.dv_sb = dv_strides[0];
  a.dv_sh = dv_strides[1];
  a.dv_sn = dv_strides[2];
  a.accumulate_fp32 = 0;
  a.stream = st;
  if (fused) {
    // the (B, Hq, Nq, W) fp32 dQ accumulator starts at zero
    if (cudaMemsetAsync(dq_accum, 0, sizeof(float) * size_t(B) * Hq * Nq * W, st) != cudaSuccess)
      return FA_ERR_LAUNCH;
    if ((rc = make_map(&a.tmap_q, q, B, Hq, Nq, W, q_strides, dkdv_cfg::BQ_WIDE, dtype, 1, D))) return rc;
    if ((rc = make_map(&a.tmap_do, dO, B, Hq, Nq, W, do_strides, dkdv_cfg::BQ_WIDE, dtype, 1, Dv))) return rc;
    if ((rc = make_map(&a.tmap_k, k, B, Hkv, Nk, W, k_strides, dkdv_cfg::BM, dtype, 1, D))) return rc;
    if ((rc = make_map(&a.tmap_v, v, B, Hkv, Nk, W, v_strides, dkdv_cfg::BM, dtype, 1, Dv))) return rc;
    CUtensorMap tmap_dq = {};
    if (W == 128 && (rc = make_acc_map(&tmap_dq, dq_accum, B, Hq, Nq, W))) return rc;
    a.dq = dq_accum;
    a.dq_sb = a.dq_sh = a.dq_sn = 0;
    if ((rc = launch_bwd_fused(a, tmap_dq, W))) return rc;
    return launch_dq_convert(dq_accum, dq, dq_strides[0], dq_strides[1], dq_strides[2], B, Hq, Nq, D, dtype, st, W);
  }
  // split path: dQ kernel, then dK/dV kernel
  if ((rc = make_map(&a.tmap_q, q, B, Hq, Nq, W, q_strides, dq_cfg::BM, dtype, 1, D))) return rc;
  if ((rc = make_map(&a.tmap_do, dO, B, Hq, Nq, W, do_strides, dq_cfg::BM, dtype, 1, Dv))) return rc;
  if ((rc = make_map(&a.tmap_k, k, B, Hkv, Nk, W, k_strides, dq_cfg::BN, dtype, 1, D))) return rc;
  if ((rc = make_map(&a.tmap_v, v, B, Hkv, Nk, W, v_strides, dq_cfg::BN, dtype, 1, Dv))) return rc;
  a.dq = dq;
  a.dq_sb = dq_strides[0];
  a.dq_sh = dq_strides[1];
  a.dq_sn = dq_strides[2];
  if ((rc = launch_bwd_dq(a, W))) return rc;
  const int bq = (W <= 64 && !drop) ? dkdv_cfg::BQ_WIDE : dkdv_cfg::BQ;
  if ((rc = make_map(&a.tmap_q, q, B, Hq, Nq, W, q_strides, bq, dtype, 1, D))) return rc;
  if ((rc = make_map(&a.tmap_do, dO, B, Hq, Nq, W, do_strides, bq, dtype, 1, Dv))) return rc;
  if ((rc = make_map(&a.tmap_k, k, B, Hkv, Nk, W, k_strides, dkdv_cfg::BM, dtype, 1, D))) return rc;
  if ((rc = make_map(&a.tmap_v, v, B, Hkv, Nk, W, v_strides, dkdv_cfg::BM, dtype, 1, Dv))) return rc;
  a.dq = nullptr;
  a.dq_sb = a.dq_sh = a.dq_sn = 0;
  return launch_bwd_dkdv(a, W);
}

}  // namespace
}  // namespace fa

using namespace fa;

// fp16 entry points (the reference's only dtype) and their bf16 twins.
extern "C" int fa_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq, int Hkv,
                      int Nq, int Nk, int D, const int64_t* q_strides, const int64_t* k_strides,
                      const int64_t* v_strides, const int64_t* o_strides, float softmax_scale, int causal,
                      int q_offset, int k_offset, void* stream) {
  return fwd_impl(q, k, v, o, lse, B, Hq, Hkv, Nq, Nk, D, q_strides, k_strides, v_strides, o_strides, softmax_scale,
                  causal, q_offset, k_offset, stream, DT_F16);
}
extern "C" int fa_fwd_bf16(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq, int Hkv,
                           int Nq, int Nk, int D, const int64_t* q_strides, const int64_t* k_strides,
                           const int64_t* v_strides, const int64_t* o_strides, float softmax_scale, int causal,
                           int q_offset, int k_offset, void* stream) {
  return fwd_impl(q, k, v, o, lse, B, Hq, Hkv, Nq, Nk, D, q_strides, k_strides, v_strides, o_strides, softmax_scale,
                  causal, q_offset, k_offset, stream, DT_BF16);
}

extern "C" int fa_bwd_delta(const void* o, const void* dO, float* delta, int B, int H, int N, int D,
                            const int64_t* o_strides, const int64_t* do_strides, void* stream) {
  return delta_impl(o, dO, delta, B, H, N, D, o_strides, do_strides, stream, DT_F16);
}
extern "C" int fa_bwd_delta_bf16(const void* o, const void* dO, float* delta, int B, int H, int N, int D,
                                 const int64_t* o_strides, const int64_t* do_strides, void* stream) {
  return delta_impl(o, dO, delta, B, H, N, D, o_strides, do_strides, stream, DT_BF16);
}

extern "C" int fa_bwd_dq(const void* q, const void* k, const void* v, const void* dO, const float* lse,
                         const float* delta, void* dq, int B, int Hq, int Hkv, int Nq, int Nk, int D,
                         const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                         const int64_t* do_strides, const int64_t* dq_strides, float softmax_scale, int causal,
                         int q_offset, int k_offset, int accumulate_fp32, void* stream) {
  return dq_impl(q, k, v, dO, lse, delta, dq, B, Hq, Hkv, Nq, Nk, D, q_strides, k_strides, v_strides, do_strides,
                 dq_strides, softmax_scale, causal, q_offset, k_offset, accumulate_fp32, stream, DT_F16);
}
extern "C" int fa_bwd_dq_bf16(const void* q, const void* k, const void* v, const void* dO, const float* lse,
                              const float* delta, void* dq, int B, int Hq, int Hkv, int Nq, int Nk, int D,
                              const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                              const int64_t* do_strides, const int64_t* dq_strides, float softmax_scale, int causal,
                              int q_offset, int k_offset, int accumulate_fp32, void* stream) {
  return dq_impl(q, k, v, dO, lse, delta, dq, B, Hq, Hkv, Nq, Nk, D, q_strides, k_strides, v_strides, do_strides,
                 dq_strides, softmax_scale, causal, q_offset, k_offset, accumulate_fp32, stream, DT_BF16);
}

extern "C" int fa_bwd_dkdv(const void* q, const void* k, const void* v, const void* dO, const float* lse,
                           const float* delta, void* dk, void* dv, int B, int Hq, int Hkv, int Nq, int Nk, int D,
                           const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                           const int64_t* do_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                           float softmax_scale, int causal, int q_offset, int k_offset, int accumulate_fp32,
                           void* stream) {
  return dkdv_impl(q, k, v, dO, lse, delta, dk, dv, B, Hq, Hkv, Nq, Nk, D, q_strides, k_strides, v_strides,
                   do_strides, dk_strides, dv_strides, softmax_scale, causal, q_offset, k_offset, accumulate_fp32,
                   stream, DT_F16);
}
extern "C" int fa_bwd_dkdv_bf16(const void* q, const void* k, const void* v, const void* dO, const float* lse,
                                const float* delta, void* dk, void* dv, int B, int Hq, int Hkv, int Nq, int Nk,
                                int D, const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                                const int64_t* do_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                                float softmax_scale, int causal, int q_offset, int k_offset, int accumulate_fp32,
                                void* stream) {
  return dkdv_impl(q, k, v, dO, lse, delta, dk, dv, B, Hq, Hkv, Nq, Nk, D, q_strides, k_strides, v_strides,
                   do_strides, dk_strides, dv_strides, softmax_scale, causal, q_offset, k_offset, accumulate_fp32,
                   stream, DT_BF16);
}

extern "C" int fa_merge_partial(float* o_acc, float* lse_acc, const void* o_part, const float* lse_part, int B,
                                int H, int N, int D, void* stream) {
  return merge_impl(o_acc, lse_acc, o_part, lse_part, B, H, N, D, stream, DT_F16);
}
extern "C" int fa_merge_partial_bf16(float* o_acc, float* lse_acc, const void* o_part, const float* lse_part, int B,
                                     int H, int N, int D, void* stream) {
  return merge_impl(o_acc, lse_acc, o_part, lse_part, B, H, N, D, stream, DT_BF16);
}

extern "C" int fa_bwd_preprocess(const void* o, const void* dO, float* delta, float* dq_accum, int B, int H, int N,
                                 int D, const int64_t* o_strides, const int64_t* do_strides, void* stream) {
  return preprocess_impl(o, dO, delta, dq_accum, B, H, N, D, o_strides, do_strides, stream, DT_F16);
}
extern "C" int fa_bwd_preprocess_bf16(const void* o, const void* dO, float* delta, float* dq_accum, int B, int H,
                                      int N, int D, const int64_t* o_strides, const int64_t* do_strides,
                                      void* stream) {
  return preprocess_impl(o, dO, delta, dq_accum, B, H, N, D, o_strides, do_strides, stream, DT_BF16);
}

extern "C" int fa_bwd_fused(const void* q, const void* k, const void* v, const void* dO, const float* lse,
                            const float* delta, float* dq_accum, void* dk, void* dv, int B, int Hq, int Hkv, int Nq,
                            int Nk, int D, const int64_t* q_strides, const int64_t* k_strides,
                            const int64_t* v_strides, const int64_t* do_strides, const int64_t* dk_strides,
                            const int64_t* dv_strides, float softmax_scale, int causal, int q_offset, int k_offset,
                            int accumulate_fp32, void* stream) {
  return fused_impl(q, k, v, dO, lse, delta, dq_accum, dk, dv, B, Hq, Hkv, Nq, Nk, D, q_strides, k_strides, v_strides,
                    do_strides, dk_strides, dv_strides, softmax_scale, causal, q_offset, k_offset, accumulate_fp32,
                    stream, DT_F16);
}
extern "C" int fa_bwd_fused_bf16(const void* q, const void* k, const void* v, const void* dO, const float* lse,
                                 const float* delta, float* dq_accum, void* dk, void* dv, int B, int Hq, int Hkv,
                                 int Nq, int Nk, int D, const int64_t* q_strides, const int64_t* k_strides,
                                 const int64_t* v_strides, const int64_t* do_strides, const int64_t* dk_strides,
                                 const int64_t* dv_strides, float softmax_scale, int causal, int q_offset,
                                 int k_offset, int accumulate_fp32, void* stream) {
  return fused_impl(q, k, v, dO, lse, delta, dq_accum, dk, dv, B, Hq, Hkv, Nq, Nk, D, q_strides, k_strides, v_strides,
                    do_strides, dk_strides, dv_strides, softmax_scale, causal, q_offset, k_offset, accumulate_fp32,
                    stream, DT_BF16);
}

extern "C" int fa_bwd_dq_convert(const float* dq_accum, void* dq, int B, int H, int N, int D,
                                 const int64_t* dq_strides, void* stream) {
  return convert_impl(dq_accum, dq, B, H, N, D, dq_strides, stream, DT_F16);
}
extern "C" int fa_bwd_dq_convert_bf16(const float* dq_accum, void* dq, int B, int H, int N, int D,
                                      const int64_t* dq_strides, void* stream) {
  return convert_impl(dq_accum, dq, B, H, N, D, dq_strides, stream, DT_BF16);
}

extern "C" int fa_fwd_varlen(const void* q, const void* k, const void* v, void* o, float* lse,
                             const int* cu_seqlens_q, const int* cu_seqlens_k, int B, int Hq, int Hkv,
                             int max_seqlen_q, int max_seqlen_k, int total_q, int total_k, int D, float softmax_scale,
                             int causal, int window, void* stream) {
  return fwd_varlen_impl(q, k, v, o, lse, cu_seqlens_q, cu_seqlens_k, B, Hq, Hkv, max_seqlen_q, max_seqlen_k,
                         total_q, total_k, D, softmax_scale, causal, window, stream, DT_F16);
}
extern "C" int fa_fwd_varlen_bf16(const void* q, const void* k, const void* v, void* o, float* lse,
                                  const int* cu_seqlens_q, const int* cu_seqlens_k, int B, int Hq, int Hkv,
                                  int max_seqlen_q, int max_seqlen_k, int total_q, int total_k, int D,
                                  float softmax_scale, int causal, int window, void* stream) {
  return fwd_varlen_impl(q, k, v, o, lse, cu_seqlens_q, cu_seqlens_k, B, Hq, Hkv, max_seqlen_q, max_seqlen_k,
                         total_q, total_k, D, softmax_scale, causal, window, stream, DT_BF16);
}
extern "C" int fa_bwd_varlen(const void* q, const void* k, const void* v, const void* o, const void* dO,
                             const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_accum,
                             const int* cu_seqlens_q, const int* cu_seqlens_k, int B, int Hq, int Hkv,
                             int max_seqlen_q, int max_seqlen_k, int total_q, int total_k, int D, float softmax_scale,
                             int causal, int window, int deterministic, void* stream) {
  return bwd_varlen_impl(q, k, v, o, dO, lse, dq, dk, dv, delta, dq_accum, cu_seqlens_q, cu_seqlens_k, B, Hq, Hkv,
                         max_seqlen_q, max_seqlen_k, total_q, total_k, D, softmax_scale, causal, window, deterministic, stream,
                         DT_F16);
}
extern "C" int fa_bwd_varlen_bf16(const void* q, const void* k, const void* v, const void* o, const void* dO,
                                  const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_accum,
                                  const int* cu_seqlens_q, const int* cu_seqlens_k, int B, int Hq, int Hkv,
                                  int max_seqlen_q, int max_seqlen_k, int total_q, int total_k, int D,
                                  float softmax_scale, int causal, int window, int deterministic, void* stream) {
  return bwd_varlen_impl(q, k, v, o, dO, lse, dq, dk, dv, delta, dq_accum, cu_seqlens_q, cu_seqlens_k, B, Hq, Hkv,
                         max_seqlen_q, max_seqlen_k, total_q, total_k, D, softmax_scale, causal, window, deterministic, stream,
                         DT_BF16);
}

extern "C" int fa_fwd_paged(const void* q, const void* k_cache, const void* v_cache, void* o, float* lse,
                            const int* cu_seqlens_q, const int* seqlens_k, const int* block_table, int B, int Hq,
                            int Hkv, int max_seqlen_q, int max_seqlen_k, int total_q, int num_pages, int page_size,
                            int max_pages_per_seq, int D, float softmax_scale, int causal, int window, void* stream) {
  return fwd_paged_impl(q, k_cache, v_cache, o, lse, cu_seqlens_q, seqlens_k, block_table, B, Hq, Hkv, max_seqlen_q,
                        max_seqlen_k, total_q, num_pages, page_size, max_pages_per_seq, D, softmax_scale, causal,
                        window, stream, DT_F16);
}
extern "C" int fa_fwd_paged_bf16(const void* q, const void* k_cache, const void* v_cache, void* o, float* lse,
                                 const int* cu_seqlens_q, const int* seqlens_k, const int* block_table, int B, int Hq,
                                 int Hkv, int max_seqlen_q, int max_seqlen_k, int total_q, int num_pages,
                                 int page_size, int max_pages_per_seq, int D, float softmax_scale, int causal,
                                 int window, void* stream) {
  return fwd_paged_impl(q, k_cache, v_cache, o, lse, cu_seqlens_q, seqlens_k, block_table, B, Hq, Hkv, max_seqlen_q,
                        max_seqlen_k, total_q, num_pages, page_size, max_pages_per_seq, D, softmax_scale, causal,
                        window, stream, DT_BF16);
}

extern "C" int fa_fwd_paged_split(const void* q, const void* k_cache, const void* v_cache, void* o_part,
                                  float* lse_part, const int* cu_seqlens_q, const int* seqlens_k,
                                  const int* block_table, int B, int Hq, int Hkv, int max_seqlen_q, int max_seqlen_k,
                                  int total_q, int num_pages, int page_size, int max_pages_per_seq, int D,
                                  float softmax_scale, int causal, int splits, void* stream) {
  return fwd_paged_impl(q, k_cache, v_cache, o_part, lse_part, cu_seqlens_q, seqlens_k, block_table, B, Hq, Hkv,
                        max_seqlen_q, max_seqlen_k, total_q, num_pages, page_size, max_pages_per_seq, D,
                        softmax_scale, causal, 0, stream, DT_F16, splits);
}
extern "C" int fa_fwd_paged_split_bf16(const void* q, const void* k_cache, const void* v_cache, void* o_part,
                                       float* lse_part, const int* cu_seqlens_q, const int* seqlens_k,
                                       const int* block_table, int B, int Hq, int Hkv, int max_seqlen_q,
                                       int max_seqlen_k, int total_q, int num_pages, int page_size,
                                       int max_pages_per_seq, int D, float softmax_scale, int causal, int splits,
                                       void* stream) {
  return fwd_paged_impl(q, k_cache, v_cache, o_part, lse_part, cu_seqlens_q, seqlens_k, block_table, B, Hq, Hkv,
                        max_seqlen_q, max_seqlen_k, total_q, num_pages, page_size, max_pages_per_seq, D,
                        softmax_scale, causal, 0, stream, DT_BF16, splits);
}
extern "C" int fa_combine_splits(const void* o_part, const float* lse_part, void* o, float* lse, int splits,
                                 int total_q, int H, int D, void* stream) {
  return combine_impl(o_part, lse_part, o, lse, splits, total_q, H, D, stream, DT_F16);
}
extern "C" int fa_combine_splits_bf16(const void* o_part, const float* lse_part, void* o, float* lse, int splits,
                                      int total_q, int H, int D, void* stream) {
  return combine_impl(o_part, lse_part, o, lse, splits, total_q, H, D, stream, DT_BF16);
}

extern "C" int fa_device_status(int reset) {
  if (cudaDeviceSynchronize() != cudaSuccess) return FA_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)) != cudaSuccess) return FA_ERR_LAUNCH;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)) != cudaSuccess) return FA_ERR_LAUNCH;
  }
  return v;
}

namespace fa {
namespace {
std::atomic<const char*> g_last_cuda_error{nullptr};
}  // namespace
void record_cuda_error(cudaError_t e) { g_last_cuda_error.store(cudaGetErrorString(e)); }
const char* last_cuda_error_text() {
  const char* t = g_last_cuda_error.load();
  return t ? t : "a CUDA runtime call failed";
}
}  // namespace fa

extern "C" const char* fa_status_string(int code) {
  switch (code & 0xff) {
    case FA_OK: return "ok";
    case FA_ERR_UNSUPPORTED_HEAD_DIM: return "head_dim must be one of (32, 64, 128)";
    case FA_ERR_BAD_SHAPE: return "invalid shape, pointer or scale";
    case FA_ERR_MISALIGNED: return "pointer or stride is not 16-byte aligned (TMA requirement)";
    case FA_ERR_LAUNCH: return "CUDA kernel launch failed";
    case FA_ERR_TENSOR_MAP: return "cuTensorMapEncodeTiled rejected a tensor map";
    case FA_ERR_DRIVER: return "CUDA driver entry point cuTensorMapEncodeTiled unavailable";
    case FA_ERR_DEVICE_TIMEOUT: return "a kernel wait timed out on the device";
    case FA_ERR_NO_DEVICE: return "no sm_100 CUDA device is current";
    case FA_ERR_SCRATCH_LIMIT: return "the call needs more scratch than FA_NOALLOC_SCRATCH_BYTES (32 MiB)";
    case FA_ERR_OUT_OF_MEMORY: return "out of device memory for the library's scratch array";
    case FA_ERR_CUDA: return last_cuda_error_text();
    default: return "unknown error";
  }
}

// Value head size different from the query/key head size.
extern "C" int fa_fwd_vdim(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq, int Hkv,
                           int Nq, int Nk, int D, int Dv, const int64_t* q_strides, const int64_t* k_strides,
                           const int64_t* v_strides, const int64_t* o_strides, float softmax_scale, int causal,
                           void* stream) {
  return fwd_dense_impl(q, k, v, o, lse, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides, k_strides, v_strides, o_strides,
                       softmax_scale, causal, stream, DT_F16);
}
extern "C" int fa_fwd_vdim_bf16(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq,
                                int Hkv, int Nq, int Nk, int D, int Dv, const int64_t* q_strides,
                                const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                                float softmax_scale, int causal, void* stream) {
  return fwd_dense_impl(q, k, v, o, lse, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides, k_strides, v_strides, o_strides,
                       softmax_scale, causal, stream, DT_BF16);
}
extern "C" int fa_bwd_vdim(const void* q, const void* k, const void* v, const void* o, const void* dO,
                           const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_accum, int B,
                           int Hq, int Hkv, int Nq, int Nk, int D, int Dv, const int64_t* q_strides,
                           const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                           const int64_t* do_strides, const int64_t* dq_strides, const int64_t* dk_strides,
                           const int64_t* dv_strides, float softmax_scale, int causal, int deterministic,
                           void* stream) {
  return bwd_dense_impl(q, k, v, o, dO, lse, dq, dk, dv, delta, dq_accum, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides,
                       k_strides, v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides, softmax_scale,
                       causal, deterministic, stream, DT_F16);
}
extern "C" int fa_bwd_vdim_bf16(const void* q, const void* k, const void* v, const void* o, const void* dO,
                                const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_accum, int B,
                                int Hq, int Hkv, int Nq, int Nk, int D, int Dv, const int64_t* q_strides,
                                const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                                const int64_t* do_strides, const int64_t* dq_strides, const int64_t* dk_strides,
                                const int64_t* dv_strides, float softmax_scale, int causal, int deterministic,
                                void* stream) {
  return bwd_dense_impl(q, k, v, o, dO, lse, dq, dk, dv, delta, dq_accum, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides,
                       k_strides, v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides, softmax_scale,
                       causal, deterministic, stream, DT_BF16);
}

// Dense boolean masks.
extern "C" int fa_mask_pack(const void* mask, int Bm, int Hm, int Nq, int Nk, const int64_t* mask_strides,
                            uint32_t* bits, uint32_t* bits_t, void* stream) {
  if (Bm <= 0 || Hm <= 0 || Nq <= 0 || Nk <= 0 || !mask || !mask_strides || !bits || !bits_t) return FA_ERR_BAD_SHAPE;
  for (int i = 0; i < 4; ++i)
    if (mask_strides[i] < 0) return FA_ERR_BAD_SHAPE;
  if (!aligned16(bits) || !aligned16(bits_t)) return FA_ERR_MISALIGNED;
  return launch_mask_pack(mask, mask_strides[0], mask_strides[1], mask_strides[2], mask_strides[3], Bm, Hm, Nq, Nk,
                          bits, bits_t, static_cast<cudaStream_t>(stream));
}
static int fwd_masked_entry(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq, int Hkv,
                            int Nq, int Nk, int D, int Dv, const int64_t* q_strides, const int64_t* k_strides,
                            const int64_t* v_strides, const int64_t* o_strides, const uint32_t* mask_bits,
                            const int64_t* mask_strides, float softmax_scale, int causal, void* stream, int dtype) {
  if (!mask_bits || !mask_strides) return FA_ERR_BAD_SHAPE;
  return fwd_dense_impl(q, k, v, o, lse, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides, k_strides, v_strides, o_strides,
                       softmax_scale, causal, stream, dtype, mask_bits, mask_strides);
}
extern "C" int fa_fwd_masked(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq, int Hkv,
                             int Nq, int Nk, int D, int Dv, const int64_t* q_strides, const int64_t* k_strides,
                             const int64_t* v_strides, const int64_t* o_strides, const uint32_t* mask_bits,
                             const int64_t* mask_strides, float softmax_scale, int causal, void* stream) {
  return fwd_masked_entry(q, k, v, o, lse, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides, k_strides, v_strides, o_strides,
                          mask_bits, mask_strides, softmax_scale, causal, stream, DT_F16);
}
extern "C" int fa_fwd_masked_bf16(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq,
                                  int Hkv, int Nq, int Nk, int D, int Dv, const int64_t* q_strides,
                                  const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                                  const uint32_t* mask_bits, const int64_t* mask_strides, float softmax_scale,
                                  int causal, void* stream) {
  return fwd_masked_entry(q, k, v, o, lse, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides, k_strides, v_strides, o_strides,
                          mask_bits, mask_strides, softmax_scale, causal, stream, DT_BF16);
}
static int bwd_masked_entry(const void* q, const void* k, const void* v, const void* o, const void* dO,
                            const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_accum, int B,
                            int Hq, int Hkv, int Nq, int Nk, int D, int Dv, const int64_t* q_strides,
                            const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                            const int64_t* do_strides, const int64_t* dq_strides, const int64_t* dk_strides,
                            const int64_t* dv_strides, const uint32_t* mask_bits, const int64_t* mask_strides,
                            const uint32_t* mask_bits_t, const int64_t* mask_t_strides, float softmax_scale,
                            int causal, int deterministic, void* stream, int dtype) {
  if (!mask_bits || !mask_strides || !mask_bits_t || !mask_t_strides) return FA_ERR_BAD_SHAPE;
  return bwd_dense_impl(q, k, v, o, dO, lse, dq, dk, dv, delta, dq_accum, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides,
                       k_strides, v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides, softmax_scale,
                       causal, deterministic, stream, dtype, mask_bits, mask_strides, mask_bits_t, mask_t_strides);
}
extern "C" int fa_bwd_masked(const void* q, const void* k, const void* v, const void* o, const void* dO,
                             const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_accum, int B,
                             int Hq, int Hkv, int Nq, int Nk, int D, int Dv, const int64_t* q_strides,
                             const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                             const int64_t* do_strides, const int64_t* dq_strides, const int64_t* dk_strides,
                             const int64_t* dv_strides, const uint32_t* mask_bits, const int64_t* mask_strides,
                             const uint32_t* mask_bits_t, const int64_t* mask_t_strides, float softmax_scale,
                             int causal, int deterministic, void* stream) {
  return bwd_masked_entry(q, k, v, o, dO, lse, dq, dk, dv, delta, dq_accum, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides,
                          k_strides, v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides, mask_bits,
                          mask_strides, mask_bits_t, mask_t_strides, softmax_scale, causal, deterministic, stream,
                          DT_F16);
}
extern "C" int fa_bwd_masked_bf16(const void* q, const void* k, const void* v, const void* o, const void* dO,
                                  const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_accum,
                                  int B, int Hq, int Hkv, int Nq, int Nk, int D, int Dv, const int64_t* q_strides,
                                  const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                                  const int64_t* do_strides, const int64_t* dq_strides, const int64_t* dk_strides,
                                  const int64_t* dv_strides, const uint32_t* mask_bits, const int64_t* mask_strides,
                                  const uint32_t* mask_bits_t, const int64_t* mask_t_strides, float softmax_scale,
                                  int causal, int deterministic, void* stream) {
  return bwd_masked_entry(q, k, v, o, dO, lse, dq, dk, dv, delta, dq_accum, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides,
                          k_strides, v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides, mask_bits,
                          mask_strides, mask_bits_t, mask_t_strides, softmax_scale, causal, deterministic, stream,
                          DT_BF16);
}

// Attention dropout.
static int drop_args(float p, uint64_t seed, DropArgs* d) {
  if (!(p > 0.f && p < 1.f)) return FA_ERR_BAD_SHAPE;
  long t = std::lrint(double(p) * 256.0);
  if (t < 1) t = 1;
  if (t > 255) t = 255;
  d->t = uint32_t(t);
  d->r = float(256.0 / double(256 - t));
  d->seed_lo = uint32_t(seed);
  d->seed_hi = uint32_t(seed >> 32);
  return FA_OK;
}
static int fwd_dropout_entry(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq, int Hkv,
                             int Nq, int Nk, int D, int Dv, const int64_t* q_strides, const int64_t* k_strides,
                             const int64_t* v_strides, const int64_t* o_strides, float dropout_p, uint64_t seed,
                             float softmax_scale, int causal, void* stream, int dtype) {
  DropArgs d;
  int rc = drop_args(dropout_p, seed, &d);
  if (rc) return rc;
  return fwd_dense_impl(q, k, v, o, lse, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides, k_strides, v_strides, o_strides,
                       softmax_scale, causal, stream, dtype, nullptr, nullptr, &d);
}
extern "C" int fa_fwd_dropout(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq,
                              int Hkv, int Nq, int Nk, int D, int Dv, const int64_t* q_strides,
                              const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                              float dropout_p, uint64_t seed, float softmax_scale, int causal, void* stream) {
  return fwd_dropout_entry(q, k, v, o, lse, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides, k_strides, v_strides, o_strides,
                           dropout_p, seed, softmax_scale, causal, stream, DT_F16);
}
extern "C" int fa_fwd_dropout_bf16(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq,
                                   int Hkv, int Nq, int Nk, int D, int Dv, const int64_t* q_strides,
                                   const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                                   float dropout_p, uint64_t seed, float softmax_scale, int causal, void* stream) {
  return fwd_dropout_entry(q, k, v, o, lse, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides, k_strides, v_strides, o_strides,
                           dropout_p, seed, softmax_scale, causal, stream, DT_BF16);
}
static int bwd_dropout_entry(const void* q, const void* k, const void* v, const void* o, const void* dO,
                             const float* lse, void* dq, void* dk, void* dv, float* delta, int B, int Hq, int Hkv,
                             int Nq, int Nk, int D, int Dv, const int64_t* q_strides, const int64_t* k_strides,
                             const int64_t* v_strides, const int64_t* o_strides, const int64_t* do_strides,
                             const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                             float dropout_p, uint64_t seed, float softmax_scale, int causal, void* stream,
                             int dtype) {
  DropArgs d;
  int rc = drop_args(dropout_p, seed, &d);
  if (rc) return rc;
  return bwd_dense_impl(q, k, v, o, dO, lse, dq, dk, dv, delta, nullptr, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides,
                       k_strides, v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides, softmax_scale,
                       causal, 1, stream, dtype, nullptr, nullptr, nullptr, nullptr, &d);
}
extern "C" int fa_bwd_dropout(const void* q, const void* k, const void* v, const void* o, const void* dO,
                              const float* lse, void* dq, void* dk, void* dv, float* delta, int B, int Hq, int Hkv,
                              int Nq, int Nk, int D, int Dv, const int64_t* q_strides, const int64_t* k_strides,
                              const int64_t* v_strides, const int64_t* o_strides, const int64_t* do_strides,
                              const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                              float dropout_p, uint64_t seed, float softmax_scale, int causal, void* stream) {
  return bwd_dropout_entry(q, k, v, o, dO, lse, dq, dk, dv, delta, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides, k_strides,
                           v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides, dropout_p, seed,
                           softmax_scale, causal, stream, DT_F16);
}
extern "C" int fa_bwd_dropout_bf16(const void* q, const void* k, const void* v, const void* o, const void* dO,
                                   const float* lse, void* dq, void* dk, void* dv, float* delta, int B, int Hq,
                                   int Hkv, int Nq, int Nk, int D, int Dv, const int64_t* q_strides,
                                   const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                                   const int64_t* do_strides, const int64_t* dq_strides, const int64_t* dk_strides,
                                   const int64_t* dv_strides, float dropout_p, uint64_t seed, float softmax_scale,
                                   int causal, void* stream) {
  return bwd_dropout_entry(q, k, v, o, dO, lse, dq, dk, dv, delta, B, Hq, Hkv, Nq, Nk, D, Dv, q_strides, k_strides,
                           v_strides, o_strides, do_strides, dq_strides, dk_strides, dv_strides, dropout_p, seed,
                           softmax_scale, causal, stream, DT_BF16);
}

extern "C" int fa_version(void) { return 10600; }
