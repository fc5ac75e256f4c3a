/*
 * fa_b200.h -- C ABI of the B200 (sm_100a) FlashAttention-2 library.
 *
 * Plain pointers, sizes and element strides; no torch types.  Every entry
 * point is stateless and re-entrant, launches on the given CUDA stream
 * (cudaStream_t passed as void*, NULL = legacy default stream) and returns 0
 * on success or a nonzero FA_ERR_* code.  No exceptions cross this boundary.
 *
 * Layouts: q, o, dO, dq are (B, Hq, Nq, D) fp16; k, v, dk, dv are
 * (B, Hkv, Nk, D) fp16, each with element strides {batch, head, seq} and a
 * unit stride over D.  lse and delta are (B, Hq, Nq) fp32, contiguous.
 * D is 32, 64 or 128.  Hq % Hkv == 0; query head h reads K/V head
 * h / (Hq / Hkv).  TMA needs 16-byte aligned base pointers and strides.
 *
 * lse holds the base-2 log-sum-exp of each query row in the scaled domain:
 * lse2_i = log2(sum_j exp2(scale * log2(e) * q_i . k_j)), the same unit the
 * reference saves (triton_flash_attention/attention.py:177,230).
 *
 * Positions: query row i sits at global position q_offset + i and key row j
 * at k_offset + j.  With causal != 0 a key is visible iff its position is
 * <= the query's.  Zero offsets and Nq == Nk give the reference's
 * self-attention mask (attention.py:65,300,343); nonzero offsets serve ring
 * context parallelism, where one call sees one K/V chunk.  A query row with
 * no visible key gets o = 0 and lse = -inf.
 *
 * Every entry point has a _bf16 twin with the same signature that takes
 * bf16 instead of fp16 for q, k, v, o, dO and the non-fp32 gradients (the
 * reference's kernel path is fp16 only and sends bf16 inputs to PyTorch's
 * SDPA, attention.py:653-656; here both run on the B200 kernels, with P and
 * dS rounded to the operand type).
 *
 * accumulate_fp32 (backward only): 0 writes the gradient as fp16; nonzero
 * treats the gradient pointers as fp32 buffers with the same element strides
 * and adds this call's contribution to them (ring context parallelism sums a
 * chunk's gradient over the ranks this way).
 */
#ifndef FA_B200_H
#define FA_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define FA_API __attribute__((visibility("default")))
#else
#define FA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  FA_OK = 0,
  FA_ERR_UNSUPPORTED_HEAD_DIM = 1, /* D not in {32, 64, 128} */
  FA_ERR_BAD_SHAPE = 2,            /* a size <= 0, Hq % Hkv != 0, ... */
  FA_ERR_MISALIGNED = 3,           /* pointer or stride breaks TMA's 16-byte rule */
  FA_ERR_LAUNCH = 4,               /* the CUDA launch itself failed */
  FA_ERR_TENSOR_MAP = 5,           /* cuTensorMapEncodeTiled refused a descriptor */
  FA_ERR_DRIVER = 6,               /* the driver entry point could not be resolved */
  FA_ERR_DEVICE_TIMEOUT = 7,       /* a kernel's bounded wait gave up (see fa_device_status) */
  FA_ERR_NO_DEVICE = 8,            /* no sm_100 device is current */
  FA_ERR_SCRATCH_LIMIT = 9,        /* the call needs more than FA_NOALLOC_SCRATCH_BYTES */
  FA_ERR_OUT_OF_MEMORY = 10,       /* the device had no memory for the library's scratch array */
  FA_ERR_CUDA = 11                 /* another CUDA runtime call failed (fa_status_string names it) */
};

/* Forward: O = softmax(scale * Q K^T [+ causal mask]) V and the base-2 LSE.
 * Replaces TritonAttention.forward's launch of _attn_fwd
 * (triton_flash_attention/attention.py:676-722, kernel :90-234). */
FA_API int fa_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
           int B, int Hq, int Hkv, int Nq, int Nk, int D,
           const int64_t* q_strides, const int64_t* k_strides,
           const int64_t* v_strides, const int64_t* o_strides,
           float softmax_scale, int causal, int q_offset, int k_offset,
           void* stream);

/* Backward preprocess: delta[b,h,i] = sum_d O[b,h,i,d] * dO[b,h,i,d] (fp32).
 * Replaces the _attn_bwd_preprocess launch (attention.py:731-744, kernel
 * :237-255). */
FA_API int fa_bwd_delta(const void* o, const void* dO, float* delta,
                 int B, int H, int N, int D,
                 const int64_t* o_strides, const int64_t* do_strides,
                 void* stream);

/* Backward dQ: dQ = scale * sum_j dS_ij K_j with P rebuilt from lse and
 * dS = P (dO V^T - delta).  Replaces the dQ half of _attn_bwd
 * (attention.py:507-573, inner loop :311-350). */
FA_API int fa_bwd_dq(const void* q, const void* k, const void* v, const void* dO,
              const float* lse, const float* delta, void* dq,
              int B, int Hq, int Hkv, int Nq, int Nk, int D,
              const int64_t* q_strides, const int64_t* k_strides,
              const int64_t* v_strides, const int64_t* do_strides,
              const int64_t* dq_strides,
              float softmax_scale, int causal, int q_offset, int k_offset,
              int accumulate_fp32, void* stream);

/* Backward dK/dV: dV = sum_i P^T dO, dK = scale * sum_i dS^T Q, summed over
 * the Hq/Hkv query heads of each K/V head inside one CTA (deterministic, no
 * atomics).  Replaces the dK/dV half of _attn_bwd and its GQA atomics
 * (attention.py:428-505, inner loop :258-308). */
FA_API int fa_bwd_dkdv(const void* q, const void* k, const void* v, const void* dO,
                const float* lse, const float* delta, void* dk, void* dv,
                int B, int Hq, int Hkv, int Nq, int Nk, int D,
                const int64_t* q_strides, const int64_t* k_strides,
                const int64_t* v_strides, const int64_t* do_strides,
                const int64_t* dk_strides, const int64_t* dv_strides,
                float softmax_scale, int causal, int q_offset, int k_offset,
                int accumulate_fp32, void* stream);

/* Merge a partial attention result into a running one (ring context
 * parallelism): with L = log2(2^lse_acc + 2^lse_part),
 * o_acc = o_acc 2^(lse_acc - L) + o_part 2^(lse_part - L), lse_acc = L.
 * o_acc/o_part are (B, H, N, D) fp32/fp16 contiguous, lse (B, H, N) fp32.
 * No counterpart in the reference (single GPU only). */
FA_API int fa_merge_partial(float* o_acc, float* lse_acc, const void* o_part,
                     const float* lse_part, int B, int H, int N, int D,
                     void* stream);

/* Fused backward, step 1 of 3: delta as fa_bwd_delta, and dq_accum -- the
 * caller's contiguous (B, H, N, D) fp32 buffer -- set to zero on the way
 * (dq_accum may be NULL).  Same role as fa_bwd_delta (attention.py:731-744). */
FA_API int fa_bwd_preprocess(const void* o, const void* dO, float* delta, float* dq_accum,
                      int B, int H, int N, int D,
                      const int64_t* o_strides, const int64_t* do_strides,
                      void* stream);

/* Fused backward, step 2 of 3 (D = 32, 64 or 128): dK, dV as fa_bwd_dkdv
 * and, in the same pass over the (key tile, query tile) pairs, dQ added into
 * dq_accum, the caller's contiguous (B, Hq, Nq, D) fp32 buffer (with
 * position offsets, the ring's fp32 dQ accumulator of a chunk: the partials
 * add to what it holds).  Replaces the
 * whole _attn_bwd launch (attention.py:746-783, kernel :383-573), which
 * rebuilds P and dS once for dK/dV and once for dQ; here they are built once.
 * dQ is summed with fp32 reduce-adds whose order follows the schedule, so it
 * is not bitwise reproducible run to run (dK, dV are).  The library
 * allocates nothing: dq_accum is the only scratch and the caller owns it. */
FA_API int fa_bwd_fused(const void* q, const void* k, const void* v, const void* dO,
                 const float* lse, const float* delta, float* dq_accum,
                 void* dk, void* dv,
                 int B, int Hq, int Hkv, int Nq, int Nk, int D,
                 const int64_t* q_strides, const int64_t* k_strides,
                 const int64_t* v_strides, const int64_t* do_strides,
                 const int64_t* dk_strides, const int64_t* dv_strides,
                 float softmax_scale, int causal, int q_offset, int k_offset,
                 int accumulate_fp32, void* stream);

/* Fused backward, step 3 of 3: dq (element strides {batch, head, seq}) =
 * dq_accum (contiguous (B, H, N, D) fp32) rounded to fp16. */
FA_API int fa_bwd_dq_convert(const float* dq_accum, void* dq, int B, int H, int N, int D,
                      const int64_t* dq_strides, void* stream);

/* bf16 twins of the entry points above (same arguments). */
FA_API int fa_fwd_bf16(const void* q, const void* k, const void* v, void* o, float* lse,
                int B, int Hq, int Hkv, int Nq, int Nk, int D,
                const int64_t* q_strides, const int64_t* k_strides,
                const int64_t* v_strides, const int64_t* o_strides,
                float softmax_scale, int causal, int q_offset, int k_offset,
                void* stream);
FA_API int fa_bwd_delta_bf16(const void* o, const void* dO, float* delta,
                      int B, int H, int N, int D,
                      const int64_t* o_strides, const int64_t* do_strides,
                      void* stream);
FA_API int fa_bwd_dq_bf16(const void* q, const void* k, const void* v, const void* dO,
                   const float* lse, const float* delta, void* dq,
                   int B, int Hq, int Hkv, int Nq, int Nk, int D,
                   const int64_t* q_strides, const int64_t* k_strides,
                   const int64_t* v_strides, const int64_t* do_strides,
                   const int64_t* dq_strides,
                   float softmax_scale, int causal, int q_offset, int k_offset,
                   int accumulate_fp32, void* stream);
FA_API int fa_bwd_dkdv_bf16(const void* q, const void* k, const void* v, const void* dO,
                     const float* lse, const float* delta, void* dk, void* dv,
                     int B, int Hq, int Hkv, int Nq, int Nk, int D,
                     const int64_t* q_strides, const int64_t* k_strides,
                     const int64_t* v_strides, const int64_t* do_strides,
                     const int64_t* dk_strides, const int64_t* dv_strides,
                     float softmax_scale, int causal, int q_offset, int k_offset,
                     int accumulate_fp32, void* stream);
FA_API int fa_merge_partial_bf16(float* o_acc, float* lse_acc, const void* o_part,
                          const float* lse_part, int B, int H, int N, int D,
                          void* stream);
FA_API int fa_bwd_preprocess_bf16(const void* o, const void* dO, float* delta, float* dq_accum,
                           int B, int H, int N, int D,
                           const int64_t* o_strides, const int64_t* do_strides,
                           void* stream);
FA_API int fa_bwd_fused_bf16(const void* q, const void* k, const void* v, const void* dO,
                      const float* lse, const float* delta, float* dq_accum,
                      void* dk, void* dv,
                      int B, int Hq, int Hkv, int Nq, int Nk, int D,
                      const int64_t* q_strides, const int64_t* k_strides,
                      const int64_t* v_strides, const int64_t* do_strides,
                      const int64_t* dk_strides, const int64_t* dv_strides,
                      float softmax_scale, int causal, int q_offset, int k_offset,
                      int accumulate_fp32, void* stream);
FA_API int fa_bwd_dq_convert_bf16(const float* dq_accum, void* dq, int B, int H, int N, int D,
                           const int64_t* dq_strides, void* stream);

/* Packed variable-length batches (varlen).  No counterpart in the reference,
 * which takes (B, H, N, D) tensors of one length only (attention.py:584-626);
 * this is the layout serving and packed-sequence training use.  q, o, dO, dq
 * are contiguous (total_q, Hq, D) and k, v, dk, dv contiguous
 * (total_k, Hkv, D) in the operand type; cu_seqlens_q / cu_seqlens_k are
 * device int32 arrays of B + 1 prefix sums (cu[0] = 0, cu[B] = total):
 * batch b owns query rows [cu_q[b], cu_q[b+1]) and key rows
 * [cu_k[b], cu_k[b+1]).  max_seqlen_q / max_seqlen_k must be at least the
 * longest batch's lengths (they size the launch).  lse and delta are
 * (Hq, total_q) fp32.  Causal masking is per batch and top-left aligned
 * (query i of a batch sees its keys j <= i), as in the dense calls.  A
 * batch may be empty; a query row with no visible key gets o = 0 and
 * lse = -inf.  total_q and total_k must be positive.  window > 0 (causal
 * only) is a sliding window: a query sees only the window keys ending at
 * its own position (key j is visible iff pos - window < j <= pos); 0 means
 * no window. */
FA_API int fa_fwd_varlen(const void* q, const void* k, const void* v, void* o, float* lse,
                  const int* cu_seqlens_q, const int* cu_seqlens_k, int B, int Hq, int Hkv,
                  int max_seqlen_q, int max_seqlen_k, int total_q, int total_k, int D,
                  float softmax_scale, int causal, int window, void* stream);
/* The whole varlen backward: delta (caller's (Hq, total_q) fp32 buffer) and
 * dq, dk, dv.  D <= 64 with deterministic == 0 runs the fused pass and needs
 * dq_accum, a caller's (Hq, total_q, D) fp32 scratch buffer (zeroed here);
 * otherwise the separate dQ and dK/dV kernels run (bitwise reproducible) and
 * dq_accum may be NULL. */
FA_API int fa_bwd_varlen(const void* q, const void* k, const void* v, const void* o, const void* dO,
                  const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_accum,
                  const int* cu_seqlens_q, const int* cu_seqlens_k, int B, int Hq, int Hkv,
                  int max_seqlen_q, int max_seqlen_k, int total_q, int total_k, int D,
                  float softmax_scale, int causal, int window, int deterministic, void* stream);
FA_API int fa_fwd_varlen_bf16(const void* q, const void* k, const void* v, void* o, float* lse,
                       const int* cu_seqlens_q, const int* cu_seqlens_k, int B, int Hq, int Hkv,
                       int max_seqlen_q, int max_seqlen_k, int total_q, int total_k, int D,
                       float softmax_scale, int causal, int window, void* stream);
FA_API int fa_bwd_varlen_bf16(const void* q, const void* k, const void* v, const void* o, const void* dO,
                       const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_accum,
                       const int* cu_seqlens_q, const int* cu_seqlens_k, int B, int Hq, int Hkv,
                       int max_seqlen_q, int max_seqlen_k, int total_q, int total_k, int D,
                       float softmax_scale, int causal, int window, int deterministic, void* stream);

/* Forward over a paged K/V cache.  No counterpart in the reference (it has
 * no cache); this is the layout serving engines keep keys and values in.
 * Queries, o and lse as in fa_fwd_varlen (packed (total_q, Hq, D), cu_seqlens_q,
 * lse (Hq, total_q)).  k_cache / v_cache are contiguous
 * (num_pages, page_size, Hkv, D); batch b has seqlens_k[b] keys (device int32
 * array of B), and its key j is row j % page_size of page
 * block_table[b * max_pages_per_seq + j / page_size] (device int32 array of
 * B * max_pages_per_seq).  page_size is a power of two, at least 16.  The
 * causal mask is bottom-right aligned, the KV-cache convention: query i of a
 * batch with nq queries and nk keys sees keys j <= i + nk - nq.  Cache rows
 * past a batch's length (in its last page) must hold finite values: their
 * keys are masked, but their values still meet a zero weight in the P V
 * product.  window as in fa_fwd_varlen (positions bottom-right aligned).
 * Forward only. */
FA_API int fa_fwd_paged(const void* q, const void* k_cache, const void* v_cache, void* o, float* lse,
                 const int* cu_seqlens_q, const int* seqlens_k, const int* block_table,
                 int B, int Hq, int Hkv, int max_seqlen_q, int max_seqlen_k, int total_q,
                 int num_pages, int page_size, int max_pages_per_seq, int D,
                 float softmax_scale, int causal, int window, void* stream);
FA_API int fa_fwd_paged_bf16(const void* q, const void* k_cache, const void* v_cache, void* o, float* lse,
                      const int* cu_seqlens_q, const int* seqlens_k, const int* block_table,
                      int B, int Hq, int Hkv, int max_seqlen_q, int max_seqlen_k, int total_q,
                      int num_pages, int page_size, int max_pages_per_seq, int D,
                      float softmax_scale, int causal, int window, void* stream);

/* Split-KV form of fa_fwd_paged for decode: when the (sequence, K/V head)
 * units are fewer than the SMs, each unit's key tiles are cut into `splits`
 * equal ranges of whole 128-key tiles, so that splits x units CTAs' worth of
 * work stream the cache.  Range s writes its partial output, normalised by
 * its own row sums, to o_part + s * total_q * Hq * D (o_part is
 * (splits, total_q, Hq, D), contiguous) and its base-2 log-sum-exp to
 * lse_part + s * Hq * total_q (lse_part is (splits, Hq, total_q) fp32); a
 * range that sees no key of a row writes 0 and -inf.  fa_combine_splits then
 * merges them.  Requires GQA packing (Hq / Hkv a power of two from 2 to 64,
 * max_seqlen_q * Hq / Hkv <= 256) and no window; 1 <= splits <=
 * min(FA_MAX_KV_SPLITS, key tiles).  No counterpart in the reference (no
 * paged path there). */
#define FA_MAX_KV_SPLITS 64
FA_API int fa_fwd_paged_split(const void* q, const void* k_cache, const void* v_cache, void* o_part,
                       float* lse_part, const int* cu_seqlens_q, const int* seqlens_k,
                       const int* block_table, int B, int Hq, int Hkv, int max_seqlen_q,
                       int max_seqlen_k, int total_q, int num_pages, int page_size,
                       int max_pages_per_seq, int D, float softmax_scale, int causal, int splits,
                       void* stream);
FA_API int fa_fwd_paged_split_bf16(const void* q, const void* k_cache, const void* v_cache,
                            void* o_part, float* lse_part, const int* cu_seqlens_q,
                            const int* seqlens_k, const int* block_table, int B, int Hq, int Hkv,
                            int max_seqlen_q, int max_seqlen_k, int total_q, int num_pages,
                            int page_size, int max_pages_per_seq, int D, float softmax_scale,
                            int causal, int splits, void* stream);

/* Combine the split partials of fa_fwd_paged_split: with
 * L = log2 sum_s 2^lse_part[s], o = sum_s o_part[s] 2^(lse_part[s] - L)
 * (rounded once to the operand type) and lse = L; rows every range missed
 * get 0 and -inf.  o is (total_q, H, D) contiguous, lse (H, total_q). */
FA_API int fa_combine_splits(const void* o_part, const float* lse_part, void* o, float* lse,
                      int splits, int total_q, int H, int D, void* stream);
FA_API int fa_combine_splits_bf16(const void* o_part, const float* lse_part, void* o, float* lse,
                           int splits, int total_q, int H, int D, void* stream);

/* Size of the scratch array fa_bwd_fused_noalloc uses: 32 MiB per device. */
#define FA_NOALLOC_SCRATCH_BYTES (32u << 20)

/* The whole fused backward (fa_bwd_preprocess + fa_bwd_fused +
 * fa_bwd_dq_convert; fp16, D = 32 or 64, zero position offsets) with no
 * scratch from the caller.  No counterpart in the reference: it exists for
 * callers that cannot allocate device memory -- engines and plugin hosts that
 * plan all device memory up front and forbid allocation while running, and
 * thin FFI bindings that hold tensor pointers but no device allocator.  The
 * caller passes the inputs (q, k, v, o, dO, lse) and the outputs (dq, dk, dv,
 * fp16, with their own element strides); Delta and the fp32 dQ accumulator
 * live in one file-scope __device__ array of FA_NOALLOC_SCRATCH_BYTES that
 * every device loading the library holds until exit.  A call needs
 * 4 * (roundup(B*Hq*Nq, 64) + B*Hq*Nq*D) bytes of it; larger calls return
 * FA_ERR_SCRATCH_LIMIT before touching the GPU.  The library allocates
 * nothing on this path.  The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress, with that device current); make that
 * first call before any stream capture.  When the lookup fails the call
 * returns FA_ERR_OUT_OF_MEMORY (the module that holds the array could not be
 * loaded) or FA_ERR_CUDA (any other runtime error, e.g. a lookup inside a
 * stream capture; fa_status_string(FA_ERR_CUDA) then gives CUDA's text).
 * The looked-up address is cached per device for the life of the process,
 * which assumes the device's primary context is never reset
 * (cudaDeviceReset) while the library is loaded.  All calls share the array and it
 * keeps the last call's contents (each call re-zeroes what must start at
 * zero), so calls that overlap on the GPU -- on two streams, or from two
 * host threads on one device -- race and give wrong gradients. */
FA_API int fa_bwd_fused_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dO,
                                const float* lse, void* dq, void* dk, void* dv,
                                int B, int Hq, int Hkv, int Nq, int Nk, int D,
                                const int64_t* q_strides, const int64_t* k_strides,
                                const int64_t* v_strides, const int64_t* o_strides,
                                const int64_t* do_strides, const int64_t* dq_strides,
                                const int64_t* dk_strides, const int64_t* dv_strides,
                                float softmax_scale, int causal, void* stream);

/* Attention whose value head size Dv differs from the query/key head size D
 * (dense (B, H, N, D) layout, as fa_fwd).  Replaces the reference's
 * dispatch of such inputs to PyTorch's SDPA (attention.py:639-646: the
 * Triton kernel takes one head size).  D and Dv are each 32, 64 or 128; q, k
 * are D wide, v, o, dO Dv wide; lse as in fa_fwd.  The kernels run at width
 * max(D, Dv), with the narrower operands' missing columns read as zeros, so
 * a call costs what an equal-width call of max(D, Dv) costs.  Zero position
 * offsets (no ring step).  fa_fwd_vdim also serves D == Dv. */
FA_API int fa_fwd_vdim(const void* q, const void* k, const void* v, void* o, float* lse,
                       int B, int Hq, int Hkv, int Nq, int Nk, int D, int Dv,
                       const int64_t* q_strides, const int64_t* k_strides,
                       const int64_t* v_strides, const int64_t* o_strides,
                       float softmax_scale, int causal, void* stream);
/* The whole backward for fa_fwd_vdim: delta (caller's (B, Hq, Nq) fp32
 * buffer), dq and dk (D wide), dv (Dv wide).  With max(D, Dv) <= 64 and
 * deterministic == 0 it runs the fused pass and needs dq_accum, a caller's
 * contiguous (B, Hq, Nq, max(D, Dv)) fp32 scratch buffer (zeroed here);
 * otherwise the separate dQ and dK/dV kernels run (bitwise reproducible)
 * and dq_accum may be NULL. */
FA_API int fa_bwd_vdim(const void* q, const void* k, const void* v, const void* o, const void* dO,
                       const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_accum,
                       int B, int Hq, int Hkv, int Nq, int Nk, int D, int Dv,
                       const int64_t* q_strides, const int64_t* k_strides,
                       const int64_t* v_strides, const int64_t* o_strides,
                       const int64_t* do_strides, const int64_t* dq_strides,
                       const int64_t* dk_strides, const int64_t* dv_strides,
                       float softmax_scale, int causal, int deterministic, void* stream);
FA_API int fa_fwd_vdim_bf16(const void* q, const void* k, const void* v, void* o, float* lse,
                            int B, int Hq, int Hkv, int Nq, int Nk, int D, int Dv,
                            const int64_t* q_strides, const int64_t* k_strides,
                            const int64_t* v_strides, const int64_t* o_strides,
                            float softmax_scale, int causal, void* stream);
FA_API int fa_bwd_vdim_bf16(const void* q, const void* k, const void* v, const void* o, const void* dO,
                            const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_accum,
                            int B, int Hq, int Hkv, int Nq, int Nk, int D, int Dv,
                            const int64_t* q_strides, const int64_t* k_strides,
                            const int64_t* v_strides, const int64_t* o_strides,
                            const int64_t* do_strides, const int64_t* dq_strides,
                            const int64_t* dk_strides, const int64_t* dv_strides,
                            float softmax_scale, int causal, int deterministic, void* stream);

/* Dense boolean attention masks.  No counterpart in the reference
 * (README.md:93: "Dropout and arbitrary attention masks are not currently
 * implemented").  fa_mask_pack turns a byte-per-position mask (a torch.bool
 * tensor: nonzero = the key takes part) of Bm x Hm x Nq x Nk positions with
 * element strides {batch, head, query, key} (0 broadcasts) into two
 * contiguous uint32 bit matrices:
 *   mask_bits   (Bm, Hm, Nq, roundup(Nk, 128) / 32): bit k & 31 of word k >> 5
 *               of row q is position (q, k);
 *   mask_bits_t (Bm, Hm, Nk, roundup(Nq, 128) / 32): the transpose.
 * Bits past Nq / Nk are zero.  Both buffers 16-byte aligned. */
FA_API int fa_mask_pack(const void* mask, int Bm, int Hm, int Nq, int Nk, const int64_t* mask_strides,
                        uint32_t* mask_bits, uint32_t* mask_bits_t, void* stream);
/* fa_fwd_vdim / fa_bwd_vdim with a packed mask: key k is visible to query q
 * of head h, batch b only if its bit is set (and, with causal != 0, also
 * k <= q).  mask_strides / mask_t_strides are word strides {batch, head,
 * row} of mask_bits / mask_bits_t (0 broadcasts over batches or heads; rows
 * at least the padded width; multiples of 4).  A query row that sees no key
 * gets o = 0 and lse = -inf (PyTorch's SDPA gives NaN there) and zero
 * gradients.  The forward reads mask_bits, the backward both. */
FA_API int fa_fwd_masked(const void* q, const void* k, const void* v, void* o, float* lse,
                         int B, int Hq, int Hkv, int Nq, int Nk, int D, int Dv,
                         const int64_t* q_strides, const int64_t* k_strides,
                         const int64_t* v_strides, const int64_t* o_strides,
                         const uint32_t* mask_bits, const int64_t* mask_strides,
                         float softmax_scale, int causal, void* stream);
FA_API int fa_bwd_masked(const void* q, const void* k, const void* v, const void* o, const void* dO,
                         const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_accum,
                         int B, int Hq, int Hkv, int Nq, int Nk, int D, int Dv,
                         const int64_t* q_strides, const int64_t* k_strides,
                         const int64_t* v_strides, const int64_t* o_strides,
                         const int64_t* do_strides, const int64_t* dq_strides,
                         const int64_t* dk_strides, const int64_t* dv_strides,
                         const uint32_t* mask_bits, const int64_t* mask_strides,
                         const uint32_t* mask_bits_t, const int64_t* mask_t_strides,
                         float softmax_scale, int causal, int deterministic, void* stream);
FA_API int fa_fwd_masked_bf16(const void* q, const void* k, const void* v, void* o, float* lse,
                              int B, int Hq, int Hkv, int Nq, int Nk, int D, int Dv,
                              const int64_t* q_strides, const int64_t* k_strides,
                              const int64_t* v_strides, const int64_t* o_strides,
                              const uint32_t* mask_bits, const int64_t* mask_strides,
                              float softmax_scale, int causal, void* stream);
FA_API int fa_bwd_masked_bf16(const void* q, const void* k, const void* v, const void* o, const void* dO,
                              const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_accum,
                              int B, int Hq, int Hkv, int Nq, int Nk, int D, int Dv,
                              const int64_t* q_strides, const int64_t* k_strides,
                              const int64_t* v_strides, const int64_t* o_strides,
                              const int64_t* do_strides, const int64_t* dq_strides,
                              const int64_t* dk_strides, const int64_t* dv_strides,
                              const uint32_t* mask_bits, const int64_t* mask_strides,
                              const uint32_t* mask_bits_t, const int64_t* mask_t_strides,
                              float softmax_scale, int causal, int deterministic, void* stream);

/* Attention dropout (PyTorch SDPA's dropout_p; the reference has none,
 * README.md:93).  fa_fwd_dropout is fa_fwd_vdim with the softmax
 * probabilities dropped at rate dropout_p and the kept ones scaled by
 * 1 / (1 - p); fa_bwd_dropout is its whole backward (Delta into the caller's
 * (B, Hq, Nq) fp32 buffer, then the separate dQ and dK/dV kernels; bitwise
 * reproducible).  dropout_p must lie in (0, 1) and is applied as
 * p = t / 256 with t = round(256 * dropout_p) clamped to [1, 255], the
 * scale as 256 / (256 - t).  Whether (query q, key k) of head h, batch b is
 * kept is a stateless function of (seed, b * Hq + h, q, k): one 32-bit word
 * per 2 x 2 block of positions, word = mix32(key2 ^ ((q >> 1) << 16 |
 * (k >> 1))) with the low 16 bits of each half, key2 = mix32(key_bh ^
 * ((q >> 17) << 16 | (k >> 17))), key_bh = mix32(seed_lo ^ mix32(seed_hi +
 * (b * Hq + h) * 0x9E3779B9)), mix32 the "lowbias32" hash (xorshift 16,
 * * 0x7feb352d, xorshift 15, * 0x846ca68b, xorshift 16); the position's
 * byte is byte 2 * (q & 1) + (k & 1) of the word and the value is kept iff
 * byte >= t.  The forward and the backward of one step take the same seed.
 * Dense layout, no mask, no window, no position offsets. */
FA_API int fa_fwd_dropout(const void* q, const void* k, const void* v, void* o, float* lse,
                          int B, int Hq, int Hkv, int Nq, int Nk, int D, int Dv,
                          const int64_t* q_strides, const int64_t* k_strides,
                          const int64_t* v_strides, const int64_t* o_strides,
                          float dropout_p, uint64_t seed, float softmax_scale, int causal, void* stream);
FA_API int fa_bwd_dropout(const void* q, const void* k, const void* v, const void* o, const void* dO,
                          const float* lse, void* dq, void* dk, void* dv, float* delta,
                          int B, int Hq, int Hkv, int Nq, int Nk, int D, int Dv,
                          const int64_t* q_strides, const int64_t* k_strides,
                          const int64_t* v_strides, const int64_t* o_strides,
                          const int64_t* do_strides, const int64_t* dq_strides,
                          const int64_t* dk_strides, const int64_t* dv_strides,
                          float dropout_p, uint64_t seed, float softmax_scale, int causal, void* stream);
FA_API int fa_fwd_dropout_bf16(const void* q, const void* k, const void* v, void* o, float* lse,
                               int B, int Hq, int Hkv, int Nq, int Nk, int D, int Dv,
                               const int64_t* q_strides, const int64_t* k_strides,
                               const int64_t* v_strides, const int64_t* o_strides,
                               float dropout_p, uint64_t seed, float softmax_scale, int causal, void* stream);
FA_API int fa_bwd_dropout_bf16(const void* q, const void* k, const void* v, const void* o, const void* dO,
                               const float* lse, void* dq, void* dk, void* dv, float* delta,
                               int B, int Hq, int Hkv, int Nq, int Nk, int D, int Dv,
                               const int64_t* q_strides, const int64_t* k_strides,
                               const int64_t* v_strides, const int64_t* o_strides,
                               const int64_t* do_strides, const int64_t* dq_strides,
                               const int64_t* dk_strides, const int64_t* dv_strides,
                               float dropout_p, uint64_t seed, float softmax_scale, int causal, void* stream);

/* Reads (and with reset != 0 clears) the device status word that kernels set
 * when a bounded wait gives up: 0 = healthy, else FA_ERR_DEVICE_TIMEOUT in the
 * low byte and the barrier site in bits 8..15.  Synchronises the device. */
FA_API int fa_device_status(int reset);

/* Human-readable text of an FA_ERR_* code. */
FA_API const char* fa_status_string(int code);

/* Library version: major * 10000 + minor * 100 + patch (1.1.0 adds bf16,
 * 1.2.0 the fused backward, 1.3.0 packed variable-length batches and the
 * paged K/V forward, 1.4.0 value head sizes different from D, 1.5.0 dense
 * boolean masks, 1.6.0 attention dropout). */
FA_API int fa_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FA_B200_H */
