// fa_bwd_aux.cu -- the HBM-bound helpers of the attention path.
//
//  * fa_delta_kernel: Delta_i = sum_d O_id * dO_id in fp32, the backward
//    preprocess of the reference (triton_flash_attention/attention.py:237-255).
//    Each row is read once with 16-byte loads, D/8 lanes per row, and reduced
//    with warp shuffles; a grid-stride loop sized to the SM count keeps every
//    SM streaming.  When O and dO are contiguous (the usual case) a lane's
//    vector is at element 8 * (vector index) of both, and every lane keeps
//    DELTA_UNROLL independent load pairs in flight: the strided path's
//    64-bit index arithmetic and its one pair per lane left the kernel
//    latency-bound at half the HBM rate.
//  * fa_merge_kernel: the log-sum-exp merge of ring context parallelism
//    (no counterpart in the reference).
// Both take fp16 or bf16 operands (template parameter DT).
#include "fa_kernels.h"

namespace fa {

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Dot product of 8 + 8 packed elements (fp16 or bf16) in fp32.
template <int DT>
__device__ __forceinline__ float dot8(uint4 a, uint4 b) {
  const uint32_t* ua = reinterpret_cast<const uint32_t*>(&a);
  const uint32_t* ub = reinterpret_cast<const uint32_t*>(&b);
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 fa = unpack2<DT>(ua[i]);
    const float2 fb = unpack2<DT>(ub[i]);
    acc = fmaf(fa.x, fb.x, acc);
    acc = fmaf(fa.y, fb.y, acc);
  }
  return acc;
}

constexpr int DELTA_UNROLL = 4;

template <int D, int DT>
__global__ void __launch_bounds__(256) fa_delta_kernel(const uint16_t* __restrict__ o, long long o_sb,
                                                       long long o_sh, long long o_sn,
                                                       const uint16_t* __restrict__ dO, long long do_sb,
                                                       long long do_sh, long long do_sn, float* __restrict__ delta,
                                                       float* __restrict__ zero_acc, int H, int N, long long rows,
                                                       int contiguous) {
  constexpr int TPR = D / 8;  // lanes per row, 8 elements each
  const long long total = rows * TPR;
  const long long nthreads = (long long)gridDim.x * blockDim.x;
  const int lane = int(threadIdx.x & 31);
  if (contiguous) {
    // vector idx = row * TPR + part sits at element 8 * idx of O, dO and (as
    // fp32) of the dQ accumulator; the warp's lanes stay within whole rows
    constexpr int U = DELTA_UNROLL;
    for (long long base = (long long)blockIdx.x * blockDim.x + (threadIdx.x & ~31); base < total;
         base += nthreads * U) {
      uint4 a[U], b[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long idx = base + u * nthreads + lane;
        if (idx < total) {
          a[u] = ld_nc_v4(o + idx * 8);
          b[u] = ld_nc_v4(dO + idx * 8);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const long long idx = base + u * nthreads + lane;
        const bool valid = idx < total;
        float acc = valid ? dot8<DT>(a[u], b[u]) : 0.f;
        if (valid && zero_acc) {
          float4* z = reinterpret_cast<float4*>(zero_acc + idx * 8);
          z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
          z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int off = TPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (valid && idx % TPR == 0) delta[idx / TPR] = acc;
      }
    }
    return;
  }
  for (long long base = (long long)blockIdx.x * blockDim.x + (threadIdx.x & ~31); base < total;
       base += nthreads) {
    const long long idx = base + (threadIdx.x & 31);
    const bool valid = idx < total;
    float acc = 0.f;
    long long row = 0;
    int part = 0;
    if (valid) {
      row = idx / TPR;
      part = int(idx % TPR);
      const int n = int(row % N);
      const long long bh = row / N;
      const int h = int(bh % H);
      const long long b = bh / H;
      const uint16_t* po = o + b * o_sb + h * o_sh + n * o_sn + part * 8;
      const uint16_t* pd = dO + b * do_sb + h * do_sh + n * do_sn + part * 8;
      acc = dot8<DT>(ld_nc_v4(po), ld_nc_v4(pd));
      if (zero_acc) {  // the fused backward's dQ accumulator, rows x D fp32
        float4* z = reinterpret_cast<float4*>(zero_acc + row * D + part * 8);
        z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
        z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int off = TPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (valid && part == 0) delta[row] = acc;
  }
}

template <int DT>
int launch_bwd_delta_t(const uint16_t* o, long long o_sb, long long o_sh, long long o_sn, const uint16_t* dO,
                       long long do_sb, long long do_sh, long long do_sn, float* delta, float* zero_acc, int B,
                       int H, int N, int D, cudaStream_t stream) {
  const int sms = device_sm_count();
  const long long rows = (long long)B * H * N;
  const long long work = rows * (D / 8);
  long long blocks = (work + 255) / 256;
  const long long cap = (long long)sms * 8;  // 8 x 256 threads resident per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const int contiguous = o_sn == D && o_sh == (long long)N * D && o_sb == (long long)H * N * D && do_sn == D &&
                         do_sh == (long long)N * D && do_sb == (long long)H * N * D;
  switch (D) {
    case 32:
      fa_delta_kernel<32, DT><<<unsigned(blocks), 256, 0, stream>>>(o, o_sb, o_sh, o_sn, dO, do_sb, do_sh, do_sn,
                                                                     delta, zero_acc, H, N, rows, contiguous);
      break;
    case 64:
      fa_delta_kernel<64, DT><<<unsigned(blocks), 256, 0, stream>>>(o, o_sb, o_sh, o_sn, dO, do_sb, do_sh, do_sn,
                                                                     delta, zero_acc, H, N, rows, contiguous);
      break;
    case 128:
      fa_delta_kernel<128, DT><<<unsigned(blocks), 256, 0, stream>>>(o, o_sb, o_sh, o_sn, dO, do_sb, do_sh, do_sn,
                                                                      delta, zero_acc, H, N, rows, contiguous);
      break;
    default:
      return FA_ERR_UNSUPPORTED_HEAD_DIM;
  }
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

int launch_bwd_delta(const void* o, long long o_sb, long long o_sh, long long o_sn, const void* dO,
                     long long do_sb, long long do_sh, long long do_sn, float* delta, float* zero_acc, int B, int H,
                     int N, int D, int dtype, cudaStream_t stream) {
  const uint16_t* o16 = static_cast<const uint16_t*>(o);
  const uint16_t* d16 = static_cast<const uint16_t*>(dO);
  return dtype == DT_BF16 ? launch_bwd_delta_t<DT_BF16>(o16, o_sb, o_sh, o_sn, d16, do_sb, do_sh, do_sn, delta,
                                                        zero_acc, B, H, N, D, stream)
                          : launch_bwd_delta_t<DT_F16>(o16, o_sb, o_sh, o_sn, d16, do_sb, do_sh, do_sn, delta,
                                                       zero_acc, B, H, N, D, stream);
}

// dq (operand type, element strides {sb, sh, sn, 1}) <- the first D columns
// of acc (contiguous [B, H, N, acc_w] fp32, acc_w >= D), eight elements per
// thread.
template <int DT>
__global__ void __launch_bounds__(256) fa_dq_convert_kernel(const float* __restrict__ acc, uint16_t* __restrict__ dq,
                                                            long long sb, long long sh, long long sn, int H, int N,
                                                            int D, int acc_w, long long rows) {
  const int vec_per_row = D / 8;
  const long long total = rows * vec_per_row;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long row = idx / vec_per_row;
    const int part = int(idx % vec_per_row);
    const int n = int(row % N);
    const long long bh = row / N;
    const int h = int(bh % H);
    const long long b = bh / H;
    const float4* src = reinterpret_cast<const float4*>(acc + row * acc_w + part * 8);
    const float4 x = src[0];
    const float4 y = src[1];
    uint4 pk;
    pk.x = pack2<DT>(x.x, x.y);
    pk.y = pack2<DT>(x.z, x.w);
    pk.z = pack2<DT>(y.x, y.y);
    pk.w = pack2<DT>(y.z, y.w);
    *reinterpret_cast<uint4*>(dq + b * sb + h * sh + n * sn + part * 8) = pk;
  }
}

int launch_dq_convert(const float* acc, void* dq, long long sb, long long sh, long long sn, int B, int H, int N, int D,
                      int dtype, cudaStream_t stream, int acc_w) {
  if (acc_w <= 0) acc_w = D;
  const long long rows = (long long)B * H * N;
  const long long work = rows * (D / 8);
  long long blocks = (work + 255) / 256;
  const long long cap = (long long)device_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  uint16_t* d16 = static_cast<uint16_t*>(dq);
  if (dtype == DT_BF16)
    fa_dq_convert_kernel<DT_BF16><<<unsigned(blocks), 256, 0, stream>>>(acc, d16, sb, sh, sn, H, N, D, acc_w, rows);
  else
    fa_dq_convert_kernel<DT_F16><<<unsigned(blocks), 256, 0, stream>>>(acc, d16, sb, sh, sn, H, N, D, acc_w, rows);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

// o_acc (rows x D fp32), lse_acc (rows) <- merge with o_part (fp16 or bf16), lse_part.
template <int DT>
__global__ void __launch_bounds__(256) fa_merge_kernel(float* __restrict__ o_acc, float* __restrict__ lse_acc,
                                                       const uint16_t* __restrict__ o_part,
                                                       const float* __restrict__ lse_part, long long rows, int D) {
  const int vec_per_row = D / 8;
  const long long total = rows * vec_per_row;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long row = idx / vec_per_row;
    const int part = int(idx % vec_per_row);
    const float a = lse_acc[row];
    const float bq = lse_part[row];
    const float mx = fmaxf(a, bq);
    float wa = 0.f, wb = 0.f, L = -INFINITY;
    if (mx != -INFINITY) {
      const float ea = exp2f(a - mx), eb = exp2f(bq - mx);
      const float tot = ea + eb;
      L = mx + log2f(tot);
      wa = ea / tot;
      wb = eb / tot;
    }
    float* po = o_acc + row * D + part * 8;
    const uint4 pk = *reinterpret_cast<const uint4*>(o_part + row * D + part * 8);
    float4 x0 = reinterpret_cast<float4*>(po)[0];
    float4 x1 = reinterpret_cast<float4*>(po)[1];
    const float2 p0 = unpack2<DT>(pk.x), p1 = unpack2<DT>(pk.y);
    const float2 p2 = unpack2<DT>(pk.z), p3 = unpack2<DT>(pk.w);
    x0.x = x0.x * wa + p0.x * wb;
    x0.y = x0.y * wa + p0.y * wb;
    x0.z = x0.z * wa + p1.x * wb;
    x0.w = x0.w * wa + p1.y * wb;
    x1.x = x1.x * wa + p2.x * wb;
    x1.y = x1.y * wa + p2.y * wb;
    x1.z = x1.z * wa + p3.x * wb;
    x1.w = x1.w * wa + p3.y * wb;
    reinterpret_cast<float4*>(po)[0] = x0;
    reinterpret_cast<float4*>(po)[1] = x1;
    // Every lane of the row read lse_acc[row] before this point in its own
    // iteration; the part-0 lane alone rewrites it after all lanes of the row
    // (same warp, consecutive lanes) have used the old value.
    __syncwarp(__activemask());
    if (part == 0) lse_acc[row] = L;
  }
}

// Split-KV combine: o (rows x D, operand type) and lse <- the S partials
// o_part (S x rows x D), lse_part (S x lse_stride): with L = log2 sum_s
// 2^lse_s, o = sum_s o_s 2^(lse_s - L), lse = L.  Row `row` = q * H + h of
// the packed (total_q, H, D) layout has its statistics at h * total_q + q.
template <int DT>
__global__ void __launch_bounds__(256) fa_combine_kernel(const uint16_t* __restrict__ o_part,
                                                         const float* __restrict__ lse_part,
                                                         uint16_t* __restrict__ o, float* __restrict__ lse, int S,
                                                         int total_q, int H, int D) {
  const int vec_per_row = D / 8;
  const long long rows = (long long)total_q * H;
  const long long total = rows * vec_per_row;
  const long long lse_stride = rows;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long row = idx / vec_per_row;
    const int part = int(idx % vec_per_row);
    const long long li = (long long)(row % H) * total_q + row / H;
    float mx = -INFINITY;
    for (int s = 0; s < S; ++s) mx = fmaxf(mx, lse_part[s * lse_stride + li]);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float L = -INFINITY;
    if (mx != -INFINITY) {
      float tot = 0.f;
      for (int s = 0; s < S; ++s) {
        const float wgt = exp2f(lse_part[s * lse_stride + li] - mx);
        tot += wgt;
        const uint4 pk = *reinterpret_cast<const uint4*>(o_part + (s * rows + row) * D + part * 8);
        const uint32_t w4[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 p = unpack2<DT>(w4[i]);
          acc[2 * i] += wgt * p.x;
          acc[2 * i + 1] += wgt * p.y;
        }
      }
      const float inv = 1.f / tot;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] *= inv;
      L = mx + log2f(tot);
    }
    uint4 out;
    out.x = pack2<DT>(acc[0], acc[1]);
    out.y = pack2<DT>(acc[2], acc[3]);
    out.z = pack2<DT>(acc[4], acc[5]);
    out.w = pack2<DT>(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(o + row * D + part * 8) = out;
    if (part == 0) lse[li] = L;
  }
}

int launch_combine_splits(const void* o_part, const float* lse_part, void* o, float* lse, int S, int total_q, int H,
                          int D, int dtype, cudaStream_t stream) {
  if (D != 32 && D != 64 && D != 128) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  const int sms = device_sm_count();
  long long blocks = ((long long)total_q * H * (D / 8) + 255) / 256;
  if (blocks > (long long)sms * 8) blocks = (long long)sms * 8;
  if (blocks < 1) blocks = 1;
  const uint16_t* p16 = static_cast<const uint16_t*>(o_part);
  uint16_t* o16 = static_cast<uint16_t*>(o);
  if (dtype == DT_BF16)
    fa_combine_kernel<DT_BF16><<<unsigned(blocks), 256, 0, stream>>>(p16, lse_part, o16, lse, S, total_q, H, D);
  else
    fa_combine_kernel<DT_F16><<<unsigned(blocks), 256, 0, stream>>>(p16, lse_part, o16, lse, S, total_q, H, D);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

int launch_merge_partial(float* o_acc, float* lse_acc, const void* o_part, const float* lse_part, long long rows,
                         int D, int dtype, cudaStream_t stream) {
  if (D != 32 && D != 64 && D != 128) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  const int sms = device_sm_count();
  long long blocks = (rows * (D / 8) + 255) / 256;
  if (blocks > (long long)sms * 8) blocks = (long long)sms * 8;
  if (blocks < 1) blocks = 1;
  const uint16_t* p16 = static_cast<const uint16_t*>(o_part);
  if (dtype == DT_BF16)
    fa_merge_kernel<DT_BF16><<<unsigned(blocks), 256, 0, stream>>>(o_acc, lse_acc, p16, lse_part, rows, D);
  else
    fa_merge_kernel<DT_F16><<<unsigned(blocks), 256, 0, stream>>>(o_acc, lse_acc, p16, lse_part, rows, D);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

}  // namespace fa
