// fa_noalloc.cu -- the whole fused backward (D = 32, 64, fp16) for callers
// that cannot allocate device memory.
//
// fa_bwd_fused needs two buffers besides its inputs and outputs: Delta
// (B*Hq*Nq fp32) and the fp32 dQ accumulator (B*Hq*Nq*D).  Some callers
// cannot provide them: serving engines and plugin hosts that plan all device
// memory up front and forbid allocation while they run (cudaMalloc and
// cudaFree may synchronise the device and fragment the pool), and thin FFI
// bindings that hold device pointers to their tensors but have no device
// allocator of their own.  fa_bwd_fused_noalloc takes that scratch from one
// file-scope __device__ array of FA_NOALLOC_SCRATCH_BYTES instead, which every
// device that loads this library holds until the process exits.
//
// The array's name in host code is a host-side stand-in, not a device
// address, so the host looks the address up with cudaGetSymbolAddress, once
// per device, with that device current (the first call on each device does
// this), and passes the pointer to the kernels.
//
// Every call shares the one array and it keeps the last call's contents: the
// preprocess kernel rewrites Delta and zeroes the accumulator on every call,
// so calls in sequence on one stream are independent, but calls that overlap
// on the GPU (two streams, or two host threads on one device) race on it.
#include <cuda_runtime.h>

#include <mutex>

#include "fa_kernels.h"

static constexpr size_t kScratchFloats = FA_NOALLOC_SCRATCH_BYTES / sizeof(float);

static __device__ __align__(256) float g_bwd_scratch[kScratchFloats];

namespace {

// Device address of this device's scratch array, looked up once per device.
// The cached address assumes the device's primary context is never reset
// (cudaDeviceReset) while the library is loaded: a new context loads the
// module again, possibly at another address.
float* scratch_ptr(int* rc) {
  static float* ptrs[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *rc = FA_ERR_NO_DEVICE;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_bwd_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();  // clear the error so that the next CUDA call does not report it
      if (e == cudaErrorMemoryAllocation) {
        *rc = FA_ERR_OUT_OF_MEMORY;  // the module holding the array could not be loaded
      } else if (e == cudaErrorNoDevice || e == cudaErrorInvalidDevice) {
        *rc = FA_ERR_NO_DEVICE;
      } else {
        fa::record_cuda_error(e == cudaSuccess ? cudaErrorInvalidSymbol : e);
        *rc = FA_ERR_CUDA;
      }
      return nullptr;
    }
    ptrs[dev] = static_cast<float*>(p);
  }
  *rc = FA_OK;
  return ptrs[dev];
}

}  // namespace

extern "C" int fa_bwd_fused_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dO,
                                    const float* lse, void* dq, void* dk, void* dv, int B, int Hq, int Hkv, int Nq,
                                    int Nk, int D, const int64_t* q_strides, const int64_t* k_strides,
                                    const int64_t* v_strides, const int64_t* o_strides, const int64_t* do_strides,
                                    const int64_t* dq_strides, const int64_t* dk_strides,
                                    const int64_t* dv_strides, float softmax_scale, int causal, void* stream) {
  if (D != 32 && D != 64) return FA_ERR_UNSUPPORTED_HEAD_DIM;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Nq <= 0 || Nk <= 0 || Hq % Hkv != 0) return FA_ERR_BAD_SHAPE;
  // Scratch layout: Delta (rows floats, padded to 256 bytes), then the
  // contiguous [B, Hq, Nq, D] fp32 dQ accumulator.
  const unsigned long long rows = (unsigned long long)B * Hq * Nq;
  const unsigned long long delta_floats = (rows + 63) / 64 * 64;
  const unsigned long long need = delta_floats + rows * (unsigned long long)D;
  if (need > kScratchFloats) return FA_ERR_SCRATCH_LIMIT;
  int rc = FA_OK;
  float* scratch = scratch_ptr(&rc);
  if (!scratch) return rc;
  float* delta = scratch;
  float* dq_accum = scratch + delta_floats;
  if ((rc = fa_bwd_preprocess(o, dO, delta, dq_accum, B, Hq, Nq, D, o_strides, do_strides, stream))) return rc;
  if ((rc = fa_bwd_fused(q, k, v, dO, lse, delta, dq_accum, dk, dv, B, Hq, Hkv, Nq, Nk, D, q_strides, k_strides,
                         v_strides, do_strides, dk_strides, dv_strides, softmax_scale, causal, 0, 0, 0, stream)))
    return rc;
  return fa_bwd_dq_convert(dq_accum, dq, B, Hq, Nq, D, dq_strides, stream);
}
