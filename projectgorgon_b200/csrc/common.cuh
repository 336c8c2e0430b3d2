// Shared helpers for the tree-verification kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <string>

#include "gorgon_b200.h"

namespace gorgon {

// Device-side error bits (reported by gorgon_device_error).
constexpr uint32_t kErrBadParent = 1u << 0;
constexpr uint32_t kErrBadTrimIndex = 1u << 1;
constexpr uint32_t kErrBadVerifyInput = 1u << 2;
constexpr uint32_t kErrBadSeqlen = 1u << 3;      // a sequence shorter than its tree
constexpr uint32_t kErrTimeout = 1u << 4;        // a bounded wait of a tensor-core kernel ran out
constexpr uint32_t kErrCandCapacity = 1u << 5;   // a candidate tree was cut at max_nodes

// Sets the calling thread's last-error message and returns `code`.
int set_error(int code, const std::string& msg);
// Wraps a CUDA runtime result; returns GORGON_OK or GORGON_ERR_CUDA with message.
int check_cuda(cudaError_t e, const char* what);
// Device address of the library's error word on the current device.
uint32_t* device_error_word();
// Number of SMs of the current device (cached per device).
int sm_count();
// Bound, in nanoseconds, on every wait inside the tensor-core kernels
// (2 s unless changed through gorgon_set_wait_limit_ns).
uint64_t wait_limit_ns();

__device__ __forceinline__ void raise_device_error(uint32_t* word, uint32_t bit) {
  if (word) atomicOr(word, bit);
}

template <typename T> struct Cvt;
template <> struct Cvt<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Cvt<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};

// Stores float x into out[idx] as dtype `dt` (runtime-selected output type).
__device__ __forceinline__ void store_as(void* out, int dt, int64_t idx, float x) {
  if (dt == GORGON_F32) {
    static_cast<float*>(out)[idx] = x;
  } else if (dt == GORGON_BF16) {
    static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(x);
  } else {
    static_cast<__half*>(out)[idx] = __float2half_rn(x);
  }
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline size_t dtype_bytes(int dt) { return dt == GORGON_F32 ? 4 : 2; }
inline bool dtype_ok(int dt) { return dt == GORGON_F32 || dt == GORGON_BF16 || dt == GORGON_F16; }

}  // namespace gorgon
