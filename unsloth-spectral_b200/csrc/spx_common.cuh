// Shared helpers for the spx kernels: dtype conversion, host-side status handling.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include "spx.h"

namespace spx {

// ---------------------------------------------------------------- host status ----
void set_error(const char* fmt, ...);

#define SPX_REQUIRE(cond, status, ...)   \
  do {                                   \
    if (!(cond)) {                       \
      ::spx::set_error(__VA_ARGS__);     \
      return (status);                   \
    }                                    \
  } while (0)

// Check the launch that was just enqueued.
inline int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return SPX_ERR_CUDA;
  }
  return SPX_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int dtype_size(int dt) { return dt == SPX_F32 ? 4 : 2; }
inline bool dtype_ok(int dt) { return dt == SPX_F32 || dt == SPX_F16 || dt == SPX_BF16; }

// ----------------------------------------------------------- device conversion ----
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Byte offset of the value code (rank r, token t) inside one block stored in the
// value-tile layout: 16-token tiles, each an [R][16] byte matrix whose row index is XORed
// with (tile & 7) and whose 16 tokens are stored in the order 0,1,8,9,2,3,10,11,4,5,12,13,
// 6,7,14,15.  R must be a multiple of 8 and the block length a multiple of 16.
__host__ __device__ __forceinline__ int vtile_offset(int r, int t, int R) {
  const int tt = t >> 4, x = t & 15;
  const int pos = 4 * ((x & 7) >> 1) + (x & 1) + 2 * (x >> 3);
  return (tt * R + (r ^ (tt & 7))) * 16 + pos;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace spx

// Run `body` with `T` bound to the C++ type of spx dtype `dt`.
#define SPX_DISPATCH_DTYPE(dt, T, ...)         \
  [&]() -> int {                               \
    switch (dt) {                              \
      case SPX_F32: {                          \
        using T = float;                       \
        return __VA_ARGS__();                  \
      }                                        \
      case SPX_F16: {                          \
        using T = __half;                      \
        return __VA_ARGS__();                  \
      }                                        \
      case SPX_BF16: {                         \
        using T = __nv_bfloat16;               \
        return __VA_ARGS__();                  \
      }                                        \
      default:                                 \
        ::spx::set_error("bad dtype %d", (int)(dt)); \
        return (int)SPX_ERR_UNSUPPORTED;       \
    }                                          \
  }()
