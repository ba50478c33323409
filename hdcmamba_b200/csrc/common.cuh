// Shared device/host helpers for the hdcmamba_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/hdcmamba_b200.h"

namespace hdc {

// ---------------------------------------------------------------- error state
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int launch_status(const char* what);  // also counts the launch (hdc_launch_count)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- element types
// Activation storage types: float (HDC_F32) and __nv_bfloat16 (HDC_BF16).
template <typename T> struct Vec;
template <> struct Vec<float> { static constexpr int N = 4; };           // 16 bytes
template <> struct Vec<__nv_bfloat16> { static constexpr int N = 8; };   // 16 bytes

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// fp32 -> bf16 (round to nearest even) -> fp32: the rounding a `.to(tl.bfloat16)`
// store performs in the reference kernels.
__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}
// Value after a store into a `T` buffer.
template <typename T> __device__ __forceinline__ float store_round(float v) {
  return to_f(from_f<T>(v));
}

// 16-byte vector of T converted to / from floats.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& u, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  } else {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x; f[2 * i + 1] = t.y;
    }
  }
}
template <typename T>
__device__ __forceinline__ uint4 pack16(const float* f) {
  uint4 u;
  if constexpr (sizeof(T) == 4) {
    u.x = __float_as_uint(f[0]); u.y = __float_as_uint(f[1]);
    u.z = __float_as_uint(f[2]); u.w = __float_as_uint(f[3]);
  } else {
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  }
  return u;
}

// Streaming 16-byte global accesses.
__device__ __forceinline__ uint4 ldg16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
// ldg16 when `pred`, zeros otherwise, as one predicated load: the caller does not wait
// for the data until it first uses it (a select on the loaded value would).
__device__ __forceinline__ uint4 ldg16_pred(const void* p, bool pred) {
  uint4 r;
  asm volatile(
      "{\n\t.reg .pred q;\n\t"
      "setp.ne.b32 q, %5, 0;\n\t"
      "mov.b32 %0, 0;\n\tmov.b32 %1, 0;\n\tmov.b32 %2, 0;\n\tmov.b32 %3, 0;\n\t"
      "@q ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];\n\t}"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p), "r"((int)pred));
  return r;
}
__device__ __forceinline__ void stg16(void* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};"
               :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Reference softplus with threshold 20 (hdcmamba/model.py:192): log(1 + exp(x)).
__device__ __forceinline__ float softplus20(float x) {
  return x > 20.0f ? x : logf(1.0f + expf(x));
}

// Feature width of the reference's per-head tile: max(64, next_pow2(hd)).
inline int64_t feature_block(int64_t hd) {
  int64_t b = 1;
  while (b < hd) b <<= 1;
  return b < 64 ? 64 : b;
}

// SM count of the current device (cached per device ordinal).
inline int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

}  // namespace hdc
