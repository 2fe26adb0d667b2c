// Shared device helpers of the cast_b200 library (one translation unit: capi.cu).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/cast_b200.h"

namespace cast {

// Per-device error word: kernels that meet inconsistent metadata skip the unit
// and record the first positive CAST_DEV_* code here (cast_device_error reads it).
__device__ int g_dev_error;

__device__ __forceinline__ void report(int code) { atomicCAS(&g_dev_error, 0, code); }

constexpr float kLog2e = 1.4426950408889634f;

template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};

// Load 4 consecutive elements (16-byte aligned for float, 8-byte for 16-bit types) as float4.
template <typename T> __device__ __forceinline__ float4 load4(const T* p);
template <> __device__ __forceinline__ float4 load4<float>(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
template <> __device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&u.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&u.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}
template <> __device__ __forceinline__ float4 load4<__half>(const __half* p) {
  uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  __half2 a = *reinterpret_cast<__half2*>(&u.x);
  __half2 b = *reinterpret_cast<__half2*>(&u.y);
  float2 fa = __half22float2(a), fb = __half22float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

template <typename T> __device__ __forceinline__ void store4(T* p, float4 v);
template <> __device__ __forceinline__ void store4<float>(float* p, float4 v) {
  *reinterpret_cast<float4*>(p) = v;
}
template <> __device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}
template <> __device__ __forceinline__ void store4<__half>(__half* p, float4 v) {
  __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

// Metadata of one sequence, validated against the buffer sizes the host gave.
struct SeqMeta {
  int q0, kv0, S, P;
  bool ok;
};

__device__ __forceinline__ SeqMeta load_seq(const int32_t* cu_q, const int32_t* cu_kv,
                                            const int32_t* prefix_len, const int32_t* pack_len,
                                            int b, int total_q, int total_kv, int max_pack,
                                            int max_kv) {
  SeqMeta m;
  m.q0 = cu_q[b];
  m.kv0 = cu_kv[b];
  m.S = prefix_len[b];
  m.P = pack_len[b];
  m.ok = m.q0 >= 0 && m.kv0 >= 0 && m.S >= 0 && m.P >= 0 && m.P <= max_pack &&
         (long long)m.S + m.P <= (long long)max_kv && (long long)m.q0 + m.P <= total_q &&
         (long long)m.kv0 + m.S + m.P <= (long long)total_kv;
  return m;
}

}  // namespace cast
