// Shared device helpers for the fdl_b200 library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/fdl_kvcache.h"

namespace fdl {

constexpr int kNumSMs = 148;  // B200: 2 dies x 74 SMs (queried at run time too)

// First device-side error (code, info) per device.  Written with atomicCAS so
// the first event wins; read and cleared by fdl_last_device_error().
__device__ int g_dev_status = 0;
__device__ long long g_dev_info = 0;

__device__ __forceinline__ void report(int code, long long info) {
  if (atomicCAS(&g_dev_status, 0, code) == 0) {
    atomicExch(reinterpret_cast<unsigned long long*>(&g_dev_info),
               static_cast<unsigned long long>(info));
  }
}

// Unsigned 32-bit division by a run-time constant via a 64-bit magic multiply
// (round-up method, exact for all n < 2^31 when d < 2^31).
struct FastDiv {
  uint32_t d;
  uint64_t m;
  __host__ void init(uint32_t div) {
    d = div;
    m = div ? (~0ull / div + 1) : 0;  // ceil(2^64 / d)
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    return d == 1 ? n : static_cast<uint32_t>(__umul64hi(m, n));
  }
  __device__ __forceinline__ void divmod(uint32_t n, uint32_t& q, uint32_t& r) const {
    q = div(n);
    r = n - q * d;
  }
};

template <int VEC>
struct VecT;
template <> struct VecT<16> { using T = uint4; };
template <> struct VecT<8> { using T = uint2; };
template <> struct VecT<4> { using T = uint32_t; };
template <> struct VecT<2> { using T = uint16_t; };

template <int VEC>
__device__ __forceinline__ typename VecT<VEC>::T ld_vec(const char* p) {
  return *reinterpret_cast<const typename VecT<VEC>::T*>(p);
}
template <int VEC>
__device__ __forceinline__ void st_vec(char* p, typename VecT<VEC>::T v) {
  *reinterpret_cast<typename VecT<VEC>::T*>(p) = v;
}
// Read-once stream: bypass L1 allocation, keep normal L2 policy.
__device__ __forceinline__ uint4 ld_stream16(const char* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// Write-once stream: evict-first in L2.
__device__ __forceinline__ void st_stream16(char* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Largest power-of-two vector width (bytes, <= 16) dividing every value.
inline int pick_vec(std::initializer_list<uint64_t> vals) {
  int v = 16;
  for (uint64_t x : vals) {
    while (v > 1 && (x % v) != 0) v >>= 1;
  }
  return v;
}

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FDL_OK : -static_cast<int>(e);
}

inline int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = kNumSMs;
  }
  return n;
}

}  // namespace fdl
