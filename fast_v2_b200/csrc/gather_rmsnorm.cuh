// (c) Fused gather + RMSNorm.  One warp per output row: the gathered row is
// loaded once into registers with 16-byte loads (VPL vectors per lane), the
// sum of squares is accumulated in fp32 (per lane, two sequential FMA chains
// over alternating vectors, then an xor-butterfly), and both outputs (the gathered copy and the normalised row)
// are written from registers -- one HBM read and one or two HBM writes per
// element, nothing else.
#pragma once
#include <type_traits>
#include "common.cuh"
#include "sm100_ptx.cuh"

namespace fdl {

constexpr int kNormThreads = 128;  // 4 rows per CTA

struct NormArgs {
  const char* x;
  const char* res;   // optional residual: rows become round(x + res) before the norm
  int64_t res_ss;    // residual row stride (bytes); rows are indexed like the output
  const int64_t* idx;
  int64_t idx_sb;
  const char* w;
  char* gathered;
  char* normed;
  float eps;
  int B, S, T, H;
  int64_t x_sb, x_ss, o_sb, o_ss;  // bytes
};

template <typename T> struct ElemOps;
template <> struct ElemOps<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct ElemOps<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct ElemOps<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};

// Normalise one element.  16-bit inputs follow Fast_dLLM_QwenRMSNorm.forward:
// round(x * inv) to the input dtype, then round(w * that).  fp32 inputs follow
// select_gather_rmsnorm_kernel: x * inv * w in fp32.
template <typename T>
__device__ __forceinline__ T norm_elem(float x, float inv, const T* w, int i) {
  if constexpr (sizeof(T) == 4) {
    float n = __fmul_rn(x, inv);
    if (w) n = __fmul_rn(n, ElemOps<T>::to_f(w[i]));
    return ElemOps<T>::from_f(n);
  } else {
    T n = ElemOps<T>::from_f(__fmul_rn(x, inv));
    if (w) n = ElemOps<T>::from_f(__fmul_rn(ElemOps<T>::to_f(w[i]), ElemOps<T>::to_f(n)));
    return n;
  }
}

template <typename T, int VPL>
__global__ void __launch_bounds__(kNormThreads) gather_rmsnorm_kernel(const __grid_constant__ NormArgs a) {
  constexpr int EPV = 16 / sizeof(T);  // elements per 16-byte vector
  // The weight row is staged once per CTA in shared memory (the four rows of
  // the CTA share it), so the output phase reads it at shared-memory latency
  // without holding it in registers through the reduction.
  __shared__ uint4 w_s[32 * VPL];
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (kNormThreads / 32) + (threadIdx.x >> 5);
  const int nvec = a.H / EPV;
  bool live = row < a.B * a.T;
  int b = 0, t = 0;
  int64_t src_t = 0;
  if (live) {
    b = row / a.T;
    t = row - b * a.T;
    src_t = a.idx ? a.idx[b * a.idx_sb + t] : t;
    if (src_t < 0 || src_t >= a.S) {
      if (lane == 0) report(FDL_DEV_INDEX, src_t);
      live = false;
    }
  }
  uint4 v[VPL];
  if (live) {
    const char* xr = a.x + b * a.x_sb + src_t * a.x_ss;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int vi = lane + 32 * k;
      if (vi < nvec) v[k] = ld_stream16(xr + vi * 16);
    }
  }
  // Weight staging (every thread of the CTA) is issued only after the row
  // loads, so its L2 latency overlaps them instead of preceding the index
  // load.
  if (a.w)
    for (int i = threadIdx.x; i < nvec; i += kNormThreads) w_s[i] = *reinterpret_cast<const uint4*>(a.w + i * 16);
  float acc = 0.f;
  if (live) {
    if (a.res) {
      // Residual connection (decoder layer `residual + hidden_states`): one
      // rounding to the storage dtype, then the norm of the rounded sum.
      const char* rr = a.res + static_cast<int64_t>(row) * a.res_ss;
#pragma unroll
      for (int k = 0; k < VPL; ++k) {
        const int vi = lane + 32 * k;
        if (vi < nvec) {
          // plain load: the sum may be written back over the residual in place
          const uint4 rv = *reinterpret_cast<const uint4*>(rr + vi * 16);
          if constexpr (std::is_same_v<T, __nv_bfloat16>) {
            // bf16x2 add: the exact sum rounded once, equal to the fp32 sum
            // rounded to bf16 (the fp32 rounding of a sum of two bf16 values
            // never lands on a bf16 midpoint the exact sum is not on).
            __nv_bfloat162* e2 = reinterpret_cast<__nv_bfloat162*>(&v[k]);
            const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rv);
#pragma unroll
            for (int j = 0; j < 4; ++j) e2[j] = __hadd2(e2[j], r2[j]);
          } else {
            T* e = reinterpret_cast<T*>(&v[k]);
            const T* re = reinterpret_cast<const T*>(&rv);
#pragma unroll
            for (int j = 0; j < EPV; ++j)
              e[j] = ElemOps<T>::from_f(__fadd_rn(ElemOps<T>::to_f(e[j]), ElemOps<T>::to_f(re[j])));
          }
        }
      }
    }
    // The gathered copy (or the residual sum) is final now: store it before
    // the reduction so the writes overlap the arithmetic.
    if (a.gathered) {
      char* gr = a.gathered + b * a.o_sb + t * a.o_ss;
#pragma unroll
      for (int k = 0; k < VPL; ++k) {
        const int vi = lane + 32 * k;
        if (vi < nvec) st_stream16(gr + vi * 16, v[k]);
      }
    }
    if constexpr (std::is_same_v<T, __nv_bfloat16>) {
      // Packed: a bf16 pair widens to two floats with two integer ops, and one
      // f32x2 FMA accumulates both; four chains (element parity x vector
      // parity) per lane.
      uint64_t acc2[2] = {0, 0};
#pragma unroll
      for (int k = 0; k < VPL; ++k) {
        const int vi = lane + 32 * k;
        if (vi < nvec) {
          const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[k]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint64_t f2 = ptx::pack2(__uint_as_float(u[j] << 16), __uint_as_float(u[j] & 0xFFFF0000u));
            acc2[k & 1] = ptx::fma2(f2, f2, acc2[k & 1]);
          }
        }
      }
      float a0, a1, a2, a3;
      ptx::unpack2(acc2[0], a0, a1);
      ptx::unpack2(acc2[1], a2, a3);
      acc = __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
    } else {
      // Two independent FMA chains (even / odd vectors of the lane); the
      // generic kernel uses the same order.
      float acc2[2] = {0.f, 0.f};
#pragma unroll
      for (int k = 0; k < VPL; ++k) {
        const int vi = lane + 32 * k;
        if (vi < nvec) {
          const T* e = reinterpret_cast<const T*>(&v[k]);
#pragma unroll
          for (int j = 0; j < EPV; ++j) {
            const float f = ElemOps<T>::to_f(e[j]);
            acc2[k & 1] = __fmaf_rn(f, f, acc2[k & 1]);
          }
        }
      }
      acc = __fadd_rn(acc2[0], acc2[1]);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  const float inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(acc, static_cast<float>(a.H)), a.eps));
  __syncthreads();  // w_s complete
  if (!live) return;

  char* nr = a.normed + b * a.o_sb + t * a.o_ss;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int vi = lane + 32 * k;
    if (vi < nvec) {
      const uint4 wv = a.w ? w_s[vi] : make_uint4(0, 0, 0, 0);
      uint4 o;
      if constexpr (std::is_same_v<T, __nv_bfloat16>) {
        // Per pair: f32x2 multiply by inv, one packed rounding to bf16 (the
        // reference's fp32 product then .to(bf16)), then w * n as a bf16x2
        // multiply -- the exact product rounded once, which is what the
        // reference's bf16 * bf16 (fp32 multiply, exact for 8-bit
        // mantissas, then rounding) gives.
        const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[k]);
        const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wv);
        __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
        const uint64_t inv2 = ptx::pack2(inv, inv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t f2 = ptx::pack2(__uint_as_float(u[j] << 16), __uint_as_float(u[j] & 0xFFFF0000u));
          float n0, n1;
          ptx::unpack2(ptx::mul2(f2, inv2), n0, n1);
          const __nv_bfloat162 n = __floats2bfloat162_rn(n0, n1);
          o2[j] = a.w ? __hmul2(w2[j], n) : n;
        }
      } else {
        const T* e = reinterpret_cast<const T*>(&v[k]);
        const T* we = reinterpret_cast<const T*>(&wv);
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int j = 0; j < EPV; ++j) oe[j] = norm_elem<T>(ElemOps<T>::to_f(e[j]), inv, a.w ? we : nullptr, j);
      }
      st_stream16(nr + vi * 16, o);
    }
  }
}

// Generic path (any H, any alignment): one warp per row, two passes over the
// row, scalar loads.  Same accumulation order per lane (element i goes to lane
// (i / EPV) % 32, sequential within a lane) so results match the vector path.
template <typename T>
__global__ void __launch_bounds__(kNormThreads) gather_rmsnorm_generic_kernel(const __grid_constant__ NormArgs a) {
  constexpr int EPV = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (kNormThreads / 32) + (threadIdx.x >> 5);
  if (row >= a.B * a.T) return;
  const int b = row / a.T;
  const int t = row - b * a.T;
  int64_t src_t = a.idx ? a.idx[b * a.idx_sb + t] : t;
  if (src_t < 0 || src_t >= a.S) {
    if (lane == 0) report(FDL_DEV_INDEX, src_t);
    return;
  }
  const T* xr = reinterpret_cast<const T*>(a.x + b * a.x_sb + src_t * a.x_ss);
  const T* rr = a.res ? reinterpret_cast<const T*>(a.res + static_cast<int64_t>(row) * a.res_ss) : nullptr;
  auto elem = [&](int i) -> T {
    return rr ? ElemOps<T>::from_f(__fadd_rn(ElemOps<T>::to_f(xr[i]), ElemOps<T>::to_f(rr[i]))) : xr[i];
  };
  float acc2[2] = {0.f, 0.f};
  int chunk = 0;
  for (int base = lane * EPV; base < a.H; base += 32 * EPV, ++chunk) {
    for (int j = 0; j < EPV && base + j < a.H; ++j) {
      const float f = ElemOps<T>::to_f(elem(base + j));
      acc2[chunk & 1] = __fmaf_rn(f, f, acc2[chunk & 1]);
    }
  }
  float acc = __fadd_rn(acc2[0], acc2[1]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  const float inv = __frsqrt_rn(__fadd_rn(__fdiv_rn(acc, static_cast<float>(a.H)), a.eps));
  T* gr = a.gathered ? reinterpret_cast<T*>(a.gathered + b * a.o_sb + t * a.o_ss) : nullptr;
  T* nr = reinterpret_cast<T*>(a.normed + b * a.o_sb + t * a.o_ss);
  const T* w = reinterpret_cast<const T*>(a.w);
  for (int i = lane; i < a.H; i += 32) {
    const T xv = elem(i);
    if (gr) gr[i] = xv;
    nr[i] = norm_elem<T>(ElemOps<T>::to_f(xv), inv, w, i);
  }
}

template <typename T>
inline void launch_gather_rmsnorm(const NormArgs& a, bool vec_ok, cudaStream_t s) {
  const int rows = a.B * a.T;
  const dim3 grid((rows + 3) / 4);
  const int nvec = a.H * static_cast<int>(sizeof(T)) / 16;
  if (!vec_ok || nvec > 32 * 32) {
    gather_rmsnorm_generic_kernel<T><<<grid, kNormThreads, 0, s>>>(a);
    return;
  }
  const int vpl = (nvec + 31) / 32;
  if (vpl <= 2) gather_rmsnorm_kernel<T, 2><<<grid, kNormThreads, 0, s>>>(a);
  else if (vpl <= 4) gather_rmsnorm_kernel<T, 4><<<grid, kNormThreads, 0, s>>>(a);
  else if (vpl <= 8) gather_rmsnorm_kernel<T, 8><<<grid, kNormThreads, 0, s>>>(a);
  else if (vpl <= 14) gather_rmsnorm_kernel<T, 14><<<grid, kNormThreads, 0, s>>>(a);
  else if (vpl <= 16) gather_rmsnorm_kernel<T, 16><<<grid, kNormThreads, 0, s>>>(a);
  else if (vpl <= 28) gather_rmsnorm_kernel<T, 28><<<grid, kNormThreads, 0, s>>>(a);
  else gather_rmsnorm_kernel<T, 32><<<grid, kNormThreads, 0, s>>>(a);
}

}  // namespace fdl
