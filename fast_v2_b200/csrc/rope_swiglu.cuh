// Elementwise stages of the decode forward that sit next to the KV-cache
// path, fused into single HBM passes:
//   rope_qkv_kernel  split of the fused q/k/v projection output + rotary
//                    embedding of q and k (apply_rotary_pos_emb,
//                    modeling.py:186-199) with the reference's bf16 rounding
//                    after each multiply and after the add; cos/sin are
//                    computed once per token (fp32 angle = pos * inv_freq,
//                    rounded to bf16 like Fast_dLLM_QwenRotaryEmbedding,
//                    modeling.py:545-560) and shared by every head.
//   swiglu_kernel    act = round(round(silu(gate)) * up) over the fused
//                    gate/up projection output (Fast_dLLM_QwenMLP.forward,
//                    modeling.py:163-165).
#pragma once
#include "common.cuh"

namespace fdl {

constexpr int kRopeThreads = 256;
constexpr int kRopeMaxHalf = 128;  // head_dim <= 256

struct RopeArgs {
  const __nv_bfloat16* y;  // [rows, (hq + 2 hkv) * D]
  int64_t y_rs;            // row stride (elements)
  const int64_t* pos;      // [rows]
  const float* inv_freq;   // [D / 2]
  __nv_bfloat16* q;        // [rows, hq, D]
  __nv_bfloat16* k;        // [rows, hkv, D]
  __nv_bfloat16* v;        // [rows, hkv, D]
  int rows, hq, hkv, D;
};

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__global__ void __launch_bounds__(kRopeThreads) rope_qkv_kernel(const __grid_constant__ RopeArgs a) {
  __shared__ float s_cos[kRopeMaxHalf], s_sin[kRopeMaxHalf];
  const int row = blockIdx.x;
  const int half = a.D / 2;
  const float p = static_cast<float>(a.pos[row]);
  for (int j = threadIdx.x; j < half; j += kRopeThreads) {
    float sn, cs;
    sincosf(__fmul_rn(p, a.inv_freq[j]), &sn, &cs);
    s_cos[j] = bf16r(cs);
    s_sin[j] = bf16r(sn);
  }
  __syncthreads();
  const __nv_bfloat16* yr = a.y + static_cast<int64_t>(row) * a.y_rs;
  const int vpr = half / 8;                 // 8-element vectors per half row
  const int n_rope = (a.hq + a.hkv) * vpr;  // q and k heads
  const int n_v = a.hkv * (a.D / 8);        // v copy vectors
  for (int w = threadIdx.x; w < n_rope + n_v; w += kRopeThreads) {
    if (w < n_rope) {
      const int hh = w / vpr;
      const int j0 = (w - hh * vpr) * 8;
      const __nv_bfloat16* src = yr + hh * a.D;
      const uint4 u1 = *reinterpret_cast<const uint4*>(src + j0);
      const uint4 u2 = *reinterpret_cast<const uint4*>(src + half + j0);
      const __nv_bfloat16* x1 = reinterpret_cast<const __nv_bfloat16*>(&u1);
      const __nv_bfloat16* x2 = reinterpret_cast<const __nv_bfloat16*>(&u2);
      uint4 o1, o2;
      __nv_bfloat16* y1 = reinterpret_cast<__nv_bfloat16*>(&o1);
      __nv_bfloat16* y2 = reinterpret_cast<__nv_bfloat16*>(&o2);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float c = s_cos[j0 + e], s = s_sin[j0 + e];
        const float a1 = __bfloat162float(x1[e]), a2 = __bfloat162float(x2[e]);
        // x * cos + rotate_half(x) * sin, rotate_half = cat(-x2, x1)
        y1[e] = __float2bfloat16_rn(__fadd_rn(bf16r(__fmul_rn(a1, c)), bf16r(__fmul_rn(-a2, s))));
        y2[e] = __float2bfloat16_rn(__fadd_rn(bf16r(__fmul_rn(a2, c)), bf16r(__fmul_rn(a1, s))));
      }
      __nv_bfloat16* dst = hh < a.hq ? a.q + (static_cast<int64_t>(row) * a.hq + hh) * a.D
                                     : a.k + (static_cast<int64_t>(row) * a.hkv + (hh - a.hq)) * a.D;
      *reinterpret_cast<uint4*>(dst + j0) = o1;
      *reinterpret_cast<uint4*>(dst + half + j0) = o2;
    } else {
      const int vi = w - n_rope;
      const int hv = vi / (a.D / 8);
      const int d0 = (vi - hv * (a.D / 8)) * 8;
      const uint4 u = *reinterpret_cast<const uint4*>(yr + (a.hq + a.hkv + hv) * a.D + d0);
      *reinterpret_cast<uint4*>(a.v + (static_cast<int64_t>(row) * a.hkv + hv) * a.D + d0) = u;
    }
  }
}

constexpr int kSwigluThreads = 256;

struct SwigluArgs {
  const __nv_bfloat16* gu;  // [rows, 2F]: gate then up
  int64_t gu_rs;
  __nv_bfloat16* out;       // [rows, F]
  int64_t out_rs;
  int64_t rows;
  int F;
};

__global__ void __launch_bounds__(kSwigluThreads) swiglu_kernel(const __grid_constant__ SwigluArgs a) {
  const int vpr = a.F / 8;
  const int64_t total = a.rows * vpr;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kSwigluThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kSwigluThreads) {
    const int64_t r = i / vpr;
    const int c = static_cast<int>(i - r * vpr) * 8;
    const __nv_bfloat16* row = a.gu + r * a.gu_rs;
    const uint4 ug = ld_stream16(reinterpret_cast<const char*>(row + c));
    const uint4 uu = ld_stream16(reinterpret_cast<const char*>(row + a.F + c));
    const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(&ug);
    const __nv_bfloat16* u = reinterpret_cast<const __nv_bfloat16*>(&uu);
    uint4 o;
    __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float x = __bfloat162float(g[e]);
      const float s = bf16r(__fdiv_rn(x, __fadd_rn(1.f, expf(-x))));
      y[e] = __float2bfloat16_rn(__fmul_rn(s, __bfloat162float(u[e])));
    }
    *reinterpret_cast<uint4*>(a.out + r * a.out_rs + c) = o;
  }
}

}  // namespace fdl
