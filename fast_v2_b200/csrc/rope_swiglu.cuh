// Elementwise stages of the decode forward that sit next to the KV-cache
// path, fused into single HBM passes:
//   rope_qkv_kernel  split of the fused q/k/v projection output + rotary
//                    embedding of q and k (apply_rotary_pos_emb,
//                    modeling.py:186-199) with the reference's bf16 rounding
//                    after each multiply and after the add; cos/sin are
//                    computed once per token (fp32 angle = pos * inv_freq,
//                    rounded to bf16 like Fast_dLLM_QwenRotaryEmbedding,
//                    modeling.py:545-560) and shared by every head.
//   rope_qkv_store_kernel  the same split + rotary embedding with K and V
//                    stored straight into their cache rows (append at a
//                    per-sequence start, or scatter at given positions),
//                    so no separate KV write follows the projection.
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

// Row r = b * T + t of y is token t of sequence b.  Its K and V rows go to
// kd / vd + b * d_sb + p * d_ss + head * d_sh (bytes), at position
// p = dpos[b, t] when dpos is set, else (start ? start[b] : 0) + t; a
// position outside [0, d_len) skips that row's K/V and is reported.
struct RopeStoreArgs {
  const __nv_bfloat16* y;  // [rows, (hq + 2 hkv) * D]
  int64_t y_rs;            // row stride (elements)
  const int64_t* pos;      // [rows] rotary positions
  const float* inv_freq;   // [D / 2]
  __nv_bfloat16* q;        // [rows, hq, D]
  char* kd;                // K destination
  char* vd;                // V destination
  int64_t d_sb, d_ss, d_sh;  // bytes
  const int32_t* start;    // [B] or null
  const int64_t* dpos;     // [B, T] (row stride dpos_sb) or null
  int64_t dpos_sb;
  int rows, hq, hkv, D, T, d_len;
};


__global__ void __launch_bounds__(kRopeThreads) rope_qkv_store_kernel(const __grid_constant__ RopeStoreArgs a) {
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
  const int b = row / a.T;
  const int t = row - b * a.T;
  const int64_t p_kv = a.dpos ? a.dpos[b * a.dpos_sb + t] : static_cast<int64_t>(a.start ? a.start[b] : 0) + t;
  const bool store_kv = p_kv >= 0 && p_kv < a.d_len;
  if (!store_kv && threadIdx.x == 0) report(FDL_DEV_INDEX, p_kv);
  char* krow = a.kd + b * a.d_sb + (store_kv ? p_kv : 0) * a.d_ss;
  char* vrow = a.vd + b * a.d_sb + (store_kv ? p_kv : 0) * a.d_ss;
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
      if (hh < a.hq) {
        __nv_bfloat16* dst = a.q + (static_cast<int64_t>(row) * a.hq + hh) * a.D;
        *reinterpret_cast<uint4*>(dst + j0) = o1;
        *reinterpret_cast<uint4*>(dst + half + j0) = o2;
      } else if (store_kv) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(krow + (hh - a.hq) * a.d_sh);
        *reinterpret_cast<uint4*>(dst + j0) = o1;
        *reinterpret_cast<uint4*>(dst + half + j0) = o2;
      }
    } else if (store_kv) {
      const int vi = w - n_rope;
      const int hv = vi / (a.D / 8);
      const int d0 = (vi - hv * (a.D / 8)) * 8;
      const uint4 u = *reinterpret_cast<const uint4*>(yr + (a.hq + a.hkv + hv) * a.D + d0);
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(vrow + hv * a.d_sh) + d0) = u;
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
  uint32_t total;           // rows * F / 8 vectors
  FastDiv vpr;              // F / 8 vectors per row
};

// bf16(silu(x)) exactly as torch computes it for a bf16 tensor: fp32
// x / (1 + exp(-x)) with IEEE division, rounded to bf16.
__device__ __forceinline__ float silu_bf16_exact(float x) { return bf16r(__fdiv_rn(x, __fadd_rn(1.f, expf(-x)))); }

// Same value from the special-function unit: s = x * rcp(1 + 2^(-x log2 e)).
// For every bf16 gate value it rounds to the same bf16 as the IEEE
// expression except for x in (-88.7, -87.3), where 1 + 2^(-x log2 e) is so
// large that its flush-to-zero reciprocal is 0 (gate values -87.5, -88 and
// -88.5 give -0 instead of about -5e-37); inputs below -87 take the exact
// expression.  The kernel only sees bf16 gate values, and the GPU tests check
// all 65536 of them against torch's bf16 silu.  (An earlier guard on the
// result -- within 16 fp32 ulps of a bf16 rounding midpoint, or not normal --
// cost 11% of the kernel time for the same outputs.)
__device__ __forceinline__ float silu_bf16_fast(float x) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * -1.44269504f));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + e));
  return bf16r(x * r);
}
__device__ __forceinline__ float silu_bf16(float x) {
  return x < -87.f ? silu_bf16_exact(x) : silu_bf16_fast(x);
}

// The rows x (F / 8) vectors of the output form one flat range and every
// thread owns one 16-byte vector of it (CTA c covers vectors
// [c * kSwigluThreads, (c + 1) * kSwigluThreads) across row boundaries), so
// every CTA but the last is full (a per-row grid leaves the last chunk of
// every row part-empty: 320 of 1024 vectors at F = 18944).  One vector per
// thread measured fastest on B200 at 2048 x 18944: 41.0 us against 41.7,
// 44.0 and 48.0 us with 2, 3 and 4 vectors per thread (more registers per
// thread, fewer resident warps, a longer tail of the last wave), and
// streaming stores of the output change nothing.
constexpr int kSwigluChunk = kSwigluThreads;  // vectors per CTA

__global__ void __launch_bounds__(kSwigluThreads) swiglu_kernel(const __grid_constant__ SwigluArgs a) {
  const uint32_t i = blockIdx.x * kSwigluChunk + threadIdx.x;
  if (i >= a.total) return;
  uint32_t r, v;
  a.vpr.divmod(i, r, v);
  const __nv_bfloat16* row = a.gu + static_cast<int64_t>(r) * a.gu_rs;
  const uint4 ug = ld_stream16(reinterpret_cast<const char*>(row + v * 8));
  const uint4 uu = ld_stream16(reinterpret_cast<const char*>(row + a.F + v * 8));
  const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(&ug);
  const __nv_bfloat16* u = reinterpret_cast<const __nv_bfloat16*>(&uu);
  uint4 o;
  __nv_bfloat16* y = reinterpret_cast<__nv_bfloat16*>(&o);
  float gf[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) gf[e] = __bfloat162float(g[e]);
  // One test per vector: the exact expression is needed only below -87.
  const float lo = fminf(fminf(fminf(gf[0], gf[1]), fminf(gf[2], gf[3])), fminf(fminf(gf[4], gf[5]), fminf(gf[6], gf[7])));
  if (__builtin_expect(lo < -87.f, 0)) {
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = __float2bfloat16_rn(__fmul_rn(silu_bf16(gf[e]), __bfloat162float(u[e])));
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = __float2bfloat16_rn(__fmul_rn(silu_bf16_fast(gf[e]), __bfloat162float(u[e])));
  }
  *reinterpret_cast<uint4*>(a.out + static_cast<int64_t>(r) * a.out_rs + v * 8) = o;
}

}  // namespace fdl
