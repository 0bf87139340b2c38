// Greedy sampling statistics of the block-diffusion sampler, fused over the
// vocabulary row: for logits row r (bf16, V entries)
//   p_max[r] = bf16(exp(0) / s),  s = sum_v exp(l_v - m),  m = max_v l_v
//   token[r] = the first v whose probability bf16(exp(l_v - m) / s) equals p_max
// i.e. sample_with_top_p at temperature 0 (modeling.py:2263-2269: argmax of
// the bf16 softmax, ties to the lower index) and the gathered probability of
// the chosen token (generation_functions.py:2290-2291), without materialising
// the [rows, V] probabilities or running a separate softmax, max and gather.
//
// One CTA per row, two passes over the row:
//   1. per thread an online (max, sum) over its 16-byte vectors (a rescale
//      only when the thread's max grows), merged by a fixed xor-butterfly and
//      a fixed shared-memory tree -- the same sum on every run;
//   2. the row again (L2-resident right after pass 1): only entries within
//      1/64 of m can round to p_max (exp(-1/64) / s is more than a bf16 ulp
//      below 1 / s), and for those the probability is formed exactly as in
//      pass 1's definition; the smallest index that equals p_max wins.
#pragma once
#include "common.cuh"

namespace fdl {

constexpr int kSampleThreads = 512;
constexpr int kSampleWarps = kSampleThreads / 32;
constexpr float kSampleTieWindow = 1.0f / 64.0f;

struct SampleArgs {
  const __nv_bfloat16* logits;  // [rows, V] with row stride rs (elements)
  int64_t rs;
  int V;
  int64_t* token;           // [rows]
  __nv_bfloat16* prob;      // [rows] or null
};

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  if (m2 > m) {
    s = s * expf(m - m2) + s2;
    m = m2;
  } else if (m2 != -INFINITY) {
    s += s2 * expf(m2 - m);
  }
}

__global__ void __launch_bounds__(kSampleThreads) softmax_argmax_kernel(const __grid_constant__ SampleArgs a) {
  __shared__ float sh_m[kSampleWarps], sh_s[kSampleWarps];
  __shared__ float sh_row[2];
  __shared__ int sh_idx;
  const int row = blockIdx.x;
  const __nv_bfloat16* x = a.logits + static_cast<int64_t>(row) * a.rs;
  const int nvec = a.V / 8;  // whole 16-byte vectors; the tail is handled per element
  // ---- pass 1: online max and sum of exp
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < nvec; i += kSampleThreads) {
    const uint4 u = ld_stream16(reinterpret_cast<const char*>(x) + static_cast<int64_t>(i) * 16);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
    float vmax = __bfloat162float(e[0]);
#pragma unroll
    for (int k = 1; k < 8; ++k) vmax = fmaxf(vmax, __bfloat162float(e[k]));
    if (vmax > m) {
      s = (m == -INFINITY) ? 0.f : s * expf(m - vmax);
      m = vmax;
    }
    if (m != -INFINITY) {
#pragma unroll
      for (int k = 0; k < 8; ++k) s += expf(__bfloat162float(e[k]) - m);
    }
  }
  for (int v = nvec * 8 + threadIdx.x; v < a.V; v += kSampleThreads) {
    const float l = __bfloat162float(x[v]);
    if (l > m) {
      s = (m == -INFINITY) ? 0.f : s * expf(m - l);
      m = l;
    }
    if (m != -INFINITY) s += expf(l - m);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, off);
    // Both lanes merge the same pair in the same roles (lower lane first), so
    // every lane ends with the same value.
    const bool lower = (threadIdx.x & off) == 0;
    float ma = lower ? m : m2, sa = lower ? s : s2;
    online_merge(ma, sa, lower ? m2 : m, lower ? s2 : s);
    m = ma;
    s = sa;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sh_m[warp] = m;
    sh_s[warp] = s;
  }
  if (threadIdx.x == 0) sh_idx = 0x7fffffff;
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sh_m[0], S = sh_s[0];
    for (int w = 1; w < kSampleWarps; ++w) online_merge(M, S, sh_m[w], sh_s[w]);
    sh_row[0] = M;
    sh_row[1] = S;
  }
  __syncthreads();
  const float M = sh_row[0], S = sh_row[1];
  const __nv_bfloat16 pmax = __float2bfloat16_rn(expf(0.f) / S);
  // ---- pass 2: first index whose rounded probability equals pmax
  int best = 0x7fffffff;
  const float lo = M - kSampleTieWindow;
  for (int i = threadIdx.x; i < nvec; i += kSampleThreads) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + static_cast<int64_t>(i) * 8);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float l = __bfloat162float(e[k]);
      if (l >= lo && i * 8 + k < best &&
          __bfloat16_as_ushort(__float2bfloat16_rn(expf(l - M) / S)) == __bfloat16_as_ushort(pmax))
        best = i * 8 + k;
    }
  }
  for (int v = nvec * 8 + threadIdx.x; v < a.V; v += kSampleThreads) {
    const float l = __bfloat162float(x[v]);
    if (l >= lo && v < best &&
        __bfloat16_as_ushort(__float2bfloat16_rn(expf(l - M) / S)) == __bfloat16_as_ushort(pmax))
      best = v;
  }
  if (best != 0x7fffffff) atomicMin(&sh_idx, best);
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = sh_idx;
    if (t == 0x7fffffff) {  // no finite logit in the row (all -inf or NaN)
      report(FDL_DEV_INDEX, row);
      t = 0;
    }
    a.token[row] = t;
    if (a.prob) a.prob[row] = pmax;
  }
}

}  // namespace fdl
