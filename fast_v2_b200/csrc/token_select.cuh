// Token selection that feeds the sparse gathers: which block tokens a sparse
// or FOCUS step recomputes.  One block of S <= 32 tokens per sequence, so a
// warp holds a whole row with lane = position; the selections are index work
// and must equal the CPU restatement bit for bit, so every float reduction
// runs in a fixed order (per-lane accumulation in element order, then an
// xor-shuffle butterfly) and every rounding point of the reference's bf16
// torch ops is reproduced.  Equal values rank by position, lower index first
// (torch.topk leaves that order open).
//   cosine_select_kernel     cosine similarity of each token's layer input
//                            with the cached one, the n least similar tokens
//                            in ascending order, and (optionally) the cache
//                            refreshed with the new input -- the sparse
//                            forward's selection, modeling.py:868-877.
//   focus_select_kernel      _focus_select, modeling.py:240-306.
//   focus_importance_kernel  _focus_importance, modeling.py:214-237, with the
//                            GQA head mapping done in the kernel instead of
//                            repeat_kv (floating point; checked with a
//                            tolerance).
#pragma once
#include "common.cuh"

namespace fdl {

constexpr int kSelMaxSeq = 32;
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float rmode(float x, bool bf) { return bf ? round_bf16(x) : x; }

__device__ __forceinline__ float butterfly_sum(float v) {
#pragma unroll
  for (int off = 16; off; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(kFull, v, off));
  return v;
}

// Rank of this lane's value among lanes [0, S): how many rank before it
// (greater -- or smaller when !largest -- or equal at a lower position).
__device__ __forceinline__ int warp_rank(float v, int lane, int S, bool largest) {
  int r = 0;
  for (int j = 0; j < S; ++j) {
    const float w = __shfl_sync(kFull, v, j);
    const bool better = largest ? (w > v) : (w < v);
    r += (better || (w == v && j < lane)) ? 1 : 0;
  }
  return r;
}

// Writes the selected lanes' positions in ascending order to out[0 .. popc),
// and -1 to out[popc .. fill).
__device__ __forceinline__ void emit_sorted(bool selected, int lane, int fill, int64_t* out) {
  const unsigned bits = __ballot_sync(kFull, selected);
  const int n = __popc(bits);
  if (selected) out[__popc(bits & ((1u << lane) - 1u))] = lane;
  if (lane >= n && lane < fill) out[lane] = -1;
}

// 16 bytes as 8 bf16 or 4 fp32 values.
__device__ __forceinline__ void cvt_chunk(const uint4& u, bool bf, float (&v)[8]) {
  if (bf) {
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = __bfloat162float(h[e]);
  } else {
    v[0] = __uint_as_float(u.x);
    v[1] = __uint_as_float(u.y);
    v[2] = __uint_as_float(u.z);
    v[3] = __uint_as_float(u.w);
  }
}

__device__ __forceinline__ void load_chunk(const char* p, bool bf, float (&v)[8]) {
  cvt_chunk(*reinterpret_cast<const uint4*>(p), bf, v);
}

// ------------------------------------------------------ cosine selection --
struct CosSelectArgs {
  const char* hidden;  // [B, S, H]
  const char* cached;  // [B, S, H]
  char* cache_out;     // [B, S, H] or null; may alias cached
  int64_t h_sb, h_ss, c_sb, c_ss, o_sb, o_ss;  // bytes
  int S, H, n_sel, bf;
  int64_t* idx;  // [B, n_sel], row stride idx_sb (elements)
  int64_t idx_sb;
  float* cos_out;  // [B, S] or null
};

constexpr int kCosThreads = 256;

template <bool BF>
__global__ void __launch_bounds__(kCosThreads) cosine_select_kernel(const __grid_constant__ CosSelectArgs a) {
  constexpr int VEC = BF ? 8 : 4;  // elements per 16-byte chunk
  __shared__ float s_cos[kSelMaxSeq];
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_chunk = a.H / VEC;
  const float eps = rmode(1e-8f, BF);
  for (int s = warp; s < a.S; s += kCosThreads / 32) {
    const char* x = a.hidden + b * a.h_sb + s * a.h_ss;
    const char* y = a.cached + b * a.c_sb + s * a.c_ss;
    float sx = 0.f, sy = 0.f;
    for (int c = lane; c < n_chunk; c += 32) {
      float xv[8], yv[8];
      load_chunk(x + static_cast<int64_t>(c) * 16, BF, xv);
      load_chunk(y + static_cast<int64_t>(c) * 16, BF, yv);
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        sx = __fadd_rn(sx, __fmul_rn(xv[e], xv[e]));
        sy = __fadd_rn(sy, __fmul_rn(yv[e], yv[e]));
      }
    }
    const float n1 = fmaxf(rmode(__fsqrt_rn(butterfly_sum(sx)), BF), eps);
    const float n2 = fmaxf(rmode(__fsqrt_rn(butterfly_sum(sy)), BF), eps);
    char* o = a.cache_out ? a.cache_out + b * a.o_sb + s * a.o_ss : nullptr;
    float acc = 0.f;
    for (int c = lane; c < n_chunk; c += 32) {
      const int64_t off = static_cast<int64_t>(c) * 16;
      const uint4 xu = *reinterpret_cast<const uint4*>(x + off);
      float xv[8], yv[8];
      cvt_chunk(xu, BF, xv);
      load_chunk(y + off, BF, yv);
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float p = rmode(__fmul_rn(rmode(__fdiv_rn(xv[e], n1), BF), rmode(__fdiv_rn(yv[e], n2), BF)), BF);
        acc = __fadd_rn(acc, p);
      }
      // This lane has read the cached chunk for the last time: refresh it.
      if (o) *reinterpret_cast<uint4*>(o + off) = xu;
    }
    const float cs = rmode(butterfly_sum(acc), BF);
    if (lane == 0) {
      s_cos[s] = cs;
      if (a.cos_out) a.cos_out[static_cast<int64_t>(b) * a.S + s] = cs;
    }
  }
  __syncthreads();
  if (warp == 0) {
    const float v = lane < a.S ? s_cos[lane] : 0.f;
    const int r = warp_rank(v, lane, a.S, false);
    emit_sorted(lane < a.S && r < a.n_sel, lane, 0, a.idx + b * a.idx_sb);
  }
}

// -------------------------------------------------------- FOCUS selection --
struct FocusSelectArgs {
  const char* delta;  // [B, S] bf16 or f32, row stride d_sb bytes
  int64_t d_sb;
  const uint8_t* mask;    // [B, S] bool, row stride m_sb
  int64_t m_sb;
  const uint8_t* frozen;  // [B, S] bool or null, row stride f_sb
  int64_t f_sb;
  int B, S, K, bf;
  int64_t* sel;  // [B, S] row stride sel_sb: ascending positions, then -1
  int64_t sel_sb;
  int32_t* ksel;  // [1]
};

constexpr int kFocusSelThreads = 1024;
constexpr int kFocusSelMaxRows = 4096;

__global__ void __launch_bounds__(kFocusSelThreads) focus_select_kernel(const __grid_constant__ FocusSelectArgs a) {
  __shared__ unsigned s_retain[kFocusSelMaxRows];
  __shared__ int s_max_retain, s_max_free;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool bf = a.bf != 0;
  const float neg = __uint_as_float(bf ? 0xff7f0000u : 0xff7fffffu);  // torch.finfo(dtype).min
  if (threadIdx.x == 0) {
    s_max_retain = 0;
    s_max_free = 0;
  }
  __syncthreads();
  const bool active = lane < a.S;
  for (int b = warp; b < a.B; b += kFocusSelThreads / 32) {
    const char* dp = a.delta + b * a.d_sb;
    const float d = !active ? 0.f
                    : bf    ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(dp)[lane])
                            : reinterpret_cast<const float*>(dp)[lane];
    const bool valid = active && a.mask[b * a.m_sb + lane] != 0;
    const bool frz = active && a.frozen && a.frozen[b * a.f_sb + lane] != 0;
    const float cnt = static_cast<float>(max(__popc(__ballot_sync(kFull, valid)), 1));
    const float mean = rmode(__fdiv_rn(rmode(butterfly_sum(valid ? d : 0.f), bf), cnt), bf);
    const float dev = rmode(__fsub_rn(d, mean), bf);
    const float sq = rmode(__fmul_rn(dev, dev), bf);
    const float var = rmode(__fdiv_rn(rmode(butterfly_sum(valid ? sq : 0.f), bf), cnt), bf);
    const float thr = rmode(__fadd_rn(mean, rmode(__fsqrt_rn(var), bf)), bf);
    const bool cand = valid && d >= thr;
    const unsigned cbits = __ballot_sync(kFull, cand);
    const bool adj = lane + 1 < a.S && ((cbits >> (lane + 1)) & 1u);
    const bool mustkeep = (cand || adj) && valid;
    const int rk = warp_rank(valid ? d : neg, lane, a.S, true);
    const bool topk = valid && rk < a.K;
    bool retain = active && (!valid || mustkeep || topk);
    if (a.frozen) retain = retain && !frz;
    const unsigned rbits = __ballot_sync(kFull, retain);
    const int n_free = __popc(__ballot_sync(kFull, active && !frz));
    if (lane == 0) {
      s_retain[b] = rbits;
      atomicMax(&s_max_retain, __popc(rbits));
      atomicMax(&s_max_free, n_free);
    }
  }
  __syncthreads();
  int ksel = min(max(s_max_retain, a.K), a.S);
  if (a.frozen) ksel = max(1, min(ksel, s_max_free));
  if (threadIdx.x == 0) *a.ksel = ksel;
  for (int b = warp; b < a.B; b += kFocusSelThreads / 32) {
    const char* dp = a.delta + b * a.d_sb;
    const float d = !active ? 0.f
                    : bf    ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(dp)[lane])
                            : reinterpret_cast<const float*>(dp)[lane];
    const bool retain = (s_retain[b] >> lane) & 1u;
    const bool frz = active && a.frozen && a.frozen[b * a.f_sb + lane] != 0;
    float prio = retain ? rmode(__fadd_rn(d, 1e4f), bf) : d;
    if (frz) prio = neg;
    const int rk = warp_rank(prio, lane, a.S, true);
    emit_sorted(active && rk < ksel, lane, a.S, a.sel + b * a.sel_sb);
  }
}

// ------------------------------------------------------- FOCUS importance --
struct FocusImportanceArgs {
  const char* q;  // [B, Hq, S, D] by strides (bytes)
  int64_t q_sb, q_sh, q_ss;
  const char* k;  // [B, Hkv, S, D]
  int64_t k_sb, k_sh, k_ss;
  const uint8_t* mask;  // [B, S] bool
  int64_t m_sb;
  int S, Hq, Hkv, D, bf;
  float scale;
  char* imp;  // [B, S] bf16 or f32
  int64_t imp_sb;  // bytes
};

constexpr int kImpThreads = 256;
constexpr int kImpMaxHeads = 128;
constexpr int kImpMaxDim = 128;

template <bool BF>
__global__ void __launch_bounds__(kImpThreads) focus_importance_kernel(const __grid_constant__ FocusImportanceArgs a) {
  constexpr int VEC = BF ? 8 : 4;
  __shared__ float s_k[kSelMaxSeq * kImpMaxDim];   // one KV head's keys, fp32
  __shared__ float s_col[kImpMaxHeads][kSelMaxSeq];  // per-head column sums
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr bool bf = BF;
  const int rep = a.Hq / a.Hkv;
  const bool active = lane < a.S;
  const bool qmask = active && a.mask[b * a.m_sb + lane] != 0;
  const unsigned kbits = __ballot_sync(kFull, qmask);  // key mask == query mask (same mask_idx)
  const float ninf = -__int_as_float(0x7f800000);
  for (int g = 0; g < a.Hkv; ++g) {
    __syncthreads();  // previous group's keys are no longer read
    for (int t = threadIdx.x; t < a.S * a.D; t += kImpThreads) {
      const int j = t / a.D, d = t - j * a.D;
      const char* kp = a.k + b * a.k_sb + g * a.k_sh + j * a.k_ss;
      s_k[j * a.D + d] = bf ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(kp)[d])
                            : reinterpret_cast<const float*>(kp)[d];
    }
    __syncthreads();
    for (int hr = warp; hr < rep; hr += kImpThreads / 32) {
      const int h = g * rep + hr;
      // lane = query row i: scores s[j] = q_i . k_j
      float s[kSelMaxSeq];
#pragma unroll
      for (int j = 0; j < kSelMaxSeq; ++j) s[j] = 0.f;
      const char* qp = a.q + b * a.q_sb + h * a.q_sh + (active ? lane : 0) * a.q_ss;
      for (int d0 = 0; d0 < a.D; d0 += VEC) {
        float qv[8];
        load_chunk(qp + d0 * (BF ? 2 : 4), BF, qv);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
#pragma unroll
          for (int j = 0; j < kSelMaxSeq; ++j)
            if (j < a.S) s[j] = fmaf(qv[e], s_k[j * a.D + d0 + e], s[j]);
        }
      }
      // round like torch's matmul output, scale, mask keys, max-pool over 3, mask again
      float p[kSelMaxSeq];
#pragma unroll
      for (int j = 0; j < kSelMaxSeq; ++j) {
        const bool kj = j < a.S && ((kbits >> j) & 1u);
        s[j] = kj ? rmode(__fmul_rn(rmode(s[j], bf), a.scale), bf) : ninf;
      }
      float mx = ninf;
#pragma unroll
      for (int j = 0; j < kSelMaxSeq; ++j) {
        const bool kj = j < a.S && ((kbits >> j) & 1u);
        float v = s[j];
        if (j > 0) v = fmaxf(v, s[j - 1]);
        if (j + 1 < kSelMaxSeq && j + 1 < a.S) v = fmaxf(v, s[j + 1]);
        p[j] = kj ? v : ninf;
        mx = fmaxf(mx, p[j]);
      }
      // softmax over keys (all-masked rows give 0, as nan_to_num), times the query mask
      float sum = 0.f;
      if (mx != ninf) {
#pragma unroll
        for (int j = 0; j < kSelMaxSeq; ++j) {
          p[j] = (p[j] == ninf) ? 0.f : expf(p[j] - mx);
          sum += p[j];
        }
      }
#pragma unroll
      for (int j = 0; j < kSelMaxSeq; ++j) {
        const float w = (mx != ninf && qmask) ? rmode(__fdiv_rn(p[j], sum), bf) : 0.f;
        const float col = butterfly_sum(w);  // sum over query rows
        if (lane == j) s_col[h][j] = rmode(col, bf);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < a.S) {
    const int j = threadIdx.x;
    float acc = 0.f;
    for (int h = 0; h < a.Hq; ++h) acc += s_col[h][j];
    const float v = rmode(acc, bf);
    char* out = a.imp + b * a.imp_sb;
    if (bf)
      reinterpret_cast<__nv_bfloat16*>(out)[j] = __float2bfloat16_rn(v);
    else
      reinterpret_cast<float*>(out)[j] = v;
  }
}

}  // namespace fdl
