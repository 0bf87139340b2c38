// (b) Token-sparse prefix selection: per-token key-norm score, exact top-k by
// 4-pass 8-bit radix select on the fp32 bit patterns (scores are >= 0, so
// unsigned order == float order), lower index wins ties, indices emitted in
// ascending order by a block-wide scan.  The selected rows are then moved by
// kv_gather_rows_kernel.
#pragma once
#include "common.cuh"

namespace fdl {

constexpr int kScoreThreads = 256;  // 8 rows per CTA
constexpr int kSelectThreads = 1024;

struct ScoreArgs {
  const char* k;
  const int32_t* len;
  float* score;  // [B, cap]
  int cap, elems;  // elems = H * D (bf16), multiple of 8
  int64_t sb, ss;  // bytes
};

// score[b, t] = sqrt(sum of squares of the H*D key elements of token t).
// Lane l accumulates the 8-element vectors l, l+32, l+64, ... in order with
// fp32 FMA, then the 32 lane sums are combined by an xor butterfly
// (offsets 16, 8, 4, 2, 1).  The CPU oracle restates exactly this order.
__global__ void __launch_bounds__(kScoreThreads) key_score_kernel(const __grid_constant__ ScoreArgs a) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (kScoreThreads / 32) + (threadIdx.x >> 5);
  const int b = blockIdx.y;
  int len = a.len[b];
  len = len < 0 ? 0 : (len > a.cap ? a.cap : len);
  if (t >= len) return;
  const char* row = a.k + b * a.sb + t * a.ss;
  const int nvec = a.elems / 8;
  float acc = 0.f;
  for (int vi = lane; vi < nvec; vi += 32) {
    const uint4 u = ld_stream16(row + vi * 16);
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float f = __bfloat162float(e[j]);
      acc = __fmaf_rn(f, f, acc);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  if (lane == 0) a.score[static_cast<int64_t>(b) * a.cap + t] = __fsqrt_rn(acc);
}

struct SelectArgs {
  const float* score;
  const int32_t* len;
  int32_t* sel;      // [B, max_keep]
  int32_t* out_len;  // [B]
  int cap, keep_num, keep_den, max_keep;
};

// Exclusive block scan of one int per thread (kSelectThreads threads).
__device__ __forceinline__ int block_excl_scan(int v, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = s_warp[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += y;
    }
    s_warp[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  total = s_warp[31];
  const int warp_base = warp ? s_warp[warp - 1] : 0;
  __syncthreads();
  return warp_base + x - v;
}

__global__ void __launch_bounds__(kSelectThreads) topk_select_kernel(const __grid_constant__ SelectArgs a) {
  __shared__ int s_hist[256];
  __shared__ int s_warp[32];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining;
  const int b = blockIdx.x;
  int len = a.len[b];
  if (len < 0 || len > a.cap) {
    if (threadIdx.x == 0) report(FDL_DEV_LENGTH, len);
    len = len < 0 ? 0 : a.cap;
  }
  int keep = static_cast<int>((static_cast<int64_t>(len) * a.keep_num + a.keep_den - 1) / a.keep_den);
  if (keep > len) keep = len;
  if (keep > a.max_keep) {
    if (threadIdx.x == 0) report(FDL_DEV_LENGTH, keep);
    keep = a.max_keep;
  }
  const uint32_t* key = reinterpret_cast<const uint32_t*>(a.score + static_cast<int64_t>(b) * a.cap);
  int32_t* sel = a.sel + static_cast<int64_t>(b) * a.max_keep;

  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_remaining = keep;
  }
  __syncthreads();
  uint32_t mask = 0;
  if (keep > 0) {
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int i = threadIdx.x; i < 256; i += kSelectThreads) s_hist[i] = 0;
      __syncthreads();
      const uint32_t prefix = s_prefix;
      for (int t = threadIdx.x; t < len; t += kSelectThreads) {
        const uint32_t kv = key[t];
        if ((kv & mask) == prefix) atomicAdd(&s_hist[(kv >> shift) & 255u], 1);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int rem = s_remaining, cum = 0, d = 255;
        for (; d > 0; --d) {
          if (cum + s_hist[d] >= rem) break;
          cum += s_hist[d];
        }
        s_remaining = rem - cum;
        s_prefix = prefix | (static_cast<uint32_t>(d) << shift);
      }
      mask |= 255u << shift;
      __syncthreads();
    }
  }
  const uint32_t thr = s_prefix;
  const int take_eq = s_remaining;  // how many keys equal to thr are kept
  // Contiguous chunk per thread keeps the scans in index order.
  const int chunk = (len + kSelectThreads - 1) / kSelectThreads;
  const int t0 = threadIdx.x * chunk;
  const int t1 = min(len, t0 + chunk);
  int n_eq = 0;
  if (keep > 0)
    for (int t = t0; t < t1; ++t) n_eq += (key[t] == thr);
  int tot;
  int eq_rank = block_excl_scan(n_eq, s_warp, tot);
  int n_sel = 0;
  if (keep > 0) {
    int r = eq_rank;
    for (int t = t0; t < t1; ++t) {
      const uint32_t kv = key[t];
      if (kv > thr) ++n_sel;
      else if (kv == thr) { n_sel += (r < take_eq); ++r; }
    }
  }
  int pos = block_excl_scan(n_sel, s_warp, tot);
  if (keep > 0) {
    int r = eq_rank;
    for (int t = t0; t < t1; ++t) {
      const uint32_t kv = key[t];
      bool take = false;
      if (kv > thr) take = true;
      else if (kv == thr) { take = (r < take_eq); ++r; }
      if (take) sel[pos++] = t;
    }
  }
  for (int i = keep + threadIdx.x; i < a.max_keep; i += kSelectThreads) sel[i] = -1;
  if (threadIdx.x == 0) a.out_len[b] = keep;
}

}  // namespace fdl
