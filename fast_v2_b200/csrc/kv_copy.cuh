// (a)/(b) KV-cache data movement: append, scatter, prefix gather (+GQA
// expand, + appended block), index gather.  All are HBM-bound byte copies:
// each thread moves VEC-byte vectors (16 B when every pointer, stride and row
// length allows it), a CTA covers one (batch row, K|V[, layer]) slice so the
// per-row addressing needs only two magic-number divisions per vector, and
// reads are issued before writes (UNROLL in flight per thread).
#pragma once
#include "common.cuh"

namespace fdl {

constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 4;

// ---------------------------------------------------------------- append --
struct AppendArgs {
  char* dst[2 * FDL_MAX_LAYERS];        // [kv * L + l]
  const char* src[2 * FDL_MAX_LAYERS];  // [kv * L + l]
  const int32_t* start;
  int n_new, max_seq;
  uint32_t total;  // n_new * H * vpr
  FastDiv vpr, heads;
  int64_t dsb, dss, dsh, ssb, sss, ssh;  // bytes
};

template <int VEC>
__global__ void __launch_bounds__(kCopyThreads) kv_append_kernel(const __grid_constant__ AppendArgs a) {
  using V = typename VecT<VEC>::T;
  const int b = blockIdx.y;
  const int slot = blockIdx.z;
  const int start = a.start[b];
  const char* src = a.src[slot] + b * a.ssb;
  char* dst = a.dst[slot] + b * a.dsb;
  V buf[kCopyUnroll];
  int64_t doff[kCopyUnroll];
  const uint32_t base = blockIdx.x * (kCopyThreads * kCopyUnroll) + threadIdx.x;
#pragma unroll
  for (int u = 0; u < kCopyUnroll; ++u) {
    const uint32_t f = base + u * kCopyThreads;
    doff[u] = -1;
    if (f < a.total) {
      uint32_t th, v, t, h;
      a.vpr.divmod(f, th, v);
      a.heads.divmod(th, t, h);
      const int pos = start + static_cast<int>(t);
      if (pos < 0 || pos >= a.max_seq) {
        report(FDL_DEV_INDEX, pos);
        continue;
      }
      buf[u] = ld_vec<VEC>(src + t * a.sss + h * a.ssh + v * VEC);
      doff[u] = pos * a.dss + h * a.dsh + v * VEC;
    }
  }
#pragma unroll
  for (int u = 0; u < kCopyUnroll; ++u)
    if (doff[u] >= 0) st_vec<VEC>(dst + doff[u], buf[u]);
}

// --------------------------------------------------------------- scatter --
struct ScatterArgs {
  char* dst[2];
  const char* src[2];
  const int64_t* pos;
  int64_t pos_sb;
  int n, dst_len;
  uint32_t total;  // n * H * vpr
  FastDiv vpr, heads;
  int64_t dsb, dss, dsh, ssb, sss, ssh;  // bytes
  int dedup;
};

constexpr int kScatterDedupMax = 1024;

template <int VEC>
__global__ void __launch_bounds__(kCopyThreads) kv_scatter_kernel(const __grid_constant__ ScatterArgs a) {
  using V = typename VecT<VEC>::T;
  __shared__ int64_t s_pos[kScatterDedupMax];
  __shared__ uint8_t s_win[kScatterDedupMax];
  const int b = blockIdx.y;
  const int which = blockIdx.z;
  const int64_t* pos = a.pos + b * a.pos_sb;
  if (a.dedup) {
    for (int i = threadIdx.x; i < a.n; i += kCopyThreads) s_pos[i] = pos[i];
    __syncthreads();
    // Sequential-scatter semantics: the last occurrence of a position wins.
    for (int i = threadIdx.x; i < a.n; i += kCopyThreads) {
      uint8_t win = 1;
      const int64_t p = s_pos[i];
      for (int j = i + 1; j < a.n; ++j) win &= (s_pos[j] != p);
      s_win[i] = win;
    }
    __syncthreads();
  }
  const char* src = a.src[which] + b * a.ssb;
  char* dst = a.dst[which] + b * a.dsb;
  V buf[kCopyUnroll];
  int64_t doff[kCopyUnroll];
  const uint32_t base = blockIdx.x * (kCopyThreads * kCopyUnroll) + threadIdx.x;
#pragma unroll
  for (int u = 0; u < kCopyUnroll; ++u) {
    const uint32_t f = base + u * kCopyThreads;
    doff[u] = -1;
    if (f < a.total) {
      uint32_t th, v, i, h;
      a.vpr.divmod(f, th, v);
      a.heads.divmod(th, i, h);
      const int64_t p = a.dedup ? s_pos[i] : pos[i];
      if (a.dedup && !s_win[i]) continue;
      if (p < 0 || p >= a.dst_len) {
        report(FDL_DEV_INDEX, p);
        continue;
      }
      buf[u] = ld_vec<VEC>(src + i * a.sss + h * a.ssh + v * VEC);
      doff[u] = p * a.dss + h * a.dsh + v * VEC;
    }
  }
#pragma unroll
  for (int u = 0; u < kCopyUnroll; ++u)
    if (doff[u] >= 0) st_vec<VEC>(dst + doff[u], buf[u]);
}

// --------------------------------------------------------- prefix gather --
struct GatherPrefixArgs {
  const char* pre[2];
  const char* blk[2];
  char* out[2];
  const int32_t* len;
  const int32_t* cu;
  int64_t out_rows;  // rows of the packed output (cu != nullptr)
  int prefix_cap, n_blk, rep;
  uint32_t total;  // (prefix_cap + n_blk) * Hs * vpr
  FastDiv vpr, heads;
  int64_t psb, pss, psh, bsb, bss, bsh, osb, oss, osh;  // bytes
};

template <int VEC>
__global__ void __launch_bounds__(kCopyThreads) kv_gather_prefix_kernel(const __grid_constant__ GatherPrefixArgs a) {
  using V = typename VecT<VEC>::T;
  const int b = blockIdx.y;
  const int which = blockIdx.z;
  int len = a.len[b];
  if (len < 0 || len > a.prefix_cap) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && which == 0) report(FDL_DEV_LENGTH, len);
    len = len < 0 ? 0 : a.prefix_cap;
  }
  if (a.cu) {
    // The packed range of sequence b is [cu[b], cu[b+1]); it must hold the
    // len + n_blk rows written here and lie inside the output.  A sequence
    // whose range does not is skipped whole and reported.
    const int64_t c0 = a.cu[b], c1 = a.cu[b + 1];
    if (c0 < 0 || c1 > a.out_rows || c0 + len + a.n_blk > c1) {
      if (threadIdx.x == 0 && blockIdx.x == 0 && which == 0) report(FDL_DEV_INDEX, b);
      return;
    }
  }
  const uint32_t per_tok = a.heads.d * a.vpr.d;
  const uint32_t limit = static_cast<uint32_t>(len + a.n_blk) * per_tok;
  const char* pre = a.pre[which] + b * a.psb;
  const char* blk = a.blk[which] ? a.blk[which] + b * a.bsb : nullptr;
  char* out = a.out[which] + (a.cu ? static_cast<int64_t>(a.cu[b]) * a.oss : b * a.osb);
  const uint32_t base = blockIdx.x * (kCopyThreads * kCopyUnroll) + threadIdx.x;
  V buf[kCopyUnroll];
  int64_t ooff[kCopyUnroll];
#pragma unroll
  for (int u = 0; u < kCopyUnroll; ++u) {
    const uint32_t f = base + u * kCopyThreads;
    ooff[u] = -1;
    if (f < limit) {
      uint32_t th, v, t, h;
      a.vpr.divmod(f, th, v);
      a.heads.divmod(th, t, h);
      const char* s = (static_cast<int>(t) < len)
                          ? pre + t * a.pss + h * a.psh
                          : blk + (t - len) * a.bss + h * a.bsh;
      buf[u] = ld_vec<VEC>(s + v * VEC);
      ooff[u] = t * a.oss + static_cast<int64_t>(h) * a.rep * a.osh + v * VEC;
    }
  }
#pragma unroll
  for (int u = 0; u < kCopyUnroll; ++u) {
    if (ooff[u] < 0) continue;
    for (int r = 0; r < a.rep; ++r) st_vec<VEC>(out + ooff[u] + r * a.osh, buf[u]);
  }
}

// ------------------------------------------------------------ row gather --
struct GatherRowsArgs {
  const char* src[2];
  char* out[2];
  const void* idx;
  int idx_i32;
  int64_t idx_sb;
  const int32_t* count;
  int n, src_len;
  uint32_t total;  // n * H * vpr
  FastDiv vpr, heads;
  int64_t ssb, sss, ssh, osb, oss, osh;  // bytes
};

template <int VEC>
__global__ void __launch_bounds__(kCopyThreads) kv_gather_rows_kernel(const __grid_constant__ GatherRowsArgs a) {
  using V = typename VecT<VEC>::T;
  const int b = blockIdx.y;
  const int which = blockIdx.z;
  int n = a.n;
  if (a.count) {
    const int c = a.count[b];
    n = c < 0 ? 0 : (c > a.n ? a.n : c);
  }
  const uint32_t limit = static_cast<uint32_t>(n) * a.heads.d * a.vpr.d;
  const char* src = a.src[which] + b * a.ssb;
  char* out = a.out[which] + b * a.osb;
  const uint32_t base = blockIdx.x * (kCopyThreads * kCopyUnroll) + threadIdx.x;
  V buf[kCopyUnroll];
  int64_t ooff[kCopyUnroll];
#pragma unroll
  for (int u = 0; u < kCopyUnroll; ++u) {
    const uint32_t f = base + u * kCopyThreads;
    ooff[u] = -1;
    if (f < limit) {
      uint32_t th, v, i, h;
      a.vpr.divmod(f, th, v);
      a.heads.divmod(th, i, h);
      const int64_t r = a.idx_i32
                            ? static_cast<int64_t>(static_cast<const int32_t*>(a.idx)[b * a.idx_sb + i])
                            : static_cast<const int64_t*>(a.idx)[b * a.idx_sb + i];
      if (r < 0 || r >= a.src_len) {
        report(FDL_DEV_INDEX, r);
        continue;
      }
      buf[u] = ld_vec<VEC>(src + r * a.sss + h * a.ssh + v * VEC);
      ooff[u] = i * a.oss + h * a.osh + v * VEC;
    }
  }
#pragma unroll
  for (int u = 0; u < kCopyUnroll; ++u)
    if (ooff[u] >= 0) st_vec<VEC>(out + ooff[u], buf[u]);
}

// ------------------------------------------------------ batch compaction --
// In-place gather along the batch axis of up to kCompactMaxBufs buffers:
// row i <- row active[i] for i < n_keep.  A thread owns one VEC-byte column
// of every row of one buffer and walks the rows in increasing i, so no two
// threads touch the same bytes, and when i <= active[i] for every i the
// source row of step i is still unwritten (the rows written before step i
// are all < i <= active[i]).  Every CTA checks that condition over the whole
// list before touching memory; a list outside it moves nothing and is
// reported as FDL_DEV_INDEX.  Rows with active[i] == i are not touched.
constexpr int kCompactMaxBufs = 128;
constexpr int kCompactMaxRows = 4096;
constexpr int kCompactUnroll = 8;

struct CompactArgs {
  char* buf[kCompactMaxBufs];
  const int64_t* active;
  int n_keep, batch;
  int64_t stride;  // bytes between consecutive batch rows
  uint32_t vpr;    // VEC-byte vectors per row
};

template <int VEC>
__global__ void __launch_bounds__(kCopyThreads) kv_compact_kernel(const __grid_constant__ CompactArgs a) {
  using V = typename VecT<VEC>::T;
  __shared__ int s_act[kCompactMaxRows];
  bool ok = true;
  long long bad = 0;
  for (int i = threadIdx.x; i < a.n_keep; i += kCopyThreads) {
    const int64_t s = a.active[i];
    if (s < i || s >= a.batch) {
      ok = false;
      bad = s;
    }
    s_act[i] = static_cast<int>(s);
  }
  if (!__syncthreads_and(ok)) {
    if (!ok && blockIdx.x == 0 && blockIdx.y == 0) report(FDL_DEV_INDEX, bad);
    return;
  }
  const uint32_t v = blockIdx.x * kCopyThreads + threadIdx.x;
  if (v >= a.vpr) return;
  char* col = a.buf[blockIdx.y] + static_cast<int64_t>(v) * VEC;
  for (int i0 = 0; i0 < a.n_keep; i0 += kCompactUnroll) {
    V buf[kCompactUnroll];
#pragma unroll
    for (int u = 0; u < kCompactUnroll; ++u) {
      const int i = i0 + u;
      if (i < a.n_keep && s_act[i] != i) buf[u] = ld_vec<VEC>(col + s_act[i] * a.stride);
    }
#pragma unroll
    for (int u = 0; u < kCompactUnroll; ++u) {
      const int i = i0 + u;
      if (i < a.n_keep && s_act[i] != i) st_vec<VEC>(col + i * a.stride, buf[u]);
    }
  }
}

template <template <int> class K, class Args>
inline void launch_vec(int vec, dim3 grid, const Args& a, cudaStream_t s) {
  switch (vec) {
    case 16: K<16>::launch(grid, a, s); break;
    case 8: K<8>::launch(grid, a, s); break;
    case 4: K<4>::launch(grid, a, s); break;
    default: K<2>::launch(grid, a, s); break;
  }
}

template <int VEC> struct AppendL {
  static void launch(dim3 g, const AppendArgs& a, cudaStream_t s) { kv_append_kernel<VEC><<<g, kCopyThreads, 0, s>>>(a); }
};
template <int VEC> struct ScatterL {
  static void launch(dim3 g, const ScatterArgs& a, cudaStream_t s) { kv_scatter_kernel<VEC><<<g, kCopyThreads, 0, s>>>(a); }
};
template <int VEC> struct GatherPrefixL {
  static void launch(dim3 g, const GatherPrefixArgs& a, cudaStream_t s) { kv_gather_prefix_kernel<VEC><<<g, kCopyThreads, 0, s>>>(a); }
};
template <int VEC> struct GatherRowsL {
  static void launch(dim3 g, const GatherRowsArgs& a, cudaStream_t s) { kv_gather_rows_kernel<VEC><<<g, kCopyThreads, 0, s>>>(a); }
};
template <int VEC> struct CompactL {
  static void launch(dim3 g, const CompactArgs& a, cudaStream_t s) { kv_compact_kernel<VEC><<<g, kCopyThreads, 0, s>>>(a); }
};

inline uint32_t copy_blocks(uint64_t total) {
  return static_cast<uint32_t>((total + kCopyThreads * kCopyUnroll - 1) / (kCopyThreads * kCopyUnroll));
}

}  // namespace fdl
