// fdl_b200: C-ABI entry points of the KV-cache hot path (see
// include/fdl_kvcache.h).  Single translation unit: all kernels share the
// per-device status word declared in common.cuh.
#include <cudaTypedefs.h>
#include <algorithm>
#include <initializer_list>
#include <mutex>

#include "common.cuh"
#include "kv_copy.cuh"
#include "gather_rmsnorm.cuh"
#include "sparse_prefix.cuh"
#include "block_attn.cuh"
#include "rope_swiglu.cuh"
#include "token_select.cuh"
#include "sampling.cuh"

using namespace fdl;

namespace {

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 4-D bf16 tensor map, dims (d0 innermost .. d3), strides in bytes of d1..d3.
bool make_map_4d(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3,
                 uint64_t s1, uint64_t s2, uint64_t s3, uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[4] = {d0, d1, d2, d3};
  const cuuint64_t strides[3] = {s1, s2, s3};
  const cuuint32_t box[4] = {b0, b1, b2, b3};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool attn_smem_configured() {
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  int dev = 0;
  cudaGetDevice(&dev);
  static uint64_t mask = 0;
  if (!(mask & (1ull << dev))) {
    if (cudaFuncSetAttribute(block_attn_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
            cudaSuccess ||
        cudaFuncSetAttribute(block_attn_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
            cudaSuccess)
      return false;
    mask |= 1ull << dev;
  }
  return true;
}

// Persistent attention grid or one CTA per work item.  Measured on B200: the
// persistent walk pays off when there are more items than SMs and each holds
// few key tiles (the decode steps over a short sparse prefix: the next item's
// Q and K/V loads and first MMAs hide the current item's tail and epilogue);
// with long items the per-CTA set-up is already amortised and the one-item
// form is faster.
constexpr int kPersistMaxTiles = 8;
bool attn_persistent(int64_t units, int tiles_per_unit) {
  return units > num_sms() && tiles_per_unit <= kPersistMaxTiles;
}

// Query chunk of one CTA: the G query heads of a KV head times qc queries
// form the CTA's MMA rows, at most max_rows of them, in equal chunks.
int attn_qc_for(int sq, int G, int max_rows) {
  const int cap_q = std::max(1, max_rows / G);
  const int nq = (sq + cap_q - 1) / cap_q;
  return (sq + nq - 1) / nq;
}

struct AttnPlan {
  int qc, splits;
};

// Chunking and split-KV count of one launch.  Up to 256 rows per CTA (two
// 128-row tiles, P over S) or up to 128 (one row tile: S double-buffered, P in
// its own columns -- half the rows per key tile, but twice the CTAs for the
// same work and no split-KV combine where the 256-row form needs one to fill
// the GPU).  Both forms and every split count are scored by an estimate in
// microseconds fitted to B200 measurements of both forms (batch 1-64, prefix
// 256-8192, 32 queries, 6 and 7 query heads per KV head): per CTA about 9 us
// of fixed cost plus 2.18 us per key tile with two row tiles or 1.72 us with
// one, times the waves of CTAs over the SMs; a split adds about 6 us plus the
// fp32 partial rows written and read back by the combine pass.  A forced split
// count (num_splits > 0) is kept; only the chunking is chosen then.
AttnPlan plan_attn(int batch, int sq, int G, int hkv, int tiles, int forced_splits) {
  const int sms = num_sms();
  AttnPlan best{attn_qc_for(sq, G, 256), forced_splits > 0 ? forced_splits : 1};
  double best_us = 1e300;
  const int max_s = std::min(64, std::max(1, tiles));
  int prev_qc = 0;
  for (int max_rows : {256, 128}) {
    const int qc = attn_qc_for(sq, G, max_rows);
    if (qc == prev_qc) break;  // one chunking only
    prev_qc = qc;
    const int64_t units = static_cast<int64_t>(batch) * hkv * ((sq + qc - 1) / qc);
    const double t_tile = G * qc > 128 ? 2.18 : 1.72;
    const int s_lo = forced_splits > 0 ? forced_splits : 1;
    const int s_hi = forced_splits > 0 ? forced_splits : max_s;
    for (int s = s_lo; s <= s_hi; ++s) {
      const int64_t waves = (units * s + sms - 1) / sms;
      const int per = (tiles + s - 1) / s;
      double us = static_cast<double>(waves) * (9.0 + per * t_tile);
      if (s > 1) us += 6.0 + static_cast<double>(batch) * sq * G * hkv * s * 1024.0 / 6.0e6;
      if (us < best_us) {
        best_us = us;
        best = {qc, s};
      }
    }
  }
  return best;
}

}  // namespace

extern "C" {

const char* fdl_version(void) { return "fdl_b200 0.1.0 sm_100a"; }

int fdl_kv_append(void* const* k_caches, void* const* v_caches, const void* const* k_srcs,
                  const void* const* v_srcs, int num_layers, const int32_t* start_pos, int batch, int n_new,
                  int max_seq, int heads, int head_dim, int elem_bytes, int64_t cache_sb, int64_t cache_ss,
                  int64_t cache_sh, int64_t src_sb, int64_t src_ss, int64_t src_sh, fdl_stream_t stream) {
  if (!k_caches || !v_caches || !k_srcs || !v_srcs || !start_pos) return FDL_E_NULL;
  if (num_layers < 1 || num_layers > FDL_MAX_LAYERS || batch < 1 || batch > 65535 || n_new < 0 || max_seq < 1 ||
      heads < 1 || head_dim < 1)
    return FDL_E_SHAPE;
  if (elem_bytes != 2 && elem_bytes != 4) return FDL_E_DTYPE;
  if (n_new == 0) return FDL_OK;
  AppendArgs a{};
  const int64_t rb = static_cast<int64_t>(head_dim) * elem_bytes;
  a.dsb = cache_sb * elem_bytes; a.dss = cache_ss * elem_bytes; a.dsh = cache_sh * elem_bytes;
  a.ssb = src_sb * elem_bytes; a.sss = src_ss * elem_bytes; a.ssh = src_sh * elem_bytes;
  uint64_t align_acc = 0;
  for (int l = 0; l < num_layers; ++l) {
    if (!k_caches[l] || !v_caches[l] || !k_srcs[l] || !v_srcs[l]) return FDL_E_NULL;
    a.dst[l] = static_cast<char*>(k_caches[l]);
    a.dst[num_layers + l] = static_cast<char*>(v_caches[l]);
    a.src[l] = static_cast<const char*>(k_srcs[l]);
    a.src[num_layers + l] = static_cast<const char*>(v_srcs[l]);
    align_acc |= reinterpret_cast<uintptr_t>(k_caches[l]) | reinterpret_cast<uintptr_t>(v_caches[l]) |
                 reinterpret_cast<uintptr_t>(k_srcs[l]) | reinterpret_cast<uintptr_t>(v_srcs[l]);
  }
  const int vec = pick_vec({static_cast<uint64_t>(rb), align_acc, static_cast<uint64_t>(a.dsb),
                            static_cast<uint64_t>(a.dss), static_cast<uint64_t>(a.dsh), static_cast<uint64_t>(a.ssb),
                            static_cast<uint64_t>(a.sss), static_cast<uint64_t>(a.ssh)});
  if (vec < 2) return FDL_E_ALIGN;
  const uint64_t total = static_cast<uint64_t>(n_new) * heads * (rb / vec);
  if (total >= (1ull << 31)) return FDL_E_SHAPE;
  a.start = start_pos;
  a.n_new = n_new;
  a.max_seq = max_seq;
  a.total = static_cast<uint32_t>(total);
  a.vpr.init(static_cast<uint32_t>(rb / vec));
  a.heads.init(static_cast<uint32_t>(heads));
  const dim3 grid(copy_blocks(total), batch, 2 * num_layers);
  launch_vec<AppendL>(vec, grid, a, reinterpret_cast<cudaStream_t>(stream));
  return launch_status();
}

int fdl_kv_scatter(void* k_dst, void* v_dst, const void* k_src, const void* v_src, const int64_t* pos,
                   int64_t pos_sb, int batch, int n, int dst_len, int heads, int head_dim, int elem_bytes,
                   int64_t dst_sb, int64_t dst_ss, int64_t dst_sh, int64_t src_sb, int64_t src_ss, int64_t src_sh,
                   fdl_stream_t stream) {
  if (batch < 1 || batch > 65535 || n < 0 || dst_len < 1 || heads < 1 || head_dim < 1) return FDL_E_SHAPE;
  if (elem_bytes != 2 && elem_bytes != 4) return FDL_E_DTYPE;
  if (n == 0) return FDL_OK;
  if (!k_dst || !k_src || !pos || (v_dst && !v_src)) return FDL_E_NULL;
  ScatterArgs a{};
  const int64_t rb = static_cast<int64_t>(head_dim) * elem_bytes;
  a.dst[0] = static_cast<char*>(k_dst);
  a.dst[1] = static_cast<char*>(v_dst);
  a.src[0] = static_cast<const char*>(k_src);
  a.src[1] = static_cast<const char*>(v_src);
  a.dsb = dst_sb * elem_bytes; a.dss = dst_ss * elem_bytes; a.dsh = dst_sh * elem_bytes;
  a.ssb = src_sb * elem_bytes; a.sss = src_ss * elem_bytes; a.ssh = src_sh * elem_bytes;
  const uint64_t ptrs = reinterpret_cast<uintptr_t>(k_dst) | reinterpret_cast<uintptr_t>(v_dst) |
                        reinterpret_cast<uintptr_t>(k_src) | reinterpret_cast<uintptr_t>(v_src);
  const int vec = pick_vec({static_cast<uint64_t>(rb), ptrs, static_cast<uint64_t>(a.dsb), static_cast<uint64_t>(a.dss),
                            static_cast<uint64_t>(a.dsh), static_cast<uint64_t>(a.ssb), static_cast<uint64_t>(a.sss),
                            static_cast<uint64_t>(a.ssh)});
  if (vec < 2) return FDL_E_ALIGN;
  const uint64_t total = static_cast<uint64_t>(n) * heads * (rb / vec);
  if (total >= (1ull << 31)) return FDL_E_SHAPE;
  a.pos = pos;
  a.pos_sb = pos_sb;
  a.n = n;
  a.dst_len = dst_len;
  a.total = static_cast<uint32_t>(total);
  a.vpr.init(static_cast<uint32_t>(rb / vec));
  a.heads.init(static_cast<uint32_t>(heads));
  a.dedup = n <= kScatterDedupMax ? 1 : 0;
  const dim3 grid(copy_blocks(total), batch, v_dst ? 2 : 1);
  launch_vec<ScatterL>(vec, grid, a, reinterpret_cast<cudaStream_t>(stream));
  return launch_status();
}

int fdl_kv_gather_prefix(const void* k_prefix, const void* v_prefix, const int32_t* len, int prefix_cap,
                         const void* k_block, const void* v_block, int n_blk, void* k_out, void* v_out,
                         const int32_t* cu_seqlens, int64_t out_rows, int batch, int heads, int head_dim, int rep,
                         int elem_bytes,
                         int64_t pre_sb, int64_t pre_ss, int64_t pre_sh, int64_t blk_sb, int64_t blk_ss,
                         int64_t blk_sh, int64_t out_sb, int64_t out_ss, int64_t out_sh, fdl_stream_t stream) {
  if (batch < 1 || batch > 65535 || prefix_cap < 0 || n_blk < 0 || heads < 1 || head_dim < 1 || rep < 1)
    return FDL_E_SHAPE;
  if (elem_bytes != 2 && elem_bytes != 4) return FDL_E_DTYPE;
  if (prefix_cap + n_blk == 0) return FDL_OK;
  if (!len || (!k_out && !v_out)) return FDL_E_NULL;
  if (!k_prefix || !k_out || (v_out && !v_prefix)) return FDL_E_NULL;
  if (n_blk > 0 && (!k_block || (v_out && !v_block))) return FDL_E_NULL;
  if (cu_seqlens && out_rows < 0) return FDL_E_SHAPE;
  GatherPrefixArgs a{};
  const int64_t rb = static_cast<int64_t>(head_dim) * elem_bytes;
  a.pre[0] = static_cast<const char*>(k_prefix);
  a.pre[1] = static_cast<const char*>(v_prefix);
  a.blk[0] = n_blk > 0 ? static_cast<const char*>(k_block) : nullptr;
  a.blk[1] = n_blk > 0 ? static_cast<const char*>(v_block) : nullptr;
  a.out[0] = static_cast<char*>(k_out);
  a.out[1] = static_cast<char*>(v_out);
  a.psb = pre_sb * elem_bytes; a.pss = pre_ss * elem_bytes; a.psh = pre_sh * elem_bytes;
  a.bsb = blk_sb * elem_bytes; a.bss = blk_ss * elem_bytes; a.bsh = blk_sh * elem_bytes;
  a.osb = out_sb * elem_bytes; a.oss = out_ss * elem_bytes; a.osh = out_sh * elem_bytes;
  const uint64_t ptrs = reinterpret_cast<uintptr_t>(k_prefix) | reinterpret_cast<uintptr_t>(v_prefix) |
                        reinterpret_cast<uintptr_t>(a.blk[0]) | reinterpret_cast<uintptr_t>(a.blk[1]) |
                        reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(v_out);
  const int vec = pick_vec({static_cast<uint64_t>(rb), ptrs, static_cast<uint64_t>(a.psb), static_cast<uint64_t>(a.pss),
                            static_cast<uint64_t>(a.psh), static_cast<uint64_t>(a.bsb), static_cast<uint64_t>(a.bss),
                            static_cast<uint64_t>(a.bsh), static_cast<uint64_t>(a.osb), static_cast<uint64_t>(a.oss),
                            static_cast<uint64_t>(a.osh)});
  if (vec < 2) return FDL_E_ALIGN;
  const uint64_t total = static_cast<uint64_t>(prefix_cap + n_blk) * heads * (rb / vec);
  if (total >= (1ull << 31)) return FDL_E_SHAPE;
  if (total == 0) return FDL_OK;
  a.len = len;
  a.cu = cu_seqlens;
  a.out_rows = out_rows;
  a.prefix_cap = prefix_cap;
  a.n_blk = n_blk;
  a.rep = rep;
  a.total = static_cast<uint32_t>(total);
  a.vpr.init(static_cast<uint32_t>(rb / vec));
  a.heads.init(static_cast<uint32_t>(heads));
  const dim3 grid(copy_blocks(total), batch, v_out ? 2 : 1);
  launch_vec<GatherPrefixL>(vec, grid, a, reinterpret_cast<cudaStream_t>(stream));
  return launch_status();
}

int fdl_kv_gather_rows(const void* k_src, const void* v_src, const void* idx, int idx_is_i32, int64_t idx_sb,
                       const int32_t* count, void* k_out, void* v_out, int batch, int n, int src_len, int heads,
                       int head_dim, int elem_bytes, int64_t src_sb, int64_t src_ss, int64_t src_sh, int64_t out_sb,
                       int64_t out_ss, int64_t out_sh, fdl_stream_t stream) {
  if (batch < 1 || batch > 65535 || n < 0 || src_len < 1 || heads < 1 || head_dim < 1) return FDL_E_SHAPE;
  if (elem_bytes != 2 && elem_bytes != 4) return FDL_E_DTYPE;
  if (n == 0) return FDL_OK;
  if (!k_src || !k_out || !idx || (v_out && !v_src)) return FDL_E_NULL;
  GatherRowsArgs a{};
  const int64_t rb = static_cast<int64_t>(head_dim) * elem_bytes;
  a.src[0] = static_cast<const char*>(k_src);
  a.src[1] = static_cast<const char*>(v_src);
  a.out[0] = static_cast<char*>(k_out);
  a.out[1] = static_cast<char*>(v_out);
  a.ssb = src_sb * elem_bytes; a.sss = src_ss * elem_bytes; a.ssh = src_sh * elem_bytes;
  a.osb = out_sb * elem_bytes; a.oss = out_ss * elem_bytes; a.osh = out_sh * elem_bytes;
  const uint64_t ptrs = reinterpret_cast<uintptr_t>(k_src) | reinterpret_cast<uintptr_t>(v_src) |
                        reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(v_out);
  const int vec = pick_vec({static_cast<uint64_t>(rb), ptrs, static_cast<uint64_t>(a.ssb), static_cast<uint64_t>(a.sss),
                            static_cast<uint64_t>(a.ssh), static_cast<uint64_t>(a.osb), static_cast<uint64_t>(a.oss),
                            static_cast<uint64_t>(a.osh)});
  if (vec < 2) return FDL_E_ALIGN;
  const uint64_t total = static_cast<uint64_t>(n) * heads * (rb / vec);
  if (total >= (1ull << 31)) return FDL_E_SHAPE;
  a.idx = idx;
  a.idx_i32 = idx_is_i32;
  a.idx_sb = idx_sb;
  a.count = count;
  a.n = n;
  a.src_len = src_len;
  a.total = static_cast<uint32_t>(total);
  a.vpr.init(static_cast<uint32_t>(rb / vec));
  a.heads.init(static_cast<uint32_t>(heads));
  const dim3 grid(copy_blocks(total), batch, v_out ? 2 : 1);
  launch_vec<GatherRowsL>(vec, grid, a, reinterpret_cast<cudaStream_t>(stream));
  return launch_status();
}

int fdl_kv_compact(void* const* bufs, int n_bufs, int64_t row_bytes, int64_t batch_stride, int batch,
                   const int64_t* active, int n_keep, fdl_stream_t stream) {
  if (n_keep == 0 || n_bufs == 0 || row_bytes == 0) return FDL_OK;
  if (!bufs || !active) return FDL_E_NULL;
  if (n_bufs < 0 || n_keep < 0 || batch < 1 || batch > 65535 || n_keep > batch || n_keep > kCompactMaxRows ||
      row_bytes < 0 || batch_stride < row_bytes)
    return FDL_E_SHAPE;
  uint64_t align_acc = 0;
  for (int j = 0; j < n_bufs; ++j) {
    if (!bufs[j]) return FDL_E_NULL;
    align_acc |= reinterpret_cast<uintptr_t>(bufs[j]);
  }
  const int vec = pick_vec({static_cast<uint64_t>(row_bytes), static_cast<uint64_t>(batch_stride), align_acc});
  if (vec < 2) return FDL_E_ALIGN;
  const uint64_t vpr = static_cast<uint64_t>(row_bytes) / vec;
  if (vpr >= (1ull << 31)) return FDL_E_SHAPE;
  CompactArgs a{};
  a.active = active;
  a.n_keep = n_keep;
  a.batch = batch;
  a.stride = batch_stride;
  a.vpr = static_cast<uint32_t>(vpr);
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int j0 = 0; j0 < n_bufs; j0 += kCompactMaxBufs) {
    const int nb = std::min(kCompactMaxBufs, n_bufs - j0);
    for (int j = 0; j < nb; ++j) a.buf[j] = static_cast<char*>(bufs[j0 + j]);
    const dim3 grid(static_cast<uint32_t>((vpr + kCopyThreads - 1) / kCopyThreads), nb);
    launch_vec<CompactL>(vec, grid, a, s);
    const int rc = launch_status();
    if (rc != FDL_OK) return rc;
  }
  return FDL_OK;
}

int64_t fdl_sparse_prefix_workspace_bytes(int batch, int cap) {
  const int64_t b = static_cast<int64_t>(batch) * cap * 4;
  return (b + 255) / 256 * 256;
}

int fdl_kv_sparse_prefix(const void* k, const void* v, const int32_t* len, int batch, int cap, int heads,
                         int head_dim, int64_t kv_sb, int64_t kv_ss, int64_t kv_sh, int keep_num, int keep_den,
                         int max_keep, int32_t* sel, int32_t* out_len, void* k_out, void* v_out, int64_t out_sb,
                         int64_t out_ss, int64_t out_sh, void* workspace, int64_t workspace_bytes,
                         fdl_stream_t stream) {
  if (!k || !len || !sel || !out_len || !workspace) return FDL_E_NULL;
  if ((k_out || v_out) && (!k_out || !v_out || !v)) return FDL_E_NULL;
  if (batch < 1 || batch > 65535 || cap < 1 || heads < 1 || head_dim < 1 || max_keep < 1) return FDL_E_SHAPE;
  if (keep_num < 0 || keep_den < 1 || keep_num > keep_den) return FDL_E_SHAPE;
  if ((heads * head_dim) % 8 != 0 || kv_sh != head_dim) return FDL_E_UNSUPPORTED;  // token row contiguous
  if (!aligned16(k) || ((kv_ss * 2) % 16) || ((kv_sb * 2) % 16)) return FDL_E_ALIGN;
  if (workspace_bytes < fdl_sparse_prefix_workspace_bytes(batch, cap) || !aligned16(workspace))
    return FDL_E_WORKSPACE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float* score = static_cast<float*>(workspace);
  ScoreArgs sa{static_cast<const char*>(k), len, score, cap, heads * head_dim, kv_sb * 2, kv_ss * 2};
  key_score_kernel<<<dim3((cap + 7) / 8, batch), kScoreThreads, 0, s>>>(sa);
  SelectArgs xa{score, len, sel, out_len, cap, keep_num, keep_den, max_keep};
  topk_select_kernel<<<batch, kSelectThreads, 0, s>>>(xa);
  int rc = launch_status();
  if (rc != FDL_OK || !k_out) return rc;
  return fdl_kv_gather_rows(k, v, sel, 1, max_keep, out_len, k_out, v_out, batch, max_keep, cap, heads, head_dim, 2,
                            kv_sb, kv_ss, kv_sh, out_sb, out_ss, out_sh, stream);
}

}  // extern "C"

namespace {
// Score scratch of fdl_kv_sparse_prefix_noalloc: a fixed array in device
// memory, one per device, alive until the process exits.  Host code must not
// pass `g_noalloc_scores` itself to a kernel (on the host it names a shadow
// variable, not device memory); it uses the address looked up per device.
static __device__ __align__(256) float g_noalloc_scores[FDL_NOALLOC_SCORE_MAX];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[256] = {};

// Device address of g_noalloc_scores on the current device (looked up once
// per device, with that device current).
int noalloc_scores_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return -static_cast<int>(e);
  if (dev < 0 || dev >= 256) return FDL_E_NODEVICE;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scores);
    if (e != cudaSuccess || !p) return e != cudaSuccess ? -static_cast<int>(e) : FDL_E_NODEVICE;
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return FDL_OK;
}
}  // namespace

extern "C" {

int fdl_kv_sparse_prefix_noalloc(const void* k, const void* v, const int32_t* len, int batch, int cap, int heads,
                                 int head_dim, int64_t kv_sb, int64_t kv_ss, int64_t kv_sh, int keep_num,
                                 int keep_den, int max_keep, int32_t* sel, int32_t* out_len, void* k_out,
                                 void* v_out, int64_t out_sb, int64_t out_ss, int64_t out_sh, fdl_stream_t stream) {
  if (batch < 1 || cap < 1) return FDL_E_SHAPE;
  if (static_cast<int64_t>(batch) * cap > FDL_NOALLOC_SCORE_MAX) return FDL_E_WORKSPACE;
  void* scores = nullptr;
  const int rc = noalloc_scores_address(&scores);
  if (rc != FDL_OK) return rc;
  return fdl_kv_sparse_prefix(k, v, len, batch, cap, heads, head_dim, kv_sb, kv_ss, kv_sh, keep_num, keep_den,
                              max_keep, sel, out_len, k_out, v_out, out_sb, out_ss, out_sh, scores,
                              static_cast<int64_t>(FDL_NOALLOC_SCORE_MAX) * sizeof(float), stream);
}

int fdl_gather_rmsnorm(const void* x, const int64_t* idx, int64_t idx_sb, const void* w, float eps, void* gathered,
                       void* normed, int batch, int seq, int n_tok, int hidden, int x_dtype, int64_t x_sb,
                       int64_t x_ss, int64_t out_sb, int64_t out_ss, fdl_stream_t stream) {
  if (batch < 1 || seq < 0 || n_tok < 0 || hidden < 1) return FDL_E_SHAPE;
  if (!idx && n_tok > seq) return FDL_E_SHAPE;
  if (static_cast<int64_t>(batch) * n_tok >= (1ll << 31)) return FDL_E_SHAPE;
  if (n_tok == 0) return FDL_OK;
  if (!x || !normed) return FDL_E_NULL;
  int es;
  switch (x_dtype) {
    case FDL_BF16: case FDL_F16: es = 2; break;
    case FDL_F32: es = 4; break;
    default: return FDL_E_DTYPE;
  }
  NormArgs a{};
  a.x = static_cast<const char*>(x);
  a.idx = idx;
  a.idx_sb = idx_sb;
  a.w = static_cast<const char*>(w);
  a.gathered = static_cast<char*>(gathered);
  a.normed = static_cast<char*>(normed);
  a.eps = eps;
  a.B = batch; a.S = seq; a.T = n_tok; a.H = hidden;
  a.x_sb = x_sb * es; a.x_ss = x_ss * es; a.o_sb = out_sb * es; a.o_ss = out_ss * es;
  const uint64_t ptrs = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gathered) |
                        reinterpret_cast<uintptr_t>(normed) | reinterpret_cast<uintptr_t>(w);
  const bool vec_ok = pick_vec({static_cast<uint64_t>(hidden) * es, ptrs, static_cast<uint64_t>(a.x_sb),
                                static_cast<uint64_t>(a.x_ss), static_cast<uint64_t>(a.o_sb),
                                static_cast<uint64_t>(a.o_ss)}) == 16;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (x_dtype == FDL_BF16) launch_gather_rmsnorm<__nv_bfloat16>(a, vec_ok, s);
  else if (x_dtype == FDL_F16) launch_gather_rmsnorm<__half>(a, vec_ok, s);
  else launch_gather_rmsnorm<float>(a, vec_ok, s);
  return launch_status();
}

int fdl_add_rmsnorm(const void* x, int64_t x_rs, const void* res, int64_t res_rs, const void* w, float eps,
                    void* sum_out, void* normed, int64_t out_rs, int rows, int hidden, int x_dtype,
                    fdl_stream_t stream) {
  if (rows < 0 || hidden < 1) return FDL_E_SHAPE;
  if (rows == 0) return FDL_OK;
  if (!x || !res || !normed) return FDL_E_NULL;
  int es;
  switch (x_dtype) {
    case FDL_BF16: case FDL_F16: es = 2; break;
    default: return FDL_E_DTYPE;
  }
  NormArgs a{};
  a.x = static_cast<const char*>(x);
  a.res = static_cast<const char*>(res);
  a.res_ss = res_rs * es;
  a.w = static_cast<const char*>(w);
  a.gathered = static_cast<char*>(sum_out);
  a.normed = static_cast<char*>(normed);
  a.eps = eps;
  a.B = 1; a.S = rows; a.T = rows; a.H = hidden;
  a.x_sb = 0; a.x_ss = x_rs * es; a.o_sb = 0; a.o_ss = out_rs * es;
  const uint64_t ptrs = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(res) |
                        reinterpret_cast<uintptr_t>(sum_out) | reinterpret_cast<uintptr_t>(normed) |
                        reinterpret_cast<uintptr_t>(w);
  const bool vec_ok = pick_vec({static_cast<uint64_t>(hidden) * es, ptrs, static_cast<uint64_t>(a.x_ss),
                                static_cast<uint64_t>(a.res_ss), static_cast<uint64_t>(a.o_ss)}) == 16;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (x_dtype == FDL_BF16) launch_gather_rmsnorm<__nv_bfloat16>(a, vec_ok, s);
  else launch_gather_rmsnorm<__half>(a, vec_ok, s);
  return launch_status();
}

int64_t fdl_block_attn_workspace_bytes(int batch, int sq, int hq, int head_dim, int num_splits) {
  if (num_splits <= 1) return 0;
  const int64_t rows = static_cast<int64_t>(batch) * sq * hq;
  const int64_t b = static_cast<int64_t>(num_splits) * rows * (head_dim + 1) * 4;
  return (b + 255) / 256 * 256 + 256;
}

int fdl_block_attn_auto_splits(int batch, int sq, int hq, int hkv, int cap, int n_blk) {
  if (batch < 1 || sq < 1 || hq < 1 || hkv < 1 || hq % hkv) return 1;
  const int G = hq / hkv;
  if (G > 256) return 1;
  const int tiles = (cap + kBlockN - 1) / kBlockN + (n_blk + kBlockN - 1) / kBlockN;
  return plan_attn(batch, sq, G, hkv, tiles, 0).splits;
}

int fdl_block_attn(const void* q, const void* k, const void* v, const int32_t* seqlens, int cap, const void* k_blk,
                   const void* v_blk, int n_blk, const int32_t* q_pos, int mask_block, void* out, int batch, int sq,
                   int hq, int hkv, int head_dim, float scale, int64_t q_sb, int64_t q_ss, int64_t q_sh,
                   int64_t kv_sb, int64_t kv_ss, int64_t kv_sh, int64_t blk_sb, int64_t blk_ss, int64_t blk_sh,
                   int64_t o_sb, int64_t o_ss, int64_t o_sh, int num_splits, void* workspace,
                   int64_t workspace_bytes, fdl_stream_t stream) {
  if (!q || !k || !v || !seqlens || !out) return FDL_E_NULL;
  if (n_blk > 0 && (!k_blk || !v_blk)) return FDL_E_NULL;
  if (head_dim != kHeadDim) return FDL_E_UNSUPPORTED;
  if (batch < 1 || batch > 65535 || sq < 1 || hq < 1 || hkv < 1 || hq % hkv || cap < 1 || n_blk < 0 ||
      mask_block < 0)
    return FDL_E_SHAPE;
  const int G = hq / hkv;
  if (G > 256) return FDL_E_UNSUPPORTED;
  // TMA: 16-byte aligned bases and strides; head dim contiguous.
  for (const void* p : std::initializer_list<const void*>{q, k, v, out}) if (!aligned16(p)) return FDL_E_ALIGN;
  if (n_blk > 0 && (!aligned16(k_blk) || !aligned16(v_blk))) return FDL_E_ALIGN;
  for (int64_t st : std::initializer_list<int64_t>{q_sb, q_ss, q_sh, kv_sb, kv_ss, kv_sh, o_sb, o_ss, o_sh})
    if ((st * 2) % 16) return FDL_E_ALIGN;
  if (n_blk > 0)
    for (int64_t st : std::initializer_list<int64_t>{blk_sb, blk_ss, blk_sh}) if ((st * 2) % 16) return FDL_E_ALIGN;

  if (q_sh > q_ss && sq > 1) return FDL_E_UNSUPPORTED;  // query memory must be [B, S, H, D]
  AttnParams p{};
  p.G = G;
  const AttnPlan plan = plan_attn(batch, sq, G, hkv,
                                  (cap + kBlockN - 1) / kBlockN + (n_blk + kBlockN - 1) / kBlockN, num_splits);
  p.qc = plan.qc;
  p.n_qchunks = (sq + p.qc - 1) / p.qc;
  p.n_mt = (G * p.qc + 127) / 128;
  int splits = plan.splits;
  if (splits > 1) {
    const int64_t need = fdl_block_attn_workspace_bytes(batch, sq, hq, head_dim, splits);
    if (!workspace || workspace_bytes < need) {
      if (num_splits > 0) return FDL_E_WORKSPACE;
      splits = 1;  // auto mode without room for partials: single pass
    }
  }
  const int64_t e = 2;  // bf16
  if (!make_map_4d(&p.tm_q, q, head_dim, hq, sq, batch, q_sh * e, q_ss * e, q_sb * e, 64, G, p.qc, 1))
    return FDL_E_NODEVICE;
  // K/V maps list dims in increasing stride order: (D, H, S, B) for
  // sequence-major memory (BSHD), (D, S, H, B) for head-major (BHSD).
  auto kv_maps = [&](CUtensorMap* mk, CUtensorMap* mv, const void* kp, const void* vp, int len_dim, int64_t sb,
                     int64_t ss, int64_t sh, int* hmajor) {
    *hmajor = sh > ss ? 1 : 0;
    if (*hmajor)
      return make_map_4d(mk, kp, head_dim, len_dim, hkv, batch, ss * e, sh * e, sb * e, 64, kBlockN, 1, 1) &&
             make_map_4d(mv, vp, head_dim, len_dim, hkv, batch, ss * e, sh * e, sb * e, 64, kBlockN, 1, 1);
    return make_map_4d(mk, kp, head_dim, hkv, len_dim, batch, sh * e, ss * e, sb * e, 64, 1, kBlockN, 1) &&
           make_map_4d(mv, vp, head_dim, hkv, len_dim, batch, sh * e, ss * e, sb * e, 64, 1, kBlockN, 1);
  };
  if (!kv_maps(&p.tm_k, &p.tm_v, k, v, cap, kv_sb, kv_ss, kv_sh, &p.kv_hmajor)) return FDL_E_NODEVICE;
  if (n_blk > 0) {
    if (!kv_maps(&p.tm_kb, &p.tm_vb, k_blk, v_blk, n_blk, blk_sb, blk_ss, blk_sh, &p.blk_hmajor))
      return FDL_E_NODEVICE;
  } else {
    p.tm_kb = p.tm_k;
    p.tm_vb = p.tm_v;
    p.blk_hmajor = p.kv_hmajor;
  }
  if (!attn_smem_configured()) return FDL_E_NODEVICE;
  p.seqlens = seqlens;
  p.q_pos = q_pos;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.B = batch; p.Sq = sq; p.Hq = hq; p.Hkv = hkv; p.cap = cap; p.n_blk = n_blk;
  p.mask_block = mask_block;
  p.splits = splits;
  const int64_t units = static_cast<int64_t>(splits) * hkv * p.n_qchunks * batch;
  if (units >= (1ll << 31)) return FDL_E_SHAPE;
  p.n_units = static_cast<int>(units);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o_sb = o_sb; p.o_ss = o_ss; p.o_sh = o_sh;
  const int64_t rows = static_cast<int64_t>(batch) * sq * hq;
  if (splits > 1) {
    p.ws_o = static_cast<float*>(workspace);
    p.ws_lse = p.ws_o + static_cast<int64_t>(splits) * rows * head_dim;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int tiles_all = (cap + kBlockN - 1) / kBlockN + (n_blk + kBlockN - 1) / kBlockN;
  if (attn_persistent(units, (tiles_all + splits - 1) / splits)) {
    // One CTA per SM (the kernel's shared memory allows no more), each
    // walking its share of the work items.
    block_attn_kernel<true><<<num_sms(), kAttnThreads, kSmemBytes, s>>>(p);
  } else {
    block_attn_kernel<false><<<static_cast<unsigned>(units), kAttnThreads, kSmemBytes, s>>>(p);
  }
  int rc = launch_status();
  if (rc != FDL_OK || splits == 1) return rc;
  attn_combine_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, s>>>(p.ws_o, p.ws_lse, p.out, splits, batch,
                                                                            sq, hq, o_sb, o_ss, o_sh);
  return launch_status();
}

int fdl_cosine_select(const void* hidden, const void* cached, void* cache_out, int batch, int seq, int hidden_size,
                      int dtype, int64_t h_sb, int64_t h_ss, int64_t c_sb, int64_t c_ss, int64_t o_sb, int64_t o_ss,
                      int n_select, int64_t* idx, int64_t idx_sb, float* cos_out, fdl_stream_t stream) {
  if (dtype != FDL_BF16 && dtype != FDL_F32) return FDL_E_DTYPE;
  const int esz = dtype == FDL_BF16 ? 2 : 4;
  if (batch < 0 || batch > 65535 || seq < 1 || seq > kSelMaxSeq || hidden_size < 1 ||
      (hidden_size * esz) % 16 || n_select < 0 || n_select > seq || idx_sb < n_select)
    return FDL_E_SHAPE;
  if (batch == 0) return FDL_OK;
  if (!hidden || !cached || (n_select > 0 && !idx)) return FDL_E_NULL;
  for (int64_t st : {h_sb, h_ss, c_sb, c_ss, o_sb, o_ss})
    if ((st * esz) % 16) return FDL_E_ALIGN;
  if (!aligned16(hidden) || !aligned16(cached) || (cache_out && !aligned16(cache_out))) return FDL_E_ALIGN;
  CosSelectArgs a{static_cast<const char*>(hidden), static_cast<const char*>(cached), static_cast<char*>(cache_out),
                  h_sb * esz, h_ss * esz, c_sb * esz, c_ss * esz, o_sb * esz, o_ss * esz,
                  seq, hidden_size, n_select, dtype == FDL_BF16, idx, idx_sb, cos_out};
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == FDL_BF16)
    cosine_select_kernel<true><<<batch, kCosThreads, 0, s>>>(a);
  else
    cosine_select_kernel<false><<<batch, kCosThreads, 0, s>>>(a);
  return launch_status();
}

int fdl_focus_select(const void* delta, int64_t delta_sb, const uint8_t* mask, int64_t mask_sb, const uint8_t* frozen,
                     int64_t frozen_sb, int batch, int seq, int k_floor, int dtype, int64_t* sel, int64_t sel_sb,
                     int32_t* ksel, fdl_stream_t stream) {
  if (dtype != FDL_BF16 && dtype != FDL_F32) return FDL_E_DTYPE;
  if (batch < 0 || batch > kFocusSelMaxRows || seq < 1 || seq > kSelMaxSeq || k_floor < 1 || k_floor > seq ||
      sel_sb < seq)
    return FDL_E_SHAPE;
  if (batch == 0) return FDL_OK;
  if (!delta || !mask || !sel || !ksel) return FDL_E_NULL;
  const int esz = dtype == FDL_BF16 ? 2 : 4;
  FocusSelectArgs a{static_cast<const char*>(delta), delta_sb * esz, mask, mask_sb, frozen, frozen_sb,
                    batch, seq, k_floor, dtype == FDL_BF16, sel, sel_sb, ksel};
  focus_select_kernel<<<1, kFocusSelThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return launch_status();
}

int fdl_focus_importance(const void* q, const void* k, const uint8_t* mask, int batch, int seq, int hq, int hkv,
                         int head_dim, int dtype, int64_t q_sb, int64_t q_sh, int64_t q_ss, int64_t k_sb, int64_t k_sh,
                         int64_t k_ss, int64_t mask_sb, float scaling, void* imp, int64_t imp_sb,
                         fdl_stream_t stream) {
  if (dtype != FDL_BF16 && dtype != FDL_F32) return FDL_E_DTYPE;
  const int esz = dtype == FDL_BF16 ? 2 : 4;
  if (batch < 0 || batch > 65535 || seq < 1 || seq > kSelMaxSeq || hq < 1 || hq > kImpMaxHeads || hkv < 1 ||
      hq % hkv || head_dim < 1 || head_dim > kImpMaxDim || (head_dim * esz) % 16)
    return FDL_E_SHAPE;
  if (batch == 0) return FDL_OK;
  if (!q || !k || !mask || !imp) return FDL_E_NULL;
  if (!aligned16(q) || (q_sb * esz) % 16 || (q_sh * esz) % 16 || (q_ss * esz) % 16) return FDL_E_ALIGN;
  FocusImportanceArgs a{static_cast<const char*>(q), q_sb * esz, q_sh * esz, q_ss * esz,
                        static_cast<const char*>(k), k_sb * esz, k_sh * esz, k_ss * esz,
                        mask, mask_sb, seq, hq, hkv, head_dim, dtype == FDL_BF16, scaling,
                        static_cast<char*>(imp), imp_sb * esz};
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == FDL_BF16)
    focus_importance_kernel<true><<<batch, kImpThreads, 0, s>>>(a);
  else
    focus_importance_kernel<false><<<batch, kImpThreads, 0, s>>>(a);
  return launch_status();
}

int fdl_rope_qkv(const void* y, int64_t y_rs, const int64_t* pos, const float* inv_freq, void* q, void* k, void* v,
                 int rows, int hq, int hkv, int head_dim, fdl_stream_t stream) {
  if (rows < 0 || hq < 1 || hkv < 1 || head_dim < 16 || head_dim % 16 || head_dim / 2 > kRopeMaxHalf)
    return FDL_E_SHAPE;
  if (rows == 0) return FDL_OK;
  if (!y || !pos || !inv_freq || !q || !k || !v) return FDL_E_NULL;
  if (!aligned16(y) || !aligned16(q) || !aligned16(k) || !aligned16(v) || (y_rs * 2) % 16) return FDL_E_ALIGN;
  RopeArgs a{static_cast<const __nv_bfloat16*>(y), y_rs, pos, inv_freq, static_cast<__nv_bfloat16*>(q),
             static_cast<__nv_bfloat16*>(k), static_cast<__nv_bfloat16*>(v), rows, hq, hkv, head_dim};
  rope_qkv_kernel<<<rows, kRopeThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return launch_status();
}

int fdl_rope_qkv_kv(const void* y, int64_t y_rs, const int64_t* pos, const float* inv_freq, void* q, void* k_dst,
                    void* v_dst, int64_t dst_sb, int64_t dst_ss, int64_t dst_sh, int dst_len, const int32_t* start,
                    const int64_t* dst_pos, int64_t dst_pos_sb, int batch, int n, int hq, int hkv, int head_dim,
                    fdl_stream_t stream) {
  if (batch < 0 || batch > 65535 || n < 0 || hq < 1 || hkv < 1 || head_dim < 16 || head_dim % 16 ||
      head_dim / 2 > kRopeMaxHalf || dst_len < 1 || (start && dst_pos))
    return FDL_E_SHAPE;
  const int64_t rows = static_cast<int64_t>(batch) * n;
  if (rows == 0) return FDL_OK;
  if (rows >= (1ll << 31)) return FDL_E_SHAPE;
  if (!y || !pos || !inv_freq || !q || !k_dst || !v_dst) return FDL_E_NULL;
  if (!aligned16(y) || !aligned16(q) || !aligned16(k_dst) || !aligned16(v_dst) || (y_rs * 2) % 16 ||
      (dst_sb * 2) % 16 || (dst_ss * 2) % 16 || (dst_sh * 2) % 16)
    return FDL_E_ALIGN;
  RopeStoreArgs a{static_cast<const __nv_bfloat16*>(y), y_rs, pos, inv_freq, static_cast<__nv_bfloat16*>(q),
                  static_cast<char*>(k_dst), static_cast<char*>(v_dst), dst_sb * 2, dst_ss * 2, dst_sh * 2, start,
                  dst_pos, dst_pos_sb, static_cast<int>(rows), hq, hkv, head_dim, n, dst_len};
  rope_qkv_store_kernel<<<static_cast<unsigned>(rows), kRopeThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return launch_status();
}

int fdl_swiglu(const void* gu, int64_t gu_rs, void* out, int64_t out_rs, int64_t rows, int ffn,
               fdl_stream_t stream) {
  if (rows < 0 || rows > INT32_MAX || ffn < 8 || ffn % 8) return FDL_E_SHAPE;
  if (rows == 0) return FDL_OK;
  if (!gu || !out) return FDL_E_NULL;
  if (!aligned16(gu) || !aligned16(out) || (gu_rs * 2) % 16 || (out_rs * 2) % 16) return FDL_E_ALIGN;
  const uint64_t total = static_cast<uint64_t>(rows) * (ffn / 8);
  if (total >= (1ull << 31)) return FDL_E_SHAPE;
  SwigluArgs a{static_cast<const __nv_bfloat16*>(gu), gu_rs, static_cast<__nv_bfloat16*>(out), out_rs, rows, ffn,
               static_cast<uint32_t>(total), {}};
  a.vpr.init(static_cast<uint32_t>(ffn / 8));
  const unsigned grid = static_cast<unsigned>((total + kSwigluChunk - 1) / kSwigluChunk);
  swiglu_kernel<<<grid, kSwigluThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return launch_status();
}

int fdl_softmax_argmax(const void* logits, int64_t row_stride, int rows, int vocab, int64_t* token, void* prob,
                       fdl_stream_t stream) {
  if (rows < 0 || rows > INT32_MAX || vocab < 1 || row_stride < vocab) return FDL_E_SHAPE;
  if (rows == 0) return FDL_OK;
  if (!logits || !token) return FDL_E_NULL;
  if (!aligned16(logits) || (row_stride * 2) % 16) return FDL_E_ALIGN;
  SampleArgs a{static_cast<const __nv_bfloat16*>(logits), row_stride, vocab, token,
               static_cast<__nv_bfloat16*>(prob)};
  softmax_argmax_kernel<<<static_cast<unsigned>(rows), kSampleThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return launch_status();
}

int fdl_last_device_error(int32_t* code, int64_t* info) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return -static_cast<int>(e);
  int c = 0;
  long long i = 0;
  e = cudaMemcpyFromSymbol(&c, g_dev_status, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&i, g_dev_info, sizeof(long long));
  if (e != cudaSuccess) return -static_cast<int>(e);
  const int zero = 0;
  const long long zl = 0;
  cudaMemcpyToSymbol(g_dev_status, &zero, sizeof(int));
  cudaMemcpyToSymbol(g_dev_info, &zl, sizeof(long long));
  if (code) *code = c;
  if (info) *info = i;
  return FDL_OK;
}

}  // extern "C"
