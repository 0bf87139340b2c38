// (d) Block attention over the KV cache on sm_100a: TMA -> shared memory,
// tcgen05.mma (bf16 in, fp32 accumulate in TMEM), online softmax,
// GQA packed into the MMA M dimension.
//
// One CTA = (batch row b, KV head g, query chunk, KV split).  The G = Hq/Hkv
// query heads that share KV head g, times the qc queries of the chunk, form
// R = G*qc <= 256 rows (224 for the 7B geometry: 7 heads x 32 queries),
// processed as one or two 128-row MMA tiles against the same K/V tiles -- the
// GQA expansion never touches memory.  Keys stream in tiles of 128 through a
// 2-stage TMA pipeline (64 KB of K+V per stage); each tile is also
// prefetched into L2 one tile ahead of its shared-memory load, and a stage
// is released as soon as the last row tile's P * V of that tile completes.
//
// Warp roles (320 threads):
//   warp 0      TMA producer (Q once, then K/V tiles)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..5  softmax for rows   0..127 (TMEM lanes = rows)
//   warps 6..9  softmax for rows 128..255
// Per key tile j and row tile m:
//   S_m = Q_m K_j^T          tcgen05.mma, A and B from shared memory,
//                            128 fp32 TMEM columns
//   softmax warps            S_m row read from TMEM in halves of 64
//                            columns (no register spills), row max, then
//                            P = exp2(S - max) written back as bf16 into the
//                            first 64 columns of S_m's own TMEM range;
//                            O_m is rescaled in TMEM only when the row max
//                            grows by more than 2^8 (the stale max is kept
//                            otherwise -- identical up to rounding)
//   O_m += P_m V_j           tcgen05.mma with A read from TMEM, B (V,
//                            head-dim contiguous) from shared memory
// S_m(j+1) overwrites the TMEM that P_m(j) * V_j reads; the issuer queues
// S_m(j+1) directly behind P_m(j) * V_j, relying on the tensor core running
// one thread's MMAs in issue order (operands of an MMA are read before a
// later MMA writes), as sm100 attention kernels with this TMEM layout do.
// Measured against waiting for the completion of P_m(j) * V_j first: results
// identical, +0.5% (B=64, P=8192) to +4.7% (B=16, P=4096).  Every s_full
// commit still fires only after all earlier MMAs of the thread completed, so
// S_m(j) ready implies P_m(j-1) * V_(j-1) done (O_m stable for a rescale).
// The two row tiles alternate (ping-pong) so the softmax of one tile overlaps
// the MMAs of the other.
// (Two issuers, one per row tile, keep the pipe fuller in isolation but slow
// the softmax warps, which bound the kernel, by more.)
//
// With a single row tile (R <= 128) the second tile's TMEM holds a second S
// buffer and P gets its own columns, so S(j+1) overlaps the softmax of S(j).
// Padding rows (beyond R or past the last query) count as fully visible and
// whole warps of them skip the softmax, so they never take the predicated
// path that would make their row tile wait for them.
//
// TMEM columns: S_0 [0,128) S_1 [128,256) O_0 [256,384) O_1 [384,512)
// (one row tile: S buffers [0,128) [128,256), O [256,384), P [384,448)).
// Shared memory: Q 64 KB | K 2x32 KB | V 2x32 KB | barriers.
#pragma once
#include <cuda.h>
#include "sm100_ptx.cuh"

namespace fdl {

constexpr int kAttnWarps = 10;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kBlockN = 128;
constexpr int kStages = 2;
constexpr int kHeadDim = 128;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;    // + m * 128 (one row tile: + buffer * 128)
constexpr uint32_t kTmemO = 256;  // + m * 128
constexpr uint32_t kTmemP1 = 384; // P of the single-row-tile pipeline (64 columns)
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s per wait
#ifndef FDL_ATTN_PREFETCH
#define FDL_ATTN_PREFETCH 1
#endif
constexpr int kPrefetch = FDL_ATTN_PREFETCH;  // key tiles prefetched into L2 ahead of the smem ring
#ifndef FDL_ATTN_POLY
#define FDL_ATTN_POLY 2
#endif
// Of every 8 exponential pairs of a full key tile of the one-row-tile
// pipeline, kPolyPairs are computed on the FMA pipe (ptx::exp2_poly2) and the
// rest on the special-function unit (measured on B200: +3% on 8-row
// sub-blocks at 2 of 8; the two-row-tile pipeline is 3-9% slower with any
// share, so it keeps every exponential on the special-function unit).
constexpr int kPolyPairs = FDL_ATTN_POLY;

static_assert(kPolyPairs >= 0 && kPolyPairs <= 8, "polynomial share in eighths");
// Pair i of a 16-pair chunk goes to the FMA pipe when (i * kPolyPairs) % 8 <
// kPolyPairs: the chosen pairs are spread evenly through the chunk.
__device__ __forceinline__ constexpr bool poly_pair(int i) { return (i * kPolyPairs) % 8 < kPolyPairs; }
// 2^x of a packed pair, by the polynomial or by two special-function ex2.
template <bool POLY>
__device__ __forceinline__ uint64_t exp2_pair(uint64_t x2) {
  if constexpr (POLY) {
    return ptx::exp2_poly2(x2);
  } else {
    float x0, x1;
    ptx::unpack2(x2, x0, x1);
    return ptx::pack2(ptx::ex2(x0), ptx::ex2(x1));
  }
}

constexpr uint32_t kSmemQ = 0;                        // 2 halves x 256 rows x 128 B
constexpr uint32_t kQHalf = 256 * 128;                // 32 KB
constexpr uint32_t kSmemK = 2 * kQHalf;               // 65536
constexpr uint32_t kKVHalf = kBlockN * 128;           // 16 KB (128 keys x 64 dims)
constexpr uint32_t kKVTile = 2 * kKVHalf;             // 32 KB
constexpr uint32_t kSmemV = kSmemK + kStages * kKVTile;
constexpr uint32_t kSmemBar = kSmemV + kStages * kKVTile;  // 196608
constexpr uint32_t kSmemBytes = kSmemBar + 256 + 1024;     // + barriers + alignment slack

struct AttnParams {
  CUtensorMap tm_q;   // dims (D, Hq, Sq, B), box (64, G, qc, 1)
  CUtensorMap tm_k;   // dims (D, Hkv, cap, B), box (64, 1, 64, 1); (D, cap, Hkv, B) if head-major
  CUtensorMap tm_v;
  CUtensorMap tm_kb;  // dims (D, Hkv, n_blk, B), box (64, 1, 64, 1)
  CUtensorMap tm_vb;
  const int32_t* seqlens;
  const int32_t* q_pos;
  __nv_bfloat16* out;
  float* ws_o;
  float* ws_lse;
  int B, Sq, Hq, Hkv, G, qc, n_qchunks, cap, n_blk, mask_block, splits, n_mt;
  int n_units;                // splits x Hkv x n_qchunks x B work items
  int kv_hmajor, blk_hmajor;  // 1: map dims are (D, S, H, B) (head-major memory)
  float scale_log2;
  int64_t o_sb, o_ss, o_sh;  // elements
};

struct AttnBarriers {
  uint64_t q_full;
  uint64_t q_empty;     // the current item's S MMAs are done: Q may be reloaded
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];   // S_m(j) complete (and with it P_m(j-1) * V_(j-1))
  uint64_t p_full[2];   // P_m(j) written to TMEM (4 warp arrivals)
  uint64_t pv_done[2];  // P_m(j) * V_j complete
  uint64_t s_free[2];   // single row tile: S buffer read by the softmax (4 warp arrivals)
  uint64_t fin;
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(AttnBarriers) <= 256, "barrier block");
static_assert(kSmemBytes <= 227 * 1024, "dynamic shared memory beyond the per-CTA limit");
static_assert(kTmemS + 2 * kBlockN <= kTmemO && kTmemO + 2 * kHeadDim <= kTmemCols, "TMEM: S_0, S_1, O_0, O_1");
// The one-row-tile pipeline's P sits in the columns of O_1 on purpose: with a
// single row tile O_1 is unused.  It must not reach into either S buffer or O_0.
static_assert(kTmemP1 + kBlockN / 2 <= kTmemCols, "TMEM: P of the one-row-tile pipeline");
static_assert(kTmemP1 >= kTmemO + kHeadDim, "TMEM: P of the one-row-tile pipeline overlaps O_0");
static_assert(kTmemP1 >= kTmemS + 2 * kBlockN, "TMEM: P of the one-row-tile pipeline overlaps an S buffer");
static_assert(kAttnWarps == 2 + 2 * 4, "producer, MMA issuer, 4 softmax warps per row tile");
static_assert(kSmemQ % 1024 == 0 && kSmemK % 1024 == 0 && kSmemV % 1024 == 0 && kKVTile % 1024 == 0,
              "128-byte swizzle atoms need 1024-byte aligned tiles");

struct TileInfo {
  int src;    // 0 = cache, 1 = appended block
  int key0;   // first key within its source
  int valid;  // valid keys in this tile
  int kpos0;  // absolute position of key0
};

__device__ __forceinline__ TileInfo tile_info(int i, int n1, int len, int n_blk) {
  TileInfo t;
  if (i < n1) {
    t.src = 0;
    t.key0 = i * kBlockN;
    t.valid = min(kBlockN, len - t.key0);
    t.kpos0 = t.key0;
  } else {
    t.src = 1;
    t.key0 = (i - n1) * kBlockN;
    t.valid = min(kBlockN, n_blk - t.key0);
    t.kpos0 = len + t.key0;
  }
  return t;
}

// One work item: a (sequence, KV head, query chunk, KV split).  Items are
// numbered u = (b * Hkv * n_qchunks + qch * Hkv + g) * splits + split; CTA c
// walks items c, c + gridDim.x, c + 2 * gridDim.x, ... (a persistent grid of
// at most one CTA per SM), so the next item's Q and K/V loads and its first
// MMAs overlap the current item's last tiles and epilogue.
struct WorkItem {
  int b, g, q0, split, len, n1, t_beg, T;
};

__device__ __forceinline__ WorkItem work_item(const AttnParams& p, int u, bool report_len) {
  WorkItem w;
  w.split = u % p.splits;
  const int t = u / p.splits;
  const int ny = p.Hkv * p.n_qchunks;
  const int y = t % ny;
  w.b = t / ny;
  w.g = y % p.Hkv;
  const int qch = y / p.Hkv;
  w.q0 = qch * p.qc;
  int len = p.seqlens[w.b];
  if (len < 0 || len > p.cap) {
    if (report_len && w.g == 0 && qch == 0 && w.split == 0) report(FDL_DEV_LENGTH, len);
    len = len < 0 ? 0 : p.cap;
  }
  w.len = len;
  w.n1 = (len + kBlockN - 1) / kBlockN;
  const int n2 = p.n_blk > 0 ? (p.n_blk + kBlockN - 1) / kBlockN : 0;
  const int n_all = w.n1 + n2;
  const int per = (n_all + p.splits - 1) / p.splits;
  w.t_beg = min(n_all, w.split * per);
  w.T = min(n_all, w.t_beg + per) - w.t_beg;
  return w;
}

// Wait without honouring the abort flag (used only to drain in-flight work).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = ptx::globaltimer();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (ptx::globaltimer() - t0 > kWaitTimeoutNs) break;
  }
}

// kPersistent = true: a grid of at most one CTA per SM, each walking items
// blockIdx.x, blockIdx.x + gridDim.x, ...  false: one CTA per item (the loops
// below then have a trip count of one the compiler can see, and compile to
// straight-line code).
template <bool kPersistent>
__global__ void __launch_bounds__(kAttnThreads, 1) block_attn_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  const int u_end = kPersistent ? p.n_units : static_cast<int>(blockIdx.x) + 1;
  const int u_step = kPersistent ? static_cast<int>(gridDim.x) : 1;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  AttnBarriers* bars = reinterpret_cast<AttnBarriers*>(smem + kSmemBar);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int R = p.G * p.qc;

  if (threadIdx.x == 0) {
    ptx::mbar_init(&bars->q_full, 1);
    ptx::mbar_init(&bars->q_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(&bars->kv_full[s], 1);
      ptx::mbar_init(&bars->kv_empty[s], 1);
    }
    for (int m = 0; m < 2; ++m) {
      ptx::mbar_init(&bars->s_full[m], 1);
      ptx::mbar_init(&bars->p_full[m], 4);
      ptx::mbar_init(&bars->pv_done[m], 1);
      ptx::mbar_init(&bars->s_free[m], 4);
    }
    ptx::mbar_init(&bars->fin, 1);
    bars->abort = 0;
    ptx::fence_mbar_init();
  }
  // Rows of the last MMA tile beyond R are padding: zero them so the padded
  // MMA rows compute on finite data (no Q load ever writes them).
  {
    const int pad0 = R, pad1 = p.n_mt * 128;
    const int n16 = (pad1 - pad0) * 8;  // 16-byte chunks per half
    for (int i = threadIdx.x; i < 2 * n16; i += kAttnThreads) {
      const int half = i / n16, k = i - half * n16;
      *reinterpret_cast<uint4*>(smem + kSmemQ + half * kQHalf + pad0 * 128 + k * 16) = make_uint4(0, 0, 0, 0);
    }
  }
  if (warp == 1) {
    __syncwarp();  // .sync.aligned: the whole warp, converged
    ptx::tmem_alloc(&bars->tmem_base, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------- TMA producer
    if (lane == 0) {
      ptx::prefetch_tmap(&p.tm_q);
      ptx::prefetch_tmap(&p.tm_k);
      ptx::prefetch_tmap(&p.tm_v);
      int gt = 0, nq = 0, issued = 0, q_issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < u_end; u += u_step) {
        const WorkItem it = work_item(p, u, true);
        if (it.T == 0) continue;
        // Q is single-buffered: the previous item's S MMAs must be done.
        if (nq > 0) {
          ok = ptx::mbar_wait(&bars->q_empty, (nq - 1) & 1, abort, kWaitTimeoutNs, 11);
          if (!ok) break;
        }
        const uint32_t qbytes = static_cast<uint32_t>(R) * 128u;
        ptx::mbar_arrive_expect_tx(&bars->q_full, 2 * qbytes);
        ptx::tma_load_4d(smem + kSmemQ, &p.tm_q, &bars->q_full, 0, it.g * p.G, it.q0, it.b);
        ptx::tma_load_4d(smem + kSmemQ + kQHalf, &p.tm_q, &bars->q_full, 64, it.g * p.G, it.q0, it.b);
        q_issued = nq + 1;
        // Tile j's coordinates in its source map.
        const int t_beg = it.t_beg, n1 = it.n1, len = it.len, g = it.g;
        auto coords = [=, &p](int j, const CUtensorMap*& tk, const CUtensorMap*& tv, int& c1, int& c2) {
          const TileInfo ti = tile_info(t_beg + j, n1, len, p.n_blk);
          tk = ti.src ? &p.tm_kb : &p.tm_k;
          tv = ti.src ? &p.tm_vb : &p.tm_v;
          const bool hm = ti.src ? p.blk_hmajor : p.kv_hmajor;
          c1 = hm ? ti.key0 : g;
          c2 = hm ? g : ti.key0;
        };
        for (int j = 0; j < it.T; ++j, ++gt) {
          const int st = gt % kStages;
          // L2 prefetch of the tile that will next use this stage.
          if (kPrefetch > 0 && j + kStages < it.T) {
            const CUtensorMap *tk, *tv;
            int c1, c2;
            coords(j + kStages, tk, tv, c1, c2);
            ptx::tma_prefetch_l2_4d(tk, 0, c1, c2, it.b);
            ptx::tma_prefetch_l2_4d(tk, 64, c1, c2, it.b);
            ptx::tma_prefetch_l2_4d(tv, 0, c1, c2, it.b);
            ptx::tma_prefetch_l2_4d(tv, 64, c1, c2, it.b);
          }
          if (gt >= kStages) {
            ok = ptx::mbar_wait(&bars->kv_empty[st], ((gt / kStages) - 1) & 1, abort, kWaitTimeoutNs, 1);
            if (!ok) break;
          }
          const CUtensorMap *tk, *tv;
          int c1, c2;
          coords(j, tk, tv, c1, c2);
          uint8_t* ks = smem + kSmemK + st * kKVTile;
          uint8_t* vs = smem + kSmemV + st * kKVTile;
          ptx::mbar_arrive_expect_tx(&bars->kv_full[st], 2 * kKVTile);
          ptx::tma_load_4d(ks, tk, &bars->kv_full[st], 0, c1, c2, it.b);
          ptx::tma_load_4d(ks + kKVHalf, tk, &bars->kv_full[st], 64, c1, c2, it.b);
          ptx::tma_load_4d(vs, tv, &bars->kv_full[st], 0, c1, c2, it.b);
          ptx::tma_load_4d(vs + kKVHalf, tv, &bars->kv_full[st], 64, c1, c2, it.b);
          issued = gt + 1;
        }
        ++nq;
      }
      if (*abort) {
        // Let every copy already in flight land before the CTA exits.
        if (q_issued > 0) drain_wait(&bars->q_full, (q_issued - 1) & 1);
        for (int g = max(0, issued - kStages); g < issued; ++g) drain_wait(&bars->kv_full[g % kStages], (g / kStages) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = ptx::idesc_bf16_f32(128, kBlockN, false);
      const uint32_t idesc_o = ptx::idesc_bf16_f32(128, kHeadDim, true);
      // Base descriptors built once; the (16-byte-unit) address field is
      // advanced by compile-time offsets in the issue loops.
      const uint64_t q_desc = ptx::smem_desc_sw128(ptx::smem_u32(smem + kSmemQ), 16, 1024);
      const uint64_t k_desc = ptx::smem_desc_sw128(ptx::smem_u32(smem + kSmemK), 16, 1024);
      const uint64_t v_desc = ptx::smem_desc_sw128(ptx::smem_u32(smem + kSmemV), kKVHalf, 1024);
      // S_m = Q_m * K_st^T: 8 MMAs of K = 16 over the 128 head dims.
      auto issue_s = [&](int m, int st) {
        const uint32_t d = tmem + kTmemS + m * kBlockN;
        const uint64_t qa = q_desc + static_cast<uint64_t>(m) * (128 * 128 / 16);
        const uint64_t kb = k_desc + static_cast<uint64_t>(st) * (kKVTile / 16);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          // K=16 slice kk: 32 bytes into the 128-byte swizzle row of its half.
          ptx::mma_bf16_ss(d, qa + ((kk >> 2) * kQHalf + (kk & 3) * 32) / 16,
                           kb + ((kk >> 2) * kKVHalf + (kk & 3) * 32) / 16, idesc_s, kk > 0);
        }
      };
      // O_m += P_m * V_st: 8 MMAs of K = 16 over the 128 keys.  P_m is read
      // from TMEM (8 packed columns per 16 keys); V is MN-major (head dim
      // contiguous): LBO = distance between the two 64-dim halves,
      // SBO = 8 keys x 128 B.
      auto issue_pv = [&](int m, int st, bool acc) {
        const uint32_t d = tmem + kTmemO + m * kHeadDim;
        const uint32_t a = tmem + kTmemS + m * kBlockN;
        const uint64_t vb = v_desc + static_cast<uint64_t>(st) * (kKVTile / 16);
#pragma unroll
        for (int kk = 0; kk < kBlockN / 16; ++kk)
          ptx::mma_bf16_ts(d, a + kk * 8, vb + (kk * 16 * 128) / 16, idesc_o, (acc || kk > 0) ? 1u : 0u);
      };
      // One row tile: S in buffer buf, P in its own columns.
      auto issue_s1 = [&](int buf, int st) {
        const uint32_t d = tmem + kTmemS + buf * kBlockN;
        const uint64_t kb = k_desc + static_cast<uint64_t>(st) * (kKVTile / 16);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          ptx::mma_bf16_ss(d, q_desc + ((kk >> 2) * kQHalf + (kk & 3) * 32) / 16,
                           kb + ((kk >> 2) * kKVHalf + (kk & 3) * 32) / 16, idesc_s, kk > 0);
      };
      auto issue_pv1 = [&](int st, bool acc) {
        const uint64_t vb = v_desc + static_cast<uint64_t>(st) * (kKVTile / 16);
#pragma unroll
        for (int kk = 0; kk < kBlockN / 16; ++kk)
          ptx::mma_bf16_ts(tmem + kTmemO, tmem + kTmemP1 + kk * 8, vb + (kk * 16 * 128) / 16, idesc_o,
                           (acc || kk > 0) ? 1u : 0u);
      };
      // This CTA's tiles and non-empty items over all its work items: a K/V
      // stage is released only if a later tile refills it, and q_empty is
      // committed only if a later item reloads Q (no asynchronous arrive may
      // still be pending when the CTA exits).
      int total = 0, n_items = 0;
      for (int u = blockIdx.x; u < u_end; u += u_step) {
        const int t = work_item(p, u, false).T;
        total += t;
        n_items += t > 0 ? 1 : 0;
      }
      int gt = 0, nq = 0;
      bool ok = true, issued_any = false;
      for (int u = blockIdx.x; ok && u < u_end; u += u_step) {
        const int T = work_item(p, u, false).T;
        if (T == 0) continue;
        const int g0 = gt;
        const bool reload_q = nq + 1 < n_items;
        ok = ptx::mbar_wait(&bars->q_full, nq & 1, abort, kWaitTimeoutNs, 2) &&
             ptx::mbar_wait(&bars->kv_full[g0 % kStages], (g0 / kStages) & 1, abort, kWaitTimeoutNs, 3);
        if (!ok) break;
        ptx::tc_fence_after();
        if (p.n_mt == 1) {
          // One row tile (R <= 128: sub-block rows, small GQA groups): S is
          // double-buffered in the TMEM the second tile would use and P has
          // its own columns, so S(g+1) is computed while the softmax works on
          // S(g) instead of after P(g) * V_g.  S(g) reuses the buffer of
          // S(g-2): the softmax must have read it.
          if (g0 >= 2) {
            ok = ptx::mbar_wait(&bars->s_free[g0 & 1], ((g0 - 2) >> 1) & 1, abort, kWaitTimeoutNs, 5);
            if (!ok) break;
            ptx::tc_fence_after();
          }
          issue_s1(g0 & 1, g0 % kStages);
          ptx::mma_commit(&bars->s_full[g0 & 1]);
          issued_any = true;
          if (T == 1 && reload_q) ptx::mma_commit(&bars->q_empty);
          for (int j = 0; ok && j < T; ++j) {
            const int g = g0 + j;
            const int st = g % kStages;
            if (j + 1 < T) {
              ok = ptx::mbar_wait(&bars->kv_full[(g + 1) % kStages], ((g + 1) / kStages) & 1, abort,
                                  kWaitTimeoutNs, 4);
              if (ok && g >= 1)
                ok = ptx::mbar_wait(&bars->s_free[(g + 1) & 1], ((g - 1) >> 1) & 1, abort, kWaitTimeoutNs, 5);
              if (!ok) break;
              ptx::tc_fence_after();
              issue_s1((g + 1) & 1, (g + 1) % kStages);
              ptx::mma_commit(&bars->s_full[(g + 1) & 1]);
              if (j + 1 == T - 1 && reload_q) ptx::mma_commit(&bars->q_empty);
            }
            ok = ptx::mbar_wait(&bars->p_full[0], g & 1, abort, kWaitTimeoutNs, 6);
            if (!ok) break;
            ptx::tc_fence_after();
            // The item's first P * V starts O afresh: every softmax warp read
            // the previous item's O before it arrived on this p_full.
            issue_pv1(st, j > 0);
            ptx::mma_commit(&bars->pv_done[0]);
            if (g + kStages < total) ptx::mma_commit(&bars->kv_empty[st]);
          }
        } else {
          // S_m(g0) overwrites P_m(g0 - 1) of the previous item: wait until
          // that P * V has completed.
          for (int m = 0; ok && m < p.n_mt; ++m) {
            if (g0 > 0) {
              ok = ptx::mbar_wait(&bars->pv_done[m], (g0 - 1) & 1, abort, kWaitTimeoutNs, 5);
              if (!ok) break;
              ptx::tc_fence_after();
            }
            issue_s(m, g0 % kStages);
            ptx::mma_commit(&bars->s_full[m]);
            issued_any = true;
          }
          if (!ok) break;
          if (T == 1 && reload_q) ptx::mma_commit(&bars->q_empty);
          for (int j = 0; ok && j < T; ++j) {
            const int g = g0 + j;
            const int st = g % kStages;
            const bool nxt = j + 1 < T;
            for (int m = 0; ok && m < p.n_mt; ++m) {
              ok = ptx::mbar_wait(&bars->p_full[m], g & 1, abort, kWaitTimeoutNs, 6);
              if (!ok) break;
              ptx::tc_fence_after();
              issue_pv(m, st, j > 0);
              ptx::mma_commit(&bars->pv_done[m]);
              // Stage st is free once the last row tile's P * V_g completes.
              if (m == p.n_mt - 1 && g + kStages < total) ptx::mma_commit(&bars->kv_empty[st]);
              if (nxt) {
                if (m == 0) {
                  ok = ptx::mbar_wait(&bars->kv_full[(g + 1) % kStages], ((g + 1) / kStages) & 1, abort,
                                      kWaitTimeoutNs, 4);
                  if (!ok) break;
                }
                // S_m(g+1) overwrites P_m(g), which P_m(g) * V_g (issued
                // just before by this thread) reads: issued in order behind it.
                issue_s(m, (g + 1) % kStages);
                ptx::mma_commit(&bars->s_full[m]);
                if (m == p.n_mt - 1 && j + 1 == T - 1 && reload_q) ptx::mma_commit(&bars->q_empty);
              }
            }
          }
        }
        gt += T;
        ++nq;
      }
      if (issued_any && !ok) {
        ptx::mma_commit(&bars->fin);
        drain_wait(&bars->fin, 0);
      }
    }
  } else if (warp >= 2 && (warp - 2) / 4 < p.n_mt) {
    // ------------------------------------------------------- softmax
    const int m = (warp - 2) >> 2;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const int r = m * 128 + row;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_off + kTmemS + m * kBlockN;
    const uint32_t t_o = tmem + lane_off + kTmemO + m * kHeadDim;
    int gt = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < u_end; u += u_step) {
    const WorkItem it = work_item(p, u, false);
    const int T = it.T;
    const int sq_i = r / p.G;
    const bool valid_row = (r < R) && (it.q0 + sq_i < p.Sq);
    // A warp whose 32 rows are all padding has nothing to compute: its P
    // lanes feed only O rows that are never stored, so it just keeps the
    // barrier phases (and leaves its SM sub-partition to the other warps).
    const bool pad_warp = __all_sync(0xffffffffu, !valid_row);
    // Block-causal mask as a key-position bound: key position kp is visible
    // iff kp / mask_block <= qpos / mask_block, i.e. kp < kpos_end.
    int kpos_end = 0x7fffffff;
    if (p.mask_block > 0 && valid_row) {
      const int q = it.q0 + sq_i;
      const int qpos = p.q_pos ? p.q_pos[static_cast<int64_t>(it.b) * p.Sq + q] : it.len + q;
      kpos_end = (qpos / p.mask_block + 1) * p.mask_block;
    }
    float m_used = -INFINITY, l = 0.f;
    if (p.n_mt == 1) {
      // Single row tile: S(g) in buffer g & 1, P in its own columns.
      const uint32_t t_p = tmem + lane_off + kTmemP1;
      const uint64_t sc2 = ptx::pack2(p.scale_log2, p.scale_log2);
      for (int j = 0; j < T; ++j) {
        const int g = gt + j;
        const int buf = g & 1;
        ok = __all_sync(0xffffffffu, ptx::mbar_wait(&bars->s_full[buf], (g >> 1) & 1, abort, kWaitTimeoutNs, 7));
        if (!ok) break;
        ptx::tc_fence_after();
        if (pad_warp) {
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&bars->s_free[buf]);
          // S(g+1) may be ready long before the other warps finish P(g), so a
          // padding warp takes its p_full turn for tile g only after
          // P(g-1) * V_(g-1) has completed -- i.e. after every warp arrived
          // for tile g-1.  Arriving earlier could complete phase g with this
          // warp's arrivals for g and g+1 (an early P * V, then phases out of
          // step).
          if (g > 0) {
            ok = __all_sync(0xffffffffu,
                            ptx::mbar_wait(&bars->pv_done[0], (g - 1) & 1, abort, kWaitTimeoutNs, 10));
            if (!ok) break;
          }
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(&bars->p_full[0]);
          continue;
        }
        const uint32_t t_sb = tmem + lane_off + kTmemS + buf * kBlockN;
        const TileInfo ti = tile_info(it.t_beg + j, it.n1, it.len, p.n_blk);
        const int climit = valid_row ? max(0, min(ti.valid, kpos_end - ti.kpos0)) : kBlockN;
        const bool full = __all_sync(0xffffffffu, climit == kBlockN);
        // Max of 64 columns [c0, c0 + 64) held in lo / hi.
        auto half_max = [&](const float (&lo)[32], const float (&hi)[32], int c0) {
          float mx = -INFINITY;
          if (full) {
            float a0 = lo[0], a1 = hi[0];
#pragma unroll
            for (int i = 1; i < 31; i += 2) {
              a0 = ptx::fmax3(a0, lo[i], lo[i + 1]);
              a1 = ptx::fmax3(a1, hi[i], hi[i + 1]);
            }
            mx = ptx::fmax3(a0, a1, fmaxf(lo[31], hi[31]));
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (c0 + i < climit) mx = fmaxf(mx, lo[i]);
              if (c0 + 32 + i < climit) mx = fmaxf(mx, hi[i]);
            }
          }
          return mx;
        };
        float sa[32], sb[32];
        ptx::tmem_ld32(t_sb + 64, sa);
        ptx::tmem_ld32(t_sb + 96, sb);
        ptx::tmem_wait_ld();
        float tmax = half_max(sa, sb, 64);
        ptx::tmem_ld32(t_sb + 0, sa);
        ptx::tmem_ld32(t_sb + 32, sb);
        ptx::tmem_wait_ld();
        tmax = fmaxf(tmax, half_max(sa, sb, 0));
        tmax *= p.scale_log2;
        const float m_new = fmaxf(m_used, tmax);
        const bool grow = m_new > m_used + 8.f;
        const bool rescale = grow && (m_used != -INFINITY) && j > 0;
        const float alpha = rescale ? ptx::ex2(m_used - m_new) : 1.f;
        if (grow) {
          l = (m_used == -INFINITY) ? 0.f : l * alpha;
          m_used = m_new;
        }
        // P and O are in use by P(j-1) * V_(j-1) until it completes.
        if (g > 0) {
          ok = __all_sync(0xffffffffu, ptx::mbar_wait(&bars->pv_done[0], (g - 1) & 1, abort, kWaitTimeoutNs, 8));
          if (!ok) break;
          ptx::tc_fence_after();
        }
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
          for (int ch = 0; ch < 4; ++ch) {
            float o[32];
            ptx::tmem_ld32(t_o + ch * 32, o);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            ptx::tmem_st32(t_o + ch * 32, o);
          }
        }
        const float neg_m = -m_used;
        const uint64_t nm2 = ptx::pack2(neg_m, neg_m);
        uint64_t acc2 = ptx::pack2(0.f, 0.f);
        float rsum = 0.f;
        auto emit = [&](const float (&sv)[32], int c) {
          uint32_t pk[16];
          if (full) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const uint64_t x2 = ptx::fma2(ptx::pack2(sv[2 * i], sv[2 * i + 1]), sc2, nm2);
              const uint64_t e2 = poly_pair(i) ? exp2_pair<true>(x2) : exp2_pair<false>(x2);
              acc2 = ptx::add2(acc2, e2);
              float p0, p1;
              ptx::unpack2(e2, p0, p1);
              const __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
              pk[i] = *reinterpret_cast<const uint32_t*>(&h);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int k0 = c * 32 + 2 * i;
              const float p0 = (k0 < climit) ? ptx::ex2(__fmaf_rn(sv[2 * i], p.scale_log2, neg_m)) : 0.f;
              const float p1 = (k0 + 1 < climit) ? ptx::ex2(__fmaf_rn(sv[2 * i + 1], p.scale_log2, neg_m)) : 0.f;
              rsum += p0 + p1;
              const __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
              pk[i] = *reinterpret_cast<const uint32_t*>(&h);
            }
          }
          ptx::tmem_st16(t_p + c * 16, pk);
        };
        emit(sa, 0);
        emit(sb, 1);
        ptx::tmem_ld32(t_sb + 64, sa);
        ptx::tmem_ld32(t_sb + 96, sb);
        ptx::tmem_wait_ld();
        // Every column of S(j) is in registers: its buffer may take S(j+2).
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars->s_free[buf]);
        emit(sa, 2);
        emit(sb, 3);
        float s0, s1;
        ptx::unpack2(acc2, s0, s1);
        l += rsum + (s0 + s1);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars->p_full[0]);
      }
    }
    for (int j = 0; ok && p.n_mt > 1 && j < T; ++j) {
      const int g = gt + j;
      // S_m(g) ready (and P_m(g-1) * V_(g-1) done: O_m is stable).
      ok = __all_sync(0xffffffffu, ptx::mbar_wait(&bars->s_full[m], g & 1, abort, kWaitTimeoutNs, 7));
      if (!ok) break;
      ptx::tc_fence_after();
      if (pad_warp) {
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars->p_full[m]);
        continue;
      }
      const TileInfo ti = tile_info(it.t_beg + j, it.n1, it.len, p.n_blk);
      // Visible keys of this tile for this row form a prefix of the tile.
      // Padding rows (beyond the R real rows, or past the last query) count
      // as fully visible: their results are never stored, and this keeps
      // whole warps of padding rows on the unpredicated path.
      const int climit = valid_row ? max(0, min(ti.valid, kpos_end - ti.kpos0)) : kBlockN;
      // The S row is read in halves of 64 columns so no more than 64 values
      // are live: the upper half (keys 64..127) is read first for its max,
      // then the lower half, which stays in registers; after the lower
      // half's P is written (over S columns 0..31, already consumed) the
      // upper half is read again.
      const bool full = __all_sync(0xffffffffu, climit == kBlockN);
      float sa[32], sb[32];
      // Max of 64 columns [c0, c0 + 64) held in lo / hi.
      auto half_max = [&](const float (&lo)[32], const float (&hi)[32], int c0) {
        float mx = -INFINITY;
        if (full) {
          float a0 = lo[0], a1 = hi[0];
#pragma unroll
          for (int i = 1; i < 31; i += 2) {
            a0 = ptx::fmax3(a0, lo[i], lo[i + 1]);
            a1 = ptx::fmax3(a1, hi[i], hi[i + 1]);
          }
          mx = ptx::fmax3(a0, a1, fmaxf(lo[31], hi[31]));
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (c0 + i < climit) mx = fmaxf(mx, lo[i]);
            if (c0 + 32 + i < climit) mx = fmaxf(mx, hi[i]);
          }
        }
        return mx;
      };
      ptx::tmem_ld32(t_s + 64, sa);
      ptx::tmem_ld32(t_s + 96, sb);
      ptx::tmem_wait_ld();
      float tmax = half_max(sa, sb, 64);
      ptx::tmem_ld32(t_s + 0, sa);
      ptx::tmem_ld32(t_s + 32, sb);
      ptx::tmem_wait_ld();
      tmax = fmaxf(tmax, half_max(sa, sb, 0));
      tmax *= p.scale_log2;  // scale > 0: max commutes with the scaling
      const float m_new = fmaxf(m_used, tmax);
      const bool grow = m_new > m_used + 8.f;  // true on the first finite max
      const bool rescale = grow && (m_used != -INFINITY) && j > 0;
      if (__any_sync(0xffffffffu, rescale)) {
        const float alpha = rescale ? ptx::ex2(m_used - m_new) : 1.f;
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          float o[32];
          ptx::tmem_ld32(t_o + ch * 32, o);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          ptx::tmem_st32(t_o + ch * 32, o);
        }
      }
      if (grow) {
        l = (m_used == -INFINITY) ? 0.f : l * ptx::ex2(m_used - m_new);
        m_used = m_new;
      }
      // P = exp2(S * scale - max) as bf16, packed two per column into the
      // first 64 columns of S_m (already read into registers).
      float rsum = 0.f;
      const float neg_m = -m_used;
      if (full) {
        // Packed pairs: x = S * scale - max by one f32x2 FMA, 2^x from the
        // special-function unit, the row sum by f32x2 adds.
        const uint64_t sc2 = ptx::pack2(p.scale_log2, p.scale_log2);
        const uint64_t nm2 = ptx::pack2(neg_m, neg_m);
        uint64_t acc2 = ptx::pack2(0.f, 0.f);
        auto emit_full = [&](const float (&sv)[32], int c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint64_t x2 = ptx::fma2(ptx::pack2(sv[2 * i], sv[2 * i + 1]), sc2, nm2);
            const uint64_t e2 = exp2_pair<false>(x2);
            acc2 = ptx::add2(acc2, e2);
            float p0, p1;
            ptx::unpack2(e2, p0, p1);
            const __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
            pk[i] = *reinterpret_cast<const uint32_t*>(&h);
          }
          ptx::tmem_st16(t_s + c * 16, pk);
        };
        emit_full(sa, 0);
        emit_full(sb, 1);
        ptx::tmem_ld32(t_s + 64, sa);
        ptx::tmem_ld32(t_s + 96, sb);
        ptx::tmem_wait_ld();
        emit_full(sa, 2);
        emit_full(sb, 3);
        float s0, s1;
        ptx::unpack2(acc2, s0, s1);
        rsum = s0 + s1;
      } else {
        auto emit = [&](const float (&sv)[32], int c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int k0 = c * 32 + 2 * i;
            const float p0 = (k0 < climit) ? ptx::ex2(__fmaf_rn(sv[2 * i], p.scale_log2, neg_m)) : 0.f;
            const float p1 = (k0 + 1 < climit) ? ptx::ex2(__fmaf_rn(sv[2 * i + 1], p.scale_log2, neg_m)) : 0.f;
            rsum += p0 + p1;
            const __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
            pk[i] = *reinterpret_cast<const uint32_t*>(&h);
          }
          ptx::tmem_st16(t_s + c * 16, pk);
        };
        emit(sa, 0);
        emit(sb, 1);
        ptx::tmem_ld32(t_s + 64, sa);
        ptx::tmem_ld32(t_s + 96, sb);
        ptx::tmem_wait_ld();
        emit(sa, 2);
        emit(sb, 3);
      }
      l += rsum;
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars->p_full[m]);
    }
    // The item's output coordinates, recomputed here rather than kept live
    // through the tile loops.
    const WorkItem ie = work_item(p, u, false);
    const int q = ie.q0 + sq_i;
    const int head = ie.g * p.G + (r - sq_i * p.G);
    bool have_o = ok && T > 0;
    if (have_o) {
      have_o = __all_sync(0xffffffffu, ptx::mbar_wait(&bars->pv_done[m], (gt + T - 1) & 1, abort, kWaitTimeoutNs, 9));
      ptx::tc_fence_after();
    }
    const float inv_l = (l > 0.f) ? 1.f / l : 0.f;
    if (p.splits == 1) {
      __nv_bfloat16* orow = p.out + ie.b * p.o_sb + static_cast<int64_t>(q) * p.o_ss + static_cast<int64_t>(head) * p.o_sh;
#pragma unroll 1
      for (int ch = 0; ch < 4; ++ch) {
        float o[32];
        if (have_o) {
          ptx::tmem_ld32(t_o + ch * 32, o);
          ptx::tmem_wait_ld();
        }
        if (valid_row) {
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float a0 = (have_o && l > 0.f) ? o[2 * i] * inv_l : 0.f;
            const float a1 = (have_o && l > 0.f) ? o[2 * i + 1] * inv_l : 0.f;
            const __nv_bfloat162 h = __floats2bfloat162_rn(a0, a1);
            w[i] = *reinterpret_cast<const uint32_t*>(&h);
          }
          uint4* dst = reinterpret_cast<uint4*>(orow + ch * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    } else {
      const int64_t rows = static_cast<int64_t>(p.B) * p.Sq * p.Hq;
      const int64_t wrow = static_cast<int64_t>(ie.split) * rows + (static_cast<int64_t>(ie.b) * p.Sq + q) * p.Hq + head;
#pragma unroll 1
      for (int ch = 0; ch < 4; ++ch) {
        float o[32];
        if (have_o) {
          ptx::tmem_ld32(t_o + ch * 32, o);
          ptx::tmem_wait_ld();
        }
        if (valid_row) {
          float4* dst = reinterpret_cast<float4*>(p.ws_o + wrow * kHeadDim + ch * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const bool live = have_o && l > 0.f;
            dst[i] = make_float4(live ? o[4 * i] * inv_l : 0.f, live ? o[4 * i + 1] * inv_l : 0.f,
                                 live ? o[4 * i + 2] * inv_l : 0.f, live ? o[4 * i + 3] * inv_l : 0.f);
          }
        }
      }
      if (valid_row) p.ws_lse[wrow] = (have_o && l > 0.f) ? m_used + __log2f(l) : -INFINITY;
    }
    gt += T;
    }  // work items
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// Merge split-KV partials: one warp per output row, 4 head dims per lane.
__global__ void __launch_bounds__(256) attn_combine_kernel(const float* __restrict__ ws_o,
                                                           const float* __restrict__ ws_lse,
                                                           __nv_bfloat16* __restrict__ out, int splits, int B,
                                                           int Sq, int Hq, int64_t o_sb, int64_t o_ss,
                                                           int64_t o_sh) {
  const int64_t rows = static_cast<int64_t>(B) * Sq * Hq;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, ws_lse[s * rows + row]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float den = 0.f;
  if (mx != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const float lse = ws_lse[s * rows + row];
      if (lse == -INFINITY) continue;
      const float w = ptx::ex2(lse - mx);
      const float4 o = reinterpret_cast<const float4*>(ws_o + (s * rows + row) * kHeadDim)[lane];
      acc.x += w * o.x;
      acc.y += w * o.y;
      acc.z += w * o.z;
      acc.w += w * o.w;
      den += w;
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  const int64_t h = row % Hq;
  const int64_t bq = row / Hq;
  const int64_t q = bq % Sq;
  const int64_t b = bq / Sq;
  __nv_bfloat16* o = out + b * o_sb + q * o_ss + h * o_sh + lane * 4;
  const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
  const __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
  uint2 v;
  v.x = *reinterpret_cast<const uint32_t*>(&lo);
  v.y = *reinterpret_cast<const uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(o) = v;
}

}  // namespace fdl
