// torch.library registration of the fdl_b200 C ABI (namespace `fdl`).
//
// Every op launches on torch's current CUDA stream, allocates nothing except
// where the schema returns a new tensor (flash_kvcache), and has a Meta
// implementation so torch.compile(fullgraph=True) and CUDA-graph capture can
// trace through it -- the same contract as the custom-op wrapper around
// flash_attn_with_kvcache in utils/attention_backends.py:73-120.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <vector>

#include "../../include/fdl_kvcache.h"

namespace {

using at::Tensor;

fdl_stream_t cur_stream() { return reinterpret_cast<fdl_stream_t>(at::cuda::getCurrentCUDAStream().stream()); }

void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == 0, "fdl_b200 ", what, " failed: ",
              rc > 0 ? (rc == FDL_E_NULL        ? "null pointer"
                        : rc == FDL_E_SHAPE     ? "unsupported shape"
                        : rc == FDL_E_ALIGN     ? "pointer/stride not aligned for vector access"
                        : rc == FDL_E_DTYPE     ? "unsupported dtype"
                        : rc == FDL_E_WORKSPACE ? "workspace too small"
                        : rc == FDL_E_NODEVICE  ? "device / driver entry point unavailable"
                                                : "unsupported configuration")
                     : "CUDA launch error",
              " (code ", rc, ")");
}

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "fdl: ", name, " must be a CUDA tensor");
  TORCH_CHECK(t.stride(-1) == 1, "fdl: ", name, " must be contiguous in its last dimension");
}

int elem_bytes(const Tensor& t) {
  const auto st = t.scalar_type();
  TORCH_CHECK(st == at::kBFloat16 || st == at::kHalf || st == at::kFloat, "fdl: unsupported dtype ", st);
  return static_cast<int>(t.element_size());
}

int dtype_code(const Tensor& t) {
  switch (t.scalar_type()) {
    case at::kBFloat16: return FDL_BF16;
    case at::kHalf: return FDL_F16;
    case at::kFloat: return FDL_F32;
    default: TORCH_CHECK(false, "fdl: unsupported dtype ", t.scalar_type());
  }
}

// View a 3-D [B, S, X] or 4-D [B, S, H, D] / [B, H, S, D] tensor as
// (batch, seq, heads, dim) sizes and strides; seq_dim selects 1 or 2.
struct Rows {
  int64_t B, S, H, D, sb, ss, sh;
};
Rows rows_of(const Tensor& t, int64_t seq_dim) {
  Rows r{};
  if (t.dim() == 3) {
    TORCH_CHECK(seq_dim == 1, "fdl: 3-D tensors use seq_dim 1");
    r = {t.size(0), t.size(1), 1, t.size(2), t.stride(0), t.stride(1), t.size(2)};
  } else {
    TORCH_CHECK(t.dim() == 4, "fdl: expected a 3-D or 4-D tensor, got ", t.dim(), "-D");
    TORCH_CHECK(seq_dim == 1 || seq_dim == 2, "fdl: seq_dim must be 1 or 2");
    const int64_t hd = seq_dim == 1 ? 2 : 1;
    r = {t.size(0), t.size(seq_dim), t.size(hd), t.size(3), t.stride(0), t.stride(seq_dim), t.stride(hd)};
  }
  return r;
}

// ---------------------------------------------------------------- (a)
void kv_append(at::TensorList k_caches, at::TensorList v_caches, at::TensorList k_srcs, at::TensorList v_srcs,
               const Tensor& start_pos) {
  const int64_t L = static_cast<int64_t>(k_caches.size());
  TORCH_CHECK(L >= 1 && L <= FDL_MAX_LAYERS, "fdl.kv_append: 1..", FDL_MAX_LAYERS, " layers per call");
  TORCH_CHECK(v_caches.size() == k_caches.size() && k_srcs.size() == k_caches.size() &&
                  v_srcs.size() == k_caches.size(),
              "fdl.kv_append: list lengths differ");
  TORCH_CHECK(start_pos.is_cuda() && start_pos.scalar_type() == at::kInt && start_pos.dim() == 1 &&
                  start_pos.is_contiguous(),
              "fdl.kv_append: start_pos must be a contiguous CUDA int32 [B] tensor");
  const Tensor& c0 = k_caches[0];
  const Tensor& s0 = k_srcs[0];
  TORCH_CHECK(c0.dim() == 4 && s0.dim() == 4, "fdl.kv_append: cache and source are [B, S, H, D]");
  TORCH_CHECK(c0.size(0) == s0.size(0) && c0.size(2) == s0.size(2) && c0.size(3) == s0.size(3),
              "fdl.kv_append: cache ", c0.sizes(), " vs source ", s0.sizes());
  TORCH_CHECK(start_pos.size(0) == c0.size(0), "fdl.kv_append: start_pos has ", start_pos.size(0), " rows");
  void* kc[FDL_MAX_LAYERS];
  void* vc[FDL_MAX_LAYERS];
  const void* ks[FDL_MAX_LAYERS];
  const void* vs[FDL_MAX_LAYERS];
  for (int64_t l = 0; l < L; ++l) {
    for (const Tensor* t : {&k_caches[l], &v_caches[l]}) {
      check_cuda(*t, "cache");
      TORCH_CHECK(t->sizes() == c0.sizes() && t->strides() == c0.strides() && t->dtype() == c0.dtype(),
                  "fdl.kv_append: all caches must share shape, strides and dtype");
    }
    for (const Tensor* t : {&k_srcs[l], &v_srcs[l]}) {
      check_cuda(*t, "source");
      TORCH_CHECK(t->sizes() == s0.sizes() && t->strides() == s0.strides() && t->dtype() == c0.dtype(),
                  "fdl.kv_append: all sources must share shape, strides and the cache dtype");
    }
    kc[l] = k_caches[l].data_ptr();
    vc[l] = v_caches[l].data_ptr();
    ks[l] = k_srcs[l].data_ptr();
    vs[l] = v_srcs[l].data_ptr();
  }
  c10::cuda::CUDAGuard guard(c0.device());
  check_rc(fdl_kv_append(kc, vc, ks, vs, static_cast<int>(L), start_pos.data_ptr<int32_t>(),
                         static_cast<int>(c0.size(0)), static_cast<int>(s0.size(1)), static_cast<int>(c0.size(1)),
                         static_cast<int>(c0.size(2)), static_cast<int>(c0.size(3)), elem_bytes(c0), c0.stride(0),
                         c0.stride(1), c0.stride(2), s0.stride(0), s0.stride(1), s0.stride(2), cur_stream()),
           "kv_append");
}

void kv_scatter(const Tensor& k_dst, const std::optional<Tensor>& v_dst, const Tensor& k_src,
                const std::optional<Tensor>& v_src, const Tensor& positions, int64_t seq_dim) {
  check_cuda(k_dst, "k_dst");
  check_cuda(k_src, "k_src");
  TORCH_CHECK(v_dst.has_value() == v_src.has_value(), "fdl.kv_scatter: v_dst and v_src go together");
  TORCH_CHECK(positions.is_cuda() && positions.scalar_type() == at::kLong && positions.dim() == 2 &&
                  positions.stride(1) == 1,
              "fdl.kv_scatter: positions must be a CUDA int64 [B, n] tensor with unit inner stride");
  const Rows d = rows_of(k_dst, seq_dim), s = rows_of(k_src, seq_dim);
  TORCH_CHECK(d.B == s.B && d.H == s.H && d.D == s.D && k_dst.dtype() == k_src.dtype(),
              "fdl.kv_scatter: dst ", k_dst.sizes(), " vs src ", k_src.sizes());
  TORCH_CHECK(positions.size(0) == s.B && positions.size(1) == s.S, "fdl.kv_scatter: positions ",
              positions.sizes(), " must be [B, n] = [", s.B, ", ", s.S, "]");
  if (v_dst) {
    check_cuda(*v_dst, "v_dst");
    check_cuda(*v_src, "v_src");
    TORCH_CHECK(v_dst->sizes() == k_dst.sizes() && v_dst->strides() == k_dst.strides() &&
                    v_src->sizes() == k_src.sizes() && v_src->strides() == k_src.strides() &&
                    v_dst->dtype() == k_dst.dtype() && v_src->dtype() == k_dst.dtype(),
                "fdl.kv_scatter: V tensors must match K tensors");
  }
  c10::cuda::CUDAGuard guard(k_dst.device());
  check_rc(fdl_kv_scatter(k_dst.data_ptr(), v_dst ? v_dst->data_ptr() : nullptr, k_src.data_ptr(),
                          v_src ? v_src->data_ptr() : nullptr, positions.data_ptr<int64_t>(), positions.stride(0),
                          static_cast<int>(s.B), static_cast<int>(s.S), static_cast<int>(d.S), static_cast<int>(d.H),
                          static_cast<int>(d.D), elem_bytes(k_dst), d.sb, d.ss, d.sh, s.sb, s.ss, s.sh, cur_stream()),
           "kv_scatter");
}

// ---------------------------------------------------------------- (b)
void kv_gather_prefix(const Tensor& k_prefix, const Tensor& v_prefix, const Tensor& lens,
                      const std::optional<Tensor>& k_block, const std::optional<Tensor>& v_block, int64_t rep,
                      const Tensor& k_out, const Tensor& v_out, const std::optional<Tensor>& cu_seqlens,
                      int64_t seq_dim_in, int64_t seq_dim_out) {
  for (const Tensor* t : {&k_prefix, &v_prefix, &k_out, &v_out}) check_cuda(*t, "gather tensor");
  TORCH_CHECK(lens.is_cuda() && lens.scalar_type() == at::kInt && lens.is_contiguous(),
              "fdl.kv_gather_prefix: lens must be a contiguous CUDA int32 [B] tensor");
  if (k_out.numel() == 0) return;  // every sequence empty: nothing to write
  const Rows p = rows_of(k_prefix, seq_dim_in);
  TORCH_CHECK(v_prefix.sizes() == k_prefix.sizes() && v_prefix.strides() == k_prefix.strides(),
              "fdl.kv_gather_prefix: V prefix must match K prefix");
  TORCH_CHECK(lens.numel() == p.B, "fdl.kv_gather_prefix: lens has ", lens.numel(), " rows, prefix has ", p.B);
  Rows bl{};
  int n_blk = 0;
  if (k_block) {
    TORCH_CHECK(v_block.has_value(), "fdl.kv_gather_prefix: k_block needs v_block");
    check_cuda(*k_block, "k_block");
    bl = rows_of(*k_block, seq_dim_in);
    TORCH_CHECK(bl.B == p.B && bl.H == p.H && bl.D == p.D && v_block->sizes() == k_block->sizes() &&
                    v_block->strides() == k_block->strides(),
                "fdl.kv_gather_prefix: block ", k_block->sizes(), " vs prefix ", k_prefix.sizes());
    n_blk = static_cast<int>(bl.S);
  }
  int64_t osb, oss, osh;
  const int32_t* cu = nullptr;
  if (cu_seqlens) {
    TORCH_CHECK(cu_seqlens->is_cuda() && cu_seqlens->scalar_type() == at::kInt && cu_seqlens->is_contiguous() &&
                    cu_seqlens->numel() == p.B + 1,
                "fdl.kv_gather_prefix: cu_seqlens must be a contiguous CUDA int32 [B+1] tensor");
    TORCH_CHECK(k_out.dim() == 3 && k_out.size(1) == p.H * rep && k_out.size(2) == p.D,
                "fdl.kv_gather_prefix: packed output must be [total, H*rep, D]");
    osb = 0;
    oss = k_out.stride(0);
    osh = k_out.stride(1);
    cu = cu_seqlens->data_ptr<int32_t>();
  } else {
    const Rows o = rows_of(k_out, seq_dim_out);
    TORCH_CHECK(o.B == p.B && o.H == p.H * rep && o.D == p.D && o.S >= p.S + n_blk,
                "fdl.kv_gather_prefix: output ", k_out.sizes(), " too small");
    osb = o.sb;
    oss = o.ss;
    osh = o.sh;
  }
  TORCH_CHECK(v_out.sizes() == k_out.sizes() && v_out.strides() == k_out.strides(),
              "fdl.kv_gather_prefix: V output must match K output");
  c10::cuda::CUDAGuard guard(k_prefix.device());
  check_rc(fdl_kv_gather_prefix(k_prefix.data_ptr(), v_prefix.data_ptr(), lens.data_ptr<int32_t>(),
                                static_cast<int>(p.S), k_block ? k_block->data_ptr() : nullptr,
                                v_block ? v_block->data_ptr() : nullptr, n_blk, k_out.data_ptr(), v_out.data_ptr(),
                                cu, cu ? k_out.size(0) : 0, static_cast<int>(p.B), static_cast<int>(p.H), static_cast<int>(p.D),
                                static_cast<int>(rep), elem_bytes(k_prefix), p.sb, p.ss, p.sh, bl.sb, bl.ss, bl.sh,
                                osb, oss, osh, cur_stream()),
           "kv_gather_prefix");
}

void kv_gather_rows(const Tensor& k_src, const std::optional<Tensor>& v_src, const Tensor& idx,
                    const std::optional<Tensor>& count, const Tensor& k_out, const std::optional<Tensor>& v_out,
                    int64_t seq_dim) {
  check_cuda(k_src, "k_src");
  check_cuda(k_out, "k_out");
  TORCH_CHECK(v_src.has_value() == v_out.has_value(), "fdl.kv_gather_rows: v_src and v_out go together");
  TORCH_CHECK(idx.is_cuda() && (idx.scalar_type() == at::kLong || idx.scalar_type() == at::kInt) && idx.dim() == 2 &&
                  idx.stride(1) == 1,
              "fdl.kv_gather_rows: idx must be a CUDA int64/int32 [B, n] tensor with unit inner stride");
  const Rows s = rows_of(k_src, seq_dim), o = rows_of(k_out, seq_dim);
  TORCH_CHECK(s.B == o.B && s.H == o.H && s.D == o.D && o.S >= idx.size(1) && idx.size(0) == s.B &&
                  k_src.dtype() == k_out.dtype(),
              "fdl.kv_gather_rows: src ", k_src.sizes(), " out ", k_out.sizes(), " idx ", idx.sizes());
  if (count)
    TORCH_CHECK(count->is_cuda() && count->scalar_type() == at::kInt && count->numel() == s.B &&
                    count->is_contiguous(),
                "fdl.kv_gather_rows: count must be a contiguous CUDA int32 [B] tensor");
  if (v_src)
    TORCH_CHECK(v_src->sizes() == k_src.sizes() && v_src->strides() == k_src.strides() &&
                    v_out->sizes() == k_out.sizes() && v_out->strides() == k_out.strides(),
                "fdl.kv_gather_rows: V tensors must match K tensors");
  c10::cuda::CUDAGuard guard(k_src.device());
  check_rc(fdl_kv_gather_rows(k_src.data_ptr(), v_src ? v_src->data_ptr() : nullptr, idx.data_ptr(),
                              idx.scalar_type() == at::kInt ? 1 : 0, idx.stride(0),
                              count ? count->data_ptr<int32_t>() : nullptr, k_out.data_ptr(),
                              v_out ? v_out->data_ptr() : nullptr, static_cast<int>(s.B), static_cast<int>(idx.size(1)),
                              static_cast<int>(s.S), static_cast<int>(s.H), static_cast<int>(s.D), elem_bytes(k_src),
                              s.sb, s.ss, s.sh, o.sb, o.ss, o.sh, cur_stream()),
           "kv_gather_rows");
}

// True when every batch row (dims 1..) of t is one contiguous run.
bool rows_contiguous(const Tensor& t) {
  int64_t expect = 1;
  for (int64_t d = t.dim() - 1; d >= 1; --d) {
    if (t.size(d) != 1 && t.stride(d) != expect) return false;
    expect *= t.size(d);
  }
  return true;
}

// In-place batch compaction of buffers that share the batch size, the row
// size in bytes and the batch stride in bytes: row i <- row active[i].
void kv_compact(at::TensorList bufs, const Tensor& active) {
  TORCH_CHECK(active.is_cuda() && active.scalar_type() == at::kLong && active.dim() == 1 && active.is_contiguous(),
              "fdl.kv_compact: active must be a contiguous CUDA int64 [n] tensor");
  if (bufs.empty() || active.numel() == 0) return;
  const Tensor& b0 = bufs[0];
  TORCH_CHECK(b0.dim() >= 1, "fdl.kv_compact: buffers need a batch dimension");
  const int64_t B = b0.size(0);
  TORCH_CHECK(active.numel() <= B, "fdl.kv_compact: ", active.numel(), " active rows for a batch of ", B);
  const int64_t row_bytes = (b0.numel() / B) * static_cast<int64_t>(b0.element_size());
  const int64_t stride_bytes = b0.stride(0) * static_cast<int64_t>(b0.element_size());
  std::vector<void*> ptrs;
  ptrs.reserve(bufs.size());
  for (const Tensor& t : bufs) {
    TORCH_CHECK(t.is_cuda() && t.device() == active.device(), "fdl.kv_compact: buffers must be on ", active.device());
    TORCH_CHECK(t.dim() >= 1 && t.size(0) == B, "fdl.kv_compact: all buffers must share the batch size ", B);
    TORCH_CHECK((t.numel() / B) * static_cast<int64_t>(t.element_size()) == row_bytes &&
                    t.stride(0) * static_cast<int64_t>(t.element_size()) == stride_bytes,
                "fdl.kv_compact: all buffers must share the row size and batch stride in bytes");
    TORCH_CHECK(rows_contiguous(t), "fdl.kv_compact: each batch row must be contiguous");
    ptrs.push_back(t.data_ptr());
  }
  c10::cuda::CUDAGuard guard(active.device());
  check_rc(fdl_kv_compact(ptrs.data(), static_cast<int>(ptrs.size()), row_bytes, stride_bytes, static_cast<int>(B),
                          active.data_ptr<int64_t>(), static_cast<int>(active.numel()), cur_stream()),
           "kv_compact");
}

// ---------------------------------------------------------------- (a18)
int select_dtype(const Tensor& t) {
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 || t.scalar_type() == at::kFloat,
              "fdl: token selection takes bf16 or fp32 inputs, got ", t.scalar_type());
  return t.scalar_type() == at::kBFloat16 ? FDL_BF16 : FDL_F32;
}

void check_flags(const Tensor& t, int64_t B, int64_t S, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBool && t.dim() == 2 && t.size(0) == B && t.size(1) == S &&
                  t.stride(1) == 1,
              "fdl: ", name, " must be a CUDA bool [", B, ", ", S, "] tensor with unit inner stride");
}

void cosine_select(const Tensor& hidden, const Tensor& cached, int64_t n_select, bool refresh, const Tensor& idx,
                   const std::optional<Tensor>& cos_out) {
  check_cuda(hidden, "hidden");
  check_cuda(cached, "cached");
  TORCH_CHECK(hidden.dim() == 3 && cached.sizes() == hidden.sizes() && cached.dtype() == hidden.dtype(),
              "fdl.cosine_select: hidden and cached are [B, S, H] of one dtype");
  const int64_t B = hidden.size(0), S = hidden.size(1);
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kLong && idx.dim() == 2 && idx.size(0) == B &&
                  idx.size(1) == n_select && idx.stride(1) == 1,
              "fdl.cosine_select: idx must be a CUDA int64 [B, n_select] tensor with unit inner stride");
  if (cos_out)
    TORCH_CHECK(cos_out->is_cuda() && cos_out->scalar_type() == at::kFloat && cos_out->is_contiguous() &&
                    cos_out->numel() == B * S,
                "fdl.cosine_select: cos_out must be a contiguous CUDA fp32 [B, S] tensor");
  c10::cuda::CUDAGuard guard(hidden.device());
  check_rc(fdl_cosine_select(hidden.data_ptr(), cached.data_ptr(), refresh ? cached.data_ptr() : nullptr,
                             static_cast<int>(B), static_cast<int>(S), static_cast<int>(hidden.size(2)),
                             select_dtype(hidden), hidden.stride(0), hidden.stride(1), cached.stride(0),
                             cached.stride(1), cached.stride(0), cached.stride(1), static_cast<int>(n_select),
                             idx.data_ptr<int64_t>(), idx.stride(0), cos_out ? cos_out->data_ptr<float>() : nullptr,
                             cur_stream()),
           "cosine_select");
}

void focus_select(const Tensor& delta, const Tensor& mask, const std::optional<Tensor>& frozen, int64_t k_floor,
                  const Tensor& sel, const Tensor& ksel) {
  TORCH_CHECK(delta.is_cuda() && delta.dim() == 2 && delta.stride(1) == 1,
              "fdl.focus_select: delta must be a CUDA [B, S] tensor with unit inner stride");
  const int64_t B = delta.size(0), S = delta.size(1);
  check_flags(mask, B, S, "mask");
  if (frozen) check_flags(*frozen, B, S, "frozen");
  TORCH_CHECK(sel.is_cuda() && sel.scalar_type() == at::kLong && sel.dim() == 2 && sel.size(0) == B &&
                  sel.size(1) == S && sel.stride(1) == 1,
              "fdl.focus_select: sel must be a CUDA int64 [B, S] tensor with unit inner stride");
  TORCH_CHECK(ksel.is_cuda() && ksel.scalar_type() == at::kInt && ksel.numel() >= 1,
              "fdl.focus_select: ksel must be a CUDA int32 tensor");
  c10::cuda::CUDAGuard guard(delta.device());
  check_rc(fdl_focus_select(delta.data_ptr(), delta.stride(0), reinterpret_cast<const uint8_t*>(mask.data_ptr()),
                            mask.stride(0), frozen ? reinterpret_cast<const uint8_t*>(frozen->data_ptr()) : nullptr,
                            frozen ? frozen->stride(0) : 0, static_cast<int>(B), static_cast<int>(S),
                            static_cast<int>(k_floor), select_dtype(delta), sel.data_ptr<int64_t>(), sel.stride(0),
                            ksel.data_ptr<int32_t>(), cur_stream()),
           "focus_select");
}

void focus_importance(const Tensor& q, const Tensor& k, const Tensor& mask, double scaling, const Tensor& imp) {
  check_cuda(q, "q");
  check_cuda(k, "k");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && k.size(0) == q.size(0) && k.size(2) == q.size(2) &&
                  k.size(3) == q.size(3) && k.dtype() == q.dtype(),
              "fdl.focus_importance: q [B, Hq, S, D] and k [B, Hkv, S, D] of one dtype");
  const int64_t B = q.size(0), S = q.size(2);
  check_flags(mask, B, S, "mask");
  TORCH_CHECK(imp.is_cuda() && imp.dim() == 2 && imp.size(0) == B && imp.size(1) == S && imp.stride(1) == 1 &&
                  imp.dtype() == q.dtype(),
              "fdl.focus_importance: imp must be a CUDA [B, S] tensor of q's dtype with unit inner stride");
  c10::cuda::CUDAGuard guard(q.device());
  check_rc(fdl_focus_importance(q.data_ptr(), k.data_ptr(), reinterpret_cast<const uint8_t*>(mask.data_ptr()),
                                static_cast<int>(B), static_cast<int>(S), static_cast<int>(q.size(1)),
                                static_cast<int>(k.size(1)), static_cast<int>(q.size(3)), select_dtype(q), q.stride(0),
                                q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2), mask.stride(0),
                                static_cast<float>(scaling), imp.data_ptr(), imp.stride(0), cur_stream()),
           "focus_importance");
}

void kv_sparse_prefix(const Tensor& k, const Tensor& v, const Tensor& lens, int64_t keep_num, int64_t keep_den,
                      const Tensor& sel, const Tensor& out_len, const std::optional<Tensor>& k_out,
                      const std::optional<Tensor>& v_out, const Tensor& workspace) {
  check_cuda(k, "k");
  check_cuda(v, "v");
  TORCH_CHECK(k.dim() == 4 && k.scalar_type() == at::kBFloat16 && v.sizes() == k.sizes() &&
                  v.strides() == k.strides(),
              "fdl.kv_sparse_prefix: K/V must be bf16 BSHD [B, cap, H, D] with equal layouts");
  TORCH_CHECK(lens.is_cuda() && lens.scalar_type() == at::kInt && lens.numel() == k.size(0) && lens.is_contiguous(),
              "fdl.kv_sparse_prefix: lens must be a contiguous CUDA int32 [B] tensor");
  TORCH_CHECK(sel.is_cuda() && sel.scalar_type() == at::kInt && sel.dim() == 2 && sel.size(0) == k.size(0) &&
                  sel.is_contiguous(),
              "fdl.kv_sparse_prefix: sel must be a contiguous CUDA int32 [B, max_keep] tensor");
  TORCH_CHECK(out_len.is_cuda() && out_len.scalar_type() == at::kInt && out_len.numel() == k.size(0),
              "fdl.kv_sparse_prefix: out_len must be a CUDA int32 [B] tensor");
  TORCH_CHECK(workspace.is_cuda() && workspace.is_contiguous(), "fdl.kv_sparse_prefix: workspace must be CUDA");
  TORCH_CHECK(k_out.has_value() == v_out.has_value(), "fdl.kv_sparse_prefix: k_out and v_out go together");
  int64_t osb = 0, oss = 0, osh = 0;
  if (k_out) {
    check_cuda(*k_out, "k_out");
    TORCH_CHECK(k_out->dim() == 4 && k_out->size(0) == k.size(0) && k_out->size(1) >= sel.size(1) &&
                    k_out->size(2) == k.size(2) && k_out->size(3) == k.size(3) && v_out->sizes() == k_out->sizes() &&
                    v_out->strides() == k_out->strides() && k_out->scalar_type() == at::kBFloat16,
                "fdl.kv_sparse_prefix: outputs must be bf16 [B, >=max_keep, H, D]");
    osb = k_out->stride(0);
    oss = k_out->stride(1);
    osh = k_out->stride(2);
  }
  c10::cuda::CUDAGuard guard(k.device());
  check_rc(fdl_kv_sparse_prefix(k.data_ptr(), v.data_ptr(), lens.data_ptr<int32_t>(), static_cast<int>(k.size(0)),
                                static_cast<int>(k.size(1)), static_cast<int>(k.size(2)), static_cast<int>(k.size(3)),
                                k.stride(0), k.stride(1), k.stride(2), static_cast<int>(keep_num),
                                static_cast<int>(keep_den), static_cast<int>(sel.size(1)), sel.data_ptr<int32_t>(),
                                out_len.data_ptr<int32_t>(), k_out ? k_out->data_ptr() : nullptr,
                                v_out ? v_out->data_ptr() : nullptr, osb, oss, osh, workspace.data_ptr(),
                                workspace.numel() * workspace.element_size(), cur_stream()),
           "kv_sparse_prefix");
}

// ---------------------------------------------------------------- (c)
void gather_rmsnorm(const Tensor& x, const std::optional<Tensor>& idx, const std::optional<Tensor>& weight,
                    double eps, const std::optional<Tensor>& gathered, const Tensor& normed) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 3 && x.stride(2) == 1, "fdl.gather_rmsnorm: x must be CUDA [B, S, H]");
  const int64_t B = x.size(0), S = x.size(1), H = x.size(2);
  int64_t T = S, idx_sb = 0;
  const int64_t* ip = nullptr;
  if (idx) {
    TORCH_CHECK(idx->is_cuda() && idx->scalar_type() == at::kLong && idx->dim() == 2 && idx->size(0) == B &&
                    idx->stride(1) == 1,
                "fdl.gather_rmsnorm: idx must be a CUDA int64 [B, T] tensor with unit inner stride");
    T = idx->size(1);
    idx_sb = idx->stride(0);
    ip = idx->data_ptr<int64_t>();
  }
  TORCH_CHECK(normed.is_cuda() && normed.dim() == 3 && normed.size(0) == B && normed.size(1) == T &&
                  normed.size(2) == H && normed.stride(2) == 1 && normed.dtype() == x.dtype(),
              "fdl.gather_rmsnorm: normed must be [B, T, H] with x's dtype");
  if (gathered)
    TORCH_CHECK(gathered->sizes() == normed.sizes() && gathered->strides() == normed.strides() &&
                    gathered->dtype() == x.dtype(),
                "fdl.gather_rmsnorm: gathered must match normed");
  if (weight)
    TORCH_CHECK(weight->is_cuda() && weight->dim() == 1 && weight->size(0) == H && weight->is_contiguous() &&
                    weight->dtype() == x.dtype(),
                "fdl.gather_rmsnorm: weight must be a contiguous [H] tensor with x's dtype");
  c10::cuda::CUDAGuard guard(x.device());
  check_rc(fdl_gather_rmsnorm(x.data_ptr(), ip, idx_sb, weight ? weight->data_ptr() : nullptr,
                              static_cast<float>(eps), gathered ? gathered->data_ptr() : nullptr, normed.data_ptr(),
                              static_cast<int>(B), static_cast<int>(S), static_cast<int>(T), static_cast<int>(H),
                              dtype_code(x), x.stride(0), x.stride(1), normed.stride(0), normed.stride(1),
                              cur_stream()),
           "gather_rmsnorm");
}

// ---------------------------------------------------------------- (d)
int64_t attn_workspace_bytes(int64_t batch, int64_t sq, int64_t hq, int64_t num_splits) {
  return fdl_block_attn_workspace_bytes(static_cast<int>(batch), static_cast<int>(sq), static_cast<int>(hq), 128,
                                        static_cast<int>(num_splits));
}

void block_attn(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& seqlens,
                const std::optional<Tensor>& k_blk, const std::optional<Tensor>& v_blk,
                const std::optional<Tensor>& q_pos, int64_t mask_block, double scale, const Tensor& out,
                const std::optional<Tensor>& workspace, int64_t num_splits) {
  for (const Tensor* t : {&q, &k, &v, &out}) {
    check_cuda(*t, "attention tensor");
    TORCH_CHECK(t->dim() == 4 && t->scalar_type() == at::kBFloat16, "fdl.block_attn: bf16 [B, S, H, D] tensors");
  }
  TORCH_CHECK(v.sizes() == k.sizes() && v.strides() == k.strides(), "fdl.block_attn: V must match K");
  TORCH_CHECK(out.sizes() == q.sizes(), "fdl.block_attn: out must match q");
  TORCH_CHECK(k.size(0) == q.size(0) && k.size(3) == q.size(3), "fdl.block_attn: q ", q.sizes(), " k ", k.sizes());
  TORCH_CHECK(seqlens.is_cuda() && seqlens.scalar_type() == at::kInt && seqlens.numel() == q.size(0) &&
                  seqlens.is_contiguous(),
              "fdl.block_attn: seqlens must be a contiguous CUDA int32 [B] tensor");
  int n_blk = 0;
  if (k_blk) {
    TORCH_CHECK(v_blk.has_value(), "fdl.block_attn: k_blk needs v_blk");
    check_cuda(*k_blk, "k_blk");
    TORCH_CHECK(k_blk->dim() == 4 && k_blk->size(0) == k.size(0) && k_blk->size(2) == k.size(2) &&
                    k_blk->size(3) == k.size(3) && v_blk->sizes() == k_blk->sizes() &&
                    v_blk->strides() == k_blk->strides() && k_blk->scalar_type() == at::kBFloat16,
                "fdl.block_attn: block K/V must be bf16 [B, n, Hkv, D]");
    n_blk = static_cast<int>(k_blk->size(1));
  }
  if (q_pos)
    TORCH_CHECK(q_pos->is_cuda() && q_pos->scalar_type() == at::kInt && q_pos->is_contiguous() &&
                    q_pos->numel() == q.size(0) * q.size(1),
                "fdl.block_attn: q_pos must be a contiguous CUDA int32 [B, Sq] tensor");
  void* ws = nullptr;
  int64_t ws_bytes = 0;
  if (workspace) {
    TORCH_CHECK(workspace->is_cuda() && workspace->is_contiguous(), "fdl.block_attn: workspace must be CUDA");
    ws = workspace->data_ptr();
    ws_bytes = workspace->numel() * workspace->element_size();
  }
  c10::cuda::CUDAGuard guard(q.device());
  check_rc(fdl_block_attn(q.data_ptr(), k.data_ptr(), v.data_ptr(), seqlens.data_ptr<int32_t>(),
                          static_cast<int>(k.size(1)), k_blk ? k_blk->data_ptr() : nullptr,
                          v_blk ? v_blk->data_ptr() : nullptr, n_blk, q_pos ? q_pos->data_ptr<int32_t>() : nullptr,
                          static_cast<int>(mask_block), out.data_ptr(), static_cast<int>(q.size(0)),
                          static_cast<int>(q.size(1)), static_cast<int>(q.size(2)), static_cast<int>(k.size(2)),
                          static_cast<int>(q.size(3)), static_cast<float>(scale), q.stride(0), q.stride(1),
                          q.stride(2), k.stride(0), k.stride(1), k.stride(2), k_blk ? k_blk->stride(0) : 0,
                          k_blk ? k_blk->stride(1) : 0, k_blk ? k_blk->stride(2) : 0, out.stride(0), out.stride(1),
                          out.stride(2), static_cast<int>(num_splits), ws, ws_bytes, cur_stream()),
           "block_attn");
}

// ---------------------------------------------------------------- decode forward glue
void rope_qkv(const Tensor& y, const Tensor& pos, const Tensor& inv_freq, int64_t hq, int64_t hkv, const Tensor& q,
              const Tensor& k, const Tensor& v) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.stride(-1) == 1,
              "fdl.rope_qkv: y must be a bf16 CUDA tensor with unit inner stride");
  const int64_t D = q.size(-1);
  const int64_t rows = y.numel() / y.size(-1);
  TORCH_CHECK(y.size(-1) == (hq + 2 * hkv) * D, "fdl.rope_qkv: y last dim ", y.size(-1), " != (hq+2hkv)*D");
  TORCH_CHECK(y.dim() == 2 || (y.dim() == 3 && y.stride(0) == y.size(1) * y.stride(1)),
              "fdl.rope_qkv: y rows must be uniformly strided");
  TORCH_CHECK(pos.is_cuda() && pos.scalar_type() == at::kLong && pos.is_contiguous() && pos.numel() == rows,
              "fdl.rope_qkv: pos must be a contiguous CUDA int64 tensor with one entry per row");
  TORCH_CHECK(inv_freq.is_cuda() && inv_freq.scalar_type() == at::kFloat && inv_freq.numel() == D / 2,
              "fdl.rope_qkv: inv_freq must be CUDA fp32 [D/2]");
  for (const Tensor* t : {&q, &k, &v})
    TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->scalar_type() == at::kBFloat16,
                "fdl.rope_qkv: outputs must be contiguous bf16 CUDA tensors");
  TORCH_CHECK(q.numel() == rows * hq * D && k.numel() == rows * hkv * D && v.numel() == rows * hkv * D,
              "fdl.rope_qkv: output sizes");
  c10::cuda::CUDAGuard guard(y.device());
  check_rc(fdl_rope_qkv(y.data_ptr(), y.stride(-2), pos.data_ptr<int64_t>(), inv_freq.data_ptr<float>(),
                        q.data_ptr(), k.data_ptr(), v.data_ptr(), static_cast<int>(rows), static_cast<int>(hq),
                        static_cast<int>(hkv), static_cast<int>(D), cur_stream()),
           "rope_qkv");
}

// q/k/v split + RoPE with K and V stored straight into cache rows:
// k_dst / v_dst are [B, S, H, D] (seq_dim 1) or [B, H, S, D] (seq_dim 2);
// token t of sequence b goes to position dst_pos[b, t], or start[b] + t, or t.
void rope_qkv_kv(const Tensor& y, const Tensor& pos, const Tensor& inv_freq, int64_t hq, int64_t hkv, const Tensor& q,
                 const Tensor& k_dst, const Tensor& v_dst, const std::optional<Tensor>& start,
                 const std::optional<Tensor>& dst_pos, int64_t seq_dim) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.stride(-1) == 1,
              "fdl.rope_qkv_kv: y must be a bf16 CUDA tensor with unit inner stride");
  TORCH_CHECK(q.is_cuda() && q.is_contiguous() && q.scalar_type() == at::kBFloat16 && q.dim() == 4 &&
                  q.size(2) == hq,
              "fdl.rope_qkv_kv: q must be a contiguous bf16 CUDA [B, n, hq, D] tensor");
  const int64_t B = q.size(0), n = q.size(1), D = q.size(3);
  const int64_t rows = B * n;
  TORCH_CHECK(y.numel() == rows * (hq + 2 * hkv) * D, "fdl.rope_qkv_kv: y must hold B*n rows of (hq+2hkv)*D");
  TORCH_CHECK(y.dim() == 2 || (y.dim() == 3 && y.stride(0) == y.size(1) * y.stride(1)),
              "fdl.rope_qkv_kv: y rows must be uniformly strided");
  TORCH_CHECK(pos.is_cuda() && pos.scalar_type() == at::kLong && pos.is_contiguous() && pos.numel() == rows,
              "fdl.rope_qkv_kv: pos must be a contiguous CUDA int64 tensor with one entry per row");
  TORCH_CHECK(inv_freq.is_cuda() && inv_freq.scalar_type() == at::kFloat && inv_freq.numel() == D / 2,
              "fdl.rope_qkv_kv: inv_freq must be CUDA fp32 [D/2]");
  check_cuda(k_dst, "k_dst");
  check_cuda(v_dst, "v_dst");
  const Rows d = rows_of(k_dst, seq_dim);
  TORCH_CHECK(k_dst.scalar_type() == at::kBFloat16 && v_dst.sizes() == k_dst.sizes() &&
                  v_dst.strides() == k_dst.strides() && v_dst.dtype() == k_dst.dtype(),
              "fdl.rope_qkv_kv: k_dst and v_dst must be bf16 tensors of one shape and layout");
  TORCH_CHECK(d.B == B && d.H == hkv && d.D == D, "fdl.rope_qkv_kv: destination ", k_dst.sizes(),
              " does not hold [B, *, hkv, D] = [", B, ", *, ", hkv, ", ", D, "]");
  TORCH_CHECK(!(start && dst_pos), "fdl.rope_qkv_kv: give start or dst_pos, not both");
  if (start)
    TORCH_CHECK(start->is_cuda() && start->scalar_type() == at::kInt && start->is_contiguous() && start->numel() == B,
                "fdl.rope_qkv_kv: start must be a contiguous CUDA int32 [B] tensor");
  if (dst_pos)
    TORCH_CHECK(dst_pos->is_cuda() && dst_pos->scalar_type() == at::kLong && dst_pos->dim() == 2 &&
                    dst_pos->size(0) == B && dst_pos->size(1) == n && dst_pos->stride(1) == 1,
                "fdl.rope_qkv_kv: dst_pos must be a CUDA int64 [B, n] tensor with unit inner stride");
  c10::cuda::CUDAGuard guard(y.device());
  check_rc(fdl_rope_qkv_kv(y.data_ptr(), y.stride(-2), pos.data_ptr<int64_t>(), inv_freq.data_ptr<float>(),
                           q.data_ptr(), k_dst.data_ptr(), v_dst.data_ptr(), d.sb, d.ss, d.sh, static_cast<int>(d.S),
                           start ? start->data_ptr<int32_t>() : nullptr,
                           dst_pos ? dst_pos->data_ptr<int64_t>() : nullptr, dst_pos ? dst_pos->stride(0) : 0,
                           static_cast<int>(B), static_cast<int>(n), static_cast<int>(hq), static_cast<int>(hkv),
                           static_cast<int>(D), cur_stream()),
           "rope_qkv_kv");
}

void swiglu(const Tensor& gu, const Tensor& out) {
  TORCH_CHECK(gu.is_cuda() && gu.scalar_type() == at::kBFloat16 && gu.stride(-1) == 1 && out.is_cuda() &&
                  out.scalar_type() == at::kBFloat16 && out.stride(-1) == 1,
              "fdl.swiglu: bf16 CUDA tensors with unit inner stride");
  const int64_t F = out.size(-1);
  const int64_t rows = out.numel() / F;
  TORCH_CHECK(gu.size(-1) == 2 * F && gu.numel() / gu.size(-1) == rows, "fdl.swiglu: gu must be [rows, 2F]");
  TORCH_CHECK((gu.dim() == 2 || gu.stride(0) == gu.size(1) * gu.stride(1)) &&
                  (out.dim() == 2 || out.stride(0) == out.size(1) * out.stride(1)),
              "fdl.swiglu: rows must be uniformly strided");
  c10::cuda::CUDAGuard guard(gu.device());
  check_rc(fdl_swiglu(gu.data_ptr(), gu.stride(-2), out.data_ptr(), out.stride(-2), rows, static_cast<int>(F),
                      cur_stream()),
           "swiglu");
}

// logits [..., V] bf16 with uniformly strided rows; token int64 and prob bf16
// hold one entry per row (any shape with that many contiguous elements).
void softmax_argmax(const Tensor& logits, const Tensor& token, const std::optional<Tensor>& prob) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kBFloat16 && logits.stride(-1) == 1,
              "fdl.softmax_argmax: logits must be a bf16 CUDA tensor with unit inner stride");
  const int64_t V = logits.size(-1);
  const int64_t rows = V > 0 ? logits.numel() / V : 0;
  for (int64_t d = 0; d + 2 < logits.dim(); ++d)
    TORCH_CHECK(logits.stride(d) == logits.size(d + 1) * logits.stride(d + 1),
                "fdl.softmax_argmax: logits rows must be uniformly strided");
  TORCH_CHECK(token.is_cuda() && token.scalar_type() == at::kLong && token.is_contiguous() && token.numel() == rows,
              "fdl.softmax_argmax: token must be a contiguous CUDA int64 tensor with one entry per row");
  if (prob)
    TORCH_CHECK(prob->is_cuda() && prob->scalar_type() == at::kBFloat16 && prob->is_contiguous() &&
                    prob->numel() == rows,
                "fdl.softmax_argmax: prob must be a contiguous CUDA bf16 tensor with one entry per row");
  c10::cuda::CUDAGuard guard(logits.device());
  check_rc(fdl_softmax_argmax(logits.data_ptr(), logits.dim() >= 2 ? logits.stride(-2) : V, static_cast<int>(rows),
                              static_cast<int>(V), token.data_ptr<int64_t>(), prob ? prob->data_ptr() : nullptr,
                              cur_stream()),
           "softmax_argmax");
}

// x, res, sum_out, normed: [..., H] with uniformly strided rows.  sum_out
// may be res itself (in-place residual update) or absent.
void add_rmsnorm(const Tensor& x, const Tensor& res, const std::optional<Tensor>& weight, double eps,
                 const std::optional<Tensor>& sum_out, const Tensor& normed) {
  const int64_t H = x.size(-1);
  const int64_t rows = x.numel() / H;
  auto rs = [&](const Tensor& t, const char* name) {
    TORCH_CHECK(t.is_cuda() && t.dtype() == x.dtype() && t.size(-1) == H && t.numel() / H == rows &&
                    t.stride(-1) == 1,
                "fdl.add_rmsnorm: ", name, " must be a CUDA tensor of x's dtype and shape with unit inner stride");
    for (int64_t d = 0; d + 2 < t.dim(); ++d)
      TORCH_CHECK(t.stride(d) == t.size(d + 1) * t.stride(d + 1), "fdl.add_rmsnorm: ", name,
                  " rows must be uniformly strided");
    return t.dim() >= 2 ? t.stride(-2) : H;
  };
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kHalf,
              "fdl.add_rmsnorm: bf16 or fp16 tensors");
  const int64_t x_rs = rs(x, "x"), r_rs = rs(res, "res"), o_rs = rs(normed, "normed");
  if (sum_out) TORCH_CHECK(rs(*sum_out, "sum_out") == o_rs, "fdl.add_rmsnorm: sum_out and normed row strides differ");
  if (weight)
    TORCH_CHECK(weight->is_cuda() && weight->dim() == 1 && weight->size(0) == H && weight->is_contiguous() &&
                    weight->dtype() == x.dtype(),
                "fdl.add_rmsnorm: weight must be a contiguous [H] tensor with x's dtype");
  c10::cuda::CUDAGuard guard(x.device());
  check_rc(fdl_add_rmsnorm(x.data_ptr(), x_rs, res.data_ptr(), r_rs, weight ? weight->data_ptr() : nullptr,
                           static_cast<float>(eps), sum_out ? sum_out->data_ptr() : nullptr, normed.data_ptr(), o_rs,
                           static_cast<int>(rows), static_cast<int>(H),
                           x.scalar_type() == at::kBFloat16 ? FDL_BF16 : FDL_F16, cur_stream()),
           "add_rmsnorm");
}

// Functional form with the signature of the flash_kvcache custom op of
// utils/attention_backends.py:83-86; workspace comes from torch's caching
// allocator (graph-capture safe).
Tensor flash_kvcache(const Tensor& q, const Tensor& k_cache, const Tensor& v_cache, const Tensor& cache_seqlens,
                     double softmax_scale, bool causal) {
  TORCH_CHECK(!causal, "fdl.flash_kvcache: block diffusion attention is non-causal (causal=True unsupported)");
  auto out = at::empty_like(q, q.options().memory_format(at::MemoryFormat::Contiguous));
  const int64_t B = q.size(0), Sq = q.size(1), Hq = q.size(2);
  const int64_t splits = fdl_block_attn_auto_splits(static_cast<int>(B), static_cast<int>(Sq), static_cast<int>(Hq),
                                                   static_cast<int>(k_cache.size(2)),
                                                   static_cast<int>(k_cache.size(1)), 0);
  const int64_t ws_bytes = attn_workspace_bytes(B, Sq, Hq, splits);
  std::optional<Tensor> ws;
  if (ws_bytes > 0) ws = at::empty({ws_bytes}, q.options().dtype(at::kByte));
  block_attn(q, k_cache, v_cache, cache_seqlens, std::nullopt, std::nullopt, std::nullopt, 0, softmax_scale, out, ws,
             splits);
  return out;
}

Tensor flash_kvcache_meta(const Tensor& q, const Tensor&, const Tensor&, const Tensor&, double, bool) {
  return at::empty_like(q, q.options().memory_format(at::MemoryFormat::Contiguous));
}

}  // namespace

TORCH_LIBRARY(fdl, m) {
  m.def("kv_append(Tensor(a!)[] k_caches, Tensor(b!)[] v_caches, Tensor[] k_srcs, Tensor[] v_srcs, "
        "Tensor start_pos) -> ()");
  m.def("kv_scatter(Tensor(a!) k_dst, Tensor(b!)? v_dst, Tensor k_src, Tensor? v_src, Tensor positions, "
        "int seq_dim) -> ()");
  m.def("kv_gather_prefix(Tensor k_prefix, Tensor v_prefix, Tensor lens, Tensor? k_block, Tensor? v_block, "
        "int rep, Tensor(a!) k_out, Tensor(b!) v_out, Tensor? cu_seqlens, int seq_dim_in, int seq_dim_out) -> ()");
  m.def("kv_gather_rows(Tensor k_src, Tensor? v_src, Tensor idx, Tensor? count, Tensor(a!) k_out, "
        "Tensor(b!)? v_out, int seq_dim) -> ()");
  m.def("kv_compact(Tensor(a!)[] bufs, Tensor active) -> ()");
  m.def("cosine_select(Tensor hidden, Tensor(a!) cached, int n_select, bool refresh, Tensor(b!) idx, "
        "Tensor(c!)? cos_out) -> ()");
  m.def("focus_select(Tensor delta, Tensor mask, Tensor? frozen, int k_floor, Tensor(a!) sel, Tensor(b!) ksel) -> ()");
  m.def("focus_importance(Tensor q, Tensor k, Tensor mask, float scaling, Tensor(a!) imp) -> ()");
  m.def("kv_sparse_prefix(Tensor k, Tensor v, Tensor lens, int keep_num, int keep_den, Tensor(a!) sel, "
        "Tensor(b!) out_len, Tensor(c!)? k_out, Tensor(d!)? v_out, Tensor(e!) workspace) -> ()");
  m.def("gather_rmsnorm(Tensor x, Tensor? idx, Tensor? weight, float eps, Tensor(a!)? gathered, "
        "Tensor(b!) normed) -> ()");
  m.def("block_attn(Tensor q, Tensor k, Tensor v, Tensor seqlens, Tensor? k_blk, Tensor? v_blk, Tensor? q_pos, "
        "int mask_block, float scale, Tensor(a!) out, Tensor(b!)? workspace, int num_splits) -> ()");
  m.def("flash_kvcache(Tensor q, Tensor k_cache, Tensor v_cache, Tensor cache_seqlens, float softmax_scale, "
        "bool causal) -> Tensor");
  m.def("rope_qkv(Tensor y, Tensor pos, Tensor inv_freq, int hq, int hkv, Tensor(a!) q, Tensor(b!) k, "
        "Tensor(c!) v) -> ()");
  m.def("rope_qkv_kv(Tensor y, Tensor pos, Tensor inv_freq, int hq, int hkv, Tensor(a!) q, Tensor(b!) k_dst, "
        "Tensor(c!) v_dst, Tensor? start, Tensor? dst_pos, int seq_dim) -> ()");
  m.def("swiglu(Tensor gu, Tensor(a!) out) -> ()");
  m.def("softmax_argmax(Tensor logits, Tensor(a!) token, Tensor(b!)? prob) -> ()");
  m.def("add_rmsnorm(Tensor x, Tensor res, Tensor? weight, float eps, Tensor(a!)? sum_out, Tensor(b!) normed) -> ()");
}

TORCH_LIBRARY_IMPL(fdl, CUDA, m) {
  m.impl("kv_append", &kv_append);
  m.impl("kv_scatter", &kv_scatter);
  m.impl("kv_gather_prefix", &kv_gather_prefix);
  m.impl("kv_gather_rows", &kv_gather_rows);
  m.impl("kv_compact", &kv_compact);
  m.impl("cosine_select", &cosine_select);
  m.impl("focus_select", &focus_select);
  m.impl("focus_importance", &focus_importance);
  m.impl("kv_sparse_prefix", &kv_sparse_prefix);
  m.impl("gather_rmsnorm", &gather_rmsnorm);
  m.impl("block_attn", &block_attn);
  m.impl("flash_kvcache", &flash_kvcache);
  m.impl("rope_qkv", &rope_qkv);
  m.impl("rope_qkv_kv", &rope_qkv_kv);
  m.impl("swiglu", &swiglu);
  m.impl("softmax_argmax", &softmax_argmax);
  m.impl("add_rmsnorm", &add_rmsnorm);
}

TORCH_LIBRARY_IMPL(fdl, Meta, m) {
  m.impl("kv_append", [](at::TensorList, at::TensorList, at::TensorList, at::TensorList, const Tensor&) {});
  m.impl("kv_scatter", [](const Tensor&, const std::optional<Tensor>&, const Tensor&, const std::optional<Tensor>&,
                          const Tensor&, int64_t) {});
  m.impl("kv_gather_prefix",
         [](const Tensor&, const Tensor&, const Tensor&, const std::optional<Tensor>&, const std::optional<Tensor>&,
            int64_t, const Tensor&, const Tensor&, const std::optional<Tensor>&, int64_t, int64_t) {});
  m.impl("kv_gather_rows", [](const Tensor&, const std::optional<Tensor>&, const Tensor&,
                              const std::optional<Tensor>&, const Tensor&, const std::optional<Tensor>&, int64_t) {});
  m.impl("kv_compact", [](at::TensorList, const Tensor&) {});
  m.impl("cosine_select", [](const Tensor&, const Tensor&, int64_t, bool, const Tensor&, const std::optional<Tensor>&) {});
  m.impl("focus_select", [](const Tensor&, const Tensor&, const std::optional<Tensor>&, int64_t, const Tensor&,
                            const Tensor&) {});
  m.impl("focus_importance", [](const Tensor&, const Tensor&, const Tensor&, double, const Tensor&) {});
  m.impl("kv_sparse_prefix",
         [](const Tensor&, const Tensor&, const Tensor&, int64_t, int64_t, const Tensor&, const Tensor&,
            const std::optional<Tensor>&, const std::optional<Tensor>&, const Tensor&) {});
  m.impl("gather_rmsnorm", [](const Tensor&, const std::optional<Tensor>&, const std::optional<Tensor>&, double,
                              const std::optional<Tensor>&, const Tensor&) {});
  m.impl("block_attn", [](const Tensor&, const Tensor&, const Tensor&, const Tensor&, const std::optional<Tensor>&,
                          const std::optional<Tensor>&, const std::optional<Tensor>&, int64_t, double, const Tensor&,
                          const std::optional<Tensor>&, int64_t) {});
  m.impl("flash_kvcache", &flash_kvcache_meta);
  m.impl("rope_qkv", [](const Tensor&, const Tensor&, const Tensor&, int64_t, int64_t, const Tensor&, const Tensor&,
                        const Tensor&) {});
  m.impl("rope_qkv_kv", [](const Tensor&, const Tensor&, const Tensor&, int64_t, int64_t, const Tensor&, const Tensor&,
                           const Tensor&, const std::optional<Tensor>&, const std::optional<Tensor>&, int64_t) {});
  m.impl("swiglu", [](const Tensor&, const Tensor&) {});
  m.impl("softmax_argmax", [](const Tensor&, const Tensor&, const std::optional<Tensor>&) {});
  m.impl("add_rmsnorm", [](const Tensor&, const Tensor&, const std::optional<Tensor>&, double,
                           const std::optional<Tensor>&, const Tensor&) {});
}
