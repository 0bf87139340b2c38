"""Block-diffusion decoding at Qwen2.5 geometry on the fdl KV-cache kernels.

This is the end-to-end driver of the hot path: a Qwen2-architecture
block-diffusion LM (random-init weights; the real checkpoints are not
available offline) whose every KV-cache touch -- commit append, dKV block
buffer writes, token-sparse prefix selection and gather, RMSNorm, and the
block attention over cat(prefix, block) with in-kernel GQA -- runs on the
sm_100a kernels of libfdl_b200.so.  The dense projections and the MLP are
cuBLAS GEMMs through torch.

The decode loop follows the reference's dKV sampler ``batch_sample_dkv``
(generation_functions.py:2132-2340) and its forwards
(``forward_dkv``, modeling.py:1625-1692; commit ``forward`` with
``update_past_key_values=True``):

* prefill the prompt (multiple of the block size), bridge token from the
  last logit;
* per block: 32-token block (bridge token + masks); sub-blocks of 8 decoded
  by diffusion steps -- full-block steps on refresh boundaries
  (step_in_block <= 1 or step_in_block % refresh == 0), otherwise cached
  steps that feed only the not-yet-frozen positions
  (``_dkv_fed_indices``, modeling.py:2039-2060) and read the other block K/V
  from the DynamicBlockKV buffer; each step unmasks the tokens of the current
  sub-block whose probability exceeds the threshold, and at least the most
  confident one (generation_functions.py:2290-2305);
* block complete: commit forward over the 32 final tokens appends their K/V
  to the committed cache; its last logit gives the next bridge token.

The static-cache sampler ``batch_sample_dynamo`` (generation_functions.py:
243-900, the static-cache configuration) is the ``schedule="static"`` of the
same decoder: full-block steps only, the block's K/V written as scratch rows
of the committed cache, unmasked attention over cache[:lens + T].

``sparse_keep`` (a keep fraction, e.g. 0.25) replaces the committed prefix
seen by the diffusion steps with the top-scoring prefix tokens by key norm,
re-selected once per block (no reference counterpart; see
include/fdl_kvcache.h, fdl_kv_sparse_prefix).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import _lib


@dataclass(frozen=True)
class Geometry:
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 1e6
    eps: float = 1e-6
    tie_embeddings: bool = False

    @property
    def gqa(self) -> int:
        return self.heads // self.kv_heads


QWEN25_7B = Geometry(28, 3584, 28, 4, 128, 18944, 152064)
QWEN25_1_5B = Geometry(28, 1536, 12, 2, 128, 8960, 151936, tie_embeddings=True)

MASK_ID = 151665
STOP_ID = 151645
PAD_ID = 151643


def param_count(g: Geometry) -> int:
    per = (g.heads + 2 * g.kv_heads) * g.head_dim * (g.hidden + 1) + g.hidden * g.heads * g.head_dim
    per += 3 * g.hidden * g.ffn + 2 * g.hidden
    emb = g.vocab * g.hidden
    return g.layers * per + emb * (1 if g.tie_embeddings else 2) + g.hidden


class BlockDiffusionLM:
    """Random-init Qwen2 block-diffusion LM (weights N(0, init_std), biases 0,
    norm weights 1, as Fast_dLLM_QwenPreTrainedModel._init_weights,
    modeling.py:511-522).  q/k/v and gate/up projections are stored fused."""

    def __init__(self, geo: Geometry, device="cuda", dtype=torch.bfloat16, seed: int = 0, init_std: float = 0.02,
                 init_device: str | None = None, load_ops: bool = True):
        if load_ops:
            _lib.ensure_ops()
        self.geo, self.device, self.dtype = geo, torch.device(device), dtype
        g = geo
        # Generation on the target device is fast; init_device="cpu" gives
        # bit-reproducible weights across machines (used by the parity tests).
        gd = torch.device(init_device) if init_device else self.device
        gen = torch.Generator(device=gd).manual_seed(seed)

        def normal(*shape):
            return (torch.randn(*shape, generator=gen, device=gd, dtype=torch.float32) * init_std).to(dtype).to(
                self.device)

        qkv_out = (g.heads + 2 * g.kv_heads) * g.head_dim
        self.embed = normal(g.vocab, g.hidden)
        self.layers = []
        for _ in range(g.layers):
            self.layers.append(dict(
                ln1=torch.ones(g.hidden, dtype=dtype, device=self.device),
                wqkv=normal(qkv_out, g.hidden),
                bqkv=torch.zeros(qkv_out, dtype=dtype, device=self.device),
                wo=normal(g.hidden, g.heads * g.head_dim),
                ln2=torch.ones(g.hidden, dtype=dtype, device=self.device),
                wgu=normal(2 * g.ffn, g.hidden),
                wd=normal(g.hidden, g.ffn),
            ))
        self.norm = torch.ones(g.hidden, dtype=dtype, device=self.device)
        self.lm_head = self.embed if g.tie_embeddings else normal(g.vocab, g.hidden)
        inv = 1.0 / (g.rope_theta ** (torch.arange(0, g.head_dim, 2, dtype=torch.int64).float() / g.head_dim))
        self.inv_freq = inv.to(self.device).contiguous()

    # ------------------------------------------------------------------ ops
    def rmsnorm(self, x, w):
        out = torch.empty_like(x)
        torch.ops.fdl.gather_rmsnorm(x, None, w, self.geo.eps, None, out)
        _lib.count_launches(1)
        return out

    def qkv(self, layer, x, pos):
        """Fused q/k/v projection (cuBLAS, bias in the epilogue), then one fdl
        kernel that splits it and applies the rotary embedding at integer
        positions pos [B, T]."""
        g = self.geo
        B, T, _ = x.shape
        y = torch.addmm(layer["bqkv"], x.view(B * T, -1), layer["wqkv"].t())
        q = torch.empty(B, T, g.heads, g.head_dim, dtype=self.dtype, device=self.device)
        k = torch.empty(B, T, g.kv_heads, g.head_dim, dtype=self.dtype, device=self.device)
        v = torch.empty_like(k)
        torch.ops.fdl.rope_qkv(y, pos.reshape(-1), self.inv_freq, g.heads, g.kv_heads, q, k, v)
        _lib.count_launches(1)
        return q, k, v

    def qkv_into(self, layer, x, pos, k_dst, v_dst, start=None, dst_pos=None, seq_dim: int = 1):
        """As ``qkv``, but K and V go straight into their cache rows (the
        reference's projection -> RoPE -> cache write, attention_backends.py:
        937-955, as one kernel after the GEMM): k_dst / v_dst [B, S, Hkv, D]
        (seq_dim 1) or [B, Hkv, S, D] (seq_dim 2), token t of sequence b at
        dst_pos[b, t], else start[b] + t, else t.  Returns q."""
        g = self.geo
        B, T, _ = x.shape
        y = torch.addmm(layer["bqkv"], x.view(B * T, -1), layer["wqkv"].t())
        q = torch.empty(B, T, g.heads, g.head_dim, dtype=self.dtype, device=self.device)
        torch.ops.fdl.rope_qkv_kv(y, pos.reshape(-1), self.inv_freq, g.heads, g.kv_heads, q, k_dst, v_dst, start,
                                  dst_pos, seq_dim)
        _lib.count_launches(1)
        return q

    def add_rmsnorm(self, y, h, w):
        """Residual connection and the following RMSNorm in one kernel:
        h += y in place (bf16 rounding, the layer's `residual + hidden_states`)
        and returns RMSNorm(h) with weight w."""
        out = torch.empty_like(h)
        torch.ops.fdl.add_rmsnorm(y.view_as(h), h, w, self.geo.eps, h, out)
        _lib.count_launches(1)
        return out

    def mlp(self, layer, x):
        """Fast_dLLM_QwenMLP.forward (modeling.py:163-165) on normed rows x:
        fused gate/up GEMM, one SwiGLU kernel, down GEMM.  The residual add is
        left to the caller (fused into the next RMSNorm)."""
        g = self.geo
        B, T, _ = x.shape
        gu = x.view(B * T, -1) @ layer["wgu"].t()
        act = torch.empty(B * T, g.ffn, dtype=self.dtype, device=self.device)
        torch.ops.fdl.swiglu(gu, act)
        _lib.count_launches(1)
        return (act @ layer["wd"].t()).view(B, T, -1)

    def layers_forward(self, h, attend_layer):
        """The decoder stack on hidden states h [B, T, hidden] (updated in
        place as the residual stream).  attend_layer(l, layer, x) returns the
        attention output [B, T, Hq * D] of layer l for normed input x.  Each
        residual add is fused into the RMSNorm that follows it; returns h
        after the last layer's MLP residual."""
        B, T, _ = h.shape
        y = None
        for l, layer in enumerate(self.layers):
            x = self.rmsnorm(h, layer["ln1"]) if y is None else self.add_rmsnorm(y, h, layer["ln1"])
            a = attend_layer(l, layer, x)
            x = self.add_rmsnorm(a.reshape(B * T, -1) @ layer["wo"].t(), h, layer["ln2"])
            y = self.mlp(layer, x)
        return h + y

    def logits_rows(self, h_final_normed_rows):
        return h_final_normed_rows @ self.lm_head.t()


class DecodeState:
    """Preallocated device state of one decode batch: committed KV cache
    (BSHD per layer), dKV block buffers (BHSD per layer), sparse-prefix
    buffers, per-sequence lengths and workspaces.  Nothing here is
    reallocated while decoding, so every step is CUDA-graph capturable."""

    def __init__(self, model: BlockDiffusionLM, batch: int, max_len: int, block: int = 32,
                 sparse_keep: float | None = None, fused_kv_store: bool = True):
        g, dev, dt = model.geo, model.device, model.dtype
        self.model, self.B, self.block, self.max_len = model, batch, block, max_len
        # True: the RoPE kernel stores K/V into the cache / block buffer itself
        # (fdl_rope_qkv_kv); False: RoPE, then a separate append / scatter.
        self.fused_kv_store = fused_kv_store
        self.k = [torch.zeros(batch, max_len, g.kv_heads, g.head_dim, dtype=dt, device=dev) for _ in range(g.layers)]
        self.v = [torch.zeros_like(t) for t in self.k]
        self.blk_k = [torch.zeros(batch, g.kv_heads, block, g.head_dim, dtype=dt, device=dev) for _ in range(g.layers)]
        self.blk_v = [torch.zeros_like(t) for t in self.blk_k]
        self.lens = torch.zeros(batch, dtype=torch.int32, device=dev)  # committed length per sequence
        self.zero = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.sparse_keep = sparse_keep
        if sparse_keep:
            self.keep_num, self.keep_den = float(sparse_keep).as_integer_ratio()
            self.max_keep = max(1, math.ceil(max_len * self.keep_num / self.keep_den))
            self.sp_k = [torch.zeros(batch, self.max_keep, g.kv_heads, g.head_dim, dtype=dt, device=dev)
                         for _ in range(g.layers)]
            self.sp_v = [torch.zeros_like(t) for t in self.sp_k]
            self.sp_len = [torch.zeros(batch, dtype=torch.int32, device=dev) for _ in range(g.layers)]
            self.sp_sel = torch.empty(batch, self.max_keep, dtype=torch.int32, device=dev)
            self.sp_ws = torch.empty(_lib.sparse_prefix_workspace_bytes(batch, max_len), dtype=torch.uint8,
                                     device=dev)
        ns = _lib.attn_auto_splits(batch, block, g.heads, g.kv_heads, max_len, block)
        self.attn_splits = ns
        wsb = _lib.attn_workspace_bytes(batch, block, g.heads, ns)
        self.attn_ws = torch.empty(max(1, wsb), dtype=torch.uint8, device=dev) if wsb > 0 else None

    # -------------------------------------------------------------- pieces
    def attend(self, q, l, prefix: str, k_blk, v_blk, q_pos, lens=None, mask_block=None):
        """Block attention for layer l: queries q [B, T, Hq, D] over the
        committed prefix ("full": the first `lens` rows of the cache, default
        self.lens) or the sparse prefix ("sparse") followed by the given block
        K/V (none when k_blk is None), under the block-causal mask of
        `mask_block` positions (default the block size; 0 = every key
        visible)."""
        g = self.model.geo
        out = torch.empty_like(q)
        if prefix == "sparse":
            kp, vp, lens = self.sp_k[l], self.sp_v[l], self.sp_len[l]
        else:
            kp, vp, lens = self.k[l], self.v[l], self.lens if lens is None else lens
        T = q.shape[1]
        n_blk = 0 if k_blk is None else k_blk.shape[1]
        ns = self.attn_splits if T <= self.block else _lib.attn_auto_splits(self.B, T, g.heads, g.kv_heads,
                                                                            kp.shape[1], n_blk)
        ws = self.attn_ws
        if ns > 1 and (ws is None or ws.numel() < _lib.attn_workspace_bytes(self.B, T, g.heads, ns)):
            ws = torch.empty(_lib.attn_workspace_bytes(self.B, T, g.heads, ns), dtype=torch.uint8, device=q.device)
        mb = self.block if mask_block is None else mask_block
        torch.ops.fdl.block_attn(q, kp, vp, lens, k_blk, v_blk, q_pos, mb, g.head_dim ** -0.5, out,
                                 ws if ns > 1 else None, ns)
        _lib.count_launches(2 if ns > 1 else 1)
        return out

    def select_sparse_prefix(self):
        """Per layer: keep the top keep_num/keep_den committed prefix tokens by
        key norm, gathered into the compact sparse-prefix buffers."""
        for l in range(self.model.geo.layers):
            torch.ops.fdl.kv_sparse_prefix(self.k[l], self.v[l], self.lens, self.keep_num, self.keep_den, self.sp_sel,
                                           self.sp_len[l], self.sp_k[l], self.sp_v[l], self.sp_ws)
            _lib.count_launches(3)

    # ------------------------------------------------------------ forwards
    def forward_commit(self, ids, pos, all_rows: bool = False, mask_block=None):
        """Forward over a fully decoded span (prompt prefill or a finished
        block) that appends its K/V to the committed cache at self.lens and
        attends over committed prefix + span (block-causal; mask_block=0: the
        static-cache sampler's unmasked attention over cache[:lens + T]).
        Returns the final-normed hidden state of the span's last row
        [B, hidden] (all rows [B, T, hidden] with all_rows=True)."""
        m = self.model
        B, T = ids.shape
        h = F.embedding(ids, m.embed)
        pos = pos.contiguous()
        qpos = pos.to(torch.int32).contiguous()

        # Fused store: the span's K/V go into the cache at self.lens in the
        # RoPE kernel; the attention then reads cache[:lens + T] under the
        # block-causal mask (the same keys as prefix + span).
        lens_after = self.lens + T if self.fused_kv_store else None

        def attend_layer(l, layer, x):
            if self.fused_kv_store:
                q = m.qkv_into(layer, x, pos, self.k[l], self.v[l], start=self.lens)
                return self.attend(q, l, "full", None, None, qpos, lens=lens_after, mask_block=mask_block)
            q, k, v = m.qkv(layer, x, pos)
            a = self.attend(q, l, "full", k, v, qpos, mask_block=mask_block)
            torch.ops.fdl.kv_append([self.k[l]], [self.v[l]], [k], [v], self.lens)
            _lib.count_launches(1)
            return a

        h = m.layers_forward(h, attend_layer)
        self.lens += T
        if all_rows:
            return m.rmsnorm(h, m.norm)
        return m.rmsnorm(h[:, -1:].contiguous(), m.norm)[:, 0]

    def forward_scratch(self, ids, pos):
        """Diffusion step of the static-cache sampler (batch_sample_dynamo,
        generation_functions.py:754-775, and the patched attention forward,
        utils/attention_backends.py:873-898): the block's K/V are written as
        scratch rows at the committed length (``write_scratch_compiled`` at
        ``kv_write_start``) and every query attends over cache[:lens + T]
        with no mask (``scratch_seqlens``, ``is_causal=False``).  The committed
        length does not move; the next step overwrites the same rows and the
        commit forward rewrites them with the final tokens.  Returns the
        last-layer hidden state [B, T, hidden] (before the final norm)."""
        m = self.model
        B, T = ids.shape
        h = F.embedding(ids, m.embed)
        pos = pos.contiguous()
        qpos = pos.to(torch.int32).contiguous()
        lens_after = self.lens + T

        def attend_layer(l, layer, x):
            if self.fused_kv_store:
                q = m.qkv_into(layer, x, pos, self.k[l], self.v[l], start=self.lens)
            else:
                q, k, v = m.qkv(layer, x, pos)
                torch.ops.fdl.kv_append([self.k[l]], [self.v[l]], [k], [v], self.lens)
                _lib.count_launches(1)
            return self.attend(q, l, "full", None, None, qpos, lens=lens_after, mask_block=0)

        return m.layers_forward(h, attend_layer)

    def forward_block(self, ids, pos, fed=None, seed_hidden=None, prefix="full"):
        """dKV diffusion step over the current block (forward_dkv,
        modeling.py:1625-1692).  fed=None: full step, all block positions
        recomputed and written to the block buffer (write_full); returns the
        last-layer hidden [B, blk, hidden] (the seed for cached steps).  With
        fed [B, n]: only those positions run; their K/V are scattered into the
        block buffer and their outputs scattered onto seed_hidden."""
        m = self.model
        B = ids.shape[0]
        if fed is None:
            h = F.embedding(ids, m.embed)
            p = pos
        else:
            h = F.embedding(torch.gather(ids, 1, fed), m.embed)
            p = torch.gather(pos, 1, fed)
        T = h.shape[1]
        p = p.contiguous()
        qpos = p.to(torch.int32).contiguous()

        def attend_layer(l, layer, x):
            bk, bv = self.blk_k[l], self.blk_v[l]
            if self.fused_kv_store:
                # K/V of the computed positions go straight into the block
                # buffer (BHSD): 0..blk-1 on a full step, fed[b, i] on a cached one.
                q = m.qkv_into(layer, x, p, bk, bv, dst_pos=fed, seq_dim=2)
                return self.attend(q, l, prefix, bk.transpose(1, 2), bv.transpose(1, 2), qpos)
            q, k, v = m.qkv(layer, x, p)
            if fed is None:
                torch.ops.fdl.kv_append([bk.transpose(1, 2)], [bv.transpose(1, 2)], [k], [v], self.zero)
            else:
                torch.ops.fdl.kv_scatter(bk, bv, k.transpose(1, 2), v.transpose(1, 2), fed, 2)
            _lib.count_launches(1)
            return self.attend(q, l, prefix, bk.transpose(1, 2), bv.transpose(1, 2), qpos)

        h = m.layers_forward(h, attend_layer)
        if fed is None:
            return h
        out = seed_hidden.clone()
        torch.ops.fdl.kv_scatter(out, None, h, None, fed, 1)
        _lib.count_launches(1)
        return out


def dkv_fed_indices(prv_transfer_idx: torch.Tensor, width: int | None = None):
    """_dkv_fed_indices (modeling.py:2039-2060) on the device: not-yet-frozen
    positions in ascending order, padded (with the row's first fed index) to
    the batch max -- or to `width` when given, so the step's shapes come
    from a small fixed set."""
    fed_mask = ~prv_transfer_idx
    counts = fed_mask.sum(dim=1)
    num = max(1, int(counts.max().item())) if width is None else width
    order = torch.argsort(fed_mask.to(torch.int8), dim=1, descending=True, stable=True)
    fed = order[:, :num].contiguous()
    first = fed[:, :1]
    slot = torch.arange(num, device=fed.device).unsqueeze(0)
    pad = slot >= counts.clamp(min=1).unsqueeze(1)
    return torch.where(pad, first.expand(-1, num), fed), num


class BlockDiffusionDecoder:
    """Greedy (temperature 0) block-diffusion decode of a batch with the dKV
    schedule of batch_sample_dkv (generation_functions.py:2132-2340), or with
    ``schedule="static"`` the static-cache schedule of batch_sample_dynamo
    (generation_functions.py:243-900, no block cache): every diffusion step
    is a full-block forward whose K/V are scratch rows of the committed cache
    (DecodeState.forward_scratch), and prefill, steps and commit attend with
    no mask over cache[:lens + T].

    Every diffusion step works on static device buffers (block tokens,
    positions, sub-block index, frozen masks, seed hidden states), so with
    ``use_graphs=True`` each step is one CUDA-graph replay: one graph for the
    full-block step and one per bucketed width of the cached step.  The host
    reads two scalars per step (any masks left in the sub-block; the fed
    width), as the reference's loop does."""

    def __init__(self, model: BlockDiffusionLM, batch: int, prompt_len: int, gen_len: int, block: int = 32,
                 sub_block: int = 8, threshold: float = 0.9, refresh: int = 4, sparse_keep: float | None = None,
                 fed_bucket: int = 1, mask_id: int = MASK_ID, stop_id: int = STOP_ID, pad_id: int = PAD_ID,
                 use_graphs: bool = False, fused_kv_store: bool = True, schedule: str = "dkv"):
        assert prompt_len % block == 0 and block % sub_block == 0
        if schedule not in ("dkv", "static"):
            raise ValueError(f"schedule must be 'dkv' or 'static', not {schedule!r}")
        if schedule == "static" and sparse_keep:
            raise ValueError("the static-cache schedule attends over the whole committed cache (no sparse prefix)")
        self.schedule = schedule
        # The static-cache sampler attends with no mask over cache[:lens + T]
        # in every forward, the prefill included; the dKV sampler's prefill
        # and commit are block-causal.
        self.commit_mask = 0 if schedule == "static" else None
        self.m, self.B, self.block, self.sub = model, batch, block, sub_block
        self.threshold, self.refresh, self.fed_bucket = threshold, refresh, fed_bucket
        self.mask_id, self.stop_id, self.pad_id = mask_id, stop_id, pad_id
        self.prompt_len, self.gen_len = prompt_len, gen_len
        max_len = prompt_len + gen_len + block
        max_len = (max_len + 255) // 256 * 256
        self.st = DecodeState(model, batch, max_len, block, sparse_keep, fused_kv_store)
        self.prefix = "sparse" if sparse_keep else "full"
        dev = model.device
        self.ar = torch.arange(block, device=dev)
        B, H = batch, model.geo.hidden
        self.x = torch.full((B, block), mask_id, dtype=torch.long, device=dev)
        self.pos = torch.zeros(B, block, dtype=torch.long, device=dev)
        self.prv = torch.zeros(B, block, dtype=torch.bool, device=dev)
        self.cur = torch.zeros(B, block, dtype=torch.bool, device=dev)
        self.seed = torch.zeros(B, block, H, dtype=model.dtype, device=dev)
        self.finished = torch.zeros(B, dtype=torch.bool, device=dev)
        self.sub_idx = torch.zeros(sub_block, dtype=torch.long, device=dev)
        self.status = torch.zeros(2, dtype=torch.long, device=dev)
        self.bridge_buf = torch.zeros(B, 1, dtype=torch.long, device=dev)
        self.nxt = torch.zeros(B, 1, dtype=torch.long, device=dev)
        self.status_h = torch.zeros(2, dtype=torch.long).pin_memory() if dev.type == "cuda" else torch.zeros(2, dtype=torch.long)
        self.src_idx = torch.zeros(sub_block, dtype=torch.long, device=dev)
        self.x1_buf = torch.zeros(B, sub_block, dtype=torch.long, device=dev)
        self.p_buf = torch.zeros(B, sub_block, dtype=model.dtype, device=dev)
        self._subs = [torch.arange(s, s + sub_block, device=dev) for s in range(0, block, sub_block)]
        self._srcs = [torch.clamp(t - 1, min=0) for t in self._subs]
        self.use_graphs = use_graphs
        self._graphs = {}
        self._graph_launches = {}
        self._pool = None

    # ------------------------------------------------------------- steps
    def _sample(self, h):
        """Threshold unmasking of the current sub-block (generation_functions.py:
        2285-2305) from the last-layer hidden states h [B, block, hidden].
        Logits only for the rows the sampler reads: row i of the sub-block is
        predicted by position i-1 (row 0 by itself).  As sample_with_top_p at
        temperature 0 (modeling.py:2263-2269): softmax in the logits dtype,
        argmax = first maximal probability (fdl_softmax_argmax)."""
        m = self.m
        hn = m.rmsnorm(h.index_select(1, self.src_idx).contiguous(), m.norm)
        # One fused pass over each logits row gives the argmax of the bf16
        # softmax (ties to the lower index) and its probability, without the
        # [B, sub, vocab] probabilities.
        p, x1 = self.p_buf, self.x1_buf
        torch.ops.fdl.softmax_argmax(m.logits_rows(hn), x1, p)
        _lib.count_launches(1)
        sub = self.x.index_select(1, self.sub_idx)
        mask_idx = sub == self.mask_id
        x1p = torch.where(mask_idx, p, torch.full_like(p, -math.inf))
        unmask = x1p > self.threshold
        unmask.scatter_(1, x1p.argmax(-1, keepdim=True), True)
        unmask &= mask_idx
        self.x.index_copy_(1, self.sub_idx, torch.where(unmask, x1, sub))
        self.finished |= ((x1 == self.stop_id) & unmask).any(dim=1)
        self.prv.copy_(self.cur)
        self.cur.copy_(self.x != self.mask_id)
        # Loop control for the host, computed in the step itself (inside its
        # CUDA graph): [any mask left in the current sub-block, fed width of
        # the next cached step = max over sequences of the not-frozen count].
        self.status[0] = (self.x.index_select(1, self.sub_idx) == self.mask_id).any()
        self.status[1] = (~self.prv).sum(1).max()

    def _full_step(self):
        if self.schedule == "static":
            self._sample(self.st.forward_scratch(self.x, self.pos))
            return
        h = self.st.forward_block(self.x, self.pos, prefix=self.prefix)
        self.seed.copy_(h)
        self._sample(self.seed)

    def _cached_step(self, width):
        fed, _ = dkv_fed_indices(self.prv, width)
        h = self.st.forward_block(self.x, self.pos, fed=fed, seed_hidden=self.seed, prefix=self.prefix)
        self._sample(h)

    def _begin_step(self):
        """Block set-up: [bridge, masks...] tokens, sparse prefix selection,
        positions, fresh dKV transfer masks."""
        st = self.st
        self.x.fill_(self.mask_id)
        self.x[:, :1] = self.bridge_buf
        self.x.masked_fill_(self.finished[:, None], self.pad_id)
        if self.prefix == "sparse":
            st.select_sparse_prefix()
        self.pos.copy_(st.lens.to(torch.long)[:, None] + self.ar[None, :])
        self.prv.zero_()
        self.cur.zero_()

    def _commit_step(self):
        """Commit the decoded block to the KV cache; next bridge token."""
        hl = self.st.forward_commit(self.x, self.pos, mask_block=self.commit_mask)
        nxt = self.m.logits_rows(hl).argmax(-1, keepdim=True)
        nxt.masked_fill_(self.finished[:, None], self.pad_id)
        self.nxt.copy_(nxt)

    def _step_fn(self, key):
        if key == "begin":
            return self._begin_step
        if key == "commit":
            return self._commit_step
        return self._full_step if key == "full" else (lambda: self._cached_step(key))

    def _capture(self, key):
        """Capture the step `key` ("full" or a cached width) into a CUDA graph.
        A warm-up run on a side stream precedes capture; every static buffer it
        touches is restored afterwards (the block buffers it rewrites are
        rewritten by the first full step of every block anyway)."""
        fn = self._step_fn(key)
        bufs = (self.x, self.prv, self.cur, self.seed, self.finished, self.status, self.pos, self.st.lens, self.nxt)
        snap = [t.clone() for t in bufs]
        n0 = _lib.launches
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        # A warm-up whose kernels recorded an error is not captured.
        _lib.check_device(f"BlockDiffusionDecoder capture warm-up of step {key!r}")
        for t, v in zip(bufs, snap):
            t.copy_(v)
        g = torch.cuda.CUDAGraph()
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        n1 = _lib.launches
        with torch.cuda.graph(g, pool=self._pool):
            fn()
        self._graph_launches[key] = _lib.launches - n1
        _lib.launches = n0
        for t, v in zip(bufs, snap):
            t.copy_(v)
        self._graphs[key] = g
        return g

    def capture_all(self):
        """Capture every step variant up front (full step and cached widths)."""
        if not self.use_graphs:
            return
        widths = [] if self.schedule == "static" else list(range(self.fed_bucket, self.block + 1, self.fed_bucket))
        for key in ["begin", "full", "commit"] + widths:
            if key not in self._graphs:
                self._capture(key)
        _lib.check_device("BlockDiffusionDecoder.capture_all")

    def _run(self, key):
        if not self.use_graphs:
            self._step_fn(key)()
            return
        g = self._graphs.get(key) or self._capture(key)
        g.replay()
        _lib.count_launches(self._graph_launches[key])

    # ------------------------------------------------------------- public
    def prefill(self, prompt: torch.Tensor):
        """Commit the prompt; returns the bridge token [B, 1]."""
        B, P = prompt.shape
        pos = torch.arange(P, device=prompt.device).unsqueeze(0).expand(B, -1)
        self.st.lens.zero_()
        self.finished.zero_()
        hl = self.st.forward_commit(prompt, pos, mask_block=self.commit_mask)
        bridge = self.m.logits_rows(hl).argmax(-1, keepdim=True)
        _lib.check_device("BlockDiffusionDecoder.prefill")
        return bridge

    def decode_block(self, bridge: torch.Tensor, stats: dict | None = None):
        """Decode one block: [bridge token, 31 masks] -> 32 tokens; commit;
        returns (block tokens [B, 32], next bridge [B, 1])."""
        blk = self.block
        self.bridge_buf.copy_(bridge)
        self._run("begin")
        step_in_block = 0
        n_fwd = 0
        for sb in range(blk // self.sub):
            self.sub_idx.copy_(self._subs[sb])
            self.src_idx.copy_(self._srcs[sb])
            s, e = sb * self.sub, (sb + 1) * self.sub
            more = bool((self.x[:, s:e] == self.mask_id).any())
            fed_n = int((~self.prv).sum(1).max().item()) if more else 0
            while more:
                # Every step unmasks at least one position unless the model
                # predicts the mask token itself (then the reference's loop
                # never ends); fail loudly instead of spinning.
                if n_fwd >= 4 * blk:
                    raise RuntimeError("block decode made no progress: the model keeps predicting the mask token")
                if self.schedule == "static" or step_in_block <= 1 or step_in_block % self.refresh == 0:
                    self._run("full")
                else:
                    self._run(min(blk, max(1, -(-fed_n // self.fed_bucket) * self.fed_bucket)))
                n_fwd += 1
                step_in_block += 1
                # One device-to-host read per step: the step's own status.
                self.status_h.copy_(self.status, non_blocking=True)
                if self.status.is_cuda:
                    torch.cuda.current_stream(self.status.device).synchronize()
                more, fed_n = bool(self.status_h[0]), int(self.status_h[1])
        x = self.x.clone()
        self._run("commit")
        n_fwd += 1
        nxt = self.nxt.clone()
        # Once per block: any kernel that skipped a row or gave up a wait
        # stops the decode here instead of letting it continue on bad K/V.
        _lib.check_device("BlockDiffusionDecoder.decode_block")
        if stats is not None:
            stats["forwards"] = stats.get("forwards", 0) + n_fwd
            stats["blocks"] = stats.get("blocks", 0) + 1
        return x, nxt

    def generate(self, prompt: torch.Tensor, n_blocks: int | None = None):
        bridge = self.prefill(prompt)
        n_blocks = n_blocks if n_blocks is not None else self.gen_len // self.block
        out = [prompt, bridge]
        for _ in range(n_blocks):
            blk, bridge = self.decode_block(bridge)
            out.append(blk[:, 1:])
            out.append(bridge)
        return torch.cat(out, dim=1), self.finished.clone()
