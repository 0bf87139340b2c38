#!/usr/bin/env python
"""Benchmark of the Fast-dLLM v2 KV-cache hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config NAME]

Prints ONE JSON line (rank 0).  Multi-GPU runs are launched by torchrun, one
process per GPU; sequences are sharded across ranks (no data-path collective),
so scaling is weak and `value` is the aggregate over ranks divided by the max
over ranks of the device time.

Configs (BASELINE.json `configs`):
  gather_norm   fused gather + RMSNorm, x [4, 2048, 3584] bf16, 512 idx/row
  kv_path       28-layer committed-block append + varlen prefix gather with
                GQA-7 expansion, cache [16, 4096, 4, 128] per layer and K/V
  block_attn    block attention Q [B, 32, 28, 128] over a prefix of P keys
                (--attn-b, --attn-p, --attn-sq select the point)
  compact       in-place batch compaction of the 7B decode cache (28 layers
                of K/V [64, 2304, 4, 128], every fourth slot finished)
  e2e_7b        (default) block-diffusion decode at Qwen2.5-7B geometry,
                random init, 64 sequences/GPU, prompt 1024, dKV block cache
                + token-sparse prefix; one step = one 32-token block
  e2e_1_5b      the same at Qwen2.5-1.5B geometry, 16 sequences, prompt 256,
                static cache (batch_sample_dynamo's schedule: full-block
                forward every step, block K/V as scratch rows of the cache)

Inputs are seeded synthetic tensors (the reference's datasets and weights are
not available offline).  Between timed steps the inputs rotate through buffer
sets larger than the 126 MB L2 (or are larger than L2 themselves).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

L2_BYTES = 126 * 2**20


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


# --------------------------------------------------------------------------
# clocks sampling (nvidia-smi during the timed region)
# --------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._t = None
        self.window = None

    def _run(self):
        try:
            p = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                  "--format=csv,noheader,nounits", "-lms", "100"],
                                 stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return
        try:
            while not self._stop.is_set():
                line = p.stdout.readline()
                if not line:
                    break
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    self.samples.append((time.time(), parts))
        finally:
            p.terminate()
            try:
                p.wait(timeout=5)
            except Exception:
                p.kill()

    def start(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        time.sleep(0.3)

    def mark(self, t0, t1):
        self.window = (t0, t1)

    def stop(self):
        time.sleep(0.25)
        self._stop.set()
        if self._t:
            self._t.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        t0, t1 = self.window if self.window else (0, 1e30)
        inside = [s for _, s in ((t, s) for t, s in self.samples) if True]
        win = [s for t, s in self.samples if t0 - 0.15 <= t <= t1 + 0.15] or inside[-3:]

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(s[1]) for s in win if num(s[1]) is not None]
        mx = [num(s[2]) for s in win if num(s[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in win for i in range(4) if s[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(win)}


# --------------------------------------------------------------------------
# distributed plumbing
# --------------------------------------------------------------------------
def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    from fast_v2_b200.sharding import max_over_ranks as _max

    return x if world == 1 else _max(x)


def barrier(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


# --------------------------------------------------------------------------
# kernel timing inside the timed region
# --------------------------------------------------------------------------
class KernelTimer:
    """CUDA events around every launch of the dominant kernel (on the stream
    it is launched on); `avg_ms` is its mean launch duration."""

    def __init__(self):
        self.pairs = []
        self.active = False

    def wrap(self, fn):
        if not self.active:
            return fn()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        r = fn()
        e.record()
        self.pairs.append((s, e))
        return r

    def avg_ms(self):
        if not self.pairs:
            return None
        return sum(s.elapsed_time(e) for s, e in self.pairs) / len(self.pairs)


# --------------------------------------------------------------------------
# workloads (ours)
# --------------------------------------------------------------------------
def gen(seed):
    return torch.Generator(device="cpu").manual_seed(seed)


def dgen(seed):
    """Seeded generator on the GPU: multi-GB synthetic inputs in milliseconds
    (the same values on every B200 for a given seed)."""
    return torch.Generator(device="cuda").manual_seed(seed)


def wl_gather_norm(args, rank, world, kt: KernelTimer):
    import numpy as np

    from fast_v2_b200 import ensure_ops

    ensure_ops()
    B, S, H, T = 4, 2048, 3584, 512
    nbuf = max(2, math.ceil(3 * L2_BYTES / (B * S * H * 2)))
    g = gen(1000 + rank)
    dg = dgen(1000 + rank)
    xs = [torch.randn(B, S, H, generator=dg, device="cuda").to(torch.bfloat16) for _ in range(nbuf)]
    idx = torch.stack([torch.sort(torch.randperm(S, generator=g)[:T]).values for _ in range(B)]).cuda()
    w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).cuda()
    outs = [(torch.empty(B, T, H, dtype=torch.bfloat16, device="cuda"),
             torch.empty(B, T, H, dtype=torch.bfloat16, device="cuda")) for _ in range(nbuf)]
    pair = not args.norm_only
    alg_bytes = B * T * H * 2 * (3 if pair else 2) + B * T * 8 + H * 2  # read rows, write (gathered +) normed, idx, w
    state = {"i": 0}

    def step():
        i = state["i"] % nbuf
        state["i"] += 1
        torch.ops.fdl.gather_rmsnorm(xs[i], idx, w, 1e-6, outs[i][0] if pair else None, outs[i][1])

    # end-to-end through the public API with host buffers
    from fast_v2_b200.cuda_bench.fused_sparse_extension import fused_gather_input_rmsnorm_pair

    class _Norm(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.weight = torch.nn.Parameter(w, requires_grad=False)
            self.variance_epsilon = 1e-6

    norm = _Norm()
    hx = xs[0].cpu().pin_memory()
    hidx = idx.cpu().pin_memory()
    hg = torch.empty(B, T, H, dtype=torch.bfloat16).pin_memory()
    hn = torch.empty_like(hg).pin_memory()

    def e2e_step():
        dx = hx.to("cuda", non_blocking=True)
        di = hidx.to("cuda", non_blocking=True)
        gth, nrm = fused_gather_input_rmsnorm_pair(dx, di, norm)
        hg.copy_(gth, non_blocking=True)
        hn.copy_(nrm, non_blocking=True)

    e2e_bytes = (hx.numel() * 2 + hidx.numel() * 8, hg.numel() * 2 + hn.numel() * 2)

    def cpu_sample():
        from oracle import torch_port

        hxf = xs[0][:1].cpu()
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < args.cpu_seconds or n < 2:
            torch_port.gather_input_rmsnorm(hxf, hidx[:1], w.cpu(), 1e-6)
            n += 1
        dt = (time.perf_counter() - t0) / n
        return alg_bytes / 4 / dt / 1e9, f"{n} calls of batch row 1 of 4 ([1, 2048, 3584], 512 rows)"

    return dict(
        metric="fused gather+RMSNorm throughput (algorithmic HBM GB/s)", unit="GB/s",
        units_per_step=alg_bytes / 1e9, step=step, dominant=step, graph=True, e2e_step=e2e_step,
        e2e_bytes=e2e_bytes,
        roofline=dict(bound="hbm", per_launch=alg_bytes, kernel="gather_rmsnorm_kernel"), launches_per_step=1,
        config={"workload": "gather_norm", "x": [B, S, H], "rows_per_batch": T, "dtype": "bf16",
                "outputs": "gathered + normed (pair API)" if pair else "normed only",
                "l2": f"inputs rotate over {nbuf} buffer sets ({nbuf * B * S * H * 2 / 2**20:.0f} MiB > L2)"},
        dtype="bf16", cpu_sample=cpu_sample)


def wl_kv_path(args, rank, world, kt: KernelTimer):
    from fast_v2_b200 import ensure_ops

    ensure_ops()
    L, B, S, Hkv, D, rep, n = 28, 16, 4096, 4, 128, args.kv_rep, 32
    g = gen(2000 + rank)
    lens = torch.randint(256, 2049, (B,), generator=g, dtype=torch.int32)
    dg = dgen(2001 + rank)
    kc = [torch.randn(B, S, Hkv, D, generator=dg, device="cuda").to(torch.bfloat16) for _ in range(L)]
    vc = [torch.randn(B, S, Hkv, D, generator=dg, device="cuda").to(torch.bfloat16) for _ in range(L)]
    kn = [torch.randn(B, n, Hkv, D, generator=dg, device="cuda").to(torch.bfloat16) for _ in range(L)]
    vn = [torch.randn(B, n, Hkv, D, generator=dg, device="cuda").to(torch.bfloat16) for _ in range(L)]
    dlens = lens.cuda()
    lens_after = (lens + n).cuda()
    cu = torch.zeros(B + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens + n, 0)
    total = int(cu[-1])
    dcu = cu.cuda()
    ok = torch.empty(total, Hkv * rep, D, dtype=torch.bfloat16, device="cuda")
    ov = torch.empty_like(ok)
    append_bytes = 2 * L * B * n * Hkv * D * 2 * 2  # K and V, read + write
    gather_bytes_layer = total * Hkv * D * 2 * 2 * (1 + rep)  # read once, write rep times, K and V
    alg = append_bytes + L * gather_bytes_layer

    def gather(l):
        torch.ops.fdl.kv_gather_prefix(kc[l], vc[l], lens_after, None, None, rep, ok, ov, dcu, 1, 1)

    def step():
        torch.ops.fdl.kv_append(kc, vc, kn, vn, dlens)
        for l in range(L):
            gather(l)

    dstate = {"l": 0}

    def dominant():
        gather(dstate["l"] % L)
        dstate["l"] += 1

    def cpu_sample():
        from oracle import torch_port

        layers = [0, 1]
        hk = [kc[l].cpu() for l in layers]
        hv = [vc[l].cpu() for l in layers]
        t0 = time.perf_counter()
        torch_port.append_and_gather(hk, hv, kn[0].cpu(), vn[0].cpu(), lens, rep, range(len(layers)))
        dt = (time.perf_counter() - t0) / len(layers) * L
        return alg / dt / 1e9, "2 of 28 layers (append + gather + GQA expand), scaled to 28"

    return dict(
        metric="KV append + prefix gather throughput (algorithmic HBM GB/s)", unit="GB/s",
        units_per_step=alg / 1e9, step=step, dominant=dominant, graph=True, e2e_step=None, e2e_bytes=None,
        roofline=dict(bound="hbm", per_launch=gather_bytes_layer, kernel="kv_gather_prefix_kernel"),
        launches_per_step=1 + L,
        config={"workload": "kv_path", "layers": L, "batch": B, "cache": [B, S, Hkv, D], "block": n,
                "gqa_rep": rep, "sum_len": total, "l2": f"working set {2 * L * B * S * Hkv * D * 2 / 2**30:.1f} GiB > L2"},
        dtype="bf16", cpu_sample=cpu_sample)


def wl_block_attn(args, rank, world, kt: KernelTimer):
    from fast_v2_b200 import _lib, ensure_ops

    ensure_ops()
    B, P, Sq, Hq, Hkv, D = args.attn_b, args.attn_p, args.attn_sq, args.attn_hq, args.attn_hkv, 128
    cap = P + 32
    g = dgen(3000 + rank)
    kv_bytes = B * cap * Hkv * D * 2 * 2
    nbuf = max(1, math.ceil(3 * L2_BYTES / kv_bytes)) if kv_bytes < 3 * L2_BYTES else 1
    ks = [torch.randn(B, cap, Hkv, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(nbuf)]
    vs = [torch.randn(B, cap, Hkv, D, generator=g, device="cuda").to(torch.bfloat16) for _ in range(nbuf)]
    q = (torch.randn(B, Sq, Hq, D, generator=g, device="cuda") / math.sqrt(D)).to(torch.bfloat16)
    seq = torch.full((B,), cap, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    splits = args.attn_splits or _lib.attn_auto_splits(B, Sq, Hq, Hkv, cap, 0)
    wsb = _lib.attn_workspace_bytes(B, Sq, Hq, splits)
    ws = torch.empty(max(1, wsb), dtype=torch.uint8, device="cuda")
    flops = 4 * B * Hq * Sq * cap * D
    hbm_bytes = kv_bytes + 2 * B * Sq * Hq * D * 2  # K/V + Q read + O written
    state = {"i": 0}

    def step():
        i = state["i"] % nbuf
        state["i"] += 1
        torch.ops.fdl.block_attn(q, ks[i], vs[i], seq, None, None, None, 0, D ** -0.5, out,
                                 ws if wsb > 0 else None, splits)

    def cpu_sample():
        from oracle import torch_port

        bb = 1
        hq, hk, hv = q[:bb].cpu(), ks[0][:bb].cpu(), vs[0][:bb].cpu()
        t0 = time.perf_counter()
        nrep = 0
        while time.perf_counter() - t0 < args.cpu_seconds or nrep < 1:
            torch_port.flash_kvcache_sdpa(hq, hk, hv, seq[:bb].cpu(), D ** -0.5)
            nrep += 1
        dt = (time.perf_counter() - t0) / nrep
        return flops / B * bb / dt / 1e12, f"{nrep} calls of 1 of {B} sequences (SDPA, GQA expand, seqused mask)"

    return dict(
        metric="block attention throughput (TFLOP/s)", unit="TFLOP/s", units_per_step=flops / 1e12, step=step,
        dominant=step, graph=True, e2e_step=None, e2e_bytes=None,
        roofline=dict(bound="tensor", per_launch=flops, kernel="block_attn_kernel", hbm_bytes=hbm_bytes),
        launches_per_step=1 + (1 if splits > 1 else 0),
        config={"workload": "block_attn", "batch": B, "prefix": P, "q_rows": Sq, "heads": [Hq, Hkv], "splits": splits,
                "l2": f"K/V {kv_bytes / 2**20:.0f} MiB x {nbuf} buffer sets"},
        dtype="bf16", cpu_sample=cpu_sample)


_CPU_CACHE = {}


def _cpu_time(layers, pk, pv, emb, ids, geod, past, nl):
    from oracle import torch_port

    dt = emb.dtype
    t0 = time.perf_counter()
    torch_port.dkv_full_step_forward(layers, emb[:1024], torch.ones(geod["hidden"], dtype=dt), emb[:1024], ids, pk,
                                     pv, past, geod)
    t_layers = (time.perf_counter() - t0) / nl * geod["layers"]
    x = torch.randn(8, geod["hidden"]).to(dt)
    t1 = time.perf_counter()
    torch.nn.functional.linear(x, emb)
    t_fwd = t_layers + (time.perf_counter() - t1)
    return 1.0 / t_fwd, (f"1 sequence x 1 full dKV step of the reference torch path: {nl} of {geod['layers']} "
                         f"layers timed and scaled, lm_head on 8 rows; 1 generated token per forward")


def _e2e(args, rank, world, kt, geo_name):
    from fast_v2_b200.block_decode import QWEN25_1_5B, QWEN25_7B, BlockDiffusionDecoder, BlockDiffusionLM, param_count

    if geo_name == "7b":
        geo, B, P, G, sparse, refresh, schedule = QWEN25_7B, 64, 1024, 1024, 0.25, 4, "dkv"
        cache_desc = "dynamic block KV (dKV, refresh 4) + token-sparse prefix (top 25% by key norm, per block)"
    else:
        geo, B, P, G, sparse, refresh, schedule = QWEN25_1_5B, 16, 256, 512, None, 1, "static"
        cache_desc = ("static KV cache (batch_sample_dynamo schedule): a full-block forward every step, the "
                      "block's K/V written as scratch rows of the cache, unmasked attention over cache[:len + 32]")
    B = args.e2e_batch or B
    # The decode capacity covers every block of the run (warm-up + timed + two
    # spare); G (the configured generation length) is the minimum.
    G = max(G, 32 * (args.warmup + args.steps + 2))
    cpu_only = getattr(args, "impl", "ours") == "reference"
    # One weight replica per rank: every rank builds the same seeded weights.
    model = None if cpu_only else BlockDiffusionLM(geo, device="cuda", seed=100)
    if model is not None:
        # Random weights can put the mask token on top of the argmax, which a
        # trained model never does (and which stalls the reference's unmask
        # loop); its lm_head row is zeroed so its logit stays below the max.
        from fast_v2_b200.block_decode import MASK_ID

        model.lm_head[MASK_ID].zero_()
    meta = dict(
        metric=f"generated tokens/s ({geo_name.upper()} geometry, bs{B}/GPU, block-diffusion decode)",
        unit="tokens/s", dtype="bf16",
        config={"workload": "e2e_7b" if geo_name == "7b" else "e2e_1_5b",
                "model": f"Qwen2.5-{geo_name.upper()} geometry, random init",
                "params": param_count(geo), "batch_per_gpu": B, "prompt": P, "gen": G, "block": 32, "sub_block": 8,
                "threshold": 0.9, "cache": cache_desc, "step": "one 32-token block (diffusion steps + commit)",
                "weights": "random normal(0, 0.02); lm_head row of the mask token zeroed",
                "fed_bucket": getattr(args, "fed_bucket", 1),
                "kv_store": ("fused into the RoPE kernel" if getattr(args, "kv_store", "fused") == "fused"
                             else "separate append/scatter"),
                "l2": "weights and KV cache stream from HBM every forward (>> L2)"})
    dec = None if cpu_only else BlockDiffusionDecoder(model, B, P, G, refresh=refresh, sparse_keep=sparse,
                                                      fed_bucket=getattr(args, "fed_bucket", 1), use_graphs=True,
                                                      fused_kv_store=getattr(args, "kv_store", "fused") == "fused",
                                                      schedule=schedule)
    if not cpu_only:
        # One seeded global batch of B x world prompts; each rank decodes its
        # own contiguous shard of sequences (sequence_shard), as the
        # reference's request-level data parallelism does.
        from fast_v2_b200.sharding import sequence_shard

        all_prompts = torch.randint(0, 151643, (B * world, P), generator=gen(4000))
        first, n_local = sequence_shard(B * world, world, rank)
        prompt = all_prompts[first:first + n_local].cuda()
        max_blocks = G // 32
        with torch.no_grad():
            state = {"bridge": dec.prefill(prompt), "blocks": 0, "gen": []}
            dec.capture_all()
        torch.cuda.synchronize()
        stats = {}

        def step():
            with torch.no_grad():
                state["blk"], state["bridge"] = dec.decode_block(state["bridge"], stats=stats)
            state["gen"].append(state["blk"])
            state["blocks"] += 1

        def reserve(n):
            """Untimed: make room for n more blocks, re-running the prefill
            (fresh cache at the prompt length) when the capacity would run out."""
            if state["blocks"] + n > max_blocks - 1:
                with torch.no_grad():
                    state["bridge"] = dec.prefill(prompt)
                state["blocks"] = 0
                state["gen"] = []
                torch.cuda.synchronize()

        def full_generation():
            """The reference's own tokens/s definition (eval.py:425-429,
            515-519): one whole generation -- the prompt prefill plus every
            block of the configured generation length -- from a fresh cache.
            Returns (generated tokens, device ms)."""
            n_blk = G // 32  # the cache holds prompt + G + one block
            torch.cuda.synchronize()
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            with torch.no_grad():
                bridge = dec.prefill(prompt)
                gen_blocks = []
                for _ in range(n_blk):
                    blk, bridge = dec.decode_block(bridge, stats=stats)
                    gen_blocks.append(blk)
            e0.record()
            torch.cuda.synchronize()
            state["bridge"], state["blocks"], state["gen"] = bridge, n_blk, gen_blocks
            return B * 32 * n_blk, s0.elapsed_time(e0)

        def collect():
            """This rank's generated sequences since the last prefill: prompt
            followed by every decoded 32-token block."""
            return torch.cat([prompt] + state["gen"], dim=1)

        # e2e: the host-facing call per block -- bridge token in from pinned host
        # memory, the block's 32 tokens back to pinned host memory.
        hb = torch.empty(B, 1, dtype=torch.long).pin_memory()
        hblk = torch.empty(B, 32, dtype=torch.long).pin_memory()

        def e2e_step():
            with torch.no_grad():
                hb.copy_(state["bridge"], non_blocking=True)
                bridge = hb.to("cuda", non_blocking=True)
                state["blk"], state["bridge"] = dec.decode_block(bridge, stats=stats)
                hblk.copy_(state["blk"], non_blocking=True)
            torch.cuda.current_stream().synchronize()
            state["gen"].append(state["blk"])
            state["blocks"] += 1

        # dominant kernel of ours in the step: the block attention of a full
        # diffusion step (layer 0, current prefix state)
        st = dec.st
        q = (torch.randn(B, 32, geo.heads, geo.head_dim, device="cuda") * 0.1).to(torch.bfloat16)
        kb, vb = st.blk_k[0].transpose(1, 2), st.blk_v[0].transpose(1, 2)
        qpos = dec.pos.to(torch.int32)

        def dominant():
            st.attend(q, 0, dec.prefix, kb, vb, qpos)

        def dom_work():
            lens = float((st.sp_len[0] if sparse else st.lens).float().mean().item())
            kv = B * (lens + 32) * geo.kv_heads * geo.head_dim * 2 * 2
            flops = 4 * B * geo.heads * 32 * (lens + 32) * geo.head_dim
            return kv, flops

    def cpu_sample():
        """The reference's full dKV step on the host CPU for ONE sequence at this
        geometry (oracle/torch_port.dkv_full_step_forward): 2 layers timed and
        scaled to all layers, plus the lm_head rows; with random weights one
        token is committed per forward, so tokens/s = 1 / forward time."""
        from oracle import torch_port

        gg = torch.Generator().manual_seed(7)
        D, dt = geo.head_dim, torch.bfloat16

        def rnd(*shape):
            return torch.empty(*shape, dtype=dt).normal_(0.0, 0.02, generator=gg)

        nl = 2
        if "cpu" in _CPU_CACHE:
            layers, pk, pv, emb, ids, geod, past = _CPU_CACHE["cpu"]
            return _cpu_time(layers, pk, pv, emb, ids, geod, past, nl)
        layers = [dict(wq=rnd(geo.heads * D, geo.hidden), bq=torch.zeros(geo.heads * D, dtype=dt),
                       wk=rnd(geo.kv_heads * D, geo.hidden), bk=torch.zeros(geo.kv_heads * D, dtype=dt),
                       wv=rnd(geo.kv_heads * D, geo.hidden), bv=torch.zeros(geo.kv_heads * D, dtype=dt),
                       wo=rnd(geo.hidden, geo.heads * D), ln1=torch.ones(geo.hidden, dtype=dt),
                       ln2=torch.ones(geo.hidden, dtype=dt), wg=rnd(geo.ffn, geo.hidden), wu=rnd(geo.ffn, geo.hidden),
                       wd=rnd(geo.hidden, geo.ffn)) for _ in range(nl)]
        past = P + 64
        pl = int(math.ceil(0.25 * past)) if sparse else past
        pk = [rnd(1, geo.kv_heads, pl, D) for _ in range(nl)]
        pv = [rnd(1, geo.kv_heads, pl, D) for _ in range(nl)]
        emb = rnd(geo.vocab, geo.hidden)
        ids = torch.randint(0, 1000, (1, 32), generator=gg)
        geod = dict(head_dim=D, heads=geo.heads, kv_heads=geo.kv_heads, rope_theta=geo.rope_theta, eps=geo.eps,
                    layers=geo.layers, hidden=geo.hidden)
        _CPU_CACHE["cpu"] = (layers, pk, pv, emb, ids, geod, past)
        torch_port.dkv_full_step_forward(layers[:1], emb[:1024], torch.ones(geo.hidden, dtype=dt), emb[:1024], ids,
                                         pk, pv, past, geod)  # warm-up
        return _cpu_time(layers, pk, pv, emb, ids, geod, past, nl)

    if cpu_only:
        return dict(meta, cpu_sample=cpu_sample)
    kvb, fl = dom_work()
    return dict(meta, units_per_step=B * 32, step=step, dominant=dominant, graph=False, e2e_step=e2e_step,
                collect=collect, reserve=reserve, full_generation=full_generation,
                e2e_bytes=(B * 8, B * 32 * 8),
                roofline=dict(bound="hbm", per_launch=kvb, kernel="block_attn_kernel (full dKV step, layer 0)",
                              flops=fl, dynamic=dom_work),
                launches_per_step=None, stats=stats, cpu_sample=cpu_sample)


def wl_compact(args, rank, world, kt: KernelTimer):
    """In-place batch compaction of the 7B decode cache (28 layers of K and V
    [64, 2304, 4, 128]) after every fourth slot finished: the kernel behind
    every cache class's compact_batch, one launch for all 56 buffers."""
    from fast_v2_b200 import ensure_ops

    ensure_ops()
    L, B, S, Hkv, D = 28, 64, 2304, 4, 128
    dg = torch.Generator(device="cuda").manual_seed(4000 + rank)
    bufs = [torch.randn(B, S, Hkv, D, generator=dg, device="cuda").to(torch.bfloat16) for _ in range(2 * L)]
    keep = [i for i in range(B) if i % 4 != 3]
    act = torch.tensor(keep, dtype=torch.int64, device="cuda")
    moved = sum(1 for i, a in enumerate(keep) if a != i)
    row_bytes = S * Hkv * D * 2
    alg = 2 * moved * row_bytes * 2 * L  # read + write of every moved row

    def step():
        torch.ops.fdl.kv_compact(bufs, act)

    def cpu_sample():
        from oracle import kvcache_oracle as O

        hb = [bufs[j].cpu().view(torch.int16).numpy() for j in range(2)]
        t0 = time.perf_counter()
        for h in hb:
            O.batch_compact(h, keep)
        dt = (time.perf_counter() - t0) / len(hb) * 2 * L
        return alg / dt / 1e9, "2 of 56 buffers (t[active] gather), scaled to 56"

    return dict(
        metric="batch compaction throughput (algorithmic HBM GB/s)", unit="GB/s",
        units_per_step=alg / 1e9, step=step, dominant=step, graph=True, e2e_step=None, e2e_bytes=None,
        roofline=dict(bound="hbm", per_launch=alg, kernel="kv_compact_kernel"), launches_per_step=1,
        config={"workload": "compact", "layers": L, "cache": [B, S, Hkv, D], "kept": len(keep), "moved_rows": moved,
                "l2": f"working set {2 * L * B * row_bytes / 2**30:.1f} GiB > L2"},
        dtype="bf16", cpu_sample=cpu_sample)


def wl_swiglu(args, rank, world, kt: KernelTimer):
    """SwiGLU of the 7B MLP at a full dKV step of the e2e bench: gate/up rows
    [64 x 32, 2 x 18944] bf16 -> [2048, 18944] (silu(gate) * up, the
    reference's bf16 roundings)."""
    from fast_v2_b200 import ensure_ops

    ensure_ops()
    rows, F = 64 * 32, 18944
    dg = dgen(6000 + rank)
    per = rows * 3 * F * 2
    nbuf = max(2, math.ceil(3 * L2_BYTES / per))
    gus = [(torch.randn(rows, 2 * F, generator=dg, device="cuda") * 2).to(torch.bfloat16) for _ in range(nbuf)]
    outs = [torch.empty(rows, F, dtype=torch.bfloat16, device="cuda") for _ in range(nbuf)]
    alg = rows * F * 2 * 3  # read gate + up, write the product
    state = {"i": 0}

    def step():
        i = state["i"] % nbuf
        state["i"] += 1
        torch.ops.fdl.swiglu(gus[i], outs[i])

    def cpu_sample():
        from oracle import torch_port

        h = gus[0][:64].cpu()
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < args.cpu_seconds or n < 2:
            torch_port.swiglu(h)
            n += 1
        dt = (time.perf_counter() - t0) / n
        return alg / rows * 64 / dt / 1e9, f"{n} calls on 64 of {rows} rows (silu(gate) * up in bf16 torch)"

    return dict(
        metric="SwiGLU throughput (algorithmic HBM GB/s)", unit="GB/s", units_per_step=alg / 1e9, step=step,
        dominant=step, graph=True, e2e_step=None, e2e_bytes=None,
        roofline=dict(bound="hbm", per_launch=alg, kernel="swiglu_kernel"), launches_per_step=1,
        config={"workload": "swiglu", "rows": rows, "ffn": F, "shape": "7B MLP, full dKV step of 64 sequences",
                "l2": f"inputs rotate over {nbuf} buffer sets"},
        dtype="bf16", cpu_sample=cpu_sample)


def wl_add_rmsnorm(args, rank, world, kt: KernelTimer):
    """Residual add + RMSNorm of the 7B decoder layer at a full dKV step:
    h += y (bf16) and normed = RMSNorm(h) * w over [2048, 3584] rows."""
    from fast_v2_b200 import ensure_ops

    ensure_ops()
    rows, H = 64 * 32, 3584
    dg = dgen(6100 + rank)
    per = rows * H * 2 * 4
    nbuf = max(2, math.ceil(3 * L2_BYTES / per))
    ys = [torch.randn(rows, H, generator=dg, device="cuda").to(torch.bfloat16) for _ in range(nbuf)]
    hs = [torch.randn(rows, H, generator=dg, device="cuda").to(torch.bfloat16) for _ in range(nbuf)]
    outs = [torch.empty(rows, H, dtype=torch.bfloat16, device="cuda") for _ in range(nbuf)]
    w = torch.ones(H, dtype=torch.bfloat16, device="cuda")
    alg = rows * H * 2 * 4  # read y and h; write h and normed
    state = {"i": 0}

    def step():
        i = state["i"] % nbuf
        state["i"] += 1
        torch.ops.fdl.add_rmsnorm(ys[i], hs[i], w, 1e-6, hs[i], outs[i])

    def cpu_sample():
        from oracle import torch_port

        y, h, wc = ys[0][:64].cpu(), hs[0][:64].cpu(), w.cpu()
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < args.cpu_seconds or n < 2:
            torch_port.rmsnorm(h + y, wc, 1e-6)
            n += 1
        dt = (time.perf_counter() - t0) / n
        return alg / rows * 64 / dt / 1e9, f"{n} calls on 64 of {rows} rows (residual add + Qwen RMSNorm in torch)"

    return dict(
        metric="residual add + RMSNorm throughput (algorithmic HBM GB/s)", unit="GB/s", units_per_step=alg / 1e9,
        step=step, dominant=step, graph=True, e2e_step=None, e2e_bytes=None,
        roofline=dict(bound="hbm", per_launch=alg, kernel="gather_rmsnorm_kernel (residual form)"),
        launches_per_step=1,
        config={"workload": "add_rmsnorm", "rows": rows, "hidden": H, "shape": "7B layer, full dKV step of 64 sequences",
                "l2": f"inputs rotate over {nbuf} buffer sets"},
        dtype="bf16", cpu_sample=cpu_sample)


def wl_e2e_7b(args, rank, world, kt):
    return _e2e(args, rank, world, kt, "7b")


def wl_e2e_1_5b(args, rank, world, kt):
    return _e2e(args, rank, world, kt, "1.5b")


WORKLOADS = {"gather_norm": wl_gather_norm, "kv_path": wl_kv_path, "block_attn": wl_block_attn, "compact": wl_compact,
             "swiglu": wl_swiglu, "add_rmsnorm": wl_add_rmsnorm, "e2e_7b": wl_e2e_7b, "e2e_1_5b": wl_e2e_1_5b}
DEFAULT_CONFIG = "e2e_7b"


# --------------------------------------------------------------------------
# reference arm: the reference's torch path on the host CPU
# --------------------------------------------------------------------------
def run_reference(args, world, rank):
    if rank != 0:
        return None
    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()

    class _Noop:
        active = False

        def wrap(self, fn):
            return fn()

    # Build the same workload on CPU-sized samples: reuse the cpu_sample hooks,
    # which time the restated reference torch path on this host.
    import types

    fake_args = types.SimpleNamespace(**vars(args))
    if not torch.cuda.is_available() and not args.config.startswith("e2e"):
        raise SystemExit(json.dumps({"impl": "reference", "unavailable": "needs the GPU box to stage inputs"}))
    w = WORKLOADS[args.config](fake_args, 0, 1, _Noop())
    vals = []
    for _ in range(args.warmup):
        w["cpu_sample"]()
    t_all = time.perf_counter()
    sample = ""
    for _ in range(args.steps):
        v, sample = w["cpu_sample"]()
        vals.append(v)
    wall = time.perf_counter() - t_all
    value = statistics.median(vals)
    # tokens/s samples commit one token per forward of one sequence, so one
    # step of this arm is one (scaled) forward: 1000 / value ms.  Otherwise a
    # step is one sample call.
    ms_step = 1e3 / value if w["unit"] == "tokens/s" else wall / max(1, args.steps) * 1e3
    line = {
        "impl": "reference", "metric": w["metric"], "value": value, "unit": w["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": w["dtype"],
        "data": "synthetic", "config": w["config"],
        "cpu_baseline": {"value": value, "unit": w["unit"], "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": w["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


# --------------------------------------------------------------------------
# measurement helpers
# --------------------------------------------------------------------------
def timed_region(w, steps, world, stream, sampler=None):
    """W warm-up steps are the caller's; here: optional CUDA-graph capture of
    the K steps, then the timed region bracketed by barrier + synchronize,
    CUDA events on the launching stream.  Returns (max-over-ranks ms, host
    launch tally inside the region, wall-clock window)."""
    from fast_v2_b200 import _lib as _fdl_lib

    graph = None
    if w.get("graph"):
        # Kernel-level configs: the K steps are replayed from a CUDA graph so
        # the device time is not diluted by host dispatch gaps.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(steps):
                w["step"]()
        graph.replay()
        barrier(world)
    if sampler is not None:
        sampler.start()
    barrier(world)
    launches0 = _fdl_lib.launches
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    start.record(stream)
    if graph is not None:
        graph.replay()
    else:
        for _ in range(steps):
            w["step"]()
    end.record(stream)
    torch.cuda.synchronize()
    t1 = time.time()
    launches = _fdl_lib.launches - launches0
    if sampler is not None:
        sampler.mark(t0, t1)
    barrier(world)
    if sampler is not None:
        sampler.stop()
    del graph
    return max_over_ranks(start.elapsed_time(end), world), launches, (t0, t1)


def launch_ms(fn, n, stream):
    """Mean duration of fn's own launches: n of them back to back in a CUDA
    graph, CUDA events on the launching stream."""
    gd = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gd):
        for _ in range(n):
            fn()
    gd.replay()
    torch.cuda.synchronize()
    s1, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s1.record(stream)
    gd.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    del gd
    return s1.elapsed_time(e1) / n


def roofline_of(rf, kms, peaks, traffic_key=None):
    if not kms:
        return None
    if rf["bound"] == "hbm":
        ach = rf["per_launch"] / (kms / 1e3) / 1e9
        peak = peaks["hbm_gbs"]
        roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                "traffic": None, "kernel": rf["kernel"], "launch_us": round(kms * 1e3, 2),
                "alg_bytes_per_launch": int(rf["per_launch"]), "peak_src": peaks["src"]}
        if rf.get("flops"):
            roof["tflops_achieved"] = round(rf["flops"] / (kms / 1e3) / 1e12, 1)
    else:
        ach = rf["per_launch"] / (kms / 1e3) / 1e12
        peak = peaks["bf16_tflops"]
        roof = {"bound": "tensor", "achieved": round(ach, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(ach / peak, 4), "traffic": None, "kernel": rf["kernel"], "launch_us": round(kms * 1e3, 2),
                "alg_flops_per_launch": int(rf["per_launch"]), "peak_src": peaks["src"]}
        if rf.get("hbm_bytes"):
            roof["hbm_gbs_achieved"] = round(rf["hbm_bytes"] / (kms / 1e3) / 1e9, 1)
            roof["hbm_frac"] = round(rf["hbm_bytes"] / (kms / 1e3) / 1e9 / peaks["hbm_gbs"], 4)
    tr = ROOT / "profiles" / "traffic.json"
    if traffic_key and tr.exists():
        t = json.loads(tr.read_text()).get(traffic_key)
        if t:
            roof["traffic"] = t
    return roof


def kernel_breakdown(fn):
    """Device time per kernel name over one call of fn (one untimed decode
    block), from a CUDA activity trace (torch.profiler / CUPTI).  This is an
    attribution of the step's device time to kernels, not a bench value.
    Returns [(name, launches, total_ms)] sorted by time, or None."""
    try:
        from torch.autograd import DeviceType
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        agg = {}
        for e in prof.events():
            if getattr(e, "device_type", None) != DeviceType.CUDA:
                continue
            name = e.name
            if name.startswith("Memcpy") or name.startswith("Memset"):
                continue
            dur = e.time_range.elapsed_us() / 1e3
            n, t = agg.get(name, (0, 0.0))
            agg[name] = (n + 1, t + dur)
        rows = sorted(((k, n, t) for k, (n, t) in agg.items()), key=lambda r: -r[2])
        return rows or None
    except Exception as ex:  # the trace is optional evidence; never fail the bench on it
        sys.stderr.write(f"kernel breakdown unavailable: {ex}\n")
        return None


def short_kernel_name(name: str) -> str:
    n = name
    for pre in ("void ",):
        if n.startswith(pre):
            n = n[len(pre):]
    return n.split("(")[0][:90]


# Kernel-level configs measured inside the default run (BASELINE configs 1-3
# and the two largest kernels of ours in the e2e step), each on its own
# inputs, after the headline's timed region.
KERNEL_SUITE = [
    ("gather_norm", {}, 400),
    ("kv_path", {}, 20),
    ("block_attn", {"attn_b": 64, "attn_p": 8192, "attn_sq": 32}, 40),
    ("block_attn", {"attn_b": 16, "attn_p": 8192, "attn_sq": 32}, 100),
    ("block_attn", {"attn_b": 16, "attn_p": 4096, "attn_sq": 32}, 150),
    ("block_attn", {"attn_b": 64, "attn_p": 8192, "attn_sq": 8}, 100),
    ("swiglu", {}, 200),
    ("add_rmsnorm", {}, 400),
]


def run_kernel_suite(args, rank, world, peaks, stream):
    import copy
    import gc

    out = {}
    for name, over, steps in KERNEL_SUITE:
        a = copy.copy(args)
        for k2, v2 in over.items():
            setattr(a, k2, v2)
        a.cpu_seconds = 2.0
        w = WORKLOADS[name](a, rank, world, KernelTimer())
        for _ in range(3):
            w["step"]()
        torch.cuda.synchronize()
        ms, _, _ = timed_region(w, steps, world, stream)
        value = w["units_per_step"] * steps * world / (ms / 1e3)
        kms = launch_ms(w["dominant"], max(20, min(200, steps)), stream)
        key = name if not over else f"{name}_b{a.attn_b}_p{a.attn_p}_sq{a.attn_sq}"
        cpu = None
        if rank == 0 and not args.no_cpu_baseline:
            v, sample = w["cpu_sample"]()
            cpu = {"value": v, "unit": w["unit"], "cores": torch.get_num_threads(), "kind": "port", "sample": sample}
        out[key] = {"metric": w["metric"], "value": value, "unit": w["unit"], "steps": steps,
                    "ms_per_step": ms / steps, "roofline": roofline_of(w["roofline"], kms, peaks, key),
                    "config": w["config"], "cpu_baseline": cpu}
        w.clear()
        del w
        gc.collect()
        torch.cuda.empty_cache()
    return out


def e2e_dominant(breakdown, geo_B=64):
    """The largest kernel of ours in the e2e step by device time, with a
    standalone workload of the same launch shape to time it."""
    cands = {"swiglu_kernel": "swiglu", "gather_rmsnorm_kernel": "add_rmsnorm", "block_attn_kernel": "block_attn_e2e"}
    if breakdown:
        for nm, _, _ in breakdown:
            for c, wl in cands.items():
                if c in nm:
                    return c, wl
    return "swiglu_kernel", "swiglu"


# --------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(WORKLOADS), default=DEFAULT_CONFIG)
    ap.add_argument("--attn-b", type=int, default=64)
    ap.add_argument("--attn-p", type=int, default=8192)
    ap.add_argument("--attn-sq", type=int, default=32)
    ap.add_argument("--attn-hq", type=int, default=28)
    ap.add_argument("--attn-hkv", type=int, default=4)
    ap.add_argument("--attn-splits", type=int, default=0, help="0 = the library's split-KV choice")
    ap.add_argument("--e2e-batch", type=int, default=0)
    ap.add_argument("--kv-rep", type=int, default=7, help="kv_path: GQA expansion factor of the gather (1 = none)")
    ap.add_argument("--norm-only", action="store_true", help="gather_norm: write only the normed rows")
    ap.add_argument("--fed-bucket", type=int, default=1,
                    help="cached dKV steps run at the fed width rounded up to this multiple (1 = exact, as the reference)")
    ap.add_argument("--kv-store", choices=["fused", "separate"], default="fused",
                    help="e2e: 'fused' = the RoPE kernel stores K/V into the cache itself; 'separate' = RoPE, then "
                         "an append / scatter launch")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernels", action="store_true",
                    help="e2e configs at N=1: skip the kernel-level measurements added to the line")
    ap.add_argument("--cpu-seconds", type=float, default=8.0, help="length of each CPU-baseline sample")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {"gather_norm": 2000, "kv_path": 100, "block_attn": 200, "swiglu": 500,
                      "add_rmsnorm": 1000}.get(args.config, 8)
    args.warmup = max(3, args.warmup)
    world, rank, local = setup_dist()

    if args.impl == "reference":
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    from fast_v2_b200 import _lib as _fdl_lib

    peaks = load_peaks()
    kt = KernelTimer()
    w = WORKLOADS[args.config](args, rank, world, kt)
    meta = {k: w[k] for k in ("metric", "unit", "config", "launches_per_step", "dtype")}
    for _ in range(args.warmup):
        w["step"]()
    barrier(world)
    _fdl_lib.check_device("bench warm-up")
    stream = torch.cuda.current_stream()
    sampler = ClockSampler(local)
    kt.active = not w.get("graph")
    ms_max, launches_timed, _ = timed_region(w, args.steps, world, stream, sampler)
    kt.active = False
    _fdl_lib.check_device("bench timed region")
    value = w["units_per_step"] * args.steps * world / (ms_max / 1e3)

    # end-to-end through the public API with host buffers
    e2e = None
    if w.get("e2e_step"):
        n_e2e = max(3, min(args.steps, 50))
        if w.get("reserve"):
            w["reserve"](n_e2e + 2)
        for _ in range(2):
            w["e2e_step"]()
        barrier(world)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(n_e2e):
            w["e2e_step"]()
        e2.record()
        torch.cuda.synchronize()
        ms2 = max_over_ranks(s2.elapsed_time(e2), world)
        e2e = {"value": w["units_per_step"] * n_e2e * world / (ms2 / 1e3), "unit": w["unit"],
               "h2d_bytes_per_step": w["e2e_bytes"][0], "d2h_bytes_per_step": w["e2e_bytes"][1]}
        _fdl_lib.check_device("bench end-to-end region")

    # One whole generation (prefill + all blocks), as the reference counts
    # tokens/s; device time, max over ranks.
    full_gen = None
    if w.get("full_generation") is not None:
        toks, fms = w["full_generation"]()
        fms = max_over_ranks(fms, world)
        full_gen = {"value": toks * world / (fms / 1e3), "unit": "tokens/s", "generated_tokens": toks * world,
                    "seconds": fms / 1e3, "includes": "prompt prefill + every 32-token block of the generation"}
        _fdl_lib.check_device("bench full generation")

    # Sequence-sharded output: one all-gather of every rank's whole generated
    # sequences (prompt + all blocks of the generation just timed), the only
    # collective besides the max-time reductions.
    collected = None
    if world > 1 and w.get("collect"):
        from fast_v2_b200.sharding import gather_generated

        collected = list(gather_generated(w["collect"](), pad_id=-1).shape)

    # Roofline of the dominant kernel.  Kernel-level configs: the config's own
    # kernel.  e2e configs: the largest kernel of this library in the step by
    # device time (attribution from one untimed, traced block), timed alone at
    # the step's full-block launch shape.
    rf = w["roofline"]
    breakdown = None
    dom_shares = None
    if w.get("stats") is not None and w.get("e2e_step"):
        if w.get("reserve"):
            w["reserve"](2)
        breakdown = kernel_breakdown(w["step"])
        if breakdown:
            total = sum(t for _, _, t in breakdown)
            ours = [(short_kernel_name(n), c, t) for n, c, t in breakdown if "fdl::" in n]
            dom_shares = {"source": "one untimed decode block, CUDA activity trace (torch.profiler)",
                          "device_ms": round(total, 2),
                          "fdl_share": round(sum(t for _, _, t in ours) / total, 4),
                          "fdl_kernels": [{"kernel": n, "launches": c, "ms": round(t, 3), "share": round(t / total, 4)}
                                          for n, c, t in ours[:8]],
                          "top_kernels": [{"kernel": short_kernel_name(n), "launches": c, "ms": round(t, 3),
                                           "share": round(t / total, 4)} for n, c, t in breakdown[:6]]}
    traffic_key = args.config
    kname = None
    if w.get("stats") is not None:
        kname, wl_name = e2e_dominant(breakdown)
        import copy

        a2 = copy.copy(args)
        a2.cpu_seconds = 1.0
        if wl_name == "block_attn_e2e":
            # The full dKV step's attention at the bench's mean shape: 64
            # sequences, a ~384-token sparse prefix plus the 32-key block, 32
            # queries; HBM-bound there (176 FLOP/B, below the ridge).
            a2.attn_b, a2.attn_p, a2.attn_sq = 64, 384, 32
            if args.config == "e2e_1_5b":  # 1.5B geometry: 16 sequences over the full prefix
                a2.attn_b, a2.attn_p, a2.attn_hq, a2.attn_hkv = 16, 512, 12, 2
            wd = WORKLOADS["block_attn"](a2, rank, world, KernelTimer())
            rf = dict(wd["roofline"])
            rf.update(bound="hbm", per_launch=rf["hbm_bytes"], flops=wd["units_per_step"] * 1e12,
                      kernel=f"{kname} at the e2e full-step shape ({a2.attn_b} sequences x ({a2.attn_p} + 32) keys, "
                             f"32 queries)")
        else:
            wd = WORKLOADS[wl_name](a2, rank, world, KernelTimer())
            rf = dict(wd["roofline"])
            rf["kernel"] = f"{kname} at the e2e full-block launch shape ({wd['config']['rows']} rows)"
        kms = launch_ms(wd["dominant"], 200, stream)
        traffic_key = wl_name if args.config == "e2e_7b" else None
        wd.clear()
    elif w.get("dominant") is not None:
        kms = launch_ms(w["dominant"], max(20, min(500, args.steps)), stream)
    else:
        kms = kt.avg_ms()
    roof = roofline_of(rf, kms, peaks, traffic_key)
    if roof is not None and dom_shares is not None:
        for k in dom_shares["fdl_kernels"]:
            if kname in k["kernel"]:
                roof["share_of_step"] = k["share"]
                break
        roof["step_breakdown"] = dom_shares

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        v, sample = w["cpu_sample"]()
        cpu = {"value": v, "unit": w["unit"], "cores": torch.get_num_threads(), "kind": "port", "sample": sample}
    clocks = sampler.summary()

    kernels = None
    if world == 1 and w.get("stats") is not None and not args.no_kernels:
        import gc

        w.clear()
        del w
        gc.collect()
        torch.cuda.empty_cache()
        kernels = run_kernel_suite(args, rank, world, peaks, stream)
        w = {}
    _fdl_lib.check_device("bench kernel measurements")

    if rank == 0:
        line = {
            "metric": meta["metric"], "value": value, "unit": meta["unit"], "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": meta["dtype"], "data": "synthetic",
            "config": {**meta["config"], "parallelism": f"dp{world} (sequence-sharded replicas)",
                       **({"gathered_sequences": collected} if collected else {})},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks,
            "gpu_launches": (meta["launches_per_step"] * args.steps
                             if meta["launches_per_step"] is not None else launches_timed),
            "device_status": 0,
        }
        if full_gen is not None:
            line["full_generation"] = full_gen
        if kernels is not None:
            line["kernels"] = kernels
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
