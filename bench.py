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
                static cache (full block recompute every step)

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


def wl_gather_norm(args, rank, world, kt: KernelTimer):
    import numpy as np

    from fast_v2_b200 import ensure_ops

    ensure_ops()
    B, S, H, T = 4, 2048, 3584, 512
    nbuf = max(2, math.ceil(3 * L2_BYTES / (B * S * H * 2)))
    g = gen(1000 + rank)
    xs = [torch.randn(B, S, H, generator=g).to(torch.bfloat16).cuda() for _ in range(nbuf)]
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
        while time.perf_counter() - t0 < 8.0 or n < 2:
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
    kc = [torch.randn(B, S, Hkv, D, generator=g).to(torch.bfloat16).cuda() for _ in range(L)]
    vc = [torch.randn(B, S, Hkv, D, generator=g).to(torch.bfloat16).cuda() for _ in range(L)]
    kn = [torch.randn(B, n, Hkv, D, generator=g).to(torch.bfloat16).cuda() for _ in range(L)]
    vn = [torch.randn(B, n, Hkv, D, generator=g).to(torch.bfloat16).cuda() for _ in range(L)]
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
    g = gen(3000 + rank)
    kv_bytes = B * cap * Hkv * D * 2 * 2
    nbuf = max(1, math.ceil(3 * L2_BYTES / kv_bytes)) if kv_bytes < 3 * L2_BYTES else 1
    ks = [torch.randn(B, cap, Hkv, D, generator=g).to(torch.bfloat16).cuda() for _ in range(nbuf)]
    vs = [torch.randn(B, cap, Hkv, D, generator=g).to(torch.bfloat16).cuda() for _ in range(nbuf)]
    q = (torch.randn(B, Sq, Hq, D, generator=g) / math.sqrt(D)).to(torch.bfloat16).cuda()
    seq = torch.full((B,), cap, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    splits = args.attn_splits or _lib.attn_auto_splits(B, Sq, Hq, Hkv, cap, 0)
    wsb = _lib.attn_workspace_bytes(B, Sq, Hq, splits)
    ws = torch.empty(max(1, wsb), dtype=torch.uint8, device="cuda")
    flops = 4 * B * Hq * Sq * cap * D
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
        while time.perf_counter() - t0 < 8.0 or nrep < 1:
            torch_port.flash_kvcache_sdpa(hq, hk, hv, seq[:bb].cpu(), D ** -0.5)
            nrep += 1
        dt = (time.perf_counter() - t0) / nrep
        return flops / B * bb / dt / 1e12, f"{nrep} calls of 1 of {B} sequences (SDPA, GQA expand, seqused mask)"

    return dict(
        metric="block attention throughput (TFLOP/s)", unit="TFLOP/s", units_per_step=flops / 1e12, step=step,
        dominant=step, graph=True, e2e_step=None, e2e_bytes=None,
        roofline=dict(bound="tensor", per_launch=flops, kernel="block_attn_kernel", hbm_bytes=kv_bytes),
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
        geo, B, P, G, sparse, refresh = QWEN25_7B, 64, 1024, 1024, 0.25, 4
        cache_desc = "dynamic block KV (dKV, refresh 4) + token-sparse prefix (top 25% by key norm, per block)"
    else:
        geo, B, P, G, sparse, refresh = QWEN25_1_5B, 16, 256, 512, None, 1
        cache_desc = "static KV cache, full block recompute every step"
    B = args.e2e_batch or B
    # The decode capacity covers every block of the run (warm-up + timed + two
    # spare); G (the configured generation length) is the minimum.
    G = max(G, 32 * (args.warmup + args.steps + 2))
    cpu_only = getattr(args, "impl", "ours") == "reference"
    model = None if cpu_only else BlockDiffusionLM(geo, device="cuda", seed=100 + rank)
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
                "l2": "weights and KV cache stream from HBM every forward (>> L2)"})
    dec = None if cpu_only else BlockDiffusionDecoder(model, B, P, G, refresh=refresh, sparse_keep=sparse,
                                                      fed_bucket=getattr(args, "fed_bucket", 1), use_graphs=True)
    g = gen(4000 + rank)
    if not cpu_only:
        prompt = torch.randint(0, 151643, (B, P), generator=g).cuda()
        max_blocks = G // 32
        with torch.no_grad():
            state = {"bridge": dec.prefill(prompt), "blocks": 0}
            dec.capture_all()
        torch.cuda.synchronize()
        stats = {}

        def step():
            with torch.no_grad():
                state["blk"], state["bridge"] = dec.decode_block(state["bridge"], stats=stats)
            state["blocks"] += 1

        def reserve(n):
            """Untimed: make room for n more blocks, re-running the prefill
            (fresh cache at the prompt length) when the capacity would run out."""
            if state["blocks"] + n > max_blocks - 1:
                with torch.no_grad():
                    state["bridge"] = dec.prefill(prompt)
                state["blocks"] = 0
                torch.cuda.synchronize()

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
                collect=lambda: state["blk"], reserve=reserve,
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


def wl_e2e_7b(args, rank, world, kt):
    return _e2e(args, rank, world, kt, "7b")


def wl_e2e_1_5b(args, rank, world, kt):
    return _e2e(args, rank, world, kt, "1.5b")


WORKLOADS = {"gather_norm": wl_gather_norm, "kv_path": wl_kv_path, "block_attn": wl_block_attn, "compact": wl_compact,
             "e2e_7b": wl_e2e_7b, "e2e_1_5b": wl_e2e_1_5b}
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
    line = {
        "impl": "reference", "metric": w["metric"], "value": value, "unit": w["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall / max(1, args.steps) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": w["dtype"],
        "data": "synthetic", "config": w["config"],
        "cpu_baseline": {"value": value, "unit": w["unit"], "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": w["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


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
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {"gather_norm": 2000, "kv_path": 100, "block_attn": 200}.get(args.config, 8)
    args.warmup = max(3, args.warmup)
    world, rank, local = setup_dist()

    if args.impl == "reference":
        line = run_reference(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    peaks = load_peaks()
    kt = KernelTimer()
    w = WORKLOADS[args.config](args, rank, world, kt)
    for _ in range(args.warmup):
        w["step"]()
    barrier(world)
    stream = torch.cuda.current_stream()
    graph = None
    if w.get("graph"):
        # Kernel-level configs: the K steps are replayed from a CUDA graph so
        # the device time is not diluted by host dispatch gaps.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                w["step"]()
        graph.replay()
        barrier(world)
    sampler = ClockSampler(local)
    sampler.start()
    barrier(world)
    kt.active = not w.get("graph")
    from fast_v2_b200 import _lib as _fdl_lib
    launches0 = _fdl_lib.launches
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    start.record(stream)
    if graph is not None:
        graph.replay()
    else:
        for _ in range(args.steps):
            w["step"]()
    end.record(stream)
    torch.cuda.synchronize()
    t1 = time.time()
    kt.active = False
    launches_timed = _fdl_lib.launches - launches0
    sampler.mark(t0, t1)
    barrier(world)
    sampler.stop()
    ms = start.elapsed_time(end)
    ms_max = max_over_ranks(ms, world)
    value = w["units_per_step"] * args.steps * world / (ms_max / 1e3)
    del graph

    # dominant-kernel duration: its own launches back to back in a CUDA graph,
    # timed with events on the launching stream.
    rf = w["roofline"]
    kms = None
    if w.get("dominant") is not None:
        n_dom = max(20, min(500, args.steps))
        gd = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gd):
            for _ in range(n_dom):
                w["dominant"]()
        gd.replay()
        torch.cuda.synchronize()
        s1, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s1.record(stream)
        gd.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        kms = s1.elapsed_time(e1) / n_dom
        del gd
    else:
        kms = kt.avg_ms()
    roof = None
    if rf.get("dynamic"):
        rf["per_launch"], rf["flops"] = rf["dynamic"]()
    if kms:
        if rf["bound"] == "hbm":
            ach = rf["per_launch"] / (kms / 1e3) / 1e9
            peak = peaks["hbm_gbs"]
            roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(ach / peak, 4), "traffic": None, "kernel": rf["kernel"],
                    "launch_us": round(kms * 1e3, 2), "peak_src": peaks["src"]}
            if rf.get("flops"):
                roof["tflops_achieved"] = round(rf["flops"] / (kms / 1e3) / 1e12, 1)
        else:
            ach = rf["per_launch"] / (kms / 1e3) / 1e12
            peak = peaks["bf16_tflops"]
            roof = {"bound": "tensor", "achieved": round(ach, 1), "peak": peak, "unit": "TFLOP/s",
                    "frac": round(ach / peak, 4), "traffic": None, "kernel": rf["kernel"],
                    "launch_us": round(kms * 1e3, 2), "peak_src": peaks["src"]}
            if rf.get("hbm_bytes"):
                roof["hbm_gbs_achieved"] = round(rf["hbm_bytes"] / (kms / 1e3) / 1e9, 1)
        tr = ROOT / "profiles" / "traffic.json"
        if tr.exists():
            t = json.loads(tr.read_text()).get(args.config)
            if t:
                roof["traffic"] = t

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

    # Sequence-sharded output: one all-gather of every rank's last generated
    # block after the timed regions (the only collective besides the max-time
    # reduction).
    collected = None
    if world > 1 and w.get("collect"):
        from fast_v2_b200.sharding import gather_generated

        collected = list(gather_generated(w["collect"](), pad_id=-1).shape)

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        v, sample = w["cpu_sample"]()
        cpu = {"value": v, "unit": w["unit"], "cores": torch.get_num_threads(), "kind": "port", "sample": sample}

    if rank == 0:
        line = {
            "metric": w["metric"], "value": value, "unit": w["unit"], "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": w["dtype"], "data": "synthetic",
            "config": {**w["config"], "parallelism": f"dp{world} (sequence-sharded replicas)",
                       **({"gathered_block": collected} if collected else {})},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": sampler.summary(),
            "gpu_launches": (w["launches_per_step"] * args.steps if w["launches_per_step"] is not None
                             else launches_timed),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
