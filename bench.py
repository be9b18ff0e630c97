#!/usr/bin/env python
"""Benchmark of the per-token decoder elementwise path (NanoInfer hot path).

Workload: config C5 (Qwen3-VL-2B shapes: hidden 2048, 16 q / 8 kv heads of
128, intermediate 6144, interleaved M-RoPE [24,20,20] theta 5e6, q/k text
norm). One STEP = 262,144 tokens through 28 fused layers plus the paged-KV
gather of 64 sequences x 16,384 tokens (K and V caches). The tokens and
sequences are split evenly over the ranks (strong scaling: total work per
step is fixed); every rank owns its own 16,384 x 256-slot K/V cache pair and
there is no collective on the data path.

A fused layer = residual add + input text norm, the attention prologue (q/k
norm + M-RoPE + paged store), residual add + post-attention norm, and
SiluAndMul. The projections that feed it (qkv, o_proj, gate_up, down_proj)
are out of scope: their outputs are fixed synthetic device tensors.

``value``  = token x layer passes per second with inputs resident in HBM
             (CUDA events on the launch stream, max over ranks).
``e2e``    = the same through the layer-module API with the step's host inputs
             (initial hidden states, positions, slot mapping) copied from
             pinned memory and the final hidden states copied back each step.
``--impl reference`` times the reference's CPU path on the host cores, rank 0
only: its own modules when an install is importable (``baseline/_ref`` or
``$NANOINFER_REF``), else the oracle port, on a bounded sample of the C5 step
extrapolated by per-token cost. The ``cpu_baseline`` leg of the GPU line is the
same measurement.

``configs`` = C1-C4 (the other BASELINE configs): each config's fused layer on
the GPU (CUDA-graph replay, inputs rotated past the L2) next to the same layer
on the CPU over the config's full token count.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

TOKENS = 262144
LAYERS = 28
GATHER_SEQS = 64
GATHER_LEN = 16384
CACHE_BLOCKS = 16384
H, NQ, NKV, D, INTER = 2048, 16, 8, 128, 6144
SECTIONS = (24, 20, 20)
THETA = 5e6
EPS = 1e-6
METRIC = "fused-layer tokens/s"
UNIT = "tokens/s"

# algorithmic bytes per token (bf16) of each kernel of the fused layer
BYTES = {
    "add_rms_norm": 8 * H,                                                    # x, res in; y, res out
    "qk_prologue": 2 * ((NQ + 2 * NKV) * D + NQ * D + NKV * D + 2 * NKV * D) + 8 * 3 + 4,
    "silu_and_mul": 6 * INTER,                                                # gate, up in; out
    "paged_gather": 2 * 2 * NKV * D,                                          # cache row in, out row
}
LAYER_BYTES = 2 * BYTES["add_rms_norm"] + BYTES["qk_prologue"] + BYTES["silu_and_mul"]


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--tokens", type=int, default=TOKENS, help="tokens per step (whole job)")
    p.add_argument("--layers", type=int, default=LAYERS)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-components", action="store_true", help="skip the per-kernel extras")
    p.add_argument("--component",
                   choices=("decode_attention", "step_inputs", "mrope", "rows", "visual_merge", "paged_store",
                            "head_norm", "decode_layers", "configs"),
                   default=None,
                   help="run only this standalone component (one GPU) and print its JSON")
    p.add_argument("--decode-requests", type=int, default=256,
                   help="requests of the decode-attention component (C2: 256)")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    p.add_argument("--no-configs", action="store_true", help="skip the C1-C4 table")
    p.add_argument("--config-cpu-seconds", type=float, default=2.0,
                   help="CPU budget per config of the C1-C4 table")
    p.add_argument("--cache-blocks", type=int, default=CACHE_BLOCKS,
                   help="blocks of 256 slots per K/V cache per GPU (smaller only for profiler captures)")
    return p.parse_args(argv)


# ------------------------------------------------------------------ distributed plumbing


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def shard(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous even split of ``n`` units: rank r gets [start, start + count)."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def max_over_ranks(value: float, world: int, device=None) -> float:
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ------------------------------------------------------------------ clocks


def physical_gpu(local: int) -> str:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if local < len(ids):
            return ids[local]
    return str(local)


class ClockSampler:
    """Samples ``nvidia-smi`` SM clocks / throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        return summarize_clocks(self.lines)


def summarize_clocks(lines: list[str]) -> dict | None:
    sm, smax, reasons = [], [], set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in lines:
        f = [x.strip() for x in line.split(",")]
        if len(f) < 9:
            continue
        try:
            sm.append(float(f[1]))
            smax.append(float(f[2]))
        except ValueError:
            continue
        for name, flag in zip(names, f[5:9]):
            if flag.lower() == "active":
                reasons.add(name)
    if not sm:
        return None
    top = max(sm)
    loaded = [s for s in sm if s >= 0.5 * top] or sm
    return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax) if smax else None,
            "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ GPU workload


def make_rank_inputs(rank: int, world: int, tokens_total: int, device, cache_blocks: int = CACHE_BLOCKS):
    from nano_vllm_multimodal_b200 import workloads as W

    t0, T = shard(tokens_total, rank, world)
    s0, S = shard(GATHER_SEQS, rank, world)
    seeds = W._Seeds(5, device)
    seeds.index = 100 * (rank + 1)
    n = lambda shape, mean=0.0, std=1.0: W._normal(seeds, shape, mean, std)  # noqa: E731
    inp = {
        "tokens": T,
        "hidden": n((T, H)), "residual": n((T, H)), "qkv": n((T, (NQ + 2 * NKV) * D)),
        "attn_out": n((T, H)), "gate_up": n((T, 2 * INTER)), "mlp_out": n((T, H)),
        "w_in": n((H,), 1.0, 0.1), "w_post": n((H,), 1.0, 0.1),
        "q_weight": n((D,), 1.0, 0.1), "k_weight": n((D,), 1.0, 0.1),
        "positions": torch.randint(0, 32768, (3, T), generator=seeds(), device=device),
        "slot_mapping": torch.randperm(cache_blocks * 256, generator=seeds(), device=device)[:T].to(torch.int32),
        "inv_freq": (1.0 / (THETA ** (torch.arange(0, D, 2, dtype=torch.float32) / D))).to(device),
    }
    cache_shape = (cache_blocks, 256, NKV, D)
    inp["key_cache"] = torch.full(cache_shape, -3.0, dtype=torch.bfloat16, device=device)
    inp["value_cache"] = torch.full(cache_shape, -3.0, dtype=torch.bfloat16, device=device)
    need = GATHER_LEN // 256
    inp["tables"] = torch.stack([torch.randperm(cache_blocks, generator=seeds(), device=device)[:need]
                                 for _ in range(S)]).to(torch.int32) if S else \
        torch.empty(0, need, dtype=torch.int32, device=device)
    inp["seq_lens"] = torch.full((S,), GATHER_LEN, dtype=torch.int32, device=device)
    inp["cu_seqlens"] = torch.arange(S + 1, dtype=torch.int64, device=device) * GATHER_LEN
    inp["gather_seqs"] = S
    return inp


class LaunchTimer:
    """CUDA events between consecutive launches on the current stream, per kernel
    name. One event marks each boundary: it ends one launch's interval and starts
    the next's, so a launch's duration includes the gap before its successor and
    the durations add up to the timed region. Recording two events per launch
    instead cost 1.8% of a 32,768-token step on B200 (more events between
    kernels, same kernel durations)."""

    def __init__(self):
        self.pairs: dict[str, list] = {}
        self.last = None  # the event after the previous launch

    def __call__(self, name, fn, *a, **k):
        s = self.last
        if s is None:
            s = torch.cuda.Event(enable_timing=True)
            s.record()
        out = fn(*a, **k)
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.pairs.setdefault(name, []).append((s, e))
        self.last = e
        return out

    def summary(self) -> dict[str, dict]:
        out = {}
        for name, pairs in self.pairs.items():
            ms = [s.elapsed_time(e) for s, e in pairs]
            out[name] = {"launches": len(ms), "total_ms": sum(ms), "avg_ms": sum(ms) / len(ms),
                         "p50_ms": statistics.median(ms)}
        return out


def run_step(inp, layers, timer=None):
    from nano_vllm_multimodal_b200 import ops

    call = timer if timer is not None else (lambda name, fn, *a, **k: fn(*a, **k))
    h, res = inp["hidden"], inp["residual"]
    qkv = inp["qkv"]
    q, k, v = qkv.split([NQ * D, NKV * D, NKV * D], -1)
    q, k, v = q.view(-1, NQ, D), k.view(-1, NKV, D), v.view(-1, NKV, D)
    h2 = None
    for _ in range(layers):
        _, h1 = call("add_rms_norm", ops.add_rms_norm, h, res, inp["w_in"], EPS, True)
        call("qk_prologue", ops.qk_prologue, q, k, v=v, positions=inp["positions"],
             q_weight=inp["q_weight"], k_weight=inp["k_weight"], eps=EPS,
             rope_mode=ops.ROPE_MROPE_INTERLEAVED, inv_freq=inp["inv_freq"], sections=SECTIONS,
             key_cache=inp["key_cache"], value_cache=inp["value_cache"],
             slot_mapping=inp["slot_mapping"])
        _, h2 = call("add_rms_norm", ops.add_rms_norm, inp["attn_out"], h1, inp["w_post"], EPS, True)
        call("silu_and_mul", ops.silu_and_mul, inp["gate_up"])
        h, res = inp["mlp_out"], h2
    if inp["gather_seqs"]:
        total = inp["gather_seqs"] * GATHER_LEN
        for cache in (inp["key_cache"], inp["value_cache"]):
            call("paged_gather", ops.paged_gather_varlen, cache, inp["tables"], inp["seq_lens"],
                 inp["cu_seqlens"], total, GATHER_LEN)
    return h2


def launches_per_step(layers, gather_seqs):
    return 4 * layers + (2 if gather_seqs else 0)


def layers_e2e(inp, layers, mods, hidden, positions, slot_mapping):
    """The step's 28 fused layers through the layer-module API (reference-facing calls)."""
    from nano_vllm_multimodal_b200.layers.attention import attention_prologue

    h, res = hidden, inp["residual"]
    h2 = None
    for _ in range(layers):
        _, h1 = mods["input_norm"](h, res)
        attention_prologue(inp["qkv"], num_heads=NQ, num_kv_heads=NKV, head_dim=D,
                           positions=positions, rotary_emb=mods["rope"], q_norm=mods["q_norm"],
                           k_norm=mods["k_norm"], k_cache=inp["key_cache"], v_cache=inp["value_cache"],
                           slot_mapping=slot_mapping)
        _, h2 = mods["post_norm"](inp["attn_out"], h1)
        mods["act"](inp["gate_up"])
        h, res = inp["mlp_out"], h2
    return h2


class E2EPipeline:
    """Steps with host inputs and host results, copies overlapped with compute.

    Each step copies its inputs (initial hidden states, positions, slot mapping)
    from pinned host memory and its final hidden states back to pinned host
    memory. Two device input slots and two host output buffers let step k+1's
    host->device copy (copy stream 1) and step k's device->host copy (copy
    stream 2) run while other steps compute; events order every reuse.
    """

    KEYS = ("hidden", "positions", "slot_mapping")

    def __init__(self, inp, layers, mods):
        self.inp, self.layers, self.mods = inp, layers, mods
        self.host_in = [{k: inp[k].cpu().pin_memory() for k in self.KEYS} for _ in range(2)]
        self.dev_in = [{k: torch.empty_like(inp[k]) for k in self.KEYS} for _ in range(2)]
        self.host_out = [torch.empty(inp["tokens"], H, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        self.h2d, self.d2h = torch.cuda.Stream(), torch.cuda.Stream()
        self.used = [torch.cuda.Event() for _ in range(2)]     # compute finished with dev_in[i]
        self.ready = [torch.cuda.Event() for _ in range(2)]    # dev_in[i] filled

    def bytes_per_step(self):
        h2d = sum(t.numel() * t.element_size() for t in self.host_in[0].values())
        return h2d, self.host_out[0].numel() * self.host_out[0].element_size()

    def _load(self, slot, first):
        if not first:
            self.h2d.wait_event(self.used[slot])
        with torch.cuda.stream(self.h2d):
            for k in self.KEYS:
                self.dev_in[slot][k].copy_(self.host_in[slot][k], non_blocking=True)
            self.ready[slot].record(self.h2d)

    def run(self, steps):
        compute = torch.cuda.current_stream()
        self.h2d.wait_stream(compute)
        self.d2h.wait_stream(compute)
        self._load(0, True)
        for k in range(steps):
            cur, nxt = k % 2, (k + 1) % 2
            if k + 1 < steps:
                self._load(nxt, k == 0)
            compute.wait_event(self.ready[cur])
            d = self.dev_in[cur]
            out = layers_e2e(self.inp, self.layers, self.mods, d["hidden"], d["positions"], d["slot_mapping"])
            self.used[cur].record(compute)
            self.d2h.wait_event(self.used[cur])
            with torch.cuda.stream(self.d2h):
                self.host_out[cur].copy_(out, non_blocking=True)
            out.record_stream(self.d2h)
        compute.wait_stream(self.d2h)
        compute.wait_stream(self.h2d)


def build_modules(inp, device):
    from nano_vllm_multimodal_b200.layers.activation import SiluAndMul
    from nano_vllm_multimodal_b200.layers.multimodal_rotary_embedding import MultimodalRotaryEmbedding
    from nano_vllm_multimodal_b200.layers.qwen3_vl import Qwen3VLTextRMSNorm

    def norm(n, w):
        m = Qwen3VLTextRMSNorm(n, eps=EPS).to(device=device, dtype=torch.bfloat16)
        with torch.no_grad():
            m.weight.copy_(w)
        return m

    rope = MultimodalRotaryEmbedding(head_dim=D, base=THETA, sections=SECTIONS, strategy="interleaved").to(device)
    return {"input_norm": norm(H, inp["w_in"]), "post_norm": norm(H, inp["w_post"]),
            "q_norm": norm(D, inp["q_weight"]), "k_norm": norm(D, inp["k_weight"]),
            "rope": rope, "act": SiluAndMul()}


def load_traffic_table() -> dict[str, float]:
    """DRAM bytes per token per kernel from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "dram_traffic.md"
    out = {}
    if not path.exists():
        return out
    for m in re.finditer(r"^\|\s*(\w+)\s*\|\s*([0-9.]+)\s*\|", path.read_text(), re.M):
        try:
            out[m.group(1)] = float(m.group(2))
        except ValueError:
            pass
    return out


# ------------------------------------------------------------------ CPU path of the reference


def host_threads() -> int:
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


CPU_SAMPLE_TOKENS = 2048


def cpu_c5_sample():
    """A bounded sample of the C5 step on the CPU: one fused layer over 2,048 C5
    tokens (cache of 256 blocks, slots drawn from it) and one 16,384-token
    sequence gathered from a 64-block table."""
    from nano_vllm_multimodal_b200 import workloads as W
    from oracle.cpu_layer import CpuLayer

    d = W.make_layer_inputs(5, tokens=CPU_SAMPLE_TOKENS, cache=False)
    seeds = W._Seeds(5, "cpu")
    seeds.index = 950
    d["slot_mapping"] = W._randperm(seeds, 256 * 256, CPU_SAMPLE_TOKENS)
    d["key_cache"] = torch.full((256, 256, NKV, D), -3.0, dtype=torch.bfloat16)
    d["value_cache"] = torch.full((256, 256, NKV, D), -3.0, dtype=torch.bfloat16)
    d["table"] = W._randperm(seeds, 256, GATHER_LEN // 256)
    return CpuLayer(W.C5, d), d


def cpu_sample_step(layer, d):
    """One sample step -> (layer seconds, gather seconds for K and V)."""
    t0 = time.perf_counter()
    layer(d)
    t1 = time.perf_counter()
    layer.gather(d["key_cache"], d["table"], GATHER_LEN)
    layer.gather(d["value_cache"], d["table"], GATHER_LEN)
    return t1 - t0, time.perf_counter() - t1


def cpu_extrapolate(layer_s, gather_s, reps, tokens_total=TOKENS, layers=LAYERS):
    """Per-token costs of the sample -> seconds of the whole C5 step and the metric."""
    per_layer_token = layer_s / (reps * CPU_SAMPLE_TOKENS)
    per_gather_token = gather_s / (reps * 2 * GATHER_LEN)
    step_s = per_layer_token * tokens_total * layers + per_gather_token * 2 * GATHER_SEQS * GATHER_LEN
    return step_s, tokens_total * layers / step_s


def cpu_sample_desc(kind, reps, cores):
    who = ("the reference's own modules (nanovllm.layers / models.qwen3_vl, PyTorch paged-KV backend, "
           "eager: torch.compile disabled)" if kind == "reference" else "the oracle port of the reference's ops")
    return (f"{reps} sample steps on {cores} host threads, each one fused C5 layer over {CPU_SAMPLE_TOKENS} "
            f"tokens plus one {GATHER_LEN}-token sequence gathered from K and V, run by {who}; "
            f"extrapolated by per-token cost to the C5 step ({TOKENS} tokens x {LAYERS} layers + "
            f"{GATHER_SEQS} x {GATHER_LEN}-token K/V gather)")


def cpu_baseline(budget_s: float) -> dict:
    """The CPU figure on the GPU arm's line: the same measurement as ``--impl reference``."""
    cores = host_threads()
    layer, d = cpu_c5_sample()
    cpu_sample_step(layer, d)  # warm-up
    lt = gt = 0.0
    reps, t0 = 0, time.perf_counter()
    while True:
        a, b = cpu_sample_step(layer, d)
        lt, gt, reps = lt + a, gt + b, reps + 1
        if time.perf_counter() - t0 >= budget_s:
            break
    step_s, value = cpu_extrapolate(lt, gt, reps)
    return {"value": value, "unit": UNIT, "cores": cores, "kind": layer.kind,
            "sample": cpu_sample_desc(layer.kind, reps, cores),
            "extrapolated_step_s": round(step_s, 3)}


def config_block(args, world, extra=None):
    cfg = {"workload": "C5 Qwen3-VL-2B fused elementwise layer x28 + paged-KV gather",
           "tokens_per_step": args.tokens, "layers": args.layers, "hidden": H,
           "heads": [NQ, NKV], "head_dim": D, "intermediate": INTER,
           "mrope": {"strategy": "interleaved", "sections": list(SECTIONS), "theta": THETA},
           "gather": {"sequences": GATHER_SEQS, "tokens_per_sequence": GATHER_LEN, "caches": 2},
           "cache_per_gpu": [args.cache_blocks, 256, NKV, D], "parallelism": f"token-sharded x{world}",
           "value_counts": "token x fused-layer passes per second",
           "l2": "inputs larger than L2 (every kernel's working set > 126 MB at every N)"}
    if extra:
        cfg.update(extra)
    return cfg


# ------------------------------------------------------------------ other kernels of the path


def _time_graph(calls, reps=24):
    """Average ms per call of ``reps`` calls captured back to back in one CUDA
    graph, cycling through ``calls``. Each callable owns a separate set of
    inputs, and the sets together are several times the 126 MB L2, so no call
    finds its inputs left in L2 by the call before; the outputs of all ``reps``
    calls stay alive, so none writes into a buffer an earlier call left in L2.
    The graph removes the host launch gaps of short kernels; each kernel starts
    with the L2 that its predecessor left, as inside a model step."""
    keep = []
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for c in calls:
            keep.append(c())
    torch.cuda.current_stream().wait_stream(side)
    keep.clear()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(reps):
            keep.append(calls[i % len(calls)]())
    graph.replay()
    torch.cuda.synchronize()
    best = None
    for _ in range(3):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        graph.replay()
        e.record()
        e.synchronize()
        ms = s.elapsed_time(e) / reps
        best = ms if best is None else min(best, ms)
    del graph, keep
    return best


def flush_l2(buf):
    """Flush the L2 between timed calls: write ``buf`` (4x the 126 MB L2), then read
    it back. The write evicts every earlier line; the read evicts the write's own
    dirty lines, so the timed call starts from a clean L2 holding none of its
    inputs and does not pay for writing 126 MB of the flush back to DRAM (13.5 us
    of a 0.2 ms decode-attention call). Both run outside the timed events."""
    buf.zero_()
    buf.view(torch.int64).sum()


def _time_op(fn, reps=20, warmup=3, flush=None):
    """Average ms of ``fn`` with CUDA events around each call; ``flush`` (a
    buffer larger than L2) flushes the L2 between calls (``flush_l2``), outside
    the events."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(reps):
        if flush is not None:
            flush_l2(flush)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        total += s.elapsed_time(e)
    return total / reps


def visual_merge_component(out, record, flush, seeds, rows, c3):
    """Packed-prefill visual merge at C3: 16 images x 1,024 rows, 3 DeepStack layers.
    Kernel alone (plan packed once), the whole API call (host packing included) and
    the reference's own torch path (model_runner.py:237-285, restated inline)."""
    from types import SimpleNamespace

    from nano_vllm_multimodal_b200 import ops
    from nano_vllm_multimodal_b200.layers.visual_merge import build_planned_visual_embeddings
    from nano_vllm_multimodal_b200 import workloads as W

    T, H, L, per = c3.tokens, c3.hidden, 3, 1024
    tok = W._normal(seeds, (T, H))
    feats = {}
    for i in range(rows.numel() // per):
        f = W._normal(seeds, (L + 1, per, H))
        feats[f"vision:{i}"] = SimpleNamespace(final_embedding=f[0], deepstack_embeddings=tuple(f[1:]))
    reps = tuple(SimpleNamespace(output_row=r, feature_key=f"vision:{i // per}", feature_row=i % per)
                 for i, r in enumerate(rows.tolist()))
    plan = SimpleNamespace(replacements=reps)
    R = len(reps)
    # kernel alone: the device plan and table that the API call packs
    table = torch.zeros(len(feats), 20, dtype=torch.int64)
    for k, b in enumerate(feats.values()):
        table[k, 0], table[k, 1], table[k, 2], table[k, 3] = b.final_embedding.data_ptr(), H, per, 2
        for l, d in enumerate(b.deepstack_embeddings):
            table[k, 4 + l], table[k, 12 + l] = d.data_ptr(), H
    plan_dev = torch.tensor([r.output_row for r in reps] + [i // per for i in range(R)]
                            + [i % per for i in range(R)], dtype=torch.int64, device=tok.device)
    table_dev = table.to(tok.device)
    # kernel alone, graph-timed over SETS sets of token embeddings and features
    kept = [(tok, table_dev)]
    for _ in range(SETS - 1):
        tk = W._normal(seeds, (T, H))
        tb = torch.zeros_like(table)
        fs = [W._normal(seeds, (L + 1, per, H)) for _ in range(len(feats))]
        for k, f in enumerate(fs):
            tb[k, 0], tb[k, 1], tb[k, 2], tb[k, 3] = f[0].data_ptr(), H, per, 2
            for l in range(L):
                tb[k, 4 + l], tb[k, 12 + l] = f[1 + l].data_ptr(), H
        kept.append((tk, tb.to(tok.device), fs))
    ms = _time_graph([lambda i=i: ops.visual_merge(kept[i][0], kept[i][1], L, plan_dev, R) for i in range(SETS)])
    del kept[1:]
    record("visual_merge", ms, 4 * H * (T + R * L),
           "C3: [32768,2048] tokens, 16 x 1024 image rows, 3 DeepStack layers; kernel alone, graph-timed")
    ms_api = _time_op(flush=flush, fn=lambda: build_planned_visual_embeddings(tok, plan, feats))

    def reference_path():
        merged = tok.clone()
        ds = tuple(torch.empty((R, H), device=tok.device, dtype=tok.dtype) for _ in range(L))
        groups = {}
        for idx, rp in enumerate(reps):
            groups.setdefault(rp.feature_key, []).append((idx, rp))
        for key, grouped in groups.items():
            b = feats[key]
            out_rows = torch.tensor([rp.output_row for _, rp in grouped], dtype=torch.int64, device=tok.device)
            frows = torch.tensor([rp.feature_row for _, rp in grouped], dtype=torch.int64, device=tok.device)
            merged.index_copy_(0, out_rows, b.final_embedding.index_select(0, frows).to(tok.dtype))
            vrows = torch.tensor([i for i, _ in grouped], dtype=torch.int64, device=tok.device)
            for l, emb in enumerate(b.deepstack_embeddings):
                lrows = torch.tensor([rp.feature_row for _, rp in grouped], dtype=torch.int64, device=tok.device)
                ds[l].index_copy_(0, vrows, emb.index_select(0, lrows).to(tok.dtype))
        return merged, ds

    ms_ref = _time_op(flush=flush, fn=reference_path)
    out["visual_merge"]["api_ms"] = round(ms_api, 4)
    out["visual_merge"]["reference_torch_ms"] = round(ms_ref, 4)
    out["visual_merge"]["note"] = ("api_ms: build_planned_visual_embeddings incl. host plan packing; "
                                   "reference_torch_ms: the reference's per-key index_select/index_copy_ path")


def step_inputs_component(out, device):
    """Host -> device step inputs of a C3 prefill (32,768 tokens, 16 sequences, 3-axis
    positions): the reference's one pinned tensor + one copy per array
    (model_runner.py:700-725,823-870) vs one StepInputStager copy. Host wall time
    per step (list conversion included), both from the same Python lists. Then the
    same for a decode step's five arrays (model_runner.py:892-935)."""
    from nano_vllm_multimodal_b200.step_inputs import StepInputStager

    g = torch.Generator().manual_seed(4242)
    T, B = 32768, 16
    ids = torch.randint(0, 151936, (T,), generator=g).tolist()
    pos = torch.randint(0, 32768, (3, T), generator=g).tolist()
    cuq = [i * (T // B) for i in range(B + 1)]
    slots = torch.randperm(1 << 20, generator=g)[:T].int().tolist()
    ctx = [T // B] * B
    qs = [0] * B
    tables = [list(range(i * 8, i * 8 + 8)) for i in range(B)]

    def reference():
        def cp(v, dt):
            return torch.tensor(v, dtype=dt, pin_memory=True).cuda(non_blocking=True)
        return (cp(ids, torch.int64), cp(pos, torch.int64), cp(cuq, torch.int32), cp(cuq, torch.int32),
                cp(slots, torch.int32), cp(ctx, torch.int32), cp(qs, torch.int32), cp(tables, torch.int32))

    stager = StepInputStager(device=device, slots=3)

    def staged():
        return stager.prefill_inputs(ids, pos, cuq, cuq, slots, ctx, qs, tables, position_axes=3)

    res = {}
    for name, fn in (("reference_host_ms", reference), ("staged_host_ms", staged)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(20):
            fn()
        res[name] = round((time.perf_counter() - t0) / 20 * 1e3, 3)
        torch.cuda.synchronize()
    res.update(copies_reference=8, copies_staged=1, bytes_per_step=T * 8 * 4 + T * 4 + (B + 1) * 8 + B * 8 + B * 8 * 4,
               config="C3 prefill step inputs: 32,768 tokens, 16 sequences, 3-axis positions")

    # decode (model_runner.py:892-935): 256 requests, contexts U[1, 8192], 3-axis positions
    R = 256
    dlens = torch.randint(1, 8193, (R,), generator=g).tolist()
    dids = torch.randint(0, 151936, (R,), generator=g).tolist()
    dpos = [[n - 1 for n in dlens]] * 3
    dtables = [torch.randperm(8192, generator=g)[:(n + 255) // 256].tolist() for n in dlens]
    dslots = [t[-1] * 256 + (n - 1) % 256 for t, n in zip(dtables, dlens)]

    def decode_reference():
        def cp(v, dt):
            return torch.tensor(v, dtype=dt, pin_memory=True).cuda(non_blocking=True)
        width = max(len(t) for t in dtables)
        return (cp(dids, torch.int64), cp(dpos, torch.int64), cp(dslots, torch.int32), cp(dlens, torch.int32),
                cp([t + [-1] * (width - len(t)) for t in dtables], torch.int32))

    def decode_staged():
        return stager.decode_inputs(dids, dpos, dslots, dlens, dtables, position_axes=3)

    for name, fn in (("decode_reference_host_ms", decode_reference), ("decode_staged_host_ms", decode_staged)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(50):
            fn()
        res[name] = round((time.perf_counter() - t0) / 50 * 1e3, 4)
        torch.cuda.synchronize()
    res.update(decode_copies_reference=5, decode_copies_staged=1,
               decode_config="C3 decode step inputs: 256 requests, contexts U[1, 8192], 3-axis positions")
    out["step_inputs"] = res


def decode_attention_component(out, record, flush, device, requests=256):
    """Paged decode attention at C2 decode: 256 requests, 256-token blocks, contexts
    U[1, 8192] (C2 positions U[0, 8191] plus the new token), at two head layouts:
    16/8 heads of 128 (Qwen3, GQA 2) and 16/2 (Qwen2.5-VL, GQA 8: four times the
    q.K and P.V work per cached byte). Each kernel against the roofline (the
    tensor-core kernel, the default, and the CUDA-core one), and flash-attn's own
    flash_attn_with_kvcache (the reference's decode kernel) on the same inputs."""
    from nano_vllm_multimodal_b200 import ops

    for name, NQ_, NKV_ in (("decode_attention", 16, 8), ("decode_attention_gqa8", 16, 2)):
        g = torch.Generator().manual_seed(5151)
        B, D_, BS_ = requests, 128, 256
        lens = torch.randint(1, 8193, (B,), generator=g, dtype=torch.int32)
        need = (lens + BS_ - 1) // BS_
        nblocks = int(need.sum()) + 16
        width = int(need.max())
        perm = torch.randperm(nblocks, generator=g).to(torch.int32)
        tables = torch.full((B, width), 0, dtype=torch.int32)
        at = 0
        for b in range(B):
            n = int(need[b])
            tables[b, :n] = perm[at:at + n]
            at += n
        kc = torch.randn(nblocks, BS_, NKV_, D_, device=device, dtype=torch.bfloat16)
        vc = torch.randn(nblocks, BS_, NKV_, D_, device=device, dtype=torch.bfloat16)
        q = torch.randn(B, NQ_, D_, device=device, dtype=torch.bfloat16)
        cl, tb = lens.to(device), tables.to(device)
        scale = D_ ** -0.5
        nbytes = int(lens.sum()) * NKV_ * D_ * 2 * 2 + B * NQ_ * D_ * 2 * 2 + B * 4 + int(need.sum()) * 4
        cfg = (f"C2 decode: {B} requests, {NQ_}/{NKV_} heads x 128 (GQA {NQ_ // NKV_}), 256-token blocks, "
               "contexts U[1,8192]; tensor-core kernel")
        ms = _time_op(flush=flush, fn=lambda: ops.decode_attention(q, kc, vc, cl, tb, scale, 8192))
        record(name, ms, nbytes, cfg)
        mine = ops.decode_attention(q, kc, vc, cl, tb, scale, 8192)
        ms_fma = _time_op(flush=flush, fn=lambda: ops.decode_attention(q, kc, vc, cl, tb, scale, 8192,
                                                                       variant=ops.DECODE_CUDA_CORES))
        out[name]["cuda_core_kernel_ms"] = round(ms_fma, 4)
        out[name]["cuda_core_kernel_frac"] = round(nbytes / (ms_fma / 1000.0) / 1e9 / measured_hbm_peak(), 4)
        try:
            from flash_attn import flash_attn_with_kvcache as fa

            ref = fa(q.unsqueeze(1), kc, vc, cache_seqlens=cl, block_table=tb, softmax_scale=scale, causal=True)
            diff = float((ref[:, 0].float() - mine.float()).abs().max())
            ms_fa = _time_op(flush=flush, fn=lambda: fa(q.unsqueeze(1), kc, vc, cache_seqlens=cl, block_table=tb,
                                                        softmax_scale=scale, causal=True))
            out[name]["flash_attn_ms"] = round(ms_fa, 4)
            out[name]["flash_attn_frac"] = round(nbytes / (ms_fa / 1000.0) / 1e9 / measured_hbm_peak(), 4)
            out[name]["max_abs_diff_vs_flash_attn"] = round(diff, 5)
        except Exception as e:  # the library may carry no kernels for this GPU
            out[name]["flash_attn"] = f"unavailable: {type(e).__name__}: {str(e)[:120]}"
        del kc, vc


def rows_flushed_rounds(flush, device, rounds=3):
    """The row kernels one call at a time, each after an L2 flush, in rounds of
    (embedding, DeepStack add, add + norm + DeepStack): the launch order a
    profiler capture of `--component rows` relies on. Returns ms per call of
    rounds 2.. (CUDA events around each call)."""
    from nano_vllm_multimodal_b200 import ops, workloads as W

    seeds = W._Seeds(2, device)
    seeds.index = 800
    emb = W._normal(seeds, (151936, 1024), 0.0, 0.02)
    ids = torch.randint(0, 151936, (65536,), generator=seeds(), device=device)
    c3 = W.C3
    hs = W._normal(seeds, (c3.tokens, c3.hidden))
    res = W._normal(seeds, (c3.tokens, c3.hidden))
    wn = W._normal(seeds, (c3.hidden,), 1.0, 0.1)
    vrows = W.deepstack_rows(3, c3.tokens).to(device)
    vis = W._normal(seeds, (vrows.numel(), c3.hidden))
    ridx = ops.deepstack_row_index(vrows, c3.tokens)
    fns = {"embedding": lambda: ops.embedding(ids, emb),
           "deepstack_add_inplace": lambda: ops.deepstack_add_(hs, vrows, vis),
           "add_norm_deepstack": lambda: ops.add_rms_norm_deepstack(hs, res, wn, EPS, vis, ridx)}
    ms = dict.fromkeys(fns, 0.0)
    for r in range(rounds):
        for name, fn in fns.items():
            flush_l2(flush)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            e.synchronize()
            if r > 0:
                ms[name] += s.elapsed_time(e) / (rounds - 1)
    return ms


SETS = 4  # separate input/output sets of a graph-timed component (together several times L2)


def rows_component(record, seeds, device, out=None):
    """The row kernels on their own, graph-timed over SETS input sets: the C2
    embedding (65,536 random ids into the 151,936 x 1,024 table), the C3
    DeepStack add in place and out of place, and the C3 add + norm + DeepStack
    fold (32,768 tokens, 16,384 visual rows) next to the three passes it
    replaces."""
    from nano_vllm_multimodal_b200 import ops, workloads as W

    embs = [W._normal(seeds, (151936, 1024), 0.0, 0.02) for _ in range(SETS)]
    idss = [torch.randint(0, 151936, (65536,), generator=seeds(), device=device) for _ in range(SETS)]
    ms = _time_graph([lambda i=i: ops.embedding(idss[i], embs[i]) for i in range(SETS)])
    record("embedding", ms, 65536 * (4 * 1024 + 8), "C2 table 151936x1024, 65,536 random ids")
    del embs, idss
    c3 = W.C3
    rows = W.deepstack_rows(3, c3.tokens).to(device)
    hss = [W._normal(seeds, (c3.tokens, c3.hidden)) for _ in range(SETS)]
    viss = [W._normal(seeds, (rows.numel(), c3.hidden)) for _ in range(SETS)]
    ms = _time_graph([lambda i=i: ops.deepstack_add_(hss[i], rows, viss[i]) for i in range(SETS)])
    record("deepstack_add_inplace", ms, rows.numel() * (6 * c3.hidden + 8),
           "C3: hidden [32768,2048], 16,384 image rows")
    ms = _time_graph([lambda i=i: ops.deepstack_add(hss[i], rows, viss[i]) for i in range(SETS)])
    record("deepstack_add_out_of_place", ms, c3.tokens * 4 * c3.hidden + rows.numel() * (6 * c3.hidden + 8),
           "C3, copy + add")
    # Qwen3-VL layer boundary with DeepStack folded in: rounded add + visual-row add + text norm
    ress = [W._normal(seeds, (c3.tokens, c3.hidden)) for _ in range(SETS)]
    wn = W._normal(seeds, (c3.hidden,), 1.0, 0.1)
    ridx = ops.deepstack_row_index(rows, c3.tokens)
    ms = _time_graph([lambda i=i: ops.add_rms_norm_deepstack(hss[i], ress[i], wn, EPS, viss[i], ridx)
                      for i in range(SETS)])

    def unfused(i):
        s = hss[i] + ress[i]
        ops.deepstack_add_(s, rows, viss[i])
        return ops.rms_norm(s, wn, EPS), s

    ms_unfused = _time_graph([lambda i=i: unfused(i) for i in range(SETS)])
    record("add_norm_deepstack", ms, c3.tokens * (8 * c3.hidden + 4) + rows.numel() * 2 * c3.hidden,
           "C3: [32768,2048] + 16,384 visual rows, one pass")
    if out is not None:
        out["add_norm_deepstack"]["unfused_ms"] = round(ms_unfused, 4)
        out["add_norm_deepstack"]["unfused"] = "torch add + deepstack_add_ + rms_norm"


def rope_forward_component(record, device):
    """The rotary modules' own forward (the drop-in path when a model is not
    edited to call the fused prologue: RotaryEmbedding.forward and
    MultimodalRotaryEmbedding.forward, one kernel each), graph-timed over
    separate input sets: 1-D RoPE and interleaved M-RoPE at 32,768 tokens with
    16/8 heads, chunked M-RoPE at C4 (8,312 tokens, 16/2 heads). q and k are
    strided views of the qkv rows; bytes = q and k in and out + positions."""
    from nano_vllm_multimodal_b200.layers.multimodal_rotary_embedding import MultimodalRotaryEmbedding
    from nano_vllm_multimodal_b200.layers.rotary_embedding import RotaryEmbedding

    g = torch.Generator(device=device)
    g.manual_seed(5500)

    def sets(n, T, nq, nkv, axes, maxpos):
        out = []
        for _ in range(n):
            qkv = torch.randn(T, (nq + 2 * nkv) * D, generator=g, device=device).to(torch.bfloat16)
            shape = (T,) if axes == 1 else (3, T)
            out.append((qkv[:, :nq * D].view(T, nq, D), qkv[:, nq * D:(nq + nkv) * D].view(T, nkv, D),
                        torch.randint(0, maxpos, shape, generator=g, device=device)))
        return out

    cases = (
        ("rope_forward", RotaryEmbedding(D, D, 40960, 1e6), SETS, 32768, 16, 8, 1, 40960,
         "RotaryEmbedding (Qwen3, theta 1e6): 32,768 tokens, 16/8 heads"),
        ("mrope_forward_interleaved",
         MultimodalRotaryEmbedding(head_dim=D, base=THETA, sections=SECTIONS, strategy="interleaved"),
         SETS, 32768, 16, 8, 3, 32768, "MultimodalRotaryEmbedding interleaved (Qwen3-VL): 32,768 tokens, 16/8 heads"),
        ("mrope_forward_chunked",
         MultimodalRotaryEmbedding(head_dim=D, base=1e6, sections=(16, 24, 24), strategy="chunked"),
         8, 8312, 16, 2, 3, 16384, "MultimodalRotaryEmbedding chunked (Qwen2.5-VL, C4): 8,312 tokens, 16/2 heads"),
    )
    for name, mod, n, T, nq, nkv, axes, maxpos, cfg in cases:
        mod = mod.to(device)
        st = sets(n, T, nq, nkv, axes, maxpos)
        ms = _time_graph([lambda i=i: mod(st[i][2], st[i][0], st[i][1]) for i in range(n)])
        record(name, ms, T * ((nq + nkv) * D * 2 * 2 + 8 * axes), cfg + "; graph-timed")
        del st


def mrope_component(record, device, inv_freq, tokens=32768):
    """MultimodalRotaryEmbedding.cos_sin and apply_multimodal_rotary_emb on their
    own (the model path computes cos/sin inside the fused prologue), graph-timed
    over SETS input sets: C3 shapes, 32,768 tokens x 16 heads, q a strided view
    of the qkv rows, positions uniform on [0, 32767]."""
    from nano_vllm_multimodal_b200 import ops

    g = torch.Generator(device=device)
    g.manual_seed(5300)
    n = tokens
    qkvs = [torch.randn(n, (NQ + 2 * NKV) * D, generator=g, device=device).to(torch.bfloat16)
            for _ in range(SETS)]
    qs = [t[:, :NQ * D].view(n, NQ, D) for t in qkvs]
    poss = [torch.randint(0, 32768, (3, n), generator=g, device=device) for _ in range(SETS)]
    trig = [ops.mrope_cos_sin(p, inv_freq, torch.bfloat16) for p in poss]
    ms = _time_graph([lambda i=i: ops.mrope_apply(qs[i], trig[i][0], trig[i][1], SECTIONS, True)
                      for i in range(SETS)])
    # interleaved: both halves of a head read column j < D/2, so the op needs the
    # first half of each axis row of cos and sin (every 32-byte sector of it)
    record("mrope_apply_generic", ms, n * NQ * D * 2 * 2 + 2 * 3 * n * (D // 2) * 2,
           f"C3 shapes, {n:,} tokens x 16 heads, cos/sin given (first half of each axis row read)")
    ms = _time_graph([lambda i=i: ops.mrope_cos_sin(poss[i], inv_freq, torch.bfloat16) for i in range(SETS)])
    record("mrope_cos_sin", ms, 3 * n * 8 + 2 * 3 * n * D * 2,
           f"{n:,} tokens, 3 axes (sincosf-bound: {3 * n * D // 2 / 1e6:.1f} M sincos per call)")


def component_bench(inp, device, hbm_peak):
    """The path's kernels that the fused layer does not exercise on their own,
    each at a full config size, timed with CUDA events (working sets > L2)."""
    from nano_vllm_multimodal_b200 import ops, workloads as W

    out = {}
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=device)  # 4x the 126 MB L2

    def record(name, ms, nbytes, cfg):
        gbs = nbytes / (ms / 1000.0) / 1e9
        out[name] = {"avg_ms": round(ms, 4), "bytes": int(nbytes), "achieved_gbs": round(gbs, 1),
                     "frac": round(gbs / hbm_peak, 4), "config": cfg}

    T = inp["tokens"]
    qkv = inp["qkv"]
    q = qkv[:, : NQ * D].view(-1, NQ, D)
    k = qkv[:, NQ * D:(NQ + NKV) * D].view(-1, NKV, D)
    v = qkv[:, (NQ + NKV) * D:].view(-1, NKV, D)
    ms = _time_op(flush=flush, fn=lambda: ops.paged_store(k, v, inp["key_cache"], inp["value_cache"], inp["slot_mapping"]))
    record("paged_store", ms, T * 4 * NKV * D * 2, f"C5: {T} tokens, k/v strided views of the qkv rows")
    ms = _time_op(flush=flush, fn=lambda: ops.rms_norm(q, inp["q_weight"], EPS))
    record("rms_norm_heads", ms, T * NQ * D * 2 * 2, f"C3/C5 q-norm: [{T},{NQ},{D}] strided view")
    # The step's prologue writes K/V to a random permutation of slots (the worst
    # case). A serving engine gives each sequence whole 256-slot blocks, so
    # consecutive tokens fill consecutive slots of a randomly chosen block. Both
    # placements on the same inputs, one launch at a time after an L2 flush.
    nblk = inp["key_cache"].shape[0]
    g = torch.Generator(device=device)
    g.manual_seed(5400)
    blocks = torch.randperm(nblk, generator=g, device=device)[: -(-T // 256)]
    tok = torch.arange(T, device=device)
    block_slots = (blocks[tok // 256] * 256 + tok % 256).to(torch.int32)

    def prologue(slots):
        return ops.qk_prologue(q, k, v=v, positions=inp["positions"], q_weight=inp["q_weight"],
                               k_weight=inp["k_weight"], eps=EPS, rope_mode=ops.ROPE_MROPE_INTERLEAVED,
                               inv_freq=inp["inv_freq"], sections=SECTIONS, key_cache=inp["key_cache"],
                               value_cache=inp["value_cache"], slot_mapping=slots)

    for name, slots, what in (("qk_prologue_random_slots", inp["slot_mapping"], "a random permutation of slots"),
                              ("qk_prologue_block_slots", block_slots,
                               "consecutive tokens in consecutive slots of random 256-slot blocks")):
        ms = _time_op(flush=flush, fn=lambda slots=slots: prologue(slots))
        record(name, ms, T * BYTES["qk_prologue"], f"C5: {T} tokens, K/V written to {what}")
    del block_slots, tok
    seeds = W._Seeds(2, device)
    seeds.index = 700
    rows_component(record, seeds, device, out)
    c3 = W.C3
    rows = W.deepstack_rows(3, c3.tokens).to(device)
    visual_merge_component(out, record, flush, seeds, rows, c3)
    step_inputs_component(out, device)
    decode_attention_component(out, record, flush, device)
    mrope_component(record, device, inp["inv_freq"])
    rope_forward_component(record, device)
    del flush
    out["c2_decode_layer_graph"] = decode_layer_graph(device, 2)
    out["c3_decode_layer_graph"] = decode_layer_graph(device, 3)
    return out


def decode_layer_graph(device, config=2, layers=28, replays=50):
    """A decode step's fused elementwise layer x28 (256 tokens), captured once in
    a CUDA graph and replayed: C2 (Qwen3-0.6B shapes, 1-D RoPE, 10% padded
    slots) or, with ``config=3``, Qwen3-VL-2B shapes (rounded add + text norm,
    interleaved M-RoPE computed in the kernel). Small batches are launch-bound,
    not HBM-bound: reported as time per layer."""
    from nano_vllm_multimodal_b200 import ops, workloads as W
    from nano_vllm_multimodal_b200.layers.multimodal_rotary_embedding import MultimodalRotaryEmbedding
    from nano_vllm_multimodal_b200.layers.rotary_embedding import RotaryEmbedding

    d = W.make_layer_inputs(config, tokens=256, device=device)
    shp = d["shape"]
    nq, nkv, hd = shp.num_heads, shp.num_kv_heads, shp.head_dim
    if shp.rope == "table":
        table = RotaryEmbedding(hd, hd, shp.max_position, shp.theta).to(device).cos_sin_cache
        rope = dict(rope_mode=ops.ROPE_TABLE, cos_sin_cache=table)
    else:
        mod = MultimodalRotaryEmbedding(head_dim=hd, base=shp.theta, sections=shp.sections,
                                        strategy=shp.rope).to(device)
        mode = ops.ROPE_MROPE_INTERLEAVED if shp.rope == "interleaved" else ops.ROPE_MROPE_CHUNKED
        rope = dict(rope_mode=mode, inv_freq=mod.inv_freq, sections=shp.sections)
    rounded = shp.qk_norm == "text"  # Qwen3-VL adds the residual in the activation dtype
    qkv = d["qkv"]
    q, k, v = qkv.split([nq * hd, nkv * hd, nkv * hd], -1)
    q, k, v = q.view(-1, nq, hd), k.view(-1, nkv, hd), v.view(-1, nkv, hd)

    def step():
        h, res = d["hidden"], d["residual"]
        for _ in range(layers):
            _, h1 = ops.add_rms_norm(h, res, d["w_in"], 1e-6, rounded)
            ops.qk_prologue(q, k, v=v, positions=d["positions"], q_weight=d["q_weight"], k_weight=d["k_weight"],
                            eps=1e-6, key_cache=d["key_cache"], value_cache=d["value_cache"],
                            slot_mapping=d["slot_mapping"], **rope)
            _, h2 = ops.add_rms_norm(d["attn_out"], h1, d["w_post"], 1e-6, rounded)
            ops.silu_and_mul(d["gate_up"])
            h, res = d["hidden"], h2

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(replays):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us_layer = e0.elapsed_time(e1) * 1000.0 / (replays * layers)
    del graph
    axes = 1 if shp.rope == "table" else 3
    cfg = ("C2 decode: 256 tokens, hidden 1024, 16/8 heads, 1-D RoPE (theta 1e6), 10% slots -1, I=3072"
           if config == 2 else
           "Qwen3-VL-2B decode (C3 shapes): 256 tokens, hidden 2048, 16/8 heads, text norm, interleaved "
           "M-RoPE [24,20,20] theta 5e6, I=6144")
    return {"us_per_layer": round(us_layer, 2), "launches_per_layer": 4,
            "tokens": shp.tokens if config == 2 else 256, "layers_per_graph": layers,
            "bytes_per_layer": 256 * (2 * 8 * shp.hidden + 2 * ((nq + 2 * nkv) * hd + nq * hd + nkv * hd
                                                               + 2 * nkv * hd) + 8 * axes + 4
                                      + 6 * shp.intermediate),
            "config": cfg + "; 28 layers per captured graph"}


# ------------------------------------------------------------------ per-config table (C1-C4)
L2_BYTES = 126 * 1024 * 1024


def layer_bytes(shape, tokens: int, valid: int) -> int:
    """Algorithmic bytes of one fused layer (2 x add+norm, prologue, SiluAndMul) over
    ``tokens`` tokens of which ``valid`` have a cache slot."""
    s = shape
    axes = 1 if s.rope == "table" else 3
    nq, nkv, hd = s.num_heads, s.num_kv_heads, s.head_dim
    norms = 2 * 8 * s.hidden * tokens
    prologue = tokens * (2 * ((nq + 2 * nkv) * hd + nq * hd + nkv * hd) + 8 * axes + 4) + valid * 2 * 2 * nkv * hd
    return norms + prologue + 6 * s.intermediate * tokens


def _rope_args(shape, device):
    from nano_vllm_multimodal_b200 import ops
    from nano_vllm_multimodal_b200.layers.multimodal_rotary_embedding import MultimodalRotaryEmbedding
    from nano_vllm_multimodal_b200.layers.rotary_embedding import RotaryEmbedding

    hd = shape.head_dim
    if shape.rope == "table":
        table = RotaryEmbedding(hd, hd, shape.max_position, shape.theta).to(device).cos_sin_cache
        return dict(rope_mode=ops.ROPE_TABLE, cos_sin_cache=table)
    mod = MultimodalRotaryEmbedding(head_dim=hd, base=shape.theta, sections=shape.sections,
                                    strategy=shape.rope).to(device)
    mode = ops.ROPE_MROPE_INTERLEAVED if shape.rope == "interleaved" else ops.ROPE_MROPE_CHUNKED
    return dict(rope_mode=mode, inv_freq=mod.inv_freq, sections=shape.sections)


def config_layer_gpu(config: int, device, hbm_peak: float, layers: int = 16, replays: int = 20,
                     tokens: int | None = None) -> dict:
    """One config's fused layer as the installed models run it (rounded add + text
    norm for Qwen3-VL, fused add+norm otherwise; the prologue with the config's
    q/k norm, rotary and store; SiluAndMul), ``layers`` layers captured in one CUDA
    graph and replayed. The layers cycle over enough separate activation sets that
    together they exceed 3x the L2, so bytes come from HBM."""
    import math

    from nano_vllm_multimodal_b200 import ops, workloads as W

    d = W.make_layer_inputs(config, device=device, tokens=tokens, extras=False)
    s, T = d["shape"], d["tokens"]
    valid = int((d["slot_mapping"] >= 0).sum())
    nbytes = layer_bytes(s, T, valid)
    nsets = max(2, math.ceil(3 * L2_BYTES / nbytes))
    keys = ("hidden", "residual", "qkv", "attn_out", "gate_up")
    g = torch.Generator(device=device).manual_seed(4000 + config)
    sets = [{k: d[k] for k in keys}] + [
        {k: torch.randn(d[k].shape, generator=g, device=device).to(d[k].dtype) for k in keys}
        for _ in range(nsets - 1)]
    rope = _rope_args(s, device)
    nq, nkv, hd = s.num_heads, s.num_kv_heads, s.head_dim
    text = s.qk_norm == "text"
    norm = dict(q_weight=d["q_weight"], k_weight=d["k_weight"], eps=s.eps) if s.qk_norm else {}
    views = []
    for a in sets:
        q, k, v = a["qkv"].split([nq * hd, nkv * hd, nkv * hd], -1)
        views.append((q.view(-1, nq, hd), k.view(-1, nkv, hd), v.view(-1, nkv, hd)))

    def step():
        for i in range(layers):
            a, (q, k, v) = sets[i % nsets], views[i % nsets]
            _, h1 = ops.add_rms_norm(a["hidden"], a["residual"], d["w_in"], s.eps, text)
            ops.qk_prologue(q, k, v=v, positions=d["positions"], key_cache=d["key_cache"],
                            value_cache=d["value_cache"], slot_mapping=d["slot_mapping"], **norm, **rope)
            ops.add_rms_norm(a["attn_out"], h1, d["w_post"], s.eps, text)
            ops.silu_and_mul(a["gate_up"])

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(replays):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (replays * layers)
    del graph
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"tokens": T, "us_per_layer": round(us, 3), "tokens_per_s": T / (us * 1e-6),
            "bytes_per_layer": nbytes, "achieved_gbs": round(gbs, 1), "frac": round(gbs / hbm_peak, 4),
            "input_sets": nsets, "launches_per_layer": 4, "layers_per_graph": layers}


def config_layer_cpu(config: int, budget_s: float) -> dict:
    """The same layer on the CPU over the config's full token count (the reference's
    modules when importable, else the oracle port), repeated for about ``budget_s``."""
    from nano_vllm_multimodal_b200 import workloads as W
    from oracle.cpu_layer import CpuLayer

    cores = host_threads()
    d = W.make_layer_inputs(config, extras=False)
    layer = CpuLayer(d["shape"], d)
    layer(d)  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        layer(d)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return {"cpu_tokens_per_s": d["tokens"] * reps / el, "cpu_kind": layer.kind, "cpu_cores": cores,
            "cpu_reps": reps}


CONFIG_NOTES = {
    1: "C1 Qwen3-0.6B layer: 512 tokens, hidden 1024, 16/8 heads, q/k RMSNorm, 1-D RoPE theta 1e6, I=3072",
    2: "C2 Qwen3-0.6B decode: 256 tokens, 10% slots -1, hidden 1024, 16/8 heads, 1-D RoPE, I=3072",
    3: "C3 Qwen3-VL-2B prefill: 16 x 2048 tokens, hidden 2048, 16/8 heads, text norm, interleaved "
       "M-RoPE [24,20,20] theta 5e6, I=6144",
    4: "C4 Qwen2.5-VL-3B mixed chunked step: 8192 + 120 tokens, hidden 2048, 16/2 heads, no q/k norm, "
       "chunked M-RoPE [16,24,24] theta 1e6, I=11008",
}


def config_table(device, hbm_peak: float, cpu_budget_s: float = 2.0) -> dict:
    out = {}
    for c in (1, 2, 3, 4):
        row = {"config": CONFIG_NOTES[c]}
        row.update(config_layer_gpu(c, device, hbm_peak))
        torch.cuda.empty_cache()
        if cpu_budget_s > 0:
            row.update(config_layer_cpu(c, cpu_budget_s))
            row["gpu_over_cpu"] = round(row["tokens_per_s"] / row["cpu_tokens_per_s"], 1)
        out[f"C{c}"] = row
    return out


# ------------------------------------------------------------------ arms


def reference_arm(args, rank, world):
    """The reference's CPU path on the host cores (rank 0 only): the same sample
    and extrapolation as the ``cpu_baseline`` leg of the GPU arm's line."""
    if rank != 0:
        return 0
    cores = host_threads()
    layer, d = cpu_c5_sample()
    for _ in range(max(1, args.warmup)):
        cpu_sample_step(layer, d)
    lt = gt = 0.0
    for _ in range(args.steps):
        a, b = cpu_sample_step(layer, d)
        lt, gt = lt + a, gt + b
    step_s, value = cpu_extrapolate(lt, gt, args.steps, args.tokens, args.layers)
    desc = cpu_sample_desc(layer.kind, args.steps, cores)
    cfg = config_block(args, 1, {
        "parallelism": "CPU, rank 0 only",
        "cpu_sample": {"step": f"one fused layer over {CPU_SAMPLE_TOKENS} C5 tokens + one {GATHER_LEN}-token "
                               "sequence gathered from K and V", "extrapolated_to": "the C5 step above, by "
                               "per-token cost", "gather_included": True, "kind": layer.kind}})
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * (lt + gt) / args.steps,
            "extrapolated_ms_per_c5_step": 1000 * step_s,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded, C5 shapes)", "config": cfg,
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": layer.kind, "sample": desc},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def ours_arm(args, rank, world, local):
    from nano_vllm_multimodal_b200 import ops  # noqa: F401  (loads the extension, fails loudly)

    visible = torch.cuda.device_count()
    if local >= visible:
        raise SystemExit(f"bench.py: rank {rank} wants cuda:{local} but {visible} GPU(s) are visible; "
                         f"run one rank per GPU (--nproc-per-node <= {visible})")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    if args.cache_blocks * 256 < -(-args.tokens // world) or args.cache_blocks < GATHER_LEN // 256:
        raise SystemExit("bench.py: --cache-blocks too small for the tokens per rank / gather length")
    inp = make_rank_inputs(rank, world, args.tokens, device, args.cache_blocks)
    T = inp["tokens"]
    torch.cuda.synchronize()

    # ---- warm-up + timed region (device-resident inputs)
    for _ in range(args.warmup):
        run_step(inp, args.layers)
    torch.cuda.synchronize()
    timer = LaunchTimer()
    clocks = ClockSampler(physical_gpu(local))
    if rank == 0:
        clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        run_step(inp, args.layers, timer)
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    clock = clocks.stop()
    ms = start.elapsed_time(end)
    ms_max = max_over_ranks(ms, world, device)
    kernels = timer.summary()

    tokens_job = args.tokens
    value = tokens_job * args.layers * args.steps / (ms_max / 1000.0)
    gather_tokens = inp["gather_seqs"] * GATHER_LEN
    step_bytes = T * args.layers * LAYER_BYTES + 2 * gather_tokens * BYTES["paged_gather"]
    step_bytes_job = max_over_ranks(float(step_bytes), world, device) * world

    # ---- per-kernel roofline (this rank's launches)
    hbm_peak, peak_src = measured_hbm_peak(with_source=True)
    traffic_tbl = load_traffic_table()
    per_kernel = {}
    for name, s in kernels.items():
        units = gather_tokens if name == "paged_gather" else T
        algo = BYTES[name] * units
        gbs = algo / (s["avg_ms"] / 1000.0) / 1e9
        per_kernel[name] = {"launches": s["launches"], "avg_ms": round(s["avg_ms"], 4),
                            "p50_ms": round(s["p50_ms"], 4),
                            "share": None, "bytes_per_launch": algo, "achieved_gbs": round(gbs, 1),
                            "frac": round(gbs / hbm_peak, 4)}
    total_k = sum(s["total_ms"] for s in kernels.values())
    for name, s in kernels.items():
        per_kernel[name]["share"] = round(s["total_ms"] / total_k, 4)
    dom = max(kernels, key=lambda n: kernels[n]["total_ms"])
    traffic = None
    if dom in traffic_tbl:
        traffic = traffic_tbl[dom] * (gather_tokens if dom == "paged_gather" else T)
    roofline = {"bound": "hbm", "kernel": dom, "achieved": per_kernel[dom]["achieved_gbs"],
                "peak": hbm_peak, "unit": "GB/s", "frac": per_kernel[dom]["frac"], "traffic": traffic,
                "peak_source": f"{peak_src} hbm_gbs (copy bandwidth)"}

    # ---- e2e through the layer API with host buffers in and out every step
    e2e = None
    if not args.no_e2e:
        pipe = E2EPipeline(inp, args.layers, build_modules(inp, device))
        pipe.run(max(1, args.warmup))
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        pipe.run(args.steps)
        e.record()
        torch.cuda.synchronize()
        barrier(world)
        e_ms = max_over_ranks(s.elapsed_time(e), world, device)
        h2d, d2h = pipe.bytes_per_step()
        e2e = {"value": tokens_job * args.layers * args.steps / (e_ms / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": int(max_over_ranks(float(h2d), world, device) * world),
               "d2h_bytes_per_step": int(max_over_ranks(float(d2h), world, device) * world),
               "ms_per_step": e_ms / args.steps,
               "copies": "pinned host buffers, H2D and D2H on two copy streams overlapping compute"}

    components = None
    if world == 1 and not args.no_components:
        components = component_bench(inp, device, hbm_peak)

    configs = None
    if world == 1 and not args.no_configs:
        configs = config_table(device, hbm_peak, 0.0 if args.no_cpu_baseline else args.config_cpu_seconds)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_seconds)

    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded, C5 shapes, random-init norm weights)",
        "config": config_block(args, world),
        # the long blocks first, so that a record keeping only the end of the line still holds the
        # roofline, e2e, CPU baseline, clocks and the per-kernel figures
        "components": components, "configs": configs,
        "hbm": {"algorithmic_bytes_per_step": step_bytes_job,
                "gbs": step_bytes_job / (ms_max / args.steps / 1000.0) / 1e9,
                "frac_of_peak": step_bytes_job / (ms_max / args.steps / 1000.0) / 1e9 / (hbm_peak * world),
                "peak_gbs": hbm_peak * world, "peak_note": "measured per-GPU copy bandwidth x GPUs"},
        "roofline": roofline, "e2e": e2e, "cpu_baseline": cpu, "clocks": clock,
        "gpu_launches": launches_per_step(args.layers, inp["gather_seqs"]) * args.steps,
        "kernels": per_kernel,
    }
    print(json.dumps(line), flush=True)
    return 0


def measured_hbm_peak(with_source=False):
    """HBM copy bandwidth (GB/s) from MEASURED_PEAKS.json, else the pool's fallback figure."""
    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    peak = peaks.get("hbm_gbs")
    src = "measured" if peak else "fallback"
    peak = peak or 6650.0
    return (peak, src) if with_source else peak


def component_only(name, decode_requests=256):
    """One standalone component on cuda:0 (for profiling a single kernel)."""
    from nano_vllm_multimodal_b200 import ops  # noqa: F401  (loads the extension, fails loudly)

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    hbm_peak = measured_hbm_peak()
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=device)
    out = {}

    def record(n, ms, nbytes, cfg):
        gbs = nbytes / (ms / 1000.0) / 1e9
        out[n] = {"avg_ms": round(ms, 4), "bytes": int(nbytes), "achieved_gbs": round(gbs, 1),
                  "frac": round(gbs / hbm_peak, 4), "config": cfg}

    if name == "decode_attention":
        decode_attention_component(out, record, flush, device, decode_requests)
    elif name == "rows":
        from nano_vllm_multimodal_b200 import workloads as W

        flushed = rows_flushed_rounds(flush, device)
        seeds = W._Seeds(2, device)
        seeds.index = 700
        rows_component(record, seeds, device, out)
        for k, v in flushed.items():
            out[k]["flushed_call_ms"] = round(v, 4)
    elif name == "visual_merge":
        from nano_vllm_multimodal_b200 import workloads as W

        seeds = W._Seeds(2, device)
        seeds.index = 700
        visual_merge_component(out, record, flush, seeds, W.deepstack_rows(3, W.C3.tokens).to(device), W.C3)
    elif name == "paged_store":
        # nanovllm_paged_kv::store alone at C5 head shapes: 65,536 tokens, k/v strided
        # views of qkv rows, random slots of a 1,024-block cache pair (about 2 GB in all)
        T = 65536
        g = torch.Generator(device=device).manual_seed(91)
        qkv = torch.randn(T, (NQ + 2 * NKV) * D, generator=g, device=device).to(torch.bfloat16)
        k = qkv[:, NQ * D:(NQ + NKV) * D].view(-1, NKV, D)
        v = qkv[:, (NQ + NKV) * D:].view(-1, NKV, D)
        kc = torch.zeros(1024, 256, NKV, D, dtype=torch.bfloat16, device=device)
        vc = torch.zeros_like(kc)
        slots = torch.randperm(kc.shape[0] * 256, generator=g, device=device)[:T].to(torch.int32)
        ms = _time_op(flush=flush, fn=lambda: ops.paged_store(k, v, kc, vc, slots))
        record("paged_store", ms, T * 4 * NKV * D * 2, f"C5 heads: {T} tokens, k/v strided views of the qkv rows, "
               "random slots; one call at a time after an L2 flush")
    elif name == "head_norm":
        # Qwen3 q_norm alone (RMSNorm over each head of a strided q view of the qkv
        # rows): 65,536 tokens x 16 heads of 128, bf16 weights
        T = 65536
        g = torch.Generator(device=device).manual_seed(92)
        qkv = torch.randn(T, (NQ + 2 * NKV) * D, generator=g, device=device).to(torch.bfloat16)
        q = qkv[:, : NQ * D].view(-1, NQ, D)
        w = (1.0 + 0.1 * torch.randn(D, generator=g, device=device)).to(torch.bfloat16)
        ms = _time_op(flush=flush, fn=lambda: ops.rms_norm(q, w, EPS))
        record("rms_norm_heads", ms, T * NQ * D * 2 * 2, f"q-norm: [{T},{NQ},{D}] strided view of the qkv rows; "
               "one call at a time after an L2 flush")
    elif name == "decode_layers":
        out["c2_decode_layer_graph"] = decode_layer_graph(device, 2)
        out["c3_decode_layer_graph"] = decode_layer_graph(device, 3)
    elif name == "configs":
        out.update(config_table(device, hbm_peak, 0.0))
    elif name == "mrope":
        inv = (1.0 / (THETA ** (torch.arange(0, D, 2, dtype=torch.float32) / D))).to(device)
        mrope_component(record, device, inv)
        rope_forward_component(record, device)
    else:
        step_inputs_component(out, device)
    print(json.dumps({"component": name, "peak_gbs": hbm_peak, **out}))
    return 0


def main(argv=None):
    args = parse_args(argv)
    rank, world, local = dist_env()
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    if args.component is not None:
        return component_only(args.component, args.decode_requests)
    if world != args.gpus and world == 1 and args.gpus > 1:
        print(f"bench.py: --gpus {args.gpus} needs torchrun with {args.gpus} processes", file=sys.stderr)
        return 2
    return ours_arm(args, rank, world, local)


if __name__ == "__main__":
    sys.exit(main())
