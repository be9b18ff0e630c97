"""Seeded synthetic workloads C1-C5 for the per-token elementwise path.

Every tensor gets its own ``torch.Generator`` seeded ``1000 * config + index``
so a workload is reproducible on its own, whatever else was generated before.
Parity tests build a workload on the CPU and copy it to the GPU (identical
bytes on both sides); the benchmark may build the large C5 workload directly
on the device (same shapes and distributions, different draws).

Shapes follow the reference models: Qwen3-0.6B (``nanovllm/models/qwen3.py``),
Qwen3-VL-2B (``nanovllm/models/qwen3_vl.py``) and Qwen2.5-VL-3B
(``nanovllm/models/qwen25_vl.py``). Multimodal 3-axis positions are built with
the static-image rule of ``nanovllm/multimodal/qwen3_vl_runtime.py:12-120``:
text tokens advance all three axes together from ``max_position + 1``; an image
span of LLM grid ``t x h x w`` starting at ``base`` takes
``(base + ti, base + hi, base + wi)`` and moves ``max_position`` to
``base + max(t, h, w) - 1``.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

BF16 = torch.bfloat16


@dataclass(frozen=True)
class Shape:
    name: str
    tokens: int
    hidden: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    qk_norm: str | None  # "rms" (Qwen3), "text" (Qwen3-VL) or None (Qwen2.5-VL)
    rope: str  # "table", "interleaved" or "chunked"
    theta: float
    sections: tuple[int, int, int] | None
    num_blocks: int
    block_size: int = 256
    max_position: int = 40960
    eps: float = 1e-6
    extra: dict = field(default_factory=dict)

    @property
    def qkv_width(self) -> int:
        return (self.num_heads + 2 * self.num_kv_heads) * self.head_dim


C1 = Shape("C1-qwen3-0.6b-layer", 512, 1024, 16, 8, 128, 3072, "rms", "table", 1e6, None, 64)
C2 = Shape("C2-qwen3-0.6b-decode", 256, 1024, 16, 8, 128, 3072, "rms", "table", 1e6, None, 4096,
           extra={"vocab": 151936})
C3 = Shape("C3-qwen3-vl-2b-prefill", 16 * 2048, 2048, 16, 8, 128, 6144, "text", "interleaved", 5e6,
           (24, 20, 20), 256, extra={"sequences": 16, "seq_len": 2048})
C4 = Shape("C4-qwen2.5-vl-3b-mixed", 8192 + 120, 2048, 16, 2, 128, 11008, None, "chunked", 1e6,
           (16, 24, 24), 256)
C5 = Shape("C5-qwen3-vl-2b-sweep", 262144, 2048, 16, 8, 128, 6144, "text", "interleaved", 5e6,
           (24, 20, 20), 16384, extra={"layers": 28, "gather_sequences": 64, "gather_len": 16384})

CONFIGS = {1: C1, 2: C2, 3: C3, 4: C4, 5: C5}


class _Seeds:
    """One generator per tensor: seed ``1000 * config + running index``."""

    def __init__(self, config: int, device):
        self.config = config
        self.index = 0
        self.device = torch.device(device)

    def __call__(self) -> torch.Generator:
        g = torch.Generator(device=self.device)
        g.manual_seed(1000 * self.config + self.index)
        self.index += 1
        return g


def _normal(seeds, shape, mean=0.0, std=1.0, dtype=BF16):
    g = seeds()
    t = torch.randn(shape, generator=g, device=seeds.device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    if mean != 0.0:
        t.add_(mean)
    return t.to(dtype)


def _randperm(seeds, n, k):
    g = seeds()
    return torch.randperm(n, generator=g, device=seeds.device)[:k].to(torch.int32)


def image_positions(segments):
    """3-axis positions for a prompt made of text runs and image spans.

    ``segments`` is a list of ``("text", length)`` or ``("image", t, h, w)``
    (LLM grid, already merged). Returns ``(positions [3, n] int64, image_rows)``
    where ``image_rows`` lists the prompt rows that hold image tokens.
    """
    axes = [[], [], []]
    rows = []
    max_pos = -1
    cursor = 0
    for seg in segments:
        if seg[0] == "text":
            n = seg[1]
            for a in axes:
                a.extend(range(max_pos + 1, max_pos + 1 + n))
            if n:
                max_pos += n
            cursor += n
        else:
            _, gt, gh, gw = seg
            base = max_pos + 1
            for ti in range(gt):
                for hi in range(gh):
                    for wi in range(gw):
                        axes[0].append(base + ti)
                        axes[1].append(base + hi)
                        axes[2].append(base + wi)
            n = gt * gh * gw
            rows.extend(range(cursor, cursor + n))
            cursor += n
            max_pos = max(max_pos, base + max(gt, gh, gw) - 1)
    return torch.tensor(axes, dtype=torch.int64), rows


def layer_weights(shape: Shape, seeds):
    return {
        "w_in": _normal(seeds, (shape.hidden,), 1.0, 0.1),
        "w_post": _normal(seeds, (shape.hidden,), 1.0, 0.1),
        "q_weight": _normal(seeds, (shape.head_dim,), 1.0, 0.1),
        "k_weight": _normal(seeds, (shape.head_dim,), 1.0, 0.1),
    }


def positions_for(config: int, shape: Shape, seeds, tokens: int):
    """Positions of each config: ``[T]`` for 1-D RoPE, ``[3, T]`` for M-RoPE."""
    if config == 1:
        return torch.arange(tokens, dtype=torch.int64, device=seeds.device)
    if config == 2:
        return torch.randint(0, 8192, (tokens,), generator=seeds(), device=seeds.device)
    if config == 3:
        seq_len = shape.extra["seq_len"]
        pos, _ = image_positions([("text", 512), ("image", 1, 32, 32), ("text", 512)])
        reps = -(-tokens // seq_len)
        return pos.repeat(1, reps)[:, :tokens].contiguous().to(seeds.device)
    if config == 4:
        chunk, _ = image_positions([("text", 1024), ("image", 1, 32, 64), ("text", 2048),
                                    ("image", 1, 32, 64), ("text", 1024)])
        dec = torch.randint(0, 16384, (120,), generator=seeds(), device=seeds.device).cpu()
        pos = torch.cat((chunk, dec.expand(3, -1)), dim=1)
        return pos[:, :tokens].contiguous().to(seeds.device)
    if config == 5:
        return torch.randint(0, 32768, (3, tokens), generator=seeds(), device=seeds.device)
    raise ValueError(f"unknown config {config}")


def deepstack_rows(config: int, tokens: int):
    """Global image rows of C3 (16 sequences, each 512 text + 1024 image + 512 text)."""
    if config != 3:
        return torch.empty(0, dtype=torch.int64)
    rows = []
    for s in range(-(-tokens // 2048)):
        rows.extend(r for r in range(s * 2048 + 512, s * 2048 + 1536) if r < tokens)
    return torch.tensor(rows, dtype=torch.int64)


def make_layer_inputs(config: int, *, tokens: int | None = None, device="cpu", cache=True, extras=True):
    """Inputs of one fused layer for config ``config`` (optionally truncated).

    Keys: ``hidden``, ``residual``, ``qkv``, ``attn_out``, ``gate_up``,
    ``positions``, ``slot_mapping``, ``key_cache``/``value_cache`` (prefilled
    with -3, as the reference's parity tests do), the four norm weights, and for
    C2 ``embedding``/``token_ids``, for C3 ``deepstack`` rows and tensors
    (``extras=False`` leaves those out).
    """
    shape = CONFIGS[config]
    T = shape.tokens if tokens is None else tokens
    seeds = _Seeds(config, device)
    out = {"shape": shape, "tokens": T}
    out["hidden"] = _normal(seeds, (T, shape.hidden))
    out["residual"] = _normal(seeds, (T, shape.hidden))
    out["qkv"] = _normal(seeds, (T, shape.qkv_width))
    out["attn_out"] = _normal(seeds, (T, shape.hidden))
    out["gate_up"] = _normal(seeds, (T, 2 * shape.intermediate))
    out.update(layer_weights(shape, seeds))
    out["positions"] = positions_for(config, shape, seeds, T)
    slots_total = shape.num_blocks * shape.block_size
    slots = _randperm(seeds, slots_total, T)
    if config == 2:
        g = seeds()
        skip = torch.randperm(T, generator=g, device=seeds.device)[: max(1, round(0.1 * T))]
        slots[skip] = -1
    out["slot_mapping"] = slots
    if cache:
        cshape = (shape.num_blocks, shape.block_size, shape.num_kv_heads, shape.head_dim)
        out["key_cache"] = torch.full(cshape, -3.0, dtype=BF16, device=device)
        out["value_cache"] = torch.full(cshape, -3.0, dtype=BF16, device=device)
    if config == 2 and extras:
        vocab = shape.extra["vocab"]
        out["embedding"] = _normal(seeds, (vocab, shape.hidden), 0.0, 0.02)
        out["token_ids"] = torch.randint(0, vocab, (T,), generator=seeds(), device=seeds.device)
    if config == 3 and extras:
        rows = deepstack_rows(3, T).to(device)
        out["deepstack_rows"] = rows
        out["deepstack"] = [_normal(seeds, (rows.numel(), shape.hidden)) for _ in range(3)]
    return out


def make_gather_inputs(config: int, *, sequences: int, seq_len: int, num_blocks: int,
                       block_size: int = 256, device="cpu", seed_offset: int = 500):
    """Random block tables for the paged-KV gather: each sequence gets
    ``ceil(seq_len / block_size)`` distinct physical blocks."""
    seeds = _Seeds(config, device)
    seeds.index = seed_offset
    need = -(-seq_len // block_size)
    tables = torch.stack([
        torch.randperm(num_blocks, generator=seeds(), device=seeds.device)[:need].to(torch.int32)
        for _ in range(sequences)
    ])
    return tables
