"""Child process of tests/test_gpu_pdl.py: one run of a fixed chain of this
library's kernels on seeded inputs, eagerly and then replayed from a CUDA graph,
printing a sha256 of every output as JSON. The parent runs it with programmatic
dependent launch off and on (``NIB_B200_PDL`` is read once per process).

The chain: 4 decode-sized Qwen3-VL-2B layers (rounded add + text norm, the
fused q/k norm + interleaved M-RoPE + paged store, SiluAndMul), then a paged
decode attention over the caches they filled, with contexts split over CTAs
(the split merge is the one launch that always takes a programmatic
dependency).

Usage: python tests/_pdl_child.py
"""

import hashlib
import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from nano_vllm_multimodal_b200 import ops, workloads as W  # noqa: E402
from nano_vllm_multimodal_b200.layers.multimodal_rotary_embedding import MultimodalRotaryEmbedding  # noqa: E402

LAYERS, REQUESTS = 4, 16


def digest(tensors):
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def main():
    torch.cuda.set_device(0)
    d = W.make_layer_inputs(3, tokens=256, device="cuda")
    shp = d["shape"]
    nq, nkv, hd = shp.num_heads, shp.num_kv_heads, shp.head_dim
    mod = MultimodalRotaryEmbedding(head_dim=hd, base=shp.theta, sections=shp.sections,
                                    strategy=shp.rope).to("cuda")
    rope = dict(rope_mode=ops.ROPE_MROPE_INTERLEAVED, inv_freq=mod.inv_freq, sections=shp.sections)
    q, k, v = d["qkv"].split([nq * hd, nkv * hd, nkv * hd], -1)
    q, k, v = q.view(-1, nq, hd), k.view(-1, nkv, hd), v.view(-1, nkv, hd)

    g = torch.Generator().manual_seed(7)
    blocks, bs = d["key_cache"].shape[0], d["key_cache"].shape[1]
    per = blocks // REQUESTS
    tables = torch.randperm(blocks, generator=g).to(torch.int32).view(REQUESTS, per).cuda()
    lens = torch.randint(1, per * bs + 1, (REQUESTS,), generator=g, dtype=torch.int32).cuda()
    qd = torch.randn(REQUESTS, nq, hd, generator=g).to(torch.bfloat16).cuda()

    def chain():
        outs = []
        h, res = d["hidden"], d["residual"]
        for _ in range(LAYERS):
            y, h1 = ops.add_rms_norm(h, res, d["w_in"], 1e-6, True)
            qr, kr = ops.qk_prologue(q, k, v=v, positions=d["positions"], q_weight=d["q_weight"],
                                     k_weight=d["k_weight"], eps=1e-6, key_cache=d["key_cache"],
                                     value_cache=d["value_cache"], slot_mapping=d["slot_mapping"], **rope)
            y2, h2 = ops.add_rms_norm(d["attn_out"], h1, d["w_post"], 1e-6, True)
            act = ops.silu_and_mul(d["gate_up"])
            outs += [y, h1, qr, kr, y2, h2, act]
            h, res = y2, h2
        att = ops.decode_attention(qd, d["key_cache"], d["value_cache"], lens, tables, hd ** -0.5)
        return outs + [att, d["key_cache"], d["value_cache"]]

    eager = digest(chain())
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        chain()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = chain()
    graph.replay()
    graph.replay()
    torch.cuda.synchronize()
    replayed = digest(captured)
    del graph
    print(json.dumps({"eager": eager, "graph": replayed}))


if __name__ == "__main__":
    main()
