"""``integration.install()`` against the reference's own ``nanovllm`` package (CPU).

Runs only where the NanoInfer package is importable: ``$NANOINFER_REF``, or an
install in the git-ignored ``baseline/_ref``; elsewhere it skips. Each check runs in a fresh interpreter, so the reference's modules
never enter this test session.

It imports a reference model module before ``install()`` (the model binds the
layer classes at import time), installs, and builds a small Qwen3 decoder layer
from the reference's own model code. The layer must be made of this package's
layers, and its parameter names must equal those of the same layer built without
``install()``: the reference's weight loader finds parameters by name.
"""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = Path(os.environ.get("NANOINFER_REF") or ROOT / "baseline" / "_ref")

pytestmark = pytest.mark.skipif(not (REF / "nanovllm" / "__init__.py").is_file(),
                                reason=f"NanoInfer reference not importable from {REF}")

SCRIPT = r"""
import json, sys, types
sys.path[:0] = [sys.argv[1], sys.argv[2]]
import torch.distributed as dist
dist.get_rank = lambda *a, **k: 0          # tensor-parallel layers build without a process group
dist.get_world_size = lambda *a, **k: 1
import nanovllm.models.qwen3 as q3         # binds the layer classes before install()
import nanovllm.models.qwen3_vl as q3vl
done = []
if sys.argv[3] == "install":
    from nano_vllm_multimodal_b200.integration import install
    done = install()
cfg = types.SimpleNamespace(hidden_size=128, num_attention_heads=2, num_key_value_heads=1,
                            max_position_embeddings=64, rms_norm_eps=1e-6, attention_bias=False,
                            head_dim=64, rope_theta=1e6, rope_scaling=None, intermediate_size=256,
                            hidden_act="silu")
layer = q3.Qwen3DecoderLayer(cfg)
kinds = {
    "input_layernorm": type(layer.input_layernorm).__module__,
    "q_norm": type(layer.self_attn.q_norm).__module__,
    "rotary_emb": type(layer.self_attn.rotary_emb).__module__,
    "act_fn": type(layer.mlp.act_fn).__module__,
    "qwen3_vl.Qwen3VLTextRMSNorm": q3vl.Qwen3VLTextRMSNorm.__module__,
    "qwen3_vl._add_deepstack_rows": q3vl.Qwen3VLLanguageModel._add_deepstack_rows.__module__,
}
params = sorted((n, list(p.shape)) for n, p in layer.named_parameters())
buffers = sorted(n for n, _ in layer.named_buffers())
print(json.dumps({"done": done, "kinds": kinds, "params": params, "buffers": buffers}))
"""


def _run(mode):
    env = dict(os.environ, TORCHDYNAMO_DISABLE="1")
    r = subprocess.run([sys.executable, "-c", SCRIPT, str(ROOT), str(REF), mode], capture_output=True,
                       text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_install_rebinds_the_reference_layers_and_keeps_parameter_names():
    ref = _run("reference")
    ours = _run("install")
    for what, module in ours["kinds"].items():
        assert module.startswith("nano_vllm_multimodal_b200."), (what, module)
    for what, module in ref["kinds"].items():
        assert module.startswith("nanovllm."), (what, module)
    assert ours["params"] == ref["params"]
    assert ours["buffers"] == ref["buffers"]
    for name in ("nanovllm.layers.layernorm.RMSNorm", "nanovllm.layers.attention.store_kvcache",
                 "nanovllm.layers.attention.flash_attn_with_kvcache",
                 "nanovllm.layers.paged_kv.loader.load_paged_kv_extension",
                 "nanovllm.engine.model_runner.build_planned_visual_embeddings",
                 "nanovllm.models.qwen3.RMSNorm", "nanovllm.models.qwen3.get_rope",
                 "nanovllm.models.qwen3_vl.Qwen3VLTextRMSNorm"):
        assert name in ours["done"], name
