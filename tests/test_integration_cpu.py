"""``integration.install()`` against a stand-in ``nanovllm`` package (CPU only).

The stand-in has the module layout and names of the reference (nothing of its
code): install() must rebind exactly the hot-path names, including names a
model module imported before install ran."""

import sys
import textwrap

import pytest


@pytest.fixture()
def fake_nanovllm(tmp_path, monkeypatch):
    files = {
        "nanovllm/__init__.py": "",
        "nanovllm/layers/__init__.py": "",
        "nanovllm/layers/layernorm.py": "class RMSNorm: pass\n",
        "nanovllm/layers/activation.py": "class SiluAndMul: pass\n",
        "nanovllm/layers/rotary_embedding.py": "class RotaryEmbedding: pass\ndef get_rope(*a): pass\n"
                                               "def apply_rotary_emb(*a): pass\n",
        "nanovllm/layers/multimodal_rotary_embedding.py": "class MultimodalRotaryEmbedding: pass\n"
                                                          "def apply_multimodal_rotary_emb(*a): pass\n",
        "nanovllm/layers/embed_head.py": "class VocabParallelEmbedding: pass\n",
        "nanovllm/layers/attention.py": "def store_kvcache(*a): pass\ndef flash_attn_with_kvcache(*a, **k): pass\n",
        "nanovllm/layers/paged_kv/__init__.py": "",
        "nanovllm/layers/paged_kv/loader.py": "def load_paged_kv_extension(*, verbose=False): raise RuntimeError('jit')\n",
        "nanovllm/layers/paged_kv/cuda_backend.py": "from nanovllm.layers.paged_kv.loader import load_paged_kv_extension\n",
        "nanovllm/engine/__init__.py": "",
        "nanovllm/engine/model_runner.py": textwrap.dedent("""
            from dataclasses import dataclass
            @dataclass(frozen=True)
            class PlannedVisualEmbeddings:
                final_embedding: object
                deepstack_embeddings: tuple
                visual_rows: object
            def build_planned_visual_embeddings(t, p, f): raise RuntimeError('reference')
            def merge_planned_visual_embeddings(t, p, f): raise RuntimeError('reference')
        """),
        "nanovllm/models/__init__.py": "",
        "nanovllm/models/qwen3.py": textwrap.dedent("""
            from nanovllm.layers.layernorm import RMSNorm
            from nanovllm.layers.activation import SiluAndMul
            from nanovllm.layers.rotary_embedding import get_rope
        """),
        "nanovllm/models/qwen3_vl.py": textwrap.dedent("""
            class Qwen3VLTextRMSNorm: pass
            class Qwen3VLLanguageModel:
                @staticmethod
                def _add_deepstack_rows(h, r, v): return None
        """),
    }
    for rel, text in files.items():
        p = tmp_path / rel
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_text(text)
    monkeypatch.syspath_prepend(str(tmp_path))
    for name in [m for m in sys.modules if m == "nanovllm" or m.startswith("nanovllm.")]:
        monkeypatch.delitem(sys.modules, name)
    yield
    for name in [m for m in sys.modules if m == "nanovllm" or m.startswith("nanovllm.")]:
        del sys.modules[name]


def test_install_rebinds_hot_path_names(fake_nanovllm):
    import nanovllm.models.qwen3 as q3  # imported before install: holds the old names
    import nanovllm.models.qwen3_vl as q3vl

    from nano_vllm_multimodal_b200 import integration
    from nano_vllm_multimodal_b200.layers import activation, layernorm, qwen3_vl, rotary_embedding

    done = integration.install()
    import nanovllm.layers.layernorm as ln
    import nanovllm.layers.paged_kv.cuda_backend as cb

    assert ln.RMSNorm is layernorm.RMSNorm
    assert q3.RMSNorm is layernorm.RMSNorm and q3.SiluAndMul is activation.SiluAndMul
    assert q3.get_rope is rotary_embedding.get_rope
    assert q3vl.Qwen3VLTextRMSNorm is qwen3_vl.Qwen3VLTextRMSNorm
    assert q3vl.Qwen3VLLanguageModel._add_deepstack_rows is qwen3_vl.add_deepstack_rows
    assert "nanovllm.layers.paged_kv.loader.load_paged_kv_extension" in done
    assert cb.load_paged_kv_extension.__module__ == "nano_vllm_multimodal_b200.integration"
    # the visual merge: rebound, and an empty plan returns the reference's result type
    import nanovllm.engine.model_runner as mr
    import torch
    from types import SimpleNamespace
    assert "nanovllm.engine.model_runner.build_planned_visual_embeddings" in done
    import nanovllm.layers.attention as at
    from nano_vllm_multimodal_b200.layers import attention as our_attention
    assert at.flash_attn_with_kvcache is our_attention.flash_attn_with_kvcache
    tok = torch.zeros(3, 4)
    res = mr.build_planned_visual_embeddings(tok, SimpleNamespace(replacements=()), {})
    assert type(res) is mr.PlannedVisualEmbeddings and res.final_embedding is tok
    assert mr.merge_planned_visual_embeddings(tok, SimpleNamespace(replacements=()), {}) is tok
