"""Host-side logic of the drop-in layer API (CPU only, nothing launched).

Mirrors the reference's validation tests
(``tests/test_paged_kv_backends.py:26-125``,
``tests/test_qwen3_vl_runtime.py:253-280``,
``tests/test_qwen25_vl_model.py``) against this package's modules."""

import os
from types import SimpleNamespace
from unittest.mock import patch

import numpy as np
import pytest
import torch

from nano_vllm_multimodal_b200 import workloads as W
from nano_vllm_multimodal_b200.layers.multimodal_rotary_embedding import (
    MultimodalRotaryEmbedding, apply_multimodal_rotary_emb)
from nano_vllm_multimodal_b200.layers.paged_kv import (
    create_paged_kv_backend, index_value_validation_enabled, resolve_paged_kv_backend_name,
    validate_gather_inputs, validate_store_inputs)
from nano_vllm_multimodal_b200.layers.rotary_embedding import RotaryEmbedding


def store_inputs():
    key = torch.arange(3 * 2 * 4, dtype=torch.float32).reshape(3, 2, 4)
    value = key + 100
    kc = torch.full((3, 4, 2, 4), -1.0)
    return key, value, kc, torch.full_like(kc, -1.0), torch.tensor([0, 5, -1], dtype=torch.int32)


def test_gpu_index_value_validation_is_debug_opt_in():
    cuda_t, cpu_t = SimpleNamespace(is_cuda=True), SimpleNamespace(is_cuda=False)
    with patch.dict(os.environ, {}, clear=False):
        os.environ.pop("NANOVLLM_PAGED_KV_VALIDATE_INDICES", None)
        assert not index_value_validation_enabled(cuda_t)
        assert index_value_validation_enabled(cpu_t)
    with patch.dict(os.environ, {"NANOVLLM_PAGED_KV_VALIDATE_INDICES": "1"}):
        assert index_value_validation_enabled(cuda_t)


def test_store_validation_messages():
    key, value, kc, vc, slots = store_inputs()
    d = validate_store_inputs(key, value, kc, vc, slots)
    assert (d.num_tokens, d.num_kv_heads, d.head_dim, d.num_slots) == (3, 2, 4, 12)
    cases = [((key[:2], value, kc, vc, slots), "matching shape"),
             ((key, value, kc[:, :, :1], vc, slots), "cache shape"),
             ((key, value, kc, vc, slots.to(torch.int64)), "int32"),
             ((key.transpose(1, 2), value.transpose(1, 2), kc, vc, slots), "inner dimensions")]
    for args, msg in cases:
        with pytest.raises(ValueError, match=msg):
            validate_store_inputs(*args)
    slots[1] = 12
    with pytest.raises(ValueError, match="slot"):
        validate_store_inputs(key, value, kc, vc, slots)


def test_gather_validation_messages():
    cache = torch.zeros(3, 4, 2, 4)
    table = torch.tensor([2, 0], dtype=torch.int32)
    assert validate_gather_inputs(cache, table, 6).required_blocks == 2
    with pytest.raises(ValueError, match="non-negative"):
        validate_gather_inputs(cache, table, -1)
    with pytest.raises(ValueError, match="int32"):
        validate_gather_inputs(cache, table.to(torch.int64), 6)
    with pytest.raises(ValueError, match="cover"):
        validate_gather_inputs(cache, table[:1], 6)
    with pytest.raises(ValueError, match="physical block"):
        validate_gather_inputs(cache, torch.tensor([3, 0], dtype=torch.int32), 6)


def test_backend_resolution_and_factory():
    for name in ("pytorch", "triton", "cuda"):
        assert resolve_paged_kv_backend_name(name, cuda_available=True, cuda_extension_available=True) == name
    assert resolve_paged_kv_backend_name("auto", cuda_available=True, cuda_extension_available=True) == "cuda"
    assert resolve_paged_kv_backend_name("auto", cuda_available=True, cuda_extension_available=False) == "triton"
    assert resolve_paged_kv_backend_name("auto", cuda_available=False, cuda_extension_available=False) == "pytorch"
    with pytest.raises(ValueError, match="paged_kv_backend"):
        resolve_paged_kv_backend_name("flash", cuda_available=True, cuda_extension_available=True)
    assert create_paged_kv_backend("cuda").name == "cuda"  # constructing does not build or load
    with pytest.raises(ValueError, match="unknown paged KV backend"):
        create_paged_kv_backend("pytorch")


def test_cuda_backend_rejects_cpu_tensors_and_devices():
    backend = create_paged_kv_backend("cuda")
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        backend.store(*store_inputs())
    with pytest.raises(ValueError, match="requires a CUDA device"):
        backend.allocate((2, 1, 4, 1, 8), dtype=torch.float16, device="cpu")
    with pytest.raises(ValueError, match="does not support dtype"):
        backend.allocate((2, 1, 4, 1, 8), dtype=torch.int8, device="cuda")


def test_mrope_constructor_validation():
    with pytest.raises(ValueError, match="strategy"):
        MultimodalRotaryEmbedding(head_dim=128, base=1e6, sections=(24, 20, 20), strategy="striped")
    with pytest.raises(ValueError, match="even"):
        MultimodalRotaryEmbedding(head_dim=127, base=1e6, sections=(24, 20, 20))
    with pytest.raises(ValueError, match="sum to half"):
        MultimodalRotaryEmbedding(head_dim=128, base=1e6, sections=(24, 20, 21))
    with pytest.raises(ValueError, match="three positive"):
        MultimodalRotaryEmbedding(head_dim=128, base=1e6, sections=(24, 40, 0))
    m = MultimodalRotaryEmbedding(head_dim=128, base=1e6, sections=(16, 24, 24))
    assert m.strategy == "chunked"
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    assert torch.equal(m.inv_freq, inv)


def test_apply_mrope_validation_before_launch():
    q, k = torch.randn(3, 2, 128), torch.randn(3, 1, 128)
    cos = torch.randn(3, 3, 128)
    with pytest.raises(ValueError, match=r"\[num_tokens, num_heads, head_dim\]"):
        apply_multimodal_rotary_emb(q[0], k, cos, cos, (16, 24, 24))
    with pytest.raises(ValueError, match="equal shape"):
        apply_multimodal_rotary_emb(q, k, cos, cos[:2], (16, 24, 24))
    with pytest.raises(ValueError, match="token count"):
        apply_multimodal_rotary_emb(q[:2], k[:2], cos, cos, (16, 24, 24))
    with pytest.raises(ValueError, match="same head dimension"):
        apply_multimodal_rotary_emb(q[..., :64], k[..., :64], cos, cos, (16, 24, 24))
    with pytest.raises(ValueError, match="cover the head dimension"):
        apply_multimodal_rotary_emb(q, k, cos, cos, (16, 24, 23))
    with pytest.raises(ValueError, match="strategy"):
        apply_multimodal_rotary_emb(q, k, cos, cos, (16, 24, 24), strategy="striped")
    m = MultimodalRotaryEmbedding(head_dim=128, base=1e6, sections=(16, 24, 24))
    with pytest.raises(ValueError, match=r"positions must have shape \[3, num_tokens\]"):
        m.cos_sin(torch.zeros(2, 3, dtype=torch.long), torch.float32)


def test_rotary_table_is_the_reference_recipe():
    r = RotaryEmbedding(128, 128, 64, 1e6)
    assert r.cos_sin_cache.shape == (64, 1, 128)
    assert r.cos_sin_cache.dtype == torch.float32
    assert torch.equal(r.cos_sin_cache[0, 0, :64], torch.ones(64))
    with pytest.raises(AssertionError):
        RotaryEmbedding(128, 64, 64, 1e6)


def test_embedding_module_construction_matches_reference_sharding():
    with patch("torch.distributed.get_rank", return_value=1), \
            patch("torch.distributed.get_world_size", return_value=2):
        from nano_vllm_multimodal_b200.layers.embed_head import VocabParallelEmbedding
        e = VocabParallelEmbedding(64, 16)
    assert (e.vocab_start_idx, e.vocab_end_idx, tuple(e.weight.shape)) == (32, 64, (32, 16))
    full = torch.arange(64 * 16, dtype=torch.float32).view(64, 16)
    e.weight.weight_loader(e.weight, full)
    assert torch.equal(e.weight.data, full[32:])


def test_workload_shapes_and_determinism():
    a = W.make_layer_inputs(2, tokens=256, cache=False)
    b = W.make_layer_inputs(2, tokens=256, cache=False)
    assert torch.equal(a["qkv"], b["qkv"]) and torch.equal(a["slot_mapping"], b["slot_mapping"])
    assert int((a["slot_mapping"] == -1).sum()) == 26
    assert a["qkv"].shape == (256, 32 * 128)
    c3 = W.make_layer_inputs(3, tokens=4096, cache=False)
    assert c3["positions"].shape == (3, 4096)
    assert c3["deepstack_rows"].numel() == 2048 and c3["deepstack"][0].shape == (2048, 2048)
    # image span of sequence 0: rows 512..1535, H/W axes follow the 32x32 grid
    pos = c3["positions"]
    assert pos[0, 512].item() == 512 and pos[1, 512 + 33].item() == 513 and pos[2, 512 + 33].item() == 513
    c4 = W.make_layer_inputs(4, cache=False)
    assert c4["positions"].shape == (3, 8312)
    assert torch.equal(c4["positions"][0, 8192:], c4["positions"][1, 8192:])
    tables = W.make_gather_inputs(5, sequences=3, seq_len=16384, num_blocks=1024)
    assert tables.shape == (3, 64) and all(t.unique().numel() == 64 for t in tables)


# ------------------------------------------------ visual merge: host-side validation (no GPU)


def _vm_plan(rows):
    from types import SimpleNamespace
    return SimpleNamespace(replacements=tuple(SimpleNamespace(output_row=o, feature_key=k, feature_row=f)
                                              for o, k, f in rows))


def test_visual_merge_validation_messages_match_reference():
    """model_runner.py:175-235: the same exception types and messages, in the same order."""
    from types import SimpleNamespace

    from nano_vllm_multimodal_b200.layers.visual_merge import build_planned_visual_embeddings as build

    tok = torch.zeros(5, 4)
    with pytest.raises(ValueError, match=r"token embeddings must have shape \[tokens, hidden_size\]"):
        build(torch.zeros(5), _vm_plan([(0, "a", 0)]), {})
    # no replacements: the input object itself, no payloads, empty rows
    out = build(tok, _vm_plan([]), {})
    assert out.final_embedding is tok and out.deepstack_embeddings == () and out.visual_rows.numel() == 0
    with pytest.raises(KeyError, match="missing visual feature: a"):
        build(tok, _vm_plan([(0, "a", 0)]), {})
    with pytest.raises(TypeError, match="visual feature must be a bundle: a"):
        build(tok, _vm_plan([(0, "a", 0)]), {"a": [1, 2]})
    with pytest.raises(ValueError, match="final vision embedding must be rank-2"):
        build(tok, _vm_plan([(0, "a", 0)]), {"a": torch.zeros(4)})
    with pytest.raises(ValueError, match="hidden size mismatch"):
        build(tok, _vm_plan([(0, "a", 0)]), {"a": torch.zeros(2, 3)})
    bundle1 = SimpleNamespace(final_embedding=torch.zeros(2, 4), deepstack_embeddings=(torch.zeros(2, 4),))
    with pytest.raises(ValueError, match="deepstack layer count"):
        build(tok, _vm_plan([(0, "a", 0), (1, "b", 0)]), {"a": bundle1, "b": torch.zeros(2, 4)})
    with pytest.raises(IndexError, match="visual output row is out of range: 5"):
        build(tok, _vm_plan([(5, "a", 0)]), {"a": torch.zeros(2, 4)})
    with pytest.raises(IndexError, match="visual feature row is out of range: key=a, row=2"):
        build(tok, _vm_plan([(0, "a", 2)]), {"a": torch.zeros(2, 4)})
    too_deep = SimpleNamespace(final_embedding=torch.zeros(2, 4),
                               deepstack_embeddings=tuple(torch.zeros(2, 4) for _ in range(9)))
    with pytest.raises(NotImplementedError, match="at most 8 DeepStack layers"):
        build(tok, _vm_plan([(0, "a", 0)]), {"a": too_deep})


def test_visual_merge_reports_the_first_error_in_plan_order():
    """The reference validates in one loop over the plan: a key's checks at its first
    replacement, then that replacement's rows. The vectorised checks raise the same one."""
    from nano_vllm_multimodal_b200.layers.visual_merge import build_planned_visual_embeddings as build

    tok = torch.zeros(5, 4)
    feats = {"a": torch.zeros(2, 4)}
    with pytest.raises(IndexError, match="visual output row is out of range: 9"):
        build(tok, _vm_plan([(9, "a", 0), (1, "missing", 0)]), feats)
    with pytest.raises(KeyError, match="missing visual feature: missing"):
        build(tok, _vm_plan([(1, "missing", 0), (9, "a", 0)]), feats)
    with pytest.raises(IndexError, match="feature row is out of range: key=a, row=7"):
        build(tok, _vm_plan([(0, "a", 0), (1, "a", 7), (9, "a", 0)]), feats)
    with pytest.raises(IndexError, match="visual output row is out of range: -1"):
        build(tok, _vm_plan([(0, "a", 0), (-1, "a", 7)]), feats)  # output row is checked first


def test_step_input_block_tables_are_padded_as_the_reference_pads_them():
    """prepare_block_tables (model_runner.py:696-707): rows of different lengths,
    padded on the right with -1 to the longest; an empty batch gives [0, 0]."""
    from nano_vllm_multimodal_b200.step_inputs import _padded_tables, host_array

    t = _padded_tables([[4, 5, 6], [7], [], [1, 2]])
    assert t.dtype.name == "int32" and t.shape == (4, 3)
    assert t.tolist() == [[4, 5, 6], [7, -1, -1], [-1, -1, -1], [1, 2, -1]]
    assert _padded_tables([]).shape == (0, 0)
    h = host_array(t, torch.int32)
    assert h.dtype == torch.int32 and h.shape == (4, 3) and h.tolist() == t.tolist()
    rows = tuple((5, 6, 7) for _ in range(3))  # build_decode_position_rows' tuple of tuples
    for v in (rows, [list(r) for r in rows], rows[0], list(rows[0]), np.asarray(rows)):
        h = host_array(v, torch.int64)
        assert h.dtype == torch.int64 and h.tolist() == np.asarray(v).tolist()
