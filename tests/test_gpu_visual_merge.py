"""Packed-prefill visual merge (``build_planned_visual_embeddings``) on the GPU.

Bit-exact against the reference's own output (golden fixture) and against the
oracle on larger plans: several feature keys interleaved, float32 / float16
sources converted to bf16, strided and 2-byte-aligned feature views (narrow
copy paths), final-only features, and the device-side index checks.
"""

from types import SimpleNamespace

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import ops
from nano_vllm_multimodal_b200.layers.visual_merge import (
    build_planned_visual_embeddings, merge_planned_visual_embeddings)
from tests._util import assert_bitexact

pytestmark = pytest.mark.gpu


def _plan(rows):
    return SimpleNamespace(replacements=tuple(SimpleNamespace(output_row=o, feature_key=k, feature_row=f)
                                              for o, k, f in rows))


def _bundle(final, deepstack):
    return SimpleNamespace(final_embedding=final, deepstack_embeddings=tuple(deepstack))


def test_golden_case(golden):
    c = golden["visual_merge_c3"]
    i = c["inputs"]
    keys = c["meta"]["keys"]
    feats = {keys[0]: _bundle(i["feature_a"][0].cuda(), i["feature_a"][1:].cuda().unbind(0)),
             keys[1]: _bundle(i["feature_b"][0].cuda(), i["feature_b"][1:].cuda().unbind(0))}
    plan = _plan([(o, keys[k], f) for o, k, f in i["plan"].tolist()])
    out = build_planned_visual_embeddings(i["tokens"].cuda(), plan, feats)
    assert_bitexact(out.final_embedding, c["outputs"]["final_embedding"], "merged")
    assert len(out.deepstack_embeddings) == 3
    assert_bitexact(torch.stack(out.deepstack_embeddings), c["outputs"]["deepstack"], "deepstack")
    assert out.visual_rows.tolist() == c["outputs"]["visual_rows"].tolist()
    assert out.visual_rows.dtype == torch.int64 and out.visual_rows.is_cuda


def _random_case(seed, device, tokens=3000, hidden=2048, layers=3):
    """Features built on `device` (CPU for the oracle, CUDA for the kernel) from the same
    seeded bytes; the float16 key's slices are taken on the device so that its rows keep
    a row stride of 2*hidden+1 elements (rows not 16-byte aligned)."""
    g = torch.Generator().manual_seed(seed)
    tok = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16).to(device)
    fa = torch.randn(layers + 1, 900, hidden, generator=g).to(torch.bfloat16).to(device)
    fb = torch.randn(layers + 1, 500, hidden, generator=g).to(device)
    wide = torch.randn(layers + 1, 400, 2 * hidden + 1, generator=g).to(torch.float16).to(device)
    fc = [wide[0, :, :hidden]] + [wide[1 + l, :, (1 if l == 1 else 0):(1 if l == 1 else 0) + hidden]
                                  for l in range(layers)]
    rows, out_row = [], 5
    for key, count, start in (("a", 600, 100), ("b", 300, 0), ("c", 350, 25), ("a", 200, 700)):
        for j in range(count):
            rows.append((out_row, key, start + j))
            out_row += 1 if j % 7 else 3
    assert out_row < tokens
    feats = {"a": (fa[0], tuple(fa[1:])), "b": (fb[0], tuple(fb[1:])), "c": (fc[0], tuple(fc[1:]))}
    return tok, rows, feats


def test_many_keys_mixed_dtypes_strided_and_unaligned_sources():
    tok_cpu, rows, feats_cpu = _random_case(1, "cpu")
    tok, _, feats_gpu = _random_case(1, "cuda")
    assert feats_gpu["c"][0].stride(0) == 2 * 2048 + 1 and feats_gpu["c"][1][1].data_ptr() % 16 == 2
    feats = {k: _bundle(f, ds) for k, (f, ds) in feats_gpu.items()}
    out = build_planned_visual_embeddings(tok, _plan(rows), feats)
    em, eds, erows = O.planned_visual_embeddings(tok_cpu, rows, feats_cpu)
    assert_bitexact(out.final_embedding, em, "merged")
    for l in range(3):
        assert_bitexact(out.deepstack_embeddings[l], eds[l], f"deepstack {l}")
    assert out.visual_rows.tolist() == erows.tolist()
    # merge_* returns only the merged embeddings; the inputs are not modified
    merged = merge_planned_visual_embeddings(tok, _plan(rows), feats)
    assert_bitexact(merged, em, "merge_planned_visual_embeddings")
    assert_bitexact(tok, tok_cpu, "token embeddings untouched")


def test_final_only_features_and_cpu_sources():
    g = torch.Generator().manual_seed(3)
    tok = torch.randn(64, 256, generator=g).to(torch.bfloat16)
    fa = torch.randn(10, 256, generator=g).to(torch.bfloat16)
    fb = torch.randn(6, 256, generator=g)  # float32 on the CPU: moved and converted
    rows = [(2, "a", 0), (3, "a", 1), (9, "b", 5), (10, "b", 4), (40, "a", 9)]
    out = build_planned_visual_embeddings(tok.cuda(), _plan(rows), {"a": fa.cuda(), "b": fb})
    em, eds, _ = O.planned_visual_embeddings(tok, rows, {"a": (fa, ()), "b": (fb, ())})
    assert out.deepstack_embeddings == () and eds == ()
    assert_bitexact(out.final_embedding, em, "final-only merge")


def test_device_index_checks(monkeypatch):
    """The kernel's own range checks (the host layer validates first, so drive the op
    directly): a source index past the table and a feature row past its source."""
    monkeypatch.setenv("NANOINFER_B200_VALIDATE", "1")
    tok = torch.randn(16, 64).to(torch.bfloat16).cuda()
    feat = torch.randn(4, 64).to(torch.bfloat16).cuda()
    table = torch.zeros(1, 20, dtype=torch.int64)
    table[0, 0], table[0, 1], table[0, 2], table[0, 3] = feat.data_ptr(), 64, 4, 2
    table = table.cuda()
    for bad in ([3, 5, 1, 0, 0, 9], [3, 5, 7, 0, 1, 0]):  # source 7 / feature row 9
        plan = torch.tensor(bad, dtype=torch.int64).cuda()
        with pytest.raises(ValueError, match="out of range"):
            ops.visual_merge(tok, table, 0, plan, 2)
    merged, _ = ops.visual_merge(tok, table, 0, torch.tensor([3, 5, 0, 0, 0, 3], dtype=torch.int64).cuda(), 2)
    assert_bitexact(merged[3], feat[0], "row 3")
    assert_bitexact(merged[5], feat[3], "row 5")
    assert_bitexact(merged[:3], tok[:3], "text rows")
