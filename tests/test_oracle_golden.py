"""Pin the CPU oracle: bit-exact against fixtures made by the reference's own
modules (``tests/golden/make_golden.py``) and against the known-answer
vectors of the reference's test-suite."""

import hashlib

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import workloads as W


def _eq(a, b):
    assert a.dtype == b.dtype and a.shape == b.shape, (a.dtype, b.dtype, a.shape, b.shape)
    assert torch.equal(a, b)


def _split(qkv, heads):
    nq, nkv = heads
    D = 128
    q, k, v = qkv.split([nq * D, nkv * D, nkv * D], dim=-1)
    return q.view(-1, nq, D), k.view(-1, nkv, D), v.view(-1, nkv, D)


def test_rmsnorm_add(golden):
    c = golden["rmsnorm_add_c1"]
    y, r = O.add_rms_norm(c["inputs"]["x"], c["inputs"]["residual"], c["inputs"]["weight"], 1e-6)
    _eq(y, c["outputs"]["y"])
    _eq(r, c["outputs"]["residual"])


def test_rmsnorm(golden):
    c = golden["rmsnorm_c1"]
    _eq(O.rms_norm(c["inputs"]["x"], c["inputs"]["weight"], 1e-6), c["outputs"]["y"])


def test_qk_norm_on_strided_views(golden):
    c = golden["qknorm_c1"]
    q, k, _ = _split(c["inputs"]["qkv"], (16, 8))
    _eq(O.rms_norm(q, c["inputs"]["q_weight"], 1e-6), c["outputs"]["q"])
    _eq(O.rms_norm(k, c["inputs"]["k_weight"], 1e-6), c["outputs"]["k"])


def test_silu_and_mul(golden):
    c = golden["silu_c1"]
    _eq(O.silu_and_mul(c["inputs"]["x"]), c["outputs"]["y"])


def test_rope_table_and_rotation(golden):
    c = golden["rope_c1"]
    table = O.rope_cos_sin_cache(128, 40960, 1e6)
    assert hashlib.sha256(table.numpy().tobytes()).hexdigest() == c["meta"]["table_sha256"]
    _eq(table[c["inputs"]["positions"]], c["outputs"]["table_rows"])
    q, k = O.apply_rope(c["inputs"]["positions"], c["inputs"]["q"], c["inputs"]["k"], table)
    _eq(q, c["outputs"]["q"])
    _eq(k, c["outputs"]["k"])


def test_text_rms_norm(golden):
    c = golden["textnorm_c3"]
    i = c["inputs"]
    _eq(O.text_rms_norm(i["x"], i["weight"], 1e-6), c["outputs"]["y"])
    y, s = O.add_text_rms_norm(i["x"], i["residual"], i["weight"], 1e-6)
    _eq(y, c["outputs"]["y_add"])
    _eq(s, c["outputs"]["sum"])


@pytest.mark.parametrize("name", ["mrope_interleaved_c3", "mrope_chunked_c4"])
def test_mrope(golden, name):
    c = golden[name]
    m = c["meta"]
    inv = O.mrope_inv_freq(128, m["base"])
    _eq(inv, c["outputs"]["inv_freq"])
    q, k = O.mrope_forward(c["inputs"]["positions"], c["inputs"]["q"], c["inputs"]["k"], inv,
                           m["sections"], m["strategy"])
    _eq(q, c["outputs"]["q"])
    _eq(k, c["outputs"]["k"])
    if "cos" in c["outputs"]:
        cos, sin = O.mrope_cos_sin(c["inputs"]["positions"], inv, torch.bfloat16)
        _eq(cos, c["outputs"]["cos"])
        _eq(sin, c["outputs"]["sin"])


def test_paged_store_and_gather(golden):
    c = golden["paged_c2"]
    _, k, v = _split(c["inputs"]["qkv"], (16, 8))
    kc = torch.full(c["meta"]["cache_shape"], c["meta"]["cache_fill"], dtype=torch.bfloat16)
    kc2, vc2 = O.paged_store(k, v, kc, kc.clone(), c["inputs"]["slot_mapping"])
    _eq(kc2, c["outputs"]["key_cache"])
    _eq(vc2, c["outputs"]["value_cache"])
    g = O.paged_gather(kc2, c["inputs"]["block_table"], c["meta"]["sequence_length"])
    _eq(g, c["outputs"]["gathered"])


def test_embedding(golden):
    c = golden["embedding_c2"]
    _eq(O.embedding(c["inputs"]["ids"], c["inputs"]["weight"]), c["outputs"]["y"])


def test_deepstack(golden):
    c = golden["deepstack_c3"]
    i = c["inputs"]
    _eq(O.add_deepstack_rows(i["hidden"], i["rows"], i["vis"]), c["outputs"]["y"])


def test_decode_attention(golden):
    """The float64 oracle against the reference's SDPA decode branch (CPU, bf16). That path
    rounds intermediates in bf16, so the pin is a tolerance: |oracle - reference| <=
    2^-6 * max(1, |reference|), and most elements agree exactly."""
    c = golden["decode_attention_c2"]
    i = c["inputs"]
    o = O.paged_decode_attention(i["q"], i["k_cache"], i["v_cache"], i["context_lens"],
                                 i["block_tables"], c["meta"]["scale"]).double()
    ref = c["outputs"]["out"].double()
    assert o.shape == ref.shape
    assert bool(((o - ref).abs() <= 2.0 ** -6 * ref.abs().clamp(min=1.0)).all())
    assert float((o == ref).double().mean()) > 0.6
    assert torch.equal(o[0], ref[0])  # one-token context: softmax weight 1, exact


def _visual_case(golden):
    c = golden["visual_merge_c3"]
    i = c["inputs"]
    keys = c["meta"]["keys"]
    feats = {keys[0]: (i["feature_a"][0], tuple(i["feature_a"][1:])),
             keys[1]: (i["feature_b"][0], tuple(i["feature_b"][1:]))}
    reps = [(int(o), keys[int(k)], int(f)) for o, k, f in i["plan"].tolist()]
    return c, reps, feats


def test_visual_merge(golden):
    """build_planned_visual_embeddings golden (reference run): merged rows with a float32
    source converted to bf16, three DeepStack payloads in plan order, visual rows."""
    c, reps, feats = _visual_case(golden)
    merged, payloads, rows = O.planned_visual_embeddings(c["inputs"]["tokens"], reps, feats)
    assert torch.equal(merged.view(torch.int16), c["outputs"]["final_embedding"].view(torch.int16))
    assert torch.equal(torch.stack(payloads).view(torch.int16), c["outputs"]["deepstack"].view(torch.int16))
    assert torch.equal(rows, c["outputs"]["visual_rows"])


@pytest.mark.parametrize("name", ["fused_qwen3_c1", "fused_qwen3vl_c3", "fused_qwen25vl_c4"])
def test_fused_prologue(golden, name):
    c = golden[name]
    i, m = c["inputs"], c["meta"]
    if m["rope"] == "table":
        rope = ("table", O.rope_cos_sin_cache(128, m["max_position"], m["base"]))
    else:
        rope = ("mrope", O.mrope_inv_freq(128, m["base"]), m["sections"], m["rope"])
    kc = torch.full(m["cache_shape"], m["cache_fill"], dtype=torch.bfloat16)
    q, k, kc2, vc2 = O.qk_norm_rope_store(
        i["qkv"], *m["heads"], 128, positions=i["positions"], rope=rope,
        q_weight=i["q_weight"], k_weight=i["k_weight"], eps=m["eps"], norm=m["norm"],
        key_cache=kc, value_cache=kc.clone(), slot_mapping=i["slot_mapping"])
    _eq(q, c["outputs"]["q"])
    _eq(k, c["outputs"]["k"])
    _eq(kc2, c["outputs"]["key_cache"])
    _eq(vc2, c["outputs"]["value_cache"])


# ---- known-answer vectors from the reference's own test-suite -------------------------


def test_interleaved_fixed_golden_output():
    """Values of ``tests/test_qwen3_vl_runtime.py:178-217`` (sections (2,1,1), D=8)."""
    q = torch.tensor([[[1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0]]])
    k = torch.tensor([[[8.0, 7.0, 6.0, 5.0, 4.0, 3.0, 2.0, 1.0]]])
    cos = torch.tensor([[[1.0, 101.0, 102.0, 4.0, 1.0, 101.0, 102.0, 4.0]],
                        [[201.0, 2.0, 203.0, 204.0, 201.0, 2.0, 203.0, 204.0]],
                        [[301.0, 302.0, 3.0, 304.0, 301.0, 302.0, 3.0, 304.0]]])
    sin = torch.tensor([[[10.0, 1001.0, 1002.0, 40.0, 10.0, 1001.0, 1002.0, 40.0]],
                        [[2001.0, 20.0, 2003.0, 2004.0, 2001.0, 20.0, 2003.0, 2004.0]],
                        [[3001.0, 3002.0, 30.0, 3004.0, 3001.0, 3002.0, 30.0, 3004.0]]])
    aq, ak = O.apply_mrope(q, k, cos, sin, (2, 1, 1), "interleaved")
    torch.testing.assert_close(aq, torch.tensor([[[-49.0, -116.0, -201.0, -304.0, 15.0, 52.0, 111.0, 192.0]]]))
    torch.testing.assert_close(ak, torch.tensor([[[-32.0, -46.0, -42.0, -20.0, 84.0, 146.0, 186.0, 204.0]]]))


def test_interleaved_matches_independent_fp32_rederivation():
    """``tests/test_qwen3_vl_runtime.py:41-62,219-251``: frequency layout re-derived."""
    torch.manual_seed(17)
    sections = (24, 20, 20)
    positions = torch.tensor(((0, 1, 4, 7), (0, 2, 5, 8), (0, 3, 6, 9)))
    q = torch.randn(4, 2, 128)
    k = torch.randn(4, 1, 128)
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    f = positions.float().unsqueeze(-1) * inv.view(1, 1, -1)
    sel = f[0].clone()
    for axis, off in ((1, 1), (2, 2)):
        sel[..., off:sections[axis] * 3:3] = f[axis, ..., off:sections[axis] * 3:3]
    emb = torch.cat((sel, sel), -1)
    c, s = emb.cos().unsqueeze(1), emb.sin().unsqueeze(1)

    def rot(x):
        return torch.cat((-x[..., 64:], x[..., :64]), -1)

    aq, ak = O.mrope_forward(positions, q, k, O.mrope_inv_freq(128, 1e6), sections, "interleaved")
    torch.testing.assert_close(aq, q * c + rot(q) * s)
    torch.testing.assert_close(ak, k * c + rot(k) * s)


def test_store_kat_skips_minus_one():
    """``tests/test_paged_kv_backends.py:17-23,127-137``."""
    key = torch.arange(3 * 2 * 4, dtype=torch.float32).reshape(3, 2, 4)
    value = key + 100
    kc = torch.full((3, 4, 2, 4), -1.0)
    slots = torch.tensor([0, 5, -1], dtype=torch.int32)
    k2, v2 = O.paged_store(key, value, kc, kc.clone(), slots)
    assert torch.equal(k2.flatten(0, 1)[0], key[0])
    assert torch.equal(k2.flatten(0, 1)[5], key[1])
    assert torch.equal(v2.flatten(0, 1)[5], value[1])
    assert torch.all(k2.flatten(0, 1)[1] == -1)
    assert int((k2 != -1).sum()) == 2 * 8


def test_gather_kat_nonsequential_blocks():
    """``tests/test_paged_kv_backends.py:139-147``."""
    cache = torch.arange(3 * 4 * 2 * 4, dtype=torch.float32).reshape(3, 4, 2, 4)
    table = torch.tensor([2, 0], dtype=torch.int32)
    assert torch.equal(O.paged_gather(cache, table, 6), torch.cat((cache[2], cache[0]), 0)[:6])
    assert O.paged_gather(cache, table, 0).shape == (0, 2, 4)


def test_text_norm_formula_exact_bf16():
    """``tests/test_qwen3_vl_model.py:155-171``."""
    torch.manual_seed(43)
    x = torch.randn(8, 2048, dtype=torch.bfloat16)
    w = torch.randn(2048, dtype=torch.bfloat16)
    n = x.float()
    n = n * torch.rsqrt(n.pow(2).mean(-1, keepdim=True) + 1e-6)
    assert torch.equal(O.text_rms_norm(x, w, 1e-6), w * n.to(torch.bfloat16))


def test_deepstack_empty_rows_returns_same_object():
    """``tests/test_qwen3_vl_model.py:608-617``."""
    h = torch.randn(3, 16)
    assert O.add_deepstack_rows(h, torch.empty(0, dtype=torch.long), torch.empty(0, 16)) is h


def test_workload_positions_rule():
    """Static-image positions (``tests/test_qwen3_vl_runtime.py:66-87`` example)."""
    pos, rows = W.image_positions([("text", 1), ("image", 1, 2, 2), ("text", 1),
                                   ("image", 1, 1, 2), ("text", 1)])
    expected = ((0, 1, 1, 1, 1, 3, 4, 4, 6), (0, 1, 1, 2, 2, 3, 4, 4, 6), (0, 1, 2, 1, 2, 3, 4, 5, 6))
    assert tuple(tuple(a) for a in pos.tolist()) == expected
    assert rows == [1, 2, 3, 4, 6, 7]
