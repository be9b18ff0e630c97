"""Fused q/k norm + RoPE/M-RoPE + paged store vs the reference's composition.

The oracle runs the reference's stage order on the CPU (split views, per-head
norm rounded to the dtype, rotation, store of rotated k and raw v), with the
norm statistics in the kernels' fp32 summation order (``order="kernel"``; the
norm tests bound the difference to PyTorch's own order). With that, the fused
kernel is bit-exact: q, k, cache placement, untouched slots - for M-RoPE given
the kernel's own cos/sin (``test_gpu_rope.py`` bounds those against the CPU)."""

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import ops, workloads as W
from nano_vllm_multimodal_b200.layers.attention import attention_prologue
from nano_vllm_multimodal_b200.layers.layernorm import RMSNorm
from nano_vllm_multimodal_b200.layers.multimodal_rotary_embedding import MultimodalRotaryEmbedding
from nano_vllm_multimodal_b200.layers.qwen3_vl import Qwen3VLTextRMSNorm
from nano_vllm_multimodal_b200.layers.rotary_embedding import RotaryEmbedding
from tests._util import assert_bitexact, assert_ulp

pytestmark = pytest.mark.gpu


def _golden_case(golden, name):
    c = golden[name]
    i, m = c["inputs"], c["meta"]
    nq, nkv = m["heads"]
    qkv = i["qkv"].cuda()
    q, k, v = qkv.split([nq * 128, nkv * 128, nkv * 128], -1)
    q, k, v = q.view(-1, nq, 128), k.view(-1, nkv, 128), v.view(-1, nkv, 128)
    kc = torch.full(m["cache_shape"], m["cache_fill"], dtype=torch.bfloat16, device="cuda")
    vc = kc.clone()
    if m["rope"] == "table":
        rope = dict(rope_mode=ops.ROPE_TABLE, cos_sin_cache=O.rope_cos_sin_cache(128, m["max_position"], m["base"]).cuda())
    else:
        mode = ops.ROPE_MROPE_INTERLEAVED if m["rope"] == "interleaved" else ops.ROPE_MROPE_CHUNKED
        rope = dict(rope_mode=mode, inv_freq=O.mrope_inv_freq(128, m["base"]).cuda(), sections=m["sections"])
    norm = {}
    if m["norm"]:
        norm = dict(q_weight=i["q_weight"].cuda(), k_weight=i["k_weight"].cuda(), eps=m["eps"])
    aq, ak = ops.qk_prologue(q, k, v=v, positions=i["positions"].cuda(), **norm, **rope,
                             key_cache=kc, value_cache=vc, slot_mapping=i["slot_mapping"].cuda())
    return c, aq, ak, kc, vc


@pytest.mark.parametrize("name", ["fused_qwen3_c1", "fused_qwen3vl_c3", "fused_qwen25vl_c4"])
def test_golden_fused_prologue(golden, name):
    c, aq, ak, kc, vc = _golden_case(golden, name)
    exact = c["meta"]["rope"] == "table"
    check = assert_bitexact if exact else (lambda a, e, w: assert_ulp(a, e, 1, w))
    check(aq, c["outputs"]["q"], "q")
    check(ak, c["outputs"]["k"], "k")
    # cache: V rows bit-exact, untouched slots keep -3, K rows follow k
    assert_bitexact(vc, c["outputs"]["value_cache"], "value cache")
    ref_k = c["outputs"]["key_cache"]
    untouched = (ref_k == -3).all(dim=-1).all(dim=-1)
    assert torch.equal((kc.cpu() == -3).all(dim=-1).all(dim=-1), untouched)
    check(kc, ref_k, "key cache")


def _oracle_case(config, tokens, norm, rope_kind, variant=0):
    d = W.make_layer_inputs(config, tokens=tokens)
    shp = d["shape"]
    if rope_kind == "table":
        table = O.rope_cos_sin_cache(128, shp.max_position, shp.theta)
        rope_o = ("table", table)
        rope_g = dict(rope_mode=ops.ROPE_TABLE, cos_sin_cache=table.cuda())
    else:
        inv = O.mrope_inv_freq(128, shp.theta)
        rope_o = ("mrope", inv, shp.sections, rope_kind)
        mode = ops.ROPE_MROPE_INTERLEAVED if rope_kind == "interleaved" else ops.ROPE_MROPE_CHUNKED
        rope_g = dict(rope_mode=mode, inv_freq=inv.cuda(), sections=shp.sections)
    nq, nkv = shp.num_heads, shp.num_kv_heads
    qkv = d["qkv"].cuda()
    q, k, v = qkv.split([nq * 128, nkv * 128, nkv * 128], -1)
    q, k, v = q.view(-1, nq, 128), k.view(-1, nkv, 128), v.view(-1, nkv, 128)
    kc, vc = d["key_cache"].cuda(), d["value_cache"].cuda()
    normg = dict(q_weight=d["q_weight"].cuda(), k_weight=d["k_weight"].cuda(), eps=1e-6) if norm else {}
    aq, ak = ops.qk_prologue(q, k, v=v, positions=d["positions"].cuda(), **normg, **rope_g,
                             key_cache=kc, value_cache=vc, slot_mapping=d["slot_mapping"].cuda(),
                             variant=variant)
    return d, (aq, ak, kc, vc), rope_o, rope_g


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("config,norm,rope_kind", [
    (1, "rms", "table"), (2, "rms", "table"), (3, "text", "interleaved"), (4, None, "chunked")])
def test_fused_matches_composition(config, norm, rope_kind, variant):
    """Both kernel variants (register-staged and bulk-copy pipelined)."""
    tokens = {1: 512, 2: 256, 3: 2048, 4: 8312}[config]
    d, (aq, ak, kc, vc), rope_o, rope_g = _oracle_case(config, tokens, norm, rope_kind, variant)
    shp = d["shape"]
    if rope_kind == "table":
        eq, ek, ekc, evc = O.qk_norm_rope_store(
            d["qkv"], shp.num_heads, shp.num_kv_heads, 128, positions=d["positions"], rope=rope_o,
            q_weight=d["q_weight"], k_weight=d["k_weight"], eps=1e-6, norm=norm,
            key_cache=d["key_cache"], value_cache=d["value_cache"], slot_mapping=d["slot_mapping"],
            order="kernel")
        assert_bitexact(aq, eq, "q")
        assert_bitexact(ak, ek, "k")
        assert_bitexact(kc, ekc, "key cache")
    else:
        # numerics given the kernel's own cos/sin (see test_gpu_rope.py for the trig bound)
        nq, nkv = shp.num_heads, shp.num_kv_heads
        q, k, v = d["qkv"].split([nq * 128, nkv * 128, nkv * 128], -1)
        q, k, v = q.reshape(-1, nq, 128), k.reshape(-1, nkv, 128), v.reshape(-1, nkv, 128)
        if norm == "text":
            q = O.text_rms_norm(q, d["q_weight"], 1e-6, order="kernel")
            k = O.text_rms_norm(k, d["k_weight"], 1e-6, order="kernel")
        gc, gs = ops.mrope_cos_sin(d["positions"].cuda(), rope_g["inv_freq"], torch.bfloat16)
        eq, ek = O.apply_mrope(q, k, gc.cpu(), gs.cpu(), shp.sections, rope_kind)
        assert_bitexact(aq, eq, "q")
        assert_bitexact(ak, ek, "k")
        ekc, evc = O.paged_store(ek, v, d["key_cache"], d["value_cache"], d["slot_mapping"])
        assert_bitexact(kc, ekc, "key cache")
    nkv = shp.num_kv_heads
    v_rows = d["qkv"][:, (shp.num_heads + nkv) * 128:].reshape(-1, nkv, 128)
    _, evc = O.paged_store(v_rows, v_rows, d["key_cache"], d["value_cache"], d["slot_mapping"])
    assert_bitexact(vc, evc, "value cache (raw v, untouched slots keep -3)")


@pytest.mark.parametrize("head_dim", [64, 256])
def test_fused_other_head_dims(head_dim):
    g = torch.Generator().manual_seed(head_dim)
    T, nq, nkv = 37, 4, 2
    qkv = torch.randn(T, (nq + 2 * nkv) * head_dim, generator=g).to(torch.bfloat16)
    pos = torch.randint(0, 4096, (T,), generator=g)
    slots = torch.randperm(64, generator=g)[:T].to(torch.int32)
    slots[::5] = -1
    w = (1 + 0.1 * torch.randn(head_dim, generator=g)).to(torch.bfloat16)
    table = O.rope_cos_sin_cache(head_dim, 4096, 1e6)
    kc = torch.full((4, 16, nkv, head_dim), -3.0, dtype=torch.bfloat16)
    eq, ek, ekc, evc = O.qk_norm_rope_store(qkv, nq, nkv, head_dim, positions=pos, rope=("table", table),
                                            q_weight=w, k_weight=w, eps=1e-6, norm="rms",
                                            key_cache=kc, value_cache=kc.clone(), slot_mapping=slots,
                                            order="kernel")
    gq = qkv.cuda()
    q, k, v = gq.split([nq * head_dim, nkv * head_dim, nkv * head_dim], -1)
    q, k, v = q.view(T, nq, head_dim), k.view(T, nkv, head_dim), v.view(T, nkv, head_dim)
    gkc, gvc = kc.cuda(), kc.clone().cuda()
    aq, ak = ops.qk_prologue(q, k, v=v, positions=pos.cuda(), q_weight=w.cuda(), k_weight=w.cuda(), eps=1e-6,
                             rope_mode=ops.ROPE_TABLE, cos_sin_cache=table.cuda(), key_cache=gkc,
                             value_cache=gvc, slot_mapping=slots.cuda())
    assert_bitexact(aq, eq, "q")
    assert_bitexact(ak, ek, "k")
    assert_bitexact(gkc, ekc, "kc")
    assert_bitexact(gvc, evc, "vc")


def test_attention_prologue_with_modules_all_models():
    """The layer-level helper with real modules (ours), per model family."""
    for config in (1, 3, 4):
        d = W.make_layer_inputs(config, tokens=300)
        shp = d["shape"]
        if shp.rope == "table":
            rope = RotaryEmbedding(128, 128, shp.max_position, shp.theta).cuda()
        else:
            rope = MultimodalRotaryEmbedding(head_dim=128, base=shp.theta, sections=shp.sections,
                                             strategy=shp.rope).cuda()
        qn = kn = None
        if shp.qk_norm == "rms":
            qn, kn = RMSNorm(128).to(torch.bfloat16).cuda(), RMSNorm(128).to(torch.bfloat16).cuda()
        elif shp.qk_norm == "text":
            qn, kn = Qwen3VLTextRMSNorm(128).to(torch.bfloat16).cuda(), Qwen3VLTextRMSNorm(128).to(torch.bfloat16).cuda()
        if qn is not None:
            with torch.no_grad():
                qn.weight.copy_(d["q_weight"])
                kn.weight.copy_(d["k_weight"])
        kc, vc = d["key_cache"].cuda(), d["value_cache"].cuda()
        qkv = d["qkv"].cuda()
        q, k, v = attention_prologue(qkv, num_heads=shp.num_heads, num_kv_heads=shp.num_kv_heads, head_dim=128,
                                     positions=d["positions"].cuda(), rotary_emb=rope, q_norm=qn, k_norm=kn,
                                     k_cache=kc, v_cache=vc, slot_mapping=d["slot_mapping"].cuda())
        # unfused path through the same modules must agree exactly
        q2, k2, v2 = qkv.split([shp.num_heads * 128, shp.num_kv_heads * 128, shp.num_kv_heads * 128], -1)
        q2, k2 = q2.view(-1, shp.num_heads, 128), k2.view(-1, shp.num_kv_heads, 128)
        if qn is not None:
            q2, k2 = qn(q2), kn(k2)
        q2, k2 = rope(d["positions"].cuda(), q2, k2)
        assert_bitexact(q, q2, f"C{config} q")
        assert_bitexact(k, k2, f"C{config} k")
        kc2, vc2 = d["key_cache"].cuda(), d["value_cache"].cuda()
        ops.paged_store(k2, v2.view(-1, shp.num_kv_heads, 128), kc2, vc2, d["slot_mapping"].cuda())
        assert_bitexact(kc, kc2, f"C{config} key cache")
        assert_bitexact(vc, vc2, f"C{config} value cache")


def test_prologue_skips_minus_one_and_flags_bad_slots(monkeypatch):
    monkeypatch.setenv("NANOINFER_B200_VALIDATE", "1")
    d = W.make_layer_inputs(1, tokens=64)
    qkv = d["qkv"].cuda()
    q, k, v = qkv.split([2048, 1024, 1024], -1)
    q, k, v = q.view(-1, 16, 128), k.view(-1, 8, 128), v.view(-1, 8, 128)
    table = O.rope_cos_sin_cache(128, 40960, 1e6).cuda()
    slots = d["slot_mapping"].clone()
    slots[:] = -1
    kc, vc = d["key_cache"].cuda(), d["value_cache"].cuda()
    ops.qk_prologue(q, k, v=v, positions=d["positions"].cuda(), rope_mode=ops.ROPE_TABLE, cos_sin_cache=table,
                    key_cache=kc, value_cache=vc, slot_mapping=slots.cuda())
    assert bool((kc == -3).all()) and bool((vc == -3).all())
    slots[3] = kc.shape[0] * kc.shape[1]  # one past the end: skipped and reported
    with pytest.raises(ValueError, match="slot_mapping contains a slot outside"):
        ops.qk_prologue(q, k, v=v, positions=d["positions"].cuda(), rope_mode=ops.ROPE_TABLE,
                        cos_sin_cache=table, key_cache=kc, value_cache=vc, slot_mapping=slots.cuda())
    assert bool((kc == -3).all()) and bool((vc == -3).all())


@pytest.mark.parametrize("head_dim,heads", [(64, (8, 4)), (128, (16, 8)), (128, (16, 2)), (256, (4, 2))])
@pytest.mark.parametrize("mode", ["table", "chunked", "interleaved", "none"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_pipelined_variant_bit_identical_to_register_variant(head_dim, heads, mode, dtype):
    """Same inputs through variant 1 and variant 2: every output and both caches identical,
    with and without norm / store, on a token count that is not a multiple of anything."""
    nq, nkv = heads
    T = 3001
    g = torch.Generator().manual_seed(head_dim + nq)
    qkv = torch.randn(T, (nq + 2 * nkv) * head_dim, generator=g).to(dtype).cuda()
    q, k, v = qkv.split([nq * head_dim, nkv * head_dim, nkv * head_dim], -1)
    q, k, v = q.view(T, nq, head_dim), k.view(T, nkv, head_dim), v.view(T, nkv, head_dim)
    slots = torch.randperm(64 * 64, generator=g)[:T].to(torch.int32)
    slots[::7] = -1
    w = (1 + 0.1 * torch.randn(head_dim, generator=g)).to(dtype).cuda()
    if mode == "table":
        rope = dict(rope_mode=ops.ROPE_TABLE, cos_sin_cache=O.rope_cos_sin_cache(head_dim, 8192, 1e6).cuda(),
                    positions=torch.randint(0, 8192, (T,), generator=g).cuda())
    elif mode == "none":
        rope = dict(rope_mode=ops.ROPE_NONE)
    else:
        half = head_dim // 2
        sec = (half - 2 * (half * 5 // 16), half * 5 // 16, half * 5 // 16)
        m = ops.ROPE_MROPE_INTERLEAVED if mode == "interleaved" else ops.ROPE_MROPE_CHUNKED
        rope = dict(rope_mode=m, inv_freq=O.mrope_inv_freq(head_dim, 5e6).cuda(), sections=sec,
                    positions=torch.randint(0, 32768, (3, T), generator=g).cuda())
    for norm in (True, False):
        for store in (True, False):
            outs = []
            for variant in (1, 2):
                kc = torch.full((64, 64, nkv, head_dim), -3.0, dtype=dtype, device="cuda")
                vc = kc.clone()
                extra = dict(v=v, key_cache=kc, value_cache=vc, slot_mapping=slots.cuda()) if store else {}
                nrm = dict(q_weight=w, k_weight=w, eps=1e-6) if norm else {}
                aq, ak = ops.qk_prologue(q, k, **rope, **nrm, **extra, variant=variant)
                outs.append((aq, ak, kc, vc))
            for a, b, name in zip(outs[0], outs[1], ("q", "k", "key cache", "value cache")):
                assert_bitexact(b, a, f"{name} norm={norm} store={store}")


@pytest.mark.parametrize("variant", [1, 2])
def test_fused_fp32_norm_weights(variant):
    """Qwen3 RMSNorm with float32 weights on bf16 activations (``x.to(dtype).mul_(weight)``
    keeps the activation dtype: n = bf16(x * rs), y = bf16(n * w)), 1-D RoPE and the paged
    store, through both kernels (the pipelined one then takes its 8-warp x 3-stage layout),
    bit-exact against the oracle composition in the kernels' summation order."""
    T = 3000
    d = W.make_layer_inputs(1, tokens=T)
    shp = d["shape"]
    nq, nkv = shp.num_heads, shp.num_kv_heads
    qw, kw = d["q_weight"].float(), d["k_weight"].float()
    table = O.rope_cos_sin_cache(128, shp.max_position, shp.theta)
    qkv = d["qkv"].cuda()
    q, k, v = qkv.split([nq * 128, nkv * 128, nkv * 128], -1)
    kc, vc = d["key_cache"].cuda(), d["value_cache"].cuda()
    aq, ak = ops.qk_prologue(q.view(-1, nq, 128), k.view(-1, nkv, 128), v=v.view(-1, nkv, 128),
                             positions=d["positions"].cuda(), q_weight=qw.cuda(), k_weight=kw.cuda(), eps=1e-6,
                             rope_mode=ops.ROPE_TABLE, cos_sin_cache=table.cuda(), key_cache=kc, value_cache=vc,
                             slot_mapping=d["slot_mapping"].cuda(), variant=variant)
    eq, ek, ekc, evc = O.qk_norm_rope_store(
        d["qkv"], nq, nkv, 128, positions=d["positions"], rope=("table", table), q_weight=qw, k_weight=kw,
        eps=1e-6, norm="rms", key_cache=d["key_cache"], value_cache=d["value_cache"],
        slot_mapping=d["slot_mapping"], order="kernel")
    assert_bitexact(aq, eq, "q")
    assert_bitexact(ak, ek, "k")
    assert_bitexact(kc, ekc, "key cache")
    assert_bitexact(vc, evc, "value cache")


def test_pipelined_variant_rejects_split_layouts():
    T = 64
    q = torch.randn(T, 16, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.randn(T, 8, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="pipelined variant"):
        ops.qk_prologue(q, k, rope_mode=ops.ROPE_NONE, variant=2)
    aq, ak = ops.qk_prologue(q, k, rope_mode=ops.ROPE_NONE, variant=0)  # auto: register kernel
    assert torch.equal(aq, q) and torch.equal(ak, k)


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("config,tokens,rope_kind", [(2, 256, "table"), (3, 4096, "interleaved"),
                                                     (4, 2048, "chunked")])
def test_cache_only_k_matches_the_full_prologue(variant, config, tokens, rope_kind):
    """``emit_k=False`` (decode / chunked prefill, which read k from the cache):
    the same rotated q and the same cache bytes as with the contiguous k written,
    in both kernel variants; no k comes back."""
    d = W.make_layer_inputs(config, tokens=tokens)
    shp = d["shape"]
    nq, nkv = shp.num_heads, shp.num_kv_heads
    qkv = d["qkv"].cuda()
    q, k, v = qkv.split([nq * 128, nkv * 128, nkv * 128], -1)
    q, k, v = q.view(-1, nq, 128), k.view(-1, nkv, 128), v.view(-1, nkv, 128)
    if rope_kind == "table":
        rope = dict(rope_mode=ops.ROPE_TABLE,
                    cos_sin_cache=O.rope_cos_sin_cache(128, shp.max_position, shp.theta).cuda())
    else:
        mode = ops.ROPE_MROPE_INTERLEAVED if rope_kind == "interleaved" else ops.ROPE_MROPE_CHUNKED
        rope = dict(rope_mode=mode, inv_freq=O.mrope_inv_freq(128, shp.theta).cuda(), sections=shp.sections)
    norm = dict(q_weight=d["q_weight"].cuda(), k_weight=d["k_weight"].cuda(), eps=1e-6) if shp.qk_norm else {}
    outs = []
    for emit_k in (True, False):
        kc, vc = d["key_cache"].cuda(), d["value_cache"].cuda()
        q_rot, k_rot = ops.qk_prologue(q, k, v=v, positions=d["positions"].cuda(), **norm, **rope,
                                       key_cache=kc, value_cache=vc, slot_mapping=d["slot_mapping"].cuda(),
                                       variant=variant, emit_k=emit_k)
        outs.append((q_rot, k_rot, kc, vc))
    (q1, k1, kc1, vc1), (q2, k2, kc2, vc2) = outs
    assert k2 is None and k1 is not None
    assert_bitexact(q2, q1.cpu(), "q")
    assert_bitexact(kc2, kc1.cpu(), "key cache")
    assert_bitexact(vc2, vc1.cpu(), "value cache")


def test_cache_only_k_needs_the_caches():
    q = torch.zeros(4, 2, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(4, 1, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="emit_k=False needs the caches"):
        ops.qk_prologue(q, k, emit_k=False)
