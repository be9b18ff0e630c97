"""Zero-size inputs: every op and layer module returns correctly shaped empty
outputs and touches nothing, as the reference's PyTorch ops do for an empty
batch (a scheduler step can carry no prefill or no decode tokens)."""

import pytest
import torch

import oracle as O
from nano_vllm_multimodal_b200 import ops
from nano_vllm_multimodal_b200.layers.activation import SiluAndMul
from nano_vllm_multimodal_b200.layers.attention import store_kvcache
from nano_vllm_multimodal_b200.layers.layernorm import RMSNorm
from nano_vllm_multimodal_b200.layers.multimodal_rotary_embedding import MultimodalRotaryEmbedding
from nano_vllm_multimodal_b200.layers.qwen3_vl import Qwen3VLTextRMSNorm
from nano_vllm_multimodal_b200.layers.rotary_embedding import RotaryEmbedding

pytestmark = pytest.mark.gpu

BF = torch.bfloat16
H, NQ, NKV, D = 1024, 16, 8, 128


def _e(*shape, dtype=BF):
    return torch.empty(*shape, dtype=dtype, device="cuda")


def test_elementwise_ops_on_empty_batches():
    w = torch.ones(H, dtype=BF, device="cuda")
    y, r = ops.add_rms_norm(_e(0, H), _e(0, H), w, 1e-6)
    assert y.shape == (0, H) and r.shape == (0, H)
    y, r = ops.add_rms_norm(_e(0, H), _e(0, H), w, 1e-6, True)
    assert y.shape == (0, H) and r.shape == (0, H)
    assert ops.silu_and_mul(_e(0, 2 * 3072)).shape == (0, 3072)
    assert ops.embedding(_e(0, dtype=torch.int64), torch.zeros(100, H, dtype=BF, device="cuda")).shape == (0, H)
    cos, sin = ops.mrope_cos_sin(_e(3, 0, dtype=torch.int64), O.mrope_inv_freq(D, 5e6).cuda(), BF)
    assert cos.shape == (3, 0, D) and sin.shape == (3, 0, D)
    assert ops.mrope_apply(_e(0, NQ, D), cos, sin, (24, 20, 20), True).shape == (0, NQ, D)


@pytest.mark.parametrize("variant", [0, 1, 2])
def test_prologue_on_an_empty_batch_leaves_the_cache_untouched(variant):
    qkv = _e(0, (NQ + 2 * NKV) * D)
    q, k, v = qkv.split([NQ * D, NKV * D, NKV * D], -1)
    q, k, v = q.view(0, NQ, D), k.view(0, NKV, D), v.view(0, NKV, D)
    kc = torch.full((4, 256, NKV, D), -3.0, dtype=BF, device="cuda")
    vc = kc.clone()
    w = torch.ones(D, dtype=BF, device="cuda")
    table = O.rope_cos_sin_cache(D, 1024, 1e6).cuda()
    aq, ak = ops.qk_prologue(q, k, v=v, positions=_e(0, dtype=torch.int64), q_weight=w, k_weight=w, eps=1e-6,
                             rope_mode=ops.ROPE_TABLE, cos_sin_cache=table, key_cache=kc, value_cache=vc,
                             slot_mapping=_e(0, dtype=torch.int32), variant=variant)
    assert aq.shape == (0, NQ, D) and ak.shape == (0, NKV, D)
    assert bool((kc == -3).all()) and bool((vc == -3).all())


def test_layer_modules_on_empty_batches():
    norm = RMSNorm(H).cuda().to(BF)
    assert norm(_e(0, H)).shape == (0, H)
    y, r = norm(_e(0, H), _e(0, H))
    assert y.shape == (0, H) and r.shape == (0, H)
    tnorm = Qwen3VLTextRMSNorm(D).cuda().to(BF)
    assert tnorm(_e(0, NQ, D)).shape == (0, NQ, D)
    assert SiluAndMul()(_e(0, 2 * 3072)).shape == (0, 3072)
    rope = RotaryEmbedding(D, D, 1024, 1e6).cuda()
    aq, ak = rope(_e(0, dtype=torch.int64), _e(0, NQ, D), _e(0, NKV, D))
    assert aq.shape == (0, NQ, D) and ak.shape == (0, NKV, D)
    mrope = MultimodalRotaryEmbedding(head_dim=D, base=5e6, sections=(24, 20, 20), strategy="interleaved").cuda()
    aq, ak = mrope(_e(3, 0, dtype=torch.int64), _e(0, NQ, D), _e(0, NKV, D))
    assert aq.shape == (0, NQ, D) and ak.shape == (0, NKV, D)
    kc = torch.full((4, 256, NKV, D), -3.0, dtype=BF, device="cuda")
    store_kvcache(_e(0, NKV, D), _e(0, NKV, D), kc, kc, _e(0, dtype=torch.int32))
    assert bool((kc == -3).all())


def test_gathers_and_decode_attention_on_empty_work():
    cache = torch.randn(4, 256, NKV, D, device="cuda").to(BF)
    table = torch.arange(4, dtype=torch.int32, device="cuda")
    assert ops.paged_gather(cache, table, 0).shape == (0, NKV, D)
    out = ops.paged_gather_varlen(cache, _e(0, 4, dtype=torch.int32), _e(0, dtype=torch.int32),
                                  torch.zeros(1, dtype=torch.int64, device="cuda"), 0, 0)
    assert out.shape == (0, NKV, D)
    o = ops.decode_attention(_e(0, NQ, D), cache, cache, _e(0, dtype=torch.int32), _e(0, 4, dtype=torch.int32),
                             D ** -0.5)
    assert o.shape == (0, NQ, D)
