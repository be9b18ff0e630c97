"""Fused forwards for the reference's decoder classes.

``integration.install()`` binds these as the ``forward`` methods of the
reference's own model classes, so an unchanged ``ModelRunner`` runs the fused
kernels:

* ``Qwen3Attention.forward``      (``nanovllm/models/qwen3.py:72-88``)
* ``Qwen25VLAttention.forward``   (``nanovllm/models/qwen25_vl.py:62-78``)
* ``Qwen3VLAttention.forward``    (``nanovllm/models/qwen3_vl.py:142-180``)

  split of the qkv row, per-head q/k norm, RoPE / M-RoPE and the paged K/V
  store become ONE prologue launch; the attention module then skips its own
  store (``Attention.forward_stored``).

* ``Qwen3VLDecoderLayer.forward``  (``qwen3_vl.py:226-240``) and
  ``Qwen3VLLanguageModel.forward`` (``qwen3_vl.py:346-378``)

  the separate bf16 residual adds and the DeepStack row add fold into the next
  norm (one pass: rounded add, visual-row add, text norm).

Parameter and buffer names are untouched (these are methods, not modules), so
the reference's weight loader still finds every weight. Norm and rotary state
is read from the module attributes the reference defines (``weight``/``eps``,
``cos_sin_cache``, ``inv_freq``/``sections``/``strategy``), so models built
before ``install()`` take the fused route too.
"""

from __future__ import annotations

import sys

import torch

from nano_vllm_multimodal_b200 import ops
from nano_vllm_multimodal_b200.layers.attention import _step_context, attention_prologue
from nano_vllm_multimodal_b200.layers.qwen3_vl import add_deepstack_rows

# ---------------------------------------------------------------- attention


def _prologue_then_attend(self, qkv: torch.Tensor, positions: torch.Tensor, q_norm, k_norm):
    """qkv row -> attention output, the K/V store folded into the prologue when
    the attention module can skip its own store (this package's ``Attention``)
    and the runner has attached caches. Otherwise (no caches yet, or the
    reference's ``SDPAAttention``, which stores before its gathers) the prologue
    only normalises and rotates, and the module stores as usual."""
    attn = self.attn
    k_cache, v_cache = attn.k_cache, attn.v_cache
    shape = dict(num_heads=self.num_heads, num_kv_heads=self.num_kv_heads, head_dim=self.head_dim,
                 positions=positions, rotary_emb=self.rotary_emb, q_norm=q_norm, k_norm=k_norm)
    stored = getattr(attn, "forward_stored", None)
    if stored is not None and k_cache.numel() and v_cache.numel():
        ctx = _step_context()
        # only prefill without a block table reads this step's k directly; decode
        # and prefix-cached / chunked prefill read k from the cache
        emit_k = bool(ctx.is_prefill and ctx.block_tables is None)
        q, k, v = attention_prologue(qkv, k_cache=k_cache, v_cache=v_cache,
                                     slot_mapping=ctx.slot_mapping, emit_k=emit_k, **shape)
        return stored(q, k, v)
    q, k, v = attention_prologue(qkv, **shape)
    return attn(q, k, v)


def qwen3_attention_forward(self, positions: torch.Tensor, hidden_states: torch.Tensor) -> torch.Tensor:
    """``Qwen3Attention.forward``: q/k RMSNorm only without qkv bias, as the reference."""
    qkv = self.qkv_proj(hidden_states)
    q_norm, k_norm = (None, None) if self.qkv_bias else (self.q_norm, self.k_norm)
    o = _prologue_then_attend(self, qkv, positions, q_norm, k_norm)
    return self.o_proj(o.flatten(1, -1))


def qwen25_vl_attention_forward(self, positions: torch.Tensor, hidden_states: torch.Tensor) -> torch.Tensor:
    """``Qwen25VLAttention.forward``: no q/k norm, chunked M-RoPE."""
    qkv = self.qkv_proj(hidden_states)
    o = _prologue_then_attend(self, qkv, positions, None, None)
    return self.o_proj(o.flatten(1, -1))


def _hf_aligned_linear():
    return sys.modules["nanovllm.models.qwen3_vl"].hf_aligned_linear


def qwen3_vl_attention_forward(self, positions: torch.Tensor, hidden_states: torch.Tensor) -> torch.Tensor:
    """``Qwen3VLAttention.forward``: text norm on q/k, interleaved M-RoPE.

    The SDPA backend's HF-aligned projections (``projection_mode="separate"``,
    ``output_projection_mode="hf_aligned"``) are kept as the reference computes
    them; only the part between the projections is fused."""
    if self.projection_mode == "separate":
        linear = _hf_aligned_linear()
        q_w, k_w, v_w = self.qkv_proj.weight.split((self.q_size, self.kv_size, self.kv_size), dim=0)
        qkv = torch.cat((linear(hidden_states, q_w), linear(hidden_states, k_w),
                         linear(hidden_states, v_w)), dim=-1)
    else:
        qkv = self.qkv_proj(hidden_states)
    o = _prologue_then_attend(self, qkv, positions, self.q_norm, self.k_norm).flatten(1, -1)
    if self.output_projection_mode == "hf_aligned":
        return _hf_aligned_linear()(o, self.o_proj.weight, self.o_proj.bias)
    return self.o_proj(o)


# ---------------------------------------------------------------- Qwen3-VL layer boundary


def _text_norm(norm, x: torch.Tensor, residual: torch.Tensor | None = None, deepstack=None):
    """``Qwen3VLTextRMSNorm`` (``qwen3_vl.py:68-79``) of ``x``, or of the rounded
    sum ``x + residual`` (plus the DeepStack rows) -> ``normed`` or
    ``(normed, sum)``. Works on the reference's module as well as on this
    package's: only ``weight`` and ``eps`` are read."""
    if norm.weight.dtype != x.dtype:
        raise TypeError("Qwen3VLTextRMSNorm: weight dtype must match the activations "
                        f"({norm.weight.dtype} vs {x.dtype})")
    if residual is None:
        return ops.rms_norm(x, norm.weight, norm.eps)
    if deepstack is None:
        return ops.add_rms_norm(x, residual, norm.weight, norm.eps, round_sum=True)
    visual_embedding, row_index = deepstack
    return ops.add_rms_norm_deepstack(x, residual, norm.weight, norm.eps, visual_embedding, row_index)


def qwen3_vl_decoder_layer_forward(self, positions: torch.Tensor, hidden_states: torch.Tensor,
                                   residual: torch.Tensor | None, deepstack=None):
    """``Qwen3VLDecoderLayer.forward`` in the residual form ``(x, residual)``
    that ``Qwen3DecoderLayer`` returns: the reference's layer output is
    ``x + residual`` (one bf16 rounding), which the next layer's input norm,
    or the final norm, computes in the same pass as its statistics.

    The reference loop (``qwen3_vl.py:366-370``) completes the sum itself when
    a layer returns a residual, so this form is also correct under the
    reference's own ``Qwen3VLLanguageModel.forward``.

    ``deepstack=(visual_embedding, row_index)`` adds the previous layer's
    DeepStack rows to the completed sum before the input norm (``row_index``
    from ``ops.deepstack_row_index``)."""
    if residual is None:
        if deepstack is not None:
            raise ValueError("the DeepStack fold needs the previous layer's residual")
        attention_residual = hidden_states
        hidden_states = _text_norm(self.input_layernorm, hidden_states)
    else:
        hidden_states, attention_residual = _text_norm(self.input_layernorm, hidden_states, residual,
                                                       deepstack)
    attention_out = self.self_attn(positions, hidden_states)
    hidden_states, mlp_residual = _text_norm(self.post_attention_layernorm, attention_out,
                                             attention_residual)
    return self.mlp(hidden_states), mlp_residual


def qwen3_vl_language_model_forward(self, input_ids: torch.Tensor | None, positions: torch.Tensor, *,
                                    inputs_embeds: torch.Tensor | None = None,
                                    visual_token_rows: torch.Tensor | None = None,
                                    deepstack_visual_embeds: tuple[torch.Tensor, ...] = ()) -> torch.Tensor:
    """``Qwen3VLLanguageModel.forward`` with the per-layer bf16 residual adds and
    the DeepStack adds after layers 0..2 folded into the following norm.

    Same validation (the reference's own ``_validate_inputs`` /
    ``_validate_deepstack``) and the same result: layer ``i``'s output plus
    ``deepstack_visual_embeds[i]`` at ``visual_token_rows`` feeds layer
    ``i + 1``; the final norm reads the last layer's output (plus its
    DeepStack rows when the model has no more layers than payloads).
    Layers of any other class are called as the reference loop calls them."""
    self._validate_inputs(input_ids, positions, inputs_embeds)
    hidden_states = self.embed_tokens(input_ids) if inputs_embeds is None else inputs_embeds
    self._validate_deepstack(hidden_states, visual_token_rows, deepstack_visual_embeds)

    payloads = len(deepstack_visual_embeds)
    row_index = None
    if payloads and visual_token_rows.numel():
        row_index = ops.deepstack_row_index(visual_token_rows, hidden_states.shape[0])

    def after(layer_index):
        if row_index is None or layer_index < 0 or layer_index >= payloads:
            return None
        return deepstack_visual_embeds[layer_index], row_index

    residual = None
    for layer_index, layer in enumerate(self.layers):
        pending = after(layer_index - 1)
        if type(layer).forward is qwen3_vl_decoder_layer_forward:
            hidden_states, residual = layer(positions, hidden_states, residual, pending)
            continue
        if residual is not None:  # the reference loop: complete the sum, then the rows
            hidden_states = hidden_states + residual
            residual = None
        if pending is not None:
            hidden_states = add_deepstack_rows(hidden_states, visual_token_rows, pending[0])
        hidden_states, residual = layer(positions, hidden_states, residual)

    pending = after(len(self.layers) - 1)
    if residual is None:
        if pending is not None:
            hidden_states = add_deepstack_rows(hidden_states, visual_token_rows, pending[0])
        return _text_norm(self.norm, hidden_states)
    return _text_norm(self.norm, hidden_states, residual, pending)[0]
