"""Swap this package's kernels into an installed NanoInfer (``nanovllm``).

``install()`` rebinds, inside the already-importable ``nanovllm`` package, the
hot-path names that the decoder models import at module load:

* ``nanovllm.layers.layernorm.RMSNorm``
* ``nanovllm.layers.activation.SiluAndMul``
* ``nanovllm.layers.rotary_embedding.{RotaryEmbedding, get_rope, apply_rotary_emb}``
* ``nanovllm.layers.multimodal_rotary_embedding.{MultimodalRotaryEmbedding,
  apply_multimodal_rotary_emb}``
* ``nanovllm.layers.embed_head.VocabParallelEmbedding``
* ``nanovllm.layers.attention.{store_kvcache, flash_attn_with_kvcache}`` (the
  decode attention reads the paged cache with this package's kernel; prefill
  keeps ``flash_attn_varlen_func``)
* ``nanovllm.models.qwen3_vl.Qwen3VLTextRMSNorm`` and
  ``Qwen3VLLanguageModel._add_deepstack_rows``
* ``nanovllm.engine.model_runner.{build_planned_visual_embeddings,
  merge_planned_visual_embeddings}`` (the packed-prefill visual merge, one
  kernel; results are the reference's own ``PlannedVisualEmbeddings``)
* ``nanovllm.layers.paged_kv.loader.load_paged_kv_extension`` - so the
  reference's own ``CUDAPagedKVBackend`` gets ``torch.ops.nanovllm_paged_kv``
  and ``PagedKVCache`` from this package's extension instead of JIT-building
  its sources; ``ModelRunner`` then runs unchanged with
  ``paged_kv_backend="cuda"``.

With ``fused=True`` (the default) it also binds the fused forwards of
``layers.fused_models`` into the reference's model classes, so the model code
runs the fused kernels without being edited:

* ``nanovllm.layers.attention.Attention`` -> this package's ``Attention`` (same
  interface, plus ``forward_stored`` for K/V that a prologue already wrote)
* ``Qwen3Attention.forward``, ``Qwen25VLAttention.forward``,
  ``Qwen3VLAttention.forward``: one prologue launch (q/k norm, RoPE / M-RoPE,
  paged K/V store) between the projections
* ``Qwen3VLDecoderLayer.forward``, ``Qwen3VLLanguageModel.forward``: residual
  adds and DeepStack rows folded into the norms

``fused=False`` rebinds only the per-op names above (each reference op replaced
by its kernel, the model code calling them one at a time).

Call it before ``nanovllm.models.*`` is imported (the models bind the layer
classes at import time); already-imported model modules are patched too when
they hold the names. Returns the list of rebound ``module.attribute`` names.
"""

from __future__ import annotations

import importlib
import sys


def _targets():
    from nano_vllm_multimodal_b200._lib import load_ops
    from nano_vllm_multimodal_b200.layers import activation, attention, embed_head, layernorm
    from nano_vllm_multimodal_b200.layers import multimodal_rotary_embedding as mrope
    from nano_vllm_multimodal_b200.layers import qwen3_vl, rotary_embedding, visual_merge

    def load_paged_kv_extension(*, verbose: bool = False) -> None:
        load_ops()

    def build_planned_visual_embeddings(token_embeddings, plan, features):
        runner = sys.modules.get("nanovllm.engine.model_runner")
        result_type = getattr(runner, "PlannedVisualEmbeddings", visual_merge.PlannedVisualEmbeddings)
        return visual_merge.build_planned_visual_embeddings(token_embeddings, plan, features,
                                                            result_type=result_type)

    def merge_planned_visual_embeddings(token_embeddings, plan, features):
        return build_planned_visual_embeddings(token_embeddings, plan, features).final_embedding

    return {
        "nanovllm.layers.layernorm": {"RMSNorm": layernorm.RMSNorm},
        "nanovllm.layers.activation": {"SiluAndMul": activation.SiluAndMul},
        "nanovllm.layers.rotary_embedding": {"RotaryEmbedding": rotary_embedding.RotaryEmbedding,
                                             "get_rope": rotary_embedding.get_rope,
                                             "apply_rotary_emb": rotary_embedding.apply_rotary_emb},
        "nanovllm.layers.multimodal_rotary_embedding": {
            "MultimodalRotaryEmbedding": mrope.MultimodalRotaryEmbedding,
            "apply_multimodal_rotary_emb": mrope.apply_multimodal_rotary_emb},
        "nanovllm.layers.embed_head": {"VocabParallelEmbedding": embed_head.VocabParallelEmbedding},
        "nanovllm.layers.attention": {"store_kvcache": attention.store_kvcache,
                                      "flash_attn_with_kvcache": attention.flash_attn_with_kvcache},
        "nanovllm.layers.paged_kv.loader": {"load_paged_kv_extension": load_paged_kv_extension},
        "nanovllm.layers.paged_kv.cuda_backend": {"load_paged_kv_extension": load_paged_kv_extension},
        "nanovllm.models.qwen3_vl": {"Qwen3VLTextRMSNorm": qwen3_vl.Qwen3VLTextRMSNorm},
        "nanovllm.engine.model_runner": {
            "build_planned_visual_embeddings": build_planned_visual_embeddings,
            "merge_planned_visual_embeddings": merge_planned_visual_embeddings},
    }


# names a model module imports from the layer modules above
_MODEL_MODULES = ("nanovllm.models.qwen3", "nanovllm.models.qwen25_vl", "nanovllm.models.qwen3_vl")


def _fused_forwards():
    from nano_vllm_multimodal_b200.layers import fused_models as fm
    return {
        "nanovllm.models.qwen3": {"Qwen3Attention": fm.qwen3_attention_forward},
        "nanovllm.models.qwen25_vl": {"Qwen25VLAttention": fm.qwen25_vl_attention_forward},
        "nanovllm.models.qwen3_vl": {"Qwen3VLAttention": fm.qwen3_vl_attention_forward,
                                     "Qwen3VLDecoderLayer": fm.qwen3_vl_decoder_layer_forward,
                                     "Qwen3VLLanguageModel": fm.qwen3_vl_language_model_forward},
    }


def install(fused: bool = True) -> list[str]:
    from nano_vllm_multimodal_b200.layers import attention, qwen3_vl

    targets = _targets()
    if fused:
        targets["nanovllm.layers.attention"]["Attention"] = attention.Attention
    done = []
    for mod_name, names in targets.items():
        try:
            mod = importlib.import_module(mod_name)
        except ImportError:
            continue
        for attr, obj in names.items():
            if hasattr(mod, attr):
                setattr(mod, attr, obj)
                done.append(f"{mod_name}.{attr}")
    flat = {attr: obj for names in targets.values() for attr, obj in names.items()}
    for mod_name in _MODEL_MODULES:
        mod = sys.modules.get(mod_name)
        if mod is None:
            continue
        for attr, obj in flat.items():
            if hasattr(mod, attr) and f"{mod_name}.{attr}" not in done:
                setattr(mod, attr, obj)
                done.append(f"{mod_name}.{attr}")
    lm = sys.modules.get("nanovllm.models.qwen3_vl")
    if lm is not None and hasattr(lm, "Qwen3VLLanguageModel"):
        lm.Qwen3VLLanguageModel._add_deepstack_rows = staticmethod(qwen3_vl.add_deepstack_rows)
        done.append("nanovllm.models.qwen3_vl.Qwen3VLLanguageModel._add_deepstack_rows")
    if fused:
        for mod_name, classes in _fused_forwards().items():
            try:
                mod = importlib.import_module(mod_name)
            except ImportError:
                continue
            for cls_name, forward in classes.items():
                cls = getattr(mod, cls_name, None)
                if cls is not None:
                    cls.forward = forward
                    done.append(f"{mod_name}.{cls_name}.forward")
    return done
