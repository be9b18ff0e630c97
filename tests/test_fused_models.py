"""The fused path through the reference's own model classes (``install()``).

Small Qwen3, Qwen2.5-VL and Qwen3-VL models are built from the reference's
model code (``tests/_model_step.py``) and run one prefill step (two sequences,
one padding slot, a Qwen3-VL image span with DeepStack payloads) and one
decode step. Three runs are compared:

* ``reference``: the reference's model, layers and store, untouched;
* ``perop``: ``install(fused=False)``, each op swapped for its kernel;
* ``fused``: ``install()``, the model classes' forwards running one prologue
  launch per attention layer (q/k norm + rotary + K/V store) and the Qwen3-VL
  residual adds and DeepStack rows folded into the norms.

The reference must be importable: ``$NANOINFER_REF`` or an install in the
git-ignored ``baseline/_ref`` (``python -m pip install --no-index
--no-build-isolation --no-deps --target baseline/_ref <checkout>``). Without it
the tests skip and say so. Each run is a fresh interpreter, so the reference's
modules never enter this test session.
"""

import json
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
REF = Path(os.environ.get("NANOINFER_REF") or ROOT / "baseline" / "_ref")
HAVE_REF = (REF / "nanovllm" / "__init__.py").is_file()
need_ref = pytest.mark.skipif(not HAVE_REF, reason=f"NanoInfer reference not importable from {REF} "
                              "(set NANOINFER_REF or install it into baseline/_ref)")

MODELS = ("qwen3", "qwen25_vl", "qwen3_vl")
ATTENTION_LAYERS = 2 + 2 + 3  # layers of the three small models
STEPS = 2


def _run_modes(device, tmp_path, modes=("reference", "perop", "fused")):
    env = dict(os.environ, TORCHDYNAMO_DISABLE="1")

    def one(mode):
        out = tmp_path / f"{device}_{mode}.pt"
        r = subprocess.run([sys.executable, str(ROOT / "tests" / "_model_step.py"), str(REF), device,
                            mode, str(out)], capture_output=True, text=True, env=env, timeout=900)
        assert r.returncode == 0, f"{mode}: {r.stderr[-4000:]}"
        return mode, json.loads(r.stdout.strip().splitlines()[-1]), torch.load(out)

    parallel = 3 if device == "cpu" else 1
    with ThreadPoolExecutor(parallel) as pool:
        done = list(pool.map(one, modes))
    return {m: (calls, res) for m, calls, res in done}


def _pairs(a, b):
    for model in MODELS:
        for key, x in a[model].items():
            y = b[model][key]
            if isinstance(x, list):
                assert len(x) == len(y), (model, key)
                for i, (xi, yi) in enumerate(zip(x, y)):
                    yield f"{model}.{key}[{i}]", xi, yi
            else:
                yield f"{model}.{key}", x, y


@need_ref
def test_fused_route_through_reference_models_cpu(tmp_path):
    """CPU, kernels replaced by the oracle in the reference's rounding order:
    the fused and per-op routes equal the reference's own run bit for bit, and
    the fused route launches one prologue with the store per attention layer,
    no separate store and one DeepStack fold per payload."""
    runs = _run_modes("cpu", tmp_path)
    ref = runs["reference"][1]
    for mode in ("perop", "fused"):
        for name, x, y in _pairs(runs[mode][1], ref):
            assert torch.equal(x, y), f"{mode} {name}: max diff {(x - y).abs().max().item()}"
    fused_calls, perop_calls = runs["fused"][0], runs["perop"][0]
    assert fused_calls.get("qk_prologue.store") == ATTENTION_LAYERS * STEPS
    assert "qk_prologue.nostore" not in fused_calls and "paged_store" not in fused_calls
    assert fused_calls.get("add_rms_norm_deepstack") == 3 and "deepstack_add" not in fused_calls
    assert fused_calls.get("deepstack_row_index") == 1
    # decode steps read k from the cache: no contiguous rotated k is written
    assert fused_calls.get("qk_prologue.cache_only_k") == ATTENTION_LAYERS
    # the per-op route: rotary without the store (the reference's attention stores), three DeepStack adds
    assert perop_calls.get("qk_prologue.nostore") == ATTENTION_LAYERS * STEPS
    assert "qk_prologue.store" not in perop_calls and perop_calls.get("deepstack_add") == 3


def _rel(x, t):
    return float((x.double() - t.double()).norm() / t.double().norm().clamp_min(1e-30))


@need_ref
@pytest.mark.gpu
def test_fused_route_through_reference_models_gpu(tmp_path):
    """On the B200, with this package's kernels and flash-attn for prefill:

    * the fused route equals the per-op route bit for bit: every layer output,
      both steps' final hidden states and every K/V cache (both routes use the
      same kernels; fusing changes nothing in the arithmetic);
    * the fused route is as accurate as the reference's own bf16 run on the
      GPU (eager: torch CUDA reductions, two-rounding SiluAndMul, its store,
      flash-attn's decode). Both are measured against the same model in
      float64 (``truth``: the same bf16 weights and inputs widened, attention
      as float64 SDPA). Over all of a model's tensors (squared errors summed)
      the fused route's relative error is at most 1.25x the reference's own;
      tensor by tensor at most 2x plus 2**-12 (a decode step's layer output is
      only 2 tokens x 512 values, too few for a tighter per-tensor ratio). The
      two bf16 runs are not compared element by element: each op's last-bit
      differences (1-2 ulp, bounded op by op in the other tests) spread through
      the GEMMs."""
    runs = _run_modes("cuda", tmp_path, ("reference", "perop", "fused", "truth"))
    fused, perop, ref, truth = (runs[m][1] for m in ("fused", "perop", "reference", "truth"))
    for name, x, y in _pairs(fused, perop):
        assert torch.equal(x, y), f"fused vs per-op {name}: max diff {(x - y).abs().max().item()}"
    report, sums = {}, {}
    truth_of = {name: t for name, _, t in _pairs(fused, truth)}
    for name, x, y in _pairs(fused, ref):
        t = truth_of[name].double()
        e_fused, e_ref = _rel(x, t), _rel(y, t)
        report[name] = dict(fused_rel_err=e_fused, reference_rel_err=e_ref)
        acc = sums.setdefault(name.split(".")[0], [0.0, 0.0, 0.0])
        acc[0] += float((x.double() - t).pow(2).sum())
        acc[1] += float((y.double() - t).pow(2).sum())
        acc[2] += float(t.pow(2).sum())
    for model, (ef, er, tt) in sums.items():
        report[model] = dict(fused_rel_err=(ef / tt) ** 0.5, reference_rel_err=(er / tt) ** 0.5)
    from tests._util import report_dir
    (report_dir() / "fused_models_vs_reference.json").write_text(json.dumps(report, indent=1))
    for model in sums:
        r = report[model]
        assert r["fused_rel_err"] <= 1.25 * r["reference_rel_err"], (model, r)
    for name, r in report.items():
        assert r["fused_rel_err"] <= 2 * r["reference_rel_err"] + 2.0 ** -12, (name, r)
