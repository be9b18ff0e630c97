"""This repo's paged-KV store and gather against the reference's own CUDA kernels.

The reference's only GPU kernels on this path are its ``nanovllm_paged_kv``
store / gather extension (``csrc/paged_kv/paged_kv_cuda.cu``), which
``oracle/build_ref_ext.py`` compiles for sm_100a into ``oracle/_ref`` from the
reference's sources. A child process runs it (it registers the same op
namespace as this repo's binding) on the shared seeded inputs of
``tests/_paged_kv_cases.py``:

* the reference's parity matrix (fp16/bf16/fp32 x 1/2/8 kv heads x head_dim
  64/80/128/256 x 1/8/257 tokens x contiguous / random slots with every 11th
  slot -1, caches prefilled with -3): caches after the store and the gathered
  rows must be bit-identical to this repo's;
* C5 head shapes (65,536 tokens into a 1,024-block cache pair; 16 sequences x
  16,384 tokens gathered): bit-identical results (sha256 of the caches and of
  the gathered rows), and both sides timed one call at a time after an L2
  flush. The times go to ``reference_paged_kv.json`` in the report directory
  (``tests/_util.report_dir``).

Skips where the library has not been built (no reference checkout at build time).
"""

import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from nano_vllm_multimodal_b200 import ops
from tests._paged_kv_cases import digest, parity_cases, parity_inputs, time_ms, timing_inputs

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "oracle" / "_ref" / "nanovllm_paged_kv_ref.so"

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not LIB.exists(), reason="reference extension not built (oracle/build_ref_ext.py)")]


@pytest.fixture(scope="module")
def reference(tmp_path_factory):
    out = tmp_path_factory.mktemp("ref") / "ref.pt"
    r = subprocess.run([sys.executable, str(ROOT / "tests" / "_ref_paged_kv_child.py"), str(LIB), str(out)],
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-4000:]
    return torch.load(out)


def test_parity_matrix_matches_the_reference_kernels_bit_for_bit(reference):
    for case in parity_cases():
        key, value, slots, cache_shape, table = parity_inputs(*case)
        kc = torch.full(cache_shape, -3.0, dtype=key.dtype, device="cuda")
        vc = torch.full_like(kc, -3.0)
        ops.paged_store(key.cuda(), value.cuda(), kc, vc, slots.cuda())
        n = key.shape[0] + 5
        g = ops.paged_gather(kc, table.cuda(), min(n, table.numel() * cache_shape[1]))
        rk, rv, rg = reference["parity"][case[0]]
        what = f"case {case}"
        assert torch.equal(kc.cpu().view(torch.uint8), rk.view(torch.uint8)), f"{what}: key cache"
        assert torch.equal(vc.cpu().view(torch.uint8), rv.view(torch.uint8)), f"{what}: value cache"
        assert torch.equal(g.cpu().view(torch.uint8), rg.view(torch.uint8)), f"{what}: gather"


def test_c5_shapes_match_and_are_timed_beside_the_reference(reference):
    k, v, slots, tables = timing_inputs("cuda")
    kc = torch.zeros(1024, 256, 8, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    store_ms = time_ms(lambda: ops.paged_store(k, v, kc, vc, slots), flush)
    gather_ms = time_ms(lambda: [ops.paged_gather(kc, tables[i], 16384) for i in range(16)], flush)
    lens = torch.full((16,), 16384, dtype=torch.int32, device="cuda")
    cu = torch.arange(17, dtype=torch.int64, device="cuda") * 16384
    varlen_ms = time_ms(lambda: ops.paged_gather_varlen(kc, tables, lens, cu, 16 * 16384, 16384), flush)
    assert digest(kc, vc) == reference["timing"]["store_digest"], "C5 store: caches differ from the reference's"
    assert digest(*[ops.paged_gather(kc, tables[i], 16384) for i in range(16)]) == \
        reference["timing"]["gather_digest"], "C5 gather: rows differ from the reference's"
    store_bytes = 65536 * 8 * 128 * 2 * 4          # k, v in; two cache rows out
    gather_bytes = 16 * 16384 * 8 * 128 * 2 * 2    # rows in and out
    peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"] if \
        (ROOT / "MEASURED_PEAKS.json").exists() else 6650.0
    rt = reference["timing"]
    frac = lambda b, ms: round(b / (ms / 1e3) / 1e9 / peak, 4)  # noqa: E731
    report = {
        "store": {"ours_ms": store_ms, "reference_ms": rt["store_ms"], "ours_frac": frac(store_bytes, store_ms),
                  "reference_frac": frac(store_bytes, rt["store_ms"])},
        "gather_16_sequences": {"ours_ms_16_calls": gather_ms, "ours_ms_one_varlen_launch": varlen_ms,
                                "reference_ms_16_calls": rt["gather_16_calls_ms"],
                                "ours_frac_varlen": frac(gather_bytes, varlen_ms),
                                "reference_frac": frac(gather_bytes, rt["gather_16_calls_ms"])},
        "peak_gbs": peak}
    from tests._util import report_dir
    (report_dir() / "reference_paged_kv.json").write_text(json.dumps(report, indent=1))
