"""Child process of tests/test_gpu_reference_paged_kv.py: the reference's own
paged-KV CUDA extension (compiled into oracle/_ref by oracle/build_ref_ext.py)
on the shared seeded inputs. It loads only that library, never this repo's
binding (both register the ``nanovllm_paged_kv`` namespace).

Usage: python tests/_ref_paged_kv_child.py LIB OUT.pt
"""

import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from tests._paged_kv_cases import digest, parity_cases, parity_inputs, time_ms, timing_inputs  # noqa: E402

torch.ops.load_library(sys.argv[1])
ops = torch.ops.nanovllm_paged_kv
out = {"parity": {}, "timing": {}}
for case in parity_cases():
    key, value, slots, cache_shape, table = parity_inputs(*case)
    kc = torch.full(cache_shape, -3.0, dtype=key.dtype, device="cuda")
    vc = torch.full_like(kc, -3.0)
    ops.store(key.cuda(), value.cuda(), kc, vc, slots.cuda())
    n = key.shape[0] + 5
    g = ops.gather(kc, table.cuda(), min(n, table.numel() * cache_shape[1]))
    out["parity"][case[0]] = (kc.cpu(), vc.cpu(), g.cpu())

k, v, slots, tables = timing_inputs("cuda")
kc = torch.zeros(1024, 256, 8, 128, dtype=torch.bfloat16, device="cuda")
vc = torch.zeros_like(kc)
flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device="cuda")
out["timing"]["store_ms"] = time_ms(lambda: ops.store(k, v, kc, vc, slots), flush)
out["timing"]["gather_16_calls_ms"] = time_ms(lambda: [ops.gather(kc, tables[i], 16384) for i in range(16)], flush)
out["timing"]["store_digest"] = digest(kc, vc)
out["timing"]["gather_digest"] = digest(*[ops.gather(kc, tables[i], 16384) for i in range(16)])
torch.save(out, sys.argv[2])
print("ok")
