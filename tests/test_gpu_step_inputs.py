"""One-copy staging of a step's host inputs (``StepInputStager``).

The staged tensors must equal the ones the reference creates one by one
(model_runner.py:700-725,823-870), keep their values when the ring of pinned
slots is reused while earlier copies are still queued behind other GPU work,
and grow a slot when a step needs more room.
"""

import pytest
import torch

from nano_vllm_multimodal_b200.step_inputs import StepInputStager

pytestmark = pytest.mark.gpu


def _reference_tensors(ids, pos_rows, cuq, cuk, slots, ctx, qstart, tables, axes):
    """The reference's per-array pinned tensors and copies."""
    def cp(v, dt):
        return torch.tensor(v, dtype=dt, pin_memory=True).cuda(non_blocking=True)
    out = dict(input_ids=cp(ids, torch.int64), positions=cp(pos_rows, torch.int64),
               cu_seqlens_q=cp(cuq, torch.int32), cu_seqlens_k=cp(cuk, torch.int32),
               slot_mapping=cp(slots, torch.int32), full_context_lens=cp(ctx, torch.int32),
               query_start_lens=cp(qstart, torch.int32))
    if axes == 1:
        out["positions"] = out["positions"][0]
    width = max(len(b) for b in tables)
    out["block_tables"] = cp([b + [-1] * (width - len(b)) for b in tables], torch.int32)
    return out


@pytest.mark.parametrize("axes", [1, 3])
def test_prefill_inputs_match_the_reference_tensors(axes):
    g = torch.Generator().manual_seed(axes)
    lens = [5, 300, 17, 1]
    T = sum(lens)
    ids = torch.randint(0, 151936, (T,), generator=g).tolist()
    pos_rows = torch.randint(0, 40000, (axes, T), generator=g).tolist()
    cuq = [0] + torch.tensor(lens).cumsum(0).tolist()
    cuk = [c + 3 * i for i, c in enumerate(cuq)]
    slots = torch.randint(-1, 1 << 20, (T,), generator=g).tolist()
    ctx = [n + 3 for n in lens]
    qstart = [3] * len(lens)
    tables = [[1, 2], [7, 8, 9, 10], [3], [4, 5, 6]]
    st = StepInputStager(slots=2)
    got = st.prefill_inputs(ids, pos_rows, cuq, cuk, slots, ctx, qstart, tables, position_axes=axes)
    exp = _reference_tensors(ids, pos_rows, cuq, cuk, slots, ctx, qstart, tables, axes)
    torch.cuda.synchronize()
    assert set(got) == set(exp)
    for name, t in exp.items():
        assert got[name].dtype == t.dtype and got[name].shape == t.shape, name
        assert torch.equal(got[name], t), name
        assert got[name].is_cuda


def test_ring_reuse_while_copies_are_queued():
    st = StepInputStager(slots=2, initial_bytes=64)
    a = torch.randn(2048, 2048, device="cuda")
    outs = []
    for step in range(12):
        for _ in range(4):  # keep the stream busy so that the staging copies queue behind it
            a = torch.tanh(a @ a * 1e-3)
        vals = torch.arange(10_000, dtype=torch.int64) * (step + 1)
        outs.append((vals, st.stage(vals, (list(range(step, step + 33)), torch.int32))))
    torch.cuda.synchronize()
    for step, (vals, (d64, d32)) in enumerate(outs):
        assert torch.equal(d64.cpu(), vals), step
        assert d32.tolist() == list(range(step, step + 33)), step
    assert all(b >= 10_000 * 8 for b in st.slot_bytes())  # slots grew past the 64-byte start


def test_mixed_dtypes_and_empty_arrays():
    st = StepInputStager(slots=1, initial_bytes=0)
    f = torch.randn(7, 3)
    e = torch.empty(0, dtype=torch.int32)
    out = st.stage(f, e, (list(range(5)), torch.int64), (torch.ones(2, 2, dtype=torch.int32), torch.int32))
    torch.cuda.synchronize()
    assert torch.equal(out[0].cpu(), f) and out[0].dtype == torch.float32
    assert out[1].numel() == 0 and out[1].dtype == torch.int32 and out[1].is_cuda
    assert out[2].tolist() == list(range(5))
    assert out[3].shape == (2, 2) and int(out[3].sum()) == 4
    assert st.stage() == []


@pytest.mark.parametrize("axes", [1, 3])
def test_decode_inputs_match_the_reference_tensors(axes):
    """prepare_decode's five tensors (model_runner.py:892-935): one token per
    sequence, positions len - 1 (+ the M-RoPE delta on every axis), block tables
    of different lengths padded with -1."""
    g = torch.Generator().manual_seed(10 + axes)
    B = 37
    lens = torch.randint(1, 3000, (B,), generator=g).tolist()
    ids = torch.randint(0, 151936, (B,), generator=g).tolist()
    delta = torch.randint(-500, 500, (B,), generator=g).tolist() if axes == 3 else [0] * B
    row = [n - 1 + d for n, d in zip(lens, delta)]
    pos_rows = [row for _ in range(axes)]
    tables = [torch.randperm(4096, generator=g)[:(n + 255) // 256].tolist() for n in lens]
    slots = [t[-1] * 256 + (n - 1) % 256 for t, n in zip(tables, lens)]

    def cp(v, dt):
        return torch.tensor(v, dtype=dt, pin_memory=True).cuda(non_blocking=True)
    width = max(len(t) for t in tables)
    exp = dict(input_ids=cp(ids, torch.int64), positions=cp(pos_rows, torch.int64),
               slot_mapping=cp(slots, torch.int32), context_lens=cp(lens, torch.int32),
               block_tables=cp([t + [-1] * (width - len(t)) for t in tables], torch.int32))
    if axes == 1:
        exp["positions"] = exp["positions"][0]
    st = StepInputStager(slots=2)
    for _ in range(2):  # a second step reuses the ring
        got = st.decode_inputs(ids, pos_rows, slots, lens, tables, position_axes=axes)
        torch.cuda.synchronize()
        assert set(got) == set(exp)
        for name, t in exp.items():
            assert got[name].dtype == t.dtype and got[name].shape == t.shape, name
            assert torch.equal(got[name], t), name
