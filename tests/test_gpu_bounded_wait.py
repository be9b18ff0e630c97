"""The library's one device-side wait (the bulk-copy mbarrier wait of the
pipelined attention prologue) is bounded: make it run out and check that the
kernel reports it and returns.

``nib_selftest_bounded_wait`` arms an mbarrier for 32 bytes while its bulk copy
brings only 16, so the phase never completes. With a 20 ms limit the warp must
give up, set ``NIB_DEV_TIMEOUT`` in the status word, wait (bounded) for its
other copy, which does land, and return. Nothing faults or hangs: afterwards
the same context runs an ordinary kernel of the library and the stream's own
work, and the result is still right.
"""

import ctypes
import time

import pytest
import torch

from nano_vllm_multimodal_b200 import _lib, ops

pytestmark = pytest.mark.gpu

NIB_DEV_TIMEOUT = 16  # include/nib_b200.h


def _bind():
    lib = _lib.cdll()
    f = lib.nib_selftest_bounded_wait
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    f.restype = ctypes.c_int
    lib.nib_last_error.restype = ctypes.c_char_p
    return lib, f


@pytest.mark.parametrize("limit_ms", [20, 200])
def test_wait_that_never_completes_gives_up_and_reports(limit_ms):
    lib, f = _bind()
    src = torch.arange(32, dtype=torch.uint8, device="cuda") + 7
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    drained = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    start.record(stream)
    rc = f(src.data_ptr(), limit_ms * 1_000_000, status.data_ptr(), drained.data_ptr(), stream.cuda_stream)
    end.record(stream)
    assert rc == 0, lib.nib_last_error().decode()
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1e3
    kernel_ms = start.elapsed_time(end)
    assert int(status.item()) & NIB_DEV_TIMEOUT, "the wait did not report its timeout"
    assert int(drained.item()) == 1, "the second copy did not land before the warp returned"
    # it waited about its limit, and not much longer
    assert limit_ms * 0.9 <= kernel_ms <= limit_ms + 500, (kernel_ms, limit_ms)
    assert wall_ms < limit_ms + 5000
    # the context is usable afterwards
    x = torch.randn(64, 256, dtype=torch.bfloat16, device="cuda")
    y = ops.silu_and_mul(x)
    torch.cuda.synchronize()
    ref = torch.nn.functional.silu(x[:, :128].float()) * x[:, 128:].float()
    assert torch.allclose(y.float(), ref, rtol=2 ** -7, atol=1e-6)


def test_selftest_rejects_bad_arguments():
    lib, f = _bind()
    src = torch.zeros(48, dtype=torch.uint8, device="cuda")
    word = torch.zeros(2, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert f(src.data_ptr() + 1, 10_000, word.data_ptr(), word.data_ptr() + 4, stream) == 1
    assert b"16-byte aligned" in lib.nib_last_error()
    assert f(src.data_ptr(), 10, word.data_ptr(), word.data_ptr() + 4, stream) == 1
    assert f(src.data_ptr(), 3_000_000_000, word.data_ptr(), word.data_ptr() + 4, stream) == 1
    assert f(None, 10_000, word.data_ptr(), word.data_ptr() + 4, stream) == 1
