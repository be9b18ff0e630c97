"""The C ABI library and the torch binding load and export what the header
declares (no GPU needed: nothing is launched)."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "nib_b200.h"


@pytest.fixture(scope="module")
def built():
    from nano_vllm_multimodal_b200 import _build
    _build.build()
    return _build


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^NIB_API\s+(?:int|const char\*)\s+(nib_\w+)\s*\(", text, re.M)))


def test_header_declares_the_path():
    names = declared_symbols()
    for required in ("nib_rms_norm", "nib_add_rms_norm", "nib_silu_and_mul", "nib_qk_prologue",
                     "nib_mrope_apply", "nib_mrope_cos_sin", "nib_paged_store", "nib_paged_gather",
                     "nib_paged_gather_varlen", "nib_embedding", "nib_deepstack_add", "nib_copy_rows"):
        assert required in names


def test_library_exports_every_declared_symbol(built):
    lib = ctypes.CDLL(str(built.LIB))
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in nib_b200.h but not exported"
    lib.nib_abi_version.restype = ctypes.c_int
    assert lib.nib_abi_version() == 1


def test_library_rejects_bad_arguments_without_a_gpu(built):
    """Argument checks run on the host before any CUDA call."""
    lib = ctypes.CDLL(str(built.LIB))
    lib.nib_last_error.restype = ctypes.c_char_p
    rc = lib.nib_rms_norm(2, None, ctypes.c_int64(0), ctypes.c_int64(0), ctypes.c_int64(4),
                          ctypes.c_int64(1), ctypes.c_int64(1024), 2, None, ctypes.c_float(1e-6), None, None)
    assert rc == 1 and b"null pointer" in lib.nib_last_error()
    rc = lib.nib_paged_store(2, None, ctypes.c_int64(0), None, ctypes.c_int64(0), ctypes.c_int64(-1),
                             ctypes.c_int64(8), None, None, ctypes.c_int64(8), ctypes.c_int64(8), None, None, None)
    assert rc == 1
    # zero-size work is a no-op that needs no pointers at all
    rc = lib.nib_silu_and_mul(2, None, ctypes.c_int64(0), ctypes.c_int64(0), ctypes.c_int64(64), None, None)
    assert rc == 0


def test_prologue_struct_size_is_checked(built):
    lib = ctypes.CDLL(str(built.LIB))

    class Args(ctypes.Structure):
        _fields_ = [("struct_size", ctypes.c_int32)]

    a = Args(7)
    assert lib.nib_qk_prologue(ctypes.byref(a), None) == 1


def test_torch_binding_registers_reference_and_new_ops(built):
    from nano_vllm_multimodal_b200._lib import load_ops
    load_ops()
    assert torch.ops.nanoinfer_b200.abi_version() == 1
    for op in ("store", "gather"):
        assert hasattr(torch.ops.nanovllm_paged_kv, op)
    for op in ("rms_norm", "add_rms_norm", "silu_and_mul", "qk_prologue", "mrope_apply", "mrope_cos_sin",
               "paged_gather_varlen", "embedding", "deepstack_add", "deepstack_add_"):
        assert hasattr(torch.ops.nanoinfer_b200, op)
    assert torch.classes.nanovllm_paged_kv.PagedKVCache is not None
    schema = str(torch.ops.nanovllm_paged_kv.store.default._schema)
    assert "Tensor(a!) key_cache" in schema and "Tensor(b!) value_cache" in schema


def test_cpu_tensors_fail_loudly(built):
    """No CPU kernel is registered: calling with CPU tensors raises."""
    from nano_vllm_multimodal_b200 import ops
    with pytest.raises(NotImplementedError):
        ops.rms_norm(torch.randn(2, 64), torch.ones(64), 1e-6)
    with pytest.raises(NotImplementedError):
        ops.paged_gather(torch.zeros(2, 4, 1, 8), torch.tensor([0], dtype=torch.int32), 4)
