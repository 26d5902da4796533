"""The C-ABI library builds, loads and exports every function the header
declares; argument validation works without a GPU.  CPU only."""
import ctypes
import os
import re

import pytest

from alveare_b200 import _lib, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "alveare_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(alv_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_header_declares_the_abi():
    fns = header_functions()
    assert "alv_gemv" in fns and "alv_ffn" in fns and "alv_gemv_weight_create" in fns
    assert len(fns) >= 15


def test_library_exports_every_declared_symbol(lib):
    for name in header_functions():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_signature_table_has_no_extra_entries():
    assert set(_lib.SIGNATURES) == set(header_functions())


def test_version_and_null_handling(lib):
    assert lib.alv_version() == 200
    assert lib.alv_last_error(None) == b"null context"
    assert lib.alv_ctx_destroy(None) == 1          # ALV_ERR_ARG
    assert lib.alv_sync_status(None, None) == 1
    out = ctypes.c_void_p()
    assert lib.alv_ctx_create(0, None) == 1


def test_every_entry_point_rejects_a_null_context(lib):
    """Every function taking a context returns ALV_ERR_ARG for a null one
    (all other arguments zero or null), before touching anything."""
    checked = 0
    for name, (_, args) in _lib.SIGNATURES.items():
        if not args or args[0] is not ctypes.c_void_p or name == "alv_last_error":
            continue
        vals = [0 if a in (ctypes.c_int, ctypes.c_uint32, ctypes.c_int64, ctypes.c_size_t) else None for a in args]
        assert getattr(lib, name)(*vals) == 1, name
        checked += 1
    assert checked >= 30


def test_no_device_is_reported_not_crashed(lib):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    p = ctypes.c_void_p()
    assert lib.alv_ctx_create(0, ctypes.byref(p)) == 7  # ALV_ERR_NO_DEVICE
    assert not p.value


def test_python_ops_fail_loudly_without_a_device(lib):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import numpy as np

    from alveare_b200 import Q4Weight
    with pytest.raises(_lib.AlvError):
        Q4Weight(np.zeros((16, 20), np.uint8))
