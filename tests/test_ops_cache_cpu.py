"""The key under which alveare_b200.ops keeps the resident copy of a raw
W_combined buffer (the reference's operators take the packed buffer on every
call, kernels/gemv_q/gemv_q.py:33-43): the same buffer maps to the same key
and version; a host buffer refilled with another matrix, or a torch tensor
changed in place, gets a new version, so it is repacked instead of served
stale.  Host logic only."""
import numpy as np
import pytest

from alveare_b200 import ops
from oracle import q4


def test_host_buffer_refill_changes_the_version():
    rng = np.random.default_rng(1)
    a = q4.quantize_combined(rng.normal(0, 0.02, (512, 1024)).astype(np.float32))
    b = q4.quantize_combined(rng.normal(0, 0.02, (512, 1024)).astype(np.float32))
    key, ver = ops._buffer_key(a, 512, 1024, 0)
    assert ops._buffer_key(a, 512, 1024, 0) == (key, ver)
    staging = a.copy()
    k1, v1 = ops._buffer_key(staging, 512, 1024, 0)
    staging[...] = b                      # the staging-buffer pattern: same address, new matrix
    k2, v2 = ops._buffer_key(staging, 512, 1024, 0)
    assert k1 == k2 and v1 != v2
    assert ops._buffer_key(staging, 256, 1024, 0)[0] != k2   # the shape is part of the key


def test_small_host_buffer_is_fingerprinted_whole():
    a = np.zeros((4, 20), np.uint8)
    _, v0 = ops._buffer_key(a, 4, 32, 0)
    a[3, 19] = 1
    assert ops._buffer_key(a, 4, 32, 0)[1] != v0


def test_torch_in_place_change_bumps_the_version():
    torch = pytest.importorskip("torch")
    t = torch.zeros((8, 40), dtype=torch.uint8)
    k0, v0 = ops._buffer_key(t, 8, 64, 0)
    t.add_(1)
    k1, v1 = ops._buffer_key(t, 8, 64, 0)
    assert k0 == k1 and v1 != v0
