"""Tensor-parallel FFN decomposition on CPU ranks (gloo, world size 2 and 4):
each rank computes the partial down projection of its intermediate slice with
the C oracle, an all-reduce sums them, and the result equals the full FFN.
This is the host-side logic of the multi-GPU path (alveare_b200.stack)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from alveare_b200.stack import tp_slice
from oracle import cpu, q4

H, I = 256, 1024


def _weights():
    rng = np.random.default_rng(21)
    cg = q4.quantize_combined(rng.normal(0, 0.02, (I, H)).astype(np.float32))
    cu = q4.quantize_combined(rng.normal(0, 0.02, (I, H)).astype(np.float32))
    cd = q4.quantize_combined(rng.normal(0, 0.02, (H, I)).astype(np.float32))
    x = rng.normal(0, 1, H).astype(np.float32)
    return cg, cu, cd, x


def _slice(cg, cu, cd, b, e):
    return cg[b:e], cu[b:e], np.ascontiguousarray(cd[:, b // 32 * 20:e // 32 * 20])


def _rank(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cg, cu, cd, x = _weights()
        b, e = tp_slice(I, rank, world)
        y, _ = cpu.ffn(*_slice(cg, cu, cd, b, e), x, "gelu", 1)
        t = torch.from_numpy(y.copy())
        dist.all_reduce(t)
        if rank == 0:
            np.save(out, t.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [2, 4])
def test_tp_partials_all_reduce_to_full_ffn(tmp_path, world):
    out = str(tmp_path / "y.npy")
    mp.start_processes(_rank, args=(world, _free_port(), out), nprocs=world, start_method="spawn", join=True)
    y = np.load(out)
    cg, cu, cd, x = _weights()
    ref, _, _, _ = q4.ffn(cg, cu, cd, x, "gelu")
    assert float(np.max(np.abs(y - ref)) / np.max(np.abs(ref))) <= 1e-3


def test_tp_slice_rules():
    assert tp_slice(15360, 0, 8) == (0, 1920) and tp_slice(15360, 7, 8) == (13440, 15360)
    with pytest.raises(ValueError):
        tp_slice(96, 0, 2)    # 48-wide slices are not whole 32-blocks
    with pytest.raises(ValueError):
        tp_slice(1024, 2, 2)
