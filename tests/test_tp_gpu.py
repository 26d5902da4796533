"""Tensor-parallel FFN stack across GPUs (one process per GPU, 2 and 4
ranks): each rank holds I-slice `rank` of every layer and the one-launch stack
kernel sums the ranks' partial down projections over NVLink
(alveare_b200.stack; the reference's I-split and host partial sum,
kernels/ffn_fused/ffn_fused.py:46-60, runtime/cpp/src/npu.cpp:360-377).

Checked: every rank returns the identical output; it matches the one-GPU
stack over the whole intermediate dimension up to bf16 rounding flips (the
ranks' fp32 partial sums are added in another order), and the CPU oracle's
chained FFN half-blocks (runtime/py/model.py:782-806) normwise.  The ranks'
host exchange runs over gloo; no NCCL is involved.  Skipped with fewer GPUs
than ranks: ranks of this kernel wait for one another and must never share
a GPU."""
import datetime
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from oracle import q4  # noqa: E402

H, I, L = 512, 2048, 3


def _layers(seed):
    rng = np.random.default_rng(seed)
    return [tuple(q4.quantize_combined(rng.normal(0, 0.02, shape).astype(np.float32))
                  for shape in ((I, H), (I, H), (H, I))) for _ in range(L)]


def _x0(seed):
    return q4.to_bf16(np.random.default_rng(seed).normal(0, 1, H).astype(np.float32))


def _rank(rank, world, port, act, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from alveare_b200.stack import FFNStack
    try:
        layers = _layers(500 + world)
        x = torch.from_numpy(q4.bf16_bits(_x0(7)).view(np.int16)).view(torch.bfloat16).pin_memory()
        st = FFNStack(H, I, device=rank, rank=rank, world=world, activation=act)
        for cg, cu, cd in layers:
            st.add_layer(cg, cu, cd)
        ys = []
        for _ in range(3):  # repeated steps: exchange slots alternate, counters carry over
            y = torch.empty(H, dtype=torch.bfloat16).pin_memory()
            st.forward(x, y)
            ys.append(y.view(torch.int16).numpy().copy())
        assert st.launches == 1
        st.free()
        np.save(os.path.join(out_dir, f"y{rank}.npy"), np.stack(ys))
        if rank == 0:  # the one-GPU stack over the whole I
            one = FFNStack(H, I, device=0, activation=act)
            for cg, cu, cd in layers:
                one.add_layer(cg, cu, cd)
            y = torch.empty(H, dtype=torch.bfloat16).pin_memory()
            one.forward(x, y)
            np.save(os.path.join(out_dir, "one.npy"), y.view(torch.int16).numpy().copy())
            one.free()
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,act", [(2, "gelu"), (2, "silu"), (4, "gelu")])
def test_tp_stack_ranks_agree_and_match_one_gpu_and_oracle(tmp_path, world, act):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs (ranks of this kernel must not share a GPU)")
    mp.start_processes(_rank, args=(world, _free_port(), act, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    ys = [np.load(tmp_path / f"y{r}.npy") for r in range(world)]
    for r in range(1, world):
        assert np.array_equal(ys[0], ys[r])          # every rank: identical bits
    assert all(np.array_equal(ys[0][0], ys[0][s]) for s in range(1, 3))  # repeated steps agree
    got = q4.bits_to_f32(ys[0][0].view(np.uint16))
    one = q4.bits_to_f32(np.load(tmp_path / "one.npy").view(np.uint16))
    assert np.mean(got == one) >= 0.97
    assert float(np.max(np.abs(got - one)) / np.max(np.abs(one))) <= 1e-2
    ref = _x0(7)
    for cg, cu, cd in _layers(500 + world):
        ref = q4.ffn_block_gemma4(ref, cg, cu, cd, activation=act)
    assert float(np.max(np.abs(got - ref)) / np.max(np.abs(ref))) <= 1e-2
