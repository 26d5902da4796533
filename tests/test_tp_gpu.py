"""Tensor-parallel FFN stack across GPUs (one process per GPU, 2, 4 and 8
ranks): each rank holds I-slice `rank` of every layer and the one-launch stack
kernel sums the ranks' partial down projections over NVLink
(alveare_b200.stack; the reference's I-split and host partial sum,
kernels/ffn_fused/ffn_fused.py:46-60, runtime/cpp/src/npu.cpp:360-377).

Checked:
* per layer, at the north-star 1e-3 (normwise, fp32): the summed down
  projection of layer 0 and of layer 1 (the stack probe, as every rank's
  final glue read it) against the CPU oracle's FFN (q4.ffn) on the rmsnorm of
  that layer's input -- x0 for layer 0, the one-layer stack's output for
  layer 1 (the identical bits layer 1 of the two-layer stack consumes);
* every rank returns the identical output, step after step;
* the three-layer chain against the one-GPU stack and the oracle's chained
  half-blocks (runtime/py/model.py:782-806).  The chain is held to 1e-2 and
  >= 97 % identical bits, not 1e-3: the ranks add their fp32 partial sums in
  another order than one GPU does, which flips an occasional bf16 rounding
  of the residual stream (one bf16 step is 2^-8 relative), and a flip
  propagates through the later layers' norms.  The per-layer checks above
  carry the 1e-3 bound.
The ranks' host exchange runs over gloo; no NCCL is involved.  Skipped with
fewer GPUs than ranks: ranks of this kernel wait for one another and must
never share a GPU."""
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
TOL = 1e-3


def _layers(seed):
    rng = np.random.default_rng(seed)
    return [tuple(q4.quantize_combined(rng.normal(0, 0.02, shape).astype(np.float32))
                  for shape in ((I, H), (I, H), (H, I))) for _ in range(L)]


def _x0(seed):
    return q4.to_bf16(np.random.default_rng(seed).normal(0, 1, H).astype(np.float32))


def _bits(t):
    return t.view(torch.int16).numpy().copy()


def _stack(layers, rank, world, act, probe=None):
    from alveare_b200.stack import FFNStack
    st = FFNStack(H, I, device=rank, rank=rank, world=world, activation=act)
    for cg, cu, cd in layers:
        st.add_layer(cg, cu, cd)
    if probe is not None:
        st.set_probe(probe)
    return st


def _rank(rank, world, port, act, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        layers = _layers(500 + world)
        x = torch.from_numpy(q4.bf16_bits(_x0(7)).view(np.int16)).view(torch.bfloat16).pin_memory()
        st = _stack(layers, rank, world, act)
        ys = []
        for _ in range(3):  # repeated steps: exchange slots alternate, counters carry over
            y = torch.empty(H, dtype=torch.bfloat16).pin_memory()
            st.forward(x, y)
            ys.append(_bits(y))
        assert st.launches == 1
        st.free()
        np.save(os.path.join(out_dir, f"y{rank}.npy"), np.stack(ys))
        # per-layer probes: stacks of the first one and the first two layers
        for n in (1, 2):
            probe = torch.full((H,), float("nan"), dtype=torch.float32, device=f"cuda:{rank}")
            sn = _stack(layers[:n], rank, world, act, probe=probe)
            y = torch.empty(H, dtype=torch.bfloat16).pin_memory()
            sn.forward(x, y)
            np.save(os.path.join(out_dir, f"probe{n}_{rank}.npy"), probe.cpu().numpy())
            np.save(os.path.join(out_dir, f"out{n}_{rank}.npy"), _bits(y))
            sn.free()
        if rank == 0:  # the one-GPU stack over the whole I
            one = _stack(layers, 0, 1, act)
            y = torch.empty(H, dtype=torch.bfloat16).pin_memory()
            one.forward(x, y)
            np.save(os.path.join(out_dir, "one.npy"), _bits(y))
            one.free()
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _normwise(y, ref):
    return float(np.max(np.abs(np.asarray(y, np.float64) - ref)) / np.max(np.abs(ref)))


@pytest.mark.parametrize("world,act", [(2, "gelu"), (2, "silu"), (4, "gelu"), (8, "gelu")])
def test_tp_stack_ranks_agree_and_match_one_gpu_and_oracle(tmp_path, world, act):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs (ranks of this kernel must not share a GPU)")
    mp.start_processes(_rank, args=(world, _free_port(), act, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    layers = _layers(500 + world)
    x0 = _x0(7)
    # per layer, 1e-3
    p1 = [np.load(tmp_path / f"probe1_{r}.npy") for r in range(world)]
    p2 = [np.load(tmp_path / f"probe2_{r}.npy") for r in range(world)]
    o1 = [np.load(tmp_path / f"out1_{r}.npy") for r in range(world)]
    for r in range(1, world):
        assert np.array_equal(p1[0], p1[r]) and np.array_equal(p2[0], p2[r]) and np.array_equal(o1[0], o1[r])
    d0_ref, _, _, _ = q4.ffn(*layers[0], q4.rmsnorm_gemma(x0), act)
    assert _normwise(p1[0], d0_ref) <= TOL
    x1 = q4.bits_to_f32(o1[0].view(np.uint16))
    d1_ref, _, _, _ = q4.ffn(*layers[1], q4.rmsnorm_gemma(x1), act)
    assert _normwise(p2[0], d1_ref) <= TOL
    assert np.mean(x1 == q4.to_bf16(x0 + q4.rmsnorm_gemma(q4.to_bf16(d0_ref)))) >= 0.99
    # the chain
    ys = [np.load(tmp_path / f"y{r}.npy") for r in range(world)]
    for r in range(1, world):
        assert np.array_equal(ys[0], ys[r])          # every rank: identical bits
    assert all(np.array_equal(ys[0][0], ys[0][s]) for s in range(1, 3))  # repeated steps agree
    got = q4.bits_to_f32(ys[0][0].view(np.uint16))
    one = q4.bits_to_f32(np.load(tmp_path / "one.npy").view(np.uint16))
    assert np.mean(got == one) >= 0.97
    assert _normwise(got, one) <= 1e-2
    ref = x0
    for cg, cu, cd in layers:
        ref = q4.ffn_block_gemma4(ref, cg, cu, cd, activation=act)
    assert _normwise(got, ref) <= 1e-2
