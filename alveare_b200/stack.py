"""Decode-time FFN stack: L fused-FFN half-blocks with the layer glue fused in,
optionally tensor-parallel over the intermediate dimension.

This is the decode loop's FFN call site of the reference
(runtime/cpp/src/model.cpp:404, runtime/py/model.py:782-806) moved onto the
GPU: per layer ``x2 = rmsnorm(x)``, ``down = FFN(x2)``,
``x = x + rmsnorm(down)`` (unit norm weights), with every step on the device.
Tensor parallelism splits each FFN's intermediate dimension over the ranks
(the reference's I-split across AIE cores, kernels/ffn_fused/ffn_fused.py:46-60,
lifted to GPUs), and the per-layer partial down projections are summed across
ranks (the reference's host partial sum, runtime/cpp/src/npu.cpp:360-377).
The whole step is a single persistent kernel per GPU (alv_ffn_stack_run) that
streams every layer's weights back to back; with tensor parallelism that
kernel pushes each layer's partial down projection to every peer GPU over
NVLink and meets the peers at a barrier, so no collective runs between
layers.  The per-layer path (fused=False: one kernel per layer, and with
tensor parallelism one NCCL all-reduce of H fp32 values per layer) is kept as
the baseline.  A step is captured once into a CUDA graph and replayed.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .ops import FusedFFNWeight


def tp_slice(I: int, rank: int, world: int) -> tuple[int, int]:
    """Intermediate-dimension slice [begin, end) of `rank` in a `world`-way
    tensor-parallel FFN: contiguous, 32-aligned (whole Q4 blocks of the down
    projection's rows), as the reference splits I over AIE cores
    (kernels/ffn_fused/ffn_fused.py:59-60)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    if I % (32 * world):
        raise ValueError(f"I={I} does not split into {world} slices of whole 32-blocks")
    step = I // world
    return rank * step, (rank + 1) * step


class FFNStack:
    """Resident FFN stack on one GPU (one rank of a tensor-parallel group).

    layers: list of (gate, up, down) packed Q4 buffers in the reference layout
    (torch CUDA uint8 tensors or host numpy arrays).  With ``world > 1`` this
    rank keeps intermediate slice [rank*I/world, (rank+1)*I/world) and
    ``torch.distributed`` (NCCL) must be initialized.
    """

    def __init__(self, H: int, I: int, device: int = 0, rank: int = 0, world: int = 1,
                 activation: str = "gelu", fused: bool = True):
        self.H, self.I, self.device, self.rank, self.world = H, I, device, rank, world
        self.activation = activation
        self.fused = fused
        self.stack_handle = 0
        self.i_begin, self.i_end = tp_slice(I, rank, world)
        self.layers: list[FusedFFNWeight] = []
        dev = torch.device("cuda", device)
        self.x = [torch.zeros(H, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self.down = [torch.zeros(H, dtype=torch.float32, device=dev) for _ in range(2)]
        self.out = torch.zeros(H, dtype=torch.bfloat16, device=dev)
        self.graph = None
        self.stream = torch.cuda.Stream(device=dev)
        self.probe = None

    @property
    def ctx(self):
        return _lib.context(self.device)

    def add_layer(self, gate, up, down) -> None:
        if self.stack_handle:
            raise RuntimeError("FFNStack: layers cannot be added after the first step")
        self.layers.append(FusedFFNWeight(gate, up, down, self.H, self.I, self.activation, device=self.device,
                                          i_begin=self.i_begin, i_end=self.i_end))

    def _stack(self) -> int:
        """Handle of the one-launch stack (created on first use)."""
        if not self.stack_handle:
            ctx = self.ctx
            n = len(self.layers)
            arr = (ctypes.c_uint32 * n)(*[w.handle for w in self.layers])
            h = ctypes.c_uint32()
            ctx.check(ctx.lib.alv_ffn_stack_create(ctx.ptr, arr, n, ctypes.byref(h)), "alv_ffn_stack_create")
            self.stack_handle = h.value
            if self.probe is not None:
                ctx.check(ctx.lib.alv_ffn_stack_set_probe(ctx.ptr, self.stack_handle, self.probe.data_ptr()),
                          "alv_ffn_stack_set_probe")
            if self.world > 1:
                self._connect()
        return self.stack_handle

    def set_probe(self, down_last: torch.Tensor) -> None:
        """Make every later step of the one-launch stack also write the last
        layer's down projection (H fp32, summed over the ranks) into
        `down_last`, a CUDA tensor on this device.  A checking aid: call it
        before the first step (a captured step keeps the pointer)."""
        if self.stack_handle or self.graph is not None:
            raise RuntimeError("FFNStack.set_probe: call before the first step")
        if not (down_last.is_cuda and down_last.dtype == torch.float32 and down_last.numel() >= self.H):
            raise ValueError("down_last must be a float32 CUDA tensor of at least H elements")
        self.probe = down_last

    def _connect(self) -> None:
        """Map every rank's exchange region (collective over the process
        group): export this rank's blob, all-gather, connect, then a barrier
        so that no rank's first launch waits on a peer still connecting."""
        import torch.distributed as dist
        ctx = self.ctx
        blob = (ctypes.c_ubyte * _lib.IPC_BLOB_BYTES)()
        ctx.check(ctx.lib.alv_ffn_stack_exchange(ctx.ptr, self.stack_handle, self.world, blob),
                  "alv_ffn_stack_exchange")
        blobs: list = [None] * self.world
        dist.all_gather_object(blobs, bytes(blob))
        allb = (ctypes.c_ubyte * (_lib.IPC_BLOB_BYTES * self.world)).from_buffer_copy(b"".join(blobs))
        ctx.check(ctx.lib.alv_ffn_stack_connect(ctx.ptr, self.stack_handle, self.rank, self.world, allb),
                  "alv_ffn_stack_connect")
        dist.barrier()

    def weight_bytes(self) -> int:
        """Algorithmic weight bytes of the whole stack (all ranks): 18 B per 32 weights."""
        return len(self.layers) * 3 * self.H * self.I // 32 * 18

    # -- one decode step --------------------------------------------------
    def _enqueue(self, layers_only: bool = False) -> int:
        """Enqueue one step on the current stream; returns kernels launched."""
        ctx = self.ctx
        st = torch.cuda.current_stream(self.device).cuda_stream
        if self.fused:
            ctx.check(ctx.lib.alv_ffn_stack_run(ctx.ptr, self._stack(), 1, self.x[0].data_ptr(),
                                                self.out.data_ptr(), st), "alv_ffn_stack_run")
            return 1
        n = 0
        L = len(self.layers)
        for l, w in enumerate(self.layers):
            x_in, x_out = self.x[l % 2], self.x[(l + 1) % 2]
            down_in = self.down[(l + 1) % 2].data_ptr() if l else None
            ctx.check(ctx.lib.alv_ffn_layer(ctx.ptr, w.handle, 1, x_in.data_ptr(), down_in, x_out.data_ptr(),
                                            self.down[l % 2].data_ptr(), st), "alv_ffn_layer")
            n += 1
            if self.world > 1 and not layers_only:
                torch.distributed.all_reduce(self.down[l % 2])
        if not layers_only:
            ctx.check(ctx.lib.alv_ffn_stack_finalize(ctx.ptr, 1, self.H, self.x[L % 2].data_ptr(),
                                                     self.down[(L - 1) % 2].data_ptr(), self.out.data_ptr(), st),
                      "alv_ffn_stack_finalize")
            n += 1
        return n

    def capture(self, layers_only: bool = False) -> torch.cuda.CUDAGraph:
        """Capture one step (input self.x[0] -> output self.out) into a graph."""
        with torch.cuda.stream(self.stream):
            self._enqueue(layers_only)          # warm-up outside capture
        self.stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self.launches = self._enqueue(layers_only)
        return g

    def prepare(self) -> None:
        if self.graph is None:
            self.graph = self.capture()

    def replay(self) -> None:
        self.graph.replay()

    def forward(self, x_host: torch.Tensor, y_host: torch.Tensor) -> None:
        """Public decode call with host buffers: copy x (bf16, pinned host) in,
        run the stack, copy the new residual stream back into y_host."""
        self.prepare()
        with torch.cuda.stream(self.stream):
            self.x[0].copy_(x_host, non_blocking=True)
            self.graph.replay()
            y_host.copy_(self.out, non_blocking=True)
        self.stream.synchronize()
        self.ctx.sync_status(self.stream.cuda_stream)

    def release(self) -> None:
        """Drop captured graphs (before destroying a process group)."""
        self.graph = None

    def free(self) -> None:
        """Release the stack handle and the layers' device memory.  With
        tensor parallelism this is collective: a barrier first, so no peer
        still runs a step that writes into this rank's exchange region."""
        self.graph = None
        ctx = self.ctx
        if self.stack_handle and self.world > 1 and self.fused:
            import torch.distributed as dist
            torch.cuda.synchronize(self.device)
            dist.barrier()
        if self.stack_handle:
            ctx.check(ctx.lib.alv_weight_destroy(ctx.ptr, self.stack_handle), "alv_weight_destroy")
            self.stack_handle = 0
        for w in self.layers:
            w.free()
        self.layers = []
