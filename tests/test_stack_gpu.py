"""The one-launch FFN stack (alv_ffn_stack_run) against the per-layer kernel
chain (alv_ffn_layer ... alv_ffn_stack_finalize) and against the CPU oracle's
decode-step FFN half-blocks (runtime/py/model.py:782-806 with unit norms).
The two GPU paths run the same arithmetic in the same order, so they must
agree bit for bit."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from alveare_b200 import FusedFFNWeight, _lib  # noqa: E402
from alveare_b200.stack import FFNStack  # noqa: E402
from oracle import q4  # noqa: E402


def make_layers(H, I, L, seed, scale=0.02):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(L):
        out.append(tuple(q4.quantize_combined(rng.normal(0, scale, shape).astype(np.float32))
                         for shape in ((I, H), (I, H), (H, I))))
    return out


def bf16_tensor(v):
    return torch.from_numpy(np.ascontiguousarray(q4.bf16_bits(v).view(np.int16))).cuda()


def per_layer_chain(ws, x_bits, ntok, H, keep=None):
    """alv_ffn_layer for every layer, then the finalize kernel.  With `keep`
    (a list), append each layer's (x entering its FFN, down) as numpy."""
    ctx = ws[0].ctx
    st = torch.cuda.current_stream().cuda_stream
    xb = [x_bits.clone(), torch.empty_like(x_bits)]
    dn = [torch.empty((ntok, H), dtype=torch.float32, device="cuda") for _ in range(2)]
    L = len(ws)
    for l, w in enumerate(ws):
        down_in = dn[(l + 1) % 2].data_ptr() if l else None
        ctx.check(ctx.lib.alv_ffn_layer(ctx.ptr, w.handle, ntok, xb[l % 2].data_ptr(), down_in,
                                        xb[(l + 1) % 2].data_ptr(), dn[l % 2].data_ptr(), st), "alv_ffn_layer")
        if keep is not None:
            ctx.sync_status()
            keep.append((q4.bits_to_f32(xb[(l + 1) % 2].cpu().numpy().view(np.uint16)), dn[l % 2].cpu().numpy()))
    out = torch.empty_like(x_bits)
    ctx.check(ctx.lib.alv_ffn_stack_finalize(ctx.ptr, ntok, H, xb[L % 2].data_ptr(), dn[(L - 1) % 2].data_ptr(),
                                             out.data_ptr(), st), "alv_ffn_stack_finalize")
    ctx.sync_status()
    return out.cpu().numpy()


def stack_run(ws, x_bits, ntok, probe=None):
    ctx = ws[0].ctx
    arr = (ctypes.c_uint32 * len(ws))(*[w.handle for w in ws])
    h = ctypes.c_uint32()
    ctx.check(ctx.lib.alv_ffn_stack_create(ctx.ptr, arr, len(ws), ctypes.byref(h)), "alv_ffn_stack_create")
    if probe is not None:
        ctx.check(ctx.lib.alv_ffn_stack_set_probe(ctx.ptr, h.value, probe.data_ptr()), "alv_ffn_stack_set_probe")
    out = torch.empty_like(x_bits)
    try:
        for _ in range(2):  # twice: the workspace must be left clean by a launch
            out.zero_()
            ctx.check(ctx.lib.alv_ffn_stack_run(ctx.ptr, h.value, ntok, x_bits.data_ptr(), out.data_ptr(),
                                                torch.cuda.current_stream().cuda_stream), "alv_ffn_stack_run")
            ctx.sync_status()
    finally:
        ctx.check(ctx.lib.alv_weight_destroy(ctx.ptr, h.value), "destroy stack")
    return out.cpu().numpy()


def glue_ref(x_prev, down_prev):
    """x entering a layer: bf16(x + bf16(rmsnorm(bf16(down)))) (model.py:800-806)."""
    return q4.to_bf16(x_prev + q4.rmsnorm_gemma(q4.to_bf16(down_prev)))


@pytest.mark.parametrize("ntok", [1, 2])
@pytest.mark.parametrize("act", ["gelu", "silu"])
def test_stack_equals_per_layer_chain_and_oracle(ntok, act):
    """Bit-exact against the per-layer chain; against the oracle layer by
    layer on the GPU's own layer inputs (fp32 sums in a different order may
    flip a bf16 rounding, and a flip propagates down a chain, so the chained
    output is only held to a normwise bound)."""
    H, I, L = 512, 1536, 4
    layers = make_layers(H, I, L, 900 + ntok)
    ws = [FusedFFNWeight(cg, cu, cd, H, I, act) for cg, cu, cd in layers]
    x0 = q4.to_bf16(np.random.default_rng(7).normal(0, 1, (ntok, H)).astype(np.float32))
    xt = bf16_tensor(x0)
    steps = []
    chain = per_layer_chain(ws, xt, ntok, H, keep=steps)
    fused = stack_run(ws, xt, ntok)
    assert np.array_equal(chain, fused)
    for t in range(ntok):
        x_prev, d_prev = x0[t], None
        for l, (cg, cu, cd) in enumerate(layers):
            x_gpu, d_gpu = steps[l][0][t], steps[l][1][t]
            x_ref = x_prev if d_prev is None else glue_ref(x_prev, d_prev)
            assert np.mean(x_gpu == x_ref) >= 0.99
            y_ref, _, _, _ = q4.ffn(cg, cu, cd, q4.rmsnorm_gemma(x_gpu), act)
            assert float(np.max(np.abs(d_gpu - y_ref)) / np.max(np.abs(y_ref))) <= 1e-3
            x_prev, d_prev = x_gpu, d_gpu
        out_ref = glue_ref(x_prev, d_prev)
        got = q4.bits_to_f32(fused[t].view(np.uint16))
        assert np.mean(got == out_ref) >= 0.99
        ref = x0[t]
        for cg, cu, cd in layers:
            ref = q4.ffn_block_gemma4(ref, cg, cu, cd, activation=act)
        assert float(np.max(np.abs(got - ref)) / np.max(np.abs(ref))) <= 1e-2
    for w in ws:
        w.free()


def test_stack_config4_shape_each_layer_against_oracle():
    """BASELINE config 4 layer shape (H=3840, I=15360: a down K of 15360 and
    240 down row tiles split unevenly over the SMs), two layers.  Each
    layer's fp32 down projection is checked against the CPU oracle
    (q4.ffn on the rmsnorm of the GPU's own layer input, runtime/py/model.py:
    782-806) at the north-star 1e-3, the layer inputs against the oracle's
    glue, and the one-launch stack against the per-layer chain bit for bit
    (output and the last layer's down projection through the stack probe)."""
    H, I, L = 3840, 15360, 2
    layers = make_layers(H, I, L, 77)
    ws = [FusedFFNWeight(cg, cu, cd, H, I, "gelu") for cg, cu, cd in layers]
    x0 = q4.to_bf16(np.random.default_rng(8).normal(0, 1, (1, H)).astype(np.float32))
    xt = bf16_tensor(x0)
    steps = []
    chain = per_layer_chain(ws, xt, 1, H, keep=steps)
    probe = torch.full((1, H), float("nan"), dtype=torch.float32, device="cuda")
    assert np.array_equal(chain, stack_run(ws, xt, 1, probe=probe))
    assert np.array_equal(probe.cpu().numpy(), steps[-1][1])
    x_prev, d_prev = x0[0], None
    for l, (cg, cu, cd) in enumerate(layers):
        x_gpu, d_gpu = steps[l][0][0], steps[l][1][0]
        x_ref = x_prev if d_prev is None else glue_ref(x_prev, d_prev)
        assert np.mean(x_gpu == x_ref) >= 0.99
        y_ref, _, _, _ = q4.ffn(cg, cu, cd, q4.rmsnorm_gemma(x_gpu), "gelu")
        assert float(np.max(np.abs(d_gpu - y_ref)) / np.max(np.abs(y_ref))) <= 1e-3
        x_prev, d_prev = x_gpu, d_gpu
    for w in ws:
        w.free()


def test_stack_generic_dequant_layers():
    """Layers repacked for the generic dequant path run through the generic
    instantiation of the stack kernel."""
    H, I, L = 256, 512, 3
    layers = make_layers(H, I, L, 31)
    for cg, cu, cd in layers:
        v = cd.reshape(H, I // 32, 20)
        v[0, 0, 16:18] = [0x00, 0x01]   # 2^-125
        v[1, 0, 16:18] = [0x80, 0x40]   # 4.0
    ws = [FusedFFNWeight(cg, cu, cd, H, I, "gelu") for cg, cu, cd in layers]
    assert all(w.info()[3] == 0 for w in ws)
    x0 = q4.to_bf16(np.random.default_rng(9).normal(0, 1, (1, H)).astype(np.float32))
    xt = bf16_tensor(x0)
    assert np.array_equal(per_layer_chain(ws, xt, 1, H), stack_run(ws, xt, 1))
    for w in ws:
        w.free()


def test_stack_rejects_mixed_layers_and_protects_its_layers():
    H, I = 256, 512
    (a,) = make_layers(H, I, 1, 40)
    (b,) = make_layers(H, I, 1, 41)
    v = b[2].reshape(H, I // 32, 20)
    v[0, 0, 16:18] = [0x00, 0x01]
    v[1, 0, 16:18] = [0x80, 0x40]
    wa = FusedFFNWeight(*a, H, I, "gelu")
    wb = FusedFFNWeight(*b, H, I, "gelu")
    ctx = wa.ctx
    arr = (ctypes.c_uint32 * 2)(wa.handle, wb.handle)
    h = ctypes.c_uint32()
    assert ctx.lib.alv_ffn_stack_create(ctx.ptr, arr, 2, ctypes.byref(h)) == 3  # ALV_ERR_SHAPE
    arr1 = (ctypes.c_uint32 * 1)(wa.handle)
    assert ctx.lib.alv_ffn_stack_create(ctx.ptr, arr1, 1, ctypes.byref(h)) == 0
    assert ctx.lib.alv_weight_destroy(ctx.ptr, wa.handle) == 1  # still a layer of the stack
    assert ctx.lib.alv_ffn_stack_run(ctx.ptr, h.value, 5, 0, 0, None) == 1  # null buffers
    assert ctx.lib.alv_weight_destroy(ctx.ptr, h.value) == 0
    wa.free()
    wb.free()


def test_ffnstack_fused_and_per_layer_agree():
    """The public FFNStack API: one-launch step vs per-layer kernels, both
    captured in a CUDA graph, host buffers in and out."""
    H, I, L = 512, 1024, 3
    layers = make_layers(H, I, L, 55)
    outs = []
    for fused in (True, False):
        st = FFNStack(H, I, fused=fused)
        for cg, cu, cd in layers:
            st.add_layer(cg, cu, cd)
        x = torch.from_numpy(q4.bf16_bits(q4.to_bf16(
            np.random.default_rng(3).normal(0, 1, H).astype(np.float32))).view(np.int16)).view(torch.bfloat16)
        y = torch.empty(H, dtype=torch.bfloat16).pin_memory()
        st.forward(x.pin_memory(), y)
        outs.append(y.view(torch.int16).numpy().copy())
        assert st.launches == (1 if fused else L + 1)
        st.free()
    assert np.array_equal(outs[0], outs[1])


def test_tp_stack_connect_rejects_ranks_on_one_gpu():
    """Two I-slice stacks in one process on one GPU: connect refuses (ranks of
    the tensor-parallel stack kernel wait for one another), and a slice stack
    that is not connected refuses to run.  No kernel is launched."""
    H, I = 256, 1024
    (layer,) = make_layers(H, I, 1, 60)
    ws = [FusedFFNWeight(*layer, H, I, "gelu", i_begin=b, i_end=b + I // 2) for b in (0, I // 2)]
    ctx = ws[0].ctx
    hs, blobs = [], b""
    for w in ws:
        arr = (ctypes.c_uint32 * 1)(w.handle)
        h = ctypes.c_uint32()
        ctx.check(ctx.lib.alv_ffn_stack_create(ctx.ptr, arr, 1, ctypes.byref(h)), "alv_ffn_stack_create")
        hs.append(h.value)
    x = torch.zeros(H, dtype=torch.int16, device="cuda")
    assert ctx.lib.alv_ffn_stack_run(ctx.ptr, hs[0], 1, x.data_ptr(), x.data_ptr(), None) == 1  # not connected
    for h in hs:
        blob = (ctypes.c_ubyte * _lib.IPC_BLOB_BYTES)()
        ctx.check(ctx.lib.alv_ffn_stack_exchange(ctx.ptr, h, 2, blob), "alv_ffn_stack_exchange")
        blobs += bytes(blob)
    allb = (ctypes.c_ubyte * len(blobs)).from_buffer_copy(blobs)
    assert ctx.lib.alv_ffn_stack_connect(ctx.ptr, hs[0], 0, 2, allb) == 6  # ALV_ERR_UNSUPPORTED
    assert b"same GPU" in ctx.lib.alv_last_error(ctx.ptr)
    assert ctx.lib.alv_ffn_stack_connect(ctx.ptr, hs[1], 0, 2, allb) == 1  # blobs[0] is not its blob
    for h in hs:
        ctx.check(ctx.lib.alv_weight_destroy(ctx.ptr, h), "destroy stack")
    for w in ws:
        w.free()
