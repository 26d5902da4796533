"""ffn_fused on the B200 vs the CPU oracle (restated runtime/py/model.py FFN
path with the reference's bf16 rounding points).  Tolerance (north star):
max|y - y_ref| / max|y_ref| <= 1e-3 on fp32 outputs."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from alveare_b200 import FusedFFNWeight, ffn_fused_npu, pack_ffn_fused_weights  # noqa: E402
from alveare_b200 import _lib  # noqa: E402
from oracle import q4  # noqa: E402

TOL = 1e-3


def normwise(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def make_ffn(H, I, seed, scale=0.02):
    rng = np.random.default_rng(seed)
    cg = q4.quantize_combined(rng.normal(0, scale, (I, H)).astype(np.float32))
    cu = q4.quantize_combined(rng.normal(0, scale, (I, H)).astype(np.float32))
    cd = q4.quantize_combined(rng.normal(0, scale, (H, I)).astype(np.float32))
    x = rng.normal(0, 1, H).astype(np.float32)
    return cg, cu, cd, x


def run_ffn(fw, x, ntok=1):
    ctx = fw.ctx
    xt = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    y = torch.empty((ntok, fw.H), dtype=torch.float32, device="cuda")
    rc = ctx.lib.alv_ffn(ctx.ptr, fw.handle, ntok, xt.data_ptr(), _lib.F32, y.data_ptr(), _lib.F32,
                         torch.cuda.current_stream().cuda_stream)
    ctx.check(rc, "alv_ffn")
    ctx.sync_status()
    return y.cpu().numpy()


@pytest.mark.parametrize("act", ["gelu", "silu"])
def test_ffn_reference_golden(golden_dir, act):
    g = np.load(os.path.join(golden_dir, "ffn_256x512.npz"))
    fw = pack_ffn_fused_weights(g["gate_c"], g["up_c"], g["down_c"], 256, 512, 32, 256, activation=act)
    Y = torch.zeros((1, 256), dtype=torch.float32, device="cuda")
    ffn_fused_npu(fw, torch.from_numpy(g["x"]).cuda(), Y, H=256, I=512, m_I=32, k_tile=256, activation=act)
    fw.ctx.sync_status()
    e = normwise(Y[0].cpu().numpy(), g[f"y_{act}32"])
    assert e <= TOL, e


def test_ffn_activation_switch_per_call(golden_dir):
    g = np.load(os.path.join(golden_dir, "ffn_256x512.npz"))
    fw = pack_ffn_fused_weights(g["gate_c"], g["up_c"], g["down_c"], 256, 512)
    for act in ("silu", "gelu", "silu"):
        Y = torch.zeros((4, 256), dtype=torch.float32, device="cuda")  # (n_cores, H) partials
        ffn_fused_npu(fw, torch.from_numpy(g["x"]).cuda(), Y, H=256, I=512, activation=act)
        fw.ctx.sync_status()
        assert normwise(Y.sum(0).cpu().numpy(), g[f"y_{act}32"]) <= TOL


def test_ffn_gemma3_1b_config2():
    """hidden 1152, intermediate 6912, GeGLU."""
    cg, cu, cd, x = make_ffn(1152, 6912, 0)
    ref, act, _, _ = q4.ffn(cg, cu, cd, x, "gelu")
    fw = FusedFFNWeight(cg, cu, cd, 1152, 6912, "gelu")
    y = run_ffn(fw, x)[0]
    e = normwise(y, ref)
    assert e <= TOL, e
    np.testing.assert_array_equal(run_ffn(fw, x)[0], y)  # deterministic


@pytest.mark.parametrize("H,I,act", [(32, 32, "gelu"), (96, 160, "silu"), (2048, 8192, "silu"),
                                     (3840, 1536, "gelu")])
def test_ffn_shapes(H, I, act):
    cg, cu, cd, x = make_ffn(H, I, H + I)
    ref, _, _, _ = q4.ffn(cg, cu, cd, x, act)
    fw = FusedFFNWeight(cg, cu, cd, H, I, act)
    assert normwise(run_ffn(fw, x)[0], ref) <= TOL


@pytest.mark.parametrize("ntok", [2, 3, 8])
def test_ffn_multi_token(ntok):
    H, I = 512, 1024
    cg, cu, cd, _ = make_ffn(H, I, 40 + ntok)
    X = np.random.default_rng(ntok).normal(0, 1, (ntok, H)).astype(np.float32)
    ref, _, _, _ = q4.ffn(cg, cu, cd, X, "silu")
    fw = FusedFFNWeight(cg, cu, cd, H, I, "silu")
    assert normwise(run_ffn(fw, X, ntok), ref) <= TOL


@pytest.mark.parametrize("P", [2, 4, 8])
def test_ffn_tensor_parallel_slices_sum_to_full(P):
    """The intermediate-dim split of the north star: partial down-projections
    of P slices sum to the full FFN (what the all-reduce computes)."""
    H, I = 768, 3072
    cg, cu, cd, x = make_ffn(H, I, 77)
    ref, _, _, _ = q4.ffn(cg, cu, cd, x, "gelu")
    step = I // P
    acc = np.zeros(H, np.float64)
    for p in range(P):
        fw = FusedFFNWeight(cg, cu, cd, H, I, "gelu", i_begin=p * step, i_end=(p + 1) * step)
        acc += run_ffn(fw, x)[0]
        fw.free()
    assert normwise(acc, ref) <= TOL


def test_ffn_host_buffers():
    H, I = 256, 768
    cg, cu, cd, x = make_ffn(H, I, 9)
    ref, _, _, _ = q4.ffn(cg, cu, cd, x, "gelu")
    fw = FusedFFNWeight(cg, cu, cd, H, I, "gelu")
    Y = np.zeros((1, H), np.float32)
    ffn_fused_npu(fw, x, Y, H=H, I=I, activation="gelu")
    assert normwise(Y[0], ref) <= TOL


def test_ffn_layer_stack_matches_oracle():
    """Three FFN half-blocks with the rmsnorm/residual glue fused in
    (model.py:782-806 with unit norms), chained like a decode step."""
    H, I, L = 512, 1536, 3
    layers = [make_ffn(H, I, 500 + l)[:3] for l in range(L)]
    x0 = q4.to_bf16(np.random.default_rng(1).normal(0, 1, H).astype(np.float32))
    ref = x0
    for cg, cu, cd in layers:
        ref = q4.ffn_block_gemma4(ref, cg, cu, cd)
    ws = [FusedFFNWeight(cg, cu, cd, H, I, "gelu") for cg, cu, cd in layers]
    ctx = ws[0].ctx
    st = torch.cuda.current_stream().cuda_stream
    xb = [torch.from_numpy(q4.bf16_bits(x0).view(np.int16)).cuda(), torch.empty(H, dtype=torch.int16, device="cuda")]
    dn = [torch.empty(H, dtype=torch.float32, device="cuda") for _ in range(2)]
    for l, w in enumerate(ws):
        x_in = xb[l % 2]
        x_out = xb[(l + 1) % 2]
        down_in = dn[(l + 1) % 2].data_ptr() if l else None
        ctx.check(ctx.lib.alv_ffn_layer(ctx.ptr, w.handle, 1, x_in.data_ptr(), down_in,
                                        x_out.data_ptr(), dn[l % 2].data_ptr(), st), "alv_ffn_layer")
    final = torch.empty(H, dtype=torch.int16, device="cuda")
    ctx.check(ctx.lib.alv_ffn_stack_finalize(ctx.ptr, 1, H, xb[L % 2].data_ptr(), dn[(L - 1) % 2].data_ptr(),
                                             final.data_ptr(), st), "finalize")
    ctx.sync_status()
    got = q4.bits_to_f32(final.cpu().numpy().view(np.uint16))
    # bf16 residual stream: a bf16 rounding flipped by a different fp32 sum
    # order propagates down the chain, so only a normwise bound holds here
    # (layer-by-layer parity: tests/test_stack_gpu.py)
    assert normwise(got, ref) <= 1e-2


def test_ffn_generic_dequant_path_shared_by_both_matrices():
    """A down matrix whose scales span more than the fast window forces the
    generic path for gate/up too (one kernel dequantizes both)."""
    H, I = 256, 512
    cg, cu, cd, x = make_ffn(H, I, 11)
    v = cd.reshape(H, I // 32, 20)
    v[0, 0, 16:18] = [0x00, 0x01]   # 2^-125
    v[1, 0, 16:18] = [0x80, 0x40]   # 4.0
    ref, _, _, _ = q4.ffn(cg, cu, cd, x, "gelu")
    fw = FusedFFNWeight(cg, cu, cd, H, I, "gelu")
    info = fw.info()
    assert info[3] == 0 and info[4] == 0
    assert normwise(run_ffn(fw, x)[0], ref) <= TOL


def test_ffn_fused_npu_batch_of_tokens():
    """ffn_fused_npu with a (B, H) batch: y of every token lands in row 0 of
    Y_partial (n_rows, B, H), the other rows are zeroed."""
    H, I, B = 512, 1024, 4
    cg, cu, cd, _ = make_ffn(H, I, 77)
    X = np.random.default_rng(78).normal(0, 1, (B, H)).astype(np.float32)
    ref, _, _, _ = q4.ffn(cg, cu, cd, X, "gelu")
    fw = pack_ffn_fused_weights(cg, cu, cd, H, I)
    Yp = torch.full((2, B, H), 7.0, dtype=torch.float32, device="cuda")
    ffn_fused_npu(fw, torch.from_numpy(X).cuda(), Yp, H=H, I=I, activation="gelu")
    fw.ctx.sync_status()
    assert normwise(Yp.sum(0).cpu().numpy(), ref) <= TOL
    assert torch.count_nonzero(Yp[1]) == 0
    fw.free()
