"""The DiT-block agent's fused forward on the GPU against the fake ComfyUI block's stock
forward (tests/fake_comfy.py): cluster 1 hands the fp8 QuantizedTensor of the kernel's
tensorwise norm/mod/quant to the linears, cluster 2 the SwiGLU's."""
import importlib
import sys

import numpy as np
import pytest
import torch

from fake_comfy import write_fake_comfy
from oracle import oracle as O
from test_proxy import make_fake_kitchen

pytestmark = pytest.mark.gpu


def _purge(FP):
    for name in list(sys.modules):
        if name == "comfy" or name.startswith("comfy.") or name == "comfy_kitchen" or name.startswith("comfy_kitchen."):
            del sys.modules[name]
    sys.meta_path[:] = [f for f in sys.meta_path if not isinstance(f, FP._Finder)]
    importlib.invalidate_caches()


@pytest.fixture
def patched(tmp_path, monkeypatch, request):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from thor_int8_gemm_b200 import fused_patch as FP
    from thor_int8_gemm_b200 import ops
    make_fake_kitchen(tmp_path, version="0.2.40")
    write_fake_comfy(tmp_path)
    monkeypatch.syspath_prepend(str(tmp_path))
    monkeypatch.setattr(FP, "MODE_FILE", str(tmp_path / "none"))
    monkeypatch.setenv(FP.ENV, request.param)
    _purge(FP)
    FP.install()
    import comfy.ldm.minimax.model as m
    yield m
    assert ops.device_status() == 0
    _purge(FP)


def _problem(m, S=300, d=256, ffn=512):
    blk = m.DiTBlock(d, ffn, device="cuda", seed=3)
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(S, d, generator=g, device="cuda").to(torch.bfloat16)
    t = (torch.randn(2, d, generator=g, device="cuda") * 0.3).to(torch.bfloat16)
    return blk, x, t, [(0, 170, 0), (170, S, 1)]


def _rel(a, b):
    return float((a.detach().float() - b.detach().float()).norm() / b.detach().float().norm())


@pytest.mark.parametrize("patched", ["on", "c1", "c2"], indirect=True)
def test_fused_forward_close_to_stock(patched):
    m = patched
    blk, x, t, segs = _problem(m)
    stock = m.DiTBlock.forward.__wrapped__(blk, x, t, segs, None)
    before = m.CALLS["stock"]
    out = blk(x, t, segs, None)
    assert m.CALLS["stock"] == before                    # the fused path ran
    assert not m.DiTBlock.forward._t8g_runtime.broken
    assert _rel(out, stock) < 0.02


@pytest.mark.parametrize("patched", ["c1"], indirect=True)
def test_cluster1_quantised_input_matches_oracle(patched):
    """The QuantizedTensor cluster 1 builds for norm1 equals the oracle's tensorwise
    norm/mod/quant of the reference (per-segment rows, one fp32 amax)."""
    m = patched
    rt = m.DiTBlock.forward._t8g_runtime
    blk, x, t, segs = _problem(m)
    shift, scale = blk.adaln_proj(t)[:2]
    rows = rt.row_map(segs, x.shape[0], x.device)
    qt = rt.norm_quant(blk.norm1, x, shift, scale, rows)
    xf, sh, sc = (v.float().cpu().numpy() for v in (x, shift, scale))
    w = blk.norm1.weight.detach().float().cpu().numpy()
    s_rows = O.round_bf16(1.0 + sc[rows.cpu().numpy()])
    q_o, scale_o, _, _, _ = O.rms_mod_res_tensorwise(xf, w, s_rows, sh[rows.cpu().numpy()], blk.norm1.eps)
    assert qt.params.scale.item() == scale_o
    np.testing.assert_array_equal(qt.qdata.cpu().view(torch.uint8).numpy(), q_o)


@pytest.mark.parametrize("patched", ["on"], indirect=True)
def test_per_token_rows_equal_segment_rows(patched):
    """A segment given as a tensor of per-token rows (which the reference declines) gives
    the same output as the equivalent integer-row segmentation."""
    m = patched
    blk, x, t, segs = _problem(m)
    S = x.shape[0]
    rows = torch.tensor([0] * 170 + [1] * (S - 170), device="cuda")
    a = blk(x, t, segs, None)
    b = blk(x, t, [(0, S, rows)], None)
    assert not m.DiTBlock.forward._t8g_runtime.broken
    assert torch.equal(a, b)


class _CallCounter:
    """Wraps a comfy linear: attributes pass through, calls are counted."""

    def __init__(self, inner):
        self._inner = inner
        self.calls = 0

    def __getattr__(self, name):
        return getattr(self._inner, name)

    def __call__(self, *a, **k):
        self.calls += 1
        return self._inner(*a, **k)


@pytest.mark.parametrize("patched", ["on", "c2"], indirect=True)
def test_cluster2_fp8_linears_run_on_library_kernels(patched):
    """With fp8 QuantizedTensor weights, cluster 2 runs fc1 + SwiGLU, the per-token fp8
    quantisation of act and fc2 + the gated residual on the library's fp8 GEMMs: comfy's fc1
    and fc2 are never called, and the block's output equals, bit for bit, the same steps
    done one kernel at a time (plain fp8 GEMM -> SwiGLU + per-token fp8 quant -> plain fp8
    GEMM -> the stock gated residual)."""
    from thor_int8_gemm_b200 import ops
    m = patched
    rt = m.DiTBlock.forward._t8g_runtime
    blk, x, t, segs = _problem(m, S=300, d=256, ffn=512)
    blk.mlp.fc1 = _CallCounter(blk.mlp.fc1)
    blk.mlp.fc2 = _CallCounter(blk.mlp.fc2)
    out = blk(x, t, segs, None)
    assert not rt.broken
    assert blk.mlp.fc1.calls == 0 and blk.mlp.fc2.calls == 0

    # the same block, step by step
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = blk.adaln_proj(t)
    rows = rt.row_map(segs, x.shape[0], x.device)
    if rt.c1:
        h1 = rt.norm_quant(blk.norm1, x, shift_msa, scale_msa, rows)
    else:
        h1 = m._mod_scale_shift(blk.norm1(x), shift_msa, scale_msa, segs)
    x1 = m._mod_gate(x, gate_msa, blk.attn(h1), segs)
    if rt.c1:
        h2 = rt.norm_quant(blk.norm2, x1, shift_mlp, scale_mlp, rows)
        a, a_s = h2.qdata, h2.params.scale.float().reshape(1).expand(x.shape[0]).contiguous()
    else:
        h2 = m._mod_scale_shift(blk.norm2(x1), shift_mlp, scale_mlp, segs)
        a, a_s = ops.quant_rows(h2, "fp8_e4m3")
    fc1, fc2 = blk.mlp.fc1._inner, blk.mlp.fc2._inner
    w1 = fc1.weight
    y = ops.gemm_dequant(a, w1.qdata, a_s, w1.params.scale.float().reshape(-1), fc1.bias)
    q3, s3 = ops.swiglu_quant_fc1(y, kind="fp8_e4m3")
    w2 = fc2.weight
    z = ops.gemm_dequant(q3, w2.qdata, s3, w2.params.scale.float().reshape(-1), fc2.bias)
    expect = m._mod_gate(x1, gate_mlp, z, segs)
    assert torch.equal(out, expect)
    # and the fused block stays close to comfy's stock block
    stock = m.DiTBlock.forward.__wrapped__(blk, x, t, segs, None)
    assert _rel(out, stock) < 0.02
