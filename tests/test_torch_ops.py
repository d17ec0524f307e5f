"""The t8g custom ops: fake implementations give the kernels' output shapes and dtypes
without a GPU, and a model function using them traces to a graph of t8g ops (what
torch.compile sees); the real kernels never run under tracing."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.proxy_tensor import make_fx


@pytest.fixture(scope="module")
def t8g():
    from thor_int8_gemm_b200 import torch_ops
    return torch_ops


def _fake(mode, shape, dtype):
    with mode:
        return torch.empty(shape, dtype=dtype, device="cuda")


def test_fake_shapes(t8g):
    mode = FakeTensorMode()
    x8 = _fake(mode, (300, 3072), torch.int8)
    w8 = _fake(mode, (9216, 3072), torch.int8)
    xs = _fake(mode, (300,), torch.float32)
    ws = _fake(mode, (9216,), torch.float32)
    xb = _fake(mode, (2, 150, 3072), torch.bfloat16)
    y = _fake(mode, (300, 2 * 1024), torch.bfloat16)
    mod = _fake(mode, (2, 3072), torch.bfloat16)
    with mode:
        out = torch.ops.t8g.gemm_dequant(x8, w8, xs, ws, None, torch.float16)
        assert out.shape == (300, 9216) and out.dtype == torch.float16 and out.device.type == "cuda"
        q, s = torch.ops.t8g.quant_rows(xb.view(300, 3072), "fp8_e4m3")
        assert q.shape == (300, 3072) and q.dtype == torch.float8_e4m3fn and s.shape == (300,)
        o = torch.ops.t8g.int8_linear(xb, w8, ws, None, torch.bfloat16)
        assert o.shape == (2, 150, 9216) and o.dtype == torch.bfloat16
        q, s = torch.ops.t8g.rms_mod_quant(xb.view(300, 3072), mod, mod, None, None, 150, False, 1e-6, "int8")
        assert q.shape == (300, 3072) and q.dtype == torch.int8 and s.dtype == torch.float32
        q, s = torch.ops.t8g.swiglu_quant(y, "int8")
        assert q.shape == (300, 1024) and s.shape == (300,)
        with pytest.raises(Exception):
            torch.ops.t8g.gemm_dequant(x8, _fake(mode, (9216, 1024), torch.int8), xs, ws, None, torch.bfloat16)
        a = torch.ops.t8g.gemm_swiglu(x8, w8, xs, ws, None)
        assert a.shape == (300, 4608) and a.dtype == torch.bfloat16
        q, s = torch.ops.t8g.gemm_swiglu_quant(x8, w8, xs, ws, None, "fp8_e4m3")
        assert q.shape == (300, 4608) and q.dtype == torch.float8_e4m3fn and s.shape == (300,)
        res = _fake(mode, (300, 9216), torch.bfloat16)
        g = torch.ops.t8g.gemm_gated(x8, w8, xs, ws, None, res, _fake(mode, (2, 9216), torch.bfloat16), 150)
        assert g.shape == (300, 9216) and g.dtype == torch.bfloat16


def test_mlp_traces_to_t8g_ops(t8g):
    """norm/mod/quant -> fc1 GEMM -> SwiGLU/quant -> fc2 GEMM traces without running a kernel."""
    def mlp(x, shift, scale, w1, ws1, w2, ws2):
        q, qs = torch.ops.t8g.rms_mod_quant(x, shift, scale, None, None, x.shape[0], False, 1e-6, "int8")
        y = torch.ops.t8g.gemm_dequant(q, w1, qs, ws1, None, torch.bfloat16)
        a, as_ = torch.ops.t8g.swiglu_quant(y, "int8")
        return torch.ops.t8g.gemm_dequant(a, w2, as_, ws2, None, torch.bfloat16)

    mode = FakeTensorMode()
    args = (_fake(mode, (256, 512), torch.bfloat16), _fake(mode, (1, 512), torch.bfloat16),
            _fake(mode, (1, 512), torch.bfloat16), _fake(mode, (2048, 512), torch.int8),
            _fake(mode, (2048,), torch.float32), _fake(mode, (512, 1024), torch.int8),
            _fake(mode, (512,), torch.float32))
    gm = make_fx(mlp, tracing_mode="fake")(*args)
    targets = [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]
    assert targets.count("t8g.gemm_dequant.default") == 2
    assert "t8g.rms_mod_quant.default" in targets and "t8g.swiglu_quant.default" in targets
