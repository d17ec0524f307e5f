"""The t8g custom ops under torch.compile (fullgraph, aot_eager backend) give the same bits
as the eager library calls, and the traced graph runs the CUDA kernels."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from thor_int8_gemm_b200 import ops, torch_ops
    yield ops, torch_ops
    assert ops.device_status() == 0


def test_compiled_mlp_matches_eager(mods):
    ops, _ = mods
    g = torch.Generator(device="cuda").manual_seed(3)
    T, D, F = 512, 1024, 2048
    x = torch.randn(T, D, generator=g, device="cuda").to(torch.bfloat16)
    shift = (torch.randn(1, D, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    scale = (torch.randn(1, D, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    w1, ws1 = ops.quant_rows((torch.randn(2 * F, D, generator=g, device="cuda") * 0.02).to(torch.bfloat16), "int8")
    w2, ws2 = ops.quant_rows((torch.randn(D, F, generator=g, device="cuda") * 0.02).to(torch.bfloat16), "int8")

    def mlp(x, shift, scale, w1, ws1, w2, ws2):
        q, qs = torch.ops.t8g.rms_mod_quant(x, shift, scale, None, None, x.shape[0], False, 1e-6, "int8")
        y = torch.ops.t8g.gemm_dequant(q, w1, qs, ws1, None, torch.bfloat16)
        a, as_ = torch.ops.t8g.swiglu_quant(y, "int8")
        return torch.ops.t8g.gemm_dequant(a, w2, as_, ws2, None, torch.bfloat16)

    def eager(x, shift, scale, w1, ws1, w2, ws2):
        q, qs = ops.rms_mod_quant(x, shift, scale, rows_per_mod=x.shape[0], eps=1e-6, kind="int8")
        y = ops.gemm_dequant(q, w1, qs, ws1, None)
        a, as_ = ops.swiglu_quant_fc1(y, kind="int8")
        return ops.gemm_dequant(a, w2, as_, ws2, None)

    args = (x, shift, scale, w1, ws1, w2, ws2)
    compiled = torch.compile(mlp, backend="aot_eager", fullgraph=True)
    assert torch.equal(compiled(*args), eager(*args))


def test_int8_linear_op(mods):
    ops, _ = mods
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(3, 100, 768, generator=g, device="cuda").to(torch.bfloat16)
    w, ws = ops.quant_rows((torch.randn(1536, 768, generator=g, device="cuda") * 0.02).to(torch.bfloat16), "int8")
    bias = (torch.randn(1536, generator=g, device="cuda") * 0.01).to(torch.bfloat16)
    out = torch.ops.t8g.int8_linear(x, w, ws, bias, torch.bfloat16)
    xq, xs = ops.quant_rows(x.reshape(300, 768), "int8")
    ref = ops.gemm_dequant(xq, w, xs, ws, bias).reshape(3, 100, 1536)
    assert torch.equal(out, ref)


def test_compiled_fused_block_tail_matches_eager(mods):
    """fc1 with the SwiGLU epilogue and fc2 with the gated residual, compiled, against the
    eager library calls."""
    ops, _ = mods
    g = torch.Generator(device="cuda").manual_seed(5)
    T, D, F = 512, 1024, 2048
    x = torch.randn(T, D, generator=g, device="cuda").to(torch.bfloat16)
    gate = (torch.randn(2, D, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    q, qs = ops.quant_rows(x, "int8")
    w1, ws1 = ops.quant_rows((torch.randn(2 * F, D, generator=g, device="cuda") * 0.02).to(torch.bfloat16), "int8")
    w2, ws2 = ops.quant_rows((torch.randn(D, F, generator=g, device="cuda") * 0.02).to(torch.bfloat16), "int8")
    il = ops.interleave_gate_up
    w1i, ws1i = il(w1), il(ws1)

    def tail(q, qs, w1i, ws1i, w2, ws2, x, gate):
        act = torch.ops.t8g.gemm_swiglu(q, w1i, qs, ws1i, None)
        a, as_ = torch.ops.t8g.quant_rows(act, "int8")
        return torch.ops.t8g.gemm_gated(a, w2, as_, ws2, None, x, gate, T // 2)

    def eager(q, qs, w1i, ws1i, w2, ws2, x, gate):
        a, as_ = ops.quant_rows(ops.gemm_swiglu(q, w1i, qs, ws1i), "int8")
        return ops.gemm_gated(a, w2, as_, ws2, None, x, gate, rows_per_gate=T // 2)

    args = (q, qs, w1i, ws1i, w2, ws2, x, gate)
    compiled = torch.compile(tail, backend="aot_eager", fullgraph=True)
    assert torch.equal(compiled(*args), eager(*args))

    def tail_q(q, qs, w1i, ws1i, w2, ws2, x, gate):
        a, as_ = torch.ops.t8g.gemm_swiglu_quant(q, w1i, qs, ws1i, None, "int8")
        return torch.ops.t8g.gemm_gated(a, w2, as_, ws2, None, x, gate, T // 2)

    compiled_q = torch.compile(tail_q, backend="aot_eager", fullgraph=True)
    assert torch.equal(compiled_q(*args), eager(*args))
