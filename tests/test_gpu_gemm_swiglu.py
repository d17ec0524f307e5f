"""The fc1 GEMM with the SwiGLU fused into its epilogue (t8g_gemm_i8_swiglu) against the
unfused pipeline (plain GEMM -> bf16 [M, 2F] -> SwiGLU kernel) and the oracle, bit for bit
(both use the exact sigmoid table)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from thor_int8_gemm_b200 import ops as _ops
    yield _ops
    assert _ops.device_status() == 0


def bits16(t):
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _problem(ops, M, K, F, kind, bias, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(2 * F, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    xq, xs = ops.quant_rows(x, kind)
    wq, ws = ops.quant_rows(w, kind)
    b = (torch.randn(2 * F, generator=g, device="cuda") * 0.5).to(torch.bfloat16) if bias else None
    return xq, xs, wq, ws, b


@pytest.mark.parametrize("M,K,F,bias", [(300, 3072, 1024, True), (129, 256, 128, False), (1, 512, 256, True),
                                        (2048, 3072, 12288, True), (777, 1024, 384, False)])
def test_fused_swiglu_equals_unfused_int8(ops, M, K, F, bias):
    xq, xs, wq, ws, b = _problem(ops, M, K, F, "int8", bias, M + F)
    y = ops.gemm_dequant(xq, wq, xs, ws, b)
    q_ref, qs_ref, act_ref = ops.swiglu_quant_fc1(y, kind="int8", return_act=True)
    il = ops.interleave_gate_up
    act = ops.gemm_swiglu(xq, il(wq), xs, il(ws), None if b is None else il(b))
    assert torch.equal(act, act_ref)
    q, qs = ops.quant_rows(act, "int8")
    assert torch.equal(q, q_ref) and torch.equal(qs, qs_ref)
    # and the unfused pipeline itself against the oracle on a few rows
    rows = np.unique(np.array([0, M // 2, M - 1]))
    y_o = O.gemm_i8_dequant(xq[rows].cpu().numpy(), wq.cpu().numpy(), xs[rows].cpu().numpy(), ws.cpu().numpy(),
                            None if b is None else b.float().cpu().numpy(), "bf16")
    np.testing.assert_array_equal(bits16(y[rows]), y_o)
    yf = O.bf16_to_f32(y_o)
    q_o, qs_o, act_o = O.swiglu_quant_per_token(yf[:, :F], yf[:, F:], O.QUANT_INT8)
    np.testing.assert_array_equal(bits16(act[rows]), act_o)
    np.testing.assert_array_equal(qs[rows].cpu().numpy(), qs_o)
    np.testing.assert_array_equal(q[rows].cpu().numpy(), q_o)


def test_fused_swiglu_fp8(ops):
    M, K, F = 400, 1024, 512
    xq, xs, wq, ws, b = _problem(ops, M, K, F, "fp8_e4m3", True, 5)
    y = ops.gemm_dequant(xq, wq, xs, ws, b)
    _, _, act_ref = ops.swiglu_quant_fc1(y, kind="fp8_e4m3", return_act=True)
    il = ops.interleave_gate_up
    act = ops.gemm_swiglu(xq, il(wq), xs, il(ws), il(b))
    assert torch.equal(act, act_ref)


def test_fused_swiglu_scalar_weight_scale_and_strided_out(ops):
    M, K, F = 260, 512, 256
    xq, xs, wq, _, b = _problem(ops, M, K, F, "int8", True, 9)
    ws1 = torch.full((1,), 3e-3, device="cuda")
    y = ops.gemm_dequant(xq, wq, xs, ws1, b)
    _, _, act_ref = ops.swiglu_quant_fc1(y, kind="int8", return_act=True)
    buf = torch.zeros(M, F + 64, dtype=torch.bfloat16, device="cuda")
    il = ops.interleave_gate_up
    act = ops.gemm_swiglu(xq, il(wq), xs, ws1, il(b), out=buf[:, 32:32 + F])
    assert torch.equal(act, act_ref)
    assert torch.count_nonzero(buf[:, :32]) == 0 and torch.count_nonzero(buf[:, 32 + F:]) == 0


def test_fused_swiglu_rejects(ops):
    xq, xs, wq, ws, b = _problem(ops, 64, 256, 128, "int8", True, 1)
    with pytest.raises(ValueError):
        ops.gemm_swiglu(xq, wq[:192], xs, ws[:192])           # 2F not a multiple of 256
    with pytest.raises(TypeError):
        ops.gemm_swiglu(xq, wq, xs, ws, b.float())            # bias must be bf16


@pytest.mark.parametrize("kind,in_kind", [("int8", "int8"), ("fp8_e4m3", "int8"), ("fp8_e4m3", "fp8_e4m3")])
@pytest.mark.parametrize("M,K,F", [(300, 1024, 384), (129, 256, 128), (2048, 3072, 12288)])
def test_swiglu_quant_entry_equals_quant_of_fused_act(ops, kind, in_kind, M, K, F):
    """fc1 + SwiGLU + per-token quant in one call (the epilogue's row maxima, then a streaming
    quantiser) gives act, the scales and the codes of gemm_swiglu followed by quant_rows,
    bit for bit -- including rows past the last full 128-row block."""
    xq, xs, wq, ws, b = _problem(ops, M, K, F, in_kind, True, M * 3 + F)
    il = ops.interleave_gate_up
    act_ref = ops.gemm_swiglu(xq, il(wq), xs, il(ws), il(b))
    q_ref, qs_ref = ops.quant_rows(act_ref, kind)
    q, qs, act = ops.gemm_swiglu_quant(xq, il(wq), xs, il(ws), il(b), kind=kind)
    assert torch.equal(act, act_ref)
    assert torch.equal(qs, qs_ref)
    assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8))
