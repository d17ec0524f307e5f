"""The GEMM with the DiT block's gated residual in its epilogue (t8g_gemm_i8_gated /
t8g_gemm_fp8_gated) against the unfused pipeline (plain GEMM -> bf16 y -> torch's bf16
`res + gate * y`) and against the oracle."""
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


def _problem(ops, M, N, K, kind, bias, n_gate, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    xq, xs = ops.quant_rows(x, kind)
    wq, ws = ops.quant_rows(w, kind)
    b = (torch.randn(N, generator=g, device="cuda") * 0.5).to(torch.bfloat16) if bias else None
    res = torch.randn(M, N, generator=g, device="cuda").to(torch.bfloat16)
    gate = (torch.randn(n_gate, N, generator=g, device="cuda") * 0.3).to(torch.bfloat16)
    return xq, xs, wq, ws, b, res, gate


def _stock(ops, xq, wq, xs, ws, b, res, gate_rows):
    y = ops.gemm_dequant(xq, wq, xs, ws, b)
    return res + gate_rows * y, y   # torch bf16 eager: bf16(gate * y), then bf16(res + t)


@pytest.mark.parametrize("M,N,K,bias,n_gate", [(300, 3072, 512, True, 2), (2048, 3072, 3072, True, 2),
                                               (129, 200, 256, False, 1), (64, 1000, 1024, True, 4),
                                               (1000, 9216, 384, True, 5), (4096, 520, 128, False, 2)])
def test_gated_equals_stock_int8(ops, M, N, K, bias, n_gate):
    xq, xs, wq, ws, b, res, gate = _problem(ops, M, N, K, "int8", bias, n_gate, M + N)
    T = -(-M // n_gate)   # ceil: the last gate row covers the ragged rest
    grow = torch.arange(M, device="cuda") // T
    ref, y = _stock(ops, xq, wq, xs, ws, b, res, gate[grow])
    out = ops.gemm_gated(xq, wq, xs, ws, b, res, gate, rows_per_gate=T)
    assert torch.equal(out, ref)
    # against the oracle on a few rows
    rows = np.unique(np.array([0, 1, M // 2, M - 1]))
    y_o = O.gemm_i8_dequant(xq[rows].cpu().numpy(), wq.cpu().numpy(), xs[rows].cpu().numpy(), ws.cpu().numpy(),
                            None if b is None else b.float().cpu().numpy(), "bf16")
    np.testing.assert_array_equal(bits16(y[rows]), y_o)
    o_o = O.gated_residual(res[rows].float().cpu().numpy(), gate[grow[rows]].float().cpu().numpy(), O.bf16_to_f32(y_o))
    np.testing.assert_array_equal(bits16(out[rows]), o_o)


def test_gated_in_place_and_gate_index(ops):
    M, N, K, G = 777, 3072, 1024, 6
    xq, xs, wq, ws, b, res, gate = _problem(ops, M, N, K, "int8", True, G, 11)
    idx = torch.randint(0, G, (M,), device="cuda", dtype=torch.int32)
    ref, _ = _stock(ops, xq, wq, xs, ws, b, res, gate[idx.long()])
    buf = res.clone()
    out = ops.gemm_gated(xq, wq, xs, ws, b, buf, gate, gate_index=idx, out=buf)
    assert out.data_ptr() == buf.data_ptr()
    assert torch.equal(buf, ref)


def test_gated_strided_rows(ops):
    # res and out as column slices of wider matrices (row strides > N)
    M, N, K = 512, 1024, 512
    xq, xs, wq, ws, b, res, gate = _problem(ops, M, N, K, "int8", True, 2, 3)
    wide_res = torch.zeros(M, N + 64, device="cuda", dtype=torch.bfloat16)
    wide_res[:, 32:32 + N] = res
    wide_out = torch.full((M, N + 128), 7.0, device="cuda", dtype=torch.bfloat16)
    out = ops.gemm_gated(xq, wq, xs, ws, b, wide_res[:, 32:32 + N], gate, rows_per_gate=M // 2,
                         out=wide_out[:, 64:64 + N])
    ref, _ = _stock(ops, xq, wq, xs, ws, b, res, gate[torch.arange(M, device="cuda") // (M // 2)])
    assert torch.equal(out, ref)
    assert torch.all(wide_out[:, :64] == 7.0) and torch.all(wide_out[:, 64 + N:] == 7.0)


def test_gated_fp8(ops):
    M, N, K = 600, 3072, 1024
    xq, xs, wq, ws, b, res, gate = _problem(ops, M, N, K, "fp8_e4m3", True, 2, 21)
    grow = torch.arange(M, device="cuda") // (M // 2)
    ref, _ = _stock(ops, xq, wq, xs, ws, b, res, gate[grow])
    out = ops.gemm_gated(xq, wq, xs, ws, b, res, gate, rows_per_gate=M // 2)
    # the same fp8 GEMM kernel family computes y: identical accumulation order
    assert torch.equal(out, ref)


def test_gated_repeat_deterministic(ops):
    M, N, K = 1024, 3072, 3072
    xq, xs, wq, ws, b, res, gate = _problem(ops, M, N, K, "int8", True, 2, 8)
    a = ops.gemm_gated(xq, wq, xs, ws, b, res, gate)
    for _ in range(3):
        assert torch.equal(ops.gemm_gated(xq, wq, xs, ws, b, res, gate), a)


def test_gated_rejects_bad_arguments(ops):
    M, N, K = 256, 3072, 256
    xq, xs, wq, ws, b, res, gate = _problem(ops, M, N, K, "int8", True, 2, 1)
    with pytest.raises(ValueError):
        ops.gemm_gated(xq, wq, xs, ws, b, res, gate, rows_per_gate=64)      # rows past the 2 gate rows
    with pytest.raises(ValueError):
        ops.gemm_gated(xq, wq, xs, ws, b, res[:, :1024], gate)              # res shape
    from thor_int8_gemm_b200 import _lib
    overlap = torch.empty(M + 1, N, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(_lib.T8GError):
        ops.gemm_gated(xq, wq, xs, ws, b, overlap[:M], gate, out=overlap[1:])   # out overlaps res
