"""The GEMMs at every shape the benchmark times, against the oracle on sampled rows.

Inputs follow the workload description: activations bf16 N(0, 1) with 1 % of the channels
scaled x20, quantised per token by the library's own quantiser (t8g_quant_rows, itself
checked against the oracle on the sampled rows); weights N(0, 0.02) quantised per output
channel; bias bf16 N(0, 0.01); bf16 output.  Every shape is checked on ~70 rows that
include the first and last row of the first tiles and of the matrix:

* int8, bit for bit: K = 3072 x N in {3072, 9216} x M in {8192, 32768, 112640} (the
  attention-projection sweep), the MLP's up-GEMM 32768 x 24576 x 3072 (plain and with
  the SwiGLU epilogue, whose act is checked too) and its down-GEMM 32768 x 3072 x 12288;
* fp8 e4m3, within the oracle's fp32-accumulation bound (fp8_gemm_tolerance, plus one
  output ulp): the same sweep.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

SWEEP = [(M, N, 3072) for N in (3072, 9216) for M in (8192, 32768, 112640)]
KINDS = {"int8": O.QUANT_INT8, "fp8_e4m3": O.QUANT_FP8}


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from thor_int8_gemm_b200 import ops as _ops
    yield _ops
    assert _ops.device_status() == 0, "a bounded wait ran out"


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def codes(t: torch.Tensor) -> np.ndarray:
    t = t.contiguous().cpu()
    return t.view(torch.uint8).numpy() if t.dtype == torch.float8_e4m3fn else t.numpy()


def sample_rows(M: int, seed: int) -> np.ndarray:
    edges = [0, 1, 127, 128, 255, 256, 257, M // 2, M - 129, M - 128, M - 2, M - 1]
    rnd = np.random.default_rng(seed).choice(M, 58, replace=False)
    return np.unique(np.clip(np.concatenate([edges, rnd]), 0, M - 1))


def make_problem(ops, M, N, K, kind, seed):
    """Quantised activations (1 % outlier channels x20), weights and bias on the GPU."""
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=dev)
    outliers = torch.randperm(K, generator=g, device=dev)[: max(1, K // 100)]
    x[:, outliers] *= 20.0
    x = x.to(torch.bfloat16)
    xq, xs = ops.quant_rows(x, kind)
    w = (torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wq, ws = ops.quant_rows(w, kind)
    bias = (torch.randn(N, generator=g, device=dev) * 0.01).to(torch.bfloat16)
    return x, xq, xs, wq, ws, bias


def check_quantised_rows(x, xq, xs, rows, kind):
    ridx = torch.from_numpy(rows).to(x.device)
    q_ref, s_ref = O.quant_rows(x[ridx].float().cpu().numpy(), KINDS[kind])
    np.testing.assert_array_equal(xs[ridx].cpu().numpy(), s_ref)
    np.testing.assert_array_equal(codes(xq[ridx]), q_ref)


@pytest.mark.parametrize("M,N,K", SWEEP)
def test_int8_sweep_shape_rows_bit_exact(ops, M, N, K):
    x, xq, xs, wq, ws, bias = make_problem(ops, M, N, K, "int8", M + N)
    out = ops.gemm_dequant(xq, wq, xs, ws, bias)
    rows = sample_rows(M, M * 3 + N)
    ridx = torch.from_numpy(rows).cuda()
    check_quantised_rows(x, xq, xs, rows, "int8")
    ref = O.gemm_i8_dequant(xq[ridx].cpu().numpy(), wq.cpu().numpy(), xs[ridx].cpu().numpy(), ws.cpu().numpy(),
                            bias.float().cpu().numpy(), "bf16")
    np.testing.assert_array_equal(bits16(out[ridx]), ref)


def test_int8_mlp_up_gemm_plain_and_swiglu_epilogue(ops):
    """fc1 32768 x 2*12288 x 3072: the plain GEMM's rows bit for bit, and the SwiGLU epilogue's
    act (interleaved weights) equal to the oracle's SwiGLU of those rows, bit for bit."""
    M, F, K = 32768, 12288, 3072
    x, xq, xs, wq, ws, bias = make_problem(ops, M, 2 * F, K, "int8", 77)
    rows = sample_rows(M, 78)
    ridx = torch.from_numpy(rows).cuda()
    y = ops.gemm_dequant(xq, wq, xs, ws, bias)
    y_ref = O.gemm_i8_dequant(xq[ridx].cpu().numpy(), wq.cpu().numpy(), xs[ridx].cpu().numpy(), ws.cpu().numpy(),
                              bias.float().cpu().numpy(), "bf16")
    np.testing.assert_array_equal(bits16(y[ridx]), y_ref)
    del y
    il = ops.interleave_gate_up
    act = ops.gemm_swiglu(xq, il(wq), xs, il(ws), il(bias))
    yf = O.bf16_to_f32(y_ref)
    _, _, act_ref = O.swiglu_quant_per_token(yf[:, :F], yf[:, F:], O.QUANT_INT8)
    np.testing.assert_array_equal(bits16(act[ridx]), act_ref)


def test_int8_mlp_down_gemm_k12288(ops):
    """fc2 32768 x 3072 x 12288 (K = the FFN width), sampled rows bit for bit."""
    M, N, K = 32768, 3072, 12288
    x, xq, xs, wq, ws, bias = make_problem(ops, M, N, K, "int8", 91)
    out = ops.gemm_dequant(xq, wq, xs, ws, bias)
    rows = sample_rows(M, 92)
    ridx = torch.from_numpy(rows).cuda()
    ref = O.gemm_i8_dequant(xq[ridx].cpu().numpy(), wq.cpu().numpy(), xs[ridx].cpu().numpy(), ws.cpu().numpy(),
                            bias.float().cpu().numpy(), "bf16")
    np.testing.assert_array_equal(bits16(out[ridx]), ref)


@pytest.mark.parametrize("M,N,K", SWEEP)
def test_fp8_sweep_shape_rows_within_accumulation_bound(ops, M, N, K):
    x, xq, xs, wq, ws, bias = make_problem(ops, M, N, K, "fp8_e4m3", M + N + 1)
    out = ops.gemm_dequant(xq, wq, xs, ws, bias)
    rows = sample_rows(M, M + 5 * N)
    ridx = torch.from_numpy(rows).cuda()
    check_quantised_rows(x, xq, xs, rows, "fp8_e4m3")
    aq, a_s = codes(xq[ridx]), xs[ridx].cpu().numpy()
    wc, wsc = codes(wq), ws.cpu().numpy()
    b = bias.float().cpu().numpy()
    got = O.bf16_to_f32(bits16(out[ridx])).astype(np.float64)
    ref = O.out_to_f32(O.gemm_fp8_dequant(aq, wc, a_s, wsc, b, "bf16"), "bf16").astype(np.float64)
    # both sides are bf16 roundings of float32 values within the bound: one bf16 spacing more
    spacing = np.spacing(np.maximum(np.abs(got), np.abs(ref)).astype(np.float32)).astype(np.float64) * 65536.0
    bound = O.fp8_gemm_tolerance(aq, wc, a_s, wsc, K) * 1.01 + spacing + 1e-30
    excess = np.abs(got - ref) / bound
    assert np.all(excess <= 1.0), float(excess.max())
