"""The `_C.cutlass_int8_dequant` proxy on the GPU: eligible calls launch from the DLPack
capsules through the compiled entry (no torch tensors built), the result equals the library
GEMM; declined calls reach the stock kernel; a launch the library rejects latches the proxy to
stock (src/ck_int8_patch_thor.py:143-168)."""
import pytest
import torch

from thor_int8_gemm_b200 import patch_int8 as P

pytestmark = pytest.mark.gpu


class Stock:
    def __init__(self):
        self.calls = 0

    def cutlass_int8_dequant(self, *args):
        self.calls += 1
        return "stock"


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from thor_int8_gemm_b200 import ops as _ops
    yield _ops
    assert _ops.device_status() == 0


@pytest.fixture
def fast_counter(monkeypatch):
    fn = P._capsule_entry()
    assert fn is not None, "the capsule module is not built"
    seen = []

    def counting(*a):
        try:
            r = fn(*a)
        except Exception:
            seen.append("raised")
            raise
        seen.append(r)
        return r

    monkeypatch.setattr(P, "_capsule_fn", counting)
    monkeypatch.setattr(P, "_capsule_tried", True)
    return seen


def problem(ops, M, N, K, out_dtype=torch.bfloat16, bias=True, ws1=False, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    xq, xs = ops.quant_rows(torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16), "int8")
    wq, ws = ops.quant_rows((torch.randn(N, K, generator=g, device="cuda") * 0.02).to(torch.bfloat16), "int8")
    if ws1:
        ws = ws[:1].clone()
    b = ((torch.randn(N, generator=g, device="cuda") * 0.1).to(out_dtype) if bias
         else torch.zeros(0, dtype=out_dtype, device="cuda"))
    out = torch.empty(M, N, dtype=out_dtype, device="cuda")
    return xq, wq, xs, ws, b, out


def call(proxy, ts, stream=None):
    s = torch.cuda.current_stream().cuda_stream if stream is None else stream
    return proxy.cutlass_int8_dequant(*(t.__dlpack__(stream=-1) for t in ts), 0, s)


@pytest.mark.parametrize("M,N,K,out_dtype,bias,ws1", [
    (256, 3072, 3072, torch.bfloat16, True, False), (1000, 9216, 3072, torch.bfloat16, True, False),
    (128, 520, 256, torch.float16, True, False), (300, 3072, 1024, torch.float32, False, True),
    (4096, 24576, 3072, torch.bfloat16, True, False)])
def test_fast_path_equals_library_gemm(ops, fast_counter, M, N, K, out_dtype, bias, ws1):
    stock = Stock()
    proxy = P._CProxy(stock)
    xq, wq, xs, ws, b, out = problem(ops, M, N, K, out_dtype, bias, ws1, seed=M + N)
    assert call(proxy, (xq, wq, xs.view(M, 1), ws, b, out)) is True
    assert fast_counter == [True] and stock.calls == 0
    ref = ops.gemm_dequant(xq, wq, xs, ws, b if bias else None, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_fast_path_on_a_side_stream(ops, fast_counter):
    proxy = P._CProxy(Stock())
    xq, wq, xs, ws, b, out = problem(ops, 512, 3072, 3072, seed=7)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    assert call(proxy, (xq, wq, xs, ws, b, out), stream=s.cuda_stream) is True
    s.synchronize()
    assert torch.equal(out, ops.gemm_dequant(xq, wq, xs, ws, b))


@pytest.mark.parametrize("case", ["small_m", "k_not_16", "transposed_x", "ws_numel", "bias_dtype"])
def test_declined_calls_reach_stock(ops, fast_counter, case):
    stock = Stock()
    proxy = P._CProxy(stock)
    M, N, K = (64 if case == "small_m" else 256), 256, (40 if case == "k_not_16" else 128)
    xq, wq, xs, ws, b, out = problem(ops, M, N, K if K % 16 == 0 else 48, seed=3)
    if case == "k_not_16":
        xq = torch.zeros(M, K, dtype=torch.int8, device="cuda")
        wq = torch.zeros(N, K, dtype=torch.int8, device="cuda")
    if case == "transposed_x":
        xq = xq.t().contiguous().t()
    if case == "ws_numel":
        ws = ws[:5]
    if case == "bias_dtype":
        b = b.float()
    assert call(proxy, (xq, wq, xs, ws, b, out)) == "stock"
    assert fast_counter == [None] and stock.calls == 1 and not proxy._broken


def test_rejected_launch_latches_to_stock(ops, fast_counter, capsys):
    stock = Stock()
    proxy = P._CProxy(stock)
    M, N, K = 256, 256, 128
    _, wq, xs, ws, b, out = problem(ops, M, N, K, seed=4)
    raw = torch.zeros(M * K + 1, dtype=torch.int8, device="cuda")
    x_misaligned = raw[1:].view(M, K)   # contiguous, but not 16-byte aligned: the library refuses it
    assert call(proxy, (x_misaligned, wq, xs, ws, b, out)) == "stock"
    assert proxy._broken and stock.calls == 1
    assert "B200 GEMM failed" in capsys.readouterr().err
    assert call(proxy, (x_misaligned, wq, xs, ws, b, out)) == "stock"   # latched: no second try
    assert fast_counter == ["raised"]


def test_capsule_module_takes_dlpack_1_capsules(ops):
    """DLPack 1.x ("dltensor_versioned") capsules launch the same GEMM."""
    from thor_int8_gemm_b200 import _t8g_capsule as C
    xq, wq, xs, ws, b, out = problem(ops, 512, 3072, 1024, seed=9)
    caps = [t.__dlpack__(max_version=(1, 0)) for t in (xq, wq, xs, ws, b, out)]
    assert C.cutlass_int8_dequant(*caps, torch.cuda.current_stream().cuda_stream) is True
    torch.cuda.synchronize()
    assert torch.equal(out, ops.gemm_dequant(xq, wq, xs, ws, b))


def test_wait_that_ran_out_stops_the_proxy(ops, fast_counter, capsys):
    """A kernel whose bounded wait runs out (the self-test kernel, which waits on a barrier
    nothing completes) shows on the host-visible status mirror without a synchronisation; the
    proxy reads it on its next call, reports it and serves that call and every later one from
    stock.  The device status word tells the same story and is cleared after."""
    stock = Stock()
    proxy = P._CProxy(stock)
    xq, wq, xs, ws, b, out = problem(ops, 256, 512, 256, seed=12)
    assert call(proxy, (xq, wq, xs, ws, b, out)) is True          # sets the mirror up for this device
    word = ops.status_mirror()
    assert word[0] == 0
    assert ops.wait_selftest(limit_ns=5_000_000) == 1
    assert word[0] == 0x1FF
    assert call(proxy, (xq, wq, xs, ws, b, out)) == "stock"
    err = capsys.readouterr().err
    assert "bounded device wait" in err and "0x1ff" in err
    assert proxy._broken and stock.calls == 1 and word[0] == 0
    assert call(proxy, (xq, wq, xs, ws, b, out)) == "stock" and stock.calls == 2
    assert ops.device_status() == 0x1FF
    assert ops.device_status() == 0
