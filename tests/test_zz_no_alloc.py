"""The allocation-free tensorwise norm/mod/quant entry point.

t8g_rms_mod_quant_tensorwise_noalloc exists for callers that cannot allocate device
memory when they quantise (a plugin inside a host whose allocator owns the GPU, a C
caller without a CUDA allocator, a path that cannot afford cudaMalloc's implicit
synchronisation): it keeps the amax word and the bf16 intermediate in the library's
own static device scratch instead of taking them from the caller.

These tests call it through the C ABI and compare it with the regular entry point
(t8g_rms_mod_quant_tensorwise, caller-provided buffers), bit for bit, on two calls
in a row -- the second with a smaller amax, so stale scratch from the first call
would show.  This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

QUANT = {"fp8_e4m3": (1, torch.float8_e4m3fn), "int8": (0, torch.int8)}


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from thor_int8_gemm_b200 import _lib
    return _lib


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def noalloc_call(_lib, x, shift, scale, rows_per_mod, eps, kind, want_res=True):
    S, D = x.shape
    code, qdt = QUANT[kind]
    q = torch.empty(S, D, dtype=qdt, device=x.device)
    res = torch.empty_like(x) if want_res else None
    scale_out = torch.empty((), dtype=torch.float32, device=x.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = _lib.load().t8g_rms_mod_quant_tensorwise_noalloc(
        _p(x), x.stride(0), None, _p(shift), _p(scale), shift.stride(0), None, rows_per_mod, 0, eps,
        _p(q), q.stride(0), _p(res), D, _p(scale_out), S, D, code, stream)
    _lib.check(rc)
    return q, scale_out, res


def regular_call(_lib, x, shift, scale, rows_per_mod, eps, kind):
    S, D = x.shape
    code, qdt = QUANT[kind]
    q = torch.empty(S, D, dtype=qdt, device=x.device)
    h = torch.empty_like(x)
    res = torch.empty_like(x)
    amax = torch.empty((), dtype=torch.float32, device=x.device)
    scale_out = torch.empty((), dtype=torch.float32, device=x.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = _lib.load().t8g_rms_mod_quant_tensorwise(
        _p(x), x.stride(0), None, _p(shift), _p(scale), shift.stride(0), None, rows_per_mod, 0, eps,
        _p(q), q.stride(0), _p(h), D, _p(res), D, _p(amax), _p(scale_out), S, D, code, stream)
    _lib.check(rc)
    return q, scale_out, res


def inputs(seed, S, D, n_mod, shift_mag):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(S, D, generator=g, device="cuda").to(torch.bfloat16)
    shift = (torch.randn(n_mod, D, generator=g, device="cuda") * shift_mag).to(torch.bfloat16)
    scale = (torch.randn(n_mod, D, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    return x, shift, scale


def as_bytes(t):
    return t.view(torch.uint8).cpu().numpy() if t.dtype == torch.float8_e4m3fn else t.cpu().numpy()


@pytest.mark.parametrize("kind", ["fp8_e4m3", "int8"])
def test_noalloc_matches_regular_entry_on_two_calls_in_a_row(lib, kind):
    # call 1: large shift -> large amax; call 2: small shift -> much smaller amax
    for call, (seed, S, D, n_mod, mag) in enumerate([(1, 2048, 3072, 2, 8.0), (2, 700, 5376, 1, 0.05)]):
        x, shift, scale = inputs(seed, S, D, n_mod, mag)
        rpm = S // n_mod
        q_n, s_n, r_n = noalloc_call(lib, x, shift, scale, rpm, 1e-6, kind)
        q_r, s_r, r_r = regular_call(lib, x, shift, scale, rpm, 1e-6, kind)
        torch.cuda.synchronize()
        assert s_n.item() == s_r.item(), f"call {call}: scale {s_n.item()} != {s_r.item()}"
        np.testing.assert_array_equal(as_bytes(q_n), as_bytes(q_r))
        assert torch.equal(r_n, r_r)
    from thor_int8_gemm_b200 import ops
    assert ops.device_status() == 0


def test_noalloc_without_res_output(lib):
    x, shift, scale = inputs(3, 64, 3072, 1, 0.1)
    q_n, s_n, _ = noalloc_call(lib, x, shift, scale, 64, 1e-5, "fp8_e4m3", want_res=False)
    q_r, s_r, _ = regular_call(lib, x, shift, scale, 64, 1e-5, "fp8_e4m3")
    assert s_n.item() == s_r.item()
    np.testing.assert_array_equal(as_bytes(q_n), as_bytes(q_r))


def test_noalloc_rejects_problems_larger_than_its_scratch(lib):
    S, D = 4096, 3072                               # 25.2 MB of bf16 h > 16 MiB of scratch
    x = torch.zeros(S, D, dtype=torch.bfloat16, device="cuda")
    shift = torch.zeros(1, D, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(lib.T8GError) as ei:
        noalloc_call(lib, x, shift, shift, S, 1e-6, "fp8_e4m3")
    assert ei.value.code == lib.T8G_ERR_UNSUPPORTED
    assert "exceeds the built-in scratch" in ei.value.message
