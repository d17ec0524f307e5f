"""The C-ABI library loads without a GPU, exports every symbol the public header
declares, and rejects malformed arguments on the host before touching CUDA."""
import ctypes
import os
import re

import pytest

from thor_int8_gemm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "thor_int8_gemm_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(t8g_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_expected_entry_points():
    names = declared_symbols()
    for n in ("t8g_gemm_i8_dequant", "t8g_gemm_fp8_dequant", "t8g_quant_rows", "t8g_rms_mod_quant",
              "t8g_rms_mod_quant_tensorwise", "t8g_swiglu_quant", "t8g_swiglu_quant_tensorwise",
              "t8g_device_status", "t8g_last_error", "t8g_version", "t8g_wait_selftest", "t8g_gemm_i8_swiglu",
              "t8g_gemm_fp8_swiglu", "t8g_gemm_i8_gated", "t8g_gemm_fp8_gated"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    # and the ctypes signatures cover exactly the header
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_build_targets_sm100a_only():
    from thor_int8_gemm_b200 import build
    flags = " ".join(build.NVCC_FLAGS)
    assert "arch=compute_100a,code=sm_100a" in flags and flags.count("-gencode") == 1


def test_version_and_empty_error():
    assert _lib.version() == "0.1.0"
    assert _lib.load().t8g_last_error() in (b"",) or isinstance(_lib.load().t8g_last_error(), bytes)


def _gemm(**kw):
    lib = _lib.load()
    a = dict(x=ctypes.c_void_p(16), w=ctypes.c_void_p(16), xs=ctypes.c_void_p(16), ws=ctypes.c_void_p(16),
             ws_n=1, bias=None, bias_n=0, out=ctypes.c_void_p(16), dt=0, M=128, N=128, K=128,
             ld_x=128, ld_w=128, ld_out=128, stream=None)
    a.update(kw)
    return lib.t8g_gemm_i8_dequant(a["x"], a["w"], a["xs"], a["ws"], a["ws_n"], a["bias"], a["bias_n"], a["out"],
                                   a["dt"], a["M"], a["N"], a["K"], a["ld_x"], a["ld_w"], a["ld_out"], a["stream"])


@pytest.mark.parametrize("kw,needle", [
    (dict(K=-1), "bad sizes"),
    (dict(dt=7), "out_dtype"),
    (dict(ws_n=5), "w_scale numel"),
    (dict(bias_n=3), "bias numel"),
    (dict(bias_n=128, bias=None), "bias is null"),
    (dict(ld_x=136), "16 bytes"),
    (dict(ld_x=64), "smaller than the row"),
    (dict(x=ctypes.c_void_p(8)), "16-byte aligned"),
    (dict(M=1 << 31), "2^31"),
])
def test_gemm_rejects_bad_arguments_on_host(kw, needle):
    rc = _gemm(**kw)
    assert rc in (_lib.T8G_ERR_INVALID_ARGUMENT, _lib.T8G_ERR_UNSUPPORTED)
    assert needle in _lib.load().t8g_last_error().decode()


def test_gemm_empty_problem_is_a_no_op():
    assert _gemm(M=0) == _lib.T8G_OK
    assert _gemm(N=0, x=None, w=None) == _lib.T8G_OK


def test_row_entry_points_reject_bad_shapes_on_host():
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    rc = lib.t8g_quant_rows(p, 16, p, 16, p, 4, 12, 0, None)
    assert rc == _lib.T8G_ERR_INVALID_ARGUMENT and b"multiple of 8" in lib.t8g_last_error()
    rc = lib.t8g_quant_rows(p, 49160, p, 49160, p, 4, 49160, 0, None)
    assert rc == _lib.T8G_ERR_UNSUPPORTED and b"exceeds" in lib.t8g_last_error()
    rc = lib.t8g_quant_rows(p, 64, p, 64, p, 4, 64, 5, None)
    assert rc == _lib.T8G_ERR_INVALID_ARGUMENT and b"quant_kind" in lib.t8g_last_error()
    rc = lib.t8g_swiglu_quant(p, p, 64, p, 64, None, None, 64, 4, 64, 0, None)
    assert rc == _lib.T8G_ERR_INVALID_ARGUMENT and b"q_scale" in lib.t8g_last_error()
    rc = lib.t8g_rms_mod_quant(p, 64, None, p, p, 64, None, 0, 0, 1e-6, p, 64, p, None, 64, None, 64, 4, 64, 0, None)
    assert rc == _lib.T8G_ERR_INVALID_ARGUMENT and b"rows_per_mod" in lib.t8g_last_error()
    rc = lib.t8g_rms_mod_quant_tensorwise(p, 64, None, p, p, 64, None, 1, 0, 1e-6, p, 64, None, 64, None, 64, p, p,
                                          4, 64, 1, None)
    assert rc == _lib.T8G_ERR_INVALID_ARGUMENT and b"h is null" in lib.t8g_last_error()
    assert lib.t8g_quant_rows(None, 8, None, 8, None, 0, 8, 0, None) == _lib.T8G_OK   # S == 0 is a no-op


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(ImportError, match="build it"):
        _lib.load(str(tmp_path / "nope.so"))


def test_capsule_module_declines_what_it_does_not_serve():
    """The compiled proxy entry reads DLPack capsules without consuming them and launches only
    for CUDA tensors; anything else is left to the general path (None)."""
    import torch
    from thor_int8_gemm_b200 import _t8g_capsule as C
    ts = (torch.zeros(256, 64, dtype=torch.int8), torch.zeros(32, 64, dtype=torch.int8), torch.ones(256),
          torch.ones(32), torch.zeros(0, dtype=torch.bfloat16), torch.zeros(256, 32, dtype=torch.bfloat16))
    caps = [t.__dlpack__() for t in ts]
    assert C.cutlass_int8_dequant(*caps, 0) is None                  # host tensors
    assert C.cutlass_int8_dequant(*ts, 0) is None                    # tensors, not capsules
    assert C.cutlass_int8_dequant(*caps[:6], "stream") is None       # stream not an integer
    assert all(torch.from_dlpack(c).shape == t.shape for c, t in zip(caps, ts))   # not consumed
    vcaps = [t.__dlpack__(max_version=(1, 0)) for t in ts]                # DLPack 1.x capsules
    assert C.cutlass_int8_dequant(*vcaps, 0) is None
    assert all(torch.from_dlpack(c).shape == t.shape for c, t in zip(vcaps, ts))
    with pytest.raises(TypeError):
        C.cutlass_int8_dequant(*caps)
