"""The comfy-kitchen `_C` import proxy and its installer, against a fake
comfy-kitchen package (the real one is not installable here).

Mirrors the behaviour of the reference agent src/ck_int8_patch_thor.py:
mode selection (:34-42), version guard (:178-188), eligibility (:148-156),
fallback latch (:159-167), meta-path hook (:219-240), install (:243-260).
"""
import importlib
import os
import subprocess
import sys
import textwrap

import pytest
import torch

from thor_int8_gemm_b200 import patch_int8 as P

FAKE_C = '''
CALLS = []
def cutlass_int8_dequant(x, w, x_scale, w_scale, bias, out, dtype_code, stream):
    import torch
    CALLS.append(tuple(torch.from_dlpack(t) for t in (x, w, x_scale, w_scale, bias, out)) + (dtype_code, stream))
    return "stock"
def other_op():
    return 42
'''


def make_fake_kitchen(root, version="0.2.40"):
    pkg = root / "comfy_kitchen"
    (pkg / "backends" / "cuda").mkdir(parents=True)
    (pkg / "backends" / "eager").mkdir(parents=True)
    (pkg / "__init__.py").write_text(textwrap.dedent('''
        def int8_linear(x, weight, weight_scale, bias=None, out_dtype=None, convrot=False,
                        convrot_groupsize=256, input_act=None, input_act_weight=None,
                        input_act_eps=0.0, residual=None, residual_scale=None):
            return ("eager", x)
    '''))
    (pkg / "backends" / "__init__.py").write_text("")
    (pkg / "backends" / "cuda" / "_C_fake.py").write_text(FAKE_C)
    (pkg / "backends" / "cuda" / "__init__.py").write_text("from . import _C_fake as _C\n_DISABLE_CUTLASS_INT8 = False\n")
    (pkg / "backends" / "eager" / "__init__.py").write_text("")
    (pkg / "backends" / "eager" / "quantization.py").write_text(
        "import torch\nDTYPE_CODE_TO_DTYPE = {0: torch.bfloat16, 1: torch.float16, 2: torch.float32}\n")
    dist = root / f"comfy_kitchen-{version}.dist-info"
    dist.mkdir()
    (dist / "METADATA").write_text(f"Metadata-Version: 2.1\nName: comfy-kitchen\nVersion: {version}\n")
    (dist / "RECORD").write_text("")


def _purge():
    for name in list(sys.modules):
        if name == "comfy_kitchen" or name.startswith("comfy_kitchen."):
            del sys.modules[name]
    sys.meta_path[:] = [f for f in sys.meta_path if not isinstance(f, P._Finder)]
    importlib.invalidate_caches()


@pytest.fixture
def kitchen(tmp_path, monkeypatch):
    make_fake_kitchen(tmp_path)
    monkeypatch.syspath_prepend(str(tmp_path))
    monkeypatch.delenv("CK_INT8_MODE", raising=False)
    monkeypatch.setattr(P, "MODE_FILE", str(tmp_path / "no-such-mode-file"))
    _purge()
    yield tmp_path
    _purge()


def test_read_mode_env_file_default(tmp_path, monkeypatch):
    monkeypatch.setattr(P, "MODE_FILE", str(tmp_path / "mode"))
    monkeypatch.delenv("CK_INT8_MODE", raising=False)
    assert P._read_mode() == "off"
    (tmp_path / "mode").write_text("Triton\n")
    assert P._read_mode() == "triton"
    (tmp_path / "mode").write_text("\n")
    assert P._read_mode() == "off"
    monkeypatch.setenv("CK_INT8_MODE", " B200 ")
    assert P._read_mode() == "b200"


def test_install_off_leaves_stock(kitchen):
    P.install()
    import comfy_kitchen.backends.cuda as cuda
    assert not isinstance(cuda._C, P._CProxy)
    assert not any(isinstance(f, P._Finder) for f in sys.meta_path)


@pytest.mark.parametrize("mode", ["b200", "triton"])
def test_install_after_import_swaps_C(kitchen, monkeypatch, capsys, mode):
    import comfy_kitchen.backends.cuda as cuda
    monkeypatch.setenv("CK_INT8_MODE", mode)
    P.install()
    assert isinstance(cuda._C, P._CProxy)
    assert f"[ck-int8-patch] comfy_kitchen 0.2.40 int8 mode={mode}" in capsys.readouterr().err
    P.install()                             # idempotent: no proxy of a proxy
    assert not isinstance(cuda._C._real, P._CProxy)


def test_install_before_import_uses_meta_path_hook(kitchen, monkeypatch):
    monkeypatch.setenv("CK_INT8_MODE", "b200")
    P.install()
    assert any(isinstance(f, P._Finder) for f in sys.meta_path)
    import comfy_kitchen.backends.cuda as cuda
    assert isinstance(cuda._C, P._CProxy)
    import comfy_kitchen
    assert getattr(comfy_kitchen.int8_linear, "_ck_compile_safe", False)
    assert comfy_kitchen.int8_linear("x", None, None) == ("eager", "x")      # eager calls untouched


def test_version_guard_keeps_stock(tmp_path, monkeypatch, capsys):
    make_fake_kitchen(tmp_path, version="0.2.41")
    monkeypatch.syspath_prepend(str(tmp_path))
    monkeypatch.setenv("CK_INT8_MODE", "b200")
    _purge()
    try:
        import comfy_kitchen.backends.cuda as cuda
        P.install()
        assert not isinstance(cuda._C, P._CProxy)
        assert "NOT applied: comfy-kitchen 0.2.41 is not validated" in capsys.readouterr().err
    finally:
        _purge()


def test_cublas_mode_flips_comfy_flag(kitchen, monkeypatch):
    import comfy_kitchen.backends.cuda as cuda
    monkeypatch.setenv("CK_INT8_MODE", "cublas")
    P.install()
    assert cuda._DISABLE_CUTLASS_INT8 is True
    assert not isinstance(cuda._C, P._CProxy)


def test_unknown_mode_warns_and_stays_stock(kitchen, monkeypatch, capsys):
    import comfy_kitchen.backends.cuda as cuda
    monkeypatch.setenv("CK_INT8_MODE", "fast")
    P.install()
    assert "unknown mode 'fast'" in capsys.readouterr().err
    assert not isinstance(cuda._C, P._CProxy)


def _args(M=256, N=128, K=64, *, x_dtype=torch.int8, out_dtype=torch.bfloat16, bias_n=None, bias_dtype=None,
          ws_n=None, xs_dtype=torch.float32, xs_n=None, transpose_x=False, out_shape=None):
    x = torch.zeros(K, M, dtype=torch.int8).t() if transpose_x else torch.zeros(M, K, dtype=torch.int8)
    x = x.to(x_dtype) if x_dtype != torch.int8 else x
    w = torch.zeros(N, K, dtype=torch.int8)
    xs = torch.ones(M if xs_n is None else xs_n, dtype=xs_dtype)
    ws = torch.ones(N if ws_n is None else ws_n)
    nb = N if bias_n is None else bias_n
    bias = torch.zeros(nb, dtype=bias_dtype or out_dtype)
    out = torch.empty(*(out_shape or (M, N)), dtype=out_dtype)
    return [x, w, xs, ws, bias, out]


def _call(proxy, tensors, dtype_code=0, stream=1234):
    return proxy.cutlass_int8_dequant(*(t.__dlpack__() for t in tensors), dtype_code, stream)


class Recorder:
    def __init__(self, fail=False):
        self.calls = []
        self.fail = fail

    def __call__(self, *a):
        self.calls.append(a)
        if self.fail:
            raise RuntimeError("kernel exploded")


@pytest.mark.parametrize("kw", [
    dict(M=64),                                  # M < MIN_M
    dict(K=40),                                  # K % 16
    dict(transpose_x=True),                      # non-contiguous x
    dict(x_dtype=torch.int16),                   # not int8
    dict(out_dtype=torch.int32),                 # unsupported out dtype
    dict(out_shape=(256, 64)),                   # out is not [M, N]
    dict(xs_dtype=torch.float16),                # x_scale not fp32
    dict(xs_n=3),                                # x_scale numel != M
    dict(ws_n=5),                                # w_scale numel not in (1, N)
    dict(bias_n=3),                              # bias numel not in (0, N)
    dict(bias_dtype=torch.float32),              # bias dtype != out dtype
])
def test_ineligible_calls_go_to_stock(kitchen, kw):
    import comfy_kitchen.backends.cuda as cuda
    rec = Recorder()
    proxy = P._CProxy(cuda._C, rec)
    assert _call(proxy, _args(**kw)) == "stock"
    assert not rec.calls
    assert len(cuda._C.CALLS) == 1 and cuda._C.CALLS[0][-1] == 1234


@pytest.mark.parametrize("kw", [dict(), dict(ws_n=1), dict(bias_n=0), dict(out_dtype=torch.float32),
                                dict(out_dtype=torch.float16), dict(M=128, K=16)])
def test_eligible_calls_reach_the_b200_kernel(kitchen, kw):
    import comfy_kitchen.backends.cuda as cuda
    rec = Recorder()
    proxy = P._CProxy(cuda._C, rec)
    assert _call(proxy, _args(**kw), stream=777) is True
    assert len(rec.calls) == 1 and not cuda._C.CALLS
    tx, tw, txs, tws, tb, tout, stream = rec.calls[0]
    assert tx.dtype == torch.int8 and tout.dtype == _args(**kw)[5].dtype and stream == 777


def test_failure_latches_to_stock_with_traceback(kitchen, capsys):
    import comfy_kitchen.backends.cuda as cuda
    rec = Recorder(fail=True)
    proxy = P._CProxy(cuda._C, rec)
    assert _call(proxy, _args()) == "stock"
    err = capsys.readouterr().err
    assert "[ck-int8-patch] B200 GEMM failed" in err and "Traceback" in err and "kernel exploded" in err
    assert proxy._broken
    assert _call(proxy, _args()) == "stock"
    assert len(rec.calls) == 1 and len(cuda._C.CALLS) == 2


def test_default_kernel_on_cpu_tensors_latches(kitchen, capsys):
    """The real kernel refuses CPU tensors (no CPU path); the proxy falls back."""
    import comfy_kitchen.backends.cuda as cuda
    proxy = P._CProxy(cuda._C)
    assert _call(proxy, _args()) == "stock"
    assert proxy._broken and "CUDA tensor" in capsys.readouterr().err


def test_proxy_forwards_public_attributes_only(kitchen):
    import comfy_kitchen.backends.cuda as cuda
    proxy = P._CProxy(cuda._C, Recorder())
    assert proxy.other_op() == 42
    with pytest.raises(AttributeError):
        proxy._private_thing


def test_stream_argument_normalisation():
    assert P._stream_arg(None) is None
    assert P._stream_arg(5) == 5
    assert P._stream_arg("not-a-stream") is None


def test_pth_boot_installs_proxy_in_a_fresh_interpreter(tmp_path):
    fake = tmp_path / "fake"
    fake.mkdir()
    make_fake_kitchen(fake)
    site_dir = tmp_path / "site"
    site_dir.mkdir()
    pth = P.write_pth(str(site_dir))
    assert os.path.basename(pth) == P.PTH_NAME
    code = ("import site, sys; site.addsitedir(sys.argv[1]); "
            "import comfy_kitchen.backends.cuda as c; print(type(c._C).__name__)")
    env = dict(os.environ, CK_INT8_MODE="b200", PYTHONPATH=str(fake))
    r = subprocess.run([sys.executable, "-c", code, str(site_dir)], env=env, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "_CProxy"
    assert "int8 mode=b200" in r.stderr


def test_pth_boot_never_breaks_startup(tmp_path):
    site_dir = tmp_path / "site"
    site_dir.mkdir()
    (site_dir / P.PTH_NAME).write_text(P.pth_line().replace("_pth_boot.py", "_missing_boot.py") + "\n")
    r = subprocess.run([sys.executable, "-c", "import site, sys; site.addsitedir(sys.argv[1]); print('alive')",
                        str(site_dir)], capture_output=True, text=True, timeout=120)
    assert r.stdout.strip() == "alive"


def test_interleave_gate_up_layout():
    """Blocks of 128 gate rows then the matching 128 up rows; 1-D and 2-D parameters."""
    import torch
    from thor_int8_gemm_b200 import ops
    F = 256
    w = torch.arange(2 * F).view(2 * F, 1).repeat(1, 3)
    il = ops.interleave_gate_up(w)
    order = il[:, 0].tolist()
    expect = list(range(0, 128)) + list(range(F, F + 128)) + list(range(128, 256)) + list(range(F + 128, F + 256))
    assert order == expect
    assert ops.interleave_gate_up(torch.arange(2 * F)).tolist() == expect
    import pytest
    with pytest.raises(ValueError):
        ops.interleave_gate_up(torch.zeros(384))
