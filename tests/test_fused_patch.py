"""The DiT-block agent (fused_patch) against a fake ComfyUI + comfy-kitchen: mode selection,
version guard, import hook, eligibility and the fall-back latch, on CPU (the fused path
itself needs a GPU: tests/test_gpu_fused_patch.py).  Mirrors src/ck_fused_patch.py's
behaviour (:45-54 mode, :83-101 eligibility, :179-203 latch, :206-243 hook and install)."""
import importlib
import sys

import pytest
import torch

from fake_comfy import write_fake_comfy
from test_proxy import make_fake_kitchen
from thor_int8_gemm_b200 import fused_patch as FP

TARGET = "comfy.ldm.minimax.model"


def _purge():
    for name in list(sys.modules):
        if name == "comfy" or name.startswith("comfy.") or name == "comfy_kitchen" or name.startswith("comfy_kitchen."):
            del sys.modules[name]
    sys.meta_path[:] = [f for f in sys.meta_path if not isinstance(f, FP._Finder)]
    importlib.invalidate_caches()


@pytest.fixture
def comfy_env(tmp_path, monkeypatch):
    make_fake_kitchen(tmp_path, version="0.2.40")
    write_fake_comfy(tmp_path)
    monkeypatch.syspath_prepend(str(tmp_path))
    monkeypatch.delenv(FP.ENV, raising=False)
    monkeypatch.setattr(FP, "MODE_FILE", str(tmp_path / "no-such-mode-file"))
    _purge()
    yield tmp_path
    _purge()


def _inputs(d=64, S=20, B=2):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(S, d, generator=g).to(torch.bfloat16)
    t = (torch.randn(B, d, generator=g) * 0.3).to(torch.bfloat16)
    return x, t, [(0, 12, 0), (12, S, 1)]


def test_read_mode(tmp_path, monkeypatch):
    monkeypatch.setattr(FP, "MODE_FILE", str(tmp_path / "m"))
    monkeypatch.delenv(FP.ENV, raising=False)
    assert FP._read_mode() == "off"
    (tmp_path / "m").write_text("C2\n")
    assert FP._read_mode() == "c2"
    monkeypatch.setenv(FP.ENV, "1")
    assert FP._read_mode() == "on"
    monkeypatch.setenv(FP.ENV, " c1 ")
    assert FP._read_mode() == "c1"


def test_off_leaves_the_block_stock(comfy_env, capsys):
    FP.install()
    import comfy.ldm.minimax.model as m
    assert not getattr(m.DiTBlock.forward, "_t8g_fused", False)
    assert not any(isinstance(f, FP._Finder) for f in sys.meta_path)


def test_unvalidated_kitchen_is_refused(tmp_path, monkeypatch, capsys):
    make_fake_kitchen(tmp_path, version="0.2.37")
    write_fake_comfy(tmp_path)
    monkeypatch.syspath_prepend(str(tmp_path))
    monkeypatch.setenv(FP.ENV, "on")
    _purge()
    try:
        FP.install()
        assert "not validated" in capsys.readouterr().err
        import comfy.ldm.minimax.model as m
        assert not getattr(m.DiTBlock.forward, "_t8g_fused", False)
    finally:
        _purge()


def test_unknown_mode_is_reported(comfy_env, monkeypatch, capsys):
    monkeypatch.setenv(FP.ENV, "turbo")
    FP.install()
    assert "unknown mode" in capsys.readouterr().err


@pytest.mark.parametrize("import_first", [False, True])
def test_hook_patches_and_cpu_calls_run_stock(comfy_env, monkeypatch, capsys, import_first):
    monkeypatch.setenv(FP.ENV, "on")
    if import_first:
        import comfy.ldm.minimax.model  # noqa: F401
    FP.install()
    import comfy.ldm.minimax.model as m
    assert m.DiTBlock.forward._t8g_fused
    assert "fused on B200 kernels mode=on" in capsys.readouterr().err
    blk = m.DiTBlock(64, 128)
    x, t, segs = _inputs()
    stock = m.DiTBlock.forward.__wrapped__
    ref = stock(blk, x, t, segs, None)
    before = m.CALLS["stock"]
    out = blk(x, t, segs, None)                      # CPU tensors: ineligible -> stock forward
    assert m.CALLS["stock"] == before + 1
    assert torch.equal(out, ref)
    FP.install()                                     # a second install does not wrap twice
    assert m.DiTBlock.forward.__wrapped__ is stock


def test_failure_latches_to_stock(comfy_env, monkeypatch, capsys):
    monkeypatch.setenv(FP.ENV, "on")
    FP.install()
    import comfy.ldm.minimax.model as m
    rt = m.DiTBlock.forward._t8g_runtime
    monkeypatch.setattr(rt, "eligible", lambda *a: True)

    def boom(*a, **k):
        raise RuntimeError("kernel failure stand-in")
    monkeypatch.setattr(rt, "forward", boom)
    blk = m.DiTBlock(64, 128)
    x, t, segs = _inputs()
    ref = m.DiTBlock.forward.__wrapped__(blk, x, t, segs, None)
    assert torch.equal(blk(x, t, segs, None), ref)
    assert rt.broken
    err = capsys.readouterr().err
    assert "fused path failed" in err and "kernel failure stand-in" in err
    assert torch.equal(blk(x, t, segs, None), ref)   # stays stock, warns once
    assert "fused path failed" not in capsys.readouterr().err


def test_eligibility_and_row_map(comfy_env, monkeypatch):
    monkeypatch.setenv(FP.ENV, "on")
    FP.install()
    import comfy.ldm.minimax.model as m
    rt = m.DiTBlock.forward._t8g_runtime
    blk = m.DiTBlock(64, 128)
    x, t, segs = _inputs()
    assert not rt.eligible(blk, x, segs)                             # CPU tensor
    rows = rt.row_map([(0, 3, 1), (3, 6, torch.tensor([0, 2, 1]))], 6, "cpu")
    assert rows.tolist() == [1, 1, 1, 0, 2, 1] and rows.dtype == torch.int32
    with pytest.raises(ValueError):
        rt.row_map([(0, 3, 0)], 6, "cpu")
    import comfy.model_management as mm
    monkeypatch.setattr(mm, "in_training", True)
    assert not rt.eligible(blk, x, segs)


def test_pth_boot_installs_both_agents():
    src = open(FP.__file__.replace("fused_patch.py", "_pth_boot.py")).read()
    assert "patch_int8" in src and "fused_patch" in src
