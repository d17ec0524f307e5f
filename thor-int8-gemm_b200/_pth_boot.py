"""Run by the one-line .pth file that `patch_int8.write_pth` installs: registers this
directory as the package `thor_int8_gemm_b200` and installs the two agents -- the
comfy-kitchen `_C` proxy (patch_int8) and the DiT-block agent (fused_patch), each inert
unless its own mode enables it.  Never raises (a performance patch must not break
interpreter start-up)."""
import importlib.util
import os
import sys

_DIR = os.path.dirname(os.path.abspath(__file__))
_NAME = "thor_int8_gemm_b200"


def _register():
    if _NAME in sys.modules:
        return sys.modules[_NAME]
    spec = importlib.util.spec_from_file_location(_NAME, os.path.join(_DIR, "__init__.py"),
                                                  submodule_search_locations=[_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[_NAME] = mod
    spec.loader.exec_module(mod)
    return mod


try:
    _register()
    from thor_int8_gemm_b200 import patch_int8 as _patch
    _patch.install_safely()
except Exception as _exc:  # never break interpreter start-up
    print(f"[ck-int8-patch] disabled: {_exc!r}", file=sys.stderr)
try:
    from thor_int8_gemm_b200 import fused_patch as _fused
    _fused.install_safely()
except Exception as _exc:
    print(f"[ck-fused-patch] disabled: {_exc!r}", file=sys.stderr)
