"""comfy-kitchen INT8 GEMM override that routes `_C.cutlass_int8_dequant` to this
library's sm_100a kernel.  Drop-in for the reference agent
src/ck_int8_patch_thor.py (same modes, mode file, environment variable, version
guard, eligibility rules, fallback latch and stderr tag), loaded the same way:
from a `.pth` file in site-packages (see `write_pth`), so every interpreter in the
venv gets it without code changes.

Modes (env CK_INT8_MODE, else /etc/comfy-kitchen-int8.mode, else "off"):
  off     stock comfy-kitchen
  cublas  comfy-kitchen's own cuBLAS route (sets `_DISABLE_CUTLASS_INT8`)
  b200    `_C.cutlass_int8_dequant` runs on this library's tcgen05 GEMM
  triton  accepted as a synonym of b200, so an existing mode file keeps working

Nothing here imports torch or loads the CUDA library until a call needs it;
installing never raises.
"""
from __future__ import annotations

import importlib.abc
import importlib.machinery
import os
import sys

MODE_FILE = "/etc/comfy-kitchen-int8.mode"          # src/ck_int8_patch_thor.py:26
TARGET = "comfy_kitchen.backends.cuda"               # :27
TOP = "comfy_kitchen"                                # :28
VALIDATED_KITCHEN = ("0.2.37", "0.2.40")             # :29
MIN_M = 128                                          # :30
KERNEL_MODES = ("b200", "triton")
TAG = "[ck-int8-patch]"


def _read_mode() -> str:
    """src/ck_int8_patch_thor.py:34-42."""
    m = os.environ.get("CK_INT8_MODE")
    if m:
        return m.strip().lower()
    try:
        with open(MODE_FILE) as f:
            return f.read().strip().lower() or "off"
    except OSError:
        return "off"


def _kitchen_version():
    try:
        from importlib.metadata import version
        return version("comfy-kitchen")
    except Exception:
        return None


def _b200_gemm(x8, w8, x_scale, w_scale, bias, out, stream=None):
    """The replacement kernel: this library's int8 fused-dequant GEMM on `stream`."""
    from . import ops
    return ops.gemm_dequant(x8, w8, x_scale, w_scale, bias, out=out, stream=stream)


_capsule_fn = None
_capsule_tried = False


def _capsule_entry():
    """The compiled capsule fast path (`_t8g_capsule.cutlass_int8_dequant`), or None when the
    module is not built (the general path below then serves every call)."""
    global _capsule_fn, _capsule_tried
    if not _capsule_tried:
        _capsule_tried = True
        try:
            from . import _t8g_capsule
            _capsule_fn = _t8g_capsule.cutlass_int8_dequant
        except ImportError:
            _capsule_fn = None
    return _capsule_fn


def _stream_arg(stream):
    """comfy passes the raw cudaStream_t; anything unusable means torch's current stream."""
    try:
        return None if stream is None else int(stream)
    except (TypeError, ValueError):
        return None


class _CProxy:
    """Stands in for comfy_kitchen.backends.cuda._C and takes over cutlass_int8_dequant
    (src/ck_int8_patch_thor.py:130-168)."""

    def __init__(self, real, gemm=_b200_gemm):
        self._real = real
        self._gemm = gemm
        self._broken = False

    def __getattr__(self, name):
        if name.startswith("_"):
            raise AttributeError(name)
        return getattr(self._real, name)

    def _stock(self, tensors, dtype_code, stream):
        return self._real.cutlass_int8_dequant(*(t.__dlpack__(stream=-1) for t in tensors), dtype_code, stream)

    def cutlass_int8_dequant(self, x, w, x_scale, w_scale, bias, out, dtype_code, stream):
        fast = _capsule_entry() if (self._gemm is _b200_gemm and not self._broken) else None
        if fast is not None:
            # capsules read in place (not consumed): eligible calls launch here, the rest
            # take the general path below
            try:
                if fast(x, w, x_scale, w_scale, bias, out, stream) is True:
                    return True
            except Exception as exc:  # a rejected launch: stock for the rest of the process
                import traceback
                self._broken = True
                print(f"{TAG} B200 GEMM failed ({exc!r:.200}); stock CUTLASS for the rest of this process\n"
                      + traceback.format_exc(), file=sys.stderr, flush=True)
                return self._real.cutlass_int8_dequant(x, w, x_scale, w_scale, bias, out, dtype_code, stream)
        import torch
        tensors = tuple(torch.from_dlpack(t) for t in (x, w, x_scale, w_scale, bias, out))
        tx, tw, txs, tws, tb, tout = tensors
        M, K = tx.shape if tx.dim() == 2 else (0, 0)
        N = tw.shape[0] if tw.dim() == 2 else 0
        # the CUTLASS eligibility the reference mirrors (:148-156); declined calls stay stock
        if (self._broken or M < MIN_M or K % 16
                or not (tx.is_contiguous() and tw.is_contiguous() and tout.is_contiguous())
                or tx.dtype != torch.int8 or tw.dtype != torch.int8
                or tw.dim() != 2 or tw.shape[1] != K or tuple(tout.shape) != (M, N)
                or tout.dtype not in (torch.bfloat16, torch.float16, torch.float32)
                or txs.dtype != torch.float32 or txs.numel() != M
                or tws.dtype != torch.float32 or tws.numel() not in (1, N)
                or tb.numel() not in (0, N) or (tb.numel() and tb.dtype != tout.dtype)):
            return self._stock(tensors, dtype_code, stream)
        try:
            self._gemm(tx, tw, txs, tws, tb, tout, _stream_arg(stream))
        except Exception as exc:  # stay numerically safe: stock for the rest of the process
            import traceback
            self._broken = True
            print(f"{TAG} B200 GEMM failed ({exc!r:.200}); stock CUTLASS for the rest of this process\n"
                  + traceback.format_exc(), file=sys.stderr, flush=True)
            return self._stock(tensors, dtype_code, stream)
        return True


def _apply(mod, mode):
    try:
        _apply_unguarded(mod, mode)
    except Exception as exc:
        print(f"{TAG} NOT applied ({exc!r:.200}); running stock", file=sys.stderr, flush=True)


def _apply_unguarded(mod, mode):
    """Version guard, then swap `_C` (src/ck_int8_patch_thor.py:178-188)."""
    ver = _kitchen_version()
    if ver not in VALIDATED_KITCHEN:
        print(f"{TAG} NOT applied: comfy-kitchen {ver} is not validated "
              f"({', '.join(VALIDATED_KITCHEN)}); running stock", file=sys.stderr, flush=True)
        return
    if mode == "cublas":
        mod._DISABLE_CUTLASS_INT8 = True
    elif mode in KERNEL_MODES:
        if not isinstance(mod._C, _CProxy):
            mod._C = _CProxy(mod._C)
    print(f"{TAG} comfy_kitchen {ver} int8 mode={mode}", file=sys.stderr, flush=True)


def _compile_safe_int8_linear(top):
    """While torch.compile traces, route comfy_kitchen.int8_linear through its
    registered custom op (src/ck_int8_patch_thor.py:191-216); eager calls are untouched."""
    try:
        import torch
        from comfy_kitchen.backends.eager.quantization import DTYPE_CODE_TO_DTYPE
        if _kitchen_version() not in VALIDATED_KITCHEN or getattr(top.int8_linear, "_ck_compile_safe", False):
            return
        code_of = {dt: code for code, dt in DTYPE_CODE_TO_DTYPE.items()}
        eager = top.int8_linear

        def int8_linear(x, weight, weight_scale, bias=None, out_dtype=None, convrot=False,
                        convrot_groupsize=256, input_act=None, input_act_weight=None,
                        input_act_eps=0.0, residual=None, residual_scale=None):
            if torch.compiler.is_compiling():
                return torch.ops.comfy_kitchen.int8_linear(
                    x, weight, weight_scale, bias, code_of[out_dtype or torch.bfloat16],
                    convrot, convrot_groupsize, input_act, input_act_weight, input_act_eps,
                    residual, residual_scale)
            return eager(x, weight, weight_scale, bias, out_dtype, convrot, convrot_groupsize,
                         input_act, input_act_weight, input_act_eps, residual, residual_scale)

        int8_linear._ck_compile_safe = True
        int8_linear.__wrapped__ = eager
        top.int8_linear = int8_linear
    except Exception as exc:
        print(f"{TAG} compile-safe int8_linear NOT applied ({exc!r:.200})", file=sys.stderr, flush=True)


class _Finder(importlib.abc.MetaPathFinder):
    """Applies the patch when comfy-kitchen is imported (src/ck_int8_patch_thor.py:219-240)."""

    def __init__(self, mode):
        self.mode = mode

    def find_spec(self, name, path, target=None):
        if name not in (TARGET, TOP):
            return None
        spec = importlib.machinery.PathFinder.find_spec(name, path)
        if spec is None or spec.loader is None:
            return None
        loader, mode = spec.loader, self.mode
        orig_exec = loader.exec_module

        def exec_module(module):
            orig_exec(module)
            if name == TARGET:
                _apply(module, mode)
            else:
                _compile_safe_int8_linear(module)

        loader.exec_module = exec_module
        return spec


def install():
    """src/ck_int8_patch_thor.py:243-254."""
    mode = _read_mode()
    if mode not in ("off", "cublas") + KERNEL_MODES:
        print(f"{TAG} unknown mode {mode!r} in {MODE_FILE}; running stock", file=sys.stderr, flush=True)
    if mode not in ("cublas",) + KERNEL_MODES:
        return
    if TARGET in sys.modules:
        _apply(sys.modules[TARGET], mode)
    if TOP in sys.modules and hasattr(sys.modules[TOP], "int8_linear"):
        _compile_safe_int8_linear(sys.modules[TOP])
    if TARGET not in sys.modules or TOP not in sys.modules:
        if not any(isinstance(f, _Finder) for f in sys.meta_path):
            sys.meta_path.insert(0, _Finder(mode))


def install_safely():
    try:
        install()
    except Exception as exc:  # never break interpreter start-up
        print(f"{TAG} disabled: {exc!r}", file=sys.stderr)


PTH_NAME = "zz_thor_int8_gemm_b200.pth"


def pth_line() -> str:
    """The single line of the .pth file: boot this package by path and install."""
    boot = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_pth_boot.py")
    return ("import importlib.util as _t8g_u; _t8g_s = _t8g_u.spec_from_file_location('_t8g_pth_boot', "
            f"{boot!r}); _t8g_s.loader.exec_module(_t8g_u.module_from_spec(_t8g_s))")


def write_pth(site_dir: str) -> str:
    """Write the .pth boot file into `site_dir` (a site-packages directory)."""
    path = os.path.join(site_dir, PTH_NAME)
    with open(path, "w") as f:
        f.write(pth_line() + "\n")
    return path
