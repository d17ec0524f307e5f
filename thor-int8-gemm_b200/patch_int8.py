"""comfy-kitchen INT8 GEMM override: `_C.cutlass_int8_dequant` served by this library's
sm_100a kernel.

A drop-in for the reference agent src/ck_int8_patch_thor.py: the same modes, mode file,
environment variable, comfy-kitchen version guard, eligibility rules, fall-back latch and
stderr tag, loaded the same way -- from a `.pth` file in site-packages (`write_pth`), so
every interpreter of the environment gets it without code changes.

Modes (environment CK_INT8_MODE, else /etc/comfy-kitchen-int8.mode, else "off"):
  off     stock comfy-kitchen
  cublas  comfy-kitchen's own cuBLAS route (sets its `_DISABLE_CUTLASS_INT8`)
  b200    `_C.cutlass_int8_dequant` runs on this library's tcgen05 GEMM
  triton  the reference's name for the kernel mode, accepted so an existing mode file works

Nothing here imports torch or loads the CUDA library until a call needs it; installing
never raises.
"""
from __future__ import annotations

import os

from . import _agent

# The deployment contract of the reference agent (src/ck_int8_patch_thor.py:26-30).
MODE_FILE = "/etc/comfy-kitchen-int8.mode"
ENV = "CK_INT8_MODE"
TARGET = "comfy_kitchen.backends.cuda"
TOP = "comfy_kitchen"
VALIDATED_KITCHEN = ("0.2.37", "0.2.40")
MIN_M = 128
TAG = "[ck-int8-patch]"
KERNEL_MODES = ("b200", "triton")
ACTIVE_MODES = ("cublas",) + KERNEL_MODES
KNOWN_MODES = ("off",) + ACTIVE_MODES

# meta-path finders of the agents are instances of this class
_Finder = _agent.ImportHook


def _say(message: str) -> None:
    _agent.say(TAG, message)


def _read_mode() -> str:
    return _agent.read_mode(ENV, MODE_FILE)


def _kitchen_version():
    return _agent.kitchen_version()


def _b200_gemm(x8, w8, x_scale, w_scale, bias, out, stream=None):
    """The replacement kernel: this library's int8 fused-dequant GEMM on `stream`."""
    from . import ops
    return ops.gemm_dequant(x8, w8, x_scale, w_scale, bias, out=out, stream=stream)


_capsule_fn = None
_capsule_tried = False


def _capsule_entry():
    """The compiled capsule fast path (`_t8g_capsule.cutlass_int8_dequant`), or None when the
    module is not built (the general path then serves every call)."""
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


def _decline_reason(tx, tw, txs, tws, tb, tout):
    """Why this call stays on the stock kernel, or None when this library takes it.

    The rules are the stock CUTLASS kernel's own eligibility, as the reference agent
    mirrors it (src/ck_int8_patch_thor.py:148-156), so that whatever CUTLASS would decline
    (and comfy-kitchen would then route to cuBLAS) keeps its stock route."""
    import torch
    if tx.dim() != 2 or tw.dim() != 2:
        return "x or w is not a matrix"
    (M, K), N = tx.shape, tw.shape[0]
    rules = (
        (M >= MIN_M, f"M={M} below {MIN_M}"),
        (K % 16 == 0, f"K={K} not a multiple of 16"),
        (tx.dtype == torch.int8 and tw.dtype == torch.int8, "x and w must both be int8"),
        (tw.shape[1] == K, "w is not [N, K]"),
        (tx.is_contiguous() and tw.is_contiguous() and tout.is_contiguous(), "x, w and out must be contiguous"),
        (tout.dtype in (torch.bfloat16, torch.float16, torch.float32), f"output dtype {tout.dtype}"),
        (tuple(tout.shape) == (M, N), "out is not [M, N]"),
        (txs.dtype == torch.float32 and txs.numel() == M, "x_scale is not float32 with M elements"),
        (tws.dtype == torch.float32 and tws.numel() in (1, N), "w_scale is not float32 with 1 or N elements"),
        (tb.numel() in (0, N), "bias has neither 0 nor N elements"),
        (tb.numel() == 0 or tb.dtype == tout.dtype, "bias dtype differs from the output dtype"),
    )
    return next((why for ok, why in rules if not ok), None)


class _CProxy:
    """Stands in for comfy_kitchen.backends.cuda._C (src/ck_int8_patch_thor.py:130-168):
    `cutlass_int8_dequant` goes to the B200 GEMM when the call is eligible, every other
    attribute to the real module.  The first failure of the B200 path (an exception from
    the launch) prints a traceback and sends this and every later call to stock."""

    def __init__(self, real, gemm=_b200_gemm):
        self._real = real
        self._gemm = gemm
        self._broken = False
        self._watched = {}   # device index -> the library's host-visible status word

    def _wait_ran_out(self) -> int:
        """The status a kernel of this library recorded when one of its bounded waits ran out
        (0: none), read from the host-visible mirror without synchronising.  A launch whose
        wait gave up has left its output incomplete; comfy has consumed it already, so all
        the proxy can do is stop using the library from the next call on."""
        try:
            import torch
            if not torch.cuda.is_available():
                return 0
            dev = torch.cuda.current_device()
            word = self._watched.get(dev)
            if word is None:
                if torch.cuda.is_current_stream_capturing():
                    return 0                           # set up on a later, uncaptured call
                from . import ops
                word = self._watched[dev] = ops.status_mirror(dev)
            code = word[0]
            if code:
                word[0] = 0
            return code
        except Exception:
            return 0

    def __getattr__(self, name):
        if name.startswith("_"):
            raise AttributeError(name)
        return getattr(self._real, name)

    def _give_up(self, exc) -> None:
        import sys
        import traceback
        self._broken = True
        trace = traceback.format_exc() if sys.exc_info()[0] is not None else ""
        _say(f"B200 GEMM failed ({exc!r:.200}); stock CUTLASS for the rest of this process\n" + trace)

    def _stock(self, tensors, dtype_code, stream):
        return self._real.cutlass_int8_dequant(*(t.__dlpack__(stream=-1) for t in tensors), dtype_code, stream)

    def cutlass_int8_dequant(self, x, w, x_scale, w_scale, bias, out, dtype_code, stream):
        if not self._broken and self._gemm is _b200_gemm:
            code = self._wait_ran_out()
            if code:
                self._give_up(RuntimeError(f"a bounded device wait of the B200 kernels ran out (status {code:#x}); "
                                           "an earlier output of this library may be incomplete"))
        if self._broken:
            return self._real.cutlass_int8_dequant(x, w, x_scale, w_scale, bias, out, dtype_code, stream)
        fast = _capsule_entry() if self._gemm is _b200_gemm else None
        if fast is not None:
            # the capsules are read in place, not consumed: an eligible call launches here,
            # anything else continues below with the same capsules
            try:
                if fast(x, w, x_scale, w_scale, bias, out, stream) is True:
                    return True
            except Exception as exc:
                self._give_up(exc)
                return self._real.cutlass_int8_dequant(x, w, x_scale, w_scale, bias, out, dtype_code, stream)
        import torch
        tensors = tuple(torch.from_dlpack(c) for c in (x, w, x_scale, w_scale, bias, out))
        if _decline_reason(*tensors) is not None:
            return self._stock(tensors, dtype_code, stream)
        try:
            self._gemm(*tensors, _stream_arg(stream))
        except Exception as exc:
            self._give_up(exc)
            return self._stock(tensors, dtype_code, stream)
        return True


def _apply(cuda_backend, mode: str) -> None:
    """Version guard, then the mode's change to comfy_kitchen.backends.cuda; never raises."""
    try:
        ver = _kitchen_version()
        if ver not in VALIDATED_KITCHEN:
            _say(f"NOT applied: comfy-kitchen {ver} is not validated ({', '.join(VALIDATED_KITCHEN)}); running stock")
            return
        if mode == "cublas":
            cuda_backend._DISABLE_CUTLASS_INT8 = True
        elif mode in KERNEL_MODES and not isinstance(cuda_backend._C, _CProxy):
            cuda_backend._C = _CProxy(cuda_backend._C)
        _say(f"comfy_kitchen {ver} int8 mode={mode}")
    except Exception as exc:
        _say(f"NOT applied ({exc!r:.200}); running stock")


def _compile_safe_int8_linear(top) -> None:
    """Make comfy_kitchen.int8_linear traceable by torch.compile (src/ck_int8_patch_thor.py:
    191-216): its eager body exports DLPack capsules, which FakeTensors cannot, so while
    dynamo traces, calls go to comfy-kitchen's registered custom op comfy_kitchen::int8_linear
    (which has a fake kernel) with the output dtype given as comfy's dtype code.  Eager calls
    reach the original function unchanged."""
    if not hasattr(top, "int8_linear"):
        return
    try:
        import functools
        import inspect

        import torch
        from comfy_kitchen.backends.eager.quantization import DTYPE_CODE_TO_DTYPE
        eager = top.int8_linear
        if _kitchen_version() not in VALIDATED_KITCHEN or getattr(eager, "_ck_compile_safe", False):
            return
        signature = inspect.signature(eager)
        order = list(signature.parameters)
        code_of = {dtype: code for code, dtype in DTYPE_CODE_TO_DTYPE.items()}

        @functools.wraps(eager)
        def int8_linear(*args, **kwargs):
            if not torch.compiler.is_compiling():
                return eager(*args, **kwargs)
            call = signature.bind(*args, **kwargs)
            call.apply_defaults()
            values = dict(call.arguments)
            values["out_dtype"] = code_of[values["out_dtype"] or torch.bfloat16]
            return torch.ops.comfy_kitchen.int8_linear(*(values[name] for name in order))

        int8_linear._ck_compile_safe = True
        top.int8_linear = int8_linear
    except Exception as exc:
        _say(f"compile-safe int8_linear NOT applied ({exc!r:.200})")


def install() -> None:
    """Read the mode and hook comfy-kitchen (now, or when it is imported)."""
    mode = _read_mode()
    if mode not in KNOWN_MODES:
        _say(f"unknown mode {mode!r} in {MODE_FILE}; running stock")
    if mode not in ACTIVE_MODES:
        return
    _agent.when_imported(__name__, {TARGET: lambda module: _apply(module, mode), TOP: _compile_safe_int8_linear})


def install_safely() -> None:
    try:
        install()
    except Exception as exc:  # interpreter start-up must not break
        _say(f"disabled: {exc!r}")


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
