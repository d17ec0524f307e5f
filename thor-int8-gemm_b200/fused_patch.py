"""DiT-block agent: ComfyUI's MiniMax-H3 `DiTBlock.forward` over this library's fused kernels.

It plays the part of the reference's fused-layer agent (src/ck_fused_patch.py) with the same
switches; the package's one `.pth` boot line (`patch_int8.write_pth`) installs it next to the
`_C` proxy, so a deployment replaces both reference agents with that line:
  * mode from the environment variable CK_FUSED ("1" means "on") or /etc/ck-fused.mode:
    off (default: nothing imported or patched), on (both clusters), c1, c2 (:4-10, :45-54);
  * target `comfy.ldm.minimax.model.DiTBlock.forward`, patched when that module is imported
    (a meta-path hook) or at once if it already is (:206-243);
  * comfy-kitchen must be a validated version (:41, :231-235); stderr tag [ck-fused-patch];
  * an ineligible call or any failure runs the captured stock forward, a failure for the rest
    of the process with a one-shot warning (:83-101, :179-185, :196-203).

What the fused forward runs (the block's call order is the stock one, :153-172):
  cluster 1 (on / c1): norm1 / norm2, (1 + scale) * h + shift of each batch segment and one
    tensorwise fp8 quantisation of the whole packed sequence -- one launch pair
    (t8g_rms_mod_quant_tensorwise) for all segments through a per-token modulation-row map
    -- handed to qkv_proj / fc1 as comfy's fp8 QuantizedTensor, so they skip their own
    quantisation;
  cluster 2 (on / c2): fc1's bf16 output -> SwiGLU + tensorwise fp8 (gate and up read in
    place, t8g_swiglu_quant_tensorwise) -> QuantizedTensor -> fc2.
Unlike the reference (:97-101), a segment whose row is a tensor of per-token rows (inpaint
masks) is accepted: it maps straight into the kernel's row map.
"""
from __future__ import annotations

import importlib.abc
import importlib.machinery
import os
import sys
import traceback

MODE_FILE = "/etc/ck-fused.mode"
ENV = "CK_FUSED"
TARGET = "comfy.ldm.minimax.model"
VALIDATED_KITCHEN = ("0.2.40",)
TAG = "[ck-fused-patch]"
MODES = ("on", "c1", "c2")


def _read_mode() -> str:
    env = os.environ.get(ENV)
    if env:
        env = env.strip().lower()
        return "on" if env == "1" else env
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


def _say(msg: str) -> None:
    print(f"{TAG} {msg}", file=sys.stderr, flush=True)


class _Runtime:
    """Kernels and comfy handles, bound once the target module has been imported."""

    def __init__(self, model_mod, mode: str):
        import torch
        import comfy.model_management as mm
        from comfy.quant_ops import QuantizedTensor, TensorCoreFP8E4M3Layout
        from . import ops
        self.torch, self.ops, self.mm = torch, ops, mm
        self.QT, self.Layout = QuantizedTensor, TensorCoreFP8E4M3Layout
        self.model = model_mod
        self.c1 = mode in ("on", "c1")
        self.c2 = mode in ("on", "c2")
        self.broken = False
        self.warned = False

    # ------------------------------------------------------------------ eligibility
    def eligible(self, block, x, mod_segments) -> bool:
        torch = self.torch
        if self.broken or getattr(self.mm, "in_training", False):
            return False
        if x.dim() != 2 or not x.is_cuda or x.dtype != torch.bfloat16 or not x.is_contiguous():
            return False
        if self.c1 and not (isinstance(block.attn.qkv_proj.weight, self.QT) and isinstance(block.mlp.fc1.weight, self.QT)):
            return False
        if self.c2 and not isinstance(block.mlp.fc2.weight, self.QT):
            return False
        for a, b, row in mod_segments:
            if isinstance(row, int):
                continue
            if not (isinstance(row, torch.Tensor) and row.dim() == 1 and row.numel() == b - a
                    and not row.is_floating_point()):
                return False
        return True

    def row_map(self, mod_segments, S: int, device):
        """The modulation row of every token of the packed sequence (int32 [S])."""
        torch = self.torch
        rows = torch.empty(S, dtype=torch.int32, device=device)
        covered = 0
        for a, b, row in mod_segments:
            if isinstance(row, int):
                rows[a:b] = row
            else:
                rows[a:b] = row.to(device=device, dtype=torch.int32)
            covered += b - a
        if covered != S:
            raise ValueError(f"mod_segments cover {covered} of {S} tokens")
        return rows

    # ------------------------------------------------------------------ cluster 1
    def norm_quant(self, norm, x, shift, scale, rows):
        """rms_norm(x, w) * bf16(1 + scale[row]) + shift[row] for every token, quantised to
        fp8 with one scale for the tensor; returned as the comfy fp8 QuantizedTensor."""
        torch = self.torch
        w = self.mm.cast_to(norm.weight, device=x.device)
        if w is not None:
            w = w.to(torch.bfloat16).contiguous()
        q, qscale, _h, _res = self.ops.rms_mod_quant_tensorwise(
            x, shift.to(torch.bfloat16).contiguous(), scale.to(torch.bfloat16).contiguous(), w=w, mod_index=rows,
            eps=float(norm.eps), kind="fp8_e4m3", want_res=False)
        params = self.Layout.Params(scale=qscale, orig_dtype=x.dtype, orig_shape=tuple(x.shape))
        return self.QT(q, "TensorCoreFP8E4M3Layout", params)

    # ------------------------------------------------------------------ cluster 2
    def mlp(self, mlp, h):
        y = mlp.fc1(h)
        F = y.shape[-1] // 2
        q, qscale, _act = self.ops.swiglu_quant_tensorwise(y[:, :F], y[:, F:], kind="fp8_e4m3")
        params = self.Layout.Params(scale=qscale, orig_dtype=y.dtype, orig_shape=(y.shape[0], F))
        return mlp.fc2(self.QT(q, "TensorCoreFP8E4M3Layout", params))

    # ------------------------------------------------------------------ block
    def forward(self, block, x, t_emb, mod_segments, rope_freqs, transformer_options, attention):
        model = self.model
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = block.adaln_proj(t_emb)
        attn = block.attn if attention is None else attention
        rows = self.row_map(mod_segments, x.shape[0], x.device) if self.c1 else None
        if self.c1:
            h1 = self.norm_quant(block.norm1, x, shift_msa, scale_msa, rows)
        else:
            h1 = model._mod_scale_shift(block.norm1(x), shift_msa, scale_msa, mod_segments)
        x = model._mod_gate(x, gate_msa, attn(h1, rope_freqs=rope_freqs, transformer_options=transformer_options),
                            mod_segments)
        if self.c1:
            h2 = self.norm_quant(block.norm2, x, shift_mlp, scale_mlp, rows)
        else:
            h2 = model._mod_scale_shift(block.norm2(x), shift_mlp, scale_mlp, mod_segments)
        out = self.mlp(block.mlp, h2) if self.c2 else block.mlp(h2)
        return model._mod_gate(x, gate_mlp, out, mod_segments)

    def fail(self, exc) -> None:
        self.broken = True
        if not self.warned:
            self.warned = True
            _say(f"fused path failed ({exc!r:.200}); stock DiTBlock for the rest of this process\n"
                 + traceback.format_exc())


def _apply(mod, mode: str) -> None:
    try:
        import comfy.model_management  # noqa: F401  (comfy core present)
        if not all(hasattr(mod, n) for n in ("DiTBlock", "_mod_scale_shift", "_mod_gate", "MLP")):
            _say("NOT applied: comfy.ldm.minimax.model layout not recognized; running stock")
            return
        if getattr(mod.DiTBlock.forward, "_t8g_fused", False):
            return
        rt = _Runtime(mod, mode)
        stock = mod.DiTBlock.forward

        def forward(self, x, t_emb, mod_segments, rope_freqs, transformer_options={}, attention=None):
            if not rt.broken and rt.eligible(self, x, mod_segments):
                try:
                    return rt.forward(self, x, t_emb, mod_segments, rope_freqs, transformer_options, attention)
                except Exception as exc:
                    rt.fail(exc)
            return stock(self, x, t_emb, mod_segments, rope_freqs, transformer_options=transformer_options,
                         attention=attention)

        forward._t8g_fused = True
        forward.__wrapped__ = stock
        forward._t8g_runtime = rt
        mod.DiTBlock.forward = forward
        _say(f"comfy-kitchen {_kitchen_version()} H3 DiTBlock fused on B200 kernels mode={mode} "
             f"(c1={rt.c1} c2={rt.c2})")
    except Exception as exc:
        _say(f"NOT applied ({exc!r:.200}); running stock")


class _Finder(importlib.abc.MetaPathFinder):
    """Patches the target module right after it executes."""

    def __init__(self, mode: str):
        self.mode = mode

    def find_spec(self, name, path, target=None):
        if name != TARGET:
            return None
        spec = importlib.machinery.PathFinder.find_spec(name, path)
        if spec is None or spec.loader is None:
            return None
        loader, mode = spec.loader, self.mode
        run = loader.exec_module

        def exec_module(module):
            run(module)
            _apply(module, mode)

        loader.exec_module = exec_module
        return spec


def install() -> None:
    mode = _read_mode()
    if mode not in MODES:
        if mode not in ("off", ""):
            _say(f"unknown mode {mode!r}; running stock")
        return
    ver = _kitchen_version()
    if ver not in VALIDATED_KITCHEN:
        _say(f"NOT applied: comfy-kitchen {ver} is not validated ({', '.join(VALIDATED_KITCHEN)}); running stock")
        return
    if TARGET in sys.modules:
        _apply(sys.modules[TARGET], mode)
    elif not any(isinstance(f, _Finder) for f in sys.meta_path):
        sys.meta_path.insert(0, _Finder(mode))


def install_safely() -> None:
    """install(), never raising (interpreter start-up must not break)."""
    try:
        install()
    except Exception as exc:
        _say(f"disabled: {exc!r}")
