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
  cluster 2 (on / c2): when fc1 and fc2 hold comfy fp8 QuantizedTensor weights (e4m3 codes
    with one scale, or one per output channel), the whole MLP and the block's gated residual
    run on this library's fp8 GEMMs: fc1 with the SwiGLU in its epilogue and per-token fp8
    quantisation of act (t8g_gemm_fp8_swiglu_quant; fc1's weight, scale and bias interleaved
    in 128-row gate / up blocks once per weight and cached), and fc2
    with x + gate_mlp * y in its epilogue (t8g_gemm_fp8_gated) -- neither fc1's [S, 2F]
    output nor fc2's output reaches memory, and comfy's own fp8 matmul is not called.
    Otherwise (another weight format) fc1 runs as comfy's linear and its bf16 output takes
    the reference's route: SwiGLU + tensorwise fp8 (gate and up read in place,
    t8g_swiglu_quant_tensorwise) -> QuantizedTensor -> fc2.
Unlike the reference (:97-101), a segment whose row is a tensor of per-token rows (inpaint
masks) is accepted: it maps straight into the kernel's row map.
"""
from __future__ import annotations

import traceback

from . import _agent

MODE_FILE = "/etc/ck-fused.mode"
ENV = "CK_FUSED"
TARGET = "comfy.ldm.minimax.model"
VALIDATED_KITCHEN = ("0.2.40",)
TAG = "[ck-fused-patch]"
MODES = ("on", "c1", "c2")

# meta-path finders of the agents are instances of this class
_Finder = _agent.ImportHook


def _read_mode() -> str:
    return _agent.read_mode(ENV, MODE_FILE, aliases={"1": "on"})


def _kitchen_version():
    return _agent.kitchen_version()


def _say(msg: str) -> None:
    _agent.say(TAG, msg)


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
        self._weights = {}   # (id(linear), interleaved) -> (stamp, (codes, scale, bias))

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

    def fp8_weights(self, linear, interleave: bool):
        """(e4m3 codes [N, K], float32 scale [1] or [N], bf16 bias [N] or None) of a linear whose
        weight is a comfy fp8 QuantizedTensor -- gate / up interleaved for the SwiGLU epilogue
        when asked -- or None for any other form.  Built once per weight and cached (keyed by
        the weight's storage and version, so a reloaded weight is rebuilt)."""
        torch = self.torch
        w = getattr(linear, "weight", None)
        if not isinstance(w, self.QT):
            return None
        codes, params = getattr(w, "qdata", None), getattr(w, "params", None)
        scale = getattr(params, "scale", None)
        if not (isinstance(codes, torch.Tensor) and isinstance(scale, torch.Tensor)):
            return None
        if codes.dtype != torch.float8_e4m3fn or codes.dim() != 2 or not codes.is_cuda or codes.shape[1] % 16:
            return None
        N = codes.shape[0]
        if scale.numel() not in (1, N) or (interleave and N % 256):
            return None
        bias = getattr(linear, "bias", None)
        if bias is not None and (not isinstance(bias, torch.Tensor) or bias.numel() != N):
            return None
        stamp = (codes.data_ptr(), codes._version, scale.data_ptr(), None if bias is None else bias.data_ptr())
        key = (id(linear), interleave)
        hit = self._weights.get(key)
        if hit is not None and hit[0] == stamp:
            return hit[1]
        scale = scale.to(device=codes.device, dtype=torch.float32).reshape(-1).contiguous()
        if bias is not None:
            bias = self.mm.cast_to(bias, device=codes.device, dtype=torch.bfloat16).reshape(-1).contiguous()
        codes = codes.contiguous()
        if interleave:
            il = self.ops.interleave_gate_up
            codes = il(codes)
            scale = il(scale) if scale.numel() > 1 else scale
            bias = None if bias is None else il(bias)
        value = (codes, scale, bias)
        self._weights[key] = (stamp, value)
        return value

    def mlp_and_gate(self, mlp, h, x, gate, rows):
        """x + gate[row] * fc2(SwiGLU(fc1(h))) on the library's fp8 GEMMs (cluster 2 with fp8
        weights), or None when the linears are not in that form.  h is cluster 1's fp8
        QuantizedTensor (its one scale given per row) or a bf16 tensor (quantised per token)."""
        torch = self.torch
        fc1 = self.fp8_weights(mlp.fc1, interleave=True)
        fc2 = self.fp8_weights(mlp.fc2, interleave=False)
        if fc1 is None or fc2 is None:
            return None
        (w1, s1, b1), (w2, s2, b2) = fc1, fc2
        S = x.shape[0]
        if isinstance(h, self.QT):
            a = h.qdata
            a_scale = h.params.scale.to(torch.float32).reshape(1).expand(S).contiguous()
        else:
            a, a_scale = self.ops.quant_rows(h.contiguous(), "fp8_e4m3")
        if a.dtype != torch.float8_e4m3fn or tuple(a.shape) != (S, w1.shape[1]) or w2.shape[1] != w1.shape[0] // 2:
            return None
        q, q_scale, _act = self.ops.gemm_swiglu_quant(a.contiguous(), w1, a_scale, s1, b1, kind="fp8_e4m3")
        return self.ops.gemm_gated(q, w2, q_scale, s2, b2, x, gate.to(torch.bfloat16).contiguous(), gate_index=rows)

    # ------------------------------------------------------------------ block
    def forward(self, block, x, t_emb, mod_segments, rope_freqs, transformer_options, attention):
        model = self.model
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = block.adaln_proj(t_emb)
        attn = block.attn if attention is None else attention
        rows = self.row_map(mod_segments, x.shape[0], x.device)
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
        if self.c2:
            done = self.mlp_and_gate(block.mlp, h2, x, gate_mlp, rows)
            if done is not None:
                return done
            out = self.mlp(block.mlp, h2)
        else:
            out = block.mlp(h2)
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
    _agent.when_imported(__name__, {TARGET: lambda module: _apply(module, mode)})


def install_safely() -> None:
    """install(), never raising (interpreter start-up must not break)."""
    try:
        install()
    except Exception as exc:
        _say(f"disabled: {exc!r}")
