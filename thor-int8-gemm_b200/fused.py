"""Drop-in mirror of the reference's fused-op module `ck_fused_mod_norm_quant`
(src/ck_fused_mod_norm_quant.py): same function names, arguments and return
values, computed by this library's sm_100a kernels.

    from thor_int8_gemm_b200.fused import fused_rms_mod_quant, fused_swiglu_quant

The reference's launch-tuning keyword arguments (BLOCK_K, num_warps, QBLOCK,
q_num_warps, BLOCK) are accepted and ignored: the launch shape here is fixed by
the row length.
"""
from __future__ import annotations

import torch

from . import ops

F8_E4M3_MAX = 448.0   # src/ck_fused_mod_norm_quant.py:19


def _make_scale(amax: torch.Tensor) -> torch.Tensor:
    """amax -> max(amax / 448, 1e-12) (src/ck_fused_mod_norm_quant.py:114-118)."""
    return (amax / F8_E4M3_MAX).clamp_min(1e-12)


def fused_rms_mod_quant(x: torch.Tensor, w: torch.Tensor, s: torch.Tensor, b: torch.Tensor,
                        eps: float = 1e-5, **launch_tuning):
    """rms_norm(x) * w * s + b, residual h + x, tensorwise fp8 quantisation.

    Mirrors src/ck_fused_mod_norm_quant.py:121-145: x [S, K] bf16, w/s/b [K] bf16
    (s is the multiplier itself); returns (q fp8 [S, K], scale 0-d fp32,
    h bf16 [S, K], res bf16 [S, K]).
    """
    del launch_tuning
    return ops.rms_mod_quant_tensorwise(x, b, s, w=w, rows_per_mod=x.shape[0], scale_is_multiplier=True,
                                        eps=eps, kind="fp8_e4m3", want_res=True)


def fused_swiglu_quant(gate: torch.Tensor, up: torch.Tensor, **launch_tuning):
    """silu(gate) * up with tensorwise fp8 quantisation.

    Mirrors src/ck_fused_mod_norm_quant.py:148-167: returns (q fp8, scale 0-d fp32,
    act bf16).  Like the reference it requires gate.shape == up.shape; unlike it,
    gate and up may be strided row views (for example the halves of the fc1
    output) as long as they share their strides.
    """
    del launch_tuning
    assert gate.shape == up.shape, "gate and up must have the same shape"
    shape = gate.shape
    g2 = gate.reshape(-1, shape[-1]) if gate.dim() != 2 else gate
    u2 = up.reshape(-1, shape[-1]) if up.dim() != 2 else up
    q, scale, act = ops.swiglu_quant_tensorwise(g2, u2, kind="fp8_e4m3")
    return q.reshape(shape), scale, act.reshape(shape)
