"""A DiT block whose linear layers and norm/quant ops run on this library's kernels.

Shapes follow the synthetic DiT the workload describes (hidden 3072, 24 heads of 128,
SwiGLU FFN 12288, adaLN modulation from a [B, 6*hidden] conditioning vector); weights are
random-init N(0, 0.02) and quantised per output channel.  The data flow is the
reference's fused block (src/ck_fused_patch.py:152-172) with per-token quantisation:

    h1  = rms_norm(x) * (1 + scale_msa) + shift_msa     -> int8/fp8 + per-token scale
    qkv = h1 @ Wqkv^T (fused dequant GEMM)               -> SDPA (torch, outside the hot path)
    o   = quant(attn) @ Wproj^T;  x += gate_msa * o       (gated residual: stock torch, or
                                                          the GEMM's epilogue, fused_gate)
    h2  = rms_norm(x) * (1 + scale_mlp) + shift_mlp     -> int8/fp8 + per-token scale
    y   = h2 @ Wfc1^T  [M, 2F];  a = quant(silu(y[:, :F]) * y[:, F:]) (read in place)
    z   = a @ Wfc2^T;  x += gate_mlp * z

Tokens are laid out batch-major ([B*T, hidden]); `tokens_per_batch` maps every token to
its batch element's modulation row.  Multi-GPU runs shard the token dimension (see
`shard.py`): weights and conditioning are replicated and no collective is needed.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import ops


class QuantLinear:
    """A linear layer with a per-output-channel quantised weight [N, K]."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None, kind: str = "int8"):
        if weight.dtype != torch.bfloat16:
            weight = weight.to(torch.bfloat16)
        self.kind = kind
        self.w, self.ws = ops.quant_rows(weight.contiguous(), kind)
        self.bias = None if bias is None else bias.to(torch.bfloat16).contiguous()
        self.out_features, self.in_features = weight.shape

    def __call__(self, xq: torch.Tensor, xs: torch.Tensor, out: torch.Tensor | None = None, stream=None):
        return ops.gemm_dequant(xq, self.w, xs, self.ws, self.bias, out=out, stream=stream)


class DiTBlock:
    """Synthetic DiT block (see module docstring)."""

    def __init__(self, hidden: int = 3072, heads: int = 24, ffn: int = 12288, kind: str = "int8",
                 device=None, seed: int = 0, eps: float = 1e-6, fused_mlp: bool = False,
                 fused_gate: bool = False):
        if hidden % heads:
            raise ValueError("hidden must be a multiple of heads")
        self.hidden, self.heads, self.ffn, self.kind, self.eps = hidden, heads, ffn, kind, eps
        device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=device)
        g.manual_seed(seed)

        def w(n, k):
            return (torch.randn(n, k, generator=g, device=device) * 0.02).to(torch.bfloat16)

        def b(n):
            return (torch.randn(n, generator=g, device=device) * 0.01).to(torch.bfloat16)

        self.qkv = QuantLinear(w(3 * hidden, hidden), b(3 * hidden), kind)
        self.proj = QuantLinear(w(hidden, hidden), b(hidden), kind)
        self.fc1 = QuantLinear(w(2 * ffn, hidden), b(2 * ffn), kind)
        self.fc2 = QuantLinear(w(hidden, ffn), b(hidden), kind)
        # fused_mlp: fc1 with the SwiGLU in its epilogue (gate / up rows interleaved once), which
        # also reports each row's max |act| so that act is quantised as a plain stream
        self.fused_mlp = fused_mlp
        # fused_gate: proj and fc2 apply the gated residual in their epilogue (gemm_gated)
        self.fused_gate = fused_gate
        if fused_mlp:
            il = ops.interleave_gate_up
            self.fc1_il = (il(self.fc1.w), il(self.fc1.ws), il(self.fc1.bias))

    def modulation(self, cond: torch.Tensor):
        """Split the conditioning [B, 6*hidden] into shift/scale/gate for attention and MLP."""
        return [c.contiguous() for c in cond.to(torch.bfloat16).chunk(6, dim=-1)]

    def norm_quant(self, x, shift, scale, tokens_per_batch):
        return ops.rms_mod_quant(x, shift, scale, rows_per_mod=tokens_per_batch, eps=self.eps, kind=self.kind)

    def attention(self, qkv: torch.Tensor, batch: int) -> torch.Tensor:
        M = qkv.shape[0]
        T = M // batch
        hd = self.hidden // self.heads
        q, k, v = qkv.view(batch, T, 3, self.heads, hd).permute(2, 0, 3, 1, 4)
        o = F.scaled_dot_product_attention(q, k, v)
        return o.transpose(1, 2).reshape(M, self.hidden)

    @staticmethod
    def gated(x, gate, y, batch):
        """x + gate[b] * y per batch element (the stock gated residual)."""
        M, H = x.shape
        return (x.view(batch, M // batch, H) + gate.view(batch, 1, H) * y.view(batch, M // batch, H)).view(M, H)

    def linears_and_norms(self, x, cond, batch, attn_fn=None):
        """The block with a pluggable attention (default: torch SDPA); returns the new x."""
        T = x.shape[0] // batch
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = self.modulation(cond)
        q1, s1 = self.norm_quant(x, shift_msa, scale_msa, T)
        qkv = self.qkv(q1, s1)
        attn = (attn_fn or self.attention)(qkv, batch)
        # the quantiser takes row-strided input; only a non-unit inner stride needs a copy
        aq, as_ = ops.quant_rows(attn if attn.stride(-1) == 1 else attn.contiguous(), self.kind)
        if self.fused_gate:
            p = self.proj
            x = ops.gemm_gated(aq, p.w, as_, p.ws, p.bias, x, gate_msa, rows_per_gate=T)
        else:
            x = self.gated(x, gate_msa, self.proj(aq, as_), batch)
        q2, s2 = self.norm_quant(x, shift_mlp, scale_mlp, T)
        if self.fused_mlp:
            w_il, ws_il, b_il = self.fc1_il
            q3, s3, _ = ops.gemm_swiglu_quant(q2, w_il, s2, ws_il, b_il, kind=self.kind)
        else:
            y = self.fc1(q2, s2)
            q3, s3 = ops.swiglu_quant_fc1(y, kind=self.kind)
        if self.fused_gate:
            f = self.fc2
            # x is this block's own tensor here: update it in place
            return ops.gemm_gated(q3, f.w, s3, f.ws, f.bias, x, gate_mlp, rows_per_gate=T, out=x)
        return self.gated(x, gate_mlp, self.fc2(q3, s3), batch)

    def __call__(self, x: torch.Tensor, cond: torch.Tensor, batch: int) -> torch.Tensor:
        return self.linears_and_norms(x, cond, batch)

    def linear_ops(self, M: int) -> float:
        """Integer/float ops of the four GEMMs for M tokens (2*M*N*K each)."""
        h, f = self.hidden, self.ffn
        return 2.0 * M * (3 * h * h + h * h + 2 * f * h + h * f)
