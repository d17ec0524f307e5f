"""A stand-in for the parts of ComfyUI the DiT-block agent touches (comfy is not installable
here): comfy.model_management, comfy.quant_ops (fp8 QuantizedTensor with a per-tensor scale)
and comfy.ldm.minimax.model (DiTBlock with adaLN modulation, RMSNorm, an attention stand-in
and a SwiGLU MLP over fp8 linears).  Written as source files into a temporary directory so
the agent's import hook sees a real module import."""
import textwrap

QUANT_OPS = '''
import dataclasses
import torch

F8_MAX = 448.0


class TensorCoreFP8E4M3Layout:
    @dataclasses.dataclass
    class Params:
        scale: torch.Tensor
        orig_dtype: torch.dtype
        orig_shape: tuple


class QuantizedTensor:
    def __init__(self, qdata, layout, params):
        self.qdata, self.layout, self.params = qdata, layout, params

    @classmethod
    def from_float(cls, x):
        scale = (x.float().abs().amax() / F8_MAX).clamp_min(1e-12)
        q = (x.float() / scale).clamp(-F8_MAX, F8_MAX).to(torch.float8_e4m3fn)
        return cls(q, "TensorCoreFP8E4M3Layout",
                   TensorCoreFP8E4M3Layout.Params(scale=scale, orig_dtype=x.dtype, orig_shape=tuple(x.shape)))

    def dequantize(self):
        return (self.qdata.float() * self.params.scale.float()).to(self.params.orig_dtype)
'''

MODEL = '''
import torch
from comfy.quant_ops import QuantizedTensor

CALLS = {"stock": 0}


def _mod_scale_shift(h, shift, scale, mod_segments):
    out = torch.empty_like(h)
    for a, b, row in mod_segments:
        s = 1.0 + scale[row].to(h.dtype)
        out[a:b] = h[a:b] * s + shift[row].to(h.dtype)
    return out


def _mod_gate(x, gate, y, mod_segments):
    out = x.clone()
    for a, b, row in mod_segments:
        out[a:b] = x[a:b] + gate[row].to(x.dtype) * y[a:b]
    return out


class RMSNorm(torch.nn.Module):
    def __init__(self, d, eps=1e-6):
        super().__init__()
        self.weight = torch.nn.Parameter(torch.ones(d, dtype=torch.bfloat16))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight.float()).to(x.dtype)


class QLinear:
    def __init__(self, w, bias):
        self.weight = QuantizedTensor.from_float(w)
        self.bias = bias

    def __call__(self, h):
        hq = h if isinstance(h, QuantizedTensor) else QuantizedTensor.from_float(h)
        y = hq.dequantize().float() @ self.weight.dequantize().float().t() + self.bias.float()
        return y.to(torch.bfloat16)


class MLP:
    def __init__(self, fc1, fc2):
        self.fc1, self.fc2 = fc1, fc2

    def __call__(self, h):
        g, u = self.fc1(h).chunk(2, dim=-1)
        return self.fc2((torch.nn.functional.silu(g.float()) * u.float()).to(torch.bfloat16))


class Attention:
    """Stand-in for attention: the value projection through the output projection."""

    def __init__(self, qkv_proj, out_proj, d):
        self.qkv_proj, self.out_proj, self.d = qkv_proj, out_proj, d

    def __call__(self, h, rope_freqs=None, transformer_options=None):
        return self.out_proj(self.qkv_proj(h)[:, 2 * self.d:].contiguous())


class DiTBlock(torch.nn.Module):
    def __init__(self, d, ffn, device="cpu", seed=0):
        super().__init__()
        g = torch.Generator(device=device).manual_seed(seed)

        def w(n, k):
            return (torch.randn(n, k, generator=g, device=device) * 0.05).to(torch.bfloat16)

        def b(n):
            return (torch.randn(n, generator=g, device=device) * 0.01).to(torch.bfloat16)

        self.d = d
        self.ada = w(6 * d, d)
        self.norm1 = RMSNorm(d).to(device)
        self.norm2 = RMSNorm(d).to(device)
        self.norm2.weight.data = (1.0 + torch.randn(d, generator=g, device=device) * 0.1).to(torch.bfloat16)
        self.attn = Attention(QLinear(w(3 * d, d), b(3 * d)), QLinear(w(d, d), b(d)), d)
        self.mlp = MLP(QLinear(w(2 * ffn, d), b(2 * ffn)), QLinear(w(d, ffn), b(d)))

    def adaln_proj(self, t_emb):
        return [c.contiguous() for c in (t_emb.float() @ self.ada.float().t()).to(torch.bfloat16).chunk(6, dim=-1)]

    def forward(self, x, t_emb, mod_segments, rope_freqs, transformer_options={}, attention=None):
        CALLS["stock"] += 1
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = self.adaln_proj(t_emb)
        attn = self.attn if attention is None else attention
        h1 = _mod_scale_shift(self.norm1(x), shift_msa, scale_msa, mod_segments)
        x = _mod_gate(x, gate_msa, attn(h1, rope_freqs=rope_freqs, transformer_options=transformer_options), mod_segments)
        h2 = _mod_scale_shift(self.norm2(x), shift_mlp, scale_mlp, mod_segments)
        return _mod_gate(x, gate_mlp, self.mlp(h2), mod_segments)
'''


def write_fake_comfy(root):
    pkg = root / "comfy"
    (pkg / "ldm" / "minimax").mkdir(parents=True)
    (pkg / "__init__.py").write_text("")
    (pkg / "model_management.py").write_text(textwrap.dedent('''
        in_training = False
        def cast_to(t, device=None, dtype=None):
            return None if t is None else t.to(device=device, dtype=dtype)
    '''))
    (pkg / "quant_ops.py").write_text(QUANT_OPS)
    (pkg / "ldm" / "__init__.py").write_text("")
    (pkg / "ldm" / "minimax" / "__init__.py").write_text("")
    (pkg / "ldm" / "minimax" / "model.py").write_text(MODEL)
