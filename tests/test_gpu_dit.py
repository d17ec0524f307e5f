"""The DiT block over the library kernels, stage by stage against the oracle.

Each quantised stage is compared with the oracle given the GPU's own input to that
stage (the pinning the reference uses for its fused ops: q exact given h); attention
and the gated residuals are stock torch and are not part of the comparison.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from thor_int8_gemm_b200 import dit, ops
    yield dit, ops
    assert ops.device_status() == 0


def f32(t):
    return t.float().cpu().numpy()


def bits16(t):
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def codes(t):
    t = t.contiguous().cpu()
    return t.numpy() if t.dtype == torch.int8 else t.view(torch.uint8).numpy()


def check_gemm(lin, xq, xs, out):
    ref = O.gemm_i8_dequant(codes(xq), codes(lin.w), xs.cpu().numpy(), lin.ws.cpu().numpy(), f32(lin.bias), "bf16")
    np.testing.assert_array_equal(bits16(out), ref)


@pytest.mark.parametrize("B,T,hidden,heads,ffn", [(2, 64, 256, 2, 512), (1, 300, 384, 3, 1024)])
def test_dit_block_int8_stages_and_composition(mods, B, T, hidden, heads, ffn):
    dit, ops = mods
    M = B * T
    g = torch.Generator(device="cuda").manual_seed(5)
    blk = dit.DiTBlock(hidden, heads, ffn, kind="int8", device="cuda", seed=7)
    x = torch.randn(M, hidden, generator=g, device="cuda").to(torch.bfloat16)
    cond = (torch.randn(B, 6 * hidden, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = blk.modulation(cond)

    q1, s1 = blk.norm_quant(x, shift_msa, scale_msa, T)
    q_ref, s_ref, _, _ = O.rms_mod_quant_per_token(f32(x), f32(shift_msa), f32(scale_msa), rows_per_mod=T,
                                                   eps=blk.eps, kind=O.QUANT_INT8)
    np.testing.assert_array_equal(codes(q1), q_ref)
    np.testing.assert_array_equal(s1.cpu().numpy(), s_ref)

    qkv = blk.qkv(q1, s1)
    check_gemm(blk.qkv, q1, s1, qkv)
    attn = blk.attention(qkv, B).contiguous()
    aq, as_ = ops.quant_rows(attn, "int8")
    q_ref, s_ref = O.quant_rows(f32(attn), O.QUANT_INT8)
    np.testing.assert_array_equal(codes(aq), q_ref)
    o = blk.proj(aq, as_)
    check_gemm(blk.proj, aq, as_, o)
    x2 = blk.gated(x, gate_msa, o, B)

    q2, s2 = blk.norm_quant(x2, shift_mlp, scale_mlp, T)
    q_ref, s_ref, _, _ = O.rms_mod_quant_per_token(f32(x2), f32(shift_mlp), f32(scale_mlp), rows_per_mod=T,
                                                   eps=blk.eps, kind=O.QUANT_INT8)
    np.testing.assert_array_equal(codes(q2), q_ref)
    y = blk.fc1(q2, s2)
    check_gemm(blk.fc1, q2, s2, y)
    q3, s3, act = ops.swiglu_quant_fc1(y, kind="int8", return_act=True)
    F = ffn
    q_ref, s_ref, act_ref = O.swiglu_quant_per_token(f32(y[:, :F]), f32(y[:, F:]), O.QUANT_INT8)
    np.testing.assert_array_equal(bits16(act), act_ref)
    np.testing.assert_array_equal(codes(q3), q_ref)
    z = blk.fc2(q3, s3)
    check_gemm(blk.fc2, q3, s3, z)
    x3 = blk.gated(x2, gate_mlp, z, B)

    # the block's forward is exactly this composition
    assert torch.equal(blk(x, cond, B), x3)


def test_dit_block_fp8_runs_close_to_int8(mods):
    dit, ops = mods
    B, T, hidden, heads, ffn = 2, 128, 256, 2, 512
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(B * T, hidden, generator=g, device="cuda").to(torch.bfloat16)
    cond = (torch.randn(B, 6 * hidden, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    y8 = dit.DiTBlock(hidden, heads, ffn, kind="int8", device="cuda", seed=3)(x, cond, B).float()
    yf = dit.DiTBlock(hidden, heads, ffn, kind="fp8_e4m3", device="cuda", seed=3)(x, cond, B).float()
    assert torch.isfinite(yf).all()
    rel = (yf - y8).norm() / y8.norm()
    assert rel < 0.05, float(rel)


@pytest.mark.parametrize("kind", ["int8", "fp8_e4m3"])
def test_dit_block_fused_mlp_matches(mods, kind):
    """fc1 with the SwiGLU in its epilogue gives the unfused block's output bit for bit (int8)
    and within one bf16 ulp through the block (fp8: fp32 accumulation order)."""
    dit, ops = mods
    B, T, hidden, heads, ffn = 2, 96, 256, 2, 512
    g = torch.Generator(device="cuda").manual_seed(12)
    x = torch.randn(B * T, hidden, generator=g, device="cuda").to(torch.bfloat16)
    cond = (torch.randn(B, 6 * hidden, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    plain = dit.DiTBlock(hidden, heads, ffn, kind=kind, device="cuda", seed=21)
    fused = dit.DiTBlock(hidden, heads, ffn, kind=kind, device="cuda", seed=21, fused_mlp=True)
    a, b = plain(x, cond, B), fused(x, cond, B)
    if kind == "int8":
        assert torch.equal(a, b)
    else:
        assert O.bf16_ulp_distance(bits16(a), bits16(b)).max() <= 2


@pytest.mark.parametrize("B,T,fused_mlp", [(2, 96, False), (2, 96, True), (1, 100, True), (3, 200, False)])
def test_dit_block_fused_gate_matches(mods, B, T, fused_mlp):
    """proj and fc2 with the gated residual in their epilogue give the stock block's output
    bit for bit (int8), and leave the caller's x untouched."""
    dit, ops = mods
    hidden, heads, ffn = 256, 2, 512
    g = torch.Generator(device="cuda").manual_seed(B * T)
    x = torch.randn(B * T, hidden, generator=g, device="cuda").to(torch.bfloat16)
    x0 = x.clone()
    cond = (torch.randn(B, 6 * hidden, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    plain = dit.DiTBlock(hidden, heads, ffn, kind="int8", device="cuda", seed=31)
    fused = dit.DiTBlock(hidden, heads, ffn, kind="int8", device="cuda", seed=31, fused_mlp=fused_mlp,
                         fused_gate=True)
    assert torch.equal(plain(x, cond, B), fused(x, cond, B))
    assert torch.equal(x, x0)
