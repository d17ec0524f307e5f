"""GPU parity of the row kernels: per-token quantisation, RMSNorm + modulation +
quant, SwiGLU + quant, and the reference's tensorwise two-phase forms, against
the oracle and the reference's own outputs (tests/golden/fused_golden.npz)."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
FUSED = np.load(os.path.join(HERE, "golden", "fused_golden.npz"))
KINDS = {"int8": O.QUANT_INT8, "fp8_e4m3": O.QUANT_FP8}


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from thor_int8_gemm_b200 import ops as _ops
    yield _ops
    assert _ops.device_status() == 0


def bf16_dev(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def to_bf16_bits(x_f32: np.ndarray) -> np.ndarray:
    return O.f32_to_bf16(x_f32)


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def qbits(t: torch.Tensor, kind: str) -> np.ndarray:
    t = t.contiguous().cpu()
    return t.numpy() if kind == "int8" else t.view(torch.uint8).numpy()


def bf16_ulp_diff(a, b):
    a = np.asarray(a, np.uint16).astype(np.int64)
    b = np.asarray(b, np.uint16).astype(np.int64)
    oa = np.where(a & 0x8000, -(a & 0x7FFF), a & 0x7FFF)
    ob = np.where(b & 0x8000, -(b & 0x7FFF), b & 0x7FFF)
    return np.abs(oa - ob)


@pytest.mark.parametrize("kind", ["int8", "fp8_e4m3"])
@pytest.mark.parametrize("S,D", [(1, 8), (7, 3072), (256, 3072), (33, 5376), (20000, 1024), (9, 8192), (9, 8200),
                                 (9, 12288), (3, 24576), (2, 49152)])
def test_quant_rows_bit_exact(ops, kind, S, D):
    rng = np.random.default_rng(S * 31 + D)
    x = O.round_bf16((rng.standard_normal((S, D)) * 3).astype(np.float32))
    x[0, : min(D, 16)] *= 20.0          # outlier channels
    if S > 2:
        x[2] = 0.0                       # amax = 0 row -> scale 1e-12, q = 0
    x = O.round_bf16(x)
    q, s = ops.quant_rows(bf16_dev(to_bf16_bits(x)), kind)
    q_ref, s_ref = O.quant_rows(x, KINDS[kind])
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref)
    np.testing.assert_array_equal(qbits(q, kind), q_ref)


@pytest.mark.parametrize("kind", ["int8", "fp8_e4m3"])
@pytest.mark.parametrize("D", [3072, 12288])
def test_quant_rows_strided_rows(ops, kind, D):
    """Row strides wider than the row on both sides (a column slice of a wider matrix)."""
    S = 300
    rng = np.random.default_rng(D)
    wide = O.round_bf16((rng.standard_normal((S, D + 24)) * 2).astype(np.float32))
    xd = bf16_dev(to_bf16_bits(wide))[:, 8: 8 + D]
    qbuf = torch.zeros(S, D + 40, dtype=torch.int8 if kind == "int8" else torch.float8_e4m3fn, device="cuda")
    q, s = ops.quant_rows(xd, kind, q=qbuf[:, 16: 16 + D])
    q_ref, s_ref = O.quant_rows(wide[:, 8: 8 + D], KINDS[kind])
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref)
    np.testing.assert_array_equal(qbits(q, kind), q_ref)
    np.testing.assert_array_equal(qbits(qbuf[:, :16], kind), 0)     # nothing written outside the slice


@pytest.mark.parametrize("kind", ["int8", "fp8_e4m3"])
@pytest.mark.parametrize("S,D,n_mod,with_w", [(16, 3072, 2, False), (5, 256, 1, True), (40, 5376, 4, True),
                                              (6, 12288, 3, False), (3, 30000 // 8 * 8, 1, False)])
def test_rms_mod_quant_per_token_bit_exact(ops, kind, S, D, n_mod, with_w):
    rng = np.random.default_rng(S + D + n_mod)
    x = O.round_bf16(rng.standard_normal((S, D)).astype(np.float32))
    shift = O.round_bf16((rng.standard_normal((n_mod, D)) * 0.1).astype(np.float32))
    scale = O.round_bf16((rng.standard_normal((n_mod, D)) * 0.1).astype(np.float32))
    w = O.round_bf16((np.abs(rng.standard_normal(D)) + 0.5).astype(np.float32)) if with_w else None
    mod_index = (np.arange(S) * n_mod // S).astype(np.int32)
    q, qs, h, res = ops.rms_mod_quant(bf16_dev(to_bf16_bits(x)), bf16_dev(to_bf16_bits(shift)),
                                      bf16_dev(to_bf16_bits(scale)),
                                      w=None if w is None else bf16_dev(to_bf16_bits(w)),
                                      mod_index=torch.from_numpy(mod_index).cuda(), eps=1e-6, kind=kind,
                                      return_h=True, return_res=True)
    q_ref, qs_ref, h_ref, res_ref = O.rms_mod_quant_per_token(x, shift, scale, w=w, mod_index=mod_index, eps=1e-6,
                                                              kind=KINDS[kind])
    np.testing.assert_array_equal(bits16(h), h_ref)
    np.testing.assert_array_equal(bits16(res), res_ref)
    np.testing.assert_array_equal(qs.cpu().numpy(), qs_ref)
    np.testing.assert_array_equal(qbits(q, kind), q_ref)


@pytest.mark.parametrize("kind", ["int8", "fp8_e4m3"])
@pytest.mark.parametrize("S,D,rows_per_mod", [(5000, 3072, 37), (4000, 1024, 1), (3001, 4096, 1000),
                                              (2500, 1536, 2500), (777, 2048, 100)])
def test_rms_mod_quant_batch_major_rows(ops, kind, S, D, rows_per_mod):
    """The DiT form (no weight, no h/res, rows_per_mod tokens per batch element) at the row
    lengths with register-resident kernels, with batch elements shorter and longer than a
    CTA's block of rows, against the oracle bit for bit."""
    rng = np.random.default_rng(S + D)
    n_mod = -(-S // rows_per_mod)
    x = rng.standard_normal((S, D)).astype(np.float32)
    x[1] *= 1e3
    x = O.round_bf16(x)
    shift = O.round_bf16((rng.standard_normal((n_mod, D)) * 0.1).astype(np.float32))
    scale = O.round_bf16((rng.standard_normal((n_mod, D)) * 0.1).astype(np.float32))
    q, qs = ops.rms_mod_quant(bf16_dev(to_bf16_bits(x)), bf16_dev(to_bf16_bits(shift)), bf16_dev(to_bf16_bits(scale)),
                              rows_per_mod=rows_per_mod, eps=1e-6, kind=kind)
    q_ref, qs_ref, _, _ = O.rms_mod_quant_per_token(x, shift, scale, rows_per_mod=rows_per_mod, eps=1e-6,
                                                    kind=KINDS[kind])
    np.testing.assert_array_equal(qs.cpu().numpy(), qs_ref)
    np.testing.assert_array_equal(qbits(q, kind), q_ref)


def _tie_row(kind, D):
    """A row of D values on the 8-bit format's rounding boundaries (half-integers for int8,
    e4m3 midpoints) and one bf16 ulp either side, tiled, with amax = qmax so the scale is 1."""
    if kind == "int8":
        amax, centres = 127.0, np.arange(-127, 127, dtype=np.float64) + 0.5
    else:
        fin = O._E4M3_FINITE
        mids = (fin[1:] + fin[:-1]) / 2
        amax, centres = 448.0, np.concatenate([mids, -mids])
    vals = O.round_bf16(centres.astype(np.float32))
    row = np.concatenate([vals, O.bf16_to_f32(O.f32_to_bf16(vals) + 1), O.bf16_to_f32(O.f32_to_bf16(vals) - 1)])
    row = row[np.abs(row) <= amax].astype(np.float32)
    out = np.resize(row, D).astype(np.float32)
    out[D // 2] = amax
    return out


@pytest.mark.parametrize("kind", ["int8", "fp8_e4m3"])
@pytest.mark.parametrize("D", [1024, 3072, 2560])
def test_rms_mod_quant_quantiser_ties(ops, kind, D):
    """scale = -1 makes s = bf16(1 + scale) = 0, so h = shift exactly: rows of tie values
    reach the norm kernels' quantiser in every vector slot of the register-resident
    kernels (D = 2560 takes the shared-memory warp kernel)."""
    S = 40
    rng = np.random.default_rng(D)
    x = O.round_bf16(rng.standard_normal((S, D)).astype(np.float32))
    shift = _tie_row(kind, D)[None, :]
    scale = -np.ones((1, D), np.float32)
    q, qs = ops.rms_mod_quant(bf16_dev(to_bf16_bits(x)), bf16_dev(to_bf16_bits(shift)), bf16_dev(to_bf16_bits(scale)),
                              rows_per_mod=S, eps=1e-6, kind=kind)
    q_ref, qs_ref, _, _ = O.rms_mod_quant_per_token(x, shift, scale, rows_per_mod=S, eps=1e-6, kind=KINDS[kind])
    assert np.all(qs_ref == 1.0)
    np.testing.assert_array_equal(qs.cpu().numpy(), qs_ref)
    np.testing.assert_array_equal(qbits(q, kind), q_ref)


def test_rms_mod_quant_config3_full_size(ops):
    """x [2, 56320, 3072] bf16 ~ N(0,1), shift/scale [2, 3072] ~ N(0, 0.1), eps 1e-6,
    fp8 and int8: all rows bit-exact against the oracle (one pass, no h/res)."""
    B, T, D = 2, 56320, 3072
    g = torch.Generator().manual_seed(3)
    x = torch.randn(B * T, D, generator=g).to(torch.bfloat16)
    shift = (torch.randn(B, D, generator=g) * 0.1).to(torch.bfloat16)
    scale = (torch.randn(B, D, generator=g) * 0.1).to(torch.bfloat16)
    xd = x.cuda()
    sh, sc = shift.float().numpy(), scale.float().numpy()
    for kind in ("fp8_e4m3", "int8"):
        q, qs = ops.rms_mod_quant(xd, shift.cuda(), scale.cuda(), rows_per_mod=T, eps=1e-6, kind=kind)
        qh, qsh = qbits(q, kind), qs.cpu().numpy()
        step = 7040                      # rows are independent: check in bounded-memory chunks
        for r0 in range(0, B * T, step):
            xf = x[r0:r0 + step].float().numpy()
            idx = (np.arange(r0, r0 + xf.shape[0]) // T).astype(np.int32)
            q_ref, qs_ref, _, _ = O.rms_mod_quant_per_token(xf, sh, sc, mod_index=idx, eps=1e-6, kind=KINDS[kind])
            np.testing.assert_array_equal(qsh[r0:r0 + step], qs_ref)
            np.testing.assert_array_equal(qh[r0:r0 + step], q_ref)


@pytest.mark.parametrize("i", range(int(FUSED["n_rms"])))
def test_fused_rms_mod_quant_vs_reference_golden(ops, i):
    """The reference-signature fused_rms_mod_quant against the reference's own outputs:
    h, res, the fp8 codes and the one scale, all bit for bit."""
    from thor_int8_gemm_b200.fused import fused_rms_mod_quant
    p = f"r{i}_"
    q, scale, h, res = fused_rms_mod_quant(bf16_dev(FUSED[p + "x"]), bf16_dev(FUSED[p + "w"]),
                                           bf16_dev(FUSED[p + "s"]), bf16_dev(FUSED[p + "b"]),
                                           float(FUSED[p + "eps"]))
    np.testing.assert_array_equal(bits16(h), FUSED[p + "h"])
    np.testing.assert_array_equal(bits16(res), FUSED[p + "res"])
    assert np.float32(scale.item()) == FUSED[p + "scale"][0]
    np.testing.assert_array_equal(qbits(q, "fp8_e4m3"), FUSED[p + "q"])


def test_tensorwise_segments_vs_reference_golden(ops):
    """The per-segment driver (src/ck_fused_patch.py:105-136): two batch segments,
    s = bf16(1 + scale[row]), one global amax -- bit for bit."""
    x = bf16_dev(FUSED["seg_x"])
    S_seg = int(FUSED["seg_rows"])
    q, scale, h, res = ops.rms_mod_quant_tensorwise(x, bf16_dev(FUSED["seg_shift"]), bf16_dev(FUSED["seg_scale"]),
                                                    rows_per_mod=S_seg, eps=1e-6, kind="fp8_e4m3")
    np.testing.assert_array_equal(bits16(h), FUSED["seg_h"])
    np.testing.assert_array_equal(bits16(res), FUSED["seg_res"])
    assert np.float32(scale.item()) == O.scale_from_amax(FUSED["seg_amax"][0], O.QUANT_FP8)
    np.testing.assert_array_equal(qbits(q, "fp8_e4m3"), FUSED["seg_q"])


@pytest.mark.parametrize("kind", ["fp8_e4m3", "int8"])
@pytest.mark.parametrize("S,D,n_mod,with_w", [(37, 256, 1, True), (64, 1000, 2, False), (300, 3072, 3, True),
                                              (40, 5376, 2, True), (17, 8192, 1, False), (9, 8200, 2, True),
                                              (6, 12288, 3, False), (3, 49152, 1, True)])
def test_rms_mod_quant_tensorwise_bit_exact(ops, kind, S, D, n_mod, with_w):
    """The tensorwise form (warp kernel for rows up to 16 KB, CTA kernel beyond) against
    the oracle, whose sum of squares is the reference's order: h, res, the float32 amax
    behind the one scale and every code, bit for bit, with per-token modulation rows."""
    rng = np.random.default_rng(S * 7 + D)
    x = O.round_bf16((rng.standard_normal((S, D)) * 1.5).astype(np.float32))
    x[S // 2, : min(D, 16)] *= 40.0
    x = O.round_bf16(x)
    shift = O.round_bf16((rng.standard_normal((n_mod, D)) * 0.1).astype(np.float32))
    scale = O.round_bf16((rng.standard_normal((n_mod, D)) * 0.1).astype(np.float32))
    w = O.round_bf16((np.abs(rng.standard_normal(D)) + 0.5).astype(np.float32)) if with_w else None
    mod_index = rng.integers(0, n_mod, S).astype(np.int32)
    q, qs, h, res = ops.rms_mod_quant_tensorwise(
        bf16_dev(to_bf16_bits(x)), bf16_dev(to_bf16_bits(shift)), bf16_dev(to_bf16_bits(scale)),
        w=None if w is None else bf16_dev(to_bf16_bits(w)), mod_index=torch.from_numpy(mod_index).cuda(), eps=1e-6,
        kind=kind)
    s_rows = O.mod_multiplier(scale, False)[mod_index]
    b_rows = shift[mod_index]
    x32 = x.astype(np.float32)
    inv = O.rms_inv(O.rms_sum_squares_reference(x32), D, 1e-6)
    h_ref32 = O.rms_mod_h(x32, inv, w, s_rows, b_rows)
    amax = np.float32(np.max(np.abs(h_ref32)))
    h_ref = O.f32_to_bf16(h_ref32)
    np.testing.assert_array_equal(bits16(h), h_ref)
    np.testing.assert_array_equal(bits16(res), O.f32_to_bf16((h_ref32 + x32).astype(np.float32)))
    q_ref, s_ref = O.quant_tensorwise_given(O.bf16_to_f32(h_ref), amax, KINDS[kind])
    assert np.float32(qs.item()) == s_ref
    np.testing.assert_array_equal(qbits(q, kind), q_ref)


@pytest.mark.parametrize("kind", ["fp8_e4m3", "int8"])
@pytest.mark.parametrize("B,T,D,want_res", [(3, 5000, 3072, True), (2, 1500, 4096, True), (5, 97, 1024, False),
                                            (4, 2001, 2048, True), (2, 333, 1536, False), (1, 149, 3072, True)])
def test_rms_mod_quant_tensorwise_dit_form(ops, kind, B, T, D, want_res):
    """The tensorwise form in the DiT layout (no norm weight, s = bf16(1 + scale), batch-major
    tokens): the kernel that caches one batch element's modulation per CTA block, with blocks
    that straddle batch elements (their other rows read the modulation from global memory),
    against the oracle -- h, res, the scale and every code, bit for bit."""
    rng = np.random.default_rng(B * T + D)
    S = B * T
    x = O.round_bf16((rng.standard_normal((S, D)) * 1.5).astype(np.float32))
    x[S // 3, : min(D, 16)] *= 40.0
    x = O.round_bf16(x)
    shift = O.round_bf16((rng.standard_normal((B, D)) * 0.1).astype(np.float32))
    scale = O.round_bf16((rng.standard_normal((B, D)) * 0.1).astype(np.float32))
    q, qs, h, res = ops.rms_mod_quant_tensorwise(
        bf16_dev(to_bf16_bits(x)), bf16_dev(to_bf16_bits(shift)), bf16_dev(to_bf16_bits(scale)), rows_per_mod=T,
        eps=1e-6, kind=kind, want_res=want_res)
    mod_index = np.arange(S) // T
    x32 = x.astype(np.float32)
    inv = O.rms_inv(O.rms_sum_squares_reference(x32), D, 1e-6)
    h_ref32 = O.rms_mod_h(x32, inv, None, O.mod_multiplier(scale, False)[mod_index], shift[mod_index])
    amax = np.float32(np.max(np.abs(h_ref32)))
    h_ref = O.f32_to_bf16(h_ref32)
    np.testing.assert_array_equal(bits16(h), h_ref)
    if want_res:
        np.testing.assert_array_equal(bits16(res), O.f32_to_bf16((h_ref32 + x32).astype(np.float32)))
    else:
        assert res is None
    q_ref, s_ref = O.quant_tensorwise_given(O.bf16_to_f32(h_ref), amax, KINDS[kind])
    assert np.float32(qs.item()) == s_ref
    np.testing.assert_array_equal(qbits(q, kind), q_ref)
    assert ops.device_status() == 0


@pytest.mark.parametrize("kind", ["fp8_e4m3", "int8"])
def test_tensorwise_forms_on_empty_input_give_the_floor_scale(ops, kind):
    """No rows: amax is 0, so the one scale is the 1e-12 floor (the reference's amax and quant
    kernels on an empty tensor); nothing else is written."""
    x = torch.empty(0, 3072, dtype=torch.bfloat16, device="cuda")
    mod = torch.zeros(1, 3072, dtype=torch.bfloat16, device="cuda")
    q, qs, h, res = ops.rms_mod_quant_tensorwise(x, mod, mod, eps=1e-6, kind=kind)
    assert q.shape == (0, 3072) and h.shape == (0, 3072)
    assert np.float32(qs.item()) == O.scale_from_amax(np.float32(0.0), KINDS[kind])
    y = torch.empty(0, 2 * 1024, dtype=torch.bfloat16, device="cuda")
    q, qs, act = ops.swiglu_quant_tensorwise(y[:, :1024], y[:, 1024:], kind=kind)
    assert q.shape == (0, 1024) and act.shape == (0, 1024)
    assert np.float32(qs.item()) == O.scale_from_amax(np.float32(0.0), KINDS[kind])
    assert ops.device_status() == 0


@pytest.mark.parametrize("kind", ["int8", "fp8_e4m3"])
@pytest.mark.parametrize("M,F", [(8, 512), (33, 1536), (64, 12288), (5, 16384), (3, 24576)])
def test_swiglu_quant_per_token(ops, kind, M, F):
    """act, the scales and the codes bit for bit against the oracle (exact sigmoid)."""
    rng = np.random.default_rng(M * F)
    y = O.round_bf16(rng.standard_normal((M, 2 * F)).astype(np.float32) * 2)
    y[0, :8] = [-100.0, -30.0, -0.0, 0.0, 30.0, 88.0, 1e-30, -1e-30]
    y = O.round_bf16(y)
    yd = bf16_dev(to_bf16_bits(y))
    q, qs, act = ops.swiglu_quant_fc1(yd, kind=kind, return_act=True)
    q_ref, qs_ref, act_ref = O.swiglu_quant_per_token(y[:, :F], y[:, F:], KINDS[kind])
    np.testing.assert_array_equal(bits16(act), act_ref)
    np.testing.assert_array_equal(qs.cpu().numpy(), qs_ref)
    np.testing.assert_array_equal(qbits(q, kind), q_ref)


def test_swiglu_every_bf16_gate(ops):
    """act for every bf16 gate value -- subnormals, the window -88.7 < g < -87.3 where the
    sigmoid is subnormal, g < -88.7 where exp(-g) overflows, the table's edges at
    |g| = 2^-25 and 128, the largest magnitudes, infinities and NaNs -- times four up
    values, bit for bit against the oracle (NaN for NaN); the codes too."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    F = 2048
    g = bits.reshape(-1, F)
    ups = np.array([0.5, -1.0, 1e-3, -0.75], np.float32)
    gate = np.concatenate([g] * len(ups))
    up = np.repeat(ups, g.shape[0])[:, None] * np.ones((1, F), np.float32)
    y = np.concatenate([gate, O.f32_to_bf16(up)], axis=1)
    _, _, act = ops.swiglu_quant_fc1(bf16_dev(y), kind="int8", return_act=True)
    act_ref = O.f32_to_bf16(O.silu_mul(O.bf16_to_f32(gate), O.round_bf16(up)))
    got = bits16(act)
    nan_ref = np.isnan(O.bf16_to_f32(act_ref))
    np.testing.assert_array_equal(np.isnan(O.bf16_to_f32(got)), nan_ref)
    np.testing.assert_array_equal(got[~nan_ref], act_ref[~nan_ref])
    # the quantiser end to end on the finite gates
    fin = (bits & 0x7F80) != 0x7F80
    gf = np.zeros(-(-int(fin.sum()) // F) * F, np.uint16)
    gf[: fin.sum()] = bits[fin]
    gf = gf.reshape(-1, F)
    yf = np.concatenate([np.concatenate([gf] * 2), O.f32_to_bf16(np.repeat(ups[:2], gf.shape[0])[:, None]
                                                                   * np.ones((1, F), np.float32))], axis=1)
    q, qs, _ = ops.swiglu_quant_fc1(bf16_dev(yf), kind="int8", return_act=True)
    q_ref, qs_ref, _ = O.swiglu_quant_per_token(O.bf16_to_f32(yf[:, :F]), O.bf16_to_f32(yf[:, F:]), O.QUANT_INT8)
    np.testing.assert_array_equal(qs.cpu().numpy(), qs_ref)
    np.testing.assert_array_equal(qbits(q, "int8"), q_ref)


def test_swiglu_quant_config2_shape(ops):
    """[32768, 24576] fc1 output -> SwiGLU + per-token int8 [32768, 12288], read in place:
    act, scales and codes of 256 sampled rows (tile and tail edges included) bit for bit
    against the oracle -- zero mismatches -- and every row's codes exact given its act."""
    M, F = 32768, 12288
    g = torch.Generator().manual_seed(7)
    y = torch.randn(M, 2 * F, generator=g).to(torch.bfloat16)
    q, qs, act = ops.swiglu_quant_fc1(y.cuda(), kind="int8", return_act=True)
    rng = np.random.default_rng(8)
    rows = np.unique(np.concatenate([[0, 1, 127, 128, 4097, M - 2, M - 1], rng.integers(0, M, 249)]))
    yr = y[torch.from_numpy(rows)].float().numpy()
    q_ref, qs_ref, act_ref = O.swiglu_quant_per_token(yr[:, :F], yr[:, F:], O.QUANT_INT8)
    sel = torch.from_numpy(rows).cuda()
    act_r = bits16(act[sel])
    assert int((act_r != act_ref).sum()) == 0, f"{int((act_r != act_ref).sum())} act mismatches"
    np.testing.assert_array_equal(qs[sel].cpu().numpy(), qs_ref)
    np.testing.assert_array_equal(qbits(q[sel], "int8"), q_ref)
    act_all, qh, qsh = bits16(act), qbits(q, "int8"), qs.cpu().numpy()
    for r0 in range(0, M, 4096):
        q_given, qs_given = O.quant_rows(O.bf16_to_f32(act_all[r0:r0 + 4096]), O.QUANT_INT8)
        np.testing.assert_array_equal(qsh[r0:r0 + 4096], qs_given)
        np.testing.assert_array_equal(qh[r0:r0 + 4096], q_given)


@pytest.mark.parametrize("i", range(int(FUSED["n_swiglu"])))
def test_fused_swiglu_quant_vs_reference_golden(ops, i):
    """The reference-signature fused_swiglu_quant against the reference's own outputs:
    act, the one scale and every fp8 code bit for bit."""
    from thor_int8_gemm_b200.fused import fused_swiglu_quant
    p = f"s{i}_"
    q, scale, act = fused_swiglu_quant(bf16_dev(FUSED[p + "gate"]), bf16_dev(FUSED[p + "up"]))
    np.testing.assert_array_equal(bits16(act), FUSED[p + "act"])
    assert np.float32(scale.item()) == FUSED[p + "scale"][0]
    np.testing.assert_array_equal(qbits(q, "fp8_e4m3"), FUSED[p + "q"])


def test_swiglu_tensorwise_long_rows_vs_oracle(ops):
    """The tensorwise SwiGLU over rows that take the generic kernel and two row groups per
    CTA, against the oracle: act, the float32 amax behind the scale, every code."""
    rng = np.random.default_rng(21)
    for M, F in ((50, 12288), (7, 24576), (300, 1536)):
        gate = O.round_bf16((rng.standard_normal((M, F)) * 3).astype(np.float32))
        up = O.round_bf16(rng.standard_normal((M, F)).astype(np.float32))
        q, qs, act = ops.swiglu_quant_tensorwise(bf16_dev(to_bf16_bits(gate)), bf16_dev(to_bf16_bits(up)))
        q_ref, s_ref, act_ref, _ = O.swiglu_tensorwise(gate, up)
        np.testing.assert_array_equal(bits16(act), act_ref)
        assert np.float32(qs.item()) == s_ref
        np.testing.assert_array_equal(qbits(q, "fp8_e4m3"), q_ref)


def test_row_kernels_reject_bad_shapes(ops):
    from thor_int8_gemm_b200._lib import T8GError
    x = torch.zeros(4, 12, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(T8GError, match="multiple of 8"):
        ops.quant_rows(x)
    x = torch.zeros(2, 49160, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(T8GError, match="exceeds"):
        ops.quant_rows(x)
    y = torch.zeros(2, 2 * 24584, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(T8GError, match="exceeds"):
        ops.swiglu_quant_fc1(y)


def test_bounded_wait_gives_up_and_context_survives(ops):
    """A wait on an mbarrier that nothing completes runs out after its limit,
    the kernel ends with a readable status, and the context keeps working."""
    assert ops.device_status() == 0
    assert ops.wait_selftest(limit_ns=5_000_000) == 1
    assert ops.device_status() == 0x1FF
    assert ops.device_status() == 0
    x = torch.randn(4, 64, device="cuda").to(torch.bfloat16)
    q, s = ops.quant_rows(x)
    torch.cuda.synchronize()
    assert q.shape == (4, 64)


@pytest.mark.parametrize("kind", ["int8", "fp8_e4m3"])
def test_quantiser_ties_and_format_midpoints(ops, kind):
    """Rows whose scale is exactly 1.0 and whose values sit on the rounding
    boundaries of the 8-bit format (half-integers for int8, midpoints between
    neighbouring e4m3 codes, including the subnormal ones), plus values one bf16
    ulp either side: the quantiser must round them exactly like the oracle's IEEE
    divide (ties to even)."""
    if kind == "int8":
        amax = 127.0
        centres = np.arange(-127, 127, dtype=np.float64) + 0.5
    else:
        amax = 448.0
        fin = O._E4M3_FINITE
        mids = (fin[1:] + fin[:-1]) / 2
        centres = np.concatenate([mids, -mids])
    vals = O.round_bf16(centres.astype(np.float32))
    up = O.bf16_to_f32(O.f32_to_bf16(vals) + 1)          # next bf16 away from zero
    dn = O.bf16_to_f32(O.f32_to_bf16(vals) - 1)
    row = np.concatenate([vals, up, dn]).astype(np.float32)
    row = row[np.abs(row) <= amax]
    D = ((row.size + 1 + 7) // 8) * 8
    x = np.zeros((3, D), np.float32)
    x[:, : row.size] = row
    x[:, row.size] = amax                                  # pins the row scale to exactly 1.0
    x[1] = -x[1]
    x[2] = np.roll(x[2], 5)
    q, s = ops.quant_rows(bf16_dev(to_bf16_bits(x)), kind)
    q_ref, s_ref = O.quant_rows(x, KINDS[kind])
    assert np.all(s_ref == 1.0)
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref)
    np.testing.assert_array_equal(qbits(q, kind), q_ref)


def test_row_kernels_deterministic(ops):
    """Repeat calls give identical bits (the reference's repeat check,
    bench/a2_fused_bench.py:127-128), including the tensorwise forms, whose amax is an
    atomic max (order-free)."""
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(6000, 3072, generator=g, device="cuda").to(torch.bfloat16)
    sh = (torch.randn(2, 3072, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    sc = (torch.randn(2, 3072, generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    y = torch.randn(3000, 2 * 2048, generator=g, device="cuda").to(torch.bfloat16)
    calls = [lambda: ops.quant_rows(x, "int8"),
             lambda: ops.rms_mod_quant(x, sh, sc, rows_per_mod=3000, eps=1e-6, kind="fp8_e4m3"),
             lambda: ops.rms_mod_quant_tensorwise(x, sh, sc, rows_per_mod=3000, eps=1e-6, kind="fp8_e4m3")[:3],
             lambda: ops.swiglu_quant_fc1(y, kind="int8"),
             lambda: ops.swiglu_quant_tensorwise(y[:, :2048], y[:, 2048:], kind="fp8_e4m3")]
    for fn in calls:
        a, b = fn(), fn()
        for ta, tb in zip(a, b):
            assert torch.equal(ta.view(torch.uint8) if ta.dtype == torch.float8_e4m3fn else ta,
                               tb.view(torch.uint8) if tb.dtype == torch.float8_e4m3fn else tb)
