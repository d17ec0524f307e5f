"""The oracle against the reference's own outputs (tests/golden/*.npz).

The goldens were produced by tests/golden/make_golden.py from the reference
implementation: `_gemm_intmm` (src/ck_int8_patch_intmm.py:63-71) and the Triton
kernels of src/ck_int8_patch_thor.py and src/ck_fused_mod_norm_quant.py.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GEMM = np.load(os.path.join(HERE, "golden", "gemm_golden.npz"))
FUSED = np.load(os.path.join(HERE, "golden", "fused_golden.npz"))


def bf16_ulp_diff(a_bits, b_bits):
    a = np.asarray(a_bits, np.uint16).astype(np.int64)
    b = np.asarray(b_bits, np.uint16).astype(np.int64)
    oa = np.where(a & 0x8000, -(a & 0x7FFF), a & 0x7FFF)
    ob = np.where(b & 0x8000, -(b & 0x7FFF), b & 0x7FFF)
    return np.abs(oa - ob)


def f32_ulp_diff(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)


@pytest.mark.parametrize("i", range(int(GEMM["n_cases"])))
def test_gemm_matches_reference_bit_exact(i):
    p = f"g{i}_"
    M, N, K, hb, scalar_ws = GEMM[p + "meta"]
    dt = str(GEMM[p + "dtype"])
    out = O.gemm_i8_dequant(GEMM[p + "x8"], GEMM[p + "w8"], GEMM[p + "xs"], GEMM[p + "ws"],
                            GEMM[p + "bias"] if hb else None, dt)
    assert out.shape == (M, N)
    np.testing.assert_array_equal(out, GEMM[p + "out"])


def test_int_matmul_matches_int64():
    rng = np.random.default_rng(0)
    a = rng.integers(-128, 128, (37, 80)).astype(np.int8)
    w = rng.integers(-128, 128, (29, 80)).astype(np.int8)
    ref = a.astype(np.int64) @ w.astype(np.int64).T
    np.testing.assert_array_equal(O.int_matmul_nt(a, w), ref.astype(np.int32))


def test_e4m3_conversion_matches_torch_rne():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(1)
    vals = [rng.standard_normal(20000).astype(np.float32) * s for s in (1e-3, 0.05, 1.0, 30.0, 200.0)]
    # every representable value and every midpoint between neighbours (ties)
    fin = O._E4M3_FINITE.astype(np.float32)
    mids = ((O._E4M3_FINITE[1:] + O._E4M3_FINITE[:-1]) / 2).astype(np.float32)
    vals += [fin, -fin, mids, -mids, np.array([0.0, -0.0, 448.0, -448.0], np.float32)]
    v = np.concatenate(vals)
    v = np.clip(v, -448, 448).astype(np.float32)
    ref = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(O.f32_to_e4m3(v), ref)
    np.testing.assert_array_equal(O.e4m3_to_f32(ref), torch.from_numpy(ref).view(torch.float8_e4m3fn).float().numpy())


def test_bf16_rounding_matches_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(2)
    v = np.concatenate([rng.standard_normal(50000).astype(np.float32) * 10.0 ** e for e in range(-30, 30, 6)])
    ref = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(O.f32_to_bf16(v), ref)


@pytest.mark.parametrize("i", range(int(FUSED["n_rms"])))
def test_rms_mod_tensorwise_vs_reference(i):
    """The whole reference call bit for bit: h, res, the fp8 codes and the one scale
    (the sum of squares follows the reference's own order)."""
    p = f"r{i}_"
    x = O.bf16_to_f32(FUSED[p + "x"])
    w, s, b = (O.bf16_to_f32(FUSED[p + k]) for k in "wsb")
    eps = float(FUSED[p + "eps"])
    q, scale, h, res, amax = O.rms_mod_res_tensorwise(x, w, s, b, eps)
    np.testing.assert_array_equal(h, FUSED[p + "h"])
    np.testing.assert_array_equal(res, FUSED[p + "res"])
    assert f32_ulp_diff(scale, FUSED[p + "scale"]).max() == 0
    np.testing.assert_array_equal(q, FUSED[p + "q"])
    if not np.any(FUSED[p + "x"]):
        # amax = 0 -> scale = 1e-12 (bench/a3p_device_scale_test.py:119-135)
        assert FUSED[p + "scale"][0] == np.float32(1e-12) == scale
        assert not np.any(FUSED[p + "q"] & 0x7F)


def test_rms_mod_segments_vs_reference():
    """The per-segment driver of src/ck_fused_patch.py:105-136 with s = bf16(1+scale):
    h, res, the shared float32 amax and the codes bit for bit."""
    x = O.bf16_to_f32(FUSED["seg_x"])
    shift = O.bf16_to_f32(FUSED["seg_shift"])
    scale_mod = O.bf16_to_f32(FUSED["seg_scale"])
    S_seg = int(FUSED["seg_rows"])
    rows = np.arange(x.shape[0]) // S_seg
    s = O.mod_multiplier(scale_mod, False)[rows]
    b = shift[rows]
    q, scale, h, res, amax = O.rms_mod_res_tensorwise(x, None, s, b, 1e-6)
    np.testing.assert_array_equal(h, FUSED["seg_h"])
    np.testing.assert_array_equal(res, FUSED["seg_res"])
    assert f32_ulp_diff(amax, FUSED["seg_amax"]).max() == 0
    np.testing.assert_array_equal(q, FUSED["seg_q"])


@pytest.mark.parametrize("i", range(int(FUSED["n_swiglu"])))
def test_swiglu_tensorwise_vs_reference(i):
    """act, the fp8 codes and the scale bit for bit."""
    p = f"s{i}_"
    g = O.bf16_to_f32(FUSED[p + "gate"])
    u = O.bf16_to_f32(FUSED[p + "up"])
    q, scale, act, amax = O.swiglu_tensorwise(g, u)
    np.testing.assert_array_equal(act, FUSED[p + "act"])
    assert f32_ulp_diff(scale, FUSED[p + "scale"]).max() == 0
    np.testing.assert_array_equal(q, FUSED[p + "q"])


def test_reference_order_sum_is_numpys_pairwise_sum():
    """rms_sum_squares_reference restates tl.sum as Triton's interpreter evaluates it:
    numpy's sum of the 2048-lane chunk-folded vector of squares."""
    rng = np.random.default_rng(11)
    for D in (8, 256, 1000, 2048, 3072, 5376, 8192, 8200, 12288):
        x = O.round_bf16((rng.standard_normal((4, D)) * 3).astype(np.float32))
        ss = O.rms_sum_squares_reference(x)
        nch = -(-D // 2048)
        pad = np.zeros((4, nch * 2048), np.float32)
        pad[:, :D] = x
        for r in range(4):
            lanes = np.zeros(2048, np.float32)
            for c in range(nch):
                v = pad[r, c * 2048:(c + 1) * 2048]
                lanes = (lanes + v * v).astype(np.float32)
            assert np.sum(lanes) == ss[r], (D, r)


def test_exp_f32_is_correctly_rounded_on_every_bf16_input():
    """The oracle's exponential, over every finite bf16 argument, against a 120-bit
    evaluation rounded to float32 (round half to even, subnormals and overflow included)."""
    mpmath = pytest.importorskip("mpmath")
    bits = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    x = bits[np.isfinite(bits)]
    got = O.exp_f32(x)
    with mpmath.workprec(120):
        two = mpmath.mpf(2)
        for xi, gi in zip(x.tolist(), got.tolist()):
            v = mpmath.exp(mpmath.mpf(xi))
            if v >= two ** 128:
                want = float("inf")
            else:
                _, e = mpmath.frexp(v)
                quantum = two ** max(e - 24, -149)
                want = float(mpmath.nint(v / quantum) * quantum)
                if want >= 2.0 ** 128:
                    want = float("inf")
            assert np.float32(want) == np.float32(gi), xi


def test_sigmoid_table_matches_oracle(tmp_path):
    """The kernels' build-time sigmoid table (csrc/sigmoid_table.c), looked up the way the
    kernels do it (magnitude bits clamped to [0x32FF, 0x4300], index sign * 4098 + clamped -
    0x32FF), gives the oracle's sigmoid for every finite bf16 value, and g * table value is
    NaN for every NaN or infinite g exactly where the oracle's act is NaN."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("t8g_build", os.path.join(HERE, "..", "thor-int8-gemm_b200", "build.py"))
    build = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build)
    path = build.generate_sigmoid_table(str(tmp_path / "sigmoid_table.inc"))
    text = open(path).read()
    words = [int(t, 16) for t in text.replace("u", "").replace(",", " ").split() if t.startswith("0x")]
    assert len(words) == 8200
    table = np.array(words, np.uint32).view(np.float32)
    bits = np.arange(65536, dtype=np.uint32)
    mag = np.clip(bits & 0x7FFF, 0x32FF, 0x4300)
    idx = (bits >> 15) * 4098 + mag - 0x32FF
    got = table[idx]
    g = O.bf16_to_f32(bits.astype(np.uint16))
    fin = np.isfinite(g)
    ref = O.sigmoid_f32(g)
    np.testing.assert_array_equal(got[fin].view(np.uint32), ref[fin].view(np.uint32))
    with np.errstate(invalid="ignore"):
        np.testing.assert_array_equal(np.isnan(g * got), np.isnan(O.silu_mul(g, np.ones_like(g))))


def test_rms_sum_squares_tree_matches_sequential_sum_closely():
    rng = np.random.default_rng(3)
    for D in (8, 100, 256, 3072, 5376, 12288, 30000):
        x = O.round_bf16(rng.standard_normal((3, D)).astype(np.float32))
        ss = O.rms_sum_squares(x)
        ref = (x.astype(np.float64) ** 2).sum(axis=1)
        assert np.all(np.abs(ss - ref) <= 1e-5 * ref)


def test_row_threads_rule():
    assert O.row_threads(3072) == 128
    assert O.row_threads(1024) == 64
    assert O.row_threads(5376) == 224
    assert O.row_threads(12288) == 512
    assert O.row_threads(16384) == 512
    assert O.row_threads(8) == 32
    assert O.row_threads(49152) == 512
    with pytest.raises(ValueError):
        O.row_threads(49152 + 8)


def test_per_token_quant_properties():
    rng = np.random.default_rng(4)
    x = O.round_bf16(rng.standard_normal((16, 300)).astype(np.float32))
    x[3] = 0.0
    for kind in (O.QUANT_INT8, O.QUANT_FP8):
        q, s = O.quant_rows(x, kind)
        assert s[3] == np.float32(1e-12)
        if kind == O.QUANT_INT8:
            assert np.abs(q.astype(np.int32)).max() <= 127
            # every non-zero row reaches +-127 at its amax element
            assert np.all(np.abs(q[np.arange(16) != 3]).max(axis=1) == 127)
        else:
            deq = O.e4m3_to_f32(q)
            assert np.all(np.abs(deq) <= 448)
