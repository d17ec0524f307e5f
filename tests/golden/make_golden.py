#!/usr/bin/env python3
"""Generate the golden vectors under tests/golden/ by running the REFERENCE's own code.

Run in a container that has the reference checkout (read-only) at REF_SRC:

    python tests/golden/make_golden.py [--ref /root/reference/src]

What runs, all on the CPU:

* `_gemm_intmm` from src/ck_int8_patch_intmm.py:63-71 (torch `_int_mm` + eager
  float32 epilogue) -- the reference's own runnable GEMM restatement;
* the Triton `_kernel` GEMM from src/ck_int8_patch_thor.py:67-125, and the fused
  kernels `fused_rms_mod_quant` / `fused_swiglu_quant` /
  `_rms_mod_res_amax_kernel` + `_quant_fp8_amax_kernel` from
  src/ck_fused_mod_norm_quant.py, through Triton's CPU interpreter
  (TRITON_INTERPRET=1).

The interpreter (Triton 3.6) converts float32 -> bf16 by truncation and rounds
its "RTNE" fp8 path half-up; the GPU lowers the same `.to()` calls to
`cvt.rn.bf16.f32` and `cvt.rn.satfinite.e4m3x2.f32` (round to nearest even).
This script therefore replaces the interpreter's `_convert_float` with a
round-to-nearest-even converter (torch's CPU casts) before running anything,
so the goldens model the GPU's rounding.  Nothing in the reference code is
modified.

Output: one .npz per case family, small enough to commit.
"""
from __future__ import annotations

import argparse
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

_TORCH_OF = {}


def _patch_interpreter():
    import triton.language as tl
    import triton.runtime.interpreter as interp

    _TORCH_OF.update({
        tl.float32: (torch.float32, np.int32),
        tl.bfloat16: (torch.bfloat16, np.int16),
        tl.float16: (torch.float16, np.int16),
        tl.float8e4nv: (torch.float8_e4m3fn, np.int8),
    })

    def rne_convert(inp, input_dtype, output_dtype, rounding_mode):
        src_t, src_np = _TORCH_OF[input_dtype]
        dst_t, dst_np = _TORCH_OF[output_dtype]
        arr = np.ascontiguousarray(inp).view(src_np)
        t = torch.from_numpy(arr.copy()).view(src_t)
        out = t.to(dst_t).view({1: torch.int8, 2: torch.int16, 4: torch.int32}[dst_t.itemsize])
        return out.numpy().view({1: np.uint8, 2: np.uint16, 4: np.uint32}[dst_t.itemsize])

    interp._convert_float = rne_convert


def _bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _bits8(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).numpy().copy()


def gemm_cases(pt, pi):
    """GEMM goldens from both reference implementations (they must agree)."""
    tri_gemm = pt._build_triton_gemm()
    intmm = pi._build_triton_gemm()
    cases = [
        # (M, N, K, bias, out dtype, scalar w_scale)
        (128, 128, 128, True, torch.bfloat16, False),
        (130, 136, 96, True, torch.bfloat16, False),
        (200, 264, 208, False, torch.bfloat16, False),
        (256, 256, 320, True, torch.float16, False),
        (129, 200, 144, True, torch.float32, False),
        (160, 144, 64, True, torch.bfloat16, True),
        (1, 64, 32, False, torch.bfloat16, False),
        (96, 48, 16, True, torch.bfloat16, False),
        (256, 320, 256, True, torch.bfloat16, False),
    ]
    out = {}
    g = torch.Generator().manual_seed(1234)
    for i, (M, N, K, hb, odt, scalar_ws) in enumerate(cases):
        x8 = torch.randint(-127, 128, (M, K), dtype=torch.int8, generator=g)
        w8 = torch.randint(-127, 128, (N, K), dtype=torch.int8, generator=g)
        xs = torch.rand(M, generator=g) + 0.5
        ws = (torch.rand(1, generator=g) + 0.5) if scalar_ws else (torch.rand(N, generator=g) + 0.5)
        xs = xs * 1e-2
        ws = ws * 1e-2
        bias = (torch.randn(N, generator=g) * 0.5).to(odt) if hb else torch.empty(0, dtype=odt)
        o_tri = torch.empty(M, N, dtype=odt)
        o_mm = torch.empty(M, N, dtype=odt)
        tri_gemm(x8, w8, xs, ws, bias, o_tri)
        intmm(x8, w8, xs, ws, bias, o_mm)
        if not torch.equal(o_tri, o_mm):
            raise SystemExit(f"reference GEMM implementations disagree on case {i}")
        tag = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}[odt]
        p = f"g{i}_"
        out[p + "x8"] = x8.numpy()
        out[p + "w8"] = w8.numpy()
        out[p + "xs"] = xs.numpy()
        out[p + "ws"] = ws.numpy()
        out[p + "bias"] = bias.float().numpy() if hb else np.zeros(0, np.float32)
        out[p + "out"] = o_mm.numpy() if odt == torch.float32 else _bits16(o_mm)
        out[p + "meta"] = np.array([M, N, K, int(hb), int(scalar_ws)], np.int64)
        out[p + "dtype"] = np.array(tag)
    out["n_cases"] = np.array(len(cases))
    return out


def fused_cases(fk):
    """Norm/mod/quant and SwiGLU/quant goldens from the reference Triton kernels."""
    out = {}
    g = torch.Generator().manual_seed(4321)
    # fused_rms_mod_quant(x, w, s, b, eps): distributions of bench/a3p_device_scale_test.py:110-116
    rms = [(8, 256, 1e-5, False), (6, 3072, 1e-6, False), (4, 5376, 1e-5, False), (4, 256, 1e-5, True)]
    for i, (S, K, eps, zero) in enumerate(rms):
        x = (torch.randn(S, K, generator=g) * 0.5).to(torch.bfloat16)
        if zero:
            x.zero_()
        w = (torch.randn(K, generator=g).abs() + 0.5).to(torch.bfloat16)
        s = (torch.randn(K, generator=g) * 0.1).to(torch.bfloat16)
        b = (torch.randn(K, generator=g) * 0.1).to(torch.bfloat16)
        if zero:
            b.zero_()
        q, scale, h, res = fk.fused_rms_mod_quant(x, w, s, b, eps)
        p = f"r{i}_"
        out[p + "x"], out[p + "w"], out[p + "s"], out[p + "b"] = map(_bits16, (x, w, s, b))
        out[p + "q"] = _bits8(q)
        out[p + "scale"] = scale.numpy().astype(np.float32).reshape(1)
        out[p + "h"], out[p + "res"] = _bits16(h), _bits16(res)
        out[p + "eps"] = np.array(eps, np.float64)
    out["n_rms"] = np.array(len(rms))

    # per-segment driver of src/ck_fused_patch.py:105-136 (config-3 style: two
    # batch segments, s = 1 + scale[row] in bf16, shared global amax, w = 1)
    S_seg, K = 5, 3072
    x = torch.randn(2 * S_seg, K, generator=g).to(torch.bfloat16)
    shift = (torch.randn(2, K, generator=g) * 0.1).to(torch.bfloat16)
    scale_mod = (torch.randn(2, K, generator=g) * 0.1).to(torch.bfloat16)
    w = torch.ones(K, dtype=torch.bfloat16)
    h = torch.empty_like(x)
    res = torch.empty_like(x)
    amax = torch.zeros((), dtype=torch.float32)
    eps = 1e-6
    for a, bnd, row in ((0, S_seg, 0), (S_seg, 2 * S_seg, 1)):
        s_row = 1.0 + scale_mod[row].to(x.dtype)
        sh = shift[row].to(x.dtype)
        fk._rms_mod_res_amax_kernel[(bnd - a,)](x[a:bnd], w, s_row, sh, h[a:bnd], res[a:bnd], amax, K, eps,
                                               BLOCK_K=2048, N_CHUNK=-(-K // 2048), num_warps=8)
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn)
    n = q.numel()
    fk._quant_fp8_amax_kernel[(-(-n // 4096),)](h, q, amax, fk.F8_E4M3_MAX, n, SCALE_MIN=1e-12, BLOCK=4096, num_warps=4)
    out["seg_x"], out["seg_shift"], out["seg_scale"] = map(_bits16, (x, shift, scale_mod))
    out["seg_h"], out["seg_res"], out["seg_q"] = _bits16(h), _bits16(res), _bits8(q)
    out["seg_amax"] = amax.numpy().astype(np.float32).reshape(1)
    out["seg_rows"] = np.array(S_seg)

    # fused_swiglu_quant(gate, up): distributions of bench/a2_fused_bench.py:50-51
    sw = [(8, 512, False), (4, 1536, False), (2, 12288, False), (4, 256, True)]
    for i, (S, F, zero) in enumerate(sw):
        gate = torch.randn(S, F, generator=g).to(torch.bfloat16)
        up = torch.randn(S, F, generator=g).to(torch.bfloat16)
        if zero:
            up.zero_()
        q, scale, act = fk.fused_swiglu_quant(gate, up)
        p = f"s{i}_"
        out[p + "gate"], out[p + "up"] = _bits16(gate), _bits16(up)
        out[p + "q"] = _bits8(q)
        out[p + "scale"] = scale.numpy().astype(np.float32).reshape(1)
        out[p + "act"] = _bits16(act)
    out["n_swiglu"] = np.array(len(sw))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference/src")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    _patch_interpreter()
    os.environ.pop("CK_INT8_MODE", None)   # the patch modules stay inert on import
    import ck_fused_mod_norm_quant as fk
    import ck_int8_patch_intmm as pi
    import ck_int8_patch_thor as pt

    g = gemm_cases(pt, pi)
    np.savez_compressed(os.path.join(HERE, "gemm_golden.npz"), **g)
    f = fused_cases(fk)
    np.savez_compressed(os.path.join(HERE, "fused_golden.npz"), **f)
    for name in ("gemm_golden.npz", "fused_golden.npz"):
        print(name, os.path.getsize(os.path.join(HERE, name)), "bytes")


if __name__ == "__main__":
    main()
