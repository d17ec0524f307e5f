"""thor_int8_gemm_b200 -- B200 (sm_100a) quantized linear-layer path.

Drop-in for the hot path that kylixs/thor-int8-gemm patches into comfy-kitchen:
the int8 fused-dequant GEMM behind `_C.cutlass_int8_dequant` (plus an fp8 e4m3
twin), fused RMSNorm + adaLN modulation + quantisation, and fused SwiGLU +
quantisation.  The kernels are hand-written CUDA for sm_100a behind a C ABI
(include/thor_int8_gemm_b200.h, libthor_int8_gemm_b200.so next to this file).

Submodules (imported lazily, so the import-proxy agent stays light at start-up):
  ops         torch-facing wrappers of every C entry point
  fused       mirror of the reference module ck_fused_mod_norm_quant
  patch_int8  the comfy-kitchen `_C` import proxy and its .pth installer
  build       nvcc build of the shared library
  shard       token sharding across ranks (one process per GPU)
  dit         a DiT block whose linears and norm/quant ops run on these kernels
  torch_ops   the entry points as torch custom ops (namespace t8g) for torch.compile
  fused_patch the DiT-block agent (comfy's MiniMax-H3 DiTBlock.forward on the fused kernels)
"""
import importlib

__version__ = "0.1.0"
PACKAGE_NAME = "thor_int8_gemm_b200"
_LAZY = ("ops", "fused", "patch_int8", "build", "_lib", "shard", "dit", "torch_ops", "fused_patch")


def __getattr__(name):
    if name in _LAZY:
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
