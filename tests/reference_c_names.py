"""The reference's ``_C`` operator names and the mirror function serving
each (test helper).

``make_C()`` builds a module with every ``_C.<op>_scalar`` / ``_C.<op>_simd``
(and the debug-op names) the reference's kernel tests call, each bound to the
matching ``i_whisper_b200.ops.<op>_cuda`` function. Used by the reference
suite plugins (emulated here, and the GPU replay of its recorded calls).
"""
import types

from i_whisper_b200 import ops

# reference _C name (without the _scalar/_simd suffix) -> mirror function
MIRROR = {
    "linear8": ops.linear8_cuda,
    "linear8_accum_{}_debug": ops.linear8_accum_cuda_debug,
    "linear32": ops.linear32_cuda,
    "linear32_accum_{}_debug": ops.linear32_accum_cuda_debug,
    "linear8_requant_{}_debug": ops.linear8_requant_cuda_debug,
    "linear32_requant_{}_debug": ops.linear32_requant_cuda_debug,
    "residual15": ops.residual15_cuda,
    "layernorm32": ops.layernorm32_cuda,
    "layernorm32_stats": ops.layernorm32_stats_cuda,
    "layernorm32_rsqrt": ops.layernorm32_rsqrt_cuda,
    "layernorm64": ops.layernorm64_cuda,
    "layernorm64_stats": ops.layernorm64_stats_cuda,
    "gelu": ops.gelu_cuda,
    "qk": ops.qk_cuda,
    "qk_requant_rowmax": ops.qk_requant_rowmax_cuda,
    "shift_exp": ops.shift_exp_cuda,
    "pv": ops.pv_cuda,
    "pv_norm_requant": ops.pv_norm_requant_cuda,
    "conv1d_accum": ops.conv1d_accum_cuda,
    "conv1d": ops.conv1d_cuda,
    "add_requant15": ops.add_requant15_cuda,
    "classifier_accum": ops.classifier_accum_cuda,
    "classifier": ops.classifier_cuda,
}


def make_C():
    C = types.ModuleType("i_whisper.kernels._C")
    C.rounding_rshift_debug = ops.rounding_rshift_debug_cuda
    for name, fn in MIRROR.items():
        for backend in ("scalar", "simd"):
            key = name.format(backend) if "{}" in name else f"{name}_{backend}"
            setattr(C, key, fn)
    return C


