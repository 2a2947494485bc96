"""PentaNet packed-weight path for B200 (sm_100a).

This directory is both a package (load it under any name with importlib) and a
drop-in module directory: put it on sys.path and the reference's own imports
    from penta_kernel import quantize_and_pack, penta_linear
    from pentanet_layer import PentaLinear, PentaLinearFast, convert_to_fast_inference
    from penta_avx2_wrapper import penta_unpack, penta_linear_avx2
resolve to the sm_100a implementation.
"""
from .penta_kernel import (absmean_scale, memory_stats, penta_linear, penta_linear_2bit, penta_linear_i8,
                           penta_linear_i8_prequant, penta_linear_i8w, quantize_activations_i8, quantize_and_pack,
                           quantize_and_pack_2bit, storage_bytes, unpack_weights, unpack_weights_2bit,
                           unpack_weights_i8)
from .pentanet_layer import PentaLinear, PentaLinearFast, convert_to_fast_inference

__all__ = [
    "absmean_scale", "memory_stats", "penta_linear", "penta_linear_i8", "penta_linear_i8_prequant",
    "penta_linear_i8w", "penta_linear_2bit", "quantize_and_pack_2bit", "unpack_weights_2bit",
    "quantize_activations_i8", "quantize_and_pack", "storage_bytes", "unpack_weights", "unpack_weights_i8",
    "PentaLinear", "PentaLinearFast", "convert_to_fast_inference",
]
