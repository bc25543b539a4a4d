"""salt_b200 — B200-native (sm_100a) implementation of SALT's integer event-driven forward pass
and of the float chunked affine scan of its FC layers.

Host API mirrors the reference (salt_core): EventStream, InputEvents, ConvLayer/FCLayer and their
specs, Network/run_network, QuantizedLayerParams and the offline integer codes.  The compute runs
in libsalt_b200.so (CUDA kernels behind a C ABI, include/salt_b200.h); there is no CPU fallback.
"""
from .capacity import Capacity, GrowthPolicy, LayerDiag, grown_to_fit, reduce_over_batch
from .layers import (ConvLayer, ConvQueueStructure, ConvSpec, FCLayer, FCQueueStructure, FCSpec,
                     LayerOutput, conv, fc)
from .network import InputEvents, Network, check_layer_connections, input_stream, run_network
from .quant import (MAX_REGISTER_BITS, MAX_SHIFT_BITS, OverflowMode, QuantizedLayerParams,
                    RoundMode, build_decay_table_int, delta_t_max, quantize_to_int,
                    round_half_away_from_zero, v_th_to_int)
from .stream import PAD_TIME, EventStream
from .io import (QuantizedModel, load_quantized, load_weights, network_from_dict,
                 network_to_dict, save_quantized, save_weights)
from .quant_run import (REFERENCE_FIELDS, QuantSplitOutput, check_quantized, quant_forward_split,
                        reference_arrays, run_until_fits)


def __getattr__(name):  # the CUDA-backed objects load the library lazily
    if name in ("QuantB200Backend", "QuantLayerResult", "NetworkOutput", "default_backend"):
        from . import backend
        return getattr(backend, name)
    if name in ("FloatB200Backend", "FloatLayerResult"):
        from . import float_backend
        return getattr(float_backend, name)
    if name == "NetworkPlan":
        from .plan import NetworkPlan
        return NetworkPlan
    raise AttributeError(name)


__all__ = ["REFERENCE_FIELDS", "QuantSplitOutput", "QuantizedModel", "check_quantized",
           "load_quantized", "load_weights", "network_from_dict", "network_to_dict",
           "quant_forward_split", "reference_arrays", "run_until_fits", "save_quantized",
           "save_weights", "Capacity", "ConvLayer", "ConvQueueStructure", "ConvSpec", "FCQueueStructure", "EventStream", "FCLayer", "FCSpec", "GrowthPolicy",
           "FloatB200Backend", "FloatLayerResult", "InputEvents", "LayerDiag", "LayerOutput", "MAX_REGISTER_BITS", "MAX_SHIFT_BITS",
           "Network", "NetworkPlan", "OverflowMode", "PAD_TIME", "QuantB200Backend",
           "QuantizedLayerParams", "RoundMode", "build_decay_table_int", "check_layer_connections",
           "conv", "delta_t_max", "fc", "grown_to_fit", "input_stream", "quantize_to_int",
           "reduce_over_batch", "round_half_away_from_zero", "run_network", "v_th_to_int"]
