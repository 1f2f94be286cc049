"""rustgears_b200 -- B200-native INT8 execution provider for RustGears models.

Drop-in for the reference's Npu(Int8) inference path:

    from rustgears_b200 import InferenceSession, ExecutionProvider
    sess = InferenceSession.from_module(model, ExecutionProvider.npu_int8())
    y = sess.run(x)
    print(sess.compilation_report()); print(sess.last_npu_profile())

All compute runs in librg_npu.so (hand-written sm_100a kernels behind the C
ABI in include/rg_npu.h); there is no CPU fallback.
"""
from .rtim import load_inference_layers, save_inference_model, save_layers
from .session import ExecutionProvider, InferenceSession, NpuPrecision, NpuProfile, OpRecord
from .spec import Activation, LayerSpec
from .rng import manual_seed

__all__ = ["InferenceSession", "ExecutionProvider", "NpuPrecision", "NpuProfile", "OpRecord", "LayerSpec",
           "Activation", "load_inference_layers", "save_layers", "save_inference_model", "manual_seed"]
__version__ = "0.1.0"
