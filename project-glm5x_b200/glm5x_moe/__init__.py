"""glm5x_moe -- B200 (sm_100a) routed-expert MoE sublayer for GLM-5.

Python front end over libglm5x_moe.so (C ABI: include/glm5x_moe.h). The
submodules import lazily so that `glm5x_moe.build` works before the library
exists.
"""
from __future__ import annotations

__all__ = ["GLM5XMoELayer", "NVFP4Expert", "MXFP4Expert", "GLM5XNVFP4Weight",
           "GLM5XMXFP4Weight", "quantize_nvfp4_weight", "quantize_mxfp4_weight",
           "dequantize_nvfp4", "encode_mxfp4", "decode_mxfp4", "RoutingMode",
           "RoutingPolicyConfig", "select_routing"]


def __getattr__(name):
    if name in ("GLM5XMoELayer", "NVFP4Expert", "MXFP4Expert", "GLM5XMoEForward"):
        from . import layer
        return getattr(layer, name)
    if name in ("GLM5XNVFP4Weight", "GLM5XMXFP4Weight", "quantize_nvfp4_weight",
                "quantize_mxfp4_weight", "dequantize_nvfp4", "encode_mxfp4", "decode_mxfp4"):
        from . import nvfp4
        return getattr(nvfp4, name)
    if name in ("RoutingMode", "RoutingPolicyConfig", "select_routing", "RoutingDecisions"):
        from . import routing
        return getattr(routing, name)
    raise AttributeError(name)
