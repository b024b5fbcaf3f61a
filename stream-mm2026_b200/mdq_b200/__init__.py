"""mdq_b200 - B200-native fused quantized-AdamW (MDQ) optimizer step.

Public API:
  MDQAdamWSimple, MDQAdamWSimpleFusedIO, MDQAdamW   torch.optim drop-ins
  MDQAdamWFakeQuant                                 the pure-PyTorch MDQAdamW's algorithm, fused
  fused_mdq_adamw                                   reference kernel signature
  step_multi / StepItem                             multi-tensor step
  ZeroMDQAdamW                                      state-sharded (ZeRO-1) step
"""
from .kernels import StepItem, fused_mdq_adamw, step_multi  # noqa: F401
from .optim import (MDQAdamW, MDQAdamWFakeQuant, MDQAdamWSimple,  # noqa: F401
                    MDQAdamWSimpleFusedIO)
from .zero1 import ZeroMDQAdamW  # noqa: F401

__all__ = ["MDQAdamW", "MDQAdamWFakeQuant", "MDQAdamWSimple", "MDQAdamWSimpleFusedIO", "fused_mdq_adamw",
           "step_multi", "StepItem", "ZeroMDQAdamW"]
