"""omnivoice-b200: OmniVoice's generator hot path on NVIDIA B200 (sm_100a).

The product is the C-ABI shared library libomnivoice_b200.so (include/ov_*.h)
with the C++ drop-in headers under csrc/host; this package builds it
(omnivoice_b200.build) and binds it with ctypes (omnivoice_b200._native,
omnivoice_b200.generator).
"""
from .generator import (Cancelled, ConditionalInput, DecodingConfig, GenerationResult,
                        Generator, GeneratorError, model_config, unmask_schedule)

__all__ = ["Cancelled", "ConditionalInput", "DecodingConfig", "GenerationResult", "Generator",
           "GeneratorError", "model_config", "unmask_schedule"]
