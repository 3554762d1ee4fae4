"""omni_b200: a B200-native (sm_100a) implementation of the SGLang-Omni talker
decode step behind the reference's own Python call signatures.

Python modules here mirror the reference modules they replace:

- ``sampling_kernels``   <- sglang_omni/models/qwen3_tts/sampling_kernels.py
- ``predictor_kernels``  <- sglang_omni/models/qwen3_tts/predictor_kernels.py
- ``predictor_layers``   <- sglang_omni/utils/predictor_layers.py
- ``seed``               <- sglang_omni/sampling/seed.py

All device work goes through libomni_b200.so (C ABI in include/omni_b200.h).
"""

from omni_b200._lib import OmniUnsupported, device_status, load  # noqa: F401

__version__ = "0.1.0"
