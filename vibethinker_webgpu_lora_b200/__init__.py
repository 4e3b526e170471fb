"""Emberglass B200: the int4 decode hot path of maceip/vibethinker-webgpu-lora
rebuilt for NVIDIA B200 (sm_100a) behind the reference's QwenWGPU surface."""
from ._lib import EmberglassError, lib  # noqa: F401
from .config import QWEN25_3B, small_config  # noqa: F401
from .lora import (LoraAdapter, loadLoraAdapter, moduleKeyFromTensorName, orientLora,  # noqa: F401
                   parseLoraAdapter, synthetic_adapter)
from .quantize import quantizeInt4Group, quantizeInt8RowMajor  # noqa: F401
from .runtime import QwenB200, readSafetensorsTensor  # noqa: F401
