"""kvasir_b200: B200-native (sm_100a) kernel chain for kvasir's per-layer Llama
path -- embedding gather, RMSNorm, RoPE + KV append, GQA attention (split-KV
decode, tcgen05 prefill), SiLU*mul -- behind a C ABI that mirrors kvasir's
engine/src/gpu launch wrappers (include/kvasir_b200.h)."""
from .config import ConfigError, LlamaConfig
from .gpu import (CudaError, DeviceError, Gpu, KvasirError, ShapeError, UnsupportedError,
                  check, dtype_tag)

__all__ = ["Gpu", "LlamaConfig", "ConfigError", "KvasirError", "ShapeError", "CudaError",
           "UnsupportedError", "DeviceError", "check", "dtype_tag"]
