"""krikil_rs_b200: B200 (sm_100a) fp32 implementation of krikil-rs's per-layer
inference path for the Pebble-25M hybrid Mamba2 + attention model.

The product is the C ABI library lib/libkrikil_cuda.so (include/krikil_cuda.h,
include/krikil_text.h for the tokenizer and chat template);
this package is its Python host mirror.  Importing it requires the built
library; there is no CPU fallback.
"""
from ._lib import KrikilError, LIB_PATH, launch_count  # noqa: F401
from .model import (  # noqa: F401
    GenerationEngine,
    GenerationOptions,
    GenerationResult,
    PebbleConfig,
    PebbleModel,
    PebbleState,
    SamplerConfig,
)
from .text import ChatMessage, ChatTemplateEngine, PebbleTokenizer  # noqa: F401

__all__ = [
    "KrikilError", "LIB_PATH", "launch_count", "GenerationEngine", "GenerationOptions", "GenerationResult",
    "PebbleConfig", "PebbleModel", "PebbleState", "SamplerConfig", "ChatMessage", "ChatTemplateEngine",
    "PebbleTokenizer",
]
