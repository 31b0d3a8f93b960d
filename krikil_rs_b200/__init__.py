"""krikil_rs_b200: B200 (sm_100a) fp32 implementation of krikil-rs's per-layer
inference path for the Pebble-25M hybrid Mamba2 + attention model.

The product is the C ABI library lib/libkrikil_cuda.so (include/krikil_cuda.h,
include/krikil_text.h for the tokenizer and chat template);
this package is its Python host mirror.  Using the model API requires the built
library and fails loudly without it; there is no CPU fallback.

The library is loaded on first use of a name that needs it (PEP 562 module
``__getattr__``), so the pure-numpy helpers (``krikil_rs_b200.synth``: seeded
weights and prompts) can be imported by a CPU-only process without mapping
the CUDA library.
"""
import importlib

_EXPORTS = {
    "KrikilError": "._lib", "LIB_PATH": "._lib", "launch_count": "._lib",
    "GenerationEngine": ".model", "GenerationOptions": ".model", "GenerationResult": ".model",
    "PebbleConfig": ".model", "PebbleModel": ".model", "PebbleState": ".model", "SamplerConfig": ".model",
    "ChatMessage": ".text", "ChatTemplateEngine": ".text", "PebbleTokenizer": ".text",
}

__all__ = list(_EXPORTS)


def __getattr__(name):
    mod = _EXPORTS.get(name)
    if mod is None:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    value = getattr(importlib.import_module(mod, __name__), name)
    globals()[name] = value
    return value


def __dir__():
    return sorted(set(globals()) | set(_EXPORTS))
