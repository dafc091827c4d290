"""tempo_compiler_b200: a B200 (sm_100a) backend for the four tile ops GPT-2 small launches in tempo-compiler.

The kernels (bf16 GEMM with fused bias / exact-erf GELU / residual, causal and decode attention over a resident
KV cache, LayerNorm, the residual add, and the KV-cache copies) are hand-written CUDA in ``csrc/`` and are reached
only through the C-ABI library ``libtempo_b200.so`` (``include/tempo_b200.h``). There is no CPU fallback: every
compute entry point raises if the library or a GPU is missing.

Modules:
    lib       -- loads the C-ABI library (ctypes) and maps its status codes to the reference's exceptions.
    runtime   -- drop-in replacement of the reference board runtime (``minitpu*`` API) over the library.
    images    -- the image set: manifest entries with the reference's kinds and fields, and their descriptors.
    dropin    -- GPT-2 driven through ``runtime`` with one image launch per 32-token block (the drop-in host path).
    engine    -- the B200-native GPT-2 engine: resident weights, batched prefill/decode, CUDA graphs.
    weights   -- seeded random GPT-2 weights in the reference's naming scheme.
"""

__all__ = ["lib", "runtime", "images", "dropin", "engine", "weights"]
