"""tinferno-b200: B200-native (sm_100a) decode/prefill engine for Llama-style GGUF models.

The compute path is the CUDA library built from ``csrc/`` (``lib/libtinferno_b200.so``)
behind the C-ABI declared in ``include/tinferno_b200.h``; this package is the host-side
mirror of the reference engine's ``Model`` API over that C-ABI plus the GGUF and synthetic
model tooling.
"""
