"""B200-native Shieldstral scoring prefill (curiosity-ai/llm-shield hot path).

The product is the CUDA library ``libshield_b200.so`` behind the C ABI in
``include/shield_b200.h``; this package holds its sources (``csrc/``), the
in-tree build, a ctypes binding of that ABI (``binding``) and the synthetic
checkpoint generator (``synth``).
"""
