"""shadow_infer_b200 -- the ShadowKV packed-KV data plane of ShadowInfer, rebuilt for B200 (sm_100a).

The Python surface mirrors the reference package (``shadowinfer.shadowkv``):
``PackedKVCache``, ``PrecisionPlan``, ``admit_codes`` and friends keep their
names, arguments, return values and exceptions.  Every data-plane operation
runs as a hand-written CUDA kernel in ``_lib/libshadowkv_b200.so`` (C ABI in
``include/shadowkv_b200.h``); there is no CPU fallback.
"""

__version__ = "0.1.0"
