"""hsd_b200 -- B200-native (sm_100a) verification hot path of HSD.

Hierarchical Speculative Decoding verifies packed document-region drafts
against a target VLM.  This package replaces the reference's verification
path (whlscut/HSD ``batch_generate`` + ``flex_attention_forward``) with
hand-written CUDA kernels behind a C ABI (``include/hsd_b200.h``,
``libhsd_b200.so``):

1. packed block-sparse verification attention (tcgen05 + TMEM + TMA),
2. in-place KV-cache compaction and the KV append,
3. warp-per-block acceptance fused with KMP re-alignment (exact match, and
   the logit-ratio rules below the default thresholds),
4. on-device packing metadata (tile plans from segment descriptors),
5. next tokens: the lm_head GEMM fused with the argmax (no logits written),
   the single logits the logit-ratio rules read, and a rank pass of the same
   GEMM for HunYuan's top-k / adaptive acceptance,
6. rotary embedding fused with the cache update,
7. tree decoding's continuation tries, built and packed on the device.

Python entry points: ``attention.flex_attention_forward`` (the HF attention
hook), ``loop.VerifyLoop`` / ``loop.batch_generate`` (the verification
loop), ``verify_step.VerifyStep`` (one fixed page's step, as benchmarked),
``lm_head.lm_head_argmax``, ``lm_head.probe_logits``, ``lm_head.lm_head_rank``,
``rope.rope_append``, ``trie.continuation_trees``
and ``sharding`` (pages over the GPUs of a node).

There is no CPU fallback: importing a kernel wrapper without the compiled
library raises ``HSDNativeError``.
"""
from ._native import HSDError, HSDNativeError, load  # noqa: F401

__version__ = "0.1.0"
