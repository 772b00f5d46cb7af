"""hsd_b200 -- B200-native (sm_100a) verification hot path of HSD.

Hierarchical Speculative Decoding verifies packed document-region drafts
against a target VLM.  This package replaces the reference's verification
path (whlscut/HSD ``batch_generate`` + ``flex_attention_forward``) with
hand-written CUDA kernels behind a C ABI (``include/hsd_b200.h``,
``libhsd_b200.so``):

1. packed block-sparse verification attention (tcgen05 + TMEM + TMA),
2. in-place KV-cache compaction,
3. warp-per-block acceptance fused with KMP re-alignment,
4. on-device packing metadata (tile plans from segment descriptors).

There is no CPU fallback: importing a kernel wrapper without the compiled
library raises ``HSDNativeError``.
"""
from ._native import HSDError, HSDNativeError, load  # noqa: F401

__version__ = "0.1.0"
