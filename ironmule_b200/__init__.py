"""IronMule's speculative-decoding hot path, rebuilt for NVIDIA B200 (sm_100a).

Host surface (same names as the reference's `ironmule` modules):
  speculation      n-gram drafting, greedy `accept`, WindowPolicy / StepPolicy / CollectiveIndex
  draft_model      DraftStop, Drafter, suggest_draft
  kernel_registry  spec -> digest-named kernels (bound to libimspec programs)
  qmv_k3840, qmv_shared, qmv_fast_shared, qmv_variant
                   the 4-bit affine matvec call surface, on the B200 qGEMM
Device code: libimspec.so (csrc/*.cu, C ABI in include/imspec.h), loaded by `_lib`, wrapped by `kernels`.
"""

__version__ = "0.1.0"
