"""csahca_b200 — B200-native (sm_100a) compressed-sparse-attention decode kernels.

Drop-in for the decode path of ypd666/CSAHCA: ``csahca_b200.extension`` mirrors
``hybrid_attention.extension`` and ``csahca_b200.hybrid_attention_cuda`` mirrors
the reference's native module.  Kernels live in ``libcsahca_b200.so`` (C ABI in
``include/csahca_b200.h``), built in-tree by ``python -m csahca_b200.build``.
"""

__version__ = "0.1.0"
