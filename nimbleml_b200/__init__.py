"""B200-native fused tied LM-head cross-entropy (drop-in for NimbleML's path).

Public surface, mirroring the reference's names:

* ``nimbleml_b200.kernels.fused_tied_crossentropy_forward / _backward``
  (NimbleML/kernels/fused_tied_crossentropy.py:8-48)
* ``nimbleml_b200.losses.CrossEntropyLoss.forward_tied``
  (NimbleML/losses/cross_entropy.py:109-192)
* ``nimbleml_b200.vocab_parallel`` — the vocab-sharded multi-GPU form.

The compute runs in ``libnimbleml_tied_ce.so`` (C ABI, include/nimbleml_tied_ce.h).
"""
# The library is loaded by nimbleml_b200._native_loader when the kernels or
# losses modules are imported (ImportError with the build command if it is
# missing); the package itself imports without it so the build step can run.

__version__ = "0.1.0"
