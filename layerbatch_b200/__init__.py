"""layerbatch_b200: B200-native (sm_100a) hot path of the LayerBatch inference engine.

The CUDA library (``liblb_b200.so``, built from ``csrc/``) is loaded on first use by
``layerbatch_b200._lib``; importing the package itself needs no GPU.
"""
__version__ = "0.1.0"
