"""aikit_b200 -- a B200-native (sm_100a) backend for aikit's exact int8
nearest-neighbour scan (ann.FlatI8) and its FlatBinary -> FlatI8 path.

The product is the CUDA library behind ``include/fi8.h``
(``aikit_b200/lib/libfi8_b200.so``). ``aikit_b200.ann`` mirrors the reference's
Go device seam (``ann.Backend`` / ``I8Index`` / ``I8BatchIndex`` /
``I8TopKIndex``, ann/backend.go:16-55) on top of that C ABI. There is no CPU
fallback: if the library or a GPU is missing, calls raise.
"""
from ._ffi import Fi8Error, DeclinedError, lib  # noqa: F401
