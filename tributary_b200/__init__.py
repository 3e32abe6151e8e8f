"""B200-native (sm_100a) Relational-Transformer masked attention.

The CUDA library (libtributary_b200.so, C ABI in include/rt_attention.h) is
the product; this package holds its build script, its ctypes binding and a
PyTorch host layer that mirrors the reference's attention interface.
"""
__version__ = "0.1.0"
