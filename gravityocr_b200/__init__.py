"""B200-native (sm_100a) self-speculative decode round for a GLM-OCR-shaped decoder.

The CUDA kernels live in ``csrc/`` and are reached through the C ABI declared in ``include/gravity_b200.h``
(``gravityocr_b200/_lib.py`` loads ``libgravity_b200.so``).  Importing this package does not load the library;
the first kernel call does, and raises if it is missing.
"""
__version__ = "0.1.0"
