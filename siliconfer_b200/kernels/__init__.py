"""Kernel APIs.  ``siliconfer_b200.kernels.cuda`` mirrors the reference's
``siliconfer.kernels.neon`` module (siliconfer/kernels/neon/__init__.py:230-239)."""
