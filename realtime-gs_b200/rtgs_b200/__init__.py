"""rtgs_b200: B200-native (sm_100a) Stage-1 2D gaussian image fitting.

Mirrors the reference package's Stage-1 API (``rtgs.core.gaussians2d``, ``rtgs.core.metrics``,
``rtgs.image2gs.renderer2d``, ``rtgs.image2gs.cuda_backend``, ``rtgs.image2gs.fit``,
``rtgs.image2gs.batched``) on top of one CUDA library, ``_lib/librtgs2d.so`` (C ABI in
``include/rtgs2d.h``). Importing the package does not initialise CUDA.
"""

__version__ = "0.1.0"
