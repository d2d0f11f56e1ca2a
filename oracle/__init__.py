"""CPU oracle for the Stage-1 2D gaussian splatting path (TEST INFRASTRUCTURE ONLY).

This package restates the reference's algorithm on the CPU so that the CUDA path can be checked
against it. It is imported only by ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py``; the product package (``rtgs_b200``) never imports it and has no CPU
fallback.

Pinning: every function here is checked against golden vectors produced by the reference itself
(``tests/golden/make_golden.py`` imports the reference's pure-PyTorch renderer, fit loop and
batched fit and stores their outputs under ``tests/golden/``), see ``tests/test_oracle_golden.py``.

Modules:
  render2d  support rectangles, conics, the accumulated scatter renderer (differentiable through
            torch autograd exactly like the reference), tile binning enumeration.
  fit       the native fit loop (raw reparameterisation, torch Adam, cosine schedule, PSNR log)
            for a single image and for stacked views.
"""
