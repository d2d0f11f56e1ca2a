"""Stage 1: 2D gaussian image fitting (reference: src/rtgs/image2gs)."""
