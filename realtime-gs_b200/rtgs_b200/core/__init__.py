"""Core containers and metrics (reference: src/rtgs/core)."""
