"""Functional entry points over the native kernels (mirrors the reference's Kernels/ package)."""
