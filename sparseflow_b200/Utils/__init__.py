"""Shared constants and policies (mirrors the reference's Utils/ package)."""
