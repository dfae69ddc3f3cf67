"""Graph analysis and module replacement (mirrors the reference's Core/ package)."""
