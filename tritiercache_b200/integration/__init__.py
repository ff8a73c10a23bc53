"""Hugging Face model integration (src/tri_tier/integration)."""
