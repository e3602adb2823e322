"""Serving-runtime integration (vLLM registry plumbing kept from the reference)."""
