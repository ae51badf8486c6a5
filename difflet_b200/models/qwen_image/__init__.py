"""Qwen-Image on the shared MMDiT."""
