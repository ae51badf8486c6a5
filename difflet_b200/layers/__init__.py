"""Shared model layers: RoPE tables, timestep / text embedding helpers."""
