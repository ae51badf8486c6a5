"""HunyuanVideo 1.0 / 1.5 on the shared MMDiT."""
