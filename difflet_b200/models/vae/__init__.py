"""VAE decoders: 2-D KL autoencoder (FLUX / Qwen-Image) and causal 3-D video VAEs (Wan / HunyuanVideo)."""
