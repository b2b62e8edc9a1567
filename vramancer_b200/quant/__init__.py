"""Weight quantisation: NVFP4 (e2m1 + e4m3 block-16 scales + fp32 per-tensor scale)."""
