"""Host-side planning for the fused FFN: input contract, tiling plan, implementation selection."""
