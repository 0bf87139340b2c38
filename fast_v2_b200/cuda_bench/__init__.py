"""Drop-in for the reference's cuda_bench/ extension module (fused gather + RMSNorm)."""
