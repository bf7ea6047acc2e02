"""CPU oracle of the NVFP4 MoE layer (test infrastructure only; see nvfp4_oracle)."""
