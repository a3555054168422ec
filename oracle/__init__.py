"""CPU oracle of the DWDP MoE-layer hot path: test infrastructure only (see moe_oracle)."""
