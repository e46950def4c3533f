"""CPU oracle of the NNop hot path -- test infrastructure only (see nnop_oracle)."""
