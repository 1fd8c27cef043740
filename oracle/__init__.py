"""CPU oracle (test infrastructure only; never imported by the ddq_b200 product path)."""
