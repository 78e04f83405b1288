"""CPU oracle of the attention hot path (test infrastructure; never used by the product path)."""
