"""CPU oracle for the SageAttention hot path (test infrastructure; never imported by the product)."""
