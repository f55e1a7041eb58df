"""CPU oracle for the MoE block -- test infrastructure only (never imported by the product)."""
