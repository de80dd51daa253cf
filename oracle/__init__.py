"""CPU oracle of the MoE-experts path (test infrastructure; never imported by the product)."""
