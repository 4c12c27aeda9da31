"""CPU oracle for the MoE path: test infrastructure, never part of the product path."""
