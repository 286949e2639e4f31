"""CPU oracle for the MoE hot path (test infrastructure, never product code)."""
