"""CPU oracle for the heliox_b200 hot path (test infrastructure only)."""
