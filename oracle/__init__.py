"""CPU oracle for the linear-layer hot path (test infrastructure only)."""
