"""CPU oracle for the per-layer optimizer step (test infrastructure only)."""
