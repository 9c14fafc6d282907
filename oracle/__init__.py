"""CPU oracle and reference-kernel build recipe (test infrastructure only)."""
