"""CPU oracle and reference GPU oracle (test infrastructure only)."""
