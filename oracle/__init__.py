"""CPU restatement of the reference arithmetic (test infrastructure only)."""
