"""CPU oracle for the FA2 forward (test infrastructure only)."""
