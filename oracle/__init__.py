"""CPU oracle for the sparse-conv engine (test infrastructure only; never on the product path)."""
