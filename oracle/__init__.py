"""CPU oracle of the dense-op path (test infrastructure only; see oracle.h)."""
