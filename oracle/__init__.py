"""CPU oracle of the ICTC-O3 hot path: test infrastructure, never a product path."""
