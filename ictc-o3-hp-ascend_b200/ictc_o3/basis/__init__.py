"""ICTC harmonic basis, CG tensors and path structure (host-side constants)."""
