"""MACE-ICTC interatomic potential on the ICTC-O3 CUDA backend."""
