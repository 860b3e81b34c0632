"""Higher-level O(3) operators built on the CUDA backend."""
