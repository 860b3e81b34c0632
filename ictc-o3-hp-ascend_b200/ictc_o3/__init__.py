"""ICTC-O3 operators on a B200-native (sm_100a) CUDA backend."""
__version__ = "0.1.0"
