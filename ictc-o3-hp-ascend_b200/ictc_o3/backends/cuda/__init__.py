"""B200 (sm_100a) backend: hand-written CUDA kernels behind libictc_cuda.so."""
