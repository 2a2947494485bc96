"""Oracle package: the CPU checker for the CUDA path (test infrastructure only)."""
