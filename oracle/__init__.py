"""CPU checkers for the CUDA library (test infrastructure only; see oracle.py)."""
