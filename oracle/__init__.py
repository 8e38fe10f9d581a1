"""CPU oracle for the NVFP4 linear path (test infrastructure only; see nvfp4_oracle.py)."""
