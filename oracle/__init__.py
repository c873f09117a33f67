"""CPU oracle for the NVFP4 GEMM path -- test infrastructure only (see oracle/oracle.py)."""
