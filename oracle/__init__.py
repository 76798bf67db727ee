"""CPU oracle for the W4A16 GEMV path -- test infrastructure only (see oracle.py)."""
