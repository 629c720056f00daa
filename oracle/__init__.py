"""CPU oracle for the hypno Q4_0 path (test infrastructure; see oracle.py)."""
