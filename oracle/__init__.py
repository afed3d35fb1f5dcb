"""CPU oracle (test infrastructure only; see heartmula_oracle.py)."""
