"""CPU oracle (test infrastructure only; see coalibi_oracle.py)."""
