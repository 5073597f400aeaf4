"""CPU oracle (test infrastructure only; see gw_oracle.py)."""
