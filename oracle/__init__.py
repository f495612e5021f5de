"""CPU oracle for the actkv eviction hot path: test infrastructure only (see actkv_oracle.py)."""
