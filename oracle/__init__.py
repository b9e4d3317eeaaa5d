"""CPU oracle for the optimizer step (test infrastructure only; see moteopt_oracle.py)."""
