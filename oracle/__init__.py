"""CPU oracle (test infrastructure only); see aoh_oracle.py."""
