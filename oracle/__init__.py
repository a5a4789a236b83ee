"""CPU oracle of the reference Q8 path — test infrastructure only (see q8_oracle.py)."""
