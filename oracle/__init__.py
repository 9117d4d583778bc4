"""CPU restatement of AIHost's attention path — test infrastructure only (see oracle.py)."""
