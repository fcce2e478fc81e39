"""CPU oracles for the MiniPrefix forward -- test infrastructure only (see oracle.py)."""
