"""CPU oracle of the four-op hot path (test infrastructure; see ops_oracle.py)."""
from oracle import ops_oracle  # noqa: F401
