"""CPU oracle of the SimSD hot path: TEST INFRASTRUCTURE ONLY (see oracle.py)."""
