"""TEST INFRASTRUCTURE ONLY: the CPU oracle of the replay engine (see oracle.py)."""
