"""CPU oracle of the linear path -- test infrastructure only (see reference.py)."""
