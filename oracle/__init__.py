"""CPU oracle of the Wan attention-prep path (test infrastructure only; see wan_prep.py)."""
