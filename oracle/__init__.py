"""CPU oracle for the attention forward (test infrastructure only; see reference_attention.py)."""
