"""CPU oracle for the gsplat_b200 hot path -- test infrastructure only (see oracle.py)."""
