"""TEST INFRASTRUCTURE ONLY: CPU oracle for the TriTierCache decode hot path (see oracle.py)."""
