"""TEST INFRASTRUCTURE ONLY: CPU oracle for the sdvk hot path (see oracle.h)."""
