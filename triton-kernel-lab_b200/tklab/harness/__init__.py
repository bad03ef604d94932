"""Correctness policy and validation helpers shared with the reference harness."""
