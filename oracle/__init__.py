"""CPU oracle for the attention path — test infrastructure only.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs
as the checker and the timed CPU reference; never by the product package.
"""
