"""CPU oracle of the NF4 path.  Test infrastructure only: imported by tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline legs, never by stratum_b200."""
