"""CPU oracle for the lossless BF16 weight-decode path -- TEST
INFRASTRUCTURE ONLY. Imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg; never by the afterimage_b200 product."""
