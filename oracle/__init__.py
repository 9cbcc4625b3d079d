"""TEST INFRASTRUCTURE — CPU oracle of the absorbed-MLA attention task (see mla_oracle.py).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may import it.
"""
