"""CPU oracle of the attention hot path -- test infrastructure only.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU baseline as the
checker; the drop-in modules never import it.
"""
