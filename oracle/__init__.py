"""CPU oracle for the decode path -- TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg, as the checker and the timed CPU baseline; the product never imports it.
Parity is unpinned by the reference's own golden vectors (they need real
checkpoints absent from the reference tree); see oracle/ops.py for what pins it.
"""
