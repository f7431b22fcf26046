"""CPU oracle (TEST INFRASTRUCTURE ONLY).

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU legs as the
checker / CPU baseline. The product package (codpiece_b200) never imports it.
"""
