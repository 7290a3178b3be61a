"""CPU oracle of the Zealot attention hot path -- test infrastructure only.

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline import it.
"""
