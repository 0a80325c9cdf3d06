"""CPU restatement of the reference's MoE-step algorithms — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and
its --impl reference arm) may import this package, as the checker or as the
timed CPU baseline.  Nothing in the product path imports it.
"""
