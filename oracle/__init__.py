"""CPU oracle for the drafter-loss hot path -- TEST INFRASTRUCTURE ONLY.

This package restates the reference's own correctness oracles on the CPU:
  - oracle.dpace   : losses/dpace_ref.py:8-51 (torch) and the specforge weight
                     restatement in losses/tests/test_dpace.py:21-45, plus an
                     independent float64 numpy restatement with the analytic
                     gradient;
  - oracle.dflash  : the speculators objective embedded in
                     models/dflash/tests/test_loss.py:21-49 (torch), plus a
                     float64 numpy restatement with the analytic gradient.
Pinned against golden vectors produced by the reference's own code
(tests/golden/make_golden.py, fixtures in tests/golden/).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline arm may import
this package, and only as the checker or as the timed CPU baseline. The
product path (specdec, losses, models) never touches it.
"""
