"""CPU oracle of the fused decode-sampling step (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline leg may
import this package; the product library never does.
"""
