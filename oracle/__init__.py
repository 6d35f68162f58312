"""CPU oracle for the GRU training path (test infrastructure only).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline
leg may import this package, and there only as the checker or the timed CPU
baseline.  The product path in ``rnn_kernel_b200`` never calls it.
"""
