"""CPU oracle for the B200 cached-attention path — TEST INFRASTRUCTURE ONLY.

Plain torch-CPU / numpy restatements of the reference's arithmetic for this path, each
function citing the Hy-Nomas file:line it follows.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) may import this package, and only as the checker or the timed
CPU baseline; the product package ``hy_nomas_b200`` never imports it.

Pinning: ``tests/golden/`` holds fixtures produced by running the reference's own
functions in this container (``tests/golden/make_golden.py``); ``tests/test_oracle_golden.py``
checks every restatement here against them.
"""
