"""ORACLE — test infrastructure only.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline``
leg (and its ``--impl reference`` arm) may import this package, and only as the
checker or the timed CPU baseline. The product (``cascade_cpp``) never imports
it and has no CPU fallback.

Contents
--------
* ``sha256_oracle.c`` — plain-C FIPS 180-4 restatement of
  ``compute_block_id`` (cascade_Code/cpp/src/cascade_core.cpp:47-58).
* ``store_oracle.py`` — sequential restatement of the store semantics
  (dedup, get, contains, prefix-protected demotion).
* ``Makefile`` — builds the C oracle into ``oracle/_build`` and, when the
  reference sources are present, the reference's own CPU path into
  ``oracle/_ref`` (``cascade_ref`` module via ``ref_shim.cpp``).
"""
