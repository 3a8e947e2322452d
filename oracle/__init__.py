"""CPU oracle for the block-sparse attention path (TEST INFRASTRUCTURE ONLY).

This package restates, on the CPU, the algorithms of sparse-ai's ``src/ultrametric``
hot path so that the CUDA kernels can be checked against them:

* ``block_list_oracle``  -- routing vectors -> block mask -> ascending block lists,
  and the key-block -> query-block transposition (``src/ultrametric/block_list.py``).
* ``attention_oracle``   -- masked dense softmax attention, its log-sum-exp and its
  gradients (``src/ultrametric/block_list.py:361-378``; the reference's CPU path
  ``src/ultrametric/kernel.py:574-580``).
* ``decode_oracle``      -- routed paged decode (``src/ultrametric/kernel_decode.py:129-185``).

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference itself (its torch
paths and its Triton kernels under ``TRITON_INTERPRET=1``) and stored the outputs as
fixtures in ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this oracle
against every one of them.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline leg and
its ``--impl reference`` arm) may import this package, and only as the checker or the
timed CPU baseline.  The product (``sparse-ai_b200/ultrametric``) never imports it and
has no CPU path.
"""
