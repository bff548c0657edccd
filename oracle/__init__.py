"""CPU oracle for the ragged-batch attention path.  TEST INFRASTRUCTURE ONLY.

A restatement of the reference's algorithms (nano_infer_engine, pure
PyTorch/Python) that runs on the host:

* ``paging``    - allocator, block tables and the ragged metadata
                  (query_start_loc, positions, slot mapping) as integers;
* ``attention`` - paged decode and varlen causal attention with the
                  reference's rounding sequence, in torch on the CPU;
* ``engine``    - the Llama forward over a paged cache (reference model,
                  layers and cache semantics) used as the timed CPU baseline.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only
as the checker or the baseline; the product (``nano_infer_engine_b200``)
never calls it.  It is pinned against golden vectors produced by the real
reference (``tests/golden/make_golden.py``).
"""
