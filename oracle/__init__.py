"""CPU oracle for the complex chunkwise SSD operator. This is test infrastructure only.

Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` may import
this package, and only as the checker or as the timed CPU baseline. The product path lives in
``mamba-3-lite_b200/m3ssd`` and never calls into it.

Modules:
  ssd_oracle     numpy restatement of the reference operator (chunkwise, masked before exp), the
                 naive O(T) recurrence in complex128 and its adjoint (gradients).
  ssd_torch_cpu  torch-on-CPU restatement of the reference chunkwise path with autograd; it is the
                 timed CPU baseline ("port") for forward+backward.
  cases          seeded input generators for the reference test shapes and the block shapes.
  metrics        the three error figures used for parity reports.

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference's own ``ssd_complex_chunkwise``
(models/ssd_complex.py:58-119) and its autograd on the cases in ``cases.py``, and
``tests/test_oracle.py`` checks this oracle against those fixtures.
"""
