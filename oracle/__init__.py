"""CPU oracle of the DFA hot path.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import
anything from here, and only as the checker (or as the timed CPU implementation of the
reference algorithm).  The product path in ``sparse4d-tt_b200/`` never imports it.

* ``dfa_torch``: torch fp32 restatement of the reference's PyTorch DFA
  (``test/dfa_pcc.py:211-358``), the float oracle and the timed CPU baseline.
* ``dfa_numpy``: numpy float32 restatement with explicit bilinear taps and a fixed
  evaluation order for the keypoint projection, the cross-check of ``dfa_torch`` and the
  reference for the integer outputs (depth mask, visibility, compacted indices).

Parity of both is pinned against fixtures generated from the reference itself
(``tests/golden/make_golden.py`` imports ``test/dfa_pcc.py`` and runs it).
"""
