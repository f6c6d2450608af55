"""
The oracle: a CPU restatement of the reference's arithmetic for the hot path.

TEST INFRASTRUCTURE ONLY. Only tests/, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import
anything here, and only as the checker or the timed CPU baseline; the product
(``create_graph_b200``) never imports it and has no CPU fallback.

- ``oracle.edge_attn``: forward1 / backward1 / backward2 of the masked edge
  attention in numpy float64, following kernels/edge_attn/ops.py:26-104 of the
  reference. Pinned against golden vectors the reference itself produced
  (tests/golden/make_golden.py imports it read-only).
- ``oracle.geometry``, ``oracle.segment``, ``oracle.neighbors``: numpy
  restatements of the eager geometry, segment sums and neighbour lists the
  reference leaves to model code (tests/test_semantics.py:46-69 there).
- ``oracle.step``: the reference's own algorithm for one training step, i.e.
  eager ``torch.autograd.grad(create_graph=True)`` over plain torch CPU ops
  (src/create_graph/api.py:200-211, ``exact=True``), on the model spec of
  ``create_graph_b200.mlip``; it is the timed CPU baseline.
"""
