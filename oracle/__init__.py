"""CPU oracle for the tt-splat matrix-native render/train hot path.

TEST INFRASTRUCTURE ONLY.  This package is a numpy restatement of the reference's CPU torch
path (kinginu/tt-splat ``spike/`` and ``tools/m4_train_binned.py`` and friends); every function
cites the reference file:line it follows.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it, and there only as
the checker or the timed CPU baseline.  The product path (the ``tt-splat_b200`` package and its
CUDA library) never imports, links or executes anything in here.

Parity pinning: the oracle is checked against golden vectors produced by running the reference
itself in the build container (``tests/golden/make_golden.py``) and against the known-answer
values of the reference's own tests (``spike/tests/test_transform.py:15-31``).  The SSIM term
is pinned to the reference's restatement ``tools/loss_manual.py`` only: the third-party
``pytorch_msssim`` 1.0.0 that ``spike/metrics.py:3`` calls is not installed anywhere here, so
parity against that package itself is unpinned.
"""
