"""CPU oracle for the SignRound v2 block-tuning path. TEST INFRASTRUCTURE ONLY.

Nothing in ``mround_b200`` imports this package.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may use it, and there only as the checker or as the
timed CPU baseline, never as the measured product path.

Contents, each function citing the reference file:line it restates
(paths relative to the fbaldassarri/mround tree, version 0.1.0a6):

- ``quant_fp32``  float32 fake-quant forward, codes, the straight-through
  backward in the composition MLX autodiff produces, signSGD and projection
  (``mround/core/quantizer.py``, ``mround/core/signsgd.py``,
  ``mround/reference/quantize.py``).
- ``losses_fp32``  block MSE and the outlier-suppressed MSE with a global
  threshold (``mround/core/losses.py``).
- ``packing``  MLX uint32 code packing and the affine scale/bias conversion
  (``mround/formats/packing.py``, ``mround/formats/mlx_export.py``).
- ``deltaloss``  per-layer ``sum |g * (Q(W) - W)|`` in float64
  (``mround/planner/sensitivity.py:190-229``).
- ``block_tuner``  torch-CPU float32 restatement of one decoder block and the
  per-block tuning loop (``mround/pipeline/runner.py:790-953``).

Parity is pinned: ``tests/golden/make_golden.py`` imports the reference's own
NumPy oracle (``mround/reference/*``, ``mround/planner/*``) and records its
outputs on seeded inputs; ``tests/test_oracle_golden.py`` checks this oracle
against those fixtures at the reference's own MLX-versus-NumPy tolerances
(``tests/unit/test_mlx_parity.py:58, 95-98, 213-234, 264-311``).
"""
