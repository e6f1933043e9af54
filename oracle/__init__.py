"""CPU oracle for the selective-scan / conv1d / decode-step hot path.

TEST INFRASTRUCTURE ONLY. This package is the checker, never the thing measured or shipped: only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) may import it. The product package ``mamba_metal_b200`` never imports it and
has no CPU fallback.

Contents:

- ``scan_ref``   -- NumPy restatement of the reference's own sequential CPU references for the scan
  (``experiments/09-features/test_features.py:13-43``, ``experiments/10-fp16/test_fp16.py:28-55``,
  ``experiments/18-prefill/verify_state_out.py:13-26``, ``experiments/05-pair-scan/pair_scan.py:36-42``),
  the conv1d semantics of ``mamba_metal/mamba_block.py:45-52`` and the decode-step formulas of
  ``mamba_metal/mamba_block.py:155-198``. Pinned against golden vectors produced by running those
  reference functions (``tests/golden/make_golden.py``).
- ``scan_ref.c`` -- the same sequential scan in plain C with OpenMP over (batch, channel), for sizes the
  NumPy loops cannot finish in seconds and for the timed CPU baseline. Cross-checked against
  ``scan_ref``.
- ``model_ref``  -- a float32 PyTorch-on-CPU restatement of ``MambaBlock`` / ``MambaModel`` /
  ``generate_fast`` (``mamba_metal/mamba_block.py:68-198``, ``mamba_model.py:35-127``,
  ``generate.py:65-110``) built from plain tensor ops. The reference's MLX layers (Conv1d, RMSNorm,
  Linear, softplus) are not importable here, so the model-level semantics are restated from their
  documented behaviour: parity of those layers against MLX itself is unpinned.
"""
