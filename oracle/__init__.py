"""CPU oracle for noise_b200 — TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch on the CPU, the reference algorithms that the CUDA path replaces:

- ``oracle.gpt``      the fixed 37.7M GPT of Noise (reference ``utils/model.py``).
- ``oracle.eggroll``  the EGGROLL population-perturbed forward, noise map and seed-rebuilt update
                      (reference ``archive/10M/train/val/eggroll.py``).
- ``oracle.credit``   dense restatements of the credit-readout kernels (reference
                      ``train/speedrun/moment_kernels.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may import it, and only as
the checker or the timed CPU baseline. The product path (``noise_b200``) never imports this package; it fails loudly
when its CUDA library is missing.

Parity pinning: ``tests/golden/make_golden.py`` runs the reference itself (imported read-only in the build container)
and commits its outputs under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this restatement against them.
"""
