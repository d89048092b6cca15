"""noise_b200: the B200 (sm_100a) hot path of Noise's forward-only training.

- ``noise_b200.population``: drop-in ``population_loss`` (EGGROLL's population-perturbed forward of the fixed GPT).
- ``noise_b200.moment_kernels``: drop-in credit-readout ops (the reference's ``train/speedrun/moment_kernels.py``).

All compute runs in the in-tree ``libnoise_b200.so`` (C ABI: ``include/noise_b200.h``); there is no CPU fallback.
"""
from . import _lib
from .population import (PackedGPT, gpt_loss, head_loss, member_offsets, param_shapes, population_loss,
                         population_loss_offsets)

__all__ = ['PackedGPT', 'gpt_loss', 'head_loss', 'member_offsets', 'param_shapes', 'population_loss',
           'population_loss_offsets', '_lib']
