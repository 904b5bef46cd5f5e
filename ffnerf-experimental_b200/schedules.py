"""Training schedules of the reference trainer (run_ffnerf_OG.py:49-62, 1158, 1356-1365).

lr_f(step)      = max(lr * sqrt(65536 / (B*S)) * exp(-lambda * step), LR_FLOOR),
                  lambda = lmbda_base * sqrt(B*S / 65536)
sh(step)        = clip((step - 2*T_MID) / T_MID, 0, 1)
occ(step)       = step > T_MID
color_lr(step)  = 0.15 + 0.85 * clip((step - T_MID) / T_MID, 0, 1)
"""
from __future__ import annotations

import numpy as np

LMBDA_BASE = 1e-4
LR_FLOOR = 5e-6
T_MID = 1500


def sh_multiplier_function(step):
    return np.clip((step - (2 * T_MID)) / (T_MID), 0.0, 1.0)


def occ_u_multiplier_function(step):
    return step > T_MID


def color_MLP_rel_lr_function(step):
    return 0.15 + 0.85 * min(1.0, max(0.0, (step - T_MID) / (T_MID)))


def lr_lambda(lmbda_base: float, batch_rays: int, samples_per_ray: int) -> float:
    return lmbda_base * np.sqrt((batch_rays * samples_per_ray) / (1024 * 64))


def lr_schedule(step: int, lr: float, lmbda: float, batch_rays: int, samples_per_ray: int) -> np.float32:
    return np.float32(np.maximum(lr * np.sqrt((1024 * 64) / (batch_rays * samples_per_ray)) * np.exp(-lmbda * step),
                                 LR_FLOOR))
