"""The device-resident training loop (trainer.train: GPU batch generation, Nerf.step, device metrics
and pixel-weight feedback) on the synthetic cfg1 scene.

Contracts: 1,500 steps lower the batch MSE to under a third of the first report (the model learns
the scene); the tensor-core and fp32 MLPs end within 0.5 dB PSNR of each other (mean of the last
five reports; the two trajectories differ by float rounding only); the weight maps moved away
from their initial value 16 (feedback ran).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import trainer


def _psnr(hist):
    mse = np.mean([h[1] for h in hist[-5:]])
    return -10.0 * np.log10(mse)


def test_training_loop_learns_and_precisions_agree():
    runs = {}
    for prec in ("fp16", "fp32"):
        nerf, hist = trainer.synthetic_run("cfg1", steps=1500, mlp_precision=prec, seed=0, log=False)
        assert hist[-1][1] < hist[0][1] / 3.0, hist
        runs[prec] = _psnr(hist)
    assert abs(runs["fp16"] - runs["fp32"]) < 0.5, runs
