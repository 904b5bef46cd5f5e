"""The device-resident training loop (trainer.train: GPU batch generation, Nerf.step, device metrics
and pixel-weight feedback) on the synthetic cfg1 scene.

Contracts: 2,000 steps lower the batch MSE to under a third of the first report and lift the PSNR
of renders of the training views above 15 dB (the model learns the scene); the tensor-core and
fp32 MLPs end within 1 dB of each other in that PSNR (the two trajectories differ by float rounding
only, which the training dynamics amplify).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import trainer


def test_training_loop_learns_and_precisions_agree():
    runs = {}
    for prec in ("fp16", "fp32"):
        nerf, hist, data = trainer.synthetic_run("cfg1", steps=2000, mlp_precision=prec, seed=0, log=False)
        assert hist[-1][1] < hist[0][1] / 3.0, hist
        runs[prec] = trainer.evaluate_psnr(nerf, *data)
        assert runs[prec] > 15.0, runs
    assert abs(runs["fp16"] - runs["fp32"]) < 1.0, runs
