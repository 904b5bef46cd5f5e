"""The device-resident training loop (trainer.train: GPU batch generation, Nerf.step, device metrics
and pixel-weight feedback) on the synthetic cfg1 scene.

Contracts: 2,000 steps lower the batch MSE to under a third of the first report and lift the PSNR
of renders of the training views above 15 dB (the model learns the scene); the tensor-core and
fp32 MLPs end within 1 dB of each other in that PSNR, each taken as the median of five runs.  The
trajectories differ by float rounding only, which the training dynamics amplify, and the immediate
(Hogwild) table update adds its float atomics in a different order from run to run, so one
precision's own runs spread too: measured on a B200, 17.78-19.25 dB (tensor-core MLP) and
18.38-19.26 dB (fp32 MLP) over four runs of the same seed, medians 19.13 and 19.01 dB.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import trainer


RUNS = 5


def test_training_loop_learns_and_precisions_agree():
    runs = {}
    for prec in ("fp16", "fp32"):
        runs[prec] = []
        for _ in range(RUNS):
            nerf, hist, data = trainer.synthetic_run("cfg1", steps=2000, mlp_precision=prec, seed=0, log=False)
            assert hist[-1][1] < hist[0][1] / 3.0, hist
            runs[prec].append(trainer.evaluate_psnr(nerf, *data))
            nerf.native.close()
            assert runs[prec][-1] > 15.0, runs
    med = {prec: float(np.median(v)) for prec, v in runs.items()}
    assert abs(med["fp16"] - med["fp32"]) < 1.0, runs
