"""Device batch generation (ffn_batch_generate / ffn_batch_errors / ffn_batch_feedback through
batch_gpu.GpuBatchProducer) against the host module and the reference's own feedback code.

Contracts:
  * rays and targets of the drawn (image, x, y) equal rays_targets_from_indices (the host mirror,
    pinned bit for bit to the reference by golden_rays.npz) within 2 ulp-scale (abs 1e-6) on the
    direction, exactly on origin and colour; K given, per-image K and the no-K fallback;
  * the rejection draw follows the weight map: a proposal is accepted when a uniform byte is <= its
    weight, i.e. with probability (w + 1) / 256, so with weight 255 on 1/16 of the pixels and 1
    elsewhere 16 / (16 + 15/8) = 0.895 of the weighted draws land there (+-0.01); uniform draws cover
    pixels and images evenly (+-0.01);
  * a batch depends only on its seed and inputs (two producers with one seed agree bit for bit);
  * the weight-map feedback reproduces the reference's _update_weights_u8 bit for bit on the
    golden fixture (distinct pixels), including the background cap and the median scale;
  * the device loss figures (mse, rmse, l2) equal the trainer's formulas within 1e-6 relative.
"""
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import batch_gpu as bg
import ffnerf_tools as ft

GOLD = Path(__file__).resolve().parent / "golden"


def _host_rays(prod, Ims, c2w, K):
    im = prod.im.cpu().numpy()
    x = prod.x.cpu().numpy()
    y = prod.y.cpu().numpy()
    r, t = ft.rays_targets_from_indices(im, x, y, Ims, c2w, prod.W, prod.H, K=K)
    return np.ascontiguousarray(r).view(np.float32).reshape(-1, 8), t


@pytest.mark.parametrize("kmode", ["K", "Ks", "none"])
def test_rays_match_host_module(kmode):
    g = np.load(GOLD / "golden_rays.npz")
    Ims, c2w, K, Ks = g["Ims"], g["c2w"], g["K"], g["Ks"]
    W, H = int(g["W"]), int(g["H"])
    if kmode == "Ks":
        Ims, c2w, Kuse = Ims[:2], c2w[:2], Ks
    else:
        Kuse = K if kmode == "K" else None
    prod = bg.GpuBatchProducer(Ims, c2w, Kuse, W, H, batch_rays=4096, rng_seed=5)
    rays, tg = prod.next_batch()
    torch.cuda.synchronize()
    hr, ht = _host_rays(prod, Ims, c2w, Kuse)
    r = rays.cpu().numpy()
    assert np.array_equal(r[:, :4], hr[:, :4])
    assert np.abs(r[:, 4:] - hr[:, 4:]).max() < 1e-6
    assert np.array_equal(tg.cpu().numpy(), ht)


def test_uint8_targets_and_determinism():
    g = np.load(GOLD / "golden_batch_feedback.npz")
    Ims = g["Ims"]
    N, H, W = Ims.shape[:3]
    c2w = np.tile(np.eye(4, dtype=np.float32), (N, 1, 1))
    K = np.array([[10.0, 0, W / 2], [0, 10.0, H / 2], [0, 0, 1]], np.float32)
    a = bg.GpuBatchProducer(Ims, c2w, K, W, H, batch_rays=2048, rng_seed=9)
    b = bg.GpuBatchProducer(Ims, c2w, K, W, H, batch_rays=2048, rng_seed=9)
    ra, ta = a.next_batch()
    rb, tb = b.next_batch()
    torch.cuda.synchronize()
    assert torch.equal(ra, rb) and torch.equal(ta, tb) and torch.equal(a.im, b.im)
    hr, ht = _host_rays(a, Ims, c2w, K)
    assert np.array_equal(ta.cpu().numpy(), ht)
    rc, _ = a.next_batch()                     # the next batch draws other pixels
    assert not torch.equal(rc, ra)


def test_rejection_follows_weights():
    N, H, W = 4, 64, 64
    Ims = np.zeros((N, H, W, 3), np.uint8)
    c2w = np.tile(np.eye(4, dtype=np.float32), (N, 1, 1))
    n = 1 << 20
    prod = bg.GpuBatchProducer(Ims, c2w, None, W, H, batch_rays=n, rng_seed=3, uniform_frac=0.0, max_tries=4096)
    prod.weights.fill_(1)
    prod.weights[:, :16, :16] = 255                     # 1/16 of every image
    prod.next_batch()
    torch.cuda.synchronize()
    x, y, im = prod.x.cpu().numpy(), prod.y.cpu().numpy(), prod.im.cpu().numpy()
    hot = np.mean((x < 16) & (y < 16))
    assert abs(hot - 16.0 / (16.0 + 15.0 / 8.0)) < 0.01, hot
    assert np.all(np.abs(np.bincount(im, minlength=N) / n - 1.0 / N) < 0.01)
    uni = bg.GpuBatchProducer(Ims, c2w, None, W, H, batch_rays=n, rng_seed=4, uniform_frac=1.0)
    uni.weights.copy_(prod.weights)
    uni.next_batch()
    torch.cuda.synchronize()
    x, y = uni.x.cpu().numpy(), uni.y.cpu().numpy()
    assert abs(np.mean((x < 16) & (y < 16)) - 1.0 / 16.0) < 0.01


def test_feedback_matches_reference_update():
    g = np.load(GOLD / "golden_batch_feedback.npz")
    Ims = g["Ims"]
    N, H, W = Ims.shape[:3]
    c2w = np.tile(np.eye(4, dtype=np.float32), (N, 1, 1))
    n = g["im"].size
    prod = bg.GpuBatchProducer(Ims, c2w, None, W, H, batch_rays=n, rng_seed=1, ema=0.05, bg_cap=16, fg_tau=8)
    prod.weights.copy_(torch.from_numpy(g["w_before"]))
    prod.im.copy_(torch.from_numpy(g["im"]))
    prod.x.copy_(torch.from_numpy(g["x"]))
    prod.y.copy_(torch.from_numpy(g["y"]))
    prod.err.copy_(torch.from_numpy(g["err"]))
    assert float(bg.median_like_numpy(prod.err).item()) == float(g["median"])
    prod.apply_errors()
    torch.cuda.synchronize()
    assert np.array_equal(prod.weights.cpu().numpy(), g["w_after"])
    # the per-ray error kernel: out = target + e on every channel gives e
    tg = torch.zeros((n, 4), device="cuda")
    out = tg.clone()
    out[:, :3] = torch.from_numpy(g["err"]).cuda()[:, None]
    prod.lib.ffn_batch_errors(bg._ptr(out), bg._ptr(tg), n, bg._ptr(prod.err), None, None)
    torch.cuda.synchronize()
    assert torch.allclose(prod.err.cpu(), torch.from_numpy(g["err"]), rtol=1e-6, atol=0)


def test_batch_metrics_match_trainer_formulas():
    rng = np.random.default_rng(4)
    n = 100003
    pred = rng.random((n, 4), dtype=np.float32)
    targ = rng.random((n, 4), dtype=np.float32)
    m = bg.batch_metrics(torch.from_numpy(pred).cuda(), torch.from_numpy(targ).cuda(), n).cpu().numpy()
    d = pred[:, :3].astype(np.float64) - targ[:, :3]
    mse = np.mean(d ** 2)
    ref = [mse, np.sqrt(mse), np.sqrt(np.mean(np.sum(d ** 2, axis=1)))]
    np.testing.assert_allclose(m, ref, rtol=1e-6)
