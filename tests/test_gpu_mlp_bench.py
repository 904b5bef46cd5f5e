"""The MLP microbenchmark (ffn_pack_x0 + ffn_mlp_bench) against a plain PyTorch fp32 reference of the
same computation: density MLP 32 -> 64 -> 16 and colour MLP [16 density outputs, SH16(d)] -> 64 -> 64 ->
3 with sigmoid_soft, d = (0.36, 0.48, 0.8), loss sum 0.5 (rgb - 0.5)^2, gradients summed over the
samples.  ffn_mlp_bench forms every product from compensated fp16 operand pairs (the training step's
form), with fp32 accumulation: each parameter's gradient is held to rel-L2 1e-2 of the reference (the
contract's gradient tolerance).  ffn_mlp_bench_f16 multiplies plain fp16 operands (one MMA per
product, fp32 accumulation), held to 5e-2: fp16 rounding of the activations and deltas of every layer.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import ffn_native as fn
from _helpers import rel_l2
from ffn_config import make_geometry, param_layout, param_shapes


def sh16(x, y, z):
    """Real spherical harmonics of degrees 0..3 (ffnerf_OG.cl:572-602), float64."""
    return np.array([
        0.28209479177387814, 0.4886025119029199 * y, 0.4886025119029199 * z, 0.4886025119029199 * x,
        1.0925484305920792 * x * y, 1.0925484305920792 * y * z, 0.31539156525252005 * (3 * z * z - 1),
        1.0925484305920792 * x * z, 0.5462742152960396 * (x * x - y * y),
        0.5900435899266435 * y * (3 * x * x - y * y), 2.890611442640554 * x * y * z,
        0.4570457994644658 * y * (5 * z * z - 1), 0.3731763325901154 * (5 * z * z * z - 3 * z),
        0.4570457994644658 * x * (5 * z * z - 1), 1.445305721320277 * z * (x * x - y * y),
        0.5900435899266435 * x * (x * x - 3 * y * y)])


def seeded_blob(F=2, ND=1, NC=2, seed=3):
    """He-normal hidden weights, N(0, 0.1) heads (<= 16 outputs), N(0, 0.05) biases."""
    lay, total = param_layout(F, ND, NC)
    shapes = param_shapes(F, ND, NC)
    rng = np.random.default_rng(seed)
    blob = np.zeros(total, np.float32)
    for name, (off, size) in lay.items():
        if not size:
            continue
        if name.startswith("W"):
            out_, in_ = shapes[name]
            std = 0.1 if out_ <= 16 else np.sqrt(2.0 / in_)
        else:
            std = 0.05
        blob[off:off + size] = rng.normal(0.0, std, size)
    return blob, lay, shapes


@pytest.mark.parametrize("form,tol", [("compensated", 1e-2), ("plain_f16", 5e-2)])
def test_mlp_bench_matches_torch_fp32(form, tol):
    g = make_geometry(F=2, ND=1, NC=2, spr=64, G=16, log2_entries=12, rmax=512.0)
    ctx = fn.Context(g, mlp_precision="fp16")
    blob, lay, shapes = seeded_blob()
    ctx.tensor(fn.BUF_PARAMS).copy_(torch.from_numpy(blob))
    grads = ctx.tensor(fn.BUF_GRADS)
    grads.zero_()
    table_before = ctx.tensor(fn.BUF_TABLE).clone()
    n = 1 << 14
    x = torch.randn((n, 32), generator=torch.Generator().manual_seed(5)).half()
    tiles = torch.empty(ctx.x0_tile_bytes(n), dtype=torch.uint8, device="cuda")
    ctx.pack_x0(x.cuda(), tiles, n)
    (ctx.mlp_bench if form == "compensated" else ctx.mlp_bench_f16)(tiles, n)
    torch.cuda.synchronize()
    g_all = grads.cpu().numpy()
    n_mlp = blob.size
    assert not g_all[:-n_mlp].any(), "the microbenchmark must not touch the table gradients"
    assert torch.equal(ctx.tensor(fn.BUF_TABLE), table_before)
    g_dev = g_all[-n_mlp:]

    P = {k: torch.tensor(blob[o:o + s].reshape(shapes[k]), dtype=torch.float64, requires_grad=True)
         for k, (o, s) in lay.items() if s}
    xf = x.double()
    h1 = torch.relu(xf @ P["Wd_in"].T + P["bd_0"])
    dout = h1 @ P["Wd_out"].T + P["bd_out"]
    sh = torch.tensor(sh16(0.36, 0.48, 0.8), dtype=torch.float64).expand(n, 16)
    cin = torch.cat([dout, sh], 1)
    c1 = torch.relu(cin @ P["Wc_in"].T + P["bc_0"])
    c2 = torch.relu(c1 @ P["Wc_01"].T + P["bc_1"])
    co = c2 @ P["Wc_out"].T + P["bc_out"]
    rgb = torch.sigmoid(torch.clamp(0.5 * co, -18.0, 18.0))
    (0.5 * (rgb - 0.5) ** 2).sum().backward()
    for k, t in P.items():
        o, s = lay[k]
        ref = t.grad.detach().numpy().reshape(-1)
        assert np.isfinite(g_dev[o:o + s]).all(), k
        assert rel_l2(g_dev[o:o + s], ref) < tol, (k, rel_l2(g_dev[o:o + s], ref))
    assert ctx.status() == 0


def test_mlp_bench_rejects_bad_sizes():
    g = make_geometry(F=2, ND=1, NC=2, spr=64, G=16, log2_entries=12, rmax=512.0)
    ctx = fn.Context(g, mlp_precision="fp16")
    tiles = torch.empty(ctx.x0_tile_bytes(200), dtype=torch.uint8, device="cuda")
    with pytest.raises(Exception):
        ctx.mlp_bench(tiles, 200)            # not a multiple of the 128-row tile
    ctx32 = fn.Context(g, mlp_precision="fp32")
    with pytest.raises(Exception):
        ctx32.mlp_bench(tiles, 128)          # compiled for the tensor-core MLP only
