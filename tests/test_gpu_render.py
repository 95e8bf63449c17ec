"""The fused render path (gs_render_forward / gs_render_backward, what RasterizeFunction runs)
against the reference's chain of six ops through the same module: identical forward (image,
contributor counts, transmittance, sorted ids, ranges), screen radii equal to the reference
wrapper's torch expression bit for bit, gradients within 1e-4 relative."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from test_gpu_parity import assert_grad_close, np32, scenes_small

pytestmark = pytest.mark.gpu


def op_chain(crc, sc, view, dev, grad_img):
    mu, q, s, al, A, kj = (p.to(dev).contiguous() for p in sc.params())
    R, t = view.R.to(dev).contiguous(), view.T.to(dev).contiguous()
    cam = (-torch.matmul(R.T, t)).reshape(3).contiguous()
    m2, c2, d = crc.project(sc.N, mu, q, s, R, t, view.fx, view.fy, view.cx, view.cy)
    col = crc.SH(sc.N, cam, mu, A, kj)
    op = torch.sigmoid(al).contiguous()
    img, ids, ranges, fT, nc = crc.rasterize(sc.N, d, m2, c2, col, op, view.height, view.width)
    gm, gc, gcol, ga = crc.backwards_rasterization(grad_img, m2, c2, col, op, ids, ranges, fT, nc,
                                                   sc.N, view.height, view.width)
    gA, gkj, gmu_sh = crc.backwards_SH(gcol, mu, A, kj, cam)
    gmu, gq, gs = crc.backwards_projection(gm, gc, mu, q, s, R, t, view.fx, view.fy, view.cx,
                                           view.cy)
    a, b, c = c2[:, 0], c2[:, 1], c2[:, 2]
    mid = 0.5 * (a + c)
    radius = mid + torch.sqrt(torch.clamp((0.5 * (a - c)) ** 2 + b * b, min=0.1))
    radii = 3.0 * torch.sqrt(torch.clamp(radius, min=0.0))
    return dict(img=img, ids=ids, ranges=ranges, final_T=fT, n_contrib=nc, radii=radii,
                grads=(gmu + gmu_sh, gq, gs, ga.reshape(-1), gA, gkj), mean2d_grad=gm)


@pytest.mark.parametrize("concurrent", [False, True], ids=["latency", "throughput"])
@pytest.mark.parametrize("case", list(scenes_small()), ids=lambda c: c[0])
def test_fused_render_matches_op_chain(crc, cuda_device, case, concurrent):
    """Both blend variants (GS_RENDER_CONCURRENT selects the throughput one)."""
    from custom_rasterizer_cuda.render import render_backward, render_forward

    _, sc, view = case
    dev = cuda_device
    g = torch.Generator("cpu").manual_seed(11)
    grad_img = torch.rand(view.height, view.width, 3, generator=g).to(dev)
    ref = op_chain(crc, sc, view, dev, grad_img)
    mu, q, s, al, A, kj = (p.to(dev).contiguous() for p in sc.params())
    R, t = view.R.to(dev).contiguous(), view.T.to(dev).contiguous()
    cam = (-torch.matmul(R.T, t)).reshape(3).contiguous()
    op = torch.sigmoid(al).contiguous()
    img, radii, st = render_forward(mu, q, s, op, A, kj, R, t, cam, view.fx, view.fy, view.cx,
                                    view.cy, view.height, view.width, concurrent=concurrent)
    assert st.backward_flags == (2 if concurrent else 0)
    assert torch.equal(img, ref["img"])
    assert torch.equal(st.final_T, ref["final_T"]) and torch.equal(st.n_contrib, ref["n_contrib"])
    assert torch.equal(st.sorted_ids[:st.pairs], ref["ids"])
    assert torch.equal(st.tile_ranges, ref["ranges"])
    assert torch.equal(radii, ref["radii"])
    grads = render_backward(st, grad_img, mu, q, s, A, kj, R, t, cam, view.fx, view.fy, view.cx,
                            view.cy)
    for mine, theirs, what in zip(grads[:6], ref["grads"], ("mu", "q", "s", "opacity", "A", "kj")):
        assert_grad_close(np32(mine), np32(theirs), what)
    assert_grad_close(np32(grads[6]), np32(ref["mean2d_grad"]), "mean2d")

    # accumulate mode adds into the given buffers
    bufs = tuple(torch.ones_like(x) for x in grads[:6])
    render_backward(st, grad_img, mu, q, s, A, kj, R, t, cam, view.fx, view.fy, view.cx, view.cy,
                    want_mean2d_grad=False, out=bufs)
    for acc, fresh, what in zip(bufs, grads[:6], ("mu", "q", "s", "opacity", "A", "kj")):
        assert_grad_close(np32(acc) - 1.0, np32(fresh), what + " (accumulated)")


def test_rasterize_function_attributes(cuda_device):
    """RasterizeFunction keeps the reference's class attributes: last_radii2d after the
    forward, last_mean2d_grad after the backward."""
    from gaussian_splatting.rasterizer.rasterize import RasterizeFunction, rasterize
    from gaussian_splatting.scene.gaussian import gaussian
    from gs3d_b200 import scenes

    sc = scenes.config0(0)
    g = gaussian(sc.N)
    for name, p in zip(("mu", "q", "s", "alpha", "A", "k_j"), sc.params()):
        setattr(g, name, p.to(cuda_device).requires_grad_(True))
    img = rasterize(g, sc.views[0].as_dict(cuda_device))
    assert RasterizeFunction.last_radii2d.shape == (sc.N,)
    assert RasterizeFunction.last_mean2d_grad is None
    img.sum().backward()
    assert RasterizeFunction.last_mean2d_grad.shape == (sc.N, 2)
    assert g.alpha.grad.shape == g.alpha.shape and torch.isfinite(g.alpha.grad).all()


def elongated_scene():
    """Needle-like splats (one axis about 12x the others, random orientations) of a few to a
    few dozen tiles: tilted opacity ellipses whose extent boxes are much larger than they are."""
    from gs3d_b200 import scenes

    g = torch.Generator("cpu").manual_seed(21)
    n = 20_000
    means = torch.rand(n, 3, generator=g) * 4.0 - 2.0
    sc = scenes.Scene("needles20k", *scenes._draw(g, n, means, -4.0, 0.3))
    sc.s[:, 0] += 2.5
    return "needles20k_640x360", sc, scenes.pinhole((0.5, 0.3, 7.0), 640, 360, 500.0)


@pytest.mark.parametrize("case", list(scenes_small()) + [elongated_scene()], ids=lambda c: c[0])
def test_tight_bins_keep_image_and_gradients(crc, cuda_device, case):
    """GS_RENDER_TIGHT_BINS: image, transmittance and radii identical to the reference binning,
    gradients within the atomic-order tolerance, and never more pairs."""
    from custom_rasterizer_cuda.render import render_backward, render_forward

    _, sc, view = case
    dev = cuda_device
    g = torch.Generator("cpu").manual_seed(5)
    grad_img = torch.rand(view.height, view.width, 3, generator=g).to(dev)
    mu, q, s, al, A, kj = (p.to(dev).contiguous() for p in sc.params())
    R, t = view.R.to(dev).contiguous(), view.T.to(dev).contiguous()
    cam = (-torch.matmul(R.T, t)).reshape(3).contiguous()
    op = torch.sigmoid(al).contiguous()
    res = {}
    for tight in (False, True):
        img, radii, st = render_forward(mu, q, s, op, A, kj, R, t, cam, view.fx, view.fy,
                                        view.cx, view.cy, view.height, view.width,
                                        tight_bins=tight)
        grads = render_backward(st, grad_img, mu, q, s, A, kj, R, t, cam, view.fx, view.fy,
                                view.cx, view.cy)
        res[tight] = (img, radii, st, grads)
    (img0, radii0, st0, g0), (img1, radii1, st1, g1) = res[False], res[True]
    assert torch.equal(img0, img1) and torch.equal(st0.final_T, st1.final_T)
    assert torch.equal(radii0, radii1)
    assert st1.pairs <= st0.pairs
    names = ("mu", "q", "s", "opacity", "A", "kj", "mean2d")
    if not case[0].startswith("needles"):
        for a, b, what in zip(g1, g0, names):
            assert_grad_close(np32(a), np32(b), what + " (tight bins)")
        return
    # Near-singular 2D covariances amplify the order of the float atomics in the mean, rotation
    # and log-scale gradients beyond a flat 1e-4 per element (the two binnings' tile lists
    # differ, so their blend CTAs and atomics run in different orders): those are bounded in
    # aggregate (relative L2 1e-3, at most 1% of the elements beyond the 1e-4 band), the rest
    # per element. tests/test_gpu_parity.py compares needle gradients, tight bins included,
    # with the reference's own kernels.
    for a, b, what in zip(g1, g0, names):
        a64, b64 = np32(a).astype(np.float64), np32(b).astype(np.float64)
        if what in ("mu", "q", "s"):
            rel_l2 = np.linalg.norm(a64 - b64) / np.linalg.norm(b64)
            rms = np.sqrt(np.mean(b64 * b64))
            beyond = int((np.abs(a64 - b64) > 1e-4 * (np.abs(b64) + rms)).sum())
            assert rel_l2 <= 1e-3 and beyond <= 0.01 * b64.size, (what, rel_l2, beyond)
        else:
            assert_grad_close(a64, b64, what + " (tight bins)")


def test_pair_buffers_sized_from_the_last_count(cuda_device):
    """A second render of a view gets pair buffers of the first one's count + 12.5% + 4096 (one
    attempt, no re-render); a scene whose worst case (N x tiles) is small gets buffers for that
    worst case and never waits for its count."""
    from custom_rasterizer_cuda.render import render_forward
    from gs3d_b200 import scenes

    def render(sc, view):
        mu, q, s, al, A, kj = (p.to(cuda_device).contiguous() for p in sc.params())
        R, t = view.R.to(cuda_device), view.T.to(cuda_device)
        cam = (-torch.matmul(R.T, t)).reshape(3).contiguous()
        op = torch.sigmoid(al).reshape(-1).contiguous()
        return render_forward(mu, q, s, op, A, kj, R, t, cam, view.fx, view.fy, view.cx,
                              view.cy, view.height, view.width)

    sc = scenes.config2(11, n=50_000)
    view = scenes.pinhole((0.0, 0.0, 8.0), 480, 270, 375.0)
    _, _, st1 = render(sc, view)
    _, _, st2 = render(sc, view)
    m = st1.pairs
    assert st2.capacity == m + m // 8 + 4096 and st2.pairs == m
    sc0 = scenes.config0(0)
    _, _, st0 = render(sc0, sc0.views[0])
    tiles = ((sc0.views[0].width + 15) // 16) * ((sc0.views[0].height + 15) // 16)
    assert st0.capacity == sc0.N * tiles and st0.pairs <= st0.capacity


def test_combined_per_gaussian_backward_over_views(cuda_device):
    """gs_render_backward_blend + gs_render_backward_gaussians (the training step's backward):
    one call over four views gives the same bits as one call per view accumulating in view
    order and as two calls over two views each; and it agrees (atomic-order tolerance) with one
    render_backward per view accumulating into the same buffers, statistics included."""
    from custom_rasterizer_cuda.render import (render_backward, render_backward_blend,
                                               render_backward_views, render_forward)
    from gs3d_b200 import scenes

    dev = cuda_device
    sc = scenes.config2(5, n=60_000)
    eyes = ((0.0, 0.0, 8.0), (6.0, 1.0, 5.0), (-5.0, 3.0, -6.0), (1.0, -7.0, 4.0))
    views = [scenes.pinhole(e, 480, 270, 375.0) for e in eyes]
    mu, q, s, al, A, kj = (p.to(dev).contiguous() for p in sc.params())
    op = torch.sigmoid(al).reshape(-1).contiguous()
    N = sc.N
    g = torch.Generator("cpu").manual_seed(7)
    grads = [torch.rand(v.height, v.width, 3, generator=g).to(dev) for v in views]
    cams, sums, states = [], [], []
    for v, gi in zip(views, grads):
        R, t = v.R.to(dev).contiguous(), v.T.to(dev).contiguous()
        cam = (-torch.matmul(R.T, t)).reshape(3).contiguous()
        _, _, st = render_forward(mu, q, s, op, A, kj, R, t, cam, v.fx, v.fy, v.cx, v.cy,
                                  v.height, v.width, tight_bins=True)
        sums.append(render_backward_blend(st, gi, N))
        cams.append((R, t, cam))
        states.append(st)
    entries = [(ws, R, t, cam, v.fx, v.fy, v.cx, v.cy, v.width / 2.0, v.height / 2.0)
               for ws, (R, t, cam), v in zip(sums, cams, views)]

    def fresh():
        f32 = dict(device=dev, dtype=torch.float32)
        out = (torch.full((N, 3), 7.0, **f32), torch.full((N, 4), 7.0, **f32),
               torch.full((N, 3), 7.0, **f32), torch.full((N,), 7.0, **f32),
               torch.full((N, 3), 7.0, **f32), torch.full((N, 15, 3), 7.0, **f32))
        stats = (torch.zeros(N, **f32), torch.zeros(N, **f32), torch.zeros(N, **f32))
        return out, stats

    out_all, st_all = fresh()
    render_backward_views(entries, mu, q, s, A, kj, out_all, stats=st_all)
    out_one, st_one = fresh()
    for k, e in enumerate(entries):
        render_backward_views([e], mu, q, s, A, kj, out_one, accumulate=k > 0, stats=st_one)
    out_two, st_two = fresh()
    render_backward_views(entries[:2], mu, q, s, A, kj, out_two, stats=st_two)
    render_backward_views(entries[2:], mu, q, s, A, kj, out_two, accumulate=True, stats=st_two)
    for a, b, c in zip(out_all + st_all, out_one + st_one, out_two + st_two):
        assert torch.equal(a, b) and torch.equal(a, c)
    assert int((st_all[1] > 0).sum()) > N // 2  # most Gaussians are seen by some view
    # more entries than one launch takes (GS_MAX_VIEWS_PER_CALL = 16): two launches, same bits
    many = [entries[k % len(entries)] for k in range(18)]
    out_many, st_many = fresh()
    render_backward_views(many, mu, q, s, A, kj, out_many, stats=st_many)
    out_seq, st_seq = fresh()
    for k, e in enumerate(many):
        render_backward_views([e], mu, q, s, A, kj, out_seq, accumulate=k > 0, stats=st_seq)
    for a, b in zip(out_many + st_many, out_seq + st_seq):
        assert torch.equal(a, b)
    # a workspace smaller than one view's sums is refused before any GPU work
    small = (entries[0][0][:1024],) + tuple(entries[0][1:])
    with pytest.raises(RuntimeError, match="smaller than gs_render_backward_workspace_size"):
        render_backward_views([small], mu, q, s, A, kj, fresh()[0])

    # against render_backward per view (its own blend pass: the same sums up to atomic order)
    out_ref, st_ref = fresh()
    for k, (v, gi, st, (R, t, cam)) in enumerate(zip(views, grads, states, cams)):
        render_backward(st, gi, mu, q, s, A, kj, R, t, cam, v.fx, v.fy, v.cx, v.cy,
                        want_mean2d_grad=False, out=out_ref, accumulate=k > 0,
                        stats=(*st_ref, v.width / 2.0, v.height / 2.0))
    names = ("mu", "q", "s", "opacity", "A", "kj", "norm_sum", "count", "norm_max")
    for a, b, what in zip(out_all + st_all, out_ref + st_ref, names):
        assert_grad_close(np32(a), np32(b), what + " (combined over views)")
