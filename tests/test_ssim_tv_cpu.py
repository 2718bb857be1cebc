"""CPU checks of the 3D SSIM and TV oracles (oracle/gsv_oracle.c), which the
GPU tests use as the checker: the value against an independent numpy
restatement (separable window by numpy convolution, float64) and the
analytic gradients against central finite differences. Neither loss is
part of the reference's sources (its tests call the external fused_ssim3d;
the 3D TV package is named beside it), so these checks, not golden
vectors, pin the oracle: parity of these two losses is unpinned."""
import numpy as np
import pytest

from oracle import oracle as O


def _blur_np(v, w):
    """Separable blur with zero padding: each axis padded by the window
    radius, then a 'valid' convolution (the window is symmetric)."""
    r = len(w) // 2
    out = v
    for axis in range(3):
        out = np.apply_along_axis(
            lambda row: np.convolve(np.pad(row, r), w, mode="valid"), axis, out)
    return out


def ssim_np(a, b, c1=0.01 ** 2, c2=0.03 ** 2):
    a, b = a.astype(np.float64), b.astype(np.float64)
    w = O.ssim_window()
    mx, my = _blur_np(a, w), _blur_np(b, w)
    sxx = _blur_np(a * a, w) - mx * mx
    syy = _blur_np(b * b, w) - my * my
    sxy = _blur_np(a * b, w) - mx * my
    s = ((2 * mx * my + c1) * (2 * sxy + c2)) / ((mx * mx + my * my + c1) * (sxx + syy + c2))
    return s.mean()


def tv_np(x, iso=True, eps=1e-8):
    x = x.astype(np.float64)
    d = [np.zeros_like(x) for _ in range(3)]
    d[0][:, :, :-1] = x[:, :, 1:] - x[:, :, :-1]
    d[1][:, :-1, :] = x[:, 1:, :] - x[:, :-1, :]
    d[2][:-1, :, :] = x[1:, :, :] - x[:-1, :, :]
    if iso:
        return np.sqrt(d[0] ** 2 + d[1] ** 2 + d[2] ** 2 + eps).mean()
    return (np.abs(d[0]) + np.abs(d[1]) + np.abs(d[2])).mean()


@pytest.mark.parametrize("shape", [(7, 9, 8), (12, 5, 17), (3, 3, 3)])
def test_ssim_oracle_value_and_gradient(shape):
    rng = np.random.default_rng(sum(shape))
    a = rng.random(shape).astype(np.float32)
    b = np.clip(a + 0.2 * rng.standard_normal(shape), 0, 1).astype(np.float32)
    v, g = O.ssim3d(a, b)
    assert v == pytest.approx(ssim_np(a, b), rel=1e-9, abs=1e-12)
    for idx in [(0, 0, 0), tuple(s // 2 for s in shape), tuple(s - 1 for s in shape)]:
        e = 1e-3
        ap, am = a.copy(), a.copy()
        ap[idx] += e
        am[idx] -= e
        fd = (ssim_np(ap, b) - ssim_np(am, b)) / (2 * e)
        assert g[idx] == pytest.approx(fd, rel=2e-3, abs=1e-7)


def test_ssim_oracle_identical_volumes_is_one():
    a = np.random.default_rng(1).random((6, 7, 8)).astype(np.float32)
    v, g = O.ssim3d(a, a)
    assert v == pytest.approx(1.0, abs=1e-12)
    assert np.abs(g).max() < 1e-6  # a maximum of SSIM


def test_ssim_oracle_channels_are_independent():
    rng = np.random.default_rng(2)
    a = rng.random((2, 6, 5, 7)).astype(np.float32)
    b = rng.random((2, 6, 5, 7)).astype(np.float32)
    v, g = O.ssim3d(a, b)
    v0, g0 = O.ssim3d(a[0], b[0])
    v1, g1 = O.ssim3d(a[1], b[1])
    assert v == pytest.approx((v0 + v1) / 2, rel=1e-12)
    np.testing.assert_allclose(g[0], g0 / 2, rtol=1e-6)
    np.testing.assert_allclose(g[1], g1 / 2, rtol=1e-6)


@pytest.mark.parametrize("iso", [True, False])
def test_tv_oracle_value_and_gradient(iso):
    rng = np.random.default_rng(3)
    x = rng.random((6, 7, 9)).astype(np.float32)
    v, g = O.tv3d(x, isotropic=iso)
    assert v == pytest.approx(tv_np(x, iso), rel=1e-10)
    for idx in [(0, 0, 0), (3, 3, 4), (5, 6, 8)]:
        e = 1e-4
        xp, xm = x.copy(), x.copy()
        xp[idx] += e
        xm[idx] -= e
        fd = (tv_np(xp, iso) - tv_np(xm, iso)) / (2 * e)
        assert g[idx] == pytest.approx(fd, rel=2e-3, abs=1e-6)
