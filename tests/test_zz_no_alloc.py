"""gsv_voxelize_forward_noalloc, the forward voxelization for callers that
cannot allocate device memory (their GPU memory belongs to another
allocator, or they only receive finished input/output buffers through a
foreign-function interface): called through the C ABI, it must give the
same volume as gsv_voxelize_forward (the workspace-taking entry point) on
two calls in a row, the second on smaller inputs so that records left in the
shared scratch by the first call would show up if they were read. Collected
last (file name) so that a failure here stops a -x run only after every other
test has run. Volume tolerance as in the other parity tests:
|noalloc - forward| <= 1e-5 * |forward| + 1e-6."""
import numpy as np
import pytest
import torch

from tests import _cases as K

pytestmark = pytest.mark.gpu


def _inputs(cfg):
    from gs_voxelizer_b200 import cuda as C
    pos, scale, quat, inten = (torch.from_numpy(a).cuda() for a in K.inputs(cfg))
    pr, cq, tmin, tmax, nt = C.optim_to_render_forward(
        cfg.n, pos, scale, quat, inten, cfg.vol, cfg.world, cfg.center)
    cum = torch.cumsum(nt, 0, dtype=torch.int32)
    n_isect = int(cum[-1].item())
    ids, bins = C.bin_and_sort_gaussians(cfg.n, n_isect, tmin, tmax, cum, cfg.vol)
    return pr, cq, inten, ids, bins


def _noalloc(cfg, pr, cq, inten, ids, bins):
    from gs_voxelizer_b200._lib import check, i3, lib
    C = inten.shape[1]
    out = torch.full((*cfg.vol, C), float("nan"), device="cuda")
    check(lib.gsv_voxelize_forward_noalloc(
        i3(cfg.vol), C, cfg.n, ids.numel(), ids.data_ptr(), bins.data_ptr(),
        pr.data_ptr(), cq.data_ptr(), inten.data_ptr(), out.data_ptr(),
        torch.cuda.current_stream().cuda_stream))
    return out


def test_noalloc_forward_matches_workspace_forward_twice():
    from gs_voxelizer_b200 import cuda as C
    cases = [
        K.small_config(vol=(48, 40, 56), n=3000, seed=70, channels=1,
                       scale=(0.005, 0.05)),
        K.small_config(vol=(33, 29, 41), n=1200, seed=71, channels=3,
                       scale=(0.005, 0.06)),
    ]
    for cfg in cases:
        pr, cq, inten, ids, bins = _inputs(cfg)
        got = _noalloc(cfg, pr, cq, inten, ids, bins)
        want = C.voxelize_forward(cfg.vol, ids, bins, pr, cq, inten)
        torch.cuda.synchronize()
        g = got.cpu().numpy().astype(np.float64)
        w = want.cpu().numpy().astype(np.float64)
        assert np.isfinite(g).all()
        assert w.max() > 0.1
        assert (np.abs(g - w) <= 1e-5 * np.abs(w) + 1e-6).all()


def test_noalloc_rejects_inputs_beyond_its_scratch():
    from gs_voxelizer_b200._lib import GsvError, check, i3, lib
    st = lib.gsv_voxelize_forward_noalloc(i3((16, 16, 16)), 1, 400_000, 10,
                                          None, None, None, None, None, None,
                                          None)
    assert st == 3
    with pytest.raises(GsvError, match="16 MiB scratch"):
        check(st)
