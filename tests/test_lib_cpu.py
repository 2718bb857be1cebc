"""The C-ABI library loads without a GPU, exports every function that
include/gsvox.h declares, and rejects bad arguments before touching the
device. No kernel is launched here."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    text = (ROOT / "include" / "gsvox.h").read_text()
    return re.findall(r"GSV_API\s+[\w\s\*]+?\b(gsv_\w+)\s*\(", text)


def test_header_declares_the_reference_surface():
    names = set(declared_functions())
    for fn in ("gsv_optim_to_render_forward", "gsv_optim_to_render_backward",
               "gsv_bin_and_sort_gaussians", "gsv_voxelize_forward",
               "gsv_voxelize_backward", "gsv_voxelize_backward_per_gaussian"):
        assert fn in names


def test_library_exports_every_declared_symbol():
    from gs_voxelizer_b200 import _lib
    names = declared_functions()
    assert len(names) >= 18
    for n in names:
        assert hasattr(_lib.lib, n), n
        assert n in _lib.SIGNATURES, n


def test_version_and_launch_counter():
    from gs_voxelizer_b200 import _lib
    assert _lib.version() == "0.1.0"
    assert _lib.lib.gsv_launch_count() == 0  # nothing launched on CPU


def test_workspace_queries_are_host_only():
    from gs_voxelizer_b200._lib import i3, lib
    v = i3((256, 256, 256))
    b = lib.gsv_bin_and_sort_workspace_bytes(100000, 1_500_000, v)
    assert b >= 4 * 1_500_000 + 4 * 32768
    w = lib.gsv_voxelize_workspace_bytes(100000, 1, 1_500_000, v)
    assert w >= 48 * 100000
    assert lib.gsv_voxelize_workspace_bytes(10, 5, 10, v) == 0  # C > 4
    assert lib.gsv_bin_and_sort_slab_workspace_bytes(10, 10, v, 5, 40) == 0


def test_argument_errors():
    from gs_voxelizer_b200._lib import GsvError, check, f3, i3, lib
    v = i3((16, 16, 16))
    st = lib.gsv_voxelize_forward(v, 5, 10, 10, None, None, None, None, None,
                                  None, None, 0, None)
    assert st == 2
    with pytest.raises(GsvError, match="UNSUPPORTED_CHANNELS"):
        check(st)
    st = lib.gsv_optim_to_render_forward(10, 1, None, None, None, None,
                                         i3((0, 4, 4)), f3((1, 1, 1)),
                                         f3((0, 0, 0)), None, None, None, None,
                                         None, None)
    assert st == 1
    assert b"positive" in lib.gsv_last_error()
    st = lib.gsv_bin_and_sort_gaussians(10, 100, None, None, None, v, None,
                                        None, None, 0, None)
    assert st == 1
    # workspace too small is reported, not written past
    ws = ctypes.create_string_buffer(16)
    dummy = ctypes.c_void_p(1)
    st = lib.gsv_bin_and_sort_gaussians(10, 100, dummy, dummy, None, v, dummy,
                                        dummy, ctypes.cast(ws, ctypes.c_void_p),
                                        16, None)
    assert st == 3
    st = lib.gsv_bin_and_sort_gaussians_slab(10, 100, dummy, dummy, v, 1, 9,
                                             dummy, dummy, None, 0, None)
    assert st == 1 and b"tile z range" in lib.gsv_last_error()
    assert lib.gsv_profile_kernel(7, None, None) == 1


def test_halo_argument_errors():
    """The halo entry points validate world / rank / sizes / workspace
    before any CUDA call."""
    from gs_voxelizer_b200._lib import lib
    I32, I64 = ctypes.c_int32, ctypes.c_int64
    tz = (I32 * 4)(0, 2, 2, 4)
    off = (I64 * 2)(0, 0)
    slots = (I32 * 2)(0, 5)
    dummy = ctypes.c_void_p(1)
    assert lib.gsv_halo_workspace_bytes(10, 0) == 0
    assert lib.gsv_halo_workspace_bytes(10, 65) == 0
    ws_need = lib.gsv_halo_workspace_bytes(10, 2)
    assert ws_need > 0
    # rank outside the world
    st = lib.gsv_halo_pack(10, 1, dummy, dummy, dummy, dummy, dummy, 2, 2, tz,
                           off, slots, dummy, dummy, None, dummy, ws_need, None)
    assert st == 1 and b"peer description" in lib.gsv_last_error()
    # five channels
    st = lib.gsv_halo_pack(10, 5, dummy, dummy, dummy, dummy, dummy, 2, 0, tz,
                           off, slots, dummy, dummy, None, dummy, ws_need, None)
    assert st == 1
    # workspace too small
    st = lib.gsv_halo_pack(10, 1, dummy, dummy, dummy, dummy, dummy, 2, 0, tz,
                           off, slots, dummy, dummy, None, dummy, ws_need - 1,
                           None)
    assert st == 3
    # negative slots
    bad = (I32 * 2)(0, -1)
    st = lib.gsv_halo_unpack(0, 1, 2, 0, off, bad, dummy, dummy, dummy, dummy,
                             dummy, dummy, dummy, None)
    assert st == 1
    # null receive buffer with slots to unpack
    st = lib.gsv_halo_unpack(0, 1, 2, 0, off, slots, None, dummy, dummy, dummy,
                             dummy, dummy, dummy, None)
    assert st == 1 and b"null" in lib.gsv_last_error()
    st = lib.gsv_halo_accumulate(3, 1, 2, 0, off, dummy, None, dummy, dummy,
                                 dummy, dummy, dummy, dummy, None)
    assert st == 1


def test_python_api_rejects_cpu_tensors_like_the_reference():
    from gs_voxelizer_b200 import cuda as C
    from gs_voxelizer_b200.optim_to_render import optim_to_render
    x = torch.zeros(4, 3)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        C.optim_to_render_forward(4, x, x, torch.zeros(4, 4), torch.zeros(4, 1),
                                  (8, 8, 8), (1, 1, 1), (0.5, 0.5, 0.5))
    with pytest.raises(ValueError, match="Invalid shape for pos3d"):
        optim_to_render(torch.zeros(4, 2), x, torch.zeros(4, 4), torch.zeros(4, 1),
                        (8, 8, 8), (1, 1, 1), (0.5, 0.5, 0.5))
    with pytest.raises(RuntimeError, match="MAX_CHANNELS"):
        C._channels(torch.zeros(4, 5))
    assert C.num_tiles((256, 256, 256)) == 32 ** 3
    assert C.num_tiles((100, 150, 80)) == 13 * 19 * 10


def test_slab_bounds_partition():
    from gs_voxelizer_b200.slab import slab_bounds, tile_layers
    for Z in (8, 100, 256, 2048, 2049):
        for w in (1, 2, 3, 4, 8):
            Tz = tile_layers((Z, 8, 8))
            spans = [slab_bounds((Z, 8, 8), w, r) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == Tz
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("channels,max_n", [(1, 349_525), (2, 349_525),
                                            (3, 262_144), (4, 262_144)])
def test_noalloc_limit_is_exact(channels, max_n):
    """gsv_voxelize_forward_noalloc accepts exactly max_n Gaussians (16 MiB
    of 48- or 64-byte records) and rejects max_n + 1. With no intersections
    and a null output the call stops at the output check, after the size
    check, so nothing reaches the device."""
    from gs_voxelizer_b200._lib import i3, lib
    fn = lib.gsv_voxelize_forward_noalloc
    st = fn(i3((16, 16, 16)), channels, max_n, 0, None, None, None, None, None,
            None, None)
    assert st == 1 and "out_vol is null" in lib.gsv_last_error().decode()
    st = fn(i3((16, 16, 16)), channels, max_n + 1, 0, None, None, None, None,
            None, None, None)
    assert st == 3 and "16 MiB scratch" in lib.gsv_last_error().decode()
