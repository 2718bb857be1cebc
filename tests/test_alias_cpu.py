"""The opt-in import alias: after gs_voxelizer_b200.install_alias(), the
reference's import lines resolve to this package (no GPU needed; importing
the modules loads libgsvox.so, which needs no device)."""
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_imports_resolve_after_install_alias():
    code = (
        "import gs_voxelizer_b200 as b; b.install_alias()\n"
        "from gs_voxelizer.optim_to_render import optim_to_render\n"
        "from gs_voxelizer.voxelize import voxelize_gaussians\n"
        "from gs_voxelizer.bin_and_sort_gaussians import bin_and_sort_gaussians\n"
        "import gs_voxelizer.cuda as C\n"
        "import gs_voxelizer_b200.voxelize as V\n"
        "assert voxelize_gaussians is V.voxelize_gaussians\n"
        "assert hasattr(C, 'voxelize_backward_per_gaussian')\n"
        "print('ok')\n")
    res = subprocess.run([sys.executable, "-c", code], cwd=ROOT,
                         capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr
    assert res.stdout.strip().endswith("ok")
