"""bench.py's host-side pieces that run without a GPU."""
import importlib.util
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_loads_workloads_without_the_library():
    """The reference arm takes the seeded model shapes from
    memboost_b200/workloads.py loaded by path; the package (and with it
    libmemboost_b200.so) must stay unloaded."""
    code = (
        "import importlib.util, sys\n"
        f"spec = importlib.util.spec_from_file_location('bench_under_test', {os.path.join(ROOT, 'bench.py')!r})\n"
        "b = importlib.util.module_from_spec(spec)\n"
        "sys.modules['bench_under_test'] = b\n"
        "spec.loader.exec_module(b)\n"
        "wl = b.load_workloads()\n"
        "shapes = b.model_shapes(32, wl)\n"
        "assert len(shapes) == 224 and shapes[4][1:3] == (11008, 4096), shapes[:5]\n"
        "assert not any(m.startswith('memboost_b200') for m in sys.modules), 'package loaded'\n"
        "print('ok')\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd="/tmp",
                       timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]
