"""The torch.backends entry point (reference pyproject.toml:18-19,
_autoload.py:1-2) loads the package at `import torch` without an explicit
import, and TORCH_DEVICE_BACKEND_AUTOLOAD=0 turns that off. Run in child
processes against a dist-info directory equivalent to what `pip install`
writes for this repository's pyproject.toml."""
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "mps-fp8-for-torch-and-comfyui-python-package_b200")


def _site(tmp_path):
    di = tmp_path / "fp4_fp8_for_torch_b200-1.0.0.dist-info"
    di.mkdir()
    (di / "METADATA").write_text("Metadata-Version: 2.1\nName: fp4-fp8-for-torch-b200\nVersion: 1.0.0\n")
    (di / "entry_points.txt").write_text(
        "[torch.backends]\nfp4_fp8_for_torch_mps = fp4_fp8_for_torch_mps._autoload:_autoload\n")
    return str(tmp_path)


def _run(tmp_path, extra_env=None):
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([_site(tmp_path), PKG_ROOT])
    env.update(extra_env or {})
    code = ("import sys, torch; "
            "print('loaded' if 'fp4_fp8_for_torch_mps' in sys.modules else 'absent', "
            "hasattr(torch.ops.fp8_mps, 'encode'))")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout.split()


def test_entry_point_autoloads_plugin(tmp_path):
    assert _run(tmp_path) == ["loaded", "True"]


def test_autoload_can_be_disabled(tmp_path):
    assert _run(tmp_path, {"TORCH_DEVICE_BACKEND_AUTOLOAD": "0"})[0] == "absent"
