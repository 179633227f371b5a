"""The C++20 adapter (B200MatvecAccelerator : DeepseekV4MatvecAccelerator): host-side refusal,
eviction and Governor rules over a fake device API (CPU), and the real library on a B200."""

import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
CPP = ROOT / "tests" / "cpp"


def _binary(name: str) -> Path:
    exe = CPP / name
    if not exe.exists():
        from vastloom_b200.build import reference_root

        ref = reference_root() / "include"
        if not ref.exists():
            pytest.skip(f"{name} is not built and the reference headers are absent")
        subprocess.run(["make", "-C", str(ROOT / "vastloom_b200" / "host")], check=True, capture_output=True)
        subprocess.run(["make", "-C", str(CPP), name], check=True, capture_output=True)
    return exe


def test_accelerator_host_rules():
    r = subprocess.run([str(_binary("test_accelerator"))], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "passed" in r.stdout


@pytest.mark.gpu
def test_accelerator_on_b200():
    r = subprocess.run([str(_binary("accel_gpu_check"))], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
