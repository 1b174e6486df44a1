"""The provider/runner translation unit (tests/cpp/gufo_runner_test.cpp,
the shape of the reference's provider.cpp:8-19 and runner.cpp:44-141)
compiles against the Gufo SDK stand-in headers and links against
libomnivoice_b200.so; without arguments it registers its provider into a
Registry and checks what the registry received (no GPU needed)."""
from __future__ import annotations

import subprocess


def test_provider_registers_without_a_gpu(native):
    from omnivoice_b200.build import build_test_programs
    exe = [p for p in build_test_programs() if p.name == "gufo_runner_test"][0]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0 and run.stdout.strip() == "ok", run.stdout + run.stderr
