"""Bounded waits on the GPU: every spin-wait of the kernels (bulk-copy and
pipeline mbarriers) gives up after a time limit and records an error instead
of hanging.  tests/cpp/wait_timeout.cu runs the library's own bounded wait on
a barrier that nothing arrives on; the wait must give up after its limit with
the flag set, and the context must still run the sampler afterwards."""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

ROOT = Path(__file__).resolve().parent.parent


def test_bounded_wait_gives_up_and_context_survives(cuda_lib, tmp_path):
    if not torch.cuda.is_available():
        pytest.fail("gpu tests need a CUDA device")
    from verbo_b200 import build

    so = tmp_path / "libwait_timeout.so"
    subprocess.run([build.nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-shared",
                    "-Xcompiler", "-fPIC", f"-I{ROOT / 'verbo_b200' / 'csrc'}", "-o", str(so),
                    str(ROOT / "tests" / "cpp" / "wait_timeout.cu")], check=True, capture_output=True)
    lib = ctypes.CDLL(str(so))
    gave_up, waited, limit = ctypes.c_uint(7), ctypes.c_ulonglong(0), ctypes.c_ulonglong(0)
    rc = lib.run_wait_timeout(ctypes.byref(gave_up), ctypes.byref(waited), ctypes.byref(limit))
    assert rc == 0, f"cudaError {rc}"
    assert gave_up.value == 1
    assert limit.value <= waited.value < 20 * limit.value

    import verbo_b200 as vb

    x = torch.from_numpy(np.arange(64, dtype=np.float32).reshape(2, 32)).cuda()
    ids = vb.sample(x, vb.Sampling(temp=0.0)).cpu().numpy()
    vb.check()
    assert ids.tolist() == [31, 31]
