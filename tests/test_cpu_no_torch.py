"""The package runs without the framework: device memory, streams, events and NCCL all come
from ``libtgb200.so``; torch is needed only by a caller that bootstraps ranks with
``torch.distributed``."""

from __future__ import annotations

import subprocess
import sys


def test_importing_the_package_does_not_import_torch():
    code = ("import sys, tensorgrad_b200, tensorgrad_b200.nn, tensorgrad_b200.optim, "
            "tensorgrad_b200.func, tensorgrad_b200.distributed as d; "
            "assert d.world_size() == 1 and d.rank() == 0; "
            "print('torch' in sys.modules)")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=300, env={"PATH": "/usr/bin:/bin", "WORLD_SIZE": "1"})
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "False"
