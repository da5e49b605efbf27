"""Shared pytest configuration.

* registers the ``gpu`` marker (tests that need a B200 and the built CUDA library);
* puts the package root (``smooth-attn_b200/``) and the repo root on ``sys.path``
  so ``import smooth_attn`` resolves to this build and ``import oracle`` to the
  CPU checker.
"""

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PKG_ROOT = ROOT / "smooth-attn_b200"
for p in (str(PKG_ROOT), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU and the built libsmooth_attn_b200.so")
