"""The drop-in Model facade compiles and links against the reference's own
host code: ChatSession, the tokenizers and ConfigManager from the reference
tree, unmodified, with yalama_b200/host/Model.cpp in place of
src/models/Model.cpp + the LibTorch ModelBase, and the engine library
(yalama_b200/host/Makefile). Running it needs a GPU (tests/test_gpu_facade.py)."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("YLM_REFERENCE_SRC", "/root/reference")
BIN = os.path.join(ROOT, "yalama_b200", "host", "_build", "facade_chat")


def test_facade_builds_against_reference_sources():
    if not os.path.isdir(os.path.join(REF, "src")):
        pytest.skip("the reference sources are not present on this machine")
    from yalama_b200 import build
    build.build()
    r = subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "yalama_b200", "host"), "-j8", f"REF={REF}",
                        f"PYTHON={sys.executable}"], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert os.path.exists(BIN)
    # it starts (all shared libraries resolve) and rejects a missing model
    u = subprocess.run([BIN], capture_output=True, text=True, timeout=60)
    assert u.returncode == 2 and "usage" in u.stderr
