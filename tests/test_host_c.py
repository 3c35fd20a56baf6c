"""The C host of the decode step (styx_b200/host/generate_moe.c) builds
against the public headers and links against the library with warnings as
errors; run without arguments it prints its usage.  Its GPU run is in
tests/test_gpu_gguf.py."""
import os
import subprocess

import pytest

from tests.host_c import LIBDIR, build


def test_c_host_builds_and_links(tmp_path):
    if not os.path.exists(os.path.join(LIBDIR, "libstyx_moe.so")):
        pytest.skip("library not built")
    exe = build(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True)
    assert r.returncode == 2 and "usage:" in r.stderr
