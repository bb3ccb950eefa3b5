"""The C consumer program (tests/consumer/consumer_linear.c): linked the way a
cgo caller links popcorn (gcc + lib/libpopcorn.a + -lcudart -lstdc++), it runs
quantize and every matmul family from five host threads on their own streams
(one on the legacy default stream) and checks the results on the host.

CPU: it builds and links against the static archive alone, and every function
of include/popcorn.h it calls comes from the archive. GPU: it runs clean.
"""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _build(tmp_path):
    binary = tmp_path / "consumer_linear"
    r = subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "consumer"), f"BIN={binary}"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return binary


def test_consumer_links_against_the_archive(tmp_path):
    binary = _build(tmp_path)
    syms = subprocess.run(["nm", str(binary)], capture_output=True, text=True, check=True).stdout
    defined = set(re.findall(r" [TW] (popcorn\w+)$", syms, flags=re.M))
    called = set(re.findall(r"\b(popcorn\w+)\(", open(os.path.join(ROOT, "tests", "consumer",
                                                                   "consumer_linear.c")).read()))
    assert called and called <= defined, called - defined
    # no shared popcorn library is involved
    ldd = subprocess.run(["ldd", str(binary)], capture_output=True, text=True).stdout
    assert "popcorn" not in ldd


@pytest.mark.gpu
def test_consumer_runs_on_many_threads_and_streams(tmp_path):
    binary = _build(tmp_path)
    r = subprocess.run([str(binary)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "consumer ok" in r.stdout
