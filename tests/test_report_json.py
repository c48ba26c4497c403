"""The `diarize` report's JSON text (csrc/report_json.h) on the CPU, through a helper
built from the same header: numbers as serde_json prints an f64 (ryu's shortest
round-trip digits and layout) and strings with serde_json's escapes, so the report
reads as the reference's does (src/bin/diarize.rs writes it with serde_json)."""

import json
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def helper(tmp_path_factory):
    exe = tmp_path_factory.mktemp("jn") / "json_number"
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-o", str(exe), os.path.join(ROOT, "tests", "json_number.cpp")],
                       capture_output=True, text=True)
    if r.returncode:
        pytest.skip("no host C++ compiler: " + r.stderr[-300:])
    return str(exe)


def _numbers(helper, values):
    r = subprocess.run([helper] + [repr(float(v)) for v in values], capture_output=True, text=True, check=True)
    return r.stdout.splitlines()


KNOWN = [  # (value, serde_json text); a list, since 0.0 and -0.0 are equal dict keys
    (60.0, "60.0"), (0.5, "0.5"), (100.0, "100.0"), (12.34, "12.34"), (-2.5, "-2.5"), (0.0, "0.0"),
    (-0.0, "-0.0"), (123456.789, "123456.789"), (0.1 + 0.2, "0.30000000000000004"),
    (1e15, "1000000000000000.0"), (9999999999999998.0, "9999999999999998.0"), (1e16, "1e16"),
    (1.5e16, "1.5e16"), (1.234e33, "1.234e33"), (0.0001, "0.0001"), (1e-5, "0.00001"), (1.25e-5, "0.0000125"),
    (1e-6, "1e-6"), (1.5e-7, "1.5e-7"), (1e300, "1e300"), (5e-324, "5e-324"),
    (1.7976931348623157e308, "1.7976931348623157e308"), (float("nan"), "null"), (float("inf"), "null"),
]


def test_known_serde_json_forms(helper):
    assert _numbers(helper, [v for v, _ in KNOWN]) == [t for _, t in KNOWN]


def _sig_digits(text):
    mant = text.lstrip("-").split("e")[0].replace(".", "").lstrip("0").rstrip("0")
    return len(mant) or 1


def test_round_trip_with_shortest_digits(helper):
    rng = np.random.default_rng(3)
    values = list(rng.standard_normal(300) * 10.0 ** rng.integers(-12, 20, 300)) + \
        [round(float(x), 3) for x in rng.random(100) * 4000] + [float(2 ** k) for k in range(-30, 60, 7)]
    out = _numbers(helper, values)
    for v, t in zip(values, out):
        assert json.loads(t) == v, (v, t)
        assert "+" not in t and "E" not in t
        assert _sig_digits(t) == _sig_digits(repr(float(v)).replace("e+", "e")), (v, t)


def test_string_escapes(helper):
    s = "clip \x00\x01\b\t\n\x0b\f\r\x1f \"q\" back\\slash /é.wav"
    r = subprocess.run([helper, "--quote"], input=s.encode(), capture_output=True, check=True)
    assert r.stdout.decode().rstrip("\n") == json.dumps(s, ensure_ascii=False)
