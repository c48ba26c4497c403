"""The library's JSON reader (csrc/json.h) through n3d_config_load, on the CPU: damaged
config files end in a Json error, never in a crash, and the limits it adds (nesting,
number range) are errors with a message."""

import json
import os
import subprocess
import sys

import pytest

import n3d

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(ROOT, "tests", "config_fuzz_worker.py")


def test_damaged_configs_never_crash(tmp_path, checkpoint_dir):
    r = subprocess.run([sys.executable, WORKER, checkpoint_dir, str(tmp_path), "5", "1500"], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, (r.returncode, r.stderr[-2000:])  # a negative code is the signal that ended it
    ends = json.loads(r.stdout.strip().splitlines()[-1])
    assert set(ends) <= {"ok", "Json"}, ends
    assert ends["Json"] > 1000


def _load_with(tmp_path, checkpoint_dir, text):
    d = tmp_path / "c"
    d.mkdir(exist_ok=True)
    (d / "config.json").write_text(text)
    with open(os.path.join(checkpoint_dir, "processor_config.json")) as f:
        (d / "processor_config.json").write_text(f.read())
    return n3d.Config.load(str(d))


@pytest.mark.parametrize("text,msg", [("[" * 129 + "]" * 129, "nesting too deep"),
                                      ('{"a": ' * 200 + "1" + "}" * 200, "nesting too deep"),
                                      ('{"a": 1e99999}', "number out of range"),
                                      ('{"a": -}', "bad value"),
                                      ('{"a": 1} x', "trailing characters")])
def test_parser_limits_are_errors(tmp_path, checkpoint_dir, text, msg):
    with pytest.raises(n3d.DiarizationError) as e:
        _load_with(tmp_path, checkpoint_dir, text)
    assert e.value.kind == "Json" and msg in str(e.value)


def test_python_written_config_and_nesting_at_the_limit(tmp_path, checkpoint_dir):
    """A config rewritten by Python's json module, with a shortest-round-trip float
    such as 0.30000000000000004, loads; nesting exactly at the limit is accepted."""
    with open(os.path.join(checkpoint_dir, "config.json")) as f:
        cfg = json.load(f)
    cfg["streaming_config"]["prediction_score_threshold"] = 0.1 + 0.2  # 0.30000000000000004
    c = _load_with(tmp_path, checkpoint_dir, json.dumps(cfg, indent=None))
    assert c.mode_params("ultra_low_latency")["latency_ms"] == 320
    nested = "[" * 128 + "]" * 128  # at the limit: parses (then fails on content)
    with pytest.raises(n3d.DiarizationError) as e:
        _load_with(tmp_path, checkpoint_dir, nested)
    assert "nesting" not in str(e.value)


def _canonical(v):
    if isinstance(v, bool) or v is None:
        return json.dumps(v)
    if isinstance(v, (int, float)):
        return "%.17g" % float(v)
    if isinstance(v, str):
        return '"' + v + '"'
    if isinstance(v, list):
        return "[" + ",".join(_canonical(x) for x in v) + "]"
    return "{" + ",".join('"%s":%s' % (k, _canonical(x)) for k, x in v.items()) + "}"


@pytest.fixture(scope="module")
def json_dump(tmp_path_factory):
    exe = tmp_path_factory.mktemp("jd") / "json_dump"
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-o", str(exe), os.path.join(ROOT, "tests", "json_dump.cpp")],
                       capture_output=True, text=True)
    if r.returncode:
        pytest.skip("no host C++ compiler: " + r.stderr[-300:])
    return str(exe)


def test_reader_matches_python_on_the_checkpoint_files(json_dump, checkpoint_dir):
    """The same reader parses the checkpoint's two configs and its safetensors header
    (417 entries of dtype, shape and byte offsets) exactly as Python's json does."""
    for name in ("config.json", "processor_config.json"):
        path = os.path.join(checkpoint_dir, name)
        with open(path) as f:
            want = _canonical(json.load(f))
        got = subprocess.run([json_dump, path], capture_output=True, text=True).stdout.strip()
        assert got == want, name
    path = os.path.join(checkpoint_dir, "model.safetensors")
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        header = json.loads(f.read(n))
    got = subprocess.run([json_dump, "--safetensors", path], capture_output=True, text=True).stdout.strip()
    assert got == _canonical(header)
    assert len(header) >= 417
