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


def test_random_count_values_never_crash_or_hang(tmp_path, checkpoint_dir):
    """Well-formed configs with random count values (zero, negative, fractional,
    strings, null, huge): each load succeeds or is a Json error, and planning every
    loaded one in all four modes ends (a division by zero or an endless schedule loop
    would crash or time out the child)."""
    r = subprocess.run([sys.executable, WORKER, checkpoint_dir, str(tmp_path), "9", "1500", "values"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (r.returncode, r.stderr[-2000:])
    ends = json.loads(r.stdout.strip().splitlines()[-1])
    assert set(ends) <= {"ok", "Json", "plan:UnsupportedAudio"}, ends
    assert ends["ok"] > 100 and ends["Json"] > 100


def _edited(checkpoint_dir, tmp_path, where, key, value):
    with open(os.path.join(checkpoint_dir, "config.json")) as f:
        cfg = json.load(f)
    with open(os.path.join(checkpoint_dir, "processor_config.json")) as f:
        proc = json.load(f)
    doc = proc if where.startswith("proc") else cfg
    sec = where.split(":")[1] if ":" in where else None
    (doc[sec] if sec else doc)[key] = value
    d = tmp_path / "e"
    d.mkdir(exist_ok=True)
    (d / "config.json").write_text(json.dumps(cfg))
    (d / "processor_config.json").write_text(json.dumps(proc))
    return str(d)


@pytest.mark.parametrize("where,key,value,ok", [
    ("cfg", "chunk_length", 0, False),                      # the offline loop steps by it
    ("proc:feature_extractor", "hop_length", 0, False),     # frame_count divides by it
    ("cfg:streaming_config", "num_speakers", 0, False),     # the cache budget divides by it
    ("cfg:streaming_config", "speaker_cache_length", 7, False),  # budget 7 / 8 - 1 < 0
    ("cfg:streaming_config", "speaker_cache_length", 8, True),   # budget 8 / 8 - 1 = 0
    ("cfg", "chunk_right_context", 0, True),                # zero look-ahead is allowed
    ("cfg:streaming_config", "fifo_length", 0, True),
    ("cfg", "fifo_length", -1, False),
    ("cfg", "chunk_length", 2.5, False),
    ("cfg", "chunk_length", "340", False),
    ("cfg", "chunk_length", None, False),
    ("cfg", "chunk_length", 340.0, True),                   # an integral float is still a count
    ("proc:streaming_modes", "ultra_low_latency", [0, 1], False),
    ("proc:streaming_modes", "ultra_low_latency", [3, 0], True),
    ("cfg:streaming_config", "prediction_score_threshold", "0.25", False),
])
def test_count_fields_are_validated(tmp_path, checkpoint_dir, where, key, value, ok):
    d = _edited(checkpoint_dir, tmp_path, where, key, value)
    if ok:
        n3d.Config.load(d).close()
        return
    with pytest.raises(n3d.DiarizationError) as e:
        n3d.Config.load(d)
    assert e.value.kind == "Json"
