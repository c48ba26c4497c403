"""The library's checkpoint reader (csrc/safetensors.h) on the CPU, through a small
helper compiled against the same header (tests/st_dump.cpp): it reads a checkpoint as
Python does, and damaged files end in an error with the right status, never in a read
outside the file or a crash."""

import json
import os
import random
import struct
import subprocess

import numpy as np
import pytest

import synth
from conftest import tiny_config

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SAFETENSORS, DTYPE = 3, 4  # n3d_status codes


@pytest.fixture(scope="module")
def st_dump(tmp_path_factory):
    exe = tmp_path_factory.mktemp("st") / "st_dump"
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-I/usr/local/cuda/include", "-o", str(exe),
                        os.path.join(ROOT, "tests", "st_dump.cpp")], capture_output=True, text=True)
    if r.returncode:
        pytest.skip("cannot build the helper: " + r.stderr[-300:])
    return str(exe)


def _read(st_dump, path):
    r = subprocess.run([st_dump, str(path)], capture_output=True, text=True, timeout=60)
    assert r.returncode in (0, 1), (r.returncode, r.stderr)  # anything else is a crash
    return r.returncode, r.stdout


def test_reader_matches_python(st_dump, tmp_path):
    d = synth.write_checkpoint(str(tmp_path / "ck"), seed=0, cfg=tiny_config())
    path = os.path.join(d, "model.safetensors")
    rc, out = _read(st_dump, path)
    assert rc == 0
    got = {}
    for line in out.splitlines():
        name, shape, total = line.split(" ")
        got[name] = (json.loads(shape), float(total))
    want = synth.load_safetensors(path)
    assert sorted(got) == sorted(want)
    for name, arr in want.items():
        seq = float(np.add.accumulate(arr.reshape(-1).astype(np.float64))[-1]) if arr.size else 0.0
        assert got[name] == (list(arr.shape), seq), name


def _file(header, body=b"", hlen=None):
    h = json.dumps(header).encode() if not isinstance(header, bytes) else header
    return struct.pack("<Q", len(h) if hlen is None else hlen) + h + body


BODY = np.arange(12, dtype="<f4").tobytes()  # 48 bytes
OK = {"a": {"dtype": "F32", "shape": [3, 4], "data_offsets": [0, 48]}}


def _entry(**kw):
    e = dict(OK["a"])
    e.update(kw)
    return {"a": e}


CASES = {
    "short": (b"\x01\x02", SAFETENSORS, "file too short"),
    "hlen_huge": (_file(OK, BODY, hlen=2**64 - 1), SAFETENSORS, "header out of range"),
    "hlen_past_end": (_file(OK, BODY, hlen=10**6), SAFETENSORS, "header out of range"),
    "not_json": (_file(b'{"a": {', BODY), SAFETENSORS, "safetensors error"),
    "not_object": (_file([1, 2], BODY), SAFETENSORS, "not an object"),
    "entry_not_object": (_file({"a": 5}, BODY), SAFETENSORS, "bad entry a"),
    "no_dtype": (_file({"a": {"shape": [3, 4], "data_offsets": [0, 48]}}, BODY), SAFETENSORS, "bad entry a"),
    "dtype_f16": (_file(_entry(dtype="F16"), BODY), DTYPE, "dtype F16"),
    "dtype_number": (_file(_entry(dtype=3), BODY), SAFETENSORS, "bad entry a"),
    "offsets_one": (_file(_entry(data_offsets=[0]), BODY), SAFETENSORS, "bad entry a"),
    "offsets_past_end": (_file(_entry(data_offsets=[0, 52]), BODY), SAFETENSORS, "bad data offsets"),
    "offsets_reversed": (_file(_entry(data_offsets=[48, 0]), BODY), SAFETENSORS, "bad data offsets"),
    "offsets_negative": (_file(_entry(data_offsets=[-4, 44]), BODY), SAFETENSORS, "bad data offsets"),
    "offsets_fraction": (_file(_entry(data_offsets=[0, 47.5]), BODY), SAFETENSORS, "bad data offsets"),
    "offsets_strings": (_file(_entry(data_offsets=["0", "48"]), BODY), SAFETENSORS, "bad data offsets"),
    "shape_negative": (_file(_entry(shape=[-3, -4]), BODY), SAFETENSORS, "bad shape"),
    "shape_mismatch": (_file(_entry(shape=[3, 5]), BODY), SAFETENSORS, "bad data offsets"),
    "shape_overflow": (_file(_entry(shape=[40] * 13), BODY), SAFETENSORS, "bad"),  # 40^13 > 2^64
    "shape_string": (_file(_entry(shape=["3", 4]), BODY), SAFETENSORS, "bad shape"),
    "misaligned": (_file({"a": {"dtype": "F32", "shape": [11], "data_offsets": [2, 46]}}, BODY), SAFETENSORS,
                   "misaligned"),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_damaged_file_is_an_error(st_dump, tmp_path, name):
    data, status, msg = CASES[name]
    p = tmp_path / "m.safetensors"
    p.write_bytes(data)
    rc, out = _read(st_dump, p)
    assert rc == 1 and out.startswith(f"error {status} ") and msg in out, out


def test_empty_and_metadata_entries_read(st_dump, tmp_path):
    hdr = {"__metadata__": {"format": "pt"}, "z": {"dtype": "F32", "shape": [0, 7], "data_offsets": [0, 0]},
           "a": {"dtype": "F32", "shape": [3, 4], "data_offsets": [0, 48]}}
    p = tmp_path / "m.safetensors"
    h = json.dumps(hdr).encode()
    h += b" " * ((8 - (8 + len(h)) % 8) % 8)  # keep the tensor bytes 4-byte aligned
    p.write_bytes(struct.pack("<Q", len(h)) + h + BODY)
    rc, out = _read(st_dump, p)
    assert rc == 0 and out.splitlines() == ["a [3,4] 66", "z [0,7] 0"], out


def test_random_header_damage_never_crashes(st_dump, tmp_path):
    """Random edits of a real header's bytes (digits, brackets, quotes, signs) and
    random truncations: every read ends in success or a reported error."""
    src = synth.write_checkpoint(str(tmp_path / "ck"), seed=1, cfg=tiny_config())
    with open(os.path.join(src, "model.safetensors"), "rb") as f:
        raw = f.read()
    (hlen,) = struct.unpack("<Q", raw[:8])
    header, body = bytearray(raw[8:8 + hlen]), raw[8 + hlen:8 + hlen + 4096]
    rng = random.Random(4)
    alphabet = b'0123456789-.,[]{}":e '
    seen = set()
    p = tmp_path / "m.safetensors"
    for i in range(250):
        h = bytearray(header)
        for _ in range(rng.randint(1, 6)):
            h[rng.randrange(len(h))] = rng.choice(alphabet)
        data = struct.pack("<Q", len(h)) + bytes(h) + body
        if i % 5 == 0:
            data = data[:rng.randrange(len(data))]
        p.write_bytes(data)
        rc, out = _read(st_dump, p)
        seen.add(rc)
    assert 1 in seen
