"""Child process of tests/test_config_parse.py: loads damaged copies of a checkpoint's
config.json through n3d_config_load and prints how each load ended, as one JSON line.
A crash in the library's parser ends this process with a signal, which the test sees.

    python config_fuzz_worker.py CHECKPOINT_DIR WORK_DIR SEED COUNT
"""

import json
import os
import random
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "nemotron3-diarization-wgpu_b200"))

import n3d  # noqa: E402


def cases(base: str, rng: random.Random, count: int):
    """Every 7th prefix of the file, `count` random edits of 1-4 characters, and a few
    hostile documents (deep nesting, huge numbers, long escapes)."""
    for cut in range(0, len(base), 7):
        yield base[:cut]
    alphabet = '{}[]",:0123456789.eE+-tfn \\u\n\t'
    for _ in range(count):
        s = list(base)
        for _ in range(rng.randint(1, 4)):
            i = rng.randrange(len(s))
            op = rng.randrange(3)
            if op == 0:
                s[i] = rng.choice(alphabet)
            elif op == 1:
                del s[i]
            else:
                s.insert(i, rng.choice(alphabet))
        yield "".join(s)
    yield from ["[" * 100_000, '{"a":' * 50_000, "[" * 129 + "]" * 129, "1" * 100_000, "-", "1e99999", "-1e99999",
                '"' + "\\" * 10_001, '{"audio_config": []}', ""]


def main():
    ckpt, work, seed, count = sys.argv[1], sys.argv[2], int(sys.argv[3]), int(sys.argv[4])
    with open(os.path.join(ckpt, "config.json")) as f:
        base = f.read()
    os.makedirs(work, exist_ok=True)
    with open(os.path.join(ckpt, "processor_config.json")) as f, \
            open(os.path.join(work, "processor_config.json"), "w") as g:
        g.write(f.read())
    ends = {}
    for text in cases(base, random.Random(seed), count):
        with open(os.path.join(work, "config.json"), "w") as f:
            f.write(text)
        try:
            n3d.Config.load(work).close()
            end = "ok"
        except n3d.DiarizationError as e:
            end = e.kind
        ends[end] = ends.get(end, 0) + 1
    print(json.dumps(ends))


if __name__ == "__main__":
    main()
