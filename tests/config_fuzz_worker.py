"""Child process of tests/test_config_parse.py: loads damaged copies of a checkpoint's
config.json through n3d_config_load and prints how each load ended, as one JSON line.
A crash in the library's parser ends this process with a signal, which the test sees.

    python config_fuzz_worker.py CHECKPOINT_DIR WORK_DIR SEED COUNT [values]

With `values`, the file stays well-formed and every count field gets a random value
instead; each config that loads is then planned with n3d_schedule in all four modes.
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


COUNT_FIELDS = [("audio_config", "subsampling_factor"), ("head_config", "num_speakers"),
                ("streaming_config", "fifo_length"), ("streaming_config", "speaker_cache_length"),
                ("streaming_config", "speaker_cache_silence_frames_per_speaker"),
                ("streaming_config", "speaker_cache_update_period"), ("streaming_config", "subsampling_factor"),
                ("streaming_config", "num_speakers"), (None, "chunk_length"), (None, "chunk_right_context"),
                (None, "fifo_length"), (None, "speaker_cache_update_period")]
PROC_FIELDS = [("feature_extractor", "hop_length"), ("feature_extractor", "win_length"),
               ("feature_extractor", "sampling_rate"), (None, "subsampling_factor")]
MODES = ["low_latency", "very_low_latency", "ultra_low_latency", "offline"]


def values(ckpt, work, rng, count):
    """Random count values in well-formed files: loading either succeeds or is a Json
    error, and planning a loaded config ends (UnsupportedAudio at most)."""
    with open(os.path.join(ckpt, "config.json")) as f:
        cfg0 = json.load(f)
    with open(os.path.join(ckpt, "processor_config.json")) as f:
        proc0 = json.load(f)
    pick = lambda: rng.choice([0, 1, 2, 3, 7, 8, 16, 40, 160, 512, 1000, rng.randint(0, 5000), -1, 2.5, "8", None])
    ends = {}
    for _ in range(count):
        cfg, proc = json.loads(json.dumps(cfg0)), json.loads(json.dumps(proc0))
        for _ in range(rng.randint(1, 3)):
            doc, fields = (cfg, COUNT_FIELDS) if rng.random() < 0.7 else (proc, PROC_FIELDS)
            sec, key = rng.choice(fields)
            (doc[sec] if sec else doc)[key] = pick()
        if rng.random() < 0.3:
            mode = rng.choice(["low_latency", "very_low_latency", "ultra_low_latency"])
            proc["streaming_modes"][mode] = [pick(), pick()]
        with open(os.path.join(work, "config.json"), "w") as f:
            json.dump(cfg, f)
        with open(os.path.join(work, "processor_config.json"), "w") as f:
            json.dump(proc, f)
        try:
            c = n3d.Config.load(work)
        except n3d.DiarizationError as e:
            ends[e.kind] = ends.get(e.kind, 0) + 1
            continue
        ends["ok"] = ends.get("ok", 0) + 1
        for mode in MODES:
            for n in (0, 1, 5_000, 123_457):
                try:
                    c.schedule(n, mode)
                except n3d.DiarizationError as e:
                    key = "plan:" + e.kind
                    ends[key] = ends.get(key, 0) + 1
        c.close()
    return ends


def main():
    ckpt, work, seed, count = sys.argv[1], sys.argv[2], int(sys.argv[3]), int(sys.argv[4])
    if len(sys.argv) > 5 and sys.argv[5] == "values":
        os.makedirs(work, exist_ok=True)
        print(json.dumps(values(ckpt, work, random.Random(seed), count)))
        return
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
