"""Source rules of this code base, checked on every CPU test run:

* no TMA / bulk load with cluster multicast anywhere (every kernel may run in multi-GPU
  jobs, where such a load could read another GPU's memory);
* none of the batched-memcpy runtime / driver calls that are closed on the B200 pool;
* no device traps or device asserts (a failed wait records an error and returns instead);
* no code that changes GPU clocks, power limits or persistence mode;
* comments stand on their own: no references to the build's planning documents, the
  remote-execution tool or machine-local paths.

The forbidden spellings are assembled from pieces so that this file does not contain them.
"""
import os
import re
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CODE_EXT = (".py", ".cu", ".cuh", ".cpp", ".hpp", ".h", ".sh", ".cmake", ".txt")


def _files():
    out = subprocess.run(["git", "-C", ROOT, "ls-files"], capture_output=True, text=True).stdout.split()
    me = os.path.relpath(__file__, ROOT)
    return [f for f in out if f.endswith(CODE_EXT) and f != me and not f.startswith("_work/")]


def _grep(pattern, files):
    rx = re.compile(pattern)
    hits = []
    for f in files:
        try:
            with open(os.path.join(ROOT, f), errors="replace") as fh:
                for i, line in enumerate(fh, 1):
                    if rx.search(line):
                        hits.append(f"{f}:{i}: {line.strip()[:120]}")
        except OSError:
            pass
    return hits


def test_no_cluster_multicast_loads():
    mc = "multi" + "cast" + "::" + "cluster"
    hits = _grep(r"cp\.async\.bulk[^;\n]*" + re.escape(mc), _files())
    hits += _grep(re.escape("." + mc) + r"[^;\n]*\[", [f for f in _files() if f.endswith((".cu", ".cuh"))])
    # tcgen05.commit may name the qualifier (it is not a load); nothing else may
    hits = [h for h in hits if "tcgen05.commit" not in h]
    assert not hits, hits


def test_no_closed_batched_memcpy_calls():
    names = ["cuda" + "Memcpy" + "Batch" + "Async", "cuda" + "Memcpy3D" + "Batch" + "Async",
             "cu" + "Memcpy" + "Batch" + "Async", "cu" + "Memcpy3D" + "Batch" + "Async"]
    hits = _grep("|".join(map(re.escape, names)), _files())
    assert not hits, hits


def test_no_device_traps_or_asserts():
    dev = [f for f in _files() if f.endswith((".cu", ".cuh"))]
    hits = _grep(r"__" + r"trap\s*\(|\btrap\s*;|(?<![_a-z])assert\s*\(", dev)
    assert not hits, hits


def test_no_gpu_setting_changes():
    pats = [r"nvidia-smi[^\n]*\s-(" + "lgc|lmc|ac|pm|pl|rgc|rmc|mig|e" + r")\b", "lock-" + "gpu-clocks",
            "nvml" + r"DeviceSet\w*", "cuda" + "DeviceSetLimit" + r"\(\s*cudaLimitPersisting"]
    hits = _grep("|".join(pats), _files())
    assert not hits, hits


def test_comments_stand_on_their_own():
    docs = ["SURVEY", "DESIGN", "BASELINE", "VERDICT", "ADVICE"]
    pats = [r"\b(" + "|".join(docs) + r")\.md\b", r"\b(" + "|".join(docs) + r") (config|item|section)\b",
            "gpu" + "run", r"/root/", r"\b(?i:survey)'?s?\b"]
    hits = _grep("|".join(pats), _files())
    assert not hits, hits
