"""Result records and the resumable result store (CPU)."""
import json

from opengda_b200.utils.results import ResultStore, measured_peaks, record, roofline_fraction


def test_record_has_the_standard_fields():
    r = record("put GB/s", 650.0, "GB/s", 8, shape=[1 << 20], dtype="uint8", seed=1, verified=True,
               roofline=roofline_fraction(650.0, "nvlink_gbs"), size=1 << 20)
    for k in ("metric", "value", "unit", "n_gpus", "shape", "dtype", "seed", "max_over_ranks", "verified",
              "roofline", "commit", "utc"):
        assert k in r
    assert r["size"] == 1 << 20 and abs(r["roofline"]["fraction"] - 650 / 770) < 1e-9
    json.dumps(r)


def test_peaks_fall_back_and_label_the_source(tmp_path):
    p = measured_peaks(str(tmp_path / "missing.json"))
    assert p["source"] == "fallback" and p["hbm_gbs"] == 6650.0
    (tmp_path / "peaks.json").write_text(json.dumps({"hbm_gbs": 6544.0, "bf16_tflops_sustained": 1410.6}))
    p = measured_peaks(str(tmp_path / "peaks.json"))
    assert p["source"] == "measured" and p["hbm_gbs"] == 6544.0 and p["bf16_tflops"] == 1590.0
    assert "measured" in roofline_fraction(1000.0, "bf16_tflops_sustained", p)["of"]


def test_store_resumes_and_ignores_a_torn_last_line(tmp_path):
    path = str(tmp_path / "sweep.jsonl")
    s = ResultStore(path)
    assert not s.done("n=2,size=1024")
    s.add("n=2,size=1024", {"value": 1.0})
    s.add("n=2,size=4096", {"value": 2.0})
    with open(path, "a") as f:
        f.write('{"key": "n=2,size=16384", "rec')  # crash in the middle of a write
    t = ResultStore(path)
    assert t.done("n=2,size=1024") and t.done("n=2,size=4096") and not t.done("n=2,size=16384")
    assert t.get("n=2,size=4096") == {"value": 2.0} and len(list(t.records())) == 2
