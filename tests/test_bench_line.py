"""bench.py's line layout on the CPU: the encoder object (the metric's second half) ends the line, so the last
1500 characters of the output - what a record that keeps only the tail holds - still carry it, its e2e and its CPU
baseline, behind a per-config object of the size the bench prints."""
import json


def test_encoder_object_ends_the_line():
    import bench
    line = {"metric": "five-value int8 GEMM TMAC/s", "value": 126.3, "unit": "TMAC/s", "e2e": {"value": 6.9},
            "cpu_baseline": {"value": 0.43, "sample": "x" * 200}}
    sub = {"value": 1.0, "unit": "audio-s/s", "ms_per_step": 66.8, "windows": 64, "mode": "int8w",
           "weights": "vindex", "description": "dropped by compact()",
           "e2e": {"value": 1.0, "unit": "audio-s/s", "ms_per_step": 70.3, "h2d_bytes_per_step": 98095616,
                   "d2h_bytes_per_step": 61383680, "note": "dropped"}}
    extras = {"encoder": dict(sub), "decoder": dict(sub, tokens_rank0=11057), "mel": dict(sub),
              "long_audio": dict(sub)}
    cfg = {f"c{i}": {"k" * 20: 1.2345, "api": "y" * 150} for i in range(8)}   # ~1.5 KB, as the bench's
    bench.finish_line(line, extras, cfg)
    for name in ("decoder", "mel", "long_audio", "encoder"):
        line[name]["cpu"] = {"value": 43.0, "unit": "audio-s/s", "cores": 16, "kind": "reference"}
    keys = list(line)
    assert keys[-1] == "encoder" and keys.index("configs") < keys.index("decoder")
    assert "description" not in line["encoder"] and "note" not in line["encoder"]["e2e"]
    tail = json.dumps(line)[-1500:]
    assert '"encoder": {"value": 1.0' in tail and '"cpu": {"value": 43.0' in tail.split('"encoder"')[1]
