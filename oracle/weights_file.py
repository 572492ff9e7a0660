"""A model directory in phonon-2-c's on-disk format (weights.bin, weights.json, tokens.txt) from the synthetic model.
TEST INFRASTRUCTURE ONLY: it lets the reference's own engine and command-line program (csrc/main.c, engine.c) load the
synthetic weights, so that tests can run the reference end to end beside the same program linked against this
library.

Format (csrc/weights.c:115-331, 411-531): weights.json maps each tensor name to {"dtype", "shape", ...} with byte offsets
into weights.bin - float32: "numel", "offset" (4-byte aligned); int8: "offset" and "scales_offset" (one float32 scale
per column for GEMM tables, per row for the decoder's tables, which the loader expands to float32); five_value:
"signs_offset", "flags_offset", "lo_offset", "hi_offset" - plus "_meta": {"format": "phonon-2-c-weights-v1"}.
tokens.txt (csrc/tokens.c:1-60): 8193 lines, the SentencePiece pieces of ids 0..8191, then "<blank>".

The decoder's float32 tables of the synthetic model are stored as the reference stores them, int8 with a scale per row,
so the model a program loads from this directory has the decoder tables q * scale rather than the synthetic floats.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

FORMAT = "phonon-2-c-weights-v1"
# the decoder tables the loader expands from int8 rows (csrc/weights.c:500-509)
DECODER_INT8 = {"decoder.embedding.weight", "decoder.lstm.weight_ih_l0", "decoder.lstm.weight_hh_l0",
                "decoder.lstm.weight_ih_l1", "decoder.lstm.weight_hh_l1", "decoder.decoder_projector.weight",
                "joint.head.weight"}


def _rows_int8(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-row symmetric int8: scale = max |row| / 127, q = round(x / scale) (all-zero rows: scale 1, q 0)."""
    amax = np.abs(x).max(axis=1)
    scale = np.where(amax > 0, amax / 127.0, 1.0).astype(np.float32)
    q = np.clip(np.rint(x / scale[:, None]), -127, 127).astype(np.int8)
    return q, scale


def write_model_dir(model, directory) -> Path:
    """weights.bin / weights.json / tokens.txt of `model` (a phonon2_b200.model.SyntheticModel with its decoder) in
    `directory`; returns the directory."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    blob = bytearray()
    manifest: dict = {"_meta": {"format": FORMAT}}

    def put(a: np.ndarray) -> int:
        while len(blob) % 64:
            blob.append(0)
        off = len(blob)
        blob.extend(np.ascontiguousarray(a).tobytes())
        return off

    arrays = model.arrays
    for name, a in arrays.items():
        if name.endswith(".signs"):
            base = name[: -len(".signs")]
            K = a.shape[0]
            N = arrays[base + ".lo"].shape[0]
            manifest[base] = {"dtype": "five_value", "shape": [K, N], "signs_offset": put(a),
                              "flags_offset": put(arrays[base + ".flags"]), "lo_offset": put(arrays[base + ".lo"]),
                              "hi_offset": put(arrays[base + ".hi"])}
        elif name.endswith((".flags", ".lo", ".hi", ".scales")) and (name.rsplit(".", 1)[0] + ".signs" in arrays or
                                                                     name.rsplit(".", 1)[0] + ".q8" in arrays):
            continue   # written with their weight
        elif name.endswith(".q8"):
            base = name[: -len(".q8")]
            manifest[base] = {"dtype": "int8", "shape": list(a.shape), "offset": put(a),
                              "scales_offset": put(arrays[base + ".scales"])}
        elif name in DECODER_INT8:
            q, scale = _rows_int8(a.reshape(a.shape[0], -1).astype(np.float32))
            manifest[name] = {"dtype": "int8", "shape": list(q.shape), "offset": put(q), "scales_offset": put(scale)}
        else:
            a = np.ascontiguousarray(a, np.float32)
            manifest[name] = {"dtype": "float32", "shape": list(a.shape), "numel": int(a.size), "offset": put(a)}
    (d / "weights.bin").write_bytes(bytes(blob))
    (d / "weights.json").write_text(json.dumps(manifest))
    pieces = ["<unk>", "<s>", "<pad>", "<|endoftext|>"] + [("▁" if i % 3 == 0 else "") + f"t{i}"
                                                           for i in range(4, 8192)] + ["<blank>"]
    (d / "tokens.txt").write_text("\n".join(pieces) + "\n", encoding="utf-8")
    return d


def as_loaded(model):
    """`model` (a SyntheticModel) with its decoder tables replaced, in place, by what the reference's loader makes of
    them from a directory written by write_model_dir: the int8 rows expanded as (float)q * scale
    (csrc/weights.c:335-364). Returns the model."""
    d = model.struct.dec
    fields = {"decoder.embedding.weight": ("embed_w", None), "decoder.decoder_projector.weight": ("proj_w", None),
              "joint.head.weight": ("head_w", None)}
    for l in range(2):
        fields[f"decoder.lstm.weight_ih_l{l}"] = ("lstm_w_ih", l)
        fields[f"decoder.lstm.weight_hh_l{l}"] = ("lstm_w_hh", l)
    for name, (field, idx) in fields.items():
        a = model.arrays[name]
        q, scale = _rows_int8(a.reshape(a.shape[0], -1).astype(np.float32))
        w = np.ascontiguousarray((q.astype(np.float32) * scale[:, None]).astype(np.float32).reshape(a.shape))
        addr = model._keep(name, w)
        if idx is None:
            setattr(d, field, addr)
        else:
            getattr(d, field)[idx] = addr
    return model


def write_wav16(path, audio: np.ndarray, rate: int = 16000) -> None:
    """Mono 16-bit PCM WAV of float audio in [-1, 1]."""
    import wave
    pcm = np.clip(np.rint(audio * 32767.0), -32768, 32767).astype("<i2")
    with wave.open(str(path), "wb") as w:
        w.setnchannels(1)
        w.setsampwidth(2)
        w.setframerate(rate)
        w.writeframes(pcm.tobytes())
