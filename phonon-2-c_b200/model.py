"""phonon-2-c's model structs (include/phonon2.h, the reference's csrc/phonon2.h:109-206) as ctypes mirrors, and a
seeded synthetic encoder in them.

A ``SyntheticModel`` owns numpy arrays for every encoder tensor and a ``P2Model`` whose pointers point into them, the
way phonon-2-c's loader points a P2Model into its weights.bin mapping. Anything that takes a ``const P2Model *`` can
take ``ctypes.byref(model.struct)``. The decoder tables are fp32 as the loader expands them (``decoder=False`` leaves
them NULL: the encoder never reads them).

Distributions: five-value weights as ``synth.five_value`` (P(0) = 1/3, lo ~ U(0.005, 0.02), hi = lo * U(2, 4), fp16
values: the weight statistics of phonon-2-c's five-value format, csrc/blas.h:38-45); fp32 norms and biases
N(0, 0.02); LayerNorm gains ``1 + N(0, 0.02)`` by default (``gamma="unit"``) or plain N(0, 0.02) (``gamma="small"``);
convolution weights N(0, 1 / fan_in); int8 tables with int6 values and per-column scales of about 1 / (18 sqrt K), so
every layer keeps activations of order one.

``attn_out_gain`` scales the magnitudes (lo, hi) of every block's attention output projection. With the same weight
statistics everywhere (gain 1) the 24 blocks' relative-position attention averages the frames of a window into one
common vector: the encoder output then varies across time by about 7 % of its spread across dimensions, and greedy TDT
decoding (csrc/decoder.c:100-141) of it emits almost no tokens, so that end-to-end token comparisons would compare
empty lists. ``SPEECH_ATTN_OUT_GAIN`` (0.1) keeps about 60 % of the spread across time; the decoder then emits about one
token per encoder frame, dozens of distinct ids per 30 s window, with top-2 logit gaps that 1e-4 perturbations of the
encoder output do not close. Every kernel runs the same operations on either model.
"""
from __future__ import annotations

import ctypes as C
import zlib

import numpy as np

from . import synth

D, H, DH, FF, NB, KC = 1024, 8, 128, 4096, 24, 9
SUBC, NMEL, JOINT = 256, 128, 640
LSTM_LAYERS, DEC_OWNED = 2, 8
HID, EMB, VOCAB, BLANK, N_DUR = 640, 640, 8193, 8192, 5
MAX_SYMBOLS = 10   # tokens at one frame before the decoder moves on (csrc/phonon2.h:92)
LOGITS = VOCAB + N_DUR
W_F32, W_I8, W_FV = 0, 8, 5
SPEECH_ATTN_OUT_GAIN = 0.1   # the attention output gain of the model whose greedy decoding emits tokens


class Weight(C.Structure):   # csrc/phonon2.h:116-126
    _fields_ = [("kind", C.c_int), ("K", C.c_int), ("N", C.c_int),
                ("f32", C.c_void_p), ("q8", C.c_void_p), ("scales", C.c_void_p),
                ("signs", C.c_void_p), ("flags", C.c_void_p), ("lo", C.c_void_p), ("hi", C.c_void_p),
                ("codes", C.c_void_p)]


class SubsamplingWeights(C.Structure):   # csrc/phonon2.h:128-137
    _fields_ = [(n, C.c_void_p) for n in ("conv0_w", "conv0_b", "conv2_w", "conv2_b", "conv3_w", "conv3_b",
                                          "conv5_w", "conv5_b", "conv6_w", "conv6_b")] + \
               [("linear_w", Weight), ("linear_b", C.c_void_p)]


class FFWeights(C.Structure):   # csrc/phonon2.h:139-142
    _fields_ = [("linear1_w", Weight), ("linear2_w", Weight)]


class MHAWeights(C.Structure):   # csrc/phonon2.h:144-150
    _fields_ = [("qkv_w", Weight), ("pos_w", Weight), ("out_w", Weight), ("bias_u", C.c_void_p),
                ("bias_v", C.c_void_p)]


class ConvModWeights(C.Structure):   # csrc/phonon2.h:152-157
    _fields_ = [("pw1_w", Weight), ("dw_w", C.c_void_p), ("dw_b", C.c_void_p), ("pw2_w", Weight)]


class ConformerBlock(C.Structure):   # csrc/phonon2.h:159-169
    _fields_ = [("norm_ff1_w", C.c_void_p), ("norm_ff1_b", C.c_void_p), ("ff1", FFWeights),
                ("norm_sa_w", C.c_void_p), ("norm_sa_b", C.c_void_p), ("mha", MHAWeights),
                ("norm_conv_w", C.c_void_p), ("norm_conv_b", C.c_void_p), ("conv", ConvModWeights),
                ("norm_ff2_w", C.c_void_p), ("norm_ff2_b", C.c_void_p), ("ff2", FFWeights),
                ("norm_out_w", C.c_void_p), ("norm_out_b", C.c_void_p)]


class EncoderWeights(C.Structure):   # csrc/phonon2.h:177-182
    _fields_ = [("subsampling", SubsamplingWeights), ("blocks", ConformerBlock * NB), ("projector_w", Weight),
                ("projector_b", C.c_void_p)]


class DecoderWeights(C.Structure):   # csrc/phonon2.h:189-199
    _fields_ = [("embed_w", C.c_void_p), ("lstm_w_ih", C.c_void_p * LSTM_LAYERS),
                ("lstm_w_hh", C.c_void_p * LSTM_LAYERS), ("lstm_b_ih", C.c_void_p * LSTM_LAYERS),
                ("lstm_b_hh", C.c_void_p * LSTM_LAYERS), ("proj_w", C.c_void_p), ("proj_b", C.c_void_p),
                ("head_w", C.c_void_p), ("head_b", C.c_void_p), ("owned", C.c_void_p * DEC_OWNED),
                ("n_owned", C.c_int)]


class P2Model(C.Structure):   # csrc/phonon2.h:201-206
    _fields_ = [("enc", EncoderWeights), ("dec", DecoderWeights), ("map", C.c_void_p), ("map_len", C.c_size_t)]


def _seed(base: int, name: str) -> int:
    return (base * 1_000_003 + zlib.crc32(name.encode())) & 0x7FFFFFFF


class SyntheticModel:
    """A seeded random encoder laid out as phonon-2-c's P2Model (``struct``), arrays kept alive by this object."""

    def __init__(self, seed: int = 0, gamma: str = "unit", decoder: bool = True, attn_out_gain: float = 1.0):
        if gamma not in ("unit", "small"):
            raise ValueError("gamma is 'unit' or 'small'")
        self.seed, self.gamma, self.attn_out_gain = seed, gamma, float(attn_out_gain)
        self.arrays: dict[str, np.ndarray] = {}
        self.struct = P2Model()
        e = self.struct.enc
        s = e.subsampling
        s.conv0_w = self._normal("subsampling.conv.0.weight", SUBC * 9, 1 / 3)
        s.conv0_b = self._normal("subsampling.conv.0.bias", SUBC, 0.02)
        s.conv2_w = self._normal("subsampling.conv.2.weight", SUBC * 9, 1 / 3)
        s.conv2_b = self._normal("subsampling.conv.2.bias", SUBC, 0.02)
        s.conv3_w = self._normal("subsampling.conv.3.weight", SUBC * SUBC, 1 / 16)
        s.conv3_b = self._normal("subsampling.conv.3.bias", SUBC, 0.02)
        s.conv5_w = self._normal("subsampling.conv.5.weight", SUBC * 9, 1 / 3)
        s.conv5_b = self._normal("subsampling.conv.5.bias", SUBC, 0.02)
        s.conv6_w = self._normal("subsampling.conv.6.weight", SUBC * SUBC, 1 / 16)
        s.conv6_b = self._normal("subsampling.conv.6.bias", SUBC, 0.02)
        self._table(s.linear_w, "subsampling.linear.weight", SUBC * (NMEL // 8), D)
        s.linear_b = self._normal("subsampling.linear.bias", D, 0.02)
        for i in range(NB):
            b = e.blocks[i]
            p = f"layers.{i}."
            b.norm_ff1_w, b.norm_ff1_b = self._norm(p + "norm_feed_forward1")
            self._five(b.ff1.linear1_w, p + "feed_forward1.linear1.weight", D, FF)
            self._five(b.ff1.linear2_w, p + "feed_forward1.linear2.weight", FF, D)
            b.norm_sa_w, b.norm_sa_b = self._norm(p + "norm_self_att")
            self._five(b.mha.qkv_w, p + "self_attn.qkv_proj.weight", D, 3 * D)
            self._five(b.mha.pos_w, p + "self_attn.relative_k_proj.weight", D, D)
            self._five(b.mha.out_w, p + "self_attn.o_proj.weight", D, D, gain=self.attn_out_gain)
            b.mha.bias_u = self._normal(p + "self_attn.bias_u", D, 0.02)
            b.mha.bias_v = self._normal(p + "self_attn.bias_v", D, 0.02)
            b.norm_conv_w, b.norm_conv_b = self._norm(p + "norm_conv")
            self._five(b.conv.pw1_w, p + "conv.pointwise_conv1.weight", D, 2 * D)
            b.conv.dw_w = self._normal(p + "conv.depthwise_conv.weight", D * KC, 1 / 3)
            b.conv.dw_b = self._normal(p + "conv.depthwise_conv.bias", D, 0.02)
            self._five(b.conv.pw2_w, p + "conv.pointwise_conv2.weight", D, D)
            b.norm_ff2_w, b.norm_ff2_b = self._norm(p + "norm_feed_forward2")
            self._five(b.ff2.linear1_w, p + "feed_forward2.linear1.weight", D, FF)
            self._five(b.ff2.linear2_w, p + "feed_forward2.linear2.weight", FF, D)
            b.norm_out_w, b.norm_out_b = self._norm(p + "norm_out")
        self._table(e.projector_w, "encoder_projector.weight", D, JOINT)
        e.projector_b = self._normal("encoder_projector.bias", JOINT, 0.02)
        if decoder:
            self._decoder()

    def _decoder(self) -> None:
        """The TDT prediction and joint networks as the loader leaves them (csrc/weights.c:498-512): fp32 tables.
        PyTorch-style uniform(+-1/sqrt(640)) LSTM and projector weights, a zero blank embedding row, and a joint head
        whose blank logit is biased up so that blanks and tokens alternate as in speech."""
        d = self.struct.dec
        H = HID
        bound = 1.0 / np.sqrt(H)

        def uniform(name, shape):
            rng = np.random.default_rng(_seed(self.seed, name))
            return self._keep(name, rng.uniform(-bound, bound, shape).astype(np.float32))

        rng = np.random.default_rng(_seed(self.seed, "decoder.embedding.weight"))
        emb = rng.standard_normal((VOCAB, EMB)).astype(np.float32)
        emb[BLANK] = 0.0
        d.embed_w = self._keep("decoder.embedding.weight", emb)
        for l in range(LSTM_LAYERS):
            d.lstm_w_ih[l] = uniform(f"decoder.lstm.weight_ih_l{l}", (4 * H, EMB if l == 0 else H))
            d.lstm_w_hh[l] = uniform(f"decoder.lstm.weight_hh_l{l}", (4 * H, H))
            d.lstm_b_ih[l] = uniform(f"decoder.lstm.bias_ih_l{l}", (4 * H,))
            d.lstm_b_hh[l] = uniform(f"decoder.lstm.bias_hh_l{l}", (4 * H,))
        d.proj_w = uniform("decoder.decoder_projector.weight", (JOINT, H))
        d.proj_b = uniform("decoder.decoder_projector.bias", (JOINT,))
        rng = np.random.default_rng(_seed(self.seed, "joint.head.weight"))
        d.head_w = self._keep("joint.head.weight", (rng.standard_normal((LOGITS, JOINT)) / np.sqrt(JOINT)).astype(
            np.float32))
        rng = np.random.default_rng(_seed(self.seed, "joint.head.bias"))
        hb = (rng.standard_normal(LOGITS) * 0.02).astype(np.float32)
        hb[BLANK] += 2.5
        d.head_b = self._keep("joint.head.bias", hb)
        d.n_owned = 0

    # -- array makers: each stores its array and returns the address for the struct
    def _keep(self, name: str, a: np.ndarray) -> int:
        a = np.ascontiguousarray(a)
        self.arrays[name] = a
        return a.ctypes.data

    def _normal(self, name: str, n: int, std: float) -> int:
        rng = np.random.default_rng(_seed(self.seed, name))
        return self._keep(name, (rng.standard_normal(n) * std).astype(np.float32))

    def _norm(self, prefix: str) -> tuple[int, int]:
        rng = np.random.default_rng(_seed(self.seed, prefix + ".weight"))
        g = rng.standard_normal(D) * 0.02 + (1.0 if self.gamma == "unit" else 0.0)
        gw = self._keep(prefix + ".weight", g.astype(np.float32))
        return gw, self._normal(prefix + ".bias", D, 0.02)

    def _five(self, w: Weight, name: str, K: int, N: int, gain: float = 1.0) -> None:
        fv = synth.five_value(K, N, _seed(self.seed, name))
        if gain != 1.0:   # magnitudes stay fp16 values, as the format keeps them
            fv["lo"] = (fv["lo"] * np.float32(gain)).astype(np.float16).astype(np.float32)
            fv["hi"] = (fv["hi"] * np.float32(gain)).astype(np.float16).astype(np.float32)
        w.kind, w.K, w.N = W_FV, K, N
        w.signs = self._keep(name + ".signs", fv["signs"])
        w.flags = self._keep(name + ".flags", fv["flags"])
        w.lo = self._keep(name + ".lo", fv["lo"])
        w.hi = self._keep(name + ".hi", fv["hi"])

    def _table(self, w: Weight, name: str, K: int, N: int) -> None:
        rng = np.random.default_rng(_seed(self.seed, name))
        q8 = rng.integers(-31, 32, size=(K, N), dtype=np.int8)
        scales = (rng.uniform(0.5, 1.5, N) / (18.0 * np.sqrt(K))).astype(np.float32)
        w.kind, w.K, w.N = W_I8, K, N
        w.q8 = self._keep(name + ".q8", q8)
        w.scales = self._keep(name + ".scales", scales)

    def five_value(self, name: str) -> dict:
        """The synth.five_value dict of one five-value weight, by its tensor name."""
        a = self.arrays
        K = a[name + ".signs"].shape[0]
        return {"signs": a[name + ".signs"], "flags": a[name + ".flags"], "lo": a[name + ".lo"],
                "hi": a[name + ".hi"], "K": K, "N": a[name + ".lo"].shape[0]}

    @property
    def nbytes(self) -> int:
        return sum(a.nbytes for a in self.arrays.values())


def frames_after_subsampling(n_mel: int) -> int:
    """Encoder frames of n_mel mel frames: three stride-2 convolutions (csrc/encoder.c:174, 753-756)."""
    t = n_mel
    for _ in range(3):
        t = (t - 1) // 2 + 1
    return t


def mel(n_frames: int, seed: int) -> np.ndarray:
    """Synthetic log-mel features [n_frames, 128], N(0, 1) per feature (normalised features, as csrc/mel.c:200-215
    leaves them)."""
    return np.random.default_rng(seed).standard_normal((n_frames, NMEL), dtype=np.float32)


def audio(n_samples: int, seed: int) -> np.ndarray:
    """Synthetic 16 kHz audio [n_samples]: a few gliding harmonics with a syllable-rate envelope over low noise,
    seeded (speech-like spectra for the log-mel front end; no dataset is involved)."""
    rng = np.random.default_rng(seed)
    t = np.arange(n_samples) / 16000.0
    f0 = 110.0 + 60.0 * np.sin(2 * np.pi * 0.7 * t + rng.uniform(0, 6.3))
    phase = 2 * np.pi * np.cumsum(f0) / 16000.0
    x = sum((0.3 / k) * np.sin(k * phase + rng.uniform(0, 6.3)) for k in range(1, 9))
    env = 0.5 + 0.5 * np.sin(2 * np.pi * 4.0 * t + rng.uniform(0, 6.3))
    return (x * env + 0.01 * rng.standard_normal(n_samples)).astype(np.float32)


def audio_with_pauses(seconds: float, seed: int, pause_lo: float = 0.05, pause_hi: float = 1.4) -> np.ndarray:
    """Synthetic long-form 16 kHz audio: bursts of audio() (1-6 s each, random level) separated by pauses of low noise
    (pause_lo-pause_hi s), seeded - material for the segmenter, which cuts at pauses."""
    rng = np.random.default_rng(seed)
    parts, n, total = [], 0, int(seconds * 16000)
    while n < total:
        k = int(rng.uniform(1.0, 6.0) * 16000)
        parts.append(audio(k, int(rng.integers(1 << 30))) * np.float32(rng.uniform(0.2, 1.0)))
        p = int(rng.uniform(pause_lo, pause_hi) * 16000)
        parts.append((rng.standard_normal(p) * rng.uniform(0.0002, 0.002)).astype(np.float32))
        n += k + p
    return np.concatenate(parts)[:total].astype(np.float32)


def long_audio_windows(seed: int = 0, n: int = 64, lo_s: float = 25.0, hi_s: float = 35.0) -> list[int]:
    """Mel frame counts of a long-audio batch: n windows of U(lo_s, hi_s) seconds of a synthetic stream (the 25-35 s
    windows the reference's segmenter cuts, csrc/segment.c:52-87), 100 mel frames per second."""
    rng = np.random.default_rng(seed)
    return [int(round(s * 100)) for s in rng.uniform(lo_s, hi_s, n)]
