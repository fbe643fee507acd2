"""Seeded random-init decoder models and encoder outputs in parakeet.cpp's GGUF layout.

There are no real TDT/EOU GGUFs or NeMo dumps on this machine, so every test and
benchmark runs on synthetic decoders of the named geometries:

* tensor names and layout follow the converter (scripts/convert-nemo-to-gguf.py:
  TDT tensors :563-584, EOU tensors :506-525, metadata :293-352);
* 2-D weights are quantized exactly as the converter's ``add_2d`` does
  (:405-413): q8_0 through ``gguf.quants.quantize`` when ``in % 32 == 0``,
  otherwise the f16 fallback; biases are f32 (``add_f32``, :402-403);
* weights are N(0, 1/fan_in) (std = 1/sqrt(in_dim)), biases zero except the
  blank output bias, encoder outputs are N(0, 1) -- all from numpy's PCG64
  generator with a recorded seed.
"""
from __future__ import annotations

import dataclasses
import math
from typing import Dict, List, Optional, Sequence

import numpy as np

GGML_F32, GGML_F16, GGML_Q8_0 = 0, 1, 8


@dataclasses.dataclass
class Tensor:
    """One GGUF tensor: raw bytes plus ggml type id and shape (ne0 = in, ne1 = out)."""
    data: np.ndarray          # uint8 raw blocks
    type: int
    ne0: int
    ne1: int

    @property
    def nbytes(self) -> int:
        return int(self.data.nbytes)


@dataclasses.dataclass
class DecoderModel:
    model_type: str                   # "tdt" or "eou"
    d_enc: int
    pred_hidden: int
    joint_hidden: int
    n_layers: int
    vocab_size: int
    blank_id: int
    durations: List[int]
    eou_id: int
    eob_id: int
    max_symbols_per_step: int
    pieces: List[str]
    tensors: Dict[str, Tensor]
    seed: int
    wtype: str

    @property
    def v_plus_1(self) -> int:
        return self.vocab_size + 1

    @property
    def v_out(self) -> int:
        return self.v_plus_1 + (len(self.durations) if self.model_type == "tdt" else 0)

    @property
    def prefix(self) -> str:
        return "tdt" if self.model_type == "tdt" else "eou"

    def special_mask(self) -> np.ndarray:
        """1 where a tokenizer piece looks like ``<...>`` (parakeet_eou.cpp:315-319)."""
        return np.array([1 if (len(p) > 0 and p[0] == "<" and p[-1] == ">") else 0
                         for p in self.pieces], dtype=np.uint8)


def encode_2d(arr: np.ndarray, wtype: str) -> Tensor:
    """The converter's add_2d (scripts/convert-nemo-to-gguf.py:405-413)."""
    import gguf
    arr = np.ascontiguousarray(arr, dtype=np.float32)
    out_dim, in_dim = arr.shape
    if wtype == "f32":
        return Tensor(arr.view(np.uint8).reshape(-1), GGML_F32, in_dim, out_dim)
    if wtype == "q8_0" and in_dim % 32 == 0:
        packed = gguf.quants.quantize(arr, gguf.GGMLQuantizationType.Q8_0)
        return Tensor(np.ascontiguousarray(packed).reshape(-1), GGML_Q8_0, in_dim, out_dim)
    half = arr.astype(np.float16)
    return Tensor(half.view(np.uint8).reshape(-1), GGML_F16, in_dim, out_dim)


def encode_f32(vec: np.ndarray) -> Tensor:
    vec = np.ascontiguousarray(vec, dtype=np.float32).reshape(-1)
    return Tensor(vec.view(np.uint8).reshape(-1), GGML_F32, vec.shape[0], 1)


def dequantize(t: Tensor) -> np.ndarray:
    """Reference values of a tensor via gguf-py (f32 [ne1][ne0])."""
    import gguf
    if t.type == GGML_F32:
        return t.data.view(np.float32).reshape(t.ne1, t.ne0)
    if t.type == GGML_F16:
        return t.data.view(np.float16).astype(np.float32).reshape(t.ne1, t.ne0)
    if t.type == GGML_Q8_0:
        rows = t.data.reshape(t.ne1, -1)
        return gguf.quants.dequantize(rows, gguf.GGMLQuantizationType.Q8_0).reshape(t.ne1, t.ne0)
    raise ValueError(f"unsupported type {t.type}")


def _pieces(n: int, specials: Dict[int, str]) -> List[str]:
    # Plain pieces never look like "<...>", so only the listed ids are special.
    out = []
    for i in range(n):
        out.append(specials.get(i, "▁p%d" % i if i % 3 == 0 else "p%d" % i))
    return out


def make_decoder(model_type: str = "tdt", *, vocab_size: int = 8192, d_enc: int = 1024,
                 pred_hidden: int = 640, joint_hidden: int = 640, n_layers: int = 2,
                 durations: Sequence[int] = (0, 1, 2, 3, 4), wtype: str = "q8_0",
                 blank_bias: float = 2.0, seed: int = 1234,
                 eou_id: Optional[int] = None, eob_id: Optional[int] = None,
                 max_symbols_per_step: Optional[int] = None,
                 weight_scale: float = 1.0) -> DecoderModel:
    """Random-init decoder with the converter's tensor layout.

    ``weight_scale`` multiplies every weight's std (1.0 = N(0, 1/fan_in))."""
    rng = np.random.default_rng(seed)
    H, J, De = pred_hidden, joint_hidden, d_enc
    V1 = vocab_size + 1
    durs = list(durations) if model_type == "tdt" else []
    Vo = V1 + len(durs)

    def w(out_dim, in_dim):
        return (rng.standard_normal((out_dim, in_dim), dtype=np.float32)
                * np.float32(weight_scale / math.sqrt(in_dim)))

    p = "tdt" if model_type == "tdt" else "eou"
    t: Dict[str, Tensor] = {}
    t[f"{p}.predict.embed.weight"] = encode_2d(w(V1, H), wtype)
    for l in range(n_layers):
        t[f"{p}.predict.lstm.{l}.w_ih"] = encode_2d(w(4 * H, H), wtype)
        t[f"{p}.predict.lstm.{l}.w_hh"] = encode_2d(w(4 * H, H), wtype)
        t[f"{p}.predict.lstm.{l}.b_ih"] = encode_f32(np.zeros(4 * H, np.float32))
        t[f"{p}.predict.lstm.{l}.b_hh"] = encode_f32(np.zeros(4 * H, np.float32))
    t[f"{p}.joint.enc.weight"] = encode_2d(w(J, De), wtype)
    t[f"{p}.joint.enc.bias"] = encode_f32(np.zeros(J, np.float32))
    t[f"{p}.joint.pred.weight"] = encode_2d(w(J, H), wtype)
    t[f"{p}.joint.pred.bias"] = encode_f32(np.zeros(J, np.float32))
    t[f"{p}.joint.out.weight"] = encode_2d(w(Vo, J), wtype)
    b_out = np.zeros(Vo, np.float32)
    blank = vocab_size                      # blank_as_pad at vocab_size (converter :316, :344)
    b_out[blank] = np.float32(blank_bias)
    t[f"{p}.joint.out.bias"] = encode_f32(b_out)

    if model_type == "eou":
        e_id = vocab_size - 3 if eou_id is None else eou_id
        b_id = vocab_size - 2 if eob_id is None else eob_id
        pieces = _pieces(vocab_size, {0: "<unk>", e_id: "<EOU>", b_id: "<EOB>"})
        msym = 5 if max_symbols_per_step is None else max_symbols_per_step
    else:
        e_id, b_id = -1, -1
        pieces = _pieces(vocab_size, {0: "<unk>"})
        msym = 10 if max_symbols_per_step is None else max_symbols_per_step
    return DecoderModel(model_type, De, H, J, n_layers, vocab_size, blank, durs, e_id, b_id,
                        msym, pieces, t, seed, wtype)


# Named geometries of the benchmark configurations.
def tdt_0_6b(seed=1234, wtype="q8_0", blank_bias=2.0) -> DecoderModel:
    return make_decoder("tdt", vocab_size=8192, d_enc=1024, n_layers=2, wtype=wtype,
                        blank_bias=blank_bias, seed=seed)


def tdt_1_1b(seed=1234, wtype="q8_0", blank_bias=2.0) -> DecoderModel:
    return make_decoder("tdt", vocab_size=1024, d_enc=1024, n_layers=2, wtype=wtype,
                        blank_bias=blank_bias, seed=seed)


def eou_120m(seed=1234, wtype="f16", blank_bias=2.0) -> DecoderModel:
    # 1028 outputs = vocab_size + 1 with blank = vocab_size (parakeet_eou.cpp:180).
    return make_decoder("eou", vocab_size=1027, d_enc=512, n_layers=1, wtype=wtype,
                        blank_bias=blank_bias, seed=seed, eou_id=1024, eob_id=1025)


def encoder_batch(n_frames: Sequence[int], d_enc: int, seed: int = 99):
    """N(0,1) f32 encoder outputs for a ragged batch: (enc [sum T][d_enc], offsets)."""
    n = np.asarray(n_frames, dtype=np.int64)
    offs = np.zeros(len(n), dtype=np.int64)
    if len(n) > 1:
        offs[1:] = np.cumsum(n)[:-1]
    rng = np.random.default_rng(seed)
    enc = rng.standard_normal((int(n.sum()), d_enc), dtype=np.float32)
    return enc, offs


POOL_FRAMES = 65536


def encoder_pool(d_enc: int, seed: int = 99, pool_frames: int = POOL_FRAMES) -> np.ndarray:
    """One seeded N(0,1) f32 pool of encoder frames [pool_frames][d_enc]."""
    return np.random.default_rng(seed).standard_normal((pool_frames, d_enc), dtype=np.float32)


def pooled_rows(n_frames: Sequence[int], ids: Sequence[int], pool_frames: int = POOL_FRAMES) -> np.ndarray:
    """Pool row of every frame of a batch: utterance u reads pool_frames-periodic
    consecutive rows from start (u * 2654435761) mod pool_frames."""
    n = np.asarray(n_frames, dtype=np.int64)
    starts = (np.asarray(ids, dtype=np.int64) * 2654435761) % pool_frames
    rel = np.arange(int(n.sum()), dtype=np.int64) - np.repeat(np.cumsum(n) - n, n)
    return (np.repeat(starts, n) + rel) % pool_frames


def encoder_pooled(n_frames: Sequence[int], ids: Sequence[int], d_enc: int, seed: int = 99,
                   pool: Optional[np.ndarray] = None):
    """N(0,1) f32 encoder outputs for a ragged batch in which utterance ids[i] always
    gets the same frames, whichever batch or shard holds it (a rank of a multi-GPU
    run builds exactly its shard of the global batch): its frames are consecutive
    rows of one seeded pool (``pooled_rows``). Each frame is an N(0,1) vector; the
    pool keeps generation at the host's memory-copy speed for the 4096-utterance,
    1.4 M-frame batch. Returns (enc [sum T][d_enc], offsets)."""
    n = np.asarray(n_frames, dtype=np.int64)
    offs = np.zeros(len(n), dtype=np.int64)
    if len(n) > 1:
        offs[1:] = np.cumsum(n)[:-1]
    if pool is None:
        pool = encoder_pool(d_enc, seed)
    P = pool.shape[0]
    enc = np.empty((int(n.sum()), d_enc), dtype=np.float32)
    starts = (np.asarray(ids, dtype=np.int64) * 2654435761) % P     # as pooled_rows
    for o, s, t in zip(offs, starts, n):
        done = 0
        while done < t:             # consecutive pool rows, wrapping at the end
            r = (s + done) % P
            k = int(min(t - done, P - r))
            enc[o + done:o + done + k] = pool[r:r + k]
            done += k
    return enc, offs


def lengths_uniform(B: int, lo: int, hi: int, seed: int = 7) -> np.ndarray:
    return np.random.default_rng(seed).integers(lo, hi + 1, size=B).astype(np.int32)


def lengths_lognormal(B: int, median: float = 250.0, sigma: float = 0.8,
                      lo: int = 25, hi: int = 3750, seed: int = 7) -> np.ndarray:
    x = np.random.default_rng(seed).lognormal(math.log(median), sigma, size=B)
    return np.clip(np.round(x), lo, hi).astype(np.int32)


def write_gguf(model: DecoderModel, path: str) -> None:
    """Write a decoder-only GGUF with the converter's metadata keys (:293-352)."""
    import gguf
    wr = gguf.GGUFWriter(path, "parakeet")
    wr.add_string("parakeet.model.type", model.model_type)
    wr.add_uint32("parakeet.encoder.d_model", model.d_enc)
    p = model.prefix
    wr.add_uint32(f"parakeet.{p}.vocab_size", model.vocab_size)
    wr.add_uint32(f"parakeet.{p}.blank_id", model.blank_id)
    wr.add_uint32(f"parakeet.{p}.pred_hidden", model.pred_hidden)
    wr.add_uint32(f"parakeet.{p}.pred_rnn_layers", model.n_layers)
    wr.add_uint32(f"parakeet.{p}.joint_hidden", model.joint_hidden)
    if model.model_type == "tdt":
        wr.add_uint32("parakeet.tdt.num_durations", len(model.durations))
        wr.add_array("parakeet.tdt.durations", [int(x) for x in model.durations])
    else:
        wr.add_int32("parakeet.eou.eou_id", model.eou_id)
        wr.add_int32("parakeet.eou.eob_id", model.eob_id)
        wr.add_uint32("parakeet.eou.max_symbols_per_step", model.max_symbols_per_step)
    wr.add_array("tokenizer.ggml.tokens", model.pieces)
    for name, t in model.tensors.items():
        if t.type == GGML_Q8_0:
            wr.add_tensor(name, t.data.reshape(t.ne1, -1),
                          raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        elif t.type == GGML_F16:
            arr = t.data.view(np.float16)
            wr.add_tensor(name, arr.reshape(t.ne1, t.ne0) if t.ne1 > 1 else arr)
        else:
            arr = t.data.view(np.float32)
            wr.add_tensor(name, arr.reshape(t.ne1, t.ne0) if t.ne1 > 1 else arr)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()


def read_gguf(path: str) -> DecoderModel:
    """Load the decoder part of a parakeet GGUF (converter output or write_gguf).

    Metadata defaults follow the reference loader (src/parakeet_ctc.cpp:424-460):
    TDT pred_hidden/joint_hidden 640, 2 layers, 5 durations {0,1,2,3,4}, vocab 8192,
    blank = vocab; EOU 1 layer, vocab 1026, max_symbols_per_step 5, eou/eob ids
    -1 (resolved later to vocab-2 / vocab-1)."""
    from gguf import GGUFReader
    r = GGUFReader(path)

    def val(key, default):
        f = r.fields.get(key)
        return default if f is None else f.contents()

    mtype = val("parakeet.model.type", "ctc")
    if mtype not in ("tdt", "eou"):
        raise ValueError(f"{path}: model type {mtype!r} has no transducer decoder")
    p = mtype
    if p == "tdt":
        H = int(val("parakeet.tdt.pred_hidden", 640)); L = int(val("parakeet.tdt.pred_rnn_layers", 2))
        J = int(val("parakeet.tdt.joint_hidden", 640)); V = int(val("parakeet.tdt.vocab_size", 8192))
        durs = [int(x) for x in val("parakeet.tdt.durations", [0, 1, 2, 3, 4])]
        eou_id = eob_id = -1
        msym = 10
    else:
        H = int(val("parakeet.eou.pred_hidden", 640)); L = int(val("parakeet.eou.pred_rnn_layers", 1))
        J = int(val("parakeet.eou.joint_hidden", 640)); V = int(val("parakeet.eou.vocab_size", 1026))
        durs = []
        eou_id = int(val("parakeet.eou.eou_id", -1)); eob_id = int(val("parakeet.eou.eob_id", -1))
        msym = int(val("parakeet.eou.max_symbols_per_step", 5))
    blank = int(val(f"parakeet.{p}.blank_id", V))
    De = int(val("parakeet.encoder.d_model", 1024))
    pieces = [str(x) for x in val("tokenizer.ggml.tokens", [])]
    tensors: Dict[str, Tensor] = {}
    for t in r.tensors:
        if not t.name.startswith(p + "."):
            continue
        shape = [int(x) for x in t.shape]
        ne0, ne1 = shape[0], (shape[1] if len(shape) > 1 else 1)
        raw = np.ascontiguousarray(t.data).view(np.uint8).reshape(-1).copy()
        tensors[t.name] = Tensor(raw, int(t.tensor_type), ne0, ne1)
    wtype = {GGML_Q8_0: "q8_0", GGML_F16: "f16", GGML_F32: "f32"}.get(
        tensors[f"{p}.joint.out.weight"].type, "?")
    return DecoderModel(mtype, De, H, J, L, V, blank, durs, eou_id, eob_id, msym, pieces,
                        tensors, -1, wtype)
