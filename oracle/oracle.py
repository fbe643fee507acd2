"""TEST INFRASTRUCTURE ONLY: ctypes binding of the CPU oracle (liboracle.so).

The oracle restates parakeet.cpp's f32 host decoder (src/parakeet_tdt.cpp:25-177,
:813-1005; src/parakeet_eou.cpp:48-387). Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs may use it; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import sys
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")


class orc_state(C.Structure):
    _fields_ = [("h", C.c_void_p), ("c", C.c_void_p), ("pred", C.c_void_p),
                ("symbols_this_step", C.c_int32), ("initialized", C.c_int32),
                ("carry_frames", C.c_int32), ("last_token", C.c_int32),
                ("segment_start_token", C.c_int32)]


class orc_trace(C.Structure):
    _fields_ = [("max_steps", C.c_int32), ("logits", C.c_void_p), ("h", C.c_void_p),
                ("c", C.c_void_p), ("token", C.c_void_p), ("dur_idx", C.c_void_p),
                ("margin_tok", C.c_void_p), ("margin_dur", C.c_void_p), ("frame", C.c_void_p)]


_lib = None


def build() -> None:
    import subprocess
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P, I32 = C.c_void_p, C.c_int32
        L.orc_create.restype = P
        L.orc_create.argtypes = [P, C.c_char_p, I32]
        L.orc_destroy.argtypes = [P]
        L.orc_dequantize.argtypes = [P, P]
        L.orc_dims.argtypes = [P, P]
        L.orc_init_state.argtypes = [P, P]
        L.orc_tdt_decode_window.argtypes = [P, P, I32, I32, I32, P, P, I32, P, P, P]
        L.orc_eou_decode_window.argtypes = [P, P, I32, I32, I32, P, P, I32, P, P, I32, P, P, P]
        L.orc_decode_batch.restype = C.c_double
        L.orc_decode_batch.argtypes = [P, P, P, P, I32, I32, I32, P, P, P, P, P, P, P, P]
        L.orc_ctc_greedy_window.restype = I32
        L.orc_ctc_greedy_window.argtypes = [P, I32, I32, I32, P, P, I32, P, P]
        L.orc_detokenize.restype = C.c_int64
        L.orc_detokenize.argtypes = [P, P, I32, I32, I32, I32, I32, P, C.c_int64, P, C.c_int64]
        _lib = L
    return _lib


def _p(a):
    return C.c_void_p(a.ctypes.data) if a is not None else C.c_void_p(0)


def _abi():
    return sys.modules["parakeet_b200.abi"]


def dequantize(t) -> np.ndarray:
    """Restated ggml to_float of one synth.Tensor -> f32 [ne1][ne0]."""
    out = np.zeros((max(t.ne1, 1), t.ne0), np.float32)
    pt = _abi()._tensor(t)
    rc = lib().orc_dequantize(C.byref(pt), _p(out))
    if rc != 0:
        raise RuntimeError(f"orc_dequantize rc={rc}")
    return out


class Oracle:
    """CPU restatement of the reference decoder for one synthetic model."""

    def __init__(self, model, desc=None):
        self.model = model
        self._desc = desc if desc is not None else _abi().ModelDesc(model)
        err = C.create_string_buffer(256)
        h = lib().orc_create(self._desc.ref(), err, 256)
        if not h:
            raise RuntimeError("orc_create: " + err.value.decode())
        self.h = C.c_void_p(h)
        dims = np.zeros(8, np.int32)
        lib().orc_dims(self.h, _p(dims))
        self.H, self.J, self.De, self.L, self.V1, self.Vo, self.Nd, self.blank = [int(x) for x in dims]
        self.is_tdt = model.model_type == "tdt"
        self.n_logits = self.Vo if self.is_tdt else self.V1

    def __del__(self):
        try:
            if getattr(self, "h", None):
                lib().orc_destroy(self.h)
        except Exception:
            pass

    def new_state(self):
        st = {"h": np.zeros((self.L, self.H), np.float32), "c": np.zeros((self.L, self.H), np.float32),
              "pred": np.zeros(self.H, np.float32)}
        st["s"] = orc_state(_p(st["h"]), _p(st["c"]), _p(st["pred"]), 0, 0, 0, -1, 0)
        return st

    def init_state(self, st):
        lib().orc_init_state(self.h, C.byref(st["s"]))

    def decode_window(self, enc: np.ndarray, st=None, max_symbols: Optional[int] = None,
                      n_tokens_before: int = 0, trace_steps: int = 0, d_enc: Optional[int] = None):
        """One tdt_decode_window / eou_decode_window call. Returns a dict."""
        if st is None:
            st = self.new_state()
        enc = np.ascontiguousarray(enc, np.float32)
        T = int(enc.shape[0]) if enc.ndim == 2 else 0
        msym = self.model.max_symbols_per_step if max_symbols is None else max_symbols
        cap = max(1, T * max(1, msym)) + n_tokens_before
        toks = np.zeros(cap, np.int32)
        bounds = np.zeros(max(1, T), np.int32)
        nt = C.c_int32(n_tokens_before)
        nb = C.c_int32(0)
        steps = C.c_int32(0)
        tr = None
        out = {}
        if trace_steps > 0:
            S = trace_steps
            out["logits"] = np.zeros((S, self.n_logits), np.float32)
            out["h"] = np.zeros((S, self.L, self.H), np.float32)
            out["c"] = np.zeros((S, self.L, self.H), np.float32)
            out["token"] = np.full(S, -1, np.int32)
            out["dur_idx"] = np.full(S, -1, np.int32)
            out["margin_tok"] = np.zeros(S, np.float32)
            out["margin_dur"] = np.zeros(S, np.float32)
            out["frame"] = np.full(S, -1, np.int32)
            tr = orc_trace(S, _p(out["logits"]), _p(out["h"]), _p(out["c"]), _p(out["token"]),
                           _p(out["dur_idx"]), _p(out["margin_tok"]), _p(out["margin_dur"]),
                           _p(out["frame"]))
        de = self.De if d_enc is None else d_enc
        if self.is_tdt:
            rc = lib().orc_tdt_decode_window(self.h, _p(enc), T, de, msym, C.byref(st["s"]),
                                             _p(toks), cap, C.byref(nt), C.byref(steps),
                                             C.byref(tr) if tr is not None else None)
        else:
            rc = lib().orc_eou_decode_window(self.h, _p(enc), T, de, msym, C.byref(st["s"]),
                                             _p(toks), cap, C.byref(nt), _p(bounds), len(bounds),
                                             C.byref(nb), C.byref(steps),
                                             C.byref(tr) if tr is not None else None)
        out.update(rc=int(rc), tokens=toks[n_tokens_before:nt.value].copy(), steps=int(steps.value),
                   bounds=bounds[:nb.value].copy(), state=st)
        if trace_steps > 0:
            n = min(trace_steps, out["steps"])
            for k in ("logits", "h", "c", "token", "dur_idx", "margin_tok", "margin_dur", "frame"):
                out[k] = out[k][:n]
        return out

    def decode_batch(self, enc: np.ndarray, offs: np.ndarray, n_frames: np.ndarray,
                     n_threads: int = 0, max_symbols: Optional[int] = None):
        """Greedy decode of a ragged batch on host threads (the timed CPU baseline)."""
        n_frames = np.ascontiguousarray(n_frames, np.int32)
        offs = np.ascontiguousarray(offs, np.int64)
        B = len(n_frames)
        msym = self.model.max_symbols_per_step if max_symbols is None else max_symbols
        region = np.zeros(B, np.int64)
        if B > 1:
            region[1:] = np.cumsum(n_frames.astype(np.int64) * max(1, msym))[:-1]
        cap = int(n_frames.astype(np.int64).sum() * max(1, msym)) + 1
        toks = np.zeros(cap, np.int32)
        ntok = np.zeros(B, np.int32)
        steps = np.zeros(B, np.int32)
        ms = np.zeros(B, np.float64)
        bounds = nb = bregion = None
        if not self.is_tdt:
            bregion = np.zeros(B, np.int64)
            if B > 1:
                bregion[1:] = np.cumsum(n_frames.astype(np.int64))[:-1]
            bounds = np.zeros(int(n_frames.astype(np.int64).sum()) + 1, np.int32)
            nb = np.zeros(B, np.int32)
        wall = lib().orc_decode_batch(self.h, _p(np.ascontiguousarray(enc, np.float32)), _p(offs),
                                      _p(n_frames), B, msym, n_threads, _p(toks), _p(region),
                                      _p(ntok), _p(steps), _p(bounds), _p(bregion), _p(nb), _p(ms))
        if wall < 0:
            raise RuntimeError("orc_decode_batch failed")
        tokens = [toks[region[b]:region[b] + ntok[b]].copy() for b in range(B)]
        res = {"tokens": tokens, "steps": steps, "ms": ms, "wall_ms": wall}
        if not self.is_tdt:
            res["bounds"] = [bounds[bregion[b]:bregion[b] + nb[b]].copy() for b in range(B)]
        return res


def ctc_greedy_window(logits: np.ndarray, blank_id: int, prev: int = -1):
    """ctc_greedy_decode_window (src/parakeet_ctc.cpp:1831-1865) on [frames][vocab]
    logits. Returns (tokens, first frames, new prev)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, V = logits.shape
    toks = np.zeros(max(T, 1), np.int32)
    frs = np.zeros(max(T, 1), np.int32)
    n = C.c_int32(0)
    pv = C.c_int32(prev)
    rc = lib().orc_ctc_greedy_window(_p(logits), T, V, blank_id, C.byref(pv), _p(toks), T, C.byref(n), _p(frs))
    assert rc == 0
    return toks[:n.value].copy(), frs[:n.value].copy(), pv.value


def detokenize(pieces, tokens, blank_id=-1, bos_id=-1, eos_id=-1, pad_id=-1) -> bytes:
    """parakeet::detokenize (src/sentencepiece_bpe.cpp:9-37) over byte-string pieces."""
    bs = [p.encode("utf-8") if isinstance(p, str) else bytes(p) for p in pieces]
    offs = np.zeros(len(bs) + 1, np.int64)
    offs[1:] = np.cumsum([len(b) for b in bs])
    buf = np.frombuffer(b"".join(bs) or b"\0", dtype=np.uint8).copy()
    t = np.ascontiguousarray(tokens, dtype=np.int32)
    n = lib().orc_detokenize(_p(buf), _p(offs), len(bs), blank_id, bos_id, eos_id, pad_id,
                             _p(t) if len(t) else None, len(t), None, 0)
    out = np.zeros(max(n, 1), np.uint8)
    lib().orc_detokenize(_p(buf), _p(offs), len(bs), blank_id, bos_id, eos_id, pad_id,
                         _p(t) if len(t) else None, len(t), _p(out), n)
    return out[:n].tobytes()


REF_PATH = os.path.join(HERE, "_ref", "libref_detok.so")
_ref = None


def ref_detokenize(pieces, tokens, blank_id=-1, bos_id=-1, eos_id=-1, pad_id=-1):
    """The reference's own detokenize (src/sentencepiece_bpe.cpp, built into _ref/ by
    `make ref` from the reference's sources), or None when that library is absent."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_PATH):
            return None
        _ref = C.CDLL(REF_PATH)
        P, I32, I64 = C.c_void_p, C.c_int32, C.c_int64
        _ref.ref_detokenize.restype = I64
        _ref.ref_detokenize.argtypes = [P, P, I32, I32, I32, I32, I32, P, I64, P, I64]
    bs = [p.encode("utf-8") if isinstance(p, str) else bytes(p) for p in pieces]
    offs = np.zeros(len(bs) + 1, np.int64)
    offs[1:] = np.cumsum([len(b) for b in bs])
    buf = np.frombuffer(b"".join(bs) or b"\0", dtype=np.uint8).copy()
    t = np.ascontiguousarray(tokens, dtype=np.int32)
    args = (_p(buf), _p(offs), len(bs), blank_id, bos_id, eos_id, pad_id, _p(t) if len(t) else None, len(t))
    n = _ref.ref_detokenize(*args, None, 0)
    out = np.zeros(max(n, 1), np.uint8)
    _ref.ref_detokenize(*args, _p(out), n)
    return out[:n].tobytes()


# ---- the reference's own decoder (src/parakeet_tdt.cpp, src/parakeet_eou.cpp) ----
#
# Built by `make ref` from the reference's sources, unchanged, against the
# host-only ggml stand-in in oracle/ggml_host/ (oracle/_ref/libref_decoder.so).

REF_DECODER_PATH = os.path.join(HERE, "_ref", "libref_decoder.so")
_refdec = None


def ref_decoder_available() -> bool:
    return os.path.exists(REF_DECODER_PATH)


def _ref_lib():
    global _refdec
    if _refdec is None:
        if not os.path.exists(REF_DECODER_PATH):
            raise FileNotFoundError(REF_DECODER_PATH + " (make -C oracle ref with PARAKEET_REFERENCE_DIR set)")
        L = C.CDLL(REF_DECODER_PATH)
        P, I32 = C.c_void_p, C.c_int32
        L.ref_create.restype = P
        L.ref_create.argtypes = [P, C.c_char_p, I32]
        L.ref_destroy.argtypes = [P]
        L.ref_state_new.restype = P
        L.ref_state_new.argtypes = []
        L.ref_state_free.argtypes = [P]
        L.ref_state_get.argtypes = [P, P, P, P, P, P]
        L.ref_decode_window.restype = I32
        L.ref_decode_window.argtypes = [P, P, P, I32, I32, I32, P, I32, P, P, P, I32, P]
        L.ref_decode_batch.restype = C.c_double
        L.ref_decode_batch.argtypes = [P, P, P, P, I32, I32, I32, P, P, P, P, P, P, P, P]
        _refdec = L
    return _refdec


class RefState:
    """A TdtDecodeState / EouDecodeState of the reference (default-constructed:
    uninitialised, so its first window runs tdt_init_state / eou_init_state)."""

    def __init__(self, ref):
        self.ref = ref
        self.h = C.c_void_p(_ref_lib().ref_state_new())

    def __del__(self):
        try:
            if getattr(self, "h", None):
                _ref_lib().ref_state_free(self.h)
        except Exception:
            pass

    def get(self):
        r = self.ref
        h = np.zeros((r.L, r.H), np.float32)
        c = np.zeros((r.L, r.H), np.float32)
        p = np.zeros(r.H, np.float32)
        ints = np.zeros(5, np.int32)
        _ref_lib().ref_state_get(r.h, self.h, _p(h), _p(c), _p(p), _p(ints))
        return {"h": h, "c": c, "pred": p, "symbols_this_step": int(ints[0]), "initialized": int(ints[1]),
                "carry_frames": int(ints[2]), "last_token": int(ints[3]), "segment_start_token": int(ints[4])}


class Reference:
    """The reference's own CPU decoder for one synthetic model (same interface as
    Oracle.decode_window / decode_batch, without traces: the reference exposes
    no per-step logits, only its decoder state between windows)."""

    def __init__(self, model, desc=None):
        self.model = model
        self._desc = desc if desc is not None else _abi().ModelDesc(model)
        err = C.create_string_buffer(256)
        h = _ref_lib().ref_create(self._desc.ref(), err, 256)
        if not h:
            raise RuntimeError("ref_create: " + err.value.decode())
        self.h = C.c_void_p(h)
        self.is_tdt = model.model_type == "tdt"
        self.H = model.pred_hidden
        self.L = model.n_layers
        self.De = model.d_enc

    def __del__(self):
        try:
            if getattr(self, "h", None):
                _ref_lib().ref_destroy(self.h)
        except Exception:
            pass

    def new_state(self) -> RefState:
        return RefState(self)

    def decode_window(self, enc: np.ndarray, st: Optional[RefState] = None, max_symbols: Optional[int] = None,
                      tokens_before: Optional[np.ndarray] = None, d_enc: Optional[int] = None):
        """One tdt_decode_window / eou_decode_window. `tokens_before` is the running
        out_tokens list the reference appends to (EOU boundaries count it)."""
        if st is None:
            st = self.new_state()
        enc = np.ascontiguousarray(enc, np.float32)
        T = int(enc.shape[0]) if enc.ndim == 2 else 0
        msym = self.model.max_symbols_per_step if max_symbols is None else max_symbols
        before = np.zeros(0, np.int32) if tokens_before is None else np.asarray(tokens_before, np.int32)
        n0 = len(before)
        cap = max(1, T * max(1, msym)) + n0
        toks = np.zeros(cap, np.int32)
        toks[:n0] = before
        bounds = np.zeros(max(1, T), np.int32)
        nt, nb, steps = C.c_int32(n0), C.c_int32(0), C.c_int32(0)
        rc = _ref_lib().ref_decode_window(self.h, st.h, _p(enc), T, self.De if d_enc is None else d_enc, msym,
                                          _p(toks), cap, C.byref(nt), C.byref(steps), _p(bounds), len(bounds),
                                          C.byref(nb))
        return {"rc": int(rc), "tokens": toks[n0:nt.value].copy(), "steps": int(steps.value),
                "bounds": bounds[:nb.value].copy(), "state": st}

    def decode_batch(self, enc: np.ndarray, offs: np.ndarray, n_frames: np.ndarray,
                     n_threads: int = 0, max_symbols: Optional[int] = None):
        """tdt_greedy_decode / eou_greedy_decode of a ragged batch on host threads."""
        n_frames = np.ascontiguousarray(n_frames, np.int32)
        offs = np.ascontiguousarray(offs, np.int64)
        B = len(n_frames)
        msym = self.model.max_symbols_per_step if max_symbols is None else max_symbols
        region = np.zeros(B, np.int64)
        if B > 1:
            region[1:] = np.cumsum(n_frames.astype(np.int64) * max(1, msym))[:-1]
        cap = int(n_frames.astype(np.int64).sum() * max(1, msym)) + 1
        toks = np.zeros(cap, np.int32)
        ntok = np.zeros(B, np.int32)
        steps = np.zeros(B, np.int32)
        ms = np.zeros(B, np.float64)
        bounds = nb = bregion = None
        if not self.is_tdt:
            bregion = np.zeros(B, np.int64)
            if B > 1:
                bregion[1:] = np.cumsum(n_frames.astype(np.int64))[:-1]
            bounds = np.zeros(int(n_frames.astype(np.int64).sum()) + 1, np.int32)
            nb = np.zeros(B, np.int32)
        wall = _ref_lib().ref_decode_batch(self.h, _p(np.ascontiguousarray(enc, np.float32)), _p(offs),
                                           _p(n_frames), B, msym, n_threads, _p(toks), _p(region),
                                           _p(ntok), _p(steps), _p(bounds), _p(bregion), _p(nb), _p(ms))
        if wall < 0:
            raise RuntimeError("ref_decode_batch failed")
        tokens = [toks[region[b]:region[b] + ntok[b]].copy() for b in range(B)]
        res = {"tokens": tokens, "steps": steps, "ms": ms, "wall_ms": wall}
        if not self.is_tdt:
            res["bounds"] = [bounds[bregion[b]:bregion[b] + nb[b]].copy() for b in range(B)]
        return res
