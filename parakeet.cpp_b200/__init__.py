"""parakeet_b200: host-side Python mirror of libparakeet_cuda's C ABI.

The product is the C-ABI shared library ``libparakeet_cuda.so`` built from
``csrc/`` (hand-written sm_100a CUDA). This module only binds it with ctypes and
mirrors the reference's decoder entry points for tests and benchmarks:

* ``Decoder(model)``                 -> tdt_prepare_runtime / eou_prepare_runtime
* ``Decoder.decode_batch(...)``      -> tdt_greedy_decode / eou_greedy_decode (batched)
* ``Decoder.stream()`` + ``.window`` -> tdt_decode_window / eou_decode_window with state

There is no CPU fallback: if the library cannot be loaded or has no CUDA
device, calls raise.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import Optional, Sequence

import numpy as np

from . import abi
from . import synth  # noqa: F401  (re-export)

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libparakeet_cuda.so")

_lib = None


class PkError(RuntimeError):
    def __init__(self, status: int, where: str, msg: str):
        super().__init__(f"{where}: {abi.STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


def build(verbose: bool = False) -> str:
    """Compile libparakeet_cuda.so for sm_100a in-tree (nvcc via the package Makefile)."""
    subprocess.run(["make", "-C", PKG_DIR] + ([] if verbose else ["-s"]), check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run parakeet_b200.build() first")
        L = C.CDLL(LIB_PATH)
        I32, I64, P = C.c_int32, C.c_int64, C.c_void_p
        sigs = {
            "pk_create": ([P, I32, P], I32), "pk_destroy": ([P], None),
            "pk_get_info": ([P, P], I32), "pk_set_option": ([P, I32, I64], I32),
            "pk_last_error": ([], C.c_char_p), "pk_abi_version": ([], I32),
            "pk_decode_batch": ([P, P, P], I32), "pk_tokens_capacity": ([P, I32, I32], I64),
            "pk_prefetch_batch": ([P, P, P], I32),
            "pk_decode_trace": ([P, P, P, P], I32), "pk_stream_create": ([P, P], I32),
            "pk_stream_destroy": ([P], None), "pk_stream_reset": ([P], I32),
            "pk_stream_window": ([P, P, I32, I32, I32, I32, I32, P, I32, P, P, P, I32, P], I32),
            "pk_stream_get_state": ([P, P], I32), "pk_stream_set_state": ([P, P], I32),
            "pk_shard_lpt": ([P, I32, I32, P], I32), "pk_shard_balanced": ([P, I32, I32, P], I32),
            "pk_ctc_create": ([I32, I32, I32, P], I32), "pk_ctc_destroy": ([P], None),
            "pk_ctc_greedy": ([P, P, I32, P, P, I32, P, P, I64, P, P, P], I32),
            "pk_vocab_create": ([I32, P, P, I32, I32, I32, I32, I32, P], I32), "pk_vocab_destroy": ([P], None),
            "pk_detokenize": ([P, P, I32, P, I32, P, I64, P, P], I32),
        }
        for name, (args, res) in sigs.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def last_error() -> str:
    m = lib().pk_last_error()
    return m.decode() if m else ""


def _check(rc: int, where: str):
    if rc != abi.PK_OK:
        raise PkError(rc, where, last_error())


def _p(a) -> C.c_void_p:
    return C.c_void_p(0) if a is None else C.c_void_p(a.ctypes.data)


def shard_lpt(n_frames: Sequence[int], n_shards: int) -> np.ndarray:
    """pk_shard_lpt: LPT partition of utterances over devices by frame count."""
    n = np.ascontiguousarray(n_frames, np.int32)
    out = np.zeros(max(len(n), 1), np.int32)
    _check(lib().pk_shard_lpt(_p(n), len(n), n_shards, _p(out)), "pk_shard_lpt")
    return out[:len(n)]


def shard_balanced(n_frames: Sequence[int], n_shards: int) -> np.ndarray:
    """pk_shard_balanced: partition of utterances over devices that balances each
    shard's modelled decode time (its longest utterance's sequential decode and
    the per-iteration cost of its live utterances), not its frames."""
    n = np.ascontiguousarray(n_frames, np.int32)
    out = np.zeros(max(len(n), 1), np.int32)
    _check(lib().pk_shard_balanced(_p(n), len(n), n_shards, _p(out)), "pk_shard_balanced")
    return out[:len(n)]


class Decoder:
    """A libparakeet_cuda context holding one repacked decoder on one device."""

    def __init__(self, model, device: int = 0, desc: Optional[abi.ModelDesc] = None,
                 math: Optional[str] = None, bulk_min_live: Optional[int] = None):
        """math: None (library default: tensor cores when the weights allow), "tc", "f32" or
        "q8" (PK_MATH_Q8: q8_0-quantised activations, ggml's vec_dot_q8_0_q8_0 arithmetic).
        bulk_min_live: PK_OPT_BULK_MIN_LIVE (None: the library default; 0 never runs the
        tcgen05 bulk loop, 1 runs it for every iteration of a fresh batch)."""
        self.model = model
        self._desc = desc if desc is not None else abi.ModelDesc(model)
        h = C.c_void_p()
        _check(lib().pk_create(self._desc.ref(), device, C.byref(h)), "pk_create")
        self.h = h
        info = abi.pk_info()
        _check(lib().pk_get_info(self.h, C.byref(info)), "pk_get_info")
        self.info = info
        if math is not None:
            self.set_option(abi.PK_OPT_MATH, {"tc": abi.PK_MATH_TC, "f32": abi.PK_MATH_F32,
                                              "q8": abi.PK_MATH_Q8}[math])
        if bulk_min_live is not None:
            self.set_option(abi.PK_OPT_BULK_MIN_LIVE, int(bulk_min_live))

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            lib().pk_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_option(self, opt: int, value: int):
        _check(lib().pk_set_option(self.h, opt, value), "pk_set_option")

    def make_batch(self, enc, offs, n_frames, max_symbols=None, enc_on_device=False, d_enc=None,
                   ticket: int = 0):
        """A pk_batch plus the arrays it points to (keep both alive). ticket: a
        prefetch ticket whose staged copy the decode reads instead of enc."""
        n_frames = np.ascontiguousarray(n_frames, np.int32)
        offs = np.ascontiguousarray(offs, np.int64)
        b = abi.pk_batch()
        if enc_on_device:
            b.enc = C.c_void_p(int(enc))
        else:
            enc = np.ascontiguousarray(enc, np.float32)
            b.enc = _p(enc)
        b.enc_on_device = 1 if enc_on_device else 0
        b.B = len(n_frames)
        b.d_enc = self.info.d_enc if d_enc is None else d_enc
        b.max_symbols_per_step = 0 if max_symbols is None else max_symbols
        b.frame_offsets = offs.ctypes.data_as(C.POINTER(C.c_int64))
        b.n_frames = n_frames.ctypes.data_as(C.POINTER(C.c_int32))
        b.prefetch_ticket = int(ticket)
        return b, (enc, offs, n_frames)

    def _msym(self, max_symbols):
        return max_symbols if (max_symbols and max_symbols > 0) else self.info.max_symbols_per_step

    def decode_batch(self, enc, offs, n_frames, max_symbols: Optional[int] = None,
                     enc_on_device: bool = False, d_enc: Optional[int] = None,
                     want_finish: bool = False, ticket: int = 0):
        """Greedy decode of a ragged batch. Returns dict(tokens=[...], steps, ...).
        ticket: a prefetch() ticket; the decode then reads that staged copy."""
        b, keep = self.make_batch(enc, offs, n_frames, max_symbols, enc_on_device, d_enc, ticket)
        n_frames = keep[2]
        B = len(n_frames)
        cap = int(lib().pk_tokens_capacity(_p(n_frames), B, self._msym(max_symbols)))
        toks = np.zeros(max(cap, 1), np.int32)
        offs_out = np.zeros(B + 1, np.int64)
        steps = np.zeros(max(B, 1), np.int32)
        fin = np.zeros(max(B, 1), np.float32)
        r = abi.pk_result()
        r.results_on_device = 0
        r.tokens, r.tokens_cap = _p(toks), len(toks)
        r.token_offsets, r.steps = _p(offs_out), _p(steps)
        bounds = boffs = None
        if self.model.model_type == "eou":
            bounds = np.zeros(max(int(n_frames.astype(np.int64).sum()), 1), np.int32)
            boffs = np.zeros(B + 1, np.int64)
            r.eou_bounds, r.eou_bounds_cap, r.eou_offsets = _p(bounds), len(bounds), _p(boffs)
        if want_finish:
            r.finish_ms = _p(fin)
        _check(lib().pk_decode_batch(self.h, C.byref(b), C.byref(r)), "pk_decode_batch")
        out = {"tokens": [toks[offs_out[i]:offs_out[i + 1]].copy() for i in range(B)],
               "steps": steps[:B].copy(), "total_steps": int(r.total_steps),
               "loop_iterations": int(r.loop_iterations), "encproj_ms": r.encproj_ms,
               "loop_ms": r.loop_ms, "total_ms": r.total_ms, "tokens_needed": int(r.tokens_needed),
               "bulk_ms": r.bulk_ms, "bulk_iterations": int(r.bulk_iterations),
               "bulk_phase_ms": list(r.bulk_phase_ms), "bulk_steps": int(r.bulk_steps),
               "bulk_lstm_steps": int(r.bulk_lstm_steps), "bulk_screened_steps": int(r.bulk_screened_steps)}
        if bounds is not None:
            out["bounds"] = [bounds[boffs[i]:boffs[i + 1]].copy() for i in range(B)]
        if want_finish:
            out["finish_ms"] = fin[:B].copy()
        return out

    def prefetch(self, enc, offs, n_frames, d_enc: Optional[int] = None) -> int:
        """pk_prefetch_batch: start copying host encoder outputs; returns the ticket
        to pass to decode_batch (see the header for the staging rules). The arrays
        are kept alive here until two later prefetches have been made, by which time
        their copy has completed."""
        b, keep = self.make_batch(enc, offs, n_frames, d_enc=d_enc)
        t = C.c_uint64(0)
        _check(lib().pk_prefetch_batch(self.h, C.byref(b), C.byref(t)), "pk_prefetch_batch")
        self._prefetched = (getattr(self, "_prefetched", ()) + (keep,))[-2:]
        return int(t.value)

    def prefetch_raw(self, batch: abi.pk_batch):
        """Direct pk_prefetch_batch call on a prepared struct (benchmarks).
        Returns (status, ticket)."""
        t = C.c_uint64(0)
        rc = int(lib().pk_prefetch_batch(self.h, C.byref(batch), C.byref(t)))
        return rc, int(t.value)

    def decode_batch_raw(self, batch: abi.pk_batch, result: abi.pk_result) -> int:
        """Direct pk_decode_batch call on prepared structs (benchmarks)."""
        return int(lib().pk_decode_batch(self.h, C.byref(batch), C.byref(result)))

    def trace(self, enc, offs, n_frames, max_steps: int, forced_token=None, forced_dur=None,
              max_symbols: Optional[int] = None):
        """Teacher-forced run: per-step logits, device argmax and LSTM state."""
        b, keep = self.make_batch(enc, offs, n_frames, max_symbols)
        n_frames = keep[2]
        B = len(n_frames)
        I = self.info
        out = {"logits": np.zeros((B, max_steps, I.v_out), np.float32),
               "h": np.zeros((B, max_steps, I.n_layers, I.pred_hidden), np.float32),
               "c": np.zeros((B, max_steps, I.n_layers, I.pred_hidden), np.float32),
               "argmax_token": np.full((B, max_steps), -1, np.int32),
               "argmax_dur_idx": np.full((B, max_steps), -1, np.int32)}
        ft = fd = None
        if forced_token is not None:
            ft = np.full((B, max_steps), -1, np.int32)
            fd = np.zeros((B, max_steps), np.int32)
            for i in range(B):
                n = min(max_steps, len(forced_token[i]))
                ft[i, :n] = forced_token[i][:n]
                if forced_dur is not None:
                    fd[i, :n] = forced_dur[i][:n]
        t = abi.pk_trace(max_steps, _p(ft), _p(fd), _p(out["logits"]), _p(out["h"]), _p(out["c"]),
                         _p(out["argmax_token"]), _p(out["argmax_dur_idx"]))
        cap = int(lib().pk_tokens_capacity(_p(n_frames), B, self._msym(max_symbols)))
        toks = np.zeros(max(cap, 1), np.int32)
        offs_out = np.zeros(B + 1, np.int64)
        steps = np.zeros(max(B, 1), np.int32)
        r = abi.pk_result()
        r.tokens, r.tokens_cap, r.token_offsets, r.steps = _p(toks), len(toks), _p(offs_out), _p(steps)
        _check(lib().pk_decode_trace(self.h, C.byref(b), C.byref(t), C.byref(r)), "pk_decode_trace")
        out["tokens"] = [toks[offs_out[i]:offs_out[i + 1]].copy() for i in range(B)]
        out["steps"] = steps[:B].copy()
        return out

    def stream(self) -> "Stream":
        return Stream(self)


class Stream:
    """Device-resident decoder state for tdt_decode_window / eou_decode_window."""

    def __init__(self, dec: Decoder):
        self.dec = dec
        h = C.c_void_p()
        _check(lib().pk_stream_create(dec.h, C.byref(h)), "pk_stream_create")
        self.h = h
        self.n_tokens = 0

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            lib().pk_stream_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        _check(lib().pk_stream_reset(self.h), "pk_stream_reset")
        self.n_tokens = 0

    def window(self, enc: np.ndarray, max_symbols: Optional[int] = None, d_enc: Optional[int] = None):
        enc = np.ascontiguousarray(enc, np.float32)
        T = int(enc.shape[0]) if enc.ndim == 2 else 0
        msym = max_symbols if max_symbols is not None else 0
        cap = max(1, T * max(1, msym if msym > 0 else self.dec.info.max_symbols_per_step))
        toks = np.zeros(cap, np.int32)
        bounds = np.zeros(max(1, T), np.int32)
        nt, ns, nb = C.c_int32(0), C.c_int32(0), C.c_int32(0)
        de = self.dec.info.d_enc if d_enc is None else d_enc
        _check(lib().pk_stream_window(self.h, _p(enc), 0, T, de, msym, self.n_tokens, _p(toks), cap,
                                      C.byref(nt), C.byref(ns), _p(bounds), len(bounds),
                                      C.byref(nb)), "pk_stream_window")
        self.n_tokens += nt.value
        return {"tokens": toks[:nt.value].copy(), "steps": int(ns.value),
                "bounds": bounds[:nb.value].copy()}

    def get_state(self):
        I = self.dec.info
        h = np.zeros((I.n_layers, I.pred_hidden), np.float32)
        c = np.zeros_like(h)
        p = np.zeros(I.pred_hidden, np.float32)
        st = abi.pk_stream_state(_p(h), _p(c), _p(p), 0, 0, 0, 0, 0)
        _check(lib().pk_stream_get_state(self.h, C.byref(st)), "pk_stream_get_state")
        return {"h": h, "c": c, "pred": p, "symbols_this_step": st.symbols_this_step,
                "carry_frames": st.carry_frames, "initialized": st.initialized,
                "last_token": st.last_token, "segment_start_token": st.segment_start_token}

    def set_state(self, s):
        h = np.ascontiguousarray(s["h"], np.float32)
        c = np.ascontiguousarray(s["c"], np.float32)
        p = np.ascontiguousarray(s["pred"], np.float32)
        st = abi.pk_stream_state(_p(h), _p(c), _p(p), int(s["symbols_this_step"]),
                                 int(s["carry_frames"]), int(s["initialized"]),
                                 int(s["last_token"]), int(s["segment_start_token"]))
        _check(lib().pk_stream_set_state(self.h, C.byref(st)), "pk_stream_set_state")


from . import multi  # noqa: E402,F401  (needs shard_lpt defined above)


class CtcGreedy:
    """Batched CTC greedy decode (ctc_greedy_decode / ctc_greedy_decode_window,
    src/parakeet_ctc.cpp:1820-1865) on one GPU through the C ABI."""

    def __init__(self, vocab_size: int, blank_id: int, device: int = 0):
        h = C.c_void_p()
        _check(lib().pk_ctc_create(device, vocab_size, blank_id, C.byref(h)), "pk_ctc_create")
        self._h = h
        self.vocab_size, self.blank_id = vocab_size, blank_id

    def close(self):
        if getattr(self, "_h", None):
            lib().pk_ctc_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def decode(self, logits, frame_offsets, n_frames, prev=None, on_device=False, with_frames=False):
        """logits: [frames][vocab] float32 (numpy, or a device pointer int with on_device).
        Returns (token lists, frame lists or None, new prev array)."""
        n_frames = np.ascontiguousarray(n_frames, dtype=np.int32)
        B = len(n_frames)
        foff = np.ascontiguousarray(frame_offsets, dtype=np.int64)
        prev = np.full(B, -1, np.int32) if prev is None else np.array(prev, dtype=np.int32, copy=True)
        cap = int(n_frames.sum())
        toks = np.zeros(max(cap, 1), np.int32)
        frs = np.zeros(max(cap, 1), np.int32) if with_frames else None
        toff = np.zeros(B + 1, np.int64)
        need = C.c_int64(0)
        if on_device:
            lp = C.c_void_p(int(logits))
        else:
            logits = np.ascontiguousarray(logits, dtype=np.float32)
            lp = _p(logits)
        _check(lib().pk_ctc_greedy(self._h, lp, 1 if on_device else 0, _p(foff), _p(n_frames), B, _p(prev),
                                   _p(toks), cap, _p(toff), _p(frs) if with_frames else None, C.byref(need)),
               "pk_ctc_greedy")
        out = [toks[toff[b]:toff[b + 1]].copy() for b in range(B)]
        fo = [frs[toff[b]:toff[b + 1]].copy() for b in range(B)] if with_frames else None
        return out, fo, prev


class Vocab:
    """SentencePiece BPE detokenizer (parakeet::detokenize, src/sentencepiece_bpe.cpp:9-37)
    with the vocabulary held on one GPU."""

    def __init__(self, pieces, blank_id=-1, bos_id=-1, eos_id=-1, pad_id=-1, device: int = 0):
        bs = [p.encode("utf-8") if isinstance(p, str) else bytes(p) for p in pieces]
        offs = np.zeros(len(bs) + 1, np.int64)
        offs[1:] = np.cumsum([len(b) for b in bs])
        buf = np.frombuffer(b"".join(bs) or b"\0", dtype=np.uint8).copy()
        h = C.c_void_p()
        _check(lib().pk_vocab_create(device, _p(buf), _p(offs), len(bs), blank_id, bos_id, eos_id, pad_id,
                                     C.byref(h)), "pk_vocab_create")
        self._h = h
        self.n = len(bs)

    def close(self):
        if getattr(self, "_h", None):
            lib().pk_vocab_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def detokenize(self, token_lists) -> list:
        """token_lists: sequences of int ids, one per utterance. Returns bytes per utterance."""
        B = len(token_lists)
        lens = [len(t) for t in token_lists]
        toff = np.zeros(B + 1, np.int64)
        toff[1:] = np.cumsum(lens)
        toks = np.ascontiguousarray(np.concatenate([np.asarray(t, np.int32) for t in token_lists])
                                    if sum(lens) else np.zeros(1, np.int32), dtype=np.int32)
        tof = np.zeros(B + 1, np.int64)
        need = C.c_int64(0)
        rc = lib().pk_detokenize(self._h, _p(toks), 0, _p(toff), B, None, 0, _p(tof), C.byref(need))
        if rc not in (0, 7):   # PK_ERR_CAPACITY: size query
            _check(rc, "pk_detokenize")
        cap = int(need.value)
        text = np.zeros(max(cap, 1), np.uint8)
        _check(lib().pk_detokenize(self._h, _p(toks), 0, _p(toff), B, _p(text), cap, _p(tof), C.byref(need)),
               "pk_detokenize")
        return [text[tof[b]:tof[b + 1]].tobytes() for b in range(B)]
