"""ctypes mirror of include/parakeet_cuda.h (the libparakeet_cuda C ABI)."""
from __future__ import annotations

import ctypes as C
from typing import List

import numpy as np

PK_OK, PK_ERR_DMODEL, PK_ERR_INVALID, PK_ERR_MODEL, PK_ERR_CUDA = 0, 1, 2, 3, 4
PK_ERR_OOM, PK_ERR_TIMEOUT, PK_ERR_CAPACITY, PK_ERR_NO_DEVICE, PK_ERR_DEVICE = 5, 6, 7, 8, 9
PK_MODEL_TDT, PK_MODEL_EOU = 1, 2
PK_OPT_TIMEOUT_US, PK_OPT_MATH, PK_OPT_MAX_SYMBOLS, PK_OPT_TEST_STALL, PK_OPT_BULK_MIN_LIVE = 1, 2, 3, 4, 5
PK_OPT_BULK_SCREEN, PK_OPT_BULK_I8, PK_OPT_BULK_TMA_A = 6, 7, 8
PK_MATH_F32, PK_MATH_TC, PK_MATH_Q8 = 0, 1, 2

STATUS_NAMES = {0: "PK_OK", 1: "PK_ERR_DMODEL", 2: "PK_ERR_INVALID", 3: "PK_ERR_MODEL",
                4: "PK_ERR_CUDA", 5: "PK_ERR_OOM", 6: "PK_ERR_TIMEOUT", 7: "PK_ERR_CAPACITY",
                8: "PK_ERR_NO_DEVICE", 9: "PK_ERR_DEVICE"}


class pk_tensor(C.Structure):
    _fields_ = [("data", C.c_void_p), ("type", C.c_int32), ("reserved", C.c_int32),
                ("ne0", C.c_int64), ("ne1", C.c_int64), ("nbytes", C.c_uint64)]


class pk_lstm_layer(C.Structure):
    _fields_ = [("w_ih", pk_tensor), ("w_hh", pk_tensor), ("b_ih", pk_tensor), ("b_hh", pk_tensor)]


class pk_model_desc(C.Structure):
    _fields_ = [("model_type", C.c_int32), ("d_enc", C.c_int32), ("pred_hidden", C.c_int32),
                ("joint_hidden", C.c_int32), ("n_layers", C.c_int32), ("vocab_size", C.c_int32),
                ("blank_id", C.c_int32), ("num_durations", C.c_int32),
                ("durations", C.POINTER(C.c_int32)), ("eou_id", C.c_int32), ("eob_id", C.c_int32),
                ("max_symbols_per_step", C.c_int32), ("n_vocab_pieces", C.c_int32),
                ("special_piece", C.POINTER(C.c_uint8)), ("embed", pk_tensor),
                ("lstm", C.POINTER(pk_lstm_layer)), ("joint_enc_w", pk_tensor),
                ("joint_enc_b", pk_tensor), ("joint_pred_w", pk_tensor),
                ("joint_pred_b", pk_tensor), ("joint_out_w", pk_tensor),
                ("joint_out_b", pk_tensor)]


class pk_info(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "model_type", "d_enc", "pred_hidden", "joint_hidden", "n_layers", "vocab_size",
        "blank_id", "num_durations", "v_plus_1", "v_out", "eou_id", "eob_id",
        "max_symbols_per_step", "device", "sm_count", "grid_ctas")] + [
        ("weight_bytes_device", C.c_uint64)]


class pk_batch(C.Structure):
    _fields_ = [("enc", C.c_void_p), ("enc_on_device", C.c_int32), ("B", C.c_int32),
                ("d_enc", C.c_int32), ("max_symbols_per_step", C.c_int32),
                ("frame_offsets", C.POINTER(C.c_int64)), ("n_frames", C.POINTER(C.c_int32)),
                ("prefetch_ticket", C.c_uint64)]


class pk_result(C.Structure):
    _fields_ = [("results_on_device", C.c_int32), ("tokens", C.c_void_p),
                ("tokens_cap", C.c_int64), ("token_offsets", C.c_void_p), ("steps", C.c_void_p),
                ("eou_bounds", C.c_void_p), ("eou_bounds_cap", C.c_int64),
                ("eou_offsets", C.c_void_p), ("finish_ms", C.c_void_p),
                ("tokens_needed", C.c_int64), ("eou_bounds_needed", C.c_int64),
                ("total_steps", C.c_int64), ("loop_iterations", C.c_int64),
                ("emit_iterations", C.c_int64), ("kernel_launches", C.c_int64),
                ("phase_ms", C.c_double * 8),
                ("encproj_ms", C.c_double), ("loop_ms", C.c_double), ("total_ms", C.c_double),
                ("bulk_ms", C.c_double), ("bulk_iterations", C.c_int64),
                ("bulk_phase_ms", C.c_double * 20),
                ("bulk_steps", C.c_int64), ("bulk_lstm_steps", C.c_int64),
                ("bulk_screened_steps", C.c_int64)]


class pk_trace(C.Structure):
    _fields_ = [("max_steps", C.c_int32), ("forced_token", C.c_void_p),
                ("forced_dur_idx", C.c_void_p), ("logits", C.c_void_p), ("h", C.c_void_p),
                ("c", C.c_void_p), ("argmax_token", C.c_void_p), ("argmax_dur_idx", C.c_void_p)]


class pk_stream_state(C.Structure):
    _fields_ = [("h", C.c_void_p), ("c", C.c_void_p), ("pred_out", C.c_void_p),
                ("symbols_this_step", C.c_int32), ("carry_frames", C.c_int32),
                ("initialized", C.c_int32), ("last_token", C.c_int32),
                ("segment_start_token", C.c_int32)]


# Every symbol include/parakeet_cuda.h declares (checked by the CPU test suite).
EXPORTED_SYMBOLS = [
    "pk_create", "pk_destroy", "pk_get_info", "pk_set_option", "pk_last_error",
    "pk_abi_version", "pk_decode_batch", "pk_tokens_capacity", "pk_decode_trace",
    "pk_stream_create", "pk_stream_destroy", "pk_stream_reset", "pk_stream_window",
    "pk_stream_get_state", "pk_stream_set_state", "pk_shard_lpt", "pk_decode_noalloc",
    "pk_ctc_create", "pk_ctc_destroy", "pk_ctc_greedy", "pk_vocab_create", "pk_vocab_destroy",
    "pk_detokenize", "pk_prefetch_batch", "pk_shard_balanced",
]


def _tensor(t) -> pk_tensor:
    return pk_tensor(C.c_void_p(t.data.ctypes.data), t.type, 0, t.ne0, t.ne1, t.nbytes)


class ModelDesc:
    """Owns a pk_model_desc built from a synth.DecoderModel (keeps buffers alive)."""

    def __init__(self, m):
        self.model = m
        p = m.prefix
        T = m.tensors
        self.layers = (pk_lstm_layer * m.n_layers)()
        for l in range(m.n_layers):
            self.layers[l] = pk_lstm_layer(_tensor(T[f"{p}.predict.lstm.{l}.w_ih"]),
                                           _tensor(T[f"{p}.predict.lstm.{l}.w_hh"]),
                                           _tensor(T[f"{p}.predict.lstm.{l}.b_ih"]),
                                           _tensor(T[f"{p}.predict.lstm.{l}.b_hh"]))
        self.durs = np.asarray(m.durations if m.durations else [0], dtype=np.int32)
        self.special = m.special_mask()
        d = pk_model_desc()
        d.model_type = PK_MODEL_TDT if m.model_type == "tdt" else PK_MODEL_EOU
        d.d_enc, d.pred_hidden, d.joint_hidden = m.d_enc, m.pred_hidden, m.joint_hidden
        d.n_layers, d.vocab_size, d.blank_id = m.n_layers, m.vocab_size, m.blank_id
        d.num_durations = len(m.durations) if m.model_type == "tdt" else 0
        d.durations = self.durs.ctypes.data_as(C.POINTER(C.c_int32))
        d.eou_id, d.eob_id = m.eou_id, m.eob_id
        d.max_symbols_per_step = m.max_symbols_per_step
        d.n_vocab_pieces = len(self.special)
        d.special_piece = self.special.ctypes.data_as(C.POINTER(C.c_uint8))
        d.embed = _tensor(T[f"{p}.predict.embed.weight"])
        d.lstm = C.cast(self.layers, C.POINTER(pk_lstm_layer))
        d.joint_enc_w = _tensor(T[f"{p}.joint.enc.weight"])
        d.joint_enc_b = _tensor(T[f"{p}.joint.enc.bias"])
        d.joint_pred_w = _tensor(T[f"{p}.joint.pred.weight"])
        d.joint_pred_b = _tensor(T[f"{p}.joint.pred.bias"])
        d.joint_out_w = _tensor(T[f"{p}.joint.out.weight"])
        d.joint_out_b = _tensor(T[f"{p}.joint.out.bias"])
        self.desc = d

    def ref(self):
        return C.byref(self.desc)
