"""Golden outputs of the REFERENCE's own decoder for whole benchmark configurations.

Runs src/parakeet_tdt.cpp / src/parakeet_eou.cpp as built unchanged into
oracle/_ref/libref_decoder.so (``make -C oracle ref``; the build needs the reference
tree, this script does not) on every utterance of each configuration below, with all
host threads, and writes tests/golden/full/<name>.npz:

  n_tok[B], steps[B]            tokens emitted and joint evaluations per utterance
  tok_hash[B] (uint64)          blake2b-64 of the utterance's int32 token ids (little endian)
  n_bnd[B], bnd_hash[B]         EOU segment boundaries, same hash (EOU configurations)
  tokens, tok_off (small configs only): the token ids themselves

The inputs are rebuilt from seeds by the same generators the GPU tests and bench.py
use (parakeet.cpp_b200/synth.py), so the GPU box needs only these few hundred KB.

  python tests/golden/make_full_golden.py [name ...]
"""
import hashlib
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))


def tok_hash(a) -> np.uint64:
    b = np.ascontiguousarray(a, dtype="<i4").tobytes()
    return np.frombuffer(hashlib.blake2b(b, digest_size=8).digest(), dtype="<u8")[0]


def config5_lengths(S):
    """Configuration 5's utterance lengths: log-normal, median 250 frames, sigma 0.8,
    clipped to [25, 3750], 4096 utterances."""
    return S.lengths_lognormal(4096, 250.0, 0.8, 25, 3750, seed=7)


def cases(pk):
    """name -> (model factory, (enc, offs, T) factory, keep full token arrays)."""
    S = pk.synth

    def c2():
        T = S.lengths_uniform(64, 60, 1875, seed=7)
        enc, offs = S.encoder_batch(T, 1024, seed=99)
        return enc, offs, T

    def c3():
        T = np.full(256, 50, np.int32)
        enc, offs = S.encoder_batch(T, 512, seed=99)
        return enc, offs, T

    def c4():
        B, TT, pool = 1024, 750, 16384
        enc = np.random.default_rng(99).standard_normal((pool, 1024), dtype=np.float32)
        offs = (np.arange(B, dtype=np.int64) * 613) % (pool - TT + 1)
        return enc, offs, np.full(B, TT, np.int32)

    def c5(ids=None):
        """ids: only these utterances' frames (each utterance's frames depend on its id
        alone); offsets then index the returned rows, in the order of ids."""
        T = config5_lengths(S)
        ids = np.arange(len(T)) if ids is None else np.asarray(ids)
        enc, offs = S.encoder_pooled(T[ids], ids, 1024, seed=99)
        return enc, offs, T[ids]

    return {
        "config2": (lambda: S.tdt_0_6b(seed=1234), c2, True),
        "config3": (lambda: S.eou_120m(seed=1234), c3, True),
        "config4_q8_0": (lambda: S.tdt_1_1b(seed=1234, wtype="q8_0"), c4, False),
        "config4_f16": (lambda: S.tdt_1_1b(seed=1234, wtype="f16"), c4, False),
        "config5_bias0": (lambda: S.tdt_0_6b(seed=1234, blank_bias=0.0), c5, False),
        "config5_bias2": (lambda: S.tdt_0_6b(seed=1234, blank_bias=2.0), c5, False),
        "config5_bias4": (lambda: S.tdt_0_6b(seed=1234, blank_bias=4.0), c5, False),
    }


def main(names):
    from conftest import load_oracle, load_pkg
    pk = load_pkg()
    orc = load_oracle()
    if not orc.ref_decoder_available():
        sys.exit("oracle/_ref/libref_decoder.so is missing: make -C oracle ref PARAKEET_REFERENCE_DIR=...")
    out_dir = os.path.join(HERE, "full")
    os.makedirs(out_dir, exist_ok=True)
    todo = cases(pk)
    for name in names or list(todo):
        mk_model, mk_input, keep = todo[name]
        t0 = time.time()
        m = mk_model()
        enc, offs, T = mk_input()
        ref = orc.Reference(m)
        r = ref.decode_batch(enc, offs, T)
        B = len(T)
        d = {"n_tok": np.array([len(x) for x in r["tokens"]], np.int32),
             "steps": np.asarray(r["steps"], np.int32),
             "tok_hash": np.array([tok_hash(x) for x in r["tokens"]], np.uint64)}
        if "bounds" in r:
            d["n_bnd"] = np.array([len(x) for x in r["bounds"]], np.int32)
            d["bnd_hash"] = np.array([tok_hash(x) for x in r["bounds"]], np.uint64)
        if keep:
            d["tokens"] = np.concatenate(r["tokens"]).astype(np.int32) if B else np.zeros(0, np.int32)
            d["tok_off"] = np.concatenate([[0], np.cumsum(d["n_tok"], dtype=np.int64)])
            if "bounds" in r:
                d["bounds"] = np.concatenate(r["bounds"]).astype(np.int32)
        np.savez_compressed(os.path.join(out_dir, f"{name}.npz"), **d)
        print(f"{name}: B={B} frames={int(T.sum())} tokens={int(d['n_tok'].sum())} "
              f"steps={int(d['steps'].sum())} ({time.time() - t0:.0f} s)", flush=True)


if __name__ == "__main__":
    main(sys.argv[1:])
