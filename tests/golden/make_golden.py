"""Generate the golden decoder fixtures in tests/golden/ (run: python tests/golden/make_golden.py).

Each fixture is a small random-init decoder written as a GGUF (the converter's
layout, via parakeet.cpp_b200/synth.py) plus seeded encoder outputs and the
greedy-decode results of an INDEPENDENT float64 numpy restatement of the
reference decoder written here (not the C++ oracle):

* TDT: tdt_init_state / tdt_decode_window / tdt_greedy_decode
  (src/parakeet_tdt.cpp:813-1005), including carry_frames across windows;
* EOU: eou_init_state / eou_decode_window (src/parakeet_eou.cpp:206-336),
  including <EOU> boundaries + state reset, <EOB> and "<...>" piece skips.

Weights are dequantized with gguf-py (the quantizer library the reference's
converter uses), so they are exact. Decisions are made on float64 logits; the
generator refuses a seed whose decision path has a top-2 margin below 1e-4, so
an f32 implementation must reproduce the token sequences exactly.
"""
import importlib.util
import json
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def load_synth():
    path = os.path.join(ROOT, "parakeet.cpp_b200", "synth.py")
    spec = importlib.util.spec_from_file_location("pk_synth_golden", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


class F64Decoder:
    def __init__(self, m, synth):
        self.m = m
        p = m.prefix
        W = {k: synth.dequantize(t).astype(np.float64) for k, t in m.tensors.items()}
        self.embed = W[f"{p}.predict.embed.weight"]
        self.lstm = [(W[f"{p}.predict.lstm.{l}.w_ih"], W[f"{p}.predict.lstm.{l}.w_hh"],
                      W[f"{p}.predict.lstm.{l}.b_ih"].reshape(-1), W[f"{p}.predict.lstm.{l}.b_hh"].reshape(-1))
                     for l in range(m.n_layers)]
        self.enc_w, self.enc_b = W[f"{p}.joint.enc.weight"], W[f"{p}.joint.enc.bias"].reshape(-1)
        self.pred_w, self.pred_b = W[f"{p}.joint.pred.weight"], W[f"{p}.joint.pred.bias"].reshape(-1)
        self.out_w, self.out_b = W[f"{p}.joint.out.weight"], W[f"{p}.joint.out.bias"].reshape(-1)
        self.H, self.L = m.pred_hidden, m.n_layers
        self.V1 = m.vocab_size + 1
        self.n_out = m.v_out if m.model_type == "tdt" else self.V1
        self.min_margin = math.inf

    def lstm_step(self, x, h, c):
        H = self.H
        for l, (wih, whh, bih, bhh) in enumerate(self.lstm):
            g = (wih @ x + bih) + bhh + whh @ h[l]
            sig = lambda v: 1.0 / (1.0 + np.exp(-v))
            i, f, gg, o = sig(g[:H]), sig(g[H:2 * H]), np.tanh(g[2 * H:3 * H]), sig(g[3 * H:])
            c[l] = f * c[l] + i * gg
            h[l] = o * np.tanh(c[l])
            x = h[l].copy()

    def joint(self, e, pred):
        hid = (self.enc_w @ e + self.enc_b) + (self.pred_w @ pred + self.pred_b)
        hid = np.maximum(hid, 0.0)
        return self.out_w @ hid + self.out_b

    def argmax(self, v):
        idx = int(np.argmax(v))              # first maximum, like the strict '>' scan
        if len(v) > 1:
            s = np.sort(v)
            self.min_margin = min(self.min_margin, float(s[-1] - s[-2]))
        return idx

    def new_state(self):
        return {"h": np.zeros((self.L, self.H)), "c": np.zeros((self.L, self.H)), "sym": 0,
                "carry": 0, "init": False, "seg": 0, "last": -1}

    def init_state(self, st):
        st["h"][:] = 0
        st["c"][:] = 0
        st.update(sym=0, carry=0, seg=0, last=-1)
        self.lstm_step(self.embed[self.m.blank_id], st["h"], st["c"])
        st["init"] = True

    def tdt_window(self, enc, st, msym, tokens):
        steps = 0
        T = enc.shape[0]
        if T <= 0:
            return 0
        if not st["init"]:
            self.init_state(st)
        t = 0
        if st["carry"] > 0:
            t = min(st["carry"], T)
            st["carry"] -= t
        V1, durs = self.V1, self.m.durations
        while t < T:
            lg = self.joint(enc[t], st["h"][-1])
            tok = self.argmax(lg[:V1])
            di = self.argmax(lg[V1:V1 + len(durs)])
            steps += 1
            dur = durs[di]
            if tok == self.m.blank_id:
                t += max(1, dur)
                st["sym"] = 0
                continue
            tokens.append(tok)
            self.lstm_step(self.embed[tok], st["h"], st["c"])
            st["sym"] += 1
            if dur > 0 or st["sym"] >= msym:
                t += max(1, dur)
                st["sym"] = 0
        st["carry"] = max(0, t - T)
        return steps

    def eou_window(self, enc, st, msym, tokens, bounds, special):
        if not st["init"]:
            self.init_state(st)
        m = self.m
        steps = 0
        msym = max(1, msym)
        for t in range(enc.shape[0]):
            st["sym"] = 0
            while st["sym"] < msym:
                lg = self.joint(enc[t], st["h"][-1])
                steps += 1
                best = self.argmax(lg[:self.V1])
                if best == m.blank_id or best == m.eob_id:
                    break
                if best == m.eou_id:
                    if len(tokens) > st["seg"]:
                        bounds.append(len(tokens))
                        st["seg"] = len(tokens)
                    st["h"][:] = 0
                    st["c"][:] = 0
                    st["last"] = m.blank_id
                    self.lstm_step(self.embed[m.blank_id], st["h"], st["c"])
                    break
                if best < len(special) and special[best]:
                    break
                tokens.append(best)
                self.lstm_step(self.embed[best], st["h"], st["c"])
                st["last"] = best
                st["sym"] += 1
        return steps


def bump_bias(m, updates):
    key = f"{m.prefix}.joint.out.bias"
    b = m.tensors[key].data.view(np.float32)
    for idx, v in updates.items():
        b[idx] += np.float32(v)


CASES = {
    "tdt_small": dict(kind="tdt", vocab=100, De=96, H=160, J=160, L=2, wtype="q8_0",
                      durations=[0, 1, 2, 3, 4], msym=10, bias=1.8, seed=11,
                      T=[37, 1, 0, 64, 23], windows=[10, 7, 1, 19]),
    "tdt_msym2": dict(kind="tdt", vocab=60, De=64, H=64, J=96, L=2, wtype="f16",
                      durations=[0, 2, 3], msym=2, bias=1.2, seed=12,
                      T=[30, 12], windows=[5, 5, 20]),
    "eou_small": dict(kind="eou", vocab=50, De=64, H=96, J=96, L=1, wtype="f16",
                      msym=5, bias=0.3, seed=13, eou=46, eob=47,
                      extra_bias={46: 1.2, 47: 0.6, 0: 0.6},
                      T=[40, 3, 0, 25], windows=[9, 0, 12, 19]),
}


def build_case(name, c, synth):
    if c["kind"] == "tdt":
        m = synth.make_decoder("tdt", vocab_size=c["vocab"], d_enc=c["De"], pred_hidden=c["H"],
                               joint_hidden=c["J"], n_layers=c["L"], durations=c["durations"],
                               wtype=c["wtype"], blank_bias=c["bias"], seed=c["seed"],
                               max_symbols_per_step=c["msym"])
    else:
        m = synth.make_decoder("eou", vocab_size=c["vocab"], d_enc=c["De"], pred_hidden=c["H"],
                               joint_hidden=c["J"], n_layers=c["L"], wtype=c["wtype"],
                               blank_bias=c["bias"], seed=c["seed"], eou_id=c["eou"],
                               eob_id=c["eob"], max_symbols_per_step=c["msym"])
        bump_bias(m, c.get("extra_bias", {}))
    return m


def run_case(name, c, synth):
    m = build_case(name, c, synth)
    dec = F64Decoder(m, synth)
    enc, offs = synth.encoder_batch(c["T"], c["De"], seed=c["seed"] + 1000)
    special = m.special_mask()
    toks, steps, bounds = [], [], []
    for b, T in enumerate(c["T"]):
        st = dec.new_state()
        tk, bd = [], []
        e = enc[offs[b]:offs[b] + T]
        if c["kind"] == "tdt":
            s = dec.tdt_window(e, st, c["msym"], tk)
        else:
            s = dec.eou_window(e, st, c["msym"], tk, bd, special)
        toks.append(tk); steps.append(s); bounds.append(bd)
    # windowed decode of utterance 0 (Mode 2 streaming): one state across windows
    st = dec.new_state()
    wtok, wsteps, wbounds = [], [], []
    e0 = enc[offs[0]:offs[0] + c["T"][0]]
    pos = 0
    for w in c["windows"]:
        e = e0[pos:pos + w]
        pos += w
        tk, bd = [], []
        if c["kind"] == "tdt":
            s = dec.tdt_window(e, st, c["msym"], tk)
        else:
            # the reference's out_tokens keeps growing across windows in the caller
            run = [0] * len(sum(wtok, []))
            run_tokens = list(run)
            s = dec.eou_window(e, st, c["msym"], run_tokens, bd, special)
            tk = run_tokens[len(run):]
        wtok.append(tk); wsteps.append(s); wbounds.append(bd)
    assert pos == c["T"][0], name
    if dec.min_margin < 1e-4:
        raise SystemExit(f"{name}: decision margin {dec.min_margin:.2e} < 1e-4; pick another seed")
    return m, enc, offs, toks, steps, bounds, wtok, wsteps, wbounds, dec.min_margin


def main():
    synth = load_synth()
    manifest = {}
    for name, c in CASES.items():
        m, enc, offs, toks, steps, bounds, wtok, wsteps, wbounds, mm = run_case(name, c, synth)
        synth.write_gguf(m, os.path.join(HERE, f"{name}.gguf"))
        flat = lambda lists: np.asarray(sum(lists, []), np.int32)
        lens = lambda lists: np.asarray([len(x) for x in lists], np.int32)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"),
                            enc=enc, offsets=offs, n_frames=np.asarray(c["T"], np.int32),
                            tokens=flat(toks), token_counts=lens(toks),
                            steps=np.asarray(steps, np.int32),
                            bounds=flat(bounds), bound_counts=lens(bounds),
                            windows=np.asarray(c["windows"], np.int32),
                            win_tokens=flat(wtok), win_token_counts=lens(wtok),
                            win_steps=np.asarray(wsteps, np.int32),
                            win_bounds=flat(wbounds), win_bound_counts=lens(wbounds),
                            max_symbols=np.int32(c["msym"]))
        manifest[name] = {"tokens": [len(t) for t in toks], "steps": steps,
                          "bounds": [len(b) for b in bounds], "min_margin": mm,
                          "config": {k: v for k, v in c.items() if k != "extra_bias"}}
        print(name, manifest[name]["tokens"], steps, [len(b) for b in bounds], f"margin {mm:.3g}")
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    sys.exit(main())
