#!/usr/bin/env python
"""Throughput of the TDT/RNN-T greedy token loop on B200 (libparakeet_cuda).

One "step" is one pk_decode_batch call over the configuration's batch of
synthetic encoder outputs (random-init decoder weights of the named geometry):
enc-proj GEMM, the persistent step-loop kernel, token compaction.

  value : emitted tokens/s with encoder outputs resident in HBM and results left
          on the device; time = sum over the K timed calls of the library's
          CUDA-event time on its launching stream (max over ranks).
  e2e   : the same metric through the public calls with pinned HOST encoder
          outputs and HOST results, every step's copies inside the timed region:
          each step's encoder copy is prefetched (pk_prefetch_batch) while the
          previous step decodes; time = host wall clock around the K calls.
          e2e.serial: one call at a time, its copies inside the call.

Default workload: benchmark configuration 5, TDT-0.6b-v3 q8_0, a global batch of
4096 utterances with log-normal lengths (median 250 frames, sigma 0.8, clipped to
[25, 3750]), blank bias +2. With N GPUs (torchrun, one rank per GPU) each rank
decodes its shard of the same 4096 utterances (pk_shard_balanced: the longest
utterances share shards and every shard's modelled decode time is bounded;
--shard lpt for the frame-count LPT partition;
strong scaling: N = 8 is the stated 4096-over-8 case; no collective on the
decode path). Configurations 1-4
keep their per-GPU batch (weak scaling).

--impl reference times the reference's own CPU decoder (src/parakeet_tdt.cpp /
src/parakeet_eou.cpp compiled unchanged into oracle/_ref/libref_decoder.so
against a host-only ggml stand-in; the oracle restatement when that library is
absent) on all host cores.
"""
import argparse
import importlib.util
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "parakeet.cpp_b200")

CONFIGS = {
    "1": dict(model="tdt_0_6b", wtype="q8_0", B=1, lengths=("const", 125), blank_bias=2.0,
              desc="TDT-0.6b-v3 q8_0, B=1, T=125"),
    "2": dict(model="tdt_0_6b", wtype="q8_0", B=64, lengths=("uniform", 60, 1875), blank_bias=2.0,
              desc="TDT-0.6b-v3 q8_0, B=64, T~U[60,1875]"),
    "3": dict(model="eou_120m", wtype="f16", B=256, lengths=("const", 50), blank_bias=2.0,
              desc="EOU-120m f16, B=256, T=50"),
    "4": dict(model="tdt_1_1b", wtype="q8_0", B=1024, lengths=("const", 750), blank_bias=2.0,
              desc="TDT-1.1b, B=1024, T=750"),
    "5": dict(model="tdt_0_6b", wtype="q8_0", B=4096, lengths=("lognormal",), blank_bias=2.0, global_batch=True,
              desc="TDT-0.6b-v3 q8_0, global batch 4096 split over the GPUs, T lognormal(250, 0.8) in [25, 3750]"),
}
DEFAULT_CONFIG = "5"
METRIC = "tdt_greedy_decode_tokens_per_sec"
# What the default (tensor-core) step loops compute in, by weight type: exact weights;
# in the persistent loop h as int16 fixed point in two int8 digits for the q8_0 LSTM /
# pred-proj (int8 MMA, int32 per 32-wide block, f32 block scale) and the joint hidden
# layer as f16 hi + lo (22 significant bits); in the bulk loop activations and q8_0
# weights as f16 hi + lo (three tcgen05 products), the joint of large iterations
# screened by one f16 product with the candidates recomputed in f32; f32 accumulation
# and state.
DTYPE = {"q8_0": "q8_0 weights; activations as int16 fixed point (int8 MMA) or f16 hi+lo (f16 MMA, 22 bits); "
                 "screened joint: 1 f16 product + f32 recomputation of candidates; f32 accumulate",
         "f16": "f16 weights; f16 hi+lo activations; f32 accumulate",
         "f32": "f32",
         "q8": "q8_0 weights x q8_0-quantised activations (int8 MMA per 32-block, both scales; ggml "
               "vec_dot_q8_0_q8_0); f32 accumulate"}


def load(name, path, pkg_dir=None):
    if name in sys.modules:
        return sys.modules[name]
    kw = {"submodule_search_locations": [pkg_dir]} if pkg_dir else {}
    spec = importlib.util.spec_from_file_location(name, path, **kw)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pkg():
    return load("parakeet_b200", os.path.join(PKG_DIR, "__init__.py"), PKG_DIR)


def oracle_mod():
    pkg()
    return load("pk_oracle", os.path.join(ROOT, "oracle", "oracle.py"))


def make_model(pk, cfg, wtype, blank_bias):
    fn = getattr(pk.synth, cfg["model"])
    return fn(seed=1234, wtype=wtype, blank_bias=blank_bias)


def global_lengths(pk, cfg, B_total):
    kind = cfg["lengths"]
    if kind[0] == "const":
        return np.full(B_total, kind[1], np.int32)
    if kind[0] == "uniform":
        return pk.synth.lengths_uniform(B_total, kind[1], kind[2], seed=7)
    return pk.synth.lengths_lognormal(B_total, 250.0, 0.8, 25, 3750, seed=7)


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ---------------------------------------------------------------- clocks ----

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region.
    start() returns once the first sample is in, so that a timed region shorter than the
    sampling period still has one (taken as it begins)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.perf_counter()
            while not self.lines and self.proc.poll() is None and time.perf_counter() - t0 < 3.0:
                time.sleep(0.01)
        except Exception:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ CPU legs ----

def cpu_sample_run(orc_o, enc, offs, T, threads, budget_s, msym=None):
    """The reference CPU decoder on a bounded sample: the batch's first utterances,
    whole, as many as about budget_s of work on `threads` threads takes (each
    utterance truncated only if one alone would exceed that)."""
    # calibrate: one utterance of up to 40 frames
    t40 = int(min(40, max(1, T[0])))
    t0 = time.perf_counter()
    orc_o.decode_window(enc[int(offs[0]):int(offs[0]) + t40], max_symbols=msym)
    per_frame = max((time.perf_counter() - t0) / t40, 1e-5)
    frames_budget = budget_s * threads / per_frame
    cap = int(max(10, min(int(np.max(T)), frames_budget / max(1, threads))))
    Ts = np.maximum(np.minimum(T, cap), 1).astype(np.int32)
    n_utt = int(np.searchsorted(np.cumsum(Ts.astype(np.int64)), frames_budget)) + 1
    n_utt = int(min(len(T), max(threads, n_utt)))
    Ts = Ts[:n_utt]
    t0 = time.perf_counter()
    r = orc_o.decode_batch(enc, offs[:n_utt], Ts, n_threads=threads, max_symbols=msym)
    wall = time.perf_counter() - t0
    ntok = int(sum(len(x) for x in r["tokens"]))
    nsteps = int(np.sum(r["steps"]))
    return {"tokens": ntok, "steps": nsteps, "wall_s": wall, "n_utt": n_utt, "cap": cap,
            "frames": int(Ts.sum()), "p50_ms": float(np.median(r["ms"]))}


# ------------------------------------------------------------ helpers ----

def bulk_flops(model, layer0_table=True):
    """FLOPs of the tcgen05 bulk loop's matrix products: per joint evaluation (one live
    utterance in one iteration) the joint.out product 2 * joint_hidden * v_out; per
    LSTM step (an emission or an utterance's first step) the gate products of every
    layer, 2 * 4H * (in + H) with in = H (the lower layer's h), and the pred projection
    2 * joint_hidden * H. Layer 0's input projection W_ih0 . embed is a per-token table
    lookup on the int8 path (layer0_table: not counted, in = 0 for layer 0), a product
    of the embedding on the f16 path. Returns (per joint evaluation, per LSTM step)."""
    H, J = model.pred_hidden, model.joint_hidden
    joint = 2 * J * model.v_out
    lstm = model.n_layers * 2 * 4 * H * (H + H) + 2 * J * H
    if layer0_table:
        lstm -= 2 * 4 * H * H
    return joint, lstm


def profiled_traffic(config_key):
    """dram bytes per joint evaluation of the bulk-loop kernel from the committed ncu
    summary (profiles/bulk_loop_kernel_config<k>.md), or None."""
    path = os.path.join(ROOT, "profiles", f"bulk_loop_kernel_config{config_key}.md")
    if not os.path.exists(path):
        return None
    m = re.search(r"dram_bytes_per_joint_evaluation:\s*([0-9.eE+]+)", open(path).read())
    return float(m.group(1)) if m else None


def read_peaks(kind="hbm"):
    """(peak, "measured" | "fallback"): HBM copy GB/s, or the sustained cuBLAS bf16
    TFLOP/s (the bulk loop runs for a large part of every step, back to back)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return (float(d["hbm_gbs"]) if kind == "hbm" else float(d["bf16_tflops_sustained"])), "measured"
    return (6650.0 if kind == "hbm" else 1400.0), "fallback"


# ------------------------------------------------------------------ main ----

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default=DEFAULT_CONFIG, choices=sorted(CONFIGS))
    ap.add_argument("--wtype", default=None)
    ap.add_argument("--blank-bias", type=float, default=None)
    ap.add_argument("--batch", type=int, default=None,
                    help="override the batch (global for configuration 5, per GPU otherwise)")
    ap.add_argument("--bulk-min-live", type=int, default=None,
                    help="PK_OPT_BULK_MIN_LIVE: live utterances from which iterations run on the tcgen05 "
                         "bulk loop (library default when absent; 0 = never)")
    ap.add_argument("--no-screen", action="store_true",
                    help="PK_OPT_BULK_SCREEN = 0: the bulk loop's joint always takes three f16 products per "
                         "logit, never one screening product and the f32 recomputation of the candidates")
    ap.add_argument("--no-i8", action="store_true",
                    help="PK_OPT_BULK_I8 = 0: the bulk loop's LSTM and pred-proj on f16 hi/lo halves "
                         "(kind::f16) instead of int8 digits (kind::i8)")
    ap.add_argument("--math", default=None, choices=["tc", "q8", "f32"],
                    help="PK_OPT_MATH (library default when absent: tc); q8 = the optional q8_0-activation "
                         "mode (ggml's vec_dot_q8_0_q8_0 arithmetic, persistent loop only)")
    ap.add_argument("--shard", default="balanced", choices=["balanced", "lpt"],
                    help="partition of the utterances over ranks (N > 1)")
    ap.add_argument("--emulate-ranks", type=int, default=0,
                    help="one GPU: decode each of the N shards of the global batch alone and report "
                         "the slowest shard's call time (the N-GPU step time, since ranks share nothing)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget-s", type=float, default=12.0)
    ap.add_argument("--path", default="tdt", choices=["tdt", "ctc"],
                    help="tdt: the token loop (the headline); ctc: CTC greedy decode beside it (1 GPU)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 0)
    if args.path == "ctc":
        return run_ctc(args)
    if args.emulate_ranks > 0:
        return run_emulated_ranks(args)

    cfg = dict(CONFIGS[args.config])
    wtype = args.wtype or cfg["wtype"]
    blank_bias = cfg["blank_bias"] if args.blank_bias is None else args.blank_bias
    B = args.batch or cfg["B"]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    pk = pkg()
    model = make_model(pk, cfg, wtype, blank_bias)
    strong = bool(cfg.get("global_batch"))
    B_total = B if strong else B * world
    T_all = global_lengths(pk, cfg, B_total)
    idx = pk.multi.shard_indices(T_all, world, args.shard)[rank] if world > 1 else np.arange(B_total)
    shard_sizes = [int(len(x)) for x in pk.multi.shard_indices(T_all, world, args.shard)] if world > 1 else [B_total]
    if args.impl == "reference":
        # the CPU arm (rank 0 alone) decodes a bounded sample of the batch's first
        # utterances, whatever the rank count
        idx = (np.arange(B_total) if strong else idx)[:64 * host_cores()]
    T = T_all[idx].astype(np.int32)
    if strong:
        # every utterance has the same frames whichever rank decodes it
        enc, offs = pk.synth.encoder_pooled(T, idx, model.d_enc, seed=99)
    else:
        enc, offs = pk.synth.encoder_batch(T, model.d_enc, seed=99 + rank)
    config = {"workload": cfg["desc"] + (f" (wtype {wtype})" if wtype != cfg["wtype"] else ""),
              "config": args.config, "utterances_per_gpu": shard_sizes if world > 1 else int(len(T)),
              "global_batch": int(B_total),
              "frames_per_gpu": int(T.sum()), "frames_global": int(T_all.sum()), "blank_bias": blank_bias,
              "l2": f"inputs {enc.nbytes / 1e6:.0f} MB of encoder output per step (L2 is 126 MB)",
              "parallelism": f"utterance shards x{world} ({args.shard})" if world > 1 else "single GPU"}
    args.scaling = "strong" if strong else "weak"

    if args.impl == "reference":
        return run_reference(args, model, enc, offs, T, config, rank)
    return run_ours(args, pk, model, enc, offs, T, config, world, rank, local_rank, wtype, idx)


def run_emulated_ranks(args):
    """Strong scaling of a global batch over N ranks, emulated on one GPU: each rank's
    shard (--shard) decoded alone with device-resident input, W warm-up and K timed calls
    per shard (the library's CUDA events); the slowest shard's call time is the N-GPU
    step time, since ranks share no data and no collective. Prints one JSON line
    (not the bench contract's line: a measurement aid for the partition)."""
    import torch
    pk = pkg()
    cfg = dict(CONFIGS[args.config])
    if not cfg.get("global_batch"):
        print(json.dumps({"emulate_ranks": args.emulate_ranks, "unavailable": "configuration has no global batch"}))
        return 0
    wtype = args.wtype or cfg["wtype"]
    blank_bias = cfg["blank_bias"] if args.blank_bias is None else args.blank_bias
    model = make_model(pk, cfg, wtype, blank_bias)
    B_total = args.batch or cfg["B"]
    T_all = global_lengths(pk, cfg, B_total)
    shards = pk.multi.shard_indices(T_all, args.emulate_ranks, args.shard) if args.emulate_ranks > 1 \
        else [np.arange(B_total)]
    dec = pk.Decoder(model, bulk_min_live=args.bulk_min_live, math=args.math)
    times, tokens = [], 0
    for idx in shards:
        T = T_all[idx].astype(np.int32)
        enc, offs = pk.synth.encoder_pooled(T, idx, model.d_enc, seed=99)
        ed = torch.from_numpy(enc).cuda()
        torch.cuda.synchronize()
        for _ in range(args.warmup):
            dec.decode_batch(ed.data_ptr(), offs, T, enc_on_device=True)
        rs = [dec.decode_batch(ed.data_ptr(), offs, T, enc_on_device=True) for _ in range(max(1, args.steps))]
        times.append(float(np.median([r["total_ms"] for r in rs])))
        tokens += sum(len(t) for t in rs[0]["tokens"])
        del ed
    dec.close()
    slow = max(times)
    print(json.dumps({"emulate_ranks": args.emulate_ranks, "shard": args.shard, "metric": METRIC,
                      "value": tokens / (slow / 1e3), "unit": "tokens/s", "ms_per_step": slow,
                      "shard_ms": [round(t, 3) for t in times], "shard_sizes": [int(len(i)) for i in shards],
                      "config": {"workload": cfg["desc"], "global_batch": int(B_total)},
                      "timing": "each shard alone on one GPU, median of K calls (CUDA events), slowest shard"}))
    return 0


def run_ctc(args):
    """CTC greedy decode (pk_ctc_greedy, src/parakeet_ctc.cpp:1820-1865) over a config-2 sized batch
    of synthetic CTC logits (V = 1025: 1024 pieces + blank, N(0,1) with the blank raised by 2,
    mostly-blank frames as a CTC head gives): frames/s device-resident and end to end, the HBM
    roofline of reading the logits, and the oracle on one host thread. One GPU."""
    import torch
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"path": "ctc", "unavailable": "the CTC measurement runs on one GPU"}))
        return 0
    pk = pkg()
    cfg = CONFIGS[args.config]
    B = args.batch or cfg["B"]
    T = global_lengths(pk, cfg, B).astype(np.int32)
    offs = np.zeros(B, np.int64)
    offs[1:] = np.cumsum(T[:-1])
    F, V, blank = int(T.sum()), 1025, 1024
    g = torch.Generator(device="cuda").manual_seed(7)
    logits = torch.randn(F, V, device="cuda", generator=g)
    logits[:, blank] += 2.0
    host = logits.cpu().pin_memory()
    ctc = pk.CtcGreedy(V, blank)
    for _ in range(max(args.warmup, 3)):
        ctc.decode(logits.data_ptr(), offs, T, on_device=True)
    clocks = ClockSampler(0)
    clocks.start()
    ms = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        toks, _, _ = ctc.decode(logits.data_ptr(), offs, T, on_device=True)
        e1.record()
        torch.cuda.synchronize()
        ms.append(e0.elapsed_time(e1))
    clk = clocks.stop()
    ms_e2e = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        toks_h, _, _ = ctc.decode(host.numpy(), offs, T)
        e1.record()
        torch.cuda.synchronize()
        ms_e2e.append(e0.elapsed_time(e1))
    same = all(np.array_equal(a, b) for a, b in zip(toks, toks_h))
    t = float(np.mean(ms))
    peak, peak_kind = read_peaks()
    achieved = F * V * 4 / (t * 1e-3) / 1e9
    cpu = None
    if not args.no_cpu_baseline:
        orc = oracle_mod()
        L = host.numpy()
        n = fr = 0
        t0 = time.perf_counter()
        while n < B and time.perf_counter() - t0 < min(args.cpu_budget_s, 20.0):
            orc.ctc_greedy_window(L[offs[n]:offs[n] + T[n]], blank, -1)
            fr += int(T[n])
            n += 1
        wall = time.perf_counter() - t0
        cpu = {"value": fr / wall, "unit": "frames/s", "cores": 1, "kind": "port",
               "sample": f"first {n} utterances of the batch ({fr} frames), orc_ctc_greedy_window on one thread"}
    print(json.dumps({
        "path": "ctc", "metric": "ctc_greedy_frames_per_sec", "value": F / (t * 1e-3), "unit": "frames/s",
        "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": t,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic N(0,1) logits, blank raised by 2", "config": {
            "workload": f"CTC greedy, B={B} utterances of config-{args.config} lengths, V={V}",
            "frames": F, "l2": f"logits {F * V * 4 / 1e6:.0f} MB per step (L2 is 126 MB)"},
        "tokens_per_step": int(sum(len(x) for x in toks)), "clocks": clk,
        "e2e": {"value": F / (float(np.mean(ms_e2e)) * 1e-3), "unit": "frames/s",
                "h2d_bytes_per_step": F * V * 4, "d2h_bytes_per_step": int(sum(len(x) for x in toks)) * 4 + (B + 1) * 8,
                "tokens_match_device_run": same},
        "gpu_launches": 4 * args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "kernel": "ctc_argmax_kernel (+ collapse / scan / gather in the same call)",
                     "note": f"algorithmic bytes = logits read once (4 B x V per frame); time = the whole call "
                             f"(host synchronisations included); peak {peak_kind}"},
        "cpu_baseline": cpu,
    }))
    return 0


def cpu_model():
    """Host CPU model name (lscpu), or None."""
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for ln in out.splitlines():
            if ln.startswith("Model name:"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return None


def reference_decoder(model):
    """The reference's own CPU decoder (oracle/_ref/libref_decoder.so, built from the
    reference's sources) when present, else the oracle restatement: (decoder, kind)."""
    orc = oracle_mod()
    if orc.ref_decoder_available():
        return orc.Reference(model), "reference"
    return orc.Oracle(model), "port"


def run_reference(args, model, enc, offs, T, config, rank):
    if rank != 0:
        return 0
    o, kind = reference_decoder(model)
    threads = host_cores()
    budget = max(1.0, 150.0 / max(1, args.steps + min(args.warmup, 1)))
    for _ in range(min(args.warmup, 1)):
        cpu_sample_run(o, enc, offs, T, threads, min(budget, 2.0))
    toks = steps = 0
    wall = 0.0
    last = None
    for _ in range(args.steps):
        last = cpu_sample_run(o, enc, offs, T, threads, budget)
        toks += last["tokens"]
        steps += last["steps"]
        wall += last["wall_s"]
    v = toks / wall if wall > 0 else 0.0
    what = ("the reference's tdt_greedy_decode / eou_greedy_decode (src/parakeet_tdt.cpp, src/parakeet_eou.cpp "
            "built unchanged with -O3 -ffast-math -funroll-loops)" if kind == "reference" else
            "the oracle restatement of the reference's CPU decoder")
    sample = (f"first {last['n_utt']} utterances of the batch, each truncated to {last['cap']} "
              f"frames ({last['frames']} frames), one utterance per thread, {what}")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "runs_on": "host CPU cores (rank 0)",
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * wall / max(1, args.steps),
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init weights, N(0,1) encoder outputs)", "config": config,
        "steps_per_sec": steps / wall if wall > 0 else 0.0,
        "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": kind,
                         "cpu_model": cpu_model(), "sample": sample},
        "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))
    return 0


def reference_parity(args, model, tok_host, off_host, steps_host, idx):
    """Per-utterance comparison of a host result with the reference fixture of this
    workload, when one exists (configuration 5 at blank bias 0 / 2 / 4, configuration 2)."""
    import hashlib
    cfg = args.config
    bias = args.blank_bias if args.blank_bias is not None else CONFIGS[cfg]["blank_bias"]
    name = {"5": f"config5_bias{int(bias)}" if float(bias) in (0.0, 2.0, 4.0) else None,
            "2": "config2" if float(bias) == 2.0 else None}.get(cfg)
    if name is None or (args.batch is not None and args.batch != CONFIGS[cfg]["B"]) or args.wtype not in (None, "q8_0"):
        return None
    path = os.path.join(ROOT, "tests", "golden", "full", f"{name}.npz")
    if not os.path.exists(path):
        return None
    fx = np.load(path)
    same = 0
    for i, u in enumerate(idx):
        t = tok_host[int(off_host[i]):int(off_host[i + 1])]
        h = np.frombuffer(hashlib.blake2b(np.ascontiguousarray(t, dtype="<i4").tobytes(), digest_size=8).digest(),
                          dtype="<u8")[0]
        same += int(len(t) == fx["n_tok"][u] and steps_host[i] == fx["steps"][u] and h == fx["tok_hash"][u])
    return {"fixture": os.path.relpath(path, ROOT), "identical": same, "checked": len(idx)}


def run_ours(args, pk, model, enc, offs, T, config, world, rank, local_rank, wtype, idx):
    import ctypes as C
    import torch
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    torch.cuda.set_device(local_rank)
    dec = pk.Decoder(model, device=local_rank, bulk_min_live=args.bulk_min_live, math=args.math)
    if args.no_screen:
        dec.set_option(pk.abi.PK_OPT_BULK_SCREEN, 0)
    if args.no_i8:
        dec.set_option(pk.abi.PK_OPT_BULK_I8, 0)
    msym = dec.info.max_symbols_per_step
    Bn = len(T)
    cap = int(pk.lib().pk_tokens_capacity(T.ctypes.data, Bn, msym))
    # device-resident inputs / outputs for the value path
    enc_pin = torch.from_numpy(enc).pin_memory()
    enc_dev = enc_pin.to(f"cuda:{local_rank}")
    tok_dev = torch.empty(max(cap, 1), dtype=torch.int32, device=enc_dev.device)
    off_dev = torch.empty(Bn + 1, dtype=torch.int64, device=enc_dev.device)
    steps_dev = torch.empty(max(Bn, 1), dtype=torch.int32, device=enc_dev.device)
    fin = np.zeros(max(Bn, 1), np.float32)
    torch.cuda.synchronize()
    batch_dev, keep_dev = dec.make_batch(enc_dev.data_ptr(), offs, T, enc_on_device=True)
    batch_host, keep_host = dec.make_batch(enc_pin.numpy(), offs, T)

    def res_dev():
        r = pk.abi.pk_result()
        r.results_on_device = 1
        r.tokens, r.tokens_cap = C.c_void_p(tok_dev.data_ptr()), cap
        r.token_offsets, r.steps = C.c_void_p(off_dev.data_ptr()), C.c_void_p(steps_dev.data_ptr())
        r.finish_ms = C.c_void_p(fin.ctypes.data)
        return r

    tok_host = np.zeros(max(cap, 1), np.int32)
    off_host = np.zeros(Bn + 1, np.int64)
    steps_host = np.zeros(max(Bn, 1), np.int32)
    tok_host_t = torch.from_numpy(tok_host)

    def res_host():
        r = pk.abi.pk_result()
        r.tokens, r.tokens_cap = C.c_void_p(tok_host.ctypes.data), cap
        r.token_offsets, r.steps = C.c_void_p(off_host.ctypes.data), C.c_void_p(steps_host.ctypes.data)
        return r

    def call(batch, res):
        rc = dec.decode_batch_raw(batch, res)
        if rc != 0:
            raise pk.PkError(rc, "pk_decode_batch", pk.last_error())
        return res

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        call(batch_dev, res_dev())
    # ---- value: device-resident inputs ----
    clocks = ClockSampler(local_rank)
    barrier()
    clocks.start()
    t_wall = time.perf_counter()
    tot_ms = loop_ms = enc_ms = 0.0
    tokens = steps = iters = emit_iters = launches = 0
    bulk_ms = 0.0
    bulk_steps = bulk_lstm = bulk_iters = bulk_scr = 0
    phase = np.zeros(8)
    lat = None
    for _ in range(args.steps):
        r = call(batch_dev, res_dev())
        tot_ms += r.total_ms
        loop_ms += r.loop_ms
        enc_ms += r.encproj_ms
        tokens += r.tokens_needed
        steps += r.total_steps
        iters += r.loop_iterations
        emit_iters += r.emit_iterations
        launches += r.kernel_launches
        phase += np.array(r.phase_ms[:], np.float64)
        bulk_ms += r.bulk_ms
        bulk_steps += r.bulk_steps
        bulk_lstm += r.bulk_lstm_steps
        bulk_scr += r.bulk_screened_steps
        bulk_iters += r.bulk_iterations
        lat = r.encproj_ms + fin[:Bn].astype(np.float64)
    barrier()
    wall_s = time.perf_counter() - t_wall
    clk = clocks.stop()
    # ---- e2e: host buffers through the public calls, pipelined: the next step's
    # encoder copy (pk_prefetch_batch, on the library's copy stream) overlaps this
    # step's decode. Time = host wall clock around the K synchronous decode calls
    # (every copy in and out inside it), max over ranks. ----
    def prefetch(batch):
        rc, ticket = dec.prefetch_raw(batch)
        if rc != 0:
            raise pk.PkError(rc, "pk_prefetch_batch", pk.last_error())
        return ticket

    def call_staged(ticket):
        batch_host.prefetch_ticket = ticket
        try:
            return call(batch_host, res_host())
        finally:
            batch_host.prefetch_ticket = 0

    # untimed: the host-input paths once each, so that their device buffers (two
    # prefetch slots, the in-call copy's buffer) exist before timing, as in a server
    staged = [prefetch(batch_host), prefetch(batch_host)]
    call_staged(staged[0])
    call_staged(staged[1])
    call(batch_host, res_host())
    barrier()
    e2e_tokens = 0
    t_e2e = time.perf_counter()
    staged = [prefetch(batch_host)]
    for k in range(args.steps):
        if k + 1 < args.steps:
            staged.append(prefetch(batch_host))
        r = call_staged(staged.pop(0))
        e2e_tokens += r.tokens_needed
    e2e_ms = (time.perf_counter() - t_e2e) * 1e3
    barrier()
    # ---- e2e, one call at a time: the copy inside each call (the library's CUDA events) ----
    ser_ms = 0.0
    ser_tokens = 0
    for _ in range(args.steps):
        r = call(batch_host, res_host())
        ser_ms += r.total_ms
        ser_tokens += r.tokens_needed
    barrier()
    same = bool(np.array_equal(tok_host[:int(off_host[-1])], tok_dev[:int(off_host[-1])].cpu().numpy()))
    # parity: every utterance of this rank against the reference decoder's own output on
    # the same inputs (tests/golden/full, made by tests/golden/make_full_golden.py)
    par = reference_parity(args, model, tok_host, off_host, steps_host, idx)

    # Kernel figures come from one rank's launches: shards differ widely in size (the
    # balanced partition), so the roofline is taken on the rank with the most bulk-loop
    # time and the loop figures on the rank with the longest call; copy bytes add up.
    h2d = int(enc.nbytes)
    d2h = int(tokens / max(1, args.steps)) * 4 + (Bn + 1) * 8 + Bn * 4
    kern = torch.tensor([bulk_ms, float(bulk_steps), float(bulk_lstm), float(bulk_scr), float(bulk_iters),
                         loop_ms, float(iters), tot_ms, enc_ms, float(h2d), float(d2h), float(launches)]
                        + [float(x) for x in phase], dtype=torch.float64, device=enc_dev.device)
    if dist is not None:
        rows = [torch.zeros_like(kern) for _ in range(world)]
        dist.all_gather(rows, kern)
        rows = torch.stack(rows).cpu().numpy()
        rb, rp = int(np.argmax(rows[:, 0])), int(np.argmax(rows[:, 7]))
        bulk_ms, bulk_steps, bulk_lstm, bulk_scr, bulk_iters = rows[rb, 0], int(rows[rb, 1]), int(rows[rb, 2]), \
            int(rows[rb, 3]), int(rows[rb, 4])
        loop_ms, iters, enc_ms, launches = rows[rp, 5], int(rows[rp, 6]), rows[rp, 8], int(rows[rp, 11])
        phase = rows[rp, 12:].astype(np.float64)
        pl_bulk_ms, pl_bulk_iters = rows[rp, 0], int(rows[rp, 4])
        h2d, d2h = int(rows[:, 9].sum()), int(rows[:, 10].sum())
    else:
        pl_bulk_ms, pl_bulk_iters = bulk_ms, bulk_iters
    stats = torch.tensor([tot_ms, loop_ms, e2e_ms, ser_ms, float(tokens), float(steps), float(e2e_tokens),
                          float(ser_tokens), float(par["identical"] if par else 0), float(par["checked"] if par else 0)],
                         dtype=torch.float64, device=enc_dev.device)
    if dist is not None:
        mx = stats.clone()
        dist.all_reduce(mx[:4], op=dist.ReduceOp.MAX)
        sm = stats.clone()
        dist.all_reduce(sm[4:], op=dist.ReduceOp.SUM)
        stats = torch.cat([mx[:4], sm[4:]])
    (tot_ms, loop_ms_max, e2e_ms, ser_ms, tokens_all, steps_all, e2e_tokens_all,
     ser_tokens_all, par_same, par_checked) = [float(x) for x in stats.cpu()]

    result = None
    if rank == 0:
        value = tokens_all / (tot_ms / 1e3) if tot_ms > 0 else 0.0
        fj, fl = bulk_flops(model, layer0_table=not args.no_i8)
        alg_flops = fj * bulk_steps + fl * bulk_lstm
        achieved = alg_flops / (bulk_ms / 1e3) / 1e12 if bulk_ms > 0 else 0.0
        peak, peak_kind = read_peaks("tensor")
        tr = profiled_traffic(args.config)
        # tensor work issued per algorithmic product, in f16-product equivalents: the joint
        # splits activations into f16 hi + lo and q8_0 weights (scaled) into hi + lo (three
        # products; f16 weights are exact: two), its screened iterations issue one; the
        # LSTM and pred-proj issue three int8 products (each half an f16 product's time;
        # --no-i8: as the joint); the int8 layer 0 has K = H instead of 2H
        products = 3 if wtype == "q8_0" else 2
        pl = products if args.no_i8 else 1.5
        issued = ((pl * fl * bulk_lstm + fj * (products * (bulk_steps - bulk_scr) + bulk_scr))
                  / (bulk_ms / 1e3) / 1e12 if bulk_ms > 0 else 0.0)
        parity = None
        if par is not None:
            parity = {"reference_fixture": par["fixture"], "utterances_checked": int(par_checked),
                      "identical_to_reference": int(par_same),
                      "differing": int(par_checked - par_same),
                      "bar": "tokens and steps identical to the reference decoder except where the first differing "
                             "decision is an oracle near-tie (top-2 margin < 1e-3); the near-tie and teacher-forced "
                             "logit / state checks (<= 2e-3) of these utterances are tests/test_full_size.py"}
        result = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": tot_ms / args.steps,
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
            "dtype": DTYPE["q8" if args.math == "q8" else "f32" if args.math == "f32" else wtype],
            "data": "synthetic (seeded random-init weights of the named geometry, N(0,1) encoder outputs)",
            "config": config,
            "steps_per_sec": steps_all / (tot_ms / 1e3) if tot_ms > 0 else 0.0,
            "p50_utterance_latency_ms": float(np.median(lat)) if lat is not None and len(lat) else None,
            "decode_split_ms_per_step": {"encproj": enc_ms / args.steps, "loop": loop_ms / args.steps,
                                         "total": tot_ms / args.steps},
            "loop_iterations_per_step": iters / args.steps,
            "loop_us_per_iteration": {
                name: 1e3 * (phase[2 * i] + phase[2 * i + 1]) / max(1, iters)
                for i, name in enumerate(["lstm", "pred_hidden", "joint", "decision"])},
            "loop_wait_share": float((phase[1::2].sum()) / max(phase.sum(), 1e-9)),
            "gpu_launches": int(launches),
            "parity": parity,
            "clocks": clk,
            "wall_s_timed": wall_s,
            "e2e": {"value": e2e_tokens_all / (e2e_ms / 1e3) if e2e_ms > 0 else 0.0, "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms / args.steps,
                    "timing": "host wall clock around K pk_decode_batch calls on pinned host buffers, "
                              "each step's encoder copy prefetched (pk_prefetch_batch) during the "
                              "previous step's decode; max over ranks",
                    "serial": {"value": ser_tokens_all / (ser_ms / 1e3) if ser_ms > 0 else 0.0,
                               "ms_per_step": ser_ms / args.steps,
                               "timing": "one pk_decode_batch call at a time, copies inside the call, "
                                         "the library's CUDA events; max over ranks"},
                    "tokens_match_device_run": same},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak if peak else None,
                         "traffic": (tr * bulk_steps / args.steps) if tr else None,
                         "kernel": "bulk_loop_kernel",
                         "issued_tflops": issued,
                         "note": f"FLOPs of the products computed = {fj} per joint evaluation ({bulk_steps // args.steps} "
                                 f"per launch) + {fl} per LSTM step ({bulk_lstm // args.steps} per launch), "
                                 f"one product each; the kernel issues {pl} f16-product equivalents per "
                                 f"algorithmic LSTM / pred-proj product, {products} per unscreened joint product, "
                                 f"one per screened joint product ({bulk_scr // args.steps} screened "
                                 f"evaluations per launch) "
                                 f"(issued_tflops); time = the bulk kernel's CUDA events "
                                 f"({bulk_ms / args.steps:.2f} ms per launch, {bulk_iters // args.steps} iterations); "
                                 f"peak = cuBLAS bf16 sustained, {peak_kind}; traffic = dram bytes per joint "
                                 f"evaluation from the committed ncu summary x evaluations per launch"},
            "persistent_loop": {"kernel": "step_loop_kernel", "ms_per_step": (loop_ms - pl_bulk_ms) / args.steps,
                                "iterations_per_step": (iters - pl_bulk_iters) / args.steps},
        }
    if world == 1 and not args.no_cpu_baseline and rank == 0:
        o, kind = reference_decoder(model)
        threads = host_cores()
        cs = cpu_sample_run(o, enc, offs, T, threads, args.cpu_budget_s)
        result["cpu_baseline"] = {
            "value": cs["tokens"] / cs["wall_s"], "unit": "tokens/s", "cores": threads, "kind": kind,
            "cpu_model": cpu_model(),
            "sample": f"first {cs['n_utt']} utterances of the batch truncated to {cs['cap']} frames "
                      f"({cs['frames']} frames, {cs['tokens']} tokens, {cs['wall_s']:.1f} s wall), "
                      f"one utterance per thread, -O3 -ffast-math -funroll-loops",
            "steps_per_sec": cs["steps"] / cs["wall_s"], "p50_utterance_ms": cs["p50_ms"]}
    if rank == 0:
        print(json.dumps(result))
    dec.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
