"""bench.py's reference arm (the oracle on the host's cores) runs without a GPU: check
the JSON line it prints for the driver, and that ranks other than 0 print nothing."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(extra_env=None, config=("--config", "1")):
    env = dict(os.environ)
    env.update(extra_env or {})
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", *config,
                        "--steps", "1", "--warmup", "0"], capture_output=True, text=True, env=env, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    return [ln for ln in p.stdout.splitlines() if ln.startswith("{")]


def test_reference_arm_line():
    lines = _run()
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "tdt_greedy_decode_tokens_per_sec" and d["unit"] == "tokens/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    for k in ("n_gpus", "steps", "warmup", "ms_per_step", "scaling", "vs_baseline", "dtype", "data", "config"):
        assert k in d, k
    # the reference's own decoder when oracle/_ref holds its build, else the restatement
    kind = "reference" if os.path.exists(os.path.join(ROOT, "oracle", "_ref", "libref_decoder.so")) else "port"
    assert d["cpu_baseline"]["kind"] == kind and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"].startswith("TDT-0.6b")


def test_reference_arm_default_workload():
    """With no flags the arm runs the headline workload (configuration 5: the 4096-utterance
    global batch, strong scaling) on a bounded sample."""
    d = json.loads(_run(config=())[0])
    assert d["config"]["config"] == "5" and d["config"]["global_batch"] == 4096
    assert d["scaling"] == "strong" and d["value"] > 0


def test_reference_arm_other_ranks_print_nothing():
    assert _run({"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"}) == []
