"""bench.py's reference arm runs on the host and prints the JSON line the driver reads (no GPU).

The arm must time the reference algorithm only: its process may not import
this package (or map its native library), and its ``config`` must be the
product arm's, word for word.
"""

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent

# Runs bench.py as __main__ and reports, after it returns, which product
# modules and shared objects the process loaded.
_PROBE = r"""
import json, runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1", "--gpus", GPUS]
try:
    runpy.run_path("bench.py", run_name="__main__")
except SystemExit as exc:
    assert not exc.code, exc.code
mods = sorted(m for m in sys.modules if m.split(".")[0] == "nano_infer_engine_b200")
maps = open("/proc/self/maps").read() if sys.platform.startswith("linux") else ""
libs = sorted({l.split()[-1] for l in maps.splitlines() if "nano_infer_engine_b200" in l})
print("PROBE " + json.dumps({"modules": mods, "libs": libs}))
"""


@pytest.mark.parametrize("gpus", [1, 2])
def test_reference_arm_prints_the_contract_line(gpus):
    probe_src = _PROBE.replace("GPUS", repr(str(gpus)))
    proc = subprocess.run([sys.executable, "-c", probe_src], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = proc.stdout.splitlines()
    out = json.loads([l for l in lines if l.startswith("{")][-1])
    probe = json.loads([l for l in lines if l.startswith("PROBE ")][-1][6:])
    assert probe == {"modules": [], "libs": []}, probe
    assert out["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "config", "cpu_baseline",
                "e2e"):
        assert key in out, key
    assert out["value"] > 0 and out["higher_is_better"] is True
    assert out["cpu_baseline"]["value"] == out["value"]
    assert out["cpu_baseline"]["kind"] in ("port", "reference") and out["cpu_baseline"]["cores"] >= 1
    assert out["e2e"]["value"] == out["value"]
    assert out["e2e"]["h2d_bytes_per_step"] == 0 and out["e2e"]["d2h_bytes_per_step"] == 0
    sys.path.insert(0, str(ROOT))
    import argparse

    import bench

    if gpus == 1:
        assert out["config"] == bench.headline_config(argparse.Namespace(requests=16), 1)
    else:  # the product arm's P/D workload (one pair at N=2), sampled on the host
        args = argparse.Namespace(new_tokens=256, pd_decode_per_prefill=None)
        k, groups = bench.pd_layout(args, gpus)
        assert (k, groups) == (1, 1)
        assert out["config"] == bench.pd_config(args, bench.pd_workload(2 * bench.PD_REQUESTS_PER_GPU), groups, k)


def test_oracle_weights_equal_the_engine_init():
    """The oracle's seeded state dict is the engine's random init, tensor for tensor."""
    import torch

    from nano_infer_engine_b200.models.llama import LlamaConfig, build_random_llama
    from oracle.weights import random_llama_state

    arch = dict(vocab_size=96, hidden_size=64, mlp_inner_size=80, num_layers=2, q_head_num=4, kv_head_num=2,
                norm_eps=1e-5, rope_type="default", rope_theta=500000.0)
    for tied in (True, False):
        cfg = LlamaConfig(**arch, tie_word_embeddings=tied, max_seq_len=128)
        model = build_random_llama(cfg, 7, 0.02, torch.bfloat16)
        state = random_llama_state(dict(arch, tie_word_embeddings=tied), 7, 0.02, torch.bfloat16)
        want = model.state_dict()
        assert sorted(state) == sorted(want)
        for name in want:
            assert state[name].dtype == want[name].dtype
            assert torch.equal(state[name], want[name]), name


def test_pd_job_gives_every_decode_rank_the_same_requests():
    """The closed-loop P/D job is weak scaling on a fixed job per decode GPU, for pairs and for
    one prefill rank feeding several decode ranks."""
    import bench
    from nano_infer_engine_b200.generation.pd_disagg import assign_groups

    base = None
    for groups, k in ((1, 1), (2, 1), (4, 1), (1, 3), (2, 3)):
        base, job = bench.pd_job(groups * k, 256)
        want = sorted(p.shape[1] for p in base)
        slots = assign_groups([p.shape[1] + 256 for p in job], groups, k)
        assert len(slots) == groups and all(len(group) == k for group in slots)
        for group in slots:
            for slot in group:
                assert sorted(job[i].shape[1] for i in slot) == want
    assert sum(p.shape[1] for p in base) == 18376
