"""bench.py's reference arm runs without a GPU: one JSON line with the
contract's keys, ``impl`` "reference", a ``cpu_baseline`` describing the run
and an ``e2e`` with no host<->device bytes; under torchrun only rank 0
prints, and every rank exits 0."""
import json
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
SMALL = ["--impl", "reference", "--steps", "2", "--warmup", "3", "--batch", "4",
         "--kv-len", "256", "--cpu-seconds", "1"]
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
        "impl", "cpu_baseline", "e2e"}


def _env():
    env = dict(os.environ)
    env["CUDA_VISIBLE_DEVICES"] = ""
    env["MASTER_ADDR"] = "127.0.0.1"
    return env


def _lines(out: str):
    return [json.loads(l) for l in out.splitlines() if l.startswith("{")]


def _check(line, n_gpus):
    assert KEYS <= set(line), KEYS - set(line)
    assert line["impl"] == "reference" and line["n_gpus"] == n_gpus
    assert line["value"] > 0 and line["higher_is_better"] is True
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == line["value"] and cb["unit"] == line["unit"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"]


def test_reference_arm_one_process():
    r = subprocess.run([sys.executable, "bench.py", *SMALL], cwd=REPO, env=_env(),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1, r.stdout
    _check(lines[0], 1)


def test_reference_arm_two_ranks_rank0_prints():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", "29531", "bench.py", "--gpus", "2",
           *SMALL]
    r = subprocess.run(cmd, cwd=REPO, env=_env(), capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1, r.stdout
    _check(lines[0], 2)


def test_decode_bytes_is_the_algorithmic_formula():
    """bench.decode_bytes: K+V rows (512 B per token at 2 kv heads x 64 x fp16,
    K and V), q and o (14 x 64 fp16 each) and one int64 block-table entry per
    visited page; 538,312,704 B at the bench point B=256 x 4096."""
    import bench

    assert bench.decode_bytes(256, 4096) == 538_312_704
    assert bench.decode_bytes(256, 4096) == 256 * 4096 * 512 + 256 * 3584 + 256 * 256 * 8
    assert bench.decode_bytes(1, 17) == 17 * 512 + 3584 + 2 * 8
