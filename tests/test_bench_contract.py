"""The one-JSON-line contract of bench.py, checked on its CPU-only reference arm.

The reference arm times the reference's own moda_attention_naive (torch on the host
CPU, from the unmodified install in baseline/_ref; the numpy restatement in oracle/
when that install is absent) on the host cores, so it runs here without a GPU; its line carries the same keys the GPU arm
prints. Under torchrun with two ranks only rank 0 prints and the other rank exits 0
without work.
"""

import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
             "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"}


def _json_lines(out):
    return [json.loads(s) for s in out.splitlines() if s.startswith("{")]


def _check_reference_line(line, n_gpus):
    assert BASE_KEYS <= set(line)
    assert line["impl"] == "reference"
    assert line["n_gpus"] == n_gpus and line["steps"] == 1 and line["warmup"] == 0
    assert line["value"] > 0 and line["ms_per_step"] > 0 and line["higher_is_better"] is True
    assert "workload" in line["config"]
    cb = line["cpu_baseline"]
    ref_installed = os.path.exists(os.path.join(REPO, "baseline", "_ref", "moda", "__init__.py"))
    assert cb["kind"] == ("reference" if ref_installed else "port")
    assert cb["cores"] >= 1 and cb["value"] == line["value"]
    assert cb["unit"] == line["unit"] and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                        "--warmup", "0"], cwd=REPO, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    _check_reference_line(lines[0], 1)


def test_reference_arm_two_ranks_rank0_only():
    env = dict(os.environ, MASTER_ADDR="127.0.0.1")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
                        "--master-port", "29611", "bench.py", "--impl", "reference",
                        "--gpus", "2", "--steps", "1", "--warmup", "0"],
                       cwd=REPO, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    _check_reference_line(lines[0], 2)


def test_row_checker_accepts_the_oracle_and_rejects_a_planted_error():
    """bench.py's per-rank row check (float64 restatement in torch) agrees with the
    oracle on small seeded inputs, and catches one wrong output row."""
    import numpy as np
    import torch
    sys.path.insert(0, REPO)
    import bench
    from oracle import moda_oracle as orc
    from helpers import seeded_inputs
    B, Hq, Hk, T, d, L = 2, 8, 2, 40, 16, 3
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=5)
    O = torch.from_numpy(orc.moda_attention_naive(*[a.astype(np.float64) for a in arrs], L))
    ts = [torch.from_numpy(a) for a in arrs]
    rows = bench.sample_rows(B, Hq, T, Hq // Hk, seed=1)
    assert all(0 <= b < B and 0 <= h < Hq and 0 <= t < T for b, h, t in rows)
    ok, worst = bench.check_rows(O, *ts, L, rows, tol=1e-9)
    assert ok and worst < 1e-9
    bad = O.clone()
    b, h, t = rows[3]
    bad[b, h, t, 0] += 0.05
    ok, worst = bench.check_rows(bad, *ts, L, rows)
    assert not ok and abs(worst - 0.05) < 1e-6


def test_side_pass_shape_options():
    """--batch / --seq / --heads / --head-dim reshape the workload of the backward and
    reference passes only, keeping its seeds; the forward headline refuses them."""
    sys.path.insert(0, REPO)
    import bench
    wl = bench.WORKLOADS["kernel"]
    r = bench.resized(wl, 1, 4096)
    assert (r["B"], r["T"], r["Hq"], r["Hk"], r["d"], r["seed"]) == (1, 4096, 32, 8, 128, wl["seed"])
    assert "B=1 " in r["desc"] and "T=4096 " in r["desc"]
    assert bench.resized(wl) is wl
    assert abs(bench.fma_peak_tflops(1965) - 74.45) < 0.01
    for args in (["--pass", "forward", "--heads", "24,8"], ["--pass", "forward", "--dtype", "fp32"],
                 ["--pass", "backward", "--heads", "24,7"], ["--pass", "model", "--head-dim", "96"]):
        res = subprocess.run([sys.executable, "bench.py", *args, "--steps", "1"], cwd=REPO,
                             capture_output=True, text=True, timeout=300)
        assert res.returncode == 2 and "error:" in res.stderr, (args, res.stderr[-300:])
