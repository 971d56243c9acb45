"""bench.py's reference arm on the CPU: the JSON line the driver reads (no GPU needed).

`bench.py --impl reference` times the oracle port of the path on the host cores, on the same
workload, metric and unit as the GPU arm; under torchrun only rank 0 prints."""

import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT


def _run(args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + args, cwd=ROOT,
                       capture_output=True, text=True, env=e, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


@pytest.mark.parametrize("workload", ["mxfp8_quantize", "decode_gemm"])
def test_reference_arm_line(workload):
    lines = _run(["--impl", "reference", "--steps", "1", "--warmup", "3", "--workload", workload,
                  "--extra", "none"])
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["steps"] == 1
    assert d["warmup"] >= 3 and d["higher_is_better"] is True
    assert d["value"] > 0 and d["unit"] in ("GB/s", "TFLOP/s")
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"] and cb["cores"] >= 1
    assert cb["kind"] == "port" and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert d["config"]["workload"].startswith(workload)


def test_reference_arm_workload_records():
    """The reference arm carries a record per extra workload, with the config dict the GPU arm
    emits for it (same function, same keys: parallelism and launch included)."""
    sys.path.insert(0, ROOT)
    import bench
    lines = _run(["--impl", "reference", "--steps", "1", "--warmup", "3",
                  "--extra", "fp8_gemm,decode_gemm"])
    d = json.loads(lines[0])
    assert set(d["workloads"]) == {"fp8_gemm", "decode_gemm"}
    for name, rec in d["workloads"].items():
        wl = bench.WORKLOADS[name](1)
        assert rec["config"] == bench.line_config(wl, 1, True), name
        assert rec["value"] > 0 and rec["unit"] == wl.unit
        assert rec["cpu_baseline"]["value"] == rec["value"]
        assert rec["e2e"]["h2d_bytes_per_step"] == 0
    head = bench.WORKLOADS["mxfp8_quantize"](1)
    assert d["config"] == bench.line_config(head, 1, True)


def test_extra_workload_selection():
    sys.path.insert(0, ROOT)
    import bench

    class A:
        extra, workload = "auto", "mxfp8_quantize"
    assert bench.extra_workloads(A, 1) == ["fp8_gemm", "mxfp8_gemm", "nvfp4_gemm",
                                           "decode_gemm"]
    assert bench.extra_workloads(A, 4)[-1] == "decode_gemm_nccl"
    A.workload = "nvfp4_gemm"
    assert bench.extra_workloads(A, 1) == []
    A.extra = "none"
    assert bench.extra_workloads(A, 1) == []
    # the multi-rank records name the entry points they run
    assert bench.WORKLOADS["nvfp4_gemm"](4).config["entry_point"] == "ptxstd_gemm_nvfp4_sharded"
    assert bench.WORKLOADS["decode_gemm"](2).config["entry_point"] == \
        "ptxstd_gemm_decode_sharded_p2p"
    assert bench.WORKLOADS["decode_gemm_nccl"](2).config["entry_point"] == \
        "ptxstd_gemm_decode_sharded"


def test_reference_arm_other_ranks_print_nothing():
    lines = _run(["--impl", "reference", "--steps", "1", "--warmup", "3", "--gpus", "2"],
                 env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert lines == []


def test_warmup_floor_and_workload_names():
    sys.path.insert(0, ROOT)
    import bench
    assert {"mxfp8_quantize", "fp8_gemm", "nvfp4_gemm", "decode_gemm", "mxfp8_gemm",
            "mxfp8_quantize_sr", "mxfp8_gemm_sparse", "mxfp6_gemm"} <= set(bench.WORKLOADS)
    for name, cls in bench.WORKLOADS.items():
        wl = cls(1)
        assert wl.unit in ("GB/s", "TFLOP/s") and wl.config["workload"], name
        assert hasattr(wl, "e2e_slots") and hasattr(wl, "e2e_compute"), name
