"""Benchmark of the narrow-float quantise / block-scaled GEMM path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload mxfp8_quantize|...] [--extra auto|none|w1,w2,...]

One JSON line on rank 0. A "step" is one pass of the hot path over one batch of synthetic input:
for ``mxfp8_quantize`` (the default, 8192 x 8192 bf16 -> E4M3 + UE8M0 per 32) one quantise
launch. ``value`` is device-timed (CUDA events on the launching stream, max over ranks) with the
inputs resident in HBM; ``e2e`` is the same metric through the public API with host buffers,
including every step's host->device copy of its inputs and device->host copy of its results,
pipelined over two buffer slots (copies on their own streams, overlapping the compute).

With the default headline the same line also carries a ``workloads`` object: one record per GEMM
configuration (``fp8_gemm`` 8192^3, ``mxfp8_gemm`` 8192^3, ``nvfp4_gemm`` 8192 x 28672 x 8192
sharded along N over the ranks, ``decode_gemm`` 16 x 57344 x 8192 sharded along N with the output
gathered to every rank; on several ranks also ``decode_gemm_nccl``), each measured in this
process with the same rules and carrying its own ``ms_per_step``, ``roofline``, ``clocks``,
``e2e`` and, on one GPU, ``cpu_baseline``.

``--impl reference`` times the reference's conversion semantics on the host cores instead (the
C oracle: the reference crate itself cannot be built here, it targets nvptx64 only), on the same
workloads, metric, unit and config.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "ptx-std_b200")]

METRIC = "Block-scaled FP8/FP4 GEMM TFLOPS/GPU (% tensor peak); quantise GB/s (% HBM)"
HBM_FALLBACK_GBS = 6650.0
BF16_FALLBACK_TFLOPS = 1590.0


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d.get("hbm_gbs", HBM_FALLBACK_GBS),
                "bf16_tflops": d.get("bf16_tflops", BF16_FALLBACK_TFLOPS),
                "source": "measured"}
    return {"hbm_gbs": HBM_FALLBACK_GBS, "bf16_tflops": BF16_FALLBACK_TFLOPS,
            "source": "fallback"}


def profiled_traffic(kernel: str):
    """DRAM bytes per launch recorded from an ncu capture of this kernel (profiles/traffic.json)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    return json.load(open(p)).get(kernel, {}).get("dram_bytes_per_launch")


# ---- clocks ---------------------------------------------------------------------------------

class ClockSampler:
    """SM clock and throttle-reason samples taken while the timed region runs.

    Polls NVML every 2 ms in a thread (reading clocks only; nothing is set), so that even a
    timed region of a few tens of milliseconds gets samples; falls back to nvidia-smi -lms 100.
    """

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap"}

    def __init__(self, device_index: int):
        self.dev = device_index
        self.samples: list[tuple[float, float, int]] = []
        self.proc = None
        self.lines: list[str] = []
        self._stop = threading.Event()
        self.nvml = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        uuid = "GPU-" + str(torch.cuda.get_device_properties(self.dev).uuid)
        return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid)

    def start(self):
        try:
            self.nvml, h = self._nvml_handle()
            nv = self.nvml
            smax = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))

            def sample():
                try:
                    sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                    r = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                    self.samples.append((sm, smax, r))
                except Exception:
                    pass

            def poll():
                while not self._stop.is_set():
                    sample()
                    time.sleep(0.002)

            # the caller's stop() also samples once itself, right after the timed region, so that
            # a region whose host thread holds the interpreter lock still gets a sample under load
            self._sample = sample
            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.nvml = None
        try:
            fields = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                      "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                      "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={fields}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self) -> dict:
        if self.nvml is not None:
            self._sample()
            self._stop.set()
            self.thread.join(timeout=2)
            sm = [x[0] for x in self.samples]
            reasons = set()
            for _, _, r in self.samples:
                for bit, name in self.REASONS.items():
                    if r & bit:
                        reasons.add(name)
            return {"sm_mhz": statistics.median(sm) if sm else None,
                    "sm_max_mhz": self.samples[0][1] if self.samples else None,
                    "reasons": sorted(reasons), "samples": len(sm), "source": "nvml 2 ms"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi 100 ms"}


# ---- distributed plumbing -------------------------------------------------------------------

class Dist:
    def __init__(self, n_gpus: int):
        import torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != n_gpus and self.world > 1:
            raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={self.world}")
        torch.cuda.set_device(self.local)
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as td
            td.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                  device_id=torch.device("cuda", self.local))
            self.pg = td

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ---- workloads --------------------------------------------------------------------------------

def _pinned_like(torch, t):
    """A pinned host buffer of t's shape and dtype."""
    return torch.empty(t.shape, dtype=t.dtype, pin_memory=True)


def _gemm_slots(torch, inputs, c):
    """Two end-to-end buffer slots of a GEMM: slot 0 reuses the device operands and output of the
    device-timed steps, slot 1 has its own; each slot has its own pinned host output."""
    slots = []
    for k in range(2):
        devs = [d if k == 0 else torch.empty_like(d) for d, _ in inputs]
        ck = c if k == 0 else torch.empty_like(c)
        slots.append({"in": [(d, h) for d, (_, h) in zip(devs, inputs)],
                      "out": [(_pinned_like(torch, ck), ck)], "args": (*devs, ck)})
    return slots


class MxFp8Quantize:
    """bf16 [8192, 8192] -> E4M3 [8192, 8192] + UE8M0 [8192, 256] (row-major scales)."""

    name = "mxfp8_quantize"
    unit = "GB/s"
    dtype = "bf16->e4m3+ue8m0"
    rows = cols = 8192
    kernel = "quantize_kernel<Mxfp8>"

    def __init__(self, world: int = 1):
        self.in_bytes = self.rows * self.cols * 2
        self.out_bytes = self.rows * self.cols + self.rows * self.cols // 32
        self.bytes = self.in_bytes + self.out_bytes  # algorithmic bytes per step
        self.config = {"workload": "mxfp8_quantize bf16 8192x8192 -> e4m3 + ue8m0/32",
                       "rows": self.rows, "cols": self.cols, "sf_layout": "row-major",
                       "l2": "inputs larger than L2 (197 MiB/step), 2 rotating buffer sets"}

    def host_input(self):
        if getattr(self, "_x", None) is None:
            from ptxstd import workloads
            self._x = workloads.mxfp8_activation(self.rows, self.cols)
        return self._x

    def setup(self, torch, x_np):
        import numpy as np
        xh = torch.from_numpy(x_np.view(np.int16)).view(torch.bfloat16)
        self.x_host = xh.pin_memory()
        self.sets = []
        for _ in range(2):
            x = self.x_host.cuda()
            q = torch.empty((self.rows, self.cols), dtype=torch.uint8, device="cuda")
            sf = torch.empty((self.rows, self.cols // 32), dtype=torch.uint8, device="cuda")
            self.sets.append((x, q, sf))

    def step(self, i):
        import ptxstd
        x, q, sf = self.sets[i % 2]
        ptxstd.quantize_mxfp8(x, out=(q, sf))
        return 1  # kernel launches

    def e2e_slots(self, torch):
        """Public API from host buffers: H2D input, quantise, D2H payload + scales."""
        return [{"in": [(x, self.x_host)], "out": [(_pinned_like(torch, q), q),
                                                   (_pinned_like(torch, sf), sf)],
                 "args": (x, q, sf)} for x, q, sf in self.sets]

    def e2e_compute(self, i, args):
        import ptxstd
        x, q, sf = args
        ptxstd.quantize_mxfp8(x, out=(q, sf))
        return 1

    def value(self, seconds_per_step: float) -> float:
        return self.bytes / seconds_per_step / 1e9

    def cpu_sample(self, threads: int, budget_s: float):
        """Oracle quantise of the full tensor, repeated up to budget_s of wall time."""
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        x = self.host_input()
        t0 = time.perf_counter()
        reps = 0
        while True:
            O.quantize_mxfp8(x, threads)
            reps += 1
            el = time.perf_counter() - t0
            if el >= budget_s or reps >= 20:
                break
        return self.bytes * reps / el / 1e9, f"{reps} x full 8192x8192 quantise"


class Fp8Gemm:
    """E4M3 A [8192, 8192] x E4M3 B [8192, 8192] (K-contiguous) -> bf16 C, per-tensor scales."""

    name = "fp8_gemm"
    unit = "TFLOP/s"
    dtype = "e4m3 x e4m3 -> f32 acc -> bf16"
    M = N = K = 8192
    kernel = "gemm_fp8_pair_kernel"
    bound = "tensor"
    peak_ratio_to_bf16 = 2.0
    peak_note = "dense FP8 = 2x bf16"

    def __init__(self, world: int = 1):
        self.flops = 2 * self.M * self.N * self.K
        self.in_bytes = (self.M + self.N) * self.K
        self.out_bytes = self.M * self.N * 2
        self.bytes = self.in_bytes + self.out_bytes
        self.config = {"workload": "fp8_gemm e4m3 8192x8192x8192 -> bf16, sa=0.75 sb=1.25",
                       "M": self.M, "N": self.N, "K": self.K,
                       "l2": "operands 128 MiB + output 128 MiB per step (> L2)"}

    def host_input(self):
        if getattr(self, "_ab", None) is None:
            from ptxstd import workloads
            self._ab = (workloads.fp8_operand(self.M, self.K, 31),
                        workloads.fp8_operand(self.N, self.K, 32))
        return self._ab

    def setup(self, torch, ab):
        self.a_host = torch.from_numpy(ab[0]).pin_memory()
        self.b_host = torch.from_numpy(ab[1]).pin_memory()
        self.a = self.a_host.cuda()
        self.b = self.b_host.cuda()
        self.c = torch.empty((self.M, self.N), dtype=torch.bfloat16, device="cuda")

    def step(self, i):
        import ptxstd
        ptxstd.gemm_fp8(self.a, self.b, 0.75, 1.25, out=self.c)
        return 1

    def e2e_slots(self, torch):
        return _gemm_slots(torch, [(self.a, self.a_host), (self.b, self.b_host)], self.c)

    def e2e_compute(self, i, args):
        import ptxstd
        a, b, c = args
        ptxstd.gemm_fp8(a, b, 0.75, 1.25, out=c)
        return 1

    def value(self, seconds_per_step: float) -> float:
        return self.flops / seconds_per_step / 1e12

    def cpu_sample(self, threads: int, budget_s: float):
        """Blocked f32 GEMM over decoded values, on a 256 x 8192 x 8192 row block (1/32 of
        the FLOPs), scaled to the unit."""
        import numpy as np

        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        A, B = self.host_input()[:2]
        rows = 256
        if getattr(self, "_dec", None) is None:
            self._dec = (O.decode(0, A[:rows].ravel()).reshape(rows, self.K),
                         O.decode(0, B.ravel()).reshape(self.N, self.K))
        da, db = self._dec
        t0 = time.perf_counter()
        O.sgemm_nt(np.ascontiguousarray(da), db, threads)
        el = time.perf_counter() - t0
        return 2 * rows * self.N * self.K / el / 1e12, "256x8192x8192 row block, f32 blocked GEMM"


class Mxfp8Gemm(Fp8Gemm):
    """MXFP8 (OCP MX) A [8192, 8192] x B [8192, 8192]: E4M3 with UE8M0 scales per 32 K elements
    in the blocked layout the quantiser writes -> bf16 C."""

    name = "mxfp8_gemm"
    dtype = "e4m3 x e4m3 (ue8m0/32 scales) -> f32 acc -> bf16"
    kernel = "gemm_mxfp8_pair_kernel"
    peak_note = "dense MXFP8 = 2x bf16"

    def __init__(self, world: int = 1):
        super().__init__(world)
        self.in_bytes += (self.M + self.N) * self.K // 32
        self.bytes = self.in_bytes + self.out_bytes
        self.config = {"workload": "mxfp8_gemm e4m3+ue8m0/32 8192x8192x8192 -> bf16",
                       "M": self.M, "N": self.N, "K": self.K,
                       "l2": "operands 132 MiB + output 128 MiB per step (> L2)"}

    def host_input(self):
        if getattr(self, "_abs", None) is None:
            import numpy as np
            a, b = super().host_input()
            rng = np.random.default_rng(33)
            # scales 2^-5 .. 2^5, as bytes in the blocked layout (any byte order is a valid input)
            self._abs = (a, b, rng.integers(122, 133, self.M * self.K // 32, dtype=np.uint8),
                         rng.integers(122, 133, self.N * self.K // 32, dtype=np.uint8))
        return self._abs

    def setup(self, torch, abs_):
        super().setup(torch, abs_[:2])
        self.sfa_host = torch.from_numpy(abs_[2]).pin_memory()
        self.sfb_host = torch.from_numpy(abs_[3]).pin_memory()
        self.sfa = self.sfa_host.cuda()
        self.sfb = self.sfb_host.cuda()

    def step(self, i):
        import ptxstd
        ptxstd.gemm_mxfp8(self.a, self.sfa, self.b, self.sfb, out=self.c)
        return 1

    def e2e_slots(self, torch):
        return _gemm_slots(torch, [(self.a, self.a_host), (self.sfa, self.sfa_host),
                                   (self.b, self.b_host), (self.sfb, self.sfb_host)], self.c)

    def e2e_compute(self, i, args):
        import ptxstd
        a, sfa, b, sfb, c = args
        ptxstd.gemm_mxfp8(a, sfa, b, sfb, out=c)
        return 1


class MxFp6Gemm(Fp8Gemm):
    """MXFP6 (OCP MX, E2M3 elements, UE8M0 per 32) A [8192, 8192] x B [8192, 8192] -> bf16 C on
    tcgen05.mma.kind::mxf8f6f4: payloads in the padded FP6 operand layout (16 six-bit codes + 4
    zero bytes per 16 bytes), quantised on the device from N(0, 1) bf16 by ptxstd_quantize_mx."""

    name = "mxfp6_gemm"
    dtype = "e2m3 x e2m3 (ue8m0/32 scales) -> f32 acc -> bf16"
    kernel = "gemm_mxfp8_pair_kernel"
    peak_note = "dense MXFP6 on kind::mxf8f6f4 = 2x bf16"

    def __init__(self, world: int = 1):
        super().__init__(world)
        self.in_bytes += (self.M + self.N) * self.K // 32
        self.bytes = self.in_bytes + self.out_bytes
        self.config = {"workload": "mxfp6_gemm e2m3+ue8m0/32 8192x8192x8192 -> bf16",
                       "M": self.M, "N": self.N, "K": self.K,
                       "layout": "FP6 16-element groups padded to 16 bytes (1 byte per element)",
                       "l2": "operands 132 MiB + output 128 MiB per step (> L2)"}

    # host_input (inherited) gives the CPU baseline its operands: the f32 blocked GEMM over decoded
    # values costs the same whatever narrow format they were decoded from

    def setup(self, torch, _):
        import ptxstd
        g = torch.Generator(device="cuda")
        g.manual_seed(6161)
        xa = torch.randn((self.M, self.K), generator=g, device="cuda").to(torch.bfloat16)
        xb = torch.randn((self.N, self.K), generator=g, device="cuda").to(torch.bfloat16)
        self.a, self.sfa = ptxstd.quantize_mx(xa, ptxstd.MX_E2M3, sf_layout=1)
        self.b, self.sfb = ptxstd.quantize_mx(xb, ptxstd.MX_E2M3, sf_layout=1)
        del xa, xb
        self.c = torch.empty((self.M, self.N), dtype=torch.bfloat16, device="cuda")
        self.host = [t.cpu().pin_memory() for t in (self.a, self.sfa, self.b, self.sfb)]

    def step(self, i):
        import ptxstd
        ptxstd.gemm_mx(self.a, ptxstd.MX_E2M3, self.sfa, self.b, ptxstd.MX_E2M3, self.sfb,
                       out=self.c)
        return 1

    def e2e_slots(self, torch):
        return _gemm_slots(torch, list(zip((self.a, self.sfa, self.b, self.sfb), self.host)),
                           self.c)

    def e2e_compute(self, i, args):
        import ptxstd
        a, sfa, b, sfb, c = args
        ptxstd.gemm_mx(a, ptxstd.MX_E2M3, sfa, b, ptxstd.MX_E2M3, sfb, out=c)
        return 1


class Mxfp8SparseGemm(Fp8Gemm):
    """2:4-sparse MXFP8: A [8192, 8192] pruned to 2:4 (vals [8192, 4096] + metadata [8192, 1024]) x
    dense B [8192, 8192], UE8M0 scales per 64 logical K -> bf16 C. TFLOP/s count the logical
    (dense-equivalent) 2 M N K; the roofline peak is 2x the dense MXFP8 figure (2:4 sparsity
    halves the tensor-core work per logical FLOP)."""

    name = "mxfp8_gemm_sparse"
    dtype = "2:4 e4m3 x e4m3 (ue8m0/64 scales) -> f32 acc -> bf16"
    kernel = "gemm_mxfp8_sparse_pair_kernel"
    peak_ratio_to_bf16 = 4.0
    peak_note = "2:4-sparse MXFP8 = 2x dense MXFP8 = 4x bf16, logical FLOPs"

    def __init__(self, world: int = 1):
        super().__init__(world)
        self.in_bytes = self.M * self.K // 2 + self.M * self.K // 8 + self.N * self.K + \
            (self.M + self.N) * self.K // 64
        self.bytes = self.in_bytes + self.out_bytes
        self.config = {"workload": "mxfp8_gemm_sparse 2:4 e4m3 x e4m3, ue8m0/64, "
                       "8192x8192x8192 (logical K) -> bf16", "M": self.M, "N": self.N,
                       "K": self.K, "l2": "operands 104 MiB + output 128 MiB per step (> L2)"}

    def host_input(self):
        if getattr(self, "_sp", None) is None:
            import numpy as np
            sys.path.insert(0, os.path.join(ROOT, "oracle"))
            a, b = super().host_input()
            rng = np.random.default_rng(34)
            self._sp = (a, b, rng.integers(122, 133, self.M * self.K // 64, dtype=np.uint8),
                        rng.integers(122, 133, self.N * self.K // 64, dtype=np.uint8))
        return self._sp

    def setup(self, torch, sp):
        import ptxstd
        super().setup(torch, sp[:2])
        # prune A on the device (the library's own 2:4 pruning)
        self.vals, self.meta = ptxstd.prune_24(self.a)
        self.vals_host = self.vals.cpu().pin_memory()
        self.meta_host = self.meta.cpu().pin_memory()
        self.sfa_host = torch.from_numpy(sp[2]).pin_memory()
        self.sfb_host = torch.from_numpy(sp[3]).pin_memory()
        self.sfa = self.sfa_host.cuda()
        self.sfb = self.sfb_host.cuda()

    def step(self, i):
        import ptxstd
        ptxstd.gemm_mxfp8_sparse(self.vals, self.meta, self.sfa, self.b, self.sfb, out=self.c)
        return 1

    def e2e_slots(self, torch):
        return _gemm_slots(torch, [(self.vals, self.vals_host), (self.meta, self.meta_host),
                                   (self.sfa, self.sfa_host), (self.b, self.b_host),
                                   (self.sfb, self.sfb_host)], self.c)

    def e2e_compute(self, i, args):
        import ptxstd
        vals, meta, sfa, b, sfb, c = args
        ptxstd.gemm_mxfp8_sparse(vals, meta, sfa, b, sfb, out=c)
        return 1

    def cpu_sample(self, threads: int, budget_s: float):
        """The same f32 blocked GEMM as the dense workloads over the decompressed A (a CPU has no
        2:4 sparse unit), on a 256-row block, scaled to the logical FLOPs."""
        return super().cpu_sample(threads, budget_s)


class Nvfp4Gemm:
    """NVFP4 MLP up-projection: A [8192, 8192] x B [28672, 8192] (E2M1 + E4M3/16 + f32 global)
    -> bf16 [8192, 28672]; B is sharded along N across ranks (no communication). On several
    ranks each step is ptxstd_gemm_nvfp4_sharded on this rank's 28672 / world columns."""

    name = "nvfp4_gemm"
    unit = "TFLOP/s"
    dtype = "e2m1 x e2m1 (e4m3/16 scales) -> f32 acc -> bf16"
    M, N, K = 8192, 28672, 8192
    kernel = "gemm_nvfp4_pair_kernel"
    bound = "tensor"
    peak_ratio_to_bf16 = 4.0
    peak_note = "dense NVFP4 = 4x bf16"
    scaling = "strong"
    parallelism = "n-shard"

    def __init__(self, world: int = 1):
        self.world = world
        self.n_local = self.N // world
        self.flops = 2 * self.M * self.n_local * self.K
        self.in_bytes = (self.M + self.n_local) * self.K // 2 + (self.M + self.n_local) * self.K // 16
        self.out_bytes = self.M * self.n_local * 2
        self.bytes = self.in_bytes + self.out_bytes
        self.config = {"workload": "nvfp4_gemm 8192x28672x8192 (MLP up-projection) -> bf16",
                       "M": self.M, "N": self.N, "K": self.K, "n_per_gpu": self.n_local,
                       "sharding": "B along N, no communication",
                       "entry_point": "ptxstd_gemm_nvfp4_sharded" if world > 1
                       else "ptxstd_gemm_nvfp4",
                       "l2": "operands 127 MiB + output 448 MiB per step (> L2)"}

    def host_input(self):
        return None

    def setup(self, torch, _):
        import ptxstd
        rank = int(os.environ.get("RANK", "0"))
        g = torch.Generator(device="cuda")
        g.manual_seed(1234)
        xa = torch.randn((self.M, self.K), generator=g, device="cuda").to(torch.bfloat16)
        g.manual_seed(5678 + rank)
        xb = torch.randn((self.n_local, self.K), generator=g, device="cuda").to(torch.bfloat16)
        self.ga = float(xa.float().abs().max()) / (448.0 * 6.0)
        self.gb = float(xb.float().abs().max()) / (448.0 * 6.0)
        self.a, self.sfa = ptxstd.quantize_nvfp4(xa, self.ga, sf_layout=1)
        self.b, self.sfb = ptxstd.quantize_nvfp4(xb, self.gb, sf_layout=1)
        del xa, xb
        self.c = torch.empty((self.M, self.n_local), dtype=torch.bfloat16, device="cuda")
        self.host = [t.cpu().pin_memory() for t in (self.a, self.sfa, self.b, self.sfb)]
        ctx = getattr(self, "ctx", None)
        self.pd = ctx.ptxstd_dist() if ctx is not None and self.world > 1 else None

    def _gemm(self, a, sfa, b, sfb, c):
        import ptxstd
        if self.pd is None:
            ptxstd.gemm_nvfp4(a, sfa, self.ga, b, sfb, self.gb, out=c)
        else:
            self.pd.gemm_nvfp4(a, sfa, self.ga, b, sfb, self.gb, self.N, out=c)
        return 1

    def step(self, i):
        return self._gemm(self.a, self.sfa, self.b, self.sfb, self.c)

    def e2e_slots(self, torch):
        return _gemm_slots(torch, list(zip((self.a, self.sfa, self.b, self.sfb), self.host)),
                           self.c)

    def e2e_compute(self, i, args):
        return self._gemm(*args)

    def value(self, seconds_per_step: float) -> float:
        return self.flops / seconds_per_step / 1e12

    def cpu_sample(self, threads: int, budget_s: float):
        """Blocked f32 GEMM over decoded values on a 128 x N x K row block."""
        import numpy as np

        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        rows = 128
        rng = np.random.default_rng(7)
        if getattr(self, "_dec", None) is None:
            self._dec = (rng.standard_normal((rows, self.K), dtype=np.float32),
                         rng.standard_normal((self.n_local, self.K), dtype=np.float32))
        da, db = self._dec
        t0 = time.perf_counter()
        O.sgemm_nt(da, db, threads)
        el = time.perf_counter() - t0
        return (2 * rows * self.n_local * self.K / el / 1e12,
                f"{rows}x{self.n_local}x{self.K} row block, f32 blocked GEMM on decoded values")


class DecodeGemm:
    """Decode step: x bf16 [16, 8192] (MXFP8 in the call) x NVFP4 W [57344, 8192] -> bf16
    [16, 57344]; W is sharded along N across ranks and every rank ends with all output columns:
    with `gather` "p2p" (default) the decode epilogue stores them into every rank's output over
    NVLink peer memory, with "nccl" an NCCL all-gather follows the GEMM. On several ranks the
    record also times the rank's GEMM alone (its own columns into a local output, no gather), so
    that the gather's share of a step is reported apart from the GEMM's."""

    name = "decode_gemm"
    unit = "GB/s"
    dtype = "mxfp8(x) x nvfp4(W) -> f16 tensor cores, f32 acc -> bf16"
    M, N, K = 16, 57344, 8192
    kernel = "gemm_decode_kernel"
    scaling = "strong"
    parallelism = "n-shard"

    def __init__(self, world: int = 1, gather: str = "p2p"):
        self.world = world
        self.gather = gather
        self.n_local = self.N // world
        w_bytes = self.n_local * self.K // 2 + self.n_local * self.K // 16
        self.bytes = w_bytes + self.M * self.K * 2 + self.M * self.n_local * 2
        self.in_bytes = self.M * self.K * 2            # per step from host: the activations
        self.out_bytes = self.M * self.N * 2           # per step to host: the gathered output
        self.gather_bytes = (world - 1) * self.M * self.n_local * 2  # NVLink bytes in per rank
        self.config = {"workload": "decode_gemm x[16,8192] bf16 -> mxfp8, W nvfp4 [57344,8192]",
                       "M": self.M, "N": self.N, "K": self.K, "n_per_gpu": self.n_local,
                       "sharding": "W along N, output columns gathered to every rank",
                       "l2": "weights 252 MiB per step (> L2), 2 rotating weight copies"}
        if world > 1:
            # (g - 1) / g of the 1,835,008-byte output crosses NVLink into every rank per step
            self.config["nvlink_bytes_in_per_rank"] = self.gather_bytes
            self.config["sharding"] = (
                "W along N; the decode epilogue stores each rank's columns into every rank's "
                "output over NVLink (CUDA IPC peer memory), no collective" if gather == "p2p"
                else "W along N, NCCL all-gather of output columns + device unshard permute")
            self.config["entry_point"] = ("ptxstd_gemm_decode_sharded_p2p" if gather == "p2p"
                                          else "ptxstd_gemm_decode_sharded")

    def host_input(self):
        return None

    def setup(self, torch, _):
        import ptxstd
        rank = int(os.environ.get("RANK", "0"))
        g = torch.Generator(device="cuda")
        g.manual_seed(4321)
        self.x = torch.randn((self.M, self.K), generator=g, device="cuda").to(torch.bfloat16)
        self.sets = []
        for copy in range(2):
            g.manual_seed(8765 + 17 * rank + copy)
            wb = (torch.randn((self.n_local, self.K), generator=g, device="cuda") * 0.02).to(
                torch.bfloat16)
            gw = float(wb.float().abs().max()) / (448.0 * 6.0)
            w, sfw = ptxstd.quantize_nvfp4(wb, gw, sf_layout=1)
            del wb
            self.sets.append((w, sfw, gw))
        self.x_host = self.x.cpu().pin_memory()
        # every rank ends the step with the full [16, N] output
        self.y = torch.empty((self.M, self.N), dtype=torch.bfloat16, device="cuda")
        self.y_local = None
        ctx = getattr(self, "ctx", None)
        self.dist = ctx.ptxstd_dist() if ctx is not None and self.world > 1 else None
        if self.dist is not None:
            self.y_local = torch.empty((self.M, self.n_local), dtype=torch.bfloat16,
                                       device="cuda")
            if self.gather == "p2p":
                self.y = self.dist.decode_p2p_output(self.N)

    def step(self, i):
        import ptxstd
        w, sfw, gw = self.sets[i % 2]
        if self.dist is None:
            ptxstd.gemm_decode(self.x, w, sfw, gw, out=self.y)
            return 2
        if self.gather == "p2p":
            # prep, decode with peer stores into every rank's y, completion wait
            self.dist.gemm_decode_p2p(self.x, w, sfw, gw, self.N)
            return 3
        # local shard, in-place NCCL all-gather over NVLink, device-side unshard permute
        self.dist.gemm_decode(self.x, w, sfw, gw, self.N, out=self.y)
        return 3

    def gemm_only_step(self):
        """The rank's GEMM over its own columns, with no gather (several ranks only)."""
        if self.dist is None:
            return None

        def run(i):
            import ptxstd
            w, sfw, gw = self.sets[i % 2]
            ptxstd.gemm_decode(self.x, w, sfw, gw, out=self.y_local)
            return 2
        return run

    def e2e_slots(self, torch):
        # the fused multi-GPU decode writes a library-owned y that the next step overwrites, so
        # each step also copies it into its slot's buffer, which the D2H copy then reads
        slots = []
        for k in range(2):
            x = self.x if k == 0 else torch.empty_like(self.x)
            y = torch.empty((self.M, self.N), dtype=torch.bfloat16, device="cuda")
            slots.append({"in": [(x, self.x_host)], "out": [(_pinned_like(torch, y), y)],
                          "args": (x, y)})
        return slots

    def e2e_compute(self, i, args):
        import ptxstd
        x, y = args
        w, sfw, gw = self.sets[i % 2]
        if self.dist is None:
            ptxstd.gemm_decode(x, w, sfw, gw, out=y)
            return 2
        if self.gather == "p2p":
            self.dist.gemm_decode_p2p(x, w, sfw, gw, self.N, out=y)
            return 3
        self.dist.gemm_decode(x, w, sfw, gw, self.N, out=y)
        return 3

    def value(self, seconds_per_step: float) -> float:
        return self.bytes / seconds_per_step / 1e9

    def cpu_sample(self, threads: int, budget_s: float):
        """f32 GEMV-shaped blocked GEMM (16 x 8192 x 8192 block of the weights)."""
        import numpy as np

        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        rng = np.random.default_rng(3)
        if getattr(self, "_dec", None) is None:
            self._dec = (rng.standard_normal((self.M, self.K), dtype=np.float32),
                         rng.standard_normal((8192, self.K), dtype=np.float32))
        a, b = self._dec
        t0 = time.perf_counter()
        O.sgemm_nt(a, b, threads)
        el = time.perf_counter() - t0
        # bytes of the NVFP4 weight block this sample covers, per second
        wbytes = 8192 * self.K // 2 + 8192 * self.K // 16
        return wbytes / el / 1e9, "16x8192x8192 block, f32 blocked GEMM on decoded weights"


class DecodeGemmNccl(DecodeGemm):
    """The decode step with the NCCL all-gather of output columns in place of the fused
    peer-store gather (the same as decode_gemm on one GPU)."""

    name = "decode_gemm_nccl"

    def __init__(self, world: int = 1):
        super().__init__(world, gather="nccl")
        self.config = dict(self.config, workload="decode_gemm_nccl x[16,8192] bf16 -> mxfp8, "
                           "W nvfp4 [57344,8192], NCCL all-gather")


class MxFp8QuantizeSR(MxFp8Quantize):
    """The same MXFP8 quantise with stochastic rounding of the elements (cvt.rs, random bits from
    SplitMix64 of a per-step seed, generated on the device)."""

    name = "mxfp8_quantize_sr"
    kernel = "quantize_kernel<Mxfp8Rs>"

    def __init__(self, world: int = 1):
        super().__init__(world)
        self.config = dict(self.config, workload="mxfp8_quantize_sr bf16 8192x8192 -> e4m3 "
                           "(stochastic rounding) + ue8m0/32", rounding="cvt.rs, SplitMix64 bits")

    def step(self, i):
        import ptxstd
        x, q, sf = self.sets[i % 2]
        ptxstd.quantize_mxfp8(x, out=(q, sf), seed=0x5EED + i)
        return 1

    def e2e_compute(self, i, args):
        import ptxstd
        x, q, sf = args
        ptxstd.quantize_mxfp8(x, out=(q, sf), seed=0x5EED + i)
        return 1

    def cpu_sample(self, threads: int, budget_s: float):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        x = self.host_input()
        t0 = time.perf_counter()
        reps = 0
        while True:
            O.quantize_mxfp8_rs(x, 0x5EED + reps, threads)
            reps += 1
            el = time.perf_counter() - t0
            if el >= budget_s or reps >= 20:
                break
        return self.bytes * reps / el / 1e9, f"{reps} x full 8192x8192 stochastic quantise"


WORKLOADS = {"mxfp8_quantize": MxFp8Quantize, "fp8_gemm": Fp8Gemm, "nvfp4_gemm": Nvfp4Gemm,
             "decode_gemm": DecodeGemm, "decode_gemm_nccl": DecodeGemmNccl,
             "mxfp8_gemm": Mxfp8Gemm,
             "mxfp8_quantize_sr": MxFp8QuantizeSR, "mxfp8_gemm_sparse": Mxfp8SparseGemm,
             "mxfp6_gemm": MxFp6Gemm}


# ---- arms -----------------------------------------------------------------------------------

# Workloads measured in the same process after the headline one, each as its own record of the
# line's "workloads" object: the GEMM configurations (E4M3 8192^3, MXFP8 8192^3, NVFP4
# 8192 x 28672 x 8192 N-sharded, decode 16 x 57344 x 8192 N-sharded). On several ranks the decode
# is measured with both gathers: the fused peer-store one and the NCCL all-gather.
EXTRA_DEFAULT = ["fp8_gemm", "mxfp8_gemm", "nvfp4_gemm", "decode_gemm"]
EXTRA_MULTI = ["decode_gemm_nccl"]


def extra_workloads(args, world: int) -> list[str]:
    if args.extra == "none":
        return []
    if args.extra != "auto":
        return [w for w in args.extra.split(",") if w]
    if args.workload != "mxfp8_quantize":
        return []
    return EXTRA_DEFAULT + (EXTRA_MULTI if world > 1 else [])


class Ctx:
    """Run state shared by the workloads of one process: torch.distributed plumbing and the
    libptxstd communicator (created on first use; every rank creates it at the same point)."""

    def __init__(self, n_gpus: int):
        self.dist = Dist(n_gpus)
        self._pd = None

    def ptxstd_dist(self):
        if self._pd is None and self.dist.world > 1:
            from ptxstd.dist import Dist as PtxDist
            self._pd = PtxDist.from_torch()
        return self._pd

    def close(self):
        if self._pd is not None:
            import torch
            torch.cuda.synchronize()
            self._pd.close()
            self._pd = None
        self.dist.close()


def uses_graph(args, wl, world: int) -> bool:
    return not args.no_graph and not (world > 1 and getattr(wl, "collective", False))


def line_config(wl, world: int, graph: bool) -> dict:
    """The config dict of a record; both arms emit exactly this dict for the same workload."""
    return dict(wl.config, parallelism=getattr(wl, "parallelism", "replicas") + str(world),
                launch=("cuda-graph replay of the K steps, after one untimed replay that "
                        "uploads the graph") if graph else "eager")


def time_steps(args, ctx, step, graph: bool):
    """W warm-up steps, then K steps bracketed by a barrier and a synchronize on both sides,
    timed with CUDA events on the launching stream. With `graph` the K steps are captured once
    into a CUDA graph and replayed (after one untimed replay that uploads it), so that the device
    time is not padded by host-side launch gaps between short kernels; the multi-GPU decode's
    NCCL all-gather is issued by libptxstd on the same stream and is captured with it.
    The clock sampler runs over the timed steps and over about 20 ms of untimed passes of the same
    K steps just before them (the same number of passes on every rank). So the clock record is
    taken under load, and the timed steps start on a busy GPU, not after an idle pause: after 20 ms
    idle, the first steps of a short timed region ran about 3 % slower on a B200.
    Returns (device ms of the K steps, max over ranks; kernel launches; clock record)."""
    import torch
    dist = ctx.dist
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    one_pass = (time.perf_counter() - t0) / max(args.warmup, 1) * args.steps
    g = None
    launches = 0
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(args.steps):
                launches += step(i)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        g.replay()  # uploads the graph
        torch.cuda.synchronize()
        one_pass = time.perf_counter() - t0
    # untimed passes before the timed one: ~20 ms, the largest count any rank asks for
    pre = int(dist.max(float(min(50, max(1, int(0.02 / max(one_pass, 1e-6)) + 1)))))
    sampler = ClockSampler(torch.cuda.current_device()) if dist.rank == 0 else None
    if sampler:
        sampler.start()
    for _ in range(pre):
        if g is not None:
            g.replay()
        else:
            for i in range(args.steps):
                step(i)
    dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    if g is not None:
        g.replay()
    else:
        for i in range(args.steps):
            launches += step(i)
    ev1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms = ev0.elapsed_time(ev1)
    clocks = sampler.stop() if sampler else None
    if g is not None:
        del g  # a graph holding NCCL calls is released before the process group goes
    return dist.max(ms), launches, clocks


def time_e2e(args, ctx, wl) -> float:
    """End to end through the public API with host buffers: every step copies its inputs from
    pinned host memory and its results back. Two buffer slots are used in turn, with the copies
    on their own streams, so that step i+1's H2D and step i's D2H overlap step i's compute
    (PCIe carries both directions at once); events keep a slot's buffers from being reused before
    its previous step has finished with them. Returns ms of the K steps, max over ranks."""
    import torch
    dist = ctx.dist
    stream = torch.cuda.current_stream()
    slots = wl.e2e_slots(torch)
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()

    def run(n):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev_in = [torch.cuda.Event() for _ in range(n)]
        ev_run = [torch.cuda.Event() for _ in range(n)]
        ev_out = [torch.cuda.Event() for _ in range(n)]
        start.record(stream)
        h2d.wait_event(start)
        d2h.wait_event(start)
        for i in range(n):
            slot = slots[i % 2]
            with torch.cuda.stream(h2d):
                if i >= 2:
                    h2d.wait_event(ev_run[i - 2])  # inputs of step i-2 consumed
                for dev, host in slot["in"]:
                    dev.copy_(host, non_blocking=True)
                ev_in[i].record(h2d)
            stream.wait_event(ev_in[i])
            if i >= 2:
                stream.wait_event(ev_out[i - 2])  # outputs of step i-2 read back
            wl.e2e_compute(i, slot["args"])
            ev_run[i].record(stream)
            with torch.cuda.stream(d2h):
                d2h.wait_event(ev_run[i])
                for host, dev in slot["out"]:
                    host.copy_(dev, non_blocking=True)
                ev_out[i].record(d2h)
        stream.wait_event(ev_out[n - 1])
        end.record(stream)
        torch.cuda.synchronize()
        return start.elapsed_time(end)

    run(3)
    dist.barrier()
    ms = run(args.steps)
    dist.barrier()
    del slots
    return dist.max(ms)


def roofline(wl, per_launch_s: float) -> dict:
    peaks = measured_peaks()
    traffic = profiled_traffic(wl.kernel)
    if getattr(wl, "bound", "hbm") == "tensor":
        # Dense FP8 runs at twice the bf16 rate on B200 (4.5 vs 2.25 PFLOP/s nominal), FP4 at
        # four times; the denominator is the measured cuBLAS bf16 burst figure times that ratio.
        peak = peaks["bf16_tflops"] * wl.peak_ratio_to_bf16
        achieved = wl.flops / per_launch_s / 1e12
        return {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1),
                "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                "peak_source": f"{peaks['source']} bf16_tflops (cuBLAS burst) x "
                               f"{wl.peak_ratio_to_bf16} ({wl.peak_note})",
                "algorithmic_flops_per_launch": wl.flops}
    achieved = wl.bytes / per_launch_s / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
            "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
            "peak_source": peaks["source"] + " hbm_gbs (burst copy)",
            "algorithmic_bytes_per_launch": wl.bytes}


def measure(args, ctx, wl, cpu_budget_s: float = 3.0) -> dict | None:
    """One workload, set up, device-timed, clock-sampled, timed end to end and (one GPU only)
    timed on the host cores; returns its record on rank 0, None on the other ranks."""
    import torch
    world = ctx.dist.world
    wl.ctx = ctx
    torch.manual_seed(0)
    wl.setup(torch, wl.host_input())
    graph = uses_graph(args, wl, world)
    ms, launches, clocks = time_steps(args, ctx, wl.step, graph)
    split = None
    only = wl.gemm_only_step() if hasattr(wl, "gemm_only_step") else None
    if only is not None:
        ms_gemm, _, _ = time_steps(args, ctx, only, graph)
        split = {"gemm_us_per_step": round(ms_gemm * 1e3 / args.steps, 2),
                 "gather_us_per_step": round((ms - ms_gemm) * 1e3 / args.steps, 2),
                 "how": "the same K steps timed again with each rank's GEMM writing only its own "
                        "columns (no gather); gather = step - that"}
    e2e_ms = time_e2e(args, ctx, wl)
    if ctx.dist.rank != 0:
        return None
    per_step_s = ms / 1e3 / args.steps
    rec = {
        "value": round(wl.value(per_step_s) * world, 2), "unit": wl.unit,
        "ms_per_step": round(ms / args.steps, 5), "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": getattr(wl, "scaling", "weak"),
        "dtype": wl.dtype, "config": line_config(wl, world, graph),
        "roofline": roofline(wl, per_step_s),
        "e2e": {"value": round(wl.value(e2e_ms / 1e3 / args.steps) * world, 2),
                "unit": wl.unit, "h2d_bytes_per_step": wl.in_bytes,
                "d2h_bytes_per_step": wl.out_bytes},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if split is not None:
        rec["split"] = split
    if world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, sample = wl.cpu_sample(threads, budget_s=cpu_budget_s)
        rec["cpu_baseline"] = {"value": round(v, 3), "unit": wl.unit, "cores": threads,
                               "kind": "port", "sample": sample}
    return rec


def _release(wl):
    import torch
    if hasattr(wl, "teardown"):
        torch.cuda.synchronize()
        wl.teardown()
    wl.__dict__.clear()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def run_ours(args, wl) -> dict | None:
    ctx = Ctx(args.gpus)
    world = ctx.dist.world
    head = measure(args, ctx, wl)
    _release(wl)
    extras = {}
    for name in extra_workloads(args, world):
        sub = WORKLOADS[name](world)
        rec = measure(args, ctx, sub, cpu_budget_s=1.0)
        _release(sub)
        if rec is not None:
            extras[name] = rec
    rank = ctx.dist.rank
    ctx.close()
    if rank != 0:
        return None
    out = {"metric": METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
           "higher_is_better": True, "scaling": head["scaling"], "vs_baseline": None,
           "dtype": head["dtype"], "data": "synthetic (seeded)", "config": head["config"],
           "roofline": head["roofline"], "e2e": head["e2e"],
           "gpu_launches": head["gpu_launches"], "clocks": head["clocks"]}
    if "cpu_baseline" in head:
        out["cpu_baseline"] = head["cpu_baseline"]
    if extras:
        out["workloads"] = extras
    return out


def reference_record(args, wl, world: int, samples: int, warmup: int) -> tuple[dict, float]:
    threads = os.cpu_count() or 1
    for _ in range(warmup):
        wl.cpu_sample(threads, budget_s=0.0)
    vals, sample = [], ""
    for _ in range(samples):
        v, sample = wl.cpu_sample(threads, budget_s=0.0)
        vals.append(v)
    v = statistics.median(vals)
    what = ("the C restatement of the reference's conversion semantics (oracle/)"
            if wl.unit == "GB/s" and not hasattr(wl, "gather") else
            "a blocked f32 GEMM (oracle/) over operands decoded by the C restatement of the "
            "reference's conversions")
    rec = {"value": round(v, 3), "unit": wl.unit, "steps": samples, "warmup": warmup,
           "higher_is_better": True, "dtype": wl.dtype,
           "config": line_config(wl, world, uses_graph(args, wl, world)),
           "cpu_baseline": {"value": round(v, 3), "unit": wl.unit, "cores": threads,
                            "kind": "port",
                            "sample": f"per step: {sample}; {what}, all host threads"},
           "e2e": {"value": round(v, 3), "unit": wl.unit, "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    return rec, v


def run_reference(args, wl) -> dict | None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    head, _ = reference_record(args, wl, world, args.steps, args.warmup)
    out = {"metric": METRIC, "value": head["value"], "unit": wl.unit, "impl": "reference",
           "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
           "higher_is_better": True, "dtype": wl.dtype, "data": "synthetic (seeded numpy)",
           "config": head["config"], "cpu_baseline": head["cpu_baseline"], "e2e": head["e2e"]}
    extras = {}
    for name in extra_workloads(args, world):
        # a bounded sample per workload (one warm-up and up to 3 timed samples of a row block of
        # the GEMM) keeps the arm within minutes
        extras[name], _ = reference_record(args, WORKLOADS[name](world), world,
                                           min(args.steps, 3), 1)
    if extras:
        out["workloads"] = extras
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="mxfp8_quantize")
    ap.add_argument("--extra", default="auto",
                    help="comma-separated workloads measured after the headline one, each as a "
                         "record of the line's 'workloads' object; 'auto' (default) = the GEMM "
                         "configurations when the headline is mxfp8_quantize; 'none'")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch the timed steps eagerly instead of replaying a CUDA graph")
    ap.add_argument("--gather", choices=["p2p", "nccl"], default="p2p",
                    help="decode_gemm on several GPUs: output columns stored into every rank "
                         "over NVLink peer memory by the GEMM itself, or NCCL all-gather")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    wl = WORKLOADS[args.workload](world)
    if args.workload == "decode_gemm" and args.gather == "nccl":
        wl = DecodeGemmNccl(world)
    res = run_reference(args, wl) if args.impl == "reference" else run_ours(args, wl)
    if res is not None:
        print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
