"""Benchmark of the paged GQA decode-attention hot path on B200.

Default workload (the B=256 x 4096 decode point): B = 256 sequences x
kv_len 4096, 14 q / 2 kv heads, head_dim 64, 16-token pages scattered by a
random permutation over the pool, fp16 N(0, 1) data. One step = one call of
the decode-attention op over the batch (split-KV load, plus merge when the
split count is above 1).

Metric: algorithmic HBM GB/s = (K/V rows read + q read + o written +
block-table entries read) / time, summed over ranks (each rank owns its own
batch and KV pool: sequences are sharded, no collective on the data path).

Legs:
  value     device time (CUDA events on the launching stream) of K steps
            with all inputs resident; inputs (537 MB of K/V) exceed L2. The
            steps run as replays of CUDA graphs of 100 calls each, as the
            engine's captured decode steps do (--eager: Python launches).
  e2e       the same metric through the C ABI from HOST buffers, as the
            engine runs a decode step: the KV pool and block table are the
            engine's resident state in HBM (copied in once), and every step
            copies that step's own inputs -- q, the new K/V row of every
            sequence, the lengths and the slot ids -- from pinned host memory,
            writes the rows (cie_kv_decode_update), runs cie_decode_attention
            and reads o back. e2e.full_pool_copy: the whole 537 MB pool and
            the block table copied from the host every step (PCIe-bound).
  roofline  dominant kernel's achieved algorithmic GB/s / measured HBM peak.
  cpu_baseline  the CPU oracle (torch fp32 gather + softmax) on the host's
            cores over a bounded sample of the same workload.
  mixed     mixed attention (512-token chunks, config 3): device time, e2e
            through the C ABI, CPU oracle.
  sweep     config 2 (B x kv_len) and config 5 (split count) points, cold L2,
            beside the reference's own Triton kernels timed on the same GPU
            (``reference_triton``, baseline/time_reference_kernels.py).
  serving   the Qwen2.5-0.5B-shape model: closed-batch capacity, the Poisson
            workload of config 4 and the same requests all queued at the start
            (``saturated``, rate = inf).

``--impl reference`` times the reference attention math on the host CPU
(the oracle port: the reference engine ships no CPU kernel of its own and
its Triton kernels need a GPU) on the same config, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "paged decode-attn HBM GB/s (% peak)"
UNIT = "GB/s"
H_Q, H_KV, D, PAGE = 14, 2, 64, 16
FALLBACK_HBM_GBS = 6650.0


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--kv-len", type=int, default=4096)
    ap.add_argument("--splits", type=int, default=0, help="KV splits (0 = library default)")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--e2e-resident-steps", type=int, default=200,
                    help="steps of the e2e leg with the KV pool resident in HBM")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="bound on the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-mixed", action="store_true", help="skip the mixed-attention lines")
    ap.add_argument("--no-serving", action="store_true",
                    help="skip the Qwen2.5-0.5B-shape model line (serving tok/s)")
    ap.add_argument("--no-poisson", action="store_true",
                    help="skip the Poisson-arrival serving run (config 4)")
    ap.add_argument("--poisson-requests", type=int, default=64, help="requests per GPU")
    ap.add_argument("--poisson-rate", type=float, default=8.0, help="arrivals/s per GPU")
    ap.add_argument("--serve-batch", type=int, default=64, help="sequences per GPU")
    ap.add_argument("--serve-steps", type=int, default=128, help="timed decode steps")
    ap.add_argument("--eager", action="store_true",
                    help="launch every timed decode call from Python instead of replaying "
                         "CUDA graphs of them")
    ap.add_argument("--no-sweep", action="store_true",
                    help="skip the config-2 / config-5 sweep and the reference Triton timings "
                         "(run at N=1 only)")
    ap.add_argument("--lm-head-only", action="store_true",
                    help="print only the fused lm_head + argmax line (profiling)")
    ap.add_argument("--sweep", action="store_true",
                    help="print one JSON line per decode sweep point (configs 2 and 5) "
                         "instead of the benchmark line")
    return ap.parse_args(argv)


# ---------------------------------------------------------------------------
# distributed plumbing (one process per GPU, NCCL only for results)
# ---------------------------------------------------------------------------

def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def dist_barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def dist_max(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def dist_sum(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def dist_done(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# measurement helpers
# ---------------------------------------------------------------------------

def measured_peak_gbs():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic_per_launch(batch: int, kv_len: int):
    """(dram read+write bytes per launch of the decode kernel, source) from the
    committed ncu summary of this workload, or (None, reason)."""
    p = REPO / "profiles" / f"decode_split_kernel_b{batch}_l{kv_len}.md"
    if not p.exists():
        return None, "no committed ncu capture of this workload"
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", p.read_text())
    if not m:
        return None, "no traffic figure in " + str(p.relative_to(REPO))
    return int(m.group(1)), ("committed ncu capture of the same workload, "
                             + str(p.relative_to(REPO)) + " (not this run)")


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        self.lines = []
        self.index = self._smi_index(device_index)

    @staticmethod
    def _smi_index(device_index: int):
        """nvidia-smi index of torch device ``device_index`` (matched by PCI bus id)."""
        try:
            props = torch.cuda.get_device_properties(device_index)
            want = "%02x:%02x.0" % (int(props.pci_bus_id), int(props.pci_device_id))
            out = subprocess.run(["nvidia-smi", "--query-gpu=index,pci.bus_id",
                                  "--format=csv,noheader"], capture_output=True, text=True,
                                 timeout=30).stdout
        except Exception:
            return None
        for ln in out.splitlines():
            idx, _, pci = (x.strip() for x in ln.partition(","))
            if pci.lower().endswith(want):
                return idx
        if not os.environ.get("CUDA_VISIBLE_DEVICES"):
            return str(device_index)
        return None

    def __enter__(self):
        if self.index is None:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.5)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() in ("active", "1"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def decode_bytes(batch: int, kv_len: int) -> int:
    kv = batch * kv_len * H_KV * D * 2 * 2
    qo = batch * H_Q * D * 2 * 2
    bt = batch * math.ceil(kv_len / PAGE) * 8
    return kv + qo + bt


# ---------------------------------------------------------------------------
# CPU legs (oracle port)
# ---------------------------------------------------------------------------

def cpu_oracle_rate(kv_len: int, seconds: float, max_seqs: int = 1 << 20):
    """Times the fp32 CPU oracle on sequences of ``kv_len`` until ``seconds``
    elapse; returns (GB/s, threads, sample description)."""
    import oracle
    from custom_inference_engine_b200 import workloads as W
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    per = 4
    c = W.make_decode_case([kv_len] * per, seed=3)
    oracle.decode_attention_fp32(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)  # warm
    t0 = time.perf_counter()
    done = 0
    while done < max_seqs:
        oracle.decode_attention_fp32(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)
        done += per
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    nbytes = decode_bytes(done, kv_len)
    return nbytes / dt / 1e9, threads, f"{done} sequences x kv_len {kv_len} ({dt:.1f} s)"


def run_reference(args, rank, world):
    """--impl reference: the reference attention math on the host CPU."""
    if rank != 0:
        return None
    per_step = max(1, min(args.batch, 8))
    import oracle
    from custom_inference_engine_b200 import workloads as W
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    c = W.make_decode_case([args.kv_len] * per_step, seed=3)
    warm = max(3, min(args.warmup, 5))
    for _ in range(warm):
        oracle.decode_attention_fp32(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)
    t0 = time.perf_counter()
    steps = 0
    while steps < args.steps:
        oracle.decode_attention_fp32(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)
        steps += 1
        if time.perf_counter() - t0 > args.cpu_seconds * 4:
            break
    dt = time.perf_counter() - t0
    gbs = decode_bytes(per_step, args.kv_len) * steps / dt / 1e9
    sample = (f"{per_step} of {args.batch} sequences x kv_len {args.kv_len} per step, "
              f"{steps} steps")
    return {
        "metric": METRIC, "value": gbs, "unit": UNIT, "impl": "reference",
        "n_gpus": world, "steps": steps, "warmup": warm,
        "ms_per_step": dt / steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32 (fp16 inputs)", "data": "synthetic",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": gbs, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": gbs, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def workload_config(args, world):
    return {
        "workload": (f"paged GQA decode attention, B={args.batch} x kv_len {args.kv_len}, "
                     f"14q/2kv heads, D=64, page 16, random page permutation"),
        "batch_per_gpu": args.batch, "kv_len": args.kv_len, "heads_q": H_Q, "heads_kv": H_KV,
        "head_dim": D, "page_size": PAGE, "parallelism": f"sequence-sharded x{world}",
        "l2": "inputs larger than L2 (K/V pools %.0f MB per GPU)" % (
            args.batch * args.kv_len * 512 / 1e6),
    }


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------

L2_FLUSH_BYTES = 256 << 20   # twice the 126 MB L2
GRAPH_CHUNK = 100            # decode calls per captured graph in the timed loop


def time_launches(fn, iters: int, flush: bool, dev):
    """Per-call device time (ms) of ``fn`` with CUDA events on the current
    stream; with ``flush`` a buffer larger than L2 is read before each call,
    outside the timed pair (a read leaves no dirty lines to write back while
    the timed kernel runs)."""
    stream = torch.cuda.current_stream()
    scratch = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev) if flush else None
    pairs = []
    for _ in range(iters):
        if flush:
            scratch.sum()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        pairs.append((a, b))
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in pairs]


def bf16_peak_tflops(sustained: bool = False):
    p = REPO / "MEASURED_PEAKS.json"
    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    if p.exists():
        try:
            return float(json.loads(p.read_text())[key]), "measured " + key
        except Exception:
            pass
    return (1400.0 if sustained else 1590.0), "fallback"


def mixed_lines(dev, iters: int = 30, cpu: bool = True, e2e_steps: int = 50):
    """Mixed attention: the 512-token-chunk variant (tensor roofline) and
    config 3 (32 sequences, chunk 1 w.p. 0.5 else U[16,512], budget 2048).

    Per case: device time per call (L2 flushed before each call), ``e2e``
    through the C ABI with the step's own inputs from pinned host memory (q,
    cu_seqlens, kv_lens, slot ids in; o out; the K/V pool and block table stay
    resident in HBM, as the engine's KV cache does) and ``cpu_baseline``: the
    fp32 CPU oracle of the same call on the host's cores."""
    from custom_inference_engine_b200 import cabi
    from custom_inference_engine_b200 import workloads as W
    from custom_inference_engine_b200.attn import core
    out = {}
    g = torch.Generator().manual_seed(1)
    kv512 = torch.randint(0, 8193, (4,), generator=g).tolist()
    chunk3, kv3 = W.config3_shape(seed=0)
    cases = {
        "mixed_512_chunks": W.make_mixed_case([512] * 4, kv512, seed=1, device=dev,
                                              generate_on_device=True),
        "mixed_config3": W.make_mixed_case(chunk3, kv3, seed=0, device=dev, max_seqlen=2048,
                                           generate_on_device=True),
    }
    peak, src = bf16_peak_tflops()
    stream = torch.cuda.current_stream()
    for name, c in cases.items():
        def fn(c=c):
            core.gqa_mixed_attention_op(c.q, c.k, c.v, max_seqlen=c.max_seqlen,
                                        cu_seqlens=c.cu_seqlens, kv_lens=c.kv_lens,
                                        slot_ids=c.slot_ids, block_table=c.block_table)
        for _ in range(3):
            fn()
        ms = statistics.median(time_launches(fn, iters, flush=True, dev=dev))
        flops = c.causal_flops()
        tflops = flops / (ms / 1e3) / 1e12
        rec = {"ms_per_call": ms, "tflops": tflops, "causal_flops": flops,
               "tensor_frac": tflops / peak, "peak_tflops": peak, "peak_source": src,
               "hbm_gbs": c.algorithmic_bytes() / (ms / 1e3) / 1e9,
               "chunks": c.chunk_lens(), "kv_lens": c.kv_lens.tolist(),
               "l2": "flushed (256 MB read) before each call"}

        # e2e: the step's inputs from pinned host memory, o back to the host
        host = {n: getattr(c, n).cpu().pin_memory()
                for n in ("q", "cu_seqlens", "kv_lens", "slot_ids")}
        dbuf = {n: torch.empty_like(getattr(c, n)) for n in host}
        o_dev = torch.empty_like(c.q)
        o_host = torch.empty(c.q.shape, dtype=c.q.dtype).pin_memory()
        B, T = c.slot_ids.shape[0], c.q.shape[1]
        ws = torch.empty(cabi.mixed_workspace_bytes(B, T, H_KV, 0, dev.index) // 4 + 1,
                         dtype=torch.float32, device=dev)

        def e2e_step(c=c):
            for n in host:
                dbuf[n].copy_(host[n], non_blocking=True)
            cabi.mixed_attention(dbuf["q"], c.k, c.v, c.max_seqlen, dbuf["cu_seqlens"],
                                 dbuf["kv_lens"], dbuf["slot_ids"], c.block_table, out=o_dev,
                                 workspace=ws)
            o_host.copy_(o_dev, non_blocking=True)
        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / e2e_steps
        rec["e2e"] = {"value": flops / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s",
                      "ms_per_step": e2e_ms, "steps": e2e_steps,
                      "h2d_bytes_per_step": sum(t.numel() * t.element_size()
                                                for t in host.values()),
                      "d2h_bytes_per_step": o_host.numel() * o_host.element_size(),
                      "path": "cie_mixed_attention via ctypes; q, cu_seqlens, kv_lens and slot "
                              "ids copied in from pinned host memory and o read back every "
                              "step; K/V pool and block table resident in HBM"}
        if cpu:
            rec["cpu_baseline"] = mixed_cpu_rate(c)
        out[name] = rec
    return out


def mixed_cpu_rate(c, seconds: float = 6.0):
    """The fp32 CPU oracle on the same mixed call (all host cores): TFLOP/s."""
    import oracle
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    args = [t.cpu() for t in (c.q, c.k, c.v)]
    meta = [t.cpu() for t in (c.cu_seqlens, c.kv_lens, c.slot_ids, c.block_table)]
    t0 = time.perf_counter()
    n = 0
    while True:
        oracle.mixed_attention_fp32(args[0], args[1], args[2], c.max_seqlen, *meta)
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": c.causal_flops() / dt / 1e12, "unit": "TFLOP/s", "cores": threads,
            "kind": "port", "sample": f"{n} call(s) of the whole case, {dt * 1e3:.0f} ms each"}


def graph_time_cold(fn, dev, n: int = 20, reps: int = 5) -> float:
    """Device time (ms) of one ``fn`` call with a cold L2 and no launch gaps:
    a CUDA graph of ``n`` x [read a 256 MB buffer, fn] minus a graph of ``n``
    x [read the buffer], replayed ``reps`` times each (median)."""
    scratch = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    sink = torch.empty(n, dtype=torch.float32, device=dev)

    def capture(with_fn):
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            torch.sum(scratch, dim=0, out=sink[0])
            if with_fn:
                fn()
        torch.cuda.current_stream().wait_stream(side)
        with torch.cuda.graph(g):
            for i in range(n):
                torch.sum(scratch, dim=0, out=sink[i])
                if with_fn:
                    fn()
        return g

    def timed(g):
        out = []
        for _ in range(reps):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            out.append(a.elapsed_time(b))
        return statistics.median(out)

    g1, g0 = capture(True), capture(False)
    g1.replay()
    g0.replay()
    torch.cuda.synchronize()
    return max(timed(g1) - timed(g0), 0.0) / n


SWEEP_POINTS = ([(b, l, 0) for l in (512, 4096, 16384)
                 for b in (1, 2, 4, 8, 16, 32, 64, 128, 256)]
                + [(8, 32768, s) for s in (4, 8, 16, 32, 64)])


def sweep_points(dev, points=SWEEP_POINTS):
    """Config 2 (B x kv_len, default split count) and config 5 (8 x 32768 per
    GPU, split count swept) points, each timed on the device with a cold L2
    (``graph_time_cold``); one dict per point."""
    from custom_inference_engine_b200 import cabi
    from custom_inference_engine_b200 import workloads as W
    from custom_inference_engine_b200.attn import core
    peak, _ = measured_peak_gbs()
    out = []
    for B, L, S in points:
        c = W.make_decode_case([L] * B, seed=5, device=dev, generate_on_device=True)
        splits = S if S > 0 else cabi.decode_default_splits(B, dev.index)

        def fn():
            core.decode_gqa_attention(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table,
                                      num_programs=splits)
        for _ in range(3):
            fn()
        ms = graph_time_cold(fn, dev)
        nbytes = decode_bytes(B, L)
        gbs = nbytes / (ms / 1e3) / 1e9
        out.append({"sweep": "config5" if S else "config2", "batch": B, "kv_len": L,
                    "num_splits": splits, "us_per_call": ms * 1e3, "gbs": gbs,
                    "frac_of_measured_hbm": gbs / peak})
        del c
        torch.cuda.empty_cache()
    return out


def reference_triton_times(points: str = "sweep"):
    """The reference's own Triton kernels timed on this GPU by
    baseline/time_reference_kernels.py (a child process: the reference registers
    the same op names), or the reason they could not be."""
    script = REPO / "baseline" / "time_reference_kernels.py"
    if not (REPO / "baseline" / "_ref" / "attn" / "core.py").exists():
        return {"unavailable": "no copy of the reference in baseline/_ref "
                               "(baseline/install_reference.py)"}
    try:
        run = subprocess.run([sys.executable, str(script), "--points", points],
                             capture_output=True, text=True, timeout=900)
    except subprocess.TimeoutExpired:
        return {"unavailable": "timed out after 900 s"}
    if run.returncode != 0:
        return {"unavailable": (run.stderr.strip().splitlines() or ["exit %d" % run.returncode])[-1]}
    return json.loads(run.stdout.strip().splitlines()[-1])


def config1_point(dev, cpu: bool = True):
    """Config 1 itself: B = 8 sequences, kv_lens ~ U[1, 2048] (torch.Generator
    seed 0), one decode call timed with a cold L2, and the fp32 CPU oracle on
    the same call (all host cores)."""
    from custom_inference_engine_b200 import workloads as W
    from custom_inference_engine_b200.attn import core
    lens = W.config1_lens()
    c = W.make_decode_case(lens, seed=0, device=dev, generate_on_device=True)

    def fn():
        core.gqa_decode_attention_op(c.q, c.k, c.v, c.lens, slot_ids=c.slot_ids,
                                     block_table=c.block_table)
    for _ in range(3):
        fn()
    ms = graph_time_cold(fn, dev)
    nbytes = c.algorithmic_bytes()
    peak, _ = measured_peak_gbs()
    out = {"sweep": "config1", "batch": len(lens), "kv_lens": lens, "us_per_call": ms * 1e3,
           "gbs": nbytes / (ms / 1e3) / 1e9, "frac_of_measured_hbm": nbytes / (ms / 1e3) / 1e9 / peak,
           "algorithmic_bytes": nbytes}
    if cpu:
        import oracle
        threads = len(os.sched_getaffinity(0))
        torch.set_num_threads(threads)
        h = [t.cpu() for t in (c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table)]
        oracle.decode_attention_fp32(*h)
        t0, n = time.perf_counter(), 0
        while time.perf_counter() - t0 < 3.0:
            oracle.decode_attention_fp32(*h)
            n += 1
        dt = (time.perf_counter() - t0) / n
        out["cpu_baseline"] = {"value": nbytes / dt / 1e9, "unit": UNIT, "cores": threads,
                               "kind": "port", "sample": f"{n} calls, {dt * 1e3:.2f} ms each"}
    return out


def sweep_with_reference(dev, cpu: bool = True):
    """Our sweep points side by side with the reference Triton kernels' times
    for the points both measure (same workloads, same timing method)."""
    ours = [config1_point(dev, cpu)] + sweep_points(dev)
    ref = reference_triton_times("sweep")
    by_point = {}
    for r in ref.get("decode", []):
        by_point[(r["batch"], r["kv_len"], r["num_programs"])] = r
    for p in ours:
        if p["sweep"] == "config1":
            r = ref.get("config1")
        else:
            key = (p["batch"], p["kv_len"], p["num_splits"] if p["sweep"] == "config5" else 16)
            r = by_point.get(key)
        if r is not None:
            p["reference_triton_us"] = r["us_per_call"]
            p["speedup_vs_reference_triton"] = r["us_per_call"] / p["us_per_call"]
    return ours, ref


def run_sweep(args, dev):
    """--sweep: one JSON line per decode sweep point (configs 2 and 5)."""
    for p in sweep_points(dev):
        print(json.dumps(p), flush=True)


def lm_head_line(dev, batch: int = 64):
    """The last-token lm_head + argmax of a decode step at the Qwen2.5-0.5B
    shape (hidden 896, vocab 151936, ``batch`` rows): the fused one-pass
    kernel (inference::lm_head_argmax) against cuBLAS's GEMM followed by this
    package's argmax, each timed with a cold L2 (``graph_time_cold``). HBM
    roofline: the weight, the hidden rows and the tokens."""
    from custom_inference_engine_b200.attn import core  # noqa: F401  (loads the ops)
    V, H = 151936, 896
    g = torch.Generator(device=dev).manual_seed(9)
    w = (torch.randn(V, H, generator=g, device=dev) * 0.02).half()
    h = torch.randn(batch, H, generator=g, device=dev).half()
    ops = torch.ops.inference
    fused = lambda: ops.lm_head_argmax(h, w)
    gemm = lambda: ops.argmax_rows(torch.nn.functional.linear(h, w))
    assert torch.equal(fused(), ops.lm_head_argmax(h, w))
    for f in (fused, gemm):
        for _ in range(3):
            f()
    ms_f = graph_time_cold(fused, dev)
    ms_g = graph_time_cold(gemm, dev)
    nbytes = V * H * 2 + batch * H * 2 + batch * 8
    peak, kind = measured_peak_gbs()
    gbs = nbytes / (ms_f / 1e3) / 1e9
    return {"batch": batch, "vocab": V, "hidden": H, "fused_us": ms_f * 1e3,
            "gemm_plus_argmax_us": ms_g * 1e3, "algorithmic_bytes": nbytes,
            "fused_gbs": gbs, "frac_of_hbm": gbs / peak, "peak_source": f"{kind} hbm_gbs",
            "timing": "cold L2, CUDA graph of 20 calls minus the same graph without them"}


def serving_line(args, rank, world, dev):
    """Qwen2.5-0.5B-shape model through the paged ops (every rank its own replica).

    Random-init model (HF initialiser, N(0, 0.02), seed 0, fp16). Per GPU,
    ``serve_batch`` prompts of uniform random ids with lognormal lengths (median
    512, sigma 0.5, capped at 4096; seed 1000 + rank) are prefilled through the
    mixed op in passes of at most 2048 tokens (each a replay of the CUDA graph
    of its token bucket, captured before timing), then ``serve_steps`` greedy decode
    steps run as one CUDA graph each (embedding, 24 layers with the paged decode
    op and the KV scatter, lm_head, argmax). Decode tok/s = sequences x steps of
    all ranks / max-over-ranks device time; the last step's tokens are read back
    to the host."""
    import numpy as np
    from custom_inference_engine_b200 import model_runner as MR

    B, K = args.serve_batch, args.serve_steps
    cfg = MR.qwen2_config()
    model = MR.random_qwen2(cfg, seed=0, device=dev)
    rng = np.random.default_rng(1000 + rank)
    plens = np.clip(np.round(np.exp(rng.normal(np.log(512.0), 0.5, size=B))), 1, 4096).astype(int)
    prompts = [rng.integers(0, cfg.vocab_size, size=int(n)).tolist() for n in plens]
    warm = 3
    cap = [int(n) + warm + K + 1 for n in plens]
    runner = MR.PagedRunner(model, max_cache_len=sum(c + MR.PAGE_SIZE for c in cap),
                            n_slots=B + 1, token_budget=2048)
    slots = list(range(1, B + 1))
    for s, c in zip(slots, cap):
        runner.admit(s, c)
    runner.capture_mixed_graphs()
    stream = torch.cuda.current_stream()
    dist_barrier(world)
    torch.cuda.synchronize()
    p0 = torch.cuda.Event(enable_timing=True)
    p1 = torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    pre = runner.prefill(slots, prompts)
    p1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = dist_max(p0.elapsed_time(p1), world, dev)
    graph = runner.decode_graph(slots, pre.first_tokens, capture=True)
    for _ in range(warm):
        graph.step()
    torch.cuda.synchronize()
    dist_barrier(world)
    torch.cuda.synchronize()
    d0 = torch.cuda.Event(enable_timing=True)
    d1 = torch.cuda.Event(enable_timing=True)
    d0.record(stream)
    for _ in range(K):
        graph.step()
    d1.record(stream)
    last = graph.tokens.cpu()
    torch.cuda.synchronize()
    decode_ms = dist_max(d0.elapsed_time(d1), world, dev)
    out = {
        "model": "Qwen2.5-0.5B shape (24 layers, hidden 896, 14q/2kv heads, D 64, MLP 4864, "
                 "vocab 151936, tied), random init N(0, 0.02), fp16, greedy",
        "decode_tok_s": B * K * world / (decode_ms / 1e3),
        "decode_ms_per_step": decode_ms / K,
        "batch_per_gpu": B, "decode_steps": K,
        "prompt_tokens_per_gpu": int(plens.sum()),
        "prefill_tok_s": float(plens.sum()) * world / (prefill_ms / 1e3),
        "prefill_passes": pre.forward_passes,
        "last_tokens_read_back": int(last.numel()),
        "workload": "closed batch: lognormal prompts (median 512) prefilled through the mixed "
                    "op in 2048-token passes, then CUDA-graphed greedy decode through the decode "
                    "op; not the Poisson scheduler workload (no request queue)",
    }
    del graph, runner
    torch.cuda.empty_cache()
    if not args.no_poisson:
        out["poisson"] = poisson_line(args, model, rank, world, dev, args.poisson_rate)
        # rate = infinity: every request is there at the start (the reference
        # benchmark's headline mode, README.md:217-227): the engine's capacity
        out["saturated"] = poisson_line(args, model, rank, world, dev, float("inf"))
    del model
    torch.cuda.empty_cache()
    return out


def poisson_line(args, model, rank, world, dev, rate):
    """Config 4 as specified: one Poisson stream of ``rate`` x N requests/s
    (seed 2000; ``rate`` = inf: all requests at the start) of prompts with
    lognormal lengths (median 512, sigma 0.5, capped at 4096) and outputs of
    U[64, 512] tokens, sharded round-robin by index over the N GPUs (each GPU
    sees about ``rate`` requests/s over the same time window), served per GPU
    through the continuous-batching loop (serving.py): 33 slots, a 1024-token
    budget per step, a 32768-token KV pool per GPU. Metrics as the reference's
    benchmark (5 % trim per GPU; host wall clock, since they are request
    timestamps): tok/s = new tokens of all GPUs / (latest end - earliest
    planned arrival over the GPUs)."""
    from custom_inference_engine_b200 import model_runner as MR
    from custom_inference_engine_b200 import serving as SV

    n_slots, budget, pool_tokens = 33, 1024, 32768
    runner = MR.PagedRunner(model, max_cache_len=pool_tokens, n_slots=n_slots,
                            token_budget=budget)
    engine = SV.RunnerEngine(runner, n_slots)
    stream = SV.poisson_requests(args.poisson_requests * world, rate * world,
                                 seed=2000, vocab=model.config.vocab_size)
    reqs = stream[rank::world]
    torch.cuda.synchronize()
    dist_barrier(world)
    out, steps = SV.serve(engine, reqs, n_slots=n_slots, token_budget=budget)
    torch.cuda.synchronize()
    m = SV.summarize(out, trim=0.05)
    tokens = dist_sum(float(m["new_tokens"]), world, dev)
    first = -dist_max(-m["first_planned_s"], world, dev)
    duration = dist_max(m["last_end_s"], world, dev) - first
    res = {
        "tok_s": tokens / duration, "tok_s_rank0": m["tok_s"], "req_s_rank0": m["req_s"],
        "duration_s": duration, "new_tokens": int(tokens), "n_measured_rank0": m["n_measured"],
        "ttft_ms_rank0": m["ttft_ms"], "tpot_ms_rank0": m["tpot_ms"], "steps_rank0": steps,
        "tok_s_per_gpu": tokens / duration / world,
        "offered_tok_s": None if math.isinf(rate) else rate * world * 288.0,
        "workload": (f"Poisson {rate:g} req/s per GPU ({rate * world:g} req/s sharded "
                     f"round-robin over {world} GPU(s))" if not math.isinf(rate) else
                     "rate = inf (every request queued at the start)") +
                    f", {args.poisson_requests} "
                    f"requests per GPU, prompts lognormal (median 512, sigma 0.5, cap 4096), "
                    f"outputs U[64,512], {n_slots} slots, budget {budget}, KV {pool_tokens} "
                    f"tokens per GPU; 5% trim; host wall clock",
    }
    del engine, runner
    return res


def resident_pool_e2e(args, rank, world, dev, host, dbuf, out_dev, out_host, S, ws, nbytes,
                      stream):
    """The decode step as the engine runs it through the C ABI: the KV pool
    and block table stay in HBM across steps (copied in once from the pinned
    host copies by the full-copy leg), and each step copies the step's own
    host inputs -- q, one new K and V row per sequence, the per-slot lengths,
    the attended lengths and the slot ids -- from pinned host memory, writes
    the rows (cie_kv_decode_update, at row L-1 of every sequence so that the
    attended length stays L), runs cie_decode_attention and reads o back."""
    from custom_inference_engine_b200 import cabi, native

    B = host["q"].shape[1]
    g = torch.Generator().manual_seed(200 + rank)
    slot_lens = torch.zeros(dbuf["block_table"].shape[0], dtype=torch.int64)
    slot_lens[host["slot_ids"]] = host["lens"] - 1
    rows = {
        "q": host["q"],
        "k_new": torch.randn(1, B, H_KV, D, generator=g).half(),
        "v_new": torch.randn(1, B, H_KV, D, generator=g).half(),
        "slot_lens": slot_lens,
        "lens": host["lens"],
        "slot_ids": host["slot_ids"],
    }
    # One pinned staging buffer holds the step's inputs (256-byte aligned
    # pieces) and crosses in one copy. Two device copies of it and two
    # output buffers let step i+1's inputs and step i-1's output cross while
    # step i computes: H2D and D2H on their own streams, ordered by events.
    offs, o = {}, 0
    for n, t in rows.items():
        offs[n] = o
        o += (t.numel() * t.element_size() + 255) // 256 * 256
    h_stage = torch.empty(o, dtype=torch.uint8).pin_memory()
    for n, t in rows.items():
        nb = t.numel() * t.element_size()
        h_stage[offs[n]:offs[n] + nb].view(t.dtype).view(t.shape).copy_(t)
    d_stage = [torch.empty(o, dtype=torch.uint8, device=dev) for _ in range(2)]
    rbufs = [{n: d[offs[n]:offs[n] + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
              for n, t in rows.items()} for d in d_stage]
    outs_dev = [out_dev, torch.empty_like(out_dev)]
    outs_host = [out_host, torch.empty(out_host.shape, dtype=out_host.dtype).pin_memory()]
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    out_read = [torch.cuda.Event() for _ in range(2)]

    def one(i):
        b = i & 1
        r = rbufs[b]
        with torch.cuda.stream(h2d_s):
            h2d_s.wait_event(done[b])        # step i-2 has finished reading d_stage[b]
            d_stage[b].copy_(h_stage, non_blocking=True)
            in_ready[b].record(h2d_s)
        stream.wait_event(in_ready[b])
        stream.wait_event(out_read[b])       # step i-2's output has left outs_dev[b]
        cabi.kv_decode_update(dbuf["k"], dbuf["v"], r["slot_lens"], r["slot_ids"],
                              dbuf["block_table"], r["k_new"], r["v_new"])
        cabi.decode_attention(r["q"], dbuf["k"], dbuf["v"], r["lens"], r["slot_ids"],
                              dbuf["block_table"], out=outs_dev[b], num_splits=S, workspace=ws)
        done[b].record(stream)
        with torch.cuda.stream(d2h_s):
            d2h_s.wait_event(done[b])
            outs_host[b].copy_(outs_dev[b], non_blocking=True)
            out_read[b].record(d2h_s)

    def run(n):
        h2d_s.wait_stream(stream)
        d2h_s.wait_stream(stream)
        for i in range(n):
            one(i)
        stream.wait_stream(h2d_s)
        stream.wait_stream(d2h_s)

    steps = max(1, args.e2e_resident_steps)
    run(3)
    torch.cuda.synchronize()
    dist_barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run(steps)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = dist_max(e0.elapsed_time(e1), world, dev)
    return {
        "value": nbytes * world * steps / (ms / 1e3) / 1e9, "unit": UNIT,
        "h2d_bytes_per_step": h_stage.numel(),
        "d2h_bytes_per_step": out_host.numel() * out_host.element_size(), "steps": steps,
        "path": ("decode step through the C ABI as the engine runs it: KV pool and block "
                 "table resident in HBM (the engine's KV cache, copied in once); per step "
                 "the step's inputs -- q, the new K/V rows, lengths and slot ids -- in one "
                 "copy from pinned host memory, cie_kv_decode_update + cie_decode_attention "
                 "via ctypes, o read back; copies of neighbouring steps overlap the step's "
                 "kernels (two buffers, copy streams)"),
        "device_error_bits": native.device_errors(dev.index, clear=True),
    }


def run_ours(args, rank, world, local):
    from custom_inference_engine_b200 import cabi, native
    from custom_inference_engine_b200 import workloads as W
    from custom_inference_engine_b200.attn import core

    dev = torch.device("cuda", torch.cuda.current_device())
    B, L = args.batch, args.kv_len
    c = W.make_decode_case([L] * B, seed=100 + rank, device=dev, generate_on_device=True)
    S = args.splits if args.splits > 0 else cabi.decode_default_splits(B, dev.index)
    launches_per_step = 1 if S == 1 else 2
    native.device_errors(dev.index, clear=True)

    def step():
        return core.decode_gqa_attention(c.q, c.k, c.v, c.lens, c.slot_ids, c.block_table,
                                         num_programs=S)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    # The engine calls the decode op inside CUDA graphs (one per decode step),
    # so by default the timed steps are replays of a graph of `chunk`
    # consecutive calls (plus one graph for a remainder); --eager launches
    # every call from Python instead.
    chunk = min(args.steps, GRAPH_CHUNK)
    graphs = []
    if not args.eager:
        for n in ([chunk] * (args.steps // chunk) + ([args.steps % chunk] if args.steps % chunk else [])):
            if graphs and n == chunk:
                graphs.append(graphs[0])
                continue
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(n):
                    step()
            g.replay()
            graphs.append(g)
        torch.cuda.synchronize()
    events = [torch.cuda.Event(enable_timing=True)
              for _ in range((len(graphs) if graphs else args.steps) + 1)]
    dist_barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clocks:
        events[0].record(stream)
        if graphs:
            for i, g in enumerate(graphs):
                g.replay()
                events[i + 1].record(stream)
        else:
            for i in range(args.steps):
                step()
                events[i + 1].record(stream)
        torch.cuda.synchronize()
    dist_barrier(world)
    torch.cuda.synchronize()
    local_ms = events[0].elapsed_time(events[-1])
    total_ms = dist_max(local_ms, world, dev)
    nbytes = decode_bytes(B, L)
    value = nbytes * world * args.steps / (total_ms / 1e3) / 1e9
    kernel_ms = local_ms / args.steps  # every step is one decode call on this stream
    achieved = nbytes / (kernel_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak_gbs()
    traffic, traffic_src = ncu_traffic_per_launch(B, L)
    errs = native.device_errors(dev.index, clear=True)

    # ---- e2e: C ABI with host buffers ---------------------------------------
    host = {n: getattr(c, n).cpu().pin_memory()
            for n in ("q", "k", "v", "lens", "slot_ids", "block_table")}
    dbuf = {n: torch.empty_like(getattr(c, n)) for n in host}
    out_dev = torch.empty_like(c.q)
    out_host = torch.empty(c.q.shape, dtype=c.q.dtype).pin_memory()
    ws_bytes = cabi.decode_workspace_bytes(B, H_Q, D, S)
    ws = torch.empty(max(ws_bytes // 4, 1), dtype=torch.float32, device=dev)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_host.numel() * out_host.element_size()

    def e2e_step():
        for n in host:
            dbuf[n].copy_(host[n], non_blocking=True)
        cabi.decode_attention(dbuf["q"], dbuf["k"], dbuf["v"], dbuf["lens"], dbuf["slot_ids"],
                              dbuf["block_table"], out=out_dev, num_splits=S,
                              workspace=ws if ws_bytes else None)
        out_host.copy_(out_dev, non_blocking=True)

    e2e_steps = max(1, args.e2e_steps)
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    dist_barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = dist_max(e0.elapsed_time(e1), world, dev)
    e2e_value = nbytes * world * e2e_steps / (e2e_ms / 1e3) / 1e9
    ok = torch.equal(out_host, step().cpu())
    resident = resident_pool_e2e(args, rank, world, dev, host, dbuf, out_dev, out_host, S,
                                 ws if ws_bytes else None, nbytes, stream)
    serving = None if args.no_serving else serving_line(args, rank, world, dev)

    result = None
    if rank == 0:
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16 in / fp32 accumulate", "data": "synthetic",
            "config": workload_config(args, world),
            "value_per_gpu": value / world,
            "num_splits": S,
            "timing": ("eager: one Python launch per call" if args.eager else
                       f"CUDA graphs of {chunk} consecutive decode calls, replayed "
                       f"(the engine's decode steps are CUDA graphs)"),
            "pct_of_peak": 100.0 * achieved / peak,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                         "traffic": traffic, "traffic_source": traffic_src,
                         "algorithmic_bytes_per_launch": nbytes,
                         "kernel": "decode_split_kernel<2>" + (" + decode_merge_kernel"
                                                               if S > 1 else "")},
            "e2e": dict(resident, full_pool_copy={
                "value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "path": "cie_decode_attention via ctypes; every step copies q, both K/V "
                        "pools, lens, slot ids and the block table from pinned host memory "
                        "and reads o back (PCIe-bound: the whole pool crosses every step)",
                "output_matches_device_leg": bool(ok)}),
            "gpu_launches": args.steps * launches_per_step,
            "clocks": clocks.summary(),
            "device_error_bits": errs,
        }
        if serving is not None:
            result["serving"] = serving
        if not args.no_mixed:
            # after the serving legs: the CPU oracle it times leaves busy
            # host threads behind, which slowed the host-bound prefill leg
            result["mixed"] = mixed_lines(dev, cpu=world == 1 and not args.no_cpu_baseline)
        if world == 1 and not args.no_sweep:
            result["sweep"], ref = sweep_with_reference(dev, cpu=not args.no_cpu_baseline)
            result["reference_triton"] = ref
            result["lm_head"] = lm_head_line(dev)
        if not args.no_cpu_baseline and world == 1:
            gbs, cores, sample = cpu_oracle_rate(L, args.cpu_seconds)
            result["cpu_baseline"] = {"value": gbs, "unit": UNIT, "cores": cores, "kind": "port",
                                      "sample": sample}
    return result


def main(argv=None):
    args = parse_args(argv)
    rank, world, local = dist_setup(args)
    try:
        if args.sweep:
            if rank == 0:
                run_sweep(args, torch.device("cuda", torch.cuda.current_device()))
            res = None
        elif args.lm_head_only:
            res = lm_head_line(torch.device("cuda", torch.cuda.current_device())) \
                if rank == 0 else None
        elif args.impl == "reference":
            res = run_reference(args, rank, world)
        else:
            res = run_ours(args, rank, world, local)
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
    finally:
        dist_done(world)


if __name__ == "__main__":
    main()
