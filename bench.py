"""Benchmark: embedding tokens/s of the GPU-worker forward pass on B200.

Workload (default, ``--workload c2``): Qwen3-Embedding-0.6B architecture, AWQ int4 weights
(group 128, seeded synthetic), one packed varlen batch of 20 sequences x 1000 tokens,
tensor parallel over ``--gpus`` ranks (TP=1 by default).  A step is one forward pass over
the batch: embedding -> 28 decoder layers -> final norm (``value``), plus last-token
pooling + L2 normalisation and the host copies for ``e2e``.

* ``value``: tokens/s with the batch resident in HBM, device time from CUDA events,
  barrier + synchronize around the K timed steps, max over ranks.
* ``e2e``: the same batch through ``GPUWorker.embed`` (the reference's ``_inference`` +
  post-process): pinned host ids/positions copied in, fp32 embeddings copied out, every
  step.
* ``roofline``: the AWQ GEMM (the dominant kernel), FLOPs of every launch in the timed
  region / CUDA-event time of those launches, against the measured dense bf16 peak.
* ``cpu_baseline``: the reference's torch forward as the CPU oracle restates it, in bf16 on
  the workload's dequantised AWQ checkpoint, over a bounded sample of the batch (2 of its
  sequences through every layer) on all host cores: one warm-up, median of 3.

``--impl reference`` times that CPU forward alone (rank 0; other ranks exit), one sample
per step, and prints the same metric.  Run multi-GPU as
``python -m torch.distributed.run --nproc-per-node N bench.py --gpus N``.
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
sys.path.insert(0, ROOT)

METRIC = "embedding tokens/sec (20x1000-tok batch)"

# DRAM bytes (read + write) of one launch of the kernel, from an `ncu --set full` capture of
# the same launch shape on one B200 (`--workload c3`, cold L2); None where not captured.
MEASURED_TRAFFIC: dict = {
    # gate_up + SiLU-and-mul on the weight panel (CTA-pair kernel), M = 20000
    ("silu", 20000, 6144, 1024): 133.0e6,
}
UNIT = "tokens/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["mes", "reference"], default="mes")
    ap.add_argument("--workload", choices=["c2", "c3", "c4", "c5", "ew"], default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the varying-batch e2e stream and the last-rows variant")
    ap.add_argument("--parallel", choices=["tp", "dp"], default="tp",
                    help="tp: one batch sharded over the ranks (tensor parallel, the "
                         "reference's layout); dp: every rank a full replica on its own batch")
    ap.add_argument("--gemm-shapes", default="qkv,o,gate_up,down",
                    help="c3 only: comma list of projection shapes to time")
    ap.add_argument("--gemm-m", default="16,256,2048,20000,120000",
                    help="c3 only: comma list of token counts M")
    ap.add_argument("--gemm-epilogue", choices=["bf16", "silu", "residual"], default="bf16",
                    help="c3 only: GEMM epilogue")
    return ap.parse_args()


def workload(name: str):
    from mes_b200 import synthetic
    if name == "c2":
        cfg = synthetic.qwen3_0_6b()
        lengths = [1000] * 20
        desc = "Qwen3-Embedding-0.6B arch, AWQ int4 g128, 20 x 1000 tokens"
    elif name == "c4":
        cfg = synthetic.qwen3_8b()
        lengths = synthetic.lengths_log_uniform(120000, 64, 4096, seed=1)
        desc = "Qwen3-Embedding-8B arch, AWQ int4 g128, 120000 tokens, log-uniform [64, 4096]"
    else:
        cfg = synthetic.qwen2_1_5b()
        lengths = synthetic.lengths_uniform(64, 16, 512, seed=1)
        desc = "Qwen2-1.5B arch, AWQ int4 g128, 64 seqs uniform [16, 512]"
    return cfg, lengths, desc


# ---------------------------------------------------------------------------- helpers
def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), d["hbm_gbs"], "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons during the timed region: NVML read every
    20 ms from a thread, with one sample taken before the region starts and one after it
    ends, so that even a region shorter than the period is covered (the fields are those of
    nvidia-smi's clocks.sm, clocks.max.sm and clocks_event_reasons.*).  Falls back to
    ``nvidia-smi -lms 200`` when NVML cannot be loaded.  Only reads; sets nothing."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_S = 0.02
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []
        self.nvml, self.samples, self.smax = None, [], None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = self._nvml_handle(pynvml)
            self.smax = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
            self.bits = [pynvml.nvmlClocksEventReasonHwSlowdown,
                         pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                         pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                         pynvml.nvmlClocksEventReasonSwPowerCap]
            self._sample()
            self.stop = threading.Event()
            self.t = threading.Thread(target=self._loop, daemon=True)
            self.t.start()
            return self
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _nvml_handle(self, pynvml):
        """NVML handle of CUDA device ``index`` (NVML numbers every GPU of the host, CUDA only
        the visible ones: match them by PCI address)."""
        try:
            import torch
            p = torch.cuda.get_device_properties(self.index)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _sample(self):
        nv = self.nvml
        sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
        reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        self.samples.append((float(sm), int(reasons)))

    def _loop(self):
        while not self.stop.wait(self.PERIOD_S):
            try:
                self._sample()
            except Exception:
                return

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.nvml is not None:
            self.stop.set()
            self.t.join(timeout=5)
            try:
                self._sample()
                self.nvml.nvmlShutdown()
            except Exception:
                pass
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, smax, reasons = [], self.smax, set()
        for clk, bits in self.samples:
            sm.append(clk)
            for n, bit in zip(self.NAMES, self.bits):
                if bits & bit:
                    reasons.add(n)
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(self.NAMES, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvml" if self.samples else "nvidia-smi"}


CPU_SAMPLE_SEQS = 2   # sequences of the workload's batch in one CPU sample


class CpuReferenceSample:
    """The reference's torch forward, restated by the CPU oracle (``oracle/model.py``,
    following ``models/qwen3.py`` / ``qwen2.py`` line by line), on a bounded sample of the
    workload: the first ``CPU_SAMPLE_SEQS`` sequences of the batch through every layer, in
    bf16 (the reference's deployment dtype), with the workload's seeded AWQ checkpoint
    dequantised exactly to dense weights (what the reference runs for a dequantised
    checkpoint; it has no AWQ path).  One ``step()`` is one such forward."""

    def __init__(self, cfg, lengths, threads: int):
        import torch
        from mes_b200 import synthetic
        from oracle import model as omodel
        torch.set_num_threads(threads)
        self.cfg, self.threads, self.omodel = cfg, threads, omodel
        self.lengths = list(lengths[:CPU_SAMPLE_SEQS])
        dense = omodel.awq_dense_weights(synthetic.awq_weights(cfg, seed=0, device="cpu"))
        self.weights = {k: v.to(torch.bfloat16) for k, v in dense.items()}
        del dense
        ids, pos, last = synthetic.packed_batch(self.lengths, cfg.vocab_size, seed=1)
        self.ids, self.pos, self.last = (torch.from_numpy(a) for a in (ids, pos, last))
        self.qk_norm = not synthetic.is_qwen2(cfg)
        self.tokens = int(sum(self.lengths))

    def step(self):
        import torch
        return self.omodel.embed(self.cfg, self.weights, self.ids, self.pos, self.last,
                                 qk_norm=self.qk_norm, dtype=torch.bfloat16)

    def describe(self) -> str:
        return (f"{len(self.lengths)} of the batch's sequences ({self.tokens} tokens) through "
                f"all {self.cfg.num_hidden_layers} layers per step, bf16, the workload's AWQ "
                f"checkpoint dequantised to dense weights, torch on {self.threads} host threads")

    def timed(self, warmup: int, repeats: int):
        """Median wall time (s) of `repeats` forwards after `warmup` untimed ones."""
        for _ in range(warmup):
            self.step()
        times = []
        for _ in range(repeats):
            t0 = time.perf_counter()
            self.step()
            times.append(time.perf_counter() - t0)
        return statistics.median(times), times


def cpu_baseline_entry(cfg, lengths, threads: int) -> dict:
    """``cpu_baseline`` of the GPU line: one warm-up, then the median of 3 forwards of the
    CPU sample (the same measurement as ``--impl reference``)."""
    sample = CpuReferenceSample(cfg, lengths, threads)
    med, times = sample.timed(warmup=1, repeats=3)
    return {"value": sample.tokens / med, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": sample.describe() + "; 1 warm-up, median of 3",
            "seconds_per_sample": times}


# ---------------------------------------------------------------------------- reference arm
def run_reference(args):
    """The reference arm: the CPU forward of ``CpuReferenceSample`` on all host threads,
    one sample per step (W untimed, K timed, each timed separately; value = tokens of a
    sample / median step time).  Rank 0 only; other ranks exit without work."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg, lengths, desc = workload(args.workload)
    threads = os.cpu_count() or 1
    sample = CpuReferenceSample(cfg, lengths, threads)
    steps = max(args.steps, 1)
    med, times = sample.timed(warmup=args.warmup, repeats=steps)
    value = sample.tokens / med
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup,
        "ms_per_step": med * 1000, "ms_per_step_is": "median wall time of one timed sample",
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded AWQ checkpoint, dequantised; seeded token ids)",
        "config": {"workload": desc, "tokens": sum(lengths), "sequences": len(lengths),
                   "sample_tokens": sample.tokens, "sample_sequences": len(sample.lengths)},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample.describe()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------- GPU arm
def run_mes(args):
    import torch
    import torch.distributed as dist

    import __graft_entry__
    __graft_entry__.build()
    from mes_b200 import _C, synthetic
    from mes_b200.core.gpu_worker import GPUWorker
    from mes_b200.schemas.config import MESConfig
    from mes_b200.ultils.loader import load_weights

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dp = args.parallel == "dp"
    import datetime
    if world > 1 and not dp:
        from mes_b200.core.gpu_worker import tp_nccl_environment
        tp_nccl_environment()
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))

    cfg, lengths, desc = workload(args.workload)
    ids, pos, last = synthetic.packed_batch(lengths, cfg.vocab_size, seed=1)
    T = len(ids)

    # Data-parallel replicas: the model is built before the process group exists, so it
    # is not sharded; the group only carries the barriers and the max over ranks.
    worker = GPUWorker(MESConfig(model_config=cfg), device=dev)
    if world > 1 and dp:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    # Seeded synthetic weights generated on the device (same seed on every rank; each
    # rank's loaders keep only its shard).
    weights = synthetic.awq_weights(cfg, seed=0, device=dev)
    load_weights(worker.model, weights)
    del weights
    torch.cuda.empty_cache()

    ids_d = torch.from_numpy(ids).to(dev)
    pos_d = torch.from_numpy(pos).to(dev)
    model = worker.model

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    def gemm_times(events):
        by_shape = {}
        for a, b, f, key in events:
            d = by_shape.setdefault(key, [0, 0.0, 0.0])
            d[0] += 1
            d[1] += a.elapsed_time(b)
            d[2] += f
        return by_shape

    from mes_b200.models.qwen2 import DecoderModel
    layout = worker.layout(pos, exact=True)   # the batch's own layout: no padding
    split = layout.split

    with torch.no_grad():
        # Eager warm-up; the last step records CUDA events around every GEMM: the dominant
        # GEMM shape and the GEMMs' share of a step.
        for _ in range(args.warmup - 1):
            model(ids_d, pos_d, overlap_split=split)
        _C.gemm_events, _C.gemm_event_kinds = [], None
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record()
        model(ids_d, pos_d, overlap_split=split)
        p1.record()
        barrier()
        probe = gemm_times(_C.gemm_events)
        gemm_share = sum(v[1] for v in probe.values()) / p0.elapsed_time(p1)
        probe_key = max(probe.items(), key=lambda kv: kv[1][1])[0]

        # The step as the server runs it: one forward captured as a CUDA graph (the
        # launches of ~230-450 kernels from Python would otherwise set the pace once the
        # forward is split over several GPUs).  Events around the dominant kind's GEMMs are
        # captured with it, so every replay times those launches on their stream.
        _C.gemm_events, _C.gemm_event_kinds = [], {probe_key[0]}
        launches0 = _C.launch_count
        graph, ids_s, pos_s, _, _ = worker.capture(layout, ids, pos)
        launches = (_C.launch_count - launches0) // 2   # capture() runs the forward twice
        captured = _C.gemm_events[len(_C.gemm_events) // 2:]
        _C.gemm_events, _C.gemm_event_kinds = None, None
        graph.replay()
        barrier()

        # ---- device-resident timed region (value) -----------------------------------
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            barrier()
            ev0.record()
            for _ in range(args.steps):
                graph.replay()
            ev1.record()
            barrier()
        dt = max_over_ranks(ev0.elapsed_time(ev1) / 1000.0)
        # The captured events hold the last timed replay's launches.
        by_shape = gemm_times(captured)
        top_key, (top_n, top_ms, top_flops) = max(by_shape.items(), key=lambda kv: kv[1][1])
        top_n *= args.steps   # per-step launch count below divides by steps
        del graph

        # ---- end-to-end through the public API (e2e) --------------------------------
        # Warm-up: the batch's first occurrences replay its token bucket's graph; from the
        # `exact_after`-th on, a graph of its exact layout (no padding).
        for _ in range(worker.exact_after + 1):
            worker.embed(ids, pos, last)
        barrier()
        t0 = time.perf_counter()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            out = worker.embed(ids, pos, last)
        e1.record()
        barrier()
        e2e_dt = max_over_ranks(max(e0.elapsed_time(e1) / 1000.0, time.perf_counter() - t0))

        # ---- e2e over a stream of batches of varying size (the server's case) ---------
        varying = None
        if args.workload == "c2" and not args.no_extras:
            varying = run_varying_stream(worker, cfg, barrier, max_over_ranks,
                                         replicas=world if dp else 1)

        # ---- flagged variant: the last layer on the pooled rows only ----------------
        last_rows = None
        if split == DecoderModel.NO_SPLIT and not args.no_extras:
            last_rows = run_last_rows(worker, ids, pos, last, args, barrier, max_over_ranks,
                                      replicas=world if dp else 1)

    err = _C.take_device_error()
    if err:
        raise RuntimeError(f"device error {err} during the benchmark")

    peak_burst, peak_sust, hbm, peak_kind = peaks()
    # Dominant kernel: the AWQ GEMM launch shape with the most device time in the timed
    # region; FLOPs per launch / mean CUDA-event duration of those launches.
    achieved = top_flops / (top_ms / 1000.0) / 1e12 if top_ms > 0 else 0.0
    kind, gm, gn, gk = top_key
    result = None
    if rank == 0:
        replicas = world if dp else 1     # each dp rank processes its own batch
        value = replicas * T * args.steps / dt
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            cpu = cpu_baseline_entry(cfg, lengths, os.cpu_count() or 1)
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt / args.steps * 1000, "higher_is_better": True,
            "scaling": "weak" if dp else "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded AWQ weights and token ids)",
            "config": {"workload": desc, "tokens": T * replicas, "sequences": len(lengths) * replicas,
                       "parallelism": f"dp{world}" if dp else f"tp{world}",
                       "l2": "inputs larger than L2 (weights + activations > 126 MB per step)"},
            "e2e": {"value": replicas * T * args.steps / e2e_dt, "unit": UNIT,
                    "h2d_bytes_per_step": int(ids.nbytes + pos.nbytes + last.nbytes),
                    "d2h_bytes_per_step": int(out.numel() * 4)},
            "e2e_varying": varying,
            "last_rows_only": last_rows,
            "gpu_launches": launches * args.steps,
            "cuda_graph": True,
            "roofline": {"kernel": f"awq_gemm ({kind} epilogue) M={gm} N={gn} K={gk}",
                         "launches": top_n // args.steps, "bound": "tensor",
                         "achieved": achieved, "peak": peak_sust,
                         "peak_kind": f"{peak_kind} bf16 sustained", "unit": "TFLOP/s",
                         "frac": achieved / peak_sust,
                         "traffic": MEASURED_TRAFFIC.get((kind, gm, gn, gk)),
                         "traffic_unit": "bytes per launch (ncu dram read+write)",
                         "all_gemm_share_of_step": gemm_share,
                         "all_gemm_share_from": "the last warm-up step"},
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(result), flush=True)
    # CUDA graphs that hold NCCL work are released before the process group goes.
    worker.release_graphs()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def run_last_rows(worker, ids, pos, last, args, barrier, max_over_ranks, replicas: int = 1):
    """Flagged variant (not the headline): the same batch with the last layer's o_proj, MLP
    and final norm computed for the B pooled rows only (``DecoderModel.forward_last_rows``;
    the embeddings are unchanged).  ``value``: CUDA-graph replays with the batch resident,
    CUDA events; ``e2e``: ``GPUWorker.embed`` in last-rows mode with host buffers."""
    import time as _time
    import torch
    T = len(ids)
    lay = worker.layout(pos, exact=True)
    n_rows = -(-len(last) // 16) * 16
    graph, _, _, rows_s, _ = worker.capture(lay, ids, pos, n_rows)
    rows = torch.zeros(n_rows, dtype=torch.int64)
    rows[:len(last)] = torch.from_numpy(last)
    rows_s.copy_(rows)
    for _ in range(2):
        graph.replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    barrier()
    dt = max_over_ranks(e0.elapsed_time(e1) / 1000.0)
    del graph
    worker.last_rows_only = True
    try:
        for _ in range(3):
            worker.embed(ids, pos, last)
        barrier()
        t0 = _time.perf_counter()
        for _ in range(args.steps):
            worker.embed(ids, pos, last)
        barrier()
        e2e_dt = max_over_ranks(_time.perf_counter() - t0)
    finally:
        worker.last_rows_only = False
    return {"value": replicas * T * args.steps / dt, "unit": UNIT,
            "ms_per_step": dt / args.steps * 1000,
            "e2e": {"value": replicas * T * args.steps / e2e_dt, "unit": UNIT},
            "flag": "last layer's o_proj, MLP and final norm on the pooled rows only "
                    "(same embeddings; not the headline number)"}


def run_varying_stream(worker, cfg, barrier, max_over_ranks, replicas: int = 1,
                       n_batches: int = 16):
    """``GPUWorker.embed`` over a seeded stream of batches of 20 sequences with lengths
    uniform in [500, 1500] (10-30 k tokens per batch, a different total each time), as the
    engine's batcher produces them.  The first pass includes the CUDA-graph captures of the
    token buckets it meets; the second pass replays them (steady state).  Wall time, max
    over ranks; tokens/s counts real tokens only."""
    import time as _time
    from mes_b200 import synthetic
    batches = []
    for i in range(n_batches):
        lens = synthetic.lengths_uniform(20, 500, 1500, seed=100 + i)
        batches.append(synthetic.packed_batch(lens, cfg.vocab_size, seed=200 + i))
    tokens = sum(len(b[0]) for b in batches)
    out = {}
    for name in ("first_pass", "steady"):
        c0 = worker.captures
        barrier()
        t0 = _time.perf_counter()
        for ids, pos, last in batches:
            worker.embed(ids, pos, last)
        barrier()
        dt = max_over_ranks(_time.perf_counter() - t0)
        out[name] = {"value": replicas * tokens / dt, "captures": worker.captures - c0}
    return {"value": out["steady"]["value"], "unit": UNIT, "batches": n_batches,
            "tokens": tokens, "tokens_per_batch": [min(len(b[0]) for b in batches),
                                                   max(len(b[0]) for b in batches)],
            "first_pass_value": out["first_pass"]["value"],
            "first_pass_captures": out["first_pass"]["captures"],
            "steady_captures": out["steady"]["captures"],
            "how": "GPUWorker.embed per batch (host ids/positions in, fp32 embeddings out), "
                   "graphs keyed on token buckets"}


COLD_L2 = ("before each launch 256 MB written, then another 256 MB read (L2 cold and clean); "
           "the launch is queued behind a GPU spin, so no host gap is timed")


def cold_launch_time(fn, args, dev) -> float:
    """Median CUDA-event time (s) of one launch of ``fn`` with a cold L2.  Before each launch
    a 256 MB buffer is written (the L2 flush) and a second 256 MB buffer read, which evicts
    the written lines so that their write-back is not timed; then the GPU spins for ~0.5 ms
    while the host queues the events and the launch, so the host's launch cost is not
    timed either."""
    import torch
    if not hasattr(cold_launch_time, "bufs"):
        cold_launch_time.bufs = (torch.empty(256 << 20, dtype=torch.uint8, device=dev),
                                 torch.ones(32 << 20, dtype=torch.int64, device=dev))
    wbuf, rbuf = cold_launch_time.bufs
    times = []
    for it in range(args.warmup + args.steps):
        wbuf.fill_(it & 0xFF)
        rbuf.sum()
        torch.cuda._sleep(1_000_000)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        if it >= args.warmup:
            times.append(e0.elapsed_time(e1) / 1000.0)
    return statistics.median(times)


GEMM_SHAPES = {
    # Qwen3-Embedding-4B projections (the GEMM microbenchmark's shapes), K x N
    "qkv": (2560, 6144), "o": (4096, 2560), "gate_up": (2560, 19456), "down": (9728, 2560),
    # Qwen3-Embedding-0.6B and -8B projections (the forward's GEMMs)
    "qkv_0.6b": (1024, 4096), "o_0.6b": (2048, 1024), "gate_up_0.6b": (1024, 6144),
    "down_0.6b": (3072, 1024),
    "qkv_8b": (4096, 6144), "o_8b": (4096, 4096), "gate_up_8b": (4096, 24576),
    "down_8b": (12288, 4096),
}


def run_gemm_micro(args):
    """AWQ W4A16 GEMM microbenchmark (one JSON line per shape and M), by default on the
    Qwen3-Embedding-4B projection shapes with the bf16 epilogue.  Each launch is timed
    alone with CUDA events and a cold L2 (``cold_launch_time``); the bound is
    min(tensor peak, arithmetic intensity x HBM).  For M > 256 a launch is the whole
    library call: the dequantisation of the weight panel and the tensor-core GEMM."""
    import torch
    import __graft_entry__
    __graft_entry__.build()
    from mes_b200 import _C, synthetic
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak_burst, _, hbm, peak_kind = peaks()
    gen = torch.Generator(device=dev).manual_seed(0)
    epi = args.gemm_epilogue
    lines = []
    clocks = ClockSampler(0).__enter__()   # over the whole run: one launch is too short
    for name in args.gemm_shapes.split(","):
        K, N = GEMM_SHAPES[name]
        qw, qz, sc = synthetic.random_awq(K, N, gen, dev)
        if epi == "silu":
            qw, qz, sc = _C.interleave_gate_up(qw, qz, sc.view(torch.int16))
            sc = sc.view(torch.float16)
        qwm, sc16 = _C.awq_repack(qw), sc.view(torch.int16)
        for M in (int(m) for m in args.gemm_m.split(",")):
            x = torch.randn(M, K, generator=gen, device=dev).to(torch.bfloat16)
            if epi == "silu":
                y = torch.empty(M, N // 2, dtype=torch.bfloat16, device=dev)
                fn = lambda: _C.awq_gemm_silu(x, qwm, qz, sc16, y)
            elif epi == "residual":
                y = torch.zeros(M, N, dtype=torch.float32, device=dev)
                fn = lambda: _C.awq_gemm_residual(x, qwm, qz, sc16, y)
            else:
                y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
                fn = lambda: _C.awq_gemm(x, qwm, qz, sc16, None, y)
            t = cold_launch_time(fn, args, dev)
            flops = 2.0 * M * N * K
            out_bytes = {"silu": M * N, "residual": 8 * M * N}.get(epi, 2 * M * N)
            nbytes = K * N / 2 + (K // 128) * N * 2.5 + 2 * M * K + out_bytes
            bound_tflops = min(peak_burst, flops / nbytes * hbm * 1e9 / 1e12)
            tf = flops / t / 1e12
            lines.append({
                "metric": "AWQ W4A16 GEMM TFLOP/s", "shape": name, "epilogue": epi, "M": M,
                "N": N, "K": K, "value": tf, "unit": "TFLOP/s", "us": t * 1e6,
                "steps": args.steps, "frac_of_tensor_peak": tf / peak_burst,
                "bound": "tensor" if bound_tflops >= peak_burst else "hbm",
                "frac_of_bound": tf / bound_tflops, "peak_kind": f"{peak_kind} bf16 burst",
                "weight_panel": bool(_C.lib().mes_awq_gemm_workspace_size(M, N, K)),
                "l2": COLD_L2})
            del x, y
    clocks.__exit__()
    for line in lines:
        line["clocks"] = clocks.summary()
        print(json.dumps(line), flush=True)


def run_elementwise_micro(args):
    """The memory-bound kernels of the forward at the 20 x 1000-token shapes of the
    Qwen3-0.6B workload (T = 20000, H = 1024, 16 q / 8 kv heads of 128, I = 3072), one JSON
    line per kernel: algorithmic HBM bytes per launch / CUDA-event time, against the HBM
    peak.  Each launch is timed alone with a cold L2 (``cold_launch_time``)."""
    import torch
    import __graft_entry__
    __graft_entry__.build()
    from mes_b200 import _C, synthetic
    from mes_b200.layers.rotary_embedding import RotaryEmbedding
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _, _, hbm, peak_kind = peaks()
    g = torch.Generator(device=dev).manual_seed(0)
    T, H, Hq, Hkv, D, I, V = 20000, 1024, 16, 8, 128, 3072, 151669
    _, pos_np, last_np = synthetic.packed_batch([1000] * 20, V, seed=1)
    pos = torch.from_numpy(pos_np).to(dev)
    last = torch.from_numpy(last_np).to(dev)
    ids = torch.randint(0, V, (T,), generator=g, device=dev)
    table = torch.randn(V, H, generator=g, device=dev).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(torch.bfloat16)
    wd = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).to(torch.bfloat16)
    res = torch.randn(T, H, generator=g, device=dev)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g, device=dev).to(torch.bfloat16)
    cache = RotaryEmbedding(D, D, 32768, 1e6).cos_sin_cache.to(dev)   # the model's fp32 table
    gu = torch.randn(T, 2 * I, generator=g, device=dev).to(torch.bfloat16)
    act = torch.empty(T, I, dtype=torch.bfloat16, device=dev)
    emb = torch.empty(T, H, dtype=torch.float32, device=dev)
    cases = [
        ("rmsnorm (fp32 residual in, bf16 out)", lambda: _C.rmsnorm(res, w, 1e-6, out),
         T * H * 4 + T * H * 2),
        ("add + rmsnorm (bf16 delta into the fp32 residual)",
         lambda: _C.add_rmsnorm_f32res(x, res, w, 1e-6, out), T * H * (2 + 8 + 2)),
        ("q/k rmsnorm + rope (in place, 16 q + 8 k heads)",
         lambda: _C.qknorm_rope(qkv, pos, cache, Hq, Hkv, D, wd, wd),
         2 * T * (Hq + Hkv) * D * 2 + T * 8),
        ("silu-and-mul (standalone)", lambda: _C.silu_mul(gu, act), T * I * 2 * 2 + T * I * 2),
        ("embedding gather (fp32 out)", lambda: _C.embedding_f32(ids, table, emb),
         T * H * 2 + T * 8 + T * H * 4),
        ("last token + L2 (20 rows)", lambda: _C.last_token_l2(out, last), 20 * H * 2 + 20 * H * 4),
        ("varlen schedule (20 sequences)", lambda: _C.varlen_schedule(pos), T * 8 + 4 * (T + 1)),
    ]
    lines = []
    with ClockSampler(0) as clocks:     # over all cases: one launch is too short to sample
        for name, fn, nbytes in cases:
            t = cold_launch_time(fn, args, dev)
            gbs = nbytes / t / 1e9
            lines.append({
                "metric": "HBM GB/s (algorithmic bytes)", "kernel": name, "value": gbs,
                "unit": "GB/s", "us": t * 1e6, "bytes": nbytes, "steps": args.steps,
                "frac_of_hbm_peak": gbs / hbm, "peak": hbm, "peak_kind": f"{peak_kind} HBM copy",
                "l2": COLD_L2})
    for line in lines:
        line["clocks"] = clocks.summary()
        print(json.dumps(line), flush=True)
    if _C.take_device_error():
        raise RuntimeError("device error in the elementwise benchmark")


def main():
    args = parse_args()
    import __graft_entry__
    __graft_entry__.load_package()
    if args.workload == "c3" and args.impl == "mes":
        run_gemm_micro(args)
        return
    if args.workload == "ew" and args.impl == "mes":
        run_elementwise_micro(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_mes(args)


if __name__ == "__main__":
    main()
